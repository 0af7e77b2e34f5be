"""Plan/execute engine, fixed workspaces and the CUDA-graph owner."""
