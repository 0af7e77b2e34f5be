"""Tests for the B200 decode hot path (CPU oracle pinning, host logic, GPU parity)."""
