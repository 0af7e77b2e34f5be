"""Decode the raw fp16/bf16 bits stored in attention.npz into torch / numpy arrays."""
import numpy as np
import torch

DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16}


def load_case(arrays, meta):
    """Return (q, k, v, pages) as torch tensors on the CPU in the case's dtype."""
    dtype = DTYPES[meta["dtype"]]
    name = meta["name"]
    q, k, v = (torch.from_numpy(np.ascontiguousarray(arrays[f"{name}/{x}"])).view(dtype)
               for x in ("q", "k", "v"))
    pages = torch.from_numpy(np.ascontiguousarray(arrays[f"{name}/pages"]))
    return q, k, v, pages


def as_f32(t):
    return t.float().numpy()
