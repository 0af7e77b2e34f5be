"""ctypes binding of the C-ABI kernel library ``libsgld_sm100.so`` (include/sgld_b200.h).

This is the only path from Python to the GPU work of the decode hot path: there is
no Triton, no torch fallback and no CPU fallback.  Importing is cheap; the library
is loaded on first use and a missing or unloadable library raises immediately.
"""
from __future__ import annotations

import ctypes
import threading

from . import _build

_I32P = ctypes.c_void_p


class PlanGeometry(ctypes.Structure):
    """sgld_plan_geometry."""
    _fields_ = [("batch_capacity", ctypes.c_int32), ("max_splits", ctypes.c_int32),
                ("max_context", ctypes.c_int32), ("groups", ctypes.c_int32),
                ("workers", ctypes.c_int32)]


PLAN_FIELDS = ("lengths", "splits", "active", "counts", "offsets", "chunk", "request", "split",
               "begin", "end", "weight", "order", "pack_first", "pack_count", "record_count",
               "num_packs", "mode", "error", "static_head", "static_next", "arrivals")


def plan_field_words(batch_capacity, max_splits, groups, workers):
    """int32 words of each plan buffer, in PLAN_FIELDS order: the layout of the single plan
    storage (sgld_plan_storage_words / sgld_plan_buffers_in_storage)."""
    b = batch_capacity
    e = b * max_splits
    t = e * groups
    return (b, b, 1, b, b + 1, b, e, e, e, e, e, e, t, t, 1, 1, 1, 1, workers, t, b * groups)


class PlanBuffersC(ctypes.Structure):
    """sgld_plan_buffers: device pointers of every plan array."""
    _fields_ = [(name, ctypes.c_void_p) for name in PLAN_FIELDS]


class DecodeArgs(ctypes.Structure):
    """sgld_decode_args."""
    _fields_ = [
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
        ("out", ctypes.c_void_p), ("pages", ctypes.c_void_p), ("indptr", ctypes.c_void_p),
        ("q_stride", ctypes.c_int64 * 3), ("k_stride", ctypes.c_int64 * 4),
        ("v_stride", ctypes.c_int64 * 4), ("pt_stride", ctypes.c_int64 * 2),
        ("kv_extent", ctypes.c_int64),
        ("dtype", ctypes.c_int32), ("query_heads", ctypes.c_int32), ("kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32), ("page_size", ctypes.c_int32), ("scale", ctypes.c_float), ("logit_cap", ctypes.c_float),
        ("kv_dtype", ctypes.c_int32), ("k_scale", ctypes.c_float), ("v_scale", ctypes.c_float),
        ("q_rows", ctypes.c_int32),
        ("k_new", ctypes.c_void_p), ("v_new", ctypes.c_void_p), ("new_loc", ctypes.c_void_p),
        ("knew_stride", ctypes.c_int64 * 3), ("vnew_stride", ctypes.c_int64 * 3),
        ("new_loc_int32", ctypes.c_int32),
        ("counter", ctypes.c_void_p), ("partial", ctypes.c_void_p), ("lse", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
    ]


DTYPE_F16, DTYPE_BF16, DTYPE_E4M3 = 0, 1, 2
STATUS = {0: "ok", 1: "invalid argument", 2: "unsupported", 3: "cuda error"}
EXPORTS = ("sgld_abi_version", "sgld_last_error", "sgld_layer_workspace_bytes", "sgld_plan_build",
           "sgld_decode_persistent", "sgld_merge_splits", "sgld_decode_persistent_noalloc",
           "sgld_decode_kernel_kind", "sgld_plan_storage_words", "sgld_plan_buffers_in_storage")
ABI_VERSION = 9
KERNEL_KINDS = {0: "mma.sync", 1: "tcgen05", 2: "tcgen05+tma", 3: "mma.sync+tma", 4: "small"}

_lock = threading.Lock()
_lib = None
_ops = None


class NativeError(RuntimeError):
    """A C-ABI call returned a non-zero sgld_status."""


def load(path=None):
    """Load (once) and return the ctypes handle; raise if the library is unavailable."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        lib_path = path or _build.library_path()
        if not lib_path.exists():
            raise RuntimeError(
                f"{lib_path} is missing: build the CUDA extension first "
                "(python -m sglang_decode._build or __graft_entry__.build()); "
                "there is no fallback implementation")
        lib = ctypes.CDLL(str(lib_path))
        lib.sgld_abi_version.restype = ctypes.c_int32
        lib.sgld_last_error.restype = ctypes.c_char_p
        lib.sgld_layer_workspace_bytes.restype = ctypes.c_size_t
        lib.sgld_layer_workspace_bytes.argtypes = [ctypes.c_int32] * 5
        lib.sgld_plan_build.restype = ctypes.c_int
        lib.sgld_plan_build.argtypes = [ctypes.POINTER(PlanBuffersC), ctypes.POINTER(PlanGeometry),
                                        ctypes.c_int32, ctypes.c_void_p, ctypes.c_int32,
                                        ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p]
        lib.sgld_decode_persistent.restype = ctypes.c_int
        lib.sgld_decode_persistent.argtypes = [ctypes.POINTER(DecodeArgs), ctypes.POINTER(PlanBuffersC),
                                               ctypes.POINTER(PlanGeometry), ctypes.c_void_p]
        lib.sgld_decode_persistent_noalloc.restype = ctypes.c_int
        lib.sgld_decode_persistent_noalloc.argtypes = lib.sgld_decode_persistent.argtypes
        lib.sgld_decode_kernel_kind.restype = ctypes.c_int
        lib.sgld_decode_kernel_kind.argtypes = lib.sgld_decode_persistent.argtypes[:3]
        lib.sgld_plan_storage_words.restype = ctypes.c_size_t
        lib.sgld_plan_storage_words.argtypes = [ctypes.POINTER(PlanGeometry)]
        lib.sgld_plan_buffers_in_storage.restype = ctypes.c_int
        lib.sgld_plan_buffers_in_storage.argtypes = [ctypes.c_void_p, ctypes.POINTER(PlanGeometry),
                                                     ctypes.POINTER(PlanBuffersC)]
        lib.sgld_merge_splits.restype = ctypes.c_int
        lib.sgld_merge_splits.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int32] * 5 + [ctypes.c_void_p]
        if lib.sgld_abi_version() != ABI_VERSION:
            raise RuntimeError(f"{lib_path}: ABI version {lib.sgld_abi_version()} != {ABI_VERSION}")
        if path is None:
            _lib = lib
        return lib


def ops():
    """The torch operator library (``torch.ops.sglang_decode``: plan_build, decode, merge),
    loaded once; it calls the C ABI of ``libsgld_sm100.so``.  Raises if it is not built."""
    global _ops
    if _ops is not None:
        return _ops
    load()                                         # the C ABI library first (version check; takes _lock)
    with _lock:
        if _ops is None:
            import torch
            path = _build.ops_library_path()
            if not path.exists():
                raise RuntimeError(f"{path} is missing: build the extension first (python -m sglang_decode._build "
                                   "or __graft_entry__.build()); there is no fallback implementation")
            torch.ops.load_library(str(path))
            _ops = torch.ops.sglang_decode
    return _ops


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().sgld_last_error().decode(errors="replace")
        kind = STATUS.get(rc, str(rc))
        if rc in (1, 2):
            raise ValueError(f"{what}: {kind}: {msg}")
        raise NativeError(f"{what}: {kind}: {msg}")


def layer_workspace_bytes(batch_capacity, query_heads, kv_heads, head_dim, max_splits) -> int:
    return int(load().sgld_layer_workspace_bytes(batch_capacity, query_heads, kv_heads, head_dim,
                                                 max_splits))


def plan_build(plan_c, geometry_c, force_mode, rules_ptr, n_rules, counters_ptr, n_counters, stream):
    rc = load().sgld_plan_build(ctypes.byref(plan_c), ctypes.byref(geometry_c), int(force_mode),
                                rules_ptr, int(n_rules), counters_ptr, int(n_counters), stream)
    check(rc, "sgld_plan_build")


def decode_persistent(args_c, plan_c, geometry_c, stream):
    rc = load().sgld_decode_persistent(ctypes.byref(args_c), ctypes.byref(plan_c),
                                       ctypes.byref(geometry_c), stream)
    check(rc, "sgld_decode_persistent")


def decode_kernel_kind(args_c, plan_c, geometry_c) -> str:
    """Name of the decode kernel sgld_decode_persistent launches for these arguments."""
    rc = load().sgld_decode_kernel_kind(ctypes.byref(args_c), ctypes.byref(plan_c), ctypes.byref(geometry_c))
    if rc < 0:
        check(-rc, "sgld_decode_kernel_kind")
    return KERNEL_KINDS[rc]


def merge_splits(partial, lse, counts, error, out, dtype, batch_capacity, query_heads, head_dim,
                 max_splits, stream):
    rc = load().sgld_merge_splits(partial, lse, counts, error, out, dtype, batch_capacity,
                                  query_heads, head_dim, max_splits, stream)
    check(rc, "sgld_merge_splits")
