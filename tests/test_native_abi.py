"""The C-ABI library loads without a GPU and matches include/*.h (no compute calls).

* every function declared in include/*.h is exported by libsgld_sm100.so;
* the ctypes structs of sglang_decode._native have the C header's size and field
  offsets (a tiny C program compiled with gcc prints them);
* host-side argument checks answer with the documented status codes and messages.
"""
import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from sglang_decode import _build, _native

ROOT = Path(__file__).resolve().parents[1]
HEADERS = sorted((ROOT / "include").glob("*.h"))
DECL = re.compile(r"^\s*(?:int|int32_t|size_t|const char\s*\*)\s+(sgld_\w+)\s*\(", re.M)


def declared_functions():
    names = []
    for h in HEADERS:
        names += DECL.findall(h.read_text())
    return names


@pytest.fixture(scope="module")
def lib():
    _build.build()
    return _native.load()


def test_header_declares_the_entry_points():
    names = declared_functions()
    for required in ("sgld_plan_build", "sgld_decode_persistent", "sgld_merge_splits",
                     "sgld_layer_workspace_bytes", "sgld_last_error", "sgld_abi_version"):
        assert required in names


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert set(_native.EXPORTS) <= set(declared_functions())


def test_abi_version_and_workspace_size(lib):
    assert lib.sgld_abi_version() == _native.ABI_VERSION
    b, hq, hkv, d, smax = 64, 32, 8, 128, 16
    slots = b * hq * smax
    assert _native.layer_workspace_bytes(b, hq, hkv, d, smax) == 8 + slots * d * 4 + slots * 4 + 4
    assert _native.layer_workspace_bytes(0, hq, hkv, d, smax) == 0


def test_host_checks_reject_bad_arguments_without_touching_a_gpu(lib):
    assert lib.sgld_plan_build(None, None, -1, None, 0, None, 0, None) == 1
    assert b"NULL" in lib.sgld_last_error()
    geo = _native.PlanGeometry(64, 100, 32768, 8, 148)          # 6400 records > 4096
    plan = _native.PlanBuffersC(**{n: 16 for n in _native.PLAN_FIELDS})
    assert lib.sgld_plan_build(ctypes.byref(plan), ctypes.byref(geo), -1, None, 0, None, 0, None) == 1
    assert b"4096" in lib.sgld_last_error()
    geo = _native.PlanGeometry(64, 16, 32768, 8, 148)
    assert lib.sgld_plan_build(ctypes.byref(plan), ctypes.byref(geo), 7, None, 0, None, 0, None) == 1
    args = _native.DecodeArgs()
    assert lib.sgld_decode_persistent(ctypes.byref(args), ctypes.byref(plan), ctypes.byref(geo), None) == 1
    args.q = args.k = args.v = args.out = args.pages = 16
    args.counter = args.partial = args.lse = args.status = 16
    args.dtype, args.query_heads, args.kv_heads, args.head_dim, args.page_size = 1, 32, 8, 96, 16
    assert lib.sgld_decode_persistent(ctypes.byref(args), ctypes.byref(plan), ctypes.byref(geo), None) == 1
    assert b"kv_dtype" in lib.sgld_last_error()                # K/V dtype must match q or be e4m3
    args.kv_dtype = args.dtype
    args.partial = 20                                          # the epilogue and merge store float4 rows
    assert lib.sgld_decode_persistent(ctypes.byref(args), ctypes.byref(plan), ctypes.byref(geo), None) == 1
    assert b"16-byte aligned" in lib.sgld_last_error()
    args.partial = 16
    for bad in (-1.0, float("nan"), float("inf")):             # the soft cap must be finite and >= 0
        args.logit_cap = bad
        assert lib.sgld_decode_persistent(ctypes.byref(args), ctypes.byref(plan), ctypes.byref(geo), None) == 1
        assert b"logit_cap" in lib.sgld_last_error()
    args.logit_cap = 0.0
    for name in ("k_scale", "v_scale"):                         # scales: finite and >= 0
        setattr(args, name, -2.0)
        assert lib.sgld_decode_persistent(ctypes.byref(args), ctypes.byref(plan), ctypes.byref(geo), None) == 1
        setattr(args, name, 0.0)
    assert lib.sgld_decode_persistent(ctypes.byref(args), ctypes.byref(plan), ctypes.byref(geo), None) == 2
    args.kv_dtype, args.head_dim = _native.DTYPE_E4M3, 64        # fp8 K/V: head_dim 128 only
    assert lib.sgld_decode_persistent(ctypes.byref(args), ctypes.byref(plan), ctypes.byref(geo), None) == 2
    assert b"fp8" in lib.sgld_last_error()
    args.kv_dtype, args.head_dim = args.dtype, 96
    assert lib.sgld_decode_persistent(ctypes.byref(args), ctypes.byref(plan), ctypes.byref(geo), None) == 2
    assert b"head dimensions" in lib.sgld_last_error()
    args.head_dim, args.query_heads = 128, 8 * 17
    assert lib.sgld_decode_persistent(ctypes.byref(args), ctypes.byref(plan), ctypes.byref(geo), None) == 2
    # q_rows and the fused KV write (every case below fails its host check before a launch)
    args.query_heads = 32
    decode = lambda: lib.sgld_decode_persistent(ctypes.byref(args), ctypes.byref(plan), ctypes.byref(geo), None)
    args.q_rows = 65                                            # more Q rows than the capacity (64)
    assert decode() == 1 and b"q_rows" in lib.sgld_last_error()
    args.q_rows, args.k_new = 0, 16                             # new rows without their slots
    assert decode() == 1 and b"new_loc" in lib.sgld_last_error()
    args.new_loc = 16                                           # slots without v_new
    assert decode() == 1 and b"k_new, v_new and new_loc" in lib.sgld_last_error()
    with pytest.raises(ValueError):
        _native.check(1, "probe")


C_LAYOUT = r"""
#include <stddef.h>
#include <stdio.h>
#include "sgld_b200.h"
#define F(S, f) printf("%s.%s %zu\n", #S, #f, offsetof(S, f));
int main(void) {
  printf("sgld_plan_geometry %zu\n", sizeof(sgld_plan_geometry));
  printf("sgld_plan_buffers %zu\n", sizeof(sgld_plan_buffers));
  printf("sgld_decode_args %zu\n", sizeof(sgld_decode_args));
  F(sgld_plan_geometry, workers) F(sgld_plan_buffers, static_next)
  F(sgld_decode_args, q_stride) F(sgld_decode_args, kv_extent) F(sgld_decode_args, dtype)
  F(sgld_decode_args, scale) F(sgld_decode_args, logit_cap) F(sgld_decode_args, kv_dtype)
  F(sgld_decode_args, k_scale) F(sgld_decode_args, v_scale) F(sgld_decode_args, q_rows)
  F(sgld_decode_args, k_new) F(sgld_decode_args, v_new) F(sgld_decode_args, new_loc)
  F(sgld_decode_args, knew_stride) F(sgld_decode_args, vnew_stride) F(sgld_decode_args, new_loc_int32)
  F(sgld_decode_args, counter) F(sgld_decode_args, partial)
  F(sgld_decode_args, lse) F(sgld_decode_args, status)
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_ctypes_structs_match_the_c_header(tmp_path):
    src = tmp_path / "layout.c"
    src.write_text(C_LAYOUT)
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", f"-I{ROOT / 'include'}", str(src), "-o", str(exe)], check=True)
    got = dict(line.rsplit(" ", 1) for line in subprocess.check_output([str(exe)], text=True).splitlines())
    want = {
        "sgld_plan_geometry": ctypes.sizeof(_native.PlanGeometry),
        "sgld_plan_buffers": ctypes.sizeof(_native.PlanBuffersC),
        "sgld_decode_args": ctypes.sizeof(_native.DecodeArgs),
        "sgld_plan_geometry.workers": _native.PlanGeometry.workers.offset,
        "sgld_plan_buffers.static_next": _native.PlanBuffersC.static_next.offset,
    }
    for field in ("q_stride", "kv_extent", "dtype", "scale", "logit_cap", "kv_dtype", "k_scale", "v_scale",
                  "q_rows", "k_new", "v_new", "new_loc", "knew_stride", "vnew_stride", "new_loc_int32",
                  "counter", "partial", "lse", "status"):
        want[f"sgld_decode_args.{field}"] = getattr(_native.DecodeArgs, field).offset
    assert {k: int(v) for k, v in got.items()} == want
