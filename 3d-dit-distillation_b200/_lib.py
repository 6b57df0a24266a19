"""ctypes binding of ``libvdit.so`` (the C ABI declared in ``include/vdit.h``).

The library is built in-tree next to this file.  Every wrapper checks the
returned status and raises ``RuntimeError`` with the library's message; there
is no fallback path: a missing library or a non-CUDA tensor is an error.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libvdit.so"

_c_i32, _c_i64, _c_f32, _c_f64, _c_sz = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_double, ctypes.c_size_t
_vp = ctypes.c_void_p

# name -> (restype, argtypes), mirrors include/vdit.h
SIGNATURES = {
    "vdit_version": (ctypes.c_char_p, []),
    "vdit_error_string": (ctypes.c_char_p, [ctypes.c_int]),
    "vdit_last_cuda_error": (ctypes.c_char_p, []),
    "vdit_launch_count": (ctypes.c_longlong, []),
    "vdit_device_error": (ctypes.c_int, [ctypes.c_int]),
    "vdit_geometry_workspace_bytes": (_c_sz, [_c_i64]),
    "vdit_lex_perm": (ctypes.c_int, [_vp, _c_i64, _vp, _vp, _vp, _vp, _c_sz, _vp]),
    "vdit_hilbert4_orders": (ctypes.c_int, [_vp, _c_i64, _c_i32, _vp, _vp, _vp, _vp, _c_sz, _vp]),
    "vdit_conv_indices": (ctypes.c_int, [_vp, _c_i64, _vp, _vp]),
    "vdit_rope3d_table": (ctypes.c_int, [_c_i32, _c_i32, _c_f64, _vp, _vp, _vp]),
    "vdit_rope2d_table": (ctypes.c_int, [_c_i32, _c_i32, _c_f64, _vp, _vp, _vp]),
    "vdit_patchify": (ctypes.c_int, [_vp, _c_i64, _vp, _c_i32, _vp, _vp]),
    "vdit_modulate": (ctypes.c_int, [_vp, _c_i64, _c_i32, _vp, _vp, _vp, _vp]),
    "vdit_gate_add_modulate": (ctypes.c_int, [_vp, _vp, _c_i64, _c_i64, _c_i32, _vp, _vp, _vp, _vp, _vp]),
    "vdit_gate_add2_modulate": (ctypes.c_int, [_vp, _vp, _c_i64, _c_i64, _c_i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "vdit_out_modulate_unpatchify": (ctypes.c_int, [_vp, _c_i64, _c_i32, _vp, _vp, _vp, _vp, _vp]),
    "vdit_unpatchify_project": (ctypes.c_int, [_vp, _c_i64, _c_i32, _vp, _vp, _vp]),
    "vdit_split_weight3": (ctypes.c_int, [_vp, _c_i32, _c_i32, _vp, _vp]),
    "vdit_qknorm_rope3d_gather": (ctypes.c_int, [_vp, _c_i64, _c_i32, _c_i32, _vp, _vp, _vp, _vp, _c_i32, _vp,
                                                 _vp, _vp, _vp]),
    "vdit_qknorm_rope2d": (ctypes.c_int, [_vp, _c_i64, _c_i32, _c_i32, _vp, _vp, _vp, _vp, _c_i32, _vp]),
    "vdit_vec_ln_modulate": (ctypes.c_int, [_vp, _c_i32, _vp, _vp, _vp, _vp]),
    "vdit_vec_gate_residual": (ctypes.c_int, [_vp, _vp, _vp, _c_i32, _vp]),
    "vdit_swiglu_packed": (ctypes.c_int, [_vp, _c_i64, _c_i32, _vp, _vp]),
    "vdit_dwconv27": (ctypes.c_int, [_vp, _c_i64, _c_i32, _vp, _vp, _vp, _vp, _c_i32, _vp]),
    "vdit_dwconv27_plan_bytes": (ctypes.c_size_t, [_c_i64]),
    "vdit_dwconv27_plan": (ctypes.c_int, [_vp, _vp, _c_i64, _vp, ctypes.c_size_t, _vp]),
    "vdit_dwconv27_swiglu_planned": (ctypes.c_int, [_vp, _c_i64, _c_i32, _vp, _vp, _vp, _vp, _vp]),
    "vdit_dwconv27_swiglu_planned_bf16w": (ctypes.c_int, [_vp, _c_i64, _c_i32, _vp, _vp, _vp, _vp, _vp]),
    "vdit_attention": (ctypes.c_int, [_vp, _c_i64, _vp, _c_i64, _vp, _c_i64, _vp, _c_i64, _vp, _vp, _vp, _c_i32,
                                      _c_i32, _c_i32, _c_f32, _vp]),
    "vdit_attention_1q_workspace_bytes": (_c_sz, [_c_i32, _c_i32, _c_i64]),
    "vdit_attention_1q_wide_workspace_bytes": (_c_sz, [_c_i32, _c_i32, _c_i64]),
    "vdit_attention_1q_wide": (ctypes.c_int, [_vp, _vp, _c_i64, _c_i64, _vp, _vp, _c_i64, _vp, _c_i32, _c_i32, _c_f32,
                                              _vp, _vp, _c_sz, _vp]),
    "vdit_attention_1q": (ctypes.c_int, [_vp, _vp, _vp, _c_i64, _c_i64, _c_i32, _c_i32, _c_f32, _vp, _vp, _c_sz,
                                         _vp]),
    "vdit_attention_1q_noalloc": (ctypes.c_int, [_vp, _vp, _vp, _c_i64, _c_i64, _c_i32, _c_i32, _c_f32, _vp, _vp]),
    "vdit_dense_conv27": (ctypes.c_int, [_vp, _c_i64, _c_i32, _c_i32, _vp, _vp, _vp, _vp, _vp]),
    "vdit_gemv": (ctypes.c_int, [_c_i32, _vp, _c_i64, _vp, _vp, _c_i64, _c_i32, _vp, _c_i64, _vp, _c_i64, _c_i32,
                                 _c_i32, _vp, _c_i64, _c_i32, _c_i32, _c_i32, _vp]),
    "vdit_linear": (ctypes.c_int, [_vp, _c_i64, _vp, _c_i64, _vp, _vp, _c_i64, _c_i64, _c_i32, _c_i32, _vp]),
    "vdit_linear_qkv_rope3d": (ctypes.c_int, [_vp, _c_i64, _vp, _c_i64, _vp, _vp, _vp, _vp, _vp, _c_i32, _vp, _vp,
                                              _vp, _c_i64, _c_i64, _c_i32, _c_i32, _c_i32, _vp]),
    "vdit_gather_rows_f32": (ctypes.c_int, [_vp, _vp, _c_i64, _c_i32, _vp, _vp]),
    "vdit_cfg_reuse_workspace_bytes": (_c_sz, []),
    "vdit_cfg_reuse_euler": (ctypes.c_int, [_vp, _vp, _vp, _vp, _c_i64, _c_f32, _c_f32, _c_f32, _c_f32, _c_f32, _c_i32,
                                            _vp, _c_sz, _vp]),
    "vdit_neg_endpoint": (ctypes.c_int, [_vp, _vp, _c_i64, _c_f32, _vp, _vp]),
    "vdit_cfg_euler": (ctypes.c_int, [_vp, _vp, _vp, _c_i64, _c_f32, _c_f32, _vp]),
    "vdit_unpermute_denorm": (ctypes.c_int, [_vp, _vp, _c_i64, _vp, _vp, _vp, _vp]),
}

_LIB = None


def load() -> ctypes.CDLL:
    """Load and type the library (no GPU needed).  Raises if it is missing."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is missing: build it with __graft_entry__.build() "
                           "(python 3d-dit-distillation_b200/csrc/build.py)")
    lib = ctypes.CDLL(os.fspath(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


def lib() -> ctypes.CDLL:
    return _LIB if _LIB is not None else load()


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().vdit_error_string(rc).decode()
        detail = lib().vdit_last_cuda_error().decode() if rc == -3 else ""
        raise RuntimeError(f"{what} failed: {msg} (code {rc}){' ' + detail if detail else ''}")


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def ptr(t) -> int:
    """Device pointer of a CUDA tensor (None -> NULL)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise RuntimeError("vdit kernels need CUDA tensors (no CPU path)")
    return t.data_ptr()


def launch_count() -> int:
    return int(lib().vdit_launch_count())


def device_error(clear: bool = True) -> int:
    return int(lib().vdit_device_error(1 if clear else 0))
