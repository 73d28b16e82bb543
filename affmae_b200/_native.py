"""ctypes binding of ``libaffmae_b200.so`` (the C ABI of include/affmae_b200.h).

The library is loaded from ``affmae_b200/_lib`` only.  There is no fallback:
if the library is missing or a call fails, a ``RuntimeError`` is raised.
Helpers here turn torch tensors into raw pointers and dtype codes; torch is
used for device memory and streams only.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

import torch

_LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libaffmae_b200.so"
_lock = threading.Lock()
_lib = None

F32, F16, BF16 = 0, 1, 2
_DTYPE_CODE = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}

_p = C.c_void_p
_i64 = C.c_int64
_i32 = C.c_int
_f32 = C.c_float
_u32 = C.c_uint32

# entry point -> argtypes (all return an int status)
SIGNATURES = {
    "affb_knn": [_p, _p, _i32, _i64, _i64, _i64, _i32, _i32, _p, _p],
    "affb_weighted_features_fwd": [_p, _p, _p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _p, _p],
    "affb_weighted_features_bwd": [_p, _p, _p, _p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _p,
                                   _p, _p],
    "affb_nbhd_attn_fwd": [_p, _p, _p, _p, _p, _p, _i32, _p, _p, _i32, _i64, _i64, _i64, _i64,
                           _i64, _f32, _p, _p, _p],
    "affb_nbhd_attn_bwd": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i32, _p, _p, _i32, _i64, _i64,
                           _i64, _i64, _i64, _f32, _p, _p, _p, _p, _p, _p, _p, _i64, _p],
    "affb_pos_bias_fwd": [_p, _p, _i32, _i64, _i64, _i64, _i64, _i64, _p, _p],
    "affb_rel_bias_fwd": [_p, _p, _p, _i32, _i64, _i64, _i64, _i64, _p, _p],
    "affb_knn2d": [_p, _p, _i64, _i64, _i64, _i32, _p, _p, _i64, _p],
    "affb_layer_norm_fwd": [_p, _i32, _p, _i32, _f32, _u32, _p, _p, _f32, _i64, _i64, _p, _p, _p, _p, _p,
                            _p],
    "affb_layer_norm_bwd": [_p, _p, _p, _i32, _p, _p, _p, _f32, _u32, _i64, _i64, _p, _p, _i32, _p, _p,
                            _p],
    "affb_rel_bias_bwd": [_p, _p, _i32, _i64, _i64, _i64, _i64, _p, _p, _p],
    "affb_head_copy": [_p, _i64, _i64, _i64, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p],
    "affb_pos_bias_bwd": [_p, _p, _i32, _i64, _i64, _i64, _i64, _i64, _p, _p],
    "affb_deform_knn_fwd": [_p, _p, _p, _p, _p, _p, _i32, _i64, _i64, _i64, _i64, _i64, _p, _p,
                            _p, _p, _p],
    "affb_deform_knn_fwd_noalloc": [_p, _p, _p, _p, _p, _p, _i32, _i64, _i64, _i64, _i64, _i64, _p,
                                    _p, _p, _p],
    "affb_deform_knn_bwd": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i32, _i64, _i64, _i64, _i64,
                            _i64, _p, _p, _p, _p, _p, _p, _p],
    "affb_deform_nbidx_fwd": [_p, _p, _p, _p, _p, _p, _i32, _i64, _i64, _i64, _i64, _i32, _i64,
                              _p, _p],
    "affb_deform_nbidx_bwd": [_p, _p, _p, _p, _p, _p, _p, _i32, _i64, _i64, _i64, _i64, _i32,
                              _i64, _p, _p, _p, _p, _p, _p],
    "affb_msdetrpc_fwd": [_p, _p, _p, _p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _p, _p],
    "affb_msdetrpc_bwd": [_p, _p, _p, _p, _p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _p, _p,
                          _p, _p],
    "affb_mssample_fwd": [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i32, _p, _p],
    "affb_mssample_bwd": [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i32, _p, _p, _p, _p],
    "affb_cast_f32": [_p, _p, _i32, _i64, _p],
    "affb_dropout_keep_mask": [_u32, _f32, _i64, _i64, _p],
    "affb_nbhd_attn_fwd_plan": [_p, _p, _p, _p, _p, _p, _i32, _p, _p, _i32, _i64, _i64, _i64, _i64, _i64, _f32,
                                _p, _p, _p, _i64, _p],
    "affb_nbhd_attn_bwd_plan": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i32, _p, _p, _i32, _i64, _i64, _i64, _i64,
                                _i64, _f32, _p, _p, _p, _p, _p, _p, _p, _i64, _p, _i64, _p],
    "affb_nbhd_build": [_p, _p, _i64, _i64, _i64, _p, _p, _p, _p],
    "affb_token_mask_apply": [_p, _i32, _i64, _i64, _i64, _i64, _p, _i64, _i64, _p, _p],
    "affb_layer_norm_res_fwd": [_p, _i32, _p, _i32, _f32, _u32, _p, _i64, _p, _p, _f32, _i64, _i64, _p, _p, _p,
                                _p, _p, _p],
    "affb_layer_norm_res_bwd": [_p, _p, _p, _p, _p, _p, _p, _f32, _u32, _p, _i64, _i64, _i64, _p, _p, _i32, _p,
                                _p, _p],
    "affb_sine_embed": [_p, _i64, _i64, _p, _p, _p, _i32, _p],
    "affb_relu_dropout_fwd": [_p, _i32, _i64, _f32, _u32, _p, _p],
    "affb_relu_dropout_bwd": [_p, _p, _i32, _i64, _f32, _p, _p],
}
OTHER_SYMBOLS = ["affb_last_error", "affb_abi_version", "affb_deform_workspace_bytes",
                 "affb_deform_noalloc_max_scratch_bytes", "affb_nbhd_attn_bwd_workspace_bytes",
                 "affb_knn2d_workspace_bytes", "affb_nbhd_tile_plan_bytes"]


def library_path() -> Path:
    return _LIB_PATH


def lib():
    """Load the CUDA library once; raise if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not _LIB_PATH.exists():
            raise RuntimeError(
                f"affmae_b200 CUDA library not found at {_LIB_PATH}; build it with "
                "`python -m affmae_b200.build` (there is no CPU fallback)")
        l = C.CDLL(str(_LIB_PATH))
        l.affb_last_error.restype = C.c_char_p
        l.affb_last_error.argtypes = []
        l.affb_abi_version.restype = C.c_int
        l.affb_abi_version.argtypes = []
        l.affb_deform_workspace_bytes.restype = C.c_int64
        l.affb_deform_workspace_bytes.argtypes = [_i64, _i64]
        l.affb_deform_noalloc_max_scratch_bytes.restype = C.c_int64
        l.affb_deform_noalloc_max_scratch_bytes.argtypes = []
        l.affb_nbhd_attn_bwd_workspace_bytes.restype = C.c_int64
        l.affb_nbhd_attn_bwd_workspace_bytes.argtypes = [_i32, _i64, _i64, _i64, _i64, _i64]
        l.affb_knn2d_workspace_bytes.restype = C.c_int64
        l.affb_knn2d_workspace_bytes.argtypes = [_i64, _i64]
        l.affb_nbhd_tile_plan_bytes.restype = C.c_int64
        l.affb_nbhd_tile_plan_bytes.argtypes = [_i32, _i64, _i64, _i64, _i64]
        for name, args in SIGNATURES.items():
            fn = getattr(l, name)
            fn.argtypes = args
            fn.restype = C.c_int
        _lib = l
        return l


CALLS = 0  # entry-point calls made by this process (the benchmark reports them per step)


def call(name: str, *args) -> None:
    """Call an entry point; raise RuntimeError carrying the library's message."""
    global CALLS
    CALLS += 1
    rc = getattr(lib(), name)(*args)
    if rc != 0:
        msg = lib().affb_last_error().decode(errors="replace")
        raise RuntimeError(f"{name} failed (code {rc}): {msg}")


def ptr(t):
    return None if t is None else t.data_ptr()


def dcode(t: torch.Tensor) -> int:
    try:
        return _DTYPE_CODE[t.dtype]
    except KeyError:
        raise RuntimeError(f"unsupported dtype {t.dtype}; expected float32, float16 or bfloat16")


def stream(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("affmae_b200 ops need CUDA tensors (there is no CPU path)")


def cast_from_f32(acc: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """fp32 accumulator -> storage dtype, via the library's cast kernel."""
    if dtype == torch.float32:
        return acc
    out = torch.empty(acc.shape, dtype=dtype, device=acc.device)
    call("affb_cast_f32", ptr(acc), ptr(out), _DTYPE_CODE[dtype], acc.numel(), stream(acc.device))
    return out


def f32(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.float32).contiguous()


def scalar_dev(power: torch.Tensor, device) -> torch.Tensor:
    """The learned temperature as a 1-element fp32 device tensor (no host sync)."""
    if not torch.is_tensor(power):
        return torch.full((1,), float(power), dtype=torch.float32, device=device)
    p = power.detach().reshape(-1)[:1]
    return p.to(device=device, dtype=torch.float32).contiguous()
