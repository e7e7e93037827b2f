"""Loader of the kvquant_b200 CUDA library (drop-in for kvquant/kernels/cuda_ops.py).

The reference JIT-builds a pybind11 extension and returns ``None`` when that
fails, silently falling back to PyTorch (kvquant/kernels/cuda_ops.py:13-46).
This package ships a prebuilt sm_100a C-ABI library (``_lib/libkvquant_b200.so``)
and binds it with ctypes; ``get_cuda_ops()`` returns an object exposing the
reference's four op names with the reference's signatures and return types
(kvquant/kernels/csrc/kvquant_ops.cu:265-270), plus the fused decode ops.

There is no CPU fallback: a missing library raises on first use
(``cuda_available()`` reports it), and ops reject non-CUDA tensors.
Errors from the library are raised as ``RuntimeError``, the exception the
reference's ``TORCH_CHECK`` produces.
"""
from __future__ import annotations

import ctypes
import math
import os
import threading
from pathlib import Path

import torch

_LIB_PATH = Path(__file__).resolve().parent.parent / "_lib" / "libkvquant_b200.so"

_c_i64 = ctypes.c_int64
_c_int = ctypes.c_int
_c_p = ctypes.c_void_p
_c_size = ctypes.c_size_t
_c_dbl = ctypes.c_double
_c_flt = ctypes.c_float

# name -> (restype, argtypes); mirrors include/kvquant_b200.h
_SIGNATURES = {
    "kvq_last_error": (ctypes.c_char_p, []),
    "kvq_version": (_c_int, []),
    "kvq_check_status": (_c_int, [_c_p]),
    "kvq_set_decode_kernels": (_c_int, [_c_int, _c_int]),
    "kvq_decode_kernels": (_c_int, []),
    "kvq_rope_apply": (_c_int, [_c_p, _c_p, _c_p, _c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                                _c_i64, _c_p]),
    "kvq_lut_matvec": (_c_int, [_c_p, _c_p, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_i64,
                                _c_int, _c_p]),
    "kvq_sparse_matvec_csr": (_c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_i64, _c_i64,
                                       _c_p]),
    "kvq_normalize": (_c_int, [_c_p, _c_i64, _c_i64, _c_p, _c_p, _c_int, _c_p, _c_p]),
    "kvq_lut_lookup": (_c_int, [_c_p, _c_p, _c_i64, _c_p, _c_p, _c_i64, _c_p]),
    "kvq_quantize_keys_workspace": (_c_size, [_c_i64, _c_i64, _c_i64]),
    "kvq_quantize_keys_plan": (_c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_p,
                                        _c_dbl, _c_int, _c_p, _c_i64, _c_p, _c_p, _c_size, _c_p]),
    "kvq_quantize_keys_emit": (_c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_p,
                                        _c_p, _c_int, _c_dbl, _c_int, _c_p, _c_i64, _c_p, _c_p,
                                        _c_i64, _c_p, _c_p, _c_p, _c_size, _c_p]),
    "kvq_quantize_values_workspace": (_c_size, [_c_i64, _c_i64, _c_i64]),
    "kvq_quantize_values_plan": (_c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_dbl,
                                          _c_int, _c_p, _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_p,
                                          _c_size, _c_p]),
    "kvq_quantize_values_emit": (_c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_p,
                                          _c_int, _c_dbl, _c_int, _c_p, _c_p, _c_i64, _c_p,
                                          _c_i64, _c_p, _c_p, _c_i64, _c_p, _c_p, _c_p,
                                          _c_size, _c_p]),
    "kvq_key_scores": (_c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_int, _c_p,
                                _c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_p]),
    "kvq_key_stats_size": (_c_size, [_c_i64, _c_i64]),
    "kvq_value_output_scores_workspace": (_c_size, [_c_i64, _c_i64, _c_i64, _c_i64]),
    "kvq_key_scores_stats": (_c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_int, _c_p,
                                      _c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_flt,
                                      _c_p, _c_p]),
    "kvq_value_output_scores": (_c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_p, _c_p,
                                         _c_int, _c_p, _c_p, _c_flt, _c_i64, _c_i64, _c_i64,
                                         _c_i64, _c_i64, _c_p, _c_p, _c_size, _c_p]),
    "kvq_key_scores_stats_at": (_c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_int,
                                         _c_p, _c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                                         _c_i64, _c_p, _c_flt, _c_p, _c_p]),
    "kvq_value_output_scores_ml": (_c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_p, _c_p,
                                            _c_int, _c_p, _c_p, _c_flt, _c_i64, _c_i64, _c_i64,
                                            _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_size, _c_p]),
    "kvq_merge_shards": (_c_int, [_c_p, _c_p, _c_i64, _c_i64, _c_p, _c_p]),
    "kvq_softmax_workspace": (_c_size, [_c_i64, _c_i64]),
    "kvq_softmax": (_c_int, [_c_p, _c_i64, _c_i64, _c_flt, _c_p, _c_p, _c_size, _c_p]),
    "kvq_value_output_workspace": (_c_size, [_c_i64, _c_i64, _c_i64, _c_i64]),
    "kvq_value_output": (_c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_p, _c_p, _c_int,
                                  _c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_p,
                                  _c_size, _c_p]),
    "kvq_value_output_noalloc": (_c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_p, _c_p,
                                          _c_int, _c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                                          _c_p, _c_p]),
    "kvq_append_keys": (_c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p,
                                 _c_p, _c_int, _c_i64, _c_p, _c_i64, _c_p, _c_p, _c_i64, _c_p,
                                 _c_p]),
    "kvq_append_values_workspace": (_c_size, [_c_i64, _c_i64]),
    "kvq_append_values": (_c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_dbl, _c_p,
                                   _c_int, _c_i64, _c_p, _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_p,
                                   _c_i64, _c_p, _c_size, _c_p, _c_p]),
    "kvq_fit_codebook_workspace": (_c_size, [_c_i64]),
    "kvq_fit_codebook": (_c_int, [_c_p, _c_p, _c_i64, _c_int, _c_int, _c_p, _c_p, _c_size, _c_p,
                                  _c_p]),
    "kvq_decode_attention_workspace": (_c_size, [_c_i64, _c_i64, _c_i64, _c_i64]),
    "kvq_decode_attention": (_c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p,
                                      _c_p, _c_p, _c_p, _c_i64, _c_p, _c_p, _c_int, _c_p,
                                      _c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_p,
                                      _c_p, _c_p, _c_size, _c_p]),
}

_lock = threading.Lock()
_lib = None
_ops = None
_load_error = None


def library_path() -> Path:
    return Path(os.environ.get("KVQ_B200_LIB", _LIB_PATH))


def load_library():
    """Loads and binds the shared library (raises OSError if it is missing)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        lib = ctypes.CDLL(str(library_path()))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def _ptr(t) -> int | None:
    if t is None:
        return None
    return t.data_ptr()


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _check(rc: int, lib) -> None:
    if rc != 0:
        msg = lib.kvq_last_error().decode("utf-8", "replace")
        raise RuntimeError(msg or f"kvquant_b200 error code {rc}")


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("all must be CUDA")


class CudaOps:
    """The module-like object returned by ``get_cuda_ops()``."""

    def __init__(self, lib):
        self.lib = lib

    # -- the reference's four ops --------------------------------------------------
    def rope_apply(self, x, cos_cache, sin_cache, pos_offset: int):
        """kvquant/kernels/csrc/kvquant_ops.cu:156-182."""
        _require_cuda(x)
        if x.dim() != 4:
            raise RuntimeError("x must be [B,H,S,D]")
        if x.dtype != torch.float16:
            raise RuntimeError("x must be fp16")
        _require_cuda(cos_cache, sin_cache)
        xc = x.contiguous()
        cc = cos_cache.to(torch.float32).contiguous()
        sc = sin_cache.to(torch.float32).contiguous()
        out = torch.empty_like(xc)
        B, H, S, D = xc.shape
        s_total = cc.shape[0] if cc.dim() >= 1 else 0
        with torch.cuda.device(x.device):
            _check(self.lib.kvq_rope_apply(_ptr(xc), _ptr(cc), _ptr(sc), _ptr(out), B, H, S, D,
                                           int(pos_offset), s_total, _stream(xc)), self.lib)
        return out

    def lut_matvec(self, qmat, lut, scale, zero, vec, per_channel: bool):
        """kvquant/kernels/csrc/kvquant_ops.cu:184-216."""
        _require_cuda(qmat, lut, scale, zero, vec)
        qc = qmat.to(torch.uint8).contiguous()
        lc = lut.to(torch.float16).contiguous()
        sc = scale.to(torch.float16).contiguous()
        zc = zero.to(torch.float16).contiguous()
        vc = vec.to(torch.float16).contiguous()
        N, D = qc.shape
        out = torch.empty(N, dtype=torch.float16, device=vc.device)
        with torch.cuda.device(vc.device):
            _check(self.lib.kvq_lut_matvec(_ptr(qc), _ptr(lc), lc.numel(), _ptr(sc), _ptr(zc),
                                           _ptr(vc), _ptr(out), N, D, int(bool(per_channel)),
                                           _stream(vc)), self.lib)
        return out

    def sparse_matvec_csr(self, row_ptr, col_idx, values, vec, R: int):
        """kvquant/kernels/csrc/kvquant_ops.cu:218-241."""
        _require_cuda(row_ptr, col_idx, values, vec)
        rp = row_ptr.to(torch.int32).contiguous()
        ci = col_idx.to(torch.int32).contiguous()
        vs = values.to(torch.float16).contiguous()
        vc = vec.to(torch.float16).contiguous()
        R = int(R)
        if rp.numel() < R + 1:
            raise RuntimeError("row_ptr must have R+1 entries")
        out = torch.empty(R, dtype=torch.float16, device=vc.device)
        with torch.cuda.device(vc.device):
            _check(self.lib.kvq_sparse_matvec_csr(_ptr(rp), _ptr(ci), _ptr(vs), _ptr(vc), _ptr(out),
                                                  R, ci.numel(), vc.numel(), _stream(vc)),
                   self.lib)
        return out

    def lut_lookup(self, x, codebook):
        """kvquant/kernels/csrc/kvquant_ops.cu:243-263: [idx int64, dq fp32], flattened."""
        _require_cuda(x, codebook)
        xc = x.reshape(-1).to(torch.float32).contiguous()
        cb = codebook.reshape(-1).to(torch.float32).contiguous()
        idx = torch.empty(xc.numel(), dtype=torch.int64, device=xc.device)
        dq = torch.empty(xc.numel(), dtype=torch.float32, device=xc.device)
        with torch.cuda.device(xc.device):
            _check(self.lib.kvq_lut_lookup(_ptr(xc), _ptr(cb), cb.numel(), _ptr(idx), _ptr(dq),
                                           xc.numel(), _stream(xc)), self.lib)
        return [idx, dq]

    def normalize(self, x, zero, scale, per_channel: bool):
        """The quantizers' n = (x - zero) / (scale + 1e-8) (kv_quantizer.py:82,104) of
        x [rows, cols] fp16, zero/scale per column (per_channel) or per row: fp32."""
        _require_cuda(x, zero, scale)
        if x.dim() != 2 or x.dtype != torch.float16:
            raise RuntimeError("x must be fp16 [rows, cols]")
        xc = x.contiguous()
        rows, cols = xc.shape
        zc = zero.to(torch.float32).contiguous()
        sc = scale.to(torch.float32).contiguous()
        if zc.numel() != (cols if per_channel else rows) or sc.numel() != zc.numel():
            raise RuntimeError("zero/scale must have one entry per column (per_channel) or row")
        out = torch.empty((rows, cols), dtype=torch.float32, device=xc.device)
        with torch.cuda.device(xc.device):
            _check(self.lib.kvq_normalize(_ptr(xc), rows, cols, _ptr(zc), _ptr(sc),
                                          int(bool(per_channel)), _ptr(out), _stream(xc)),
                   self.lib)
        return out

    # -- status --------------------------------------------------------------------
    def check_status(self, device=None):
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
        with torch.cuda.device(dev):
            _check(self.lib.kvq_check_status(torch.cuda.current_stream(dev).cuda_stream),
                   self.lib)


def _try_load():
    global _ops, _load_error
    if _ops is not None:
        return _ops
    try:
        _ops = CudaOps(load_library())
        _load_error = None
    except OSError as e:
        _load_error = repr(e)
        return None
    return _ops


def get_cuda_ops() -> CudaOps:
    """Returns the bound library object.

    Unlike the reference (which returns None and falls back to PyTorch), this
    raises when the library cannot be loaded: there is no CPU path.
    """
    ops = _try_load()
    if ops is None:
        raise RuntimeError(
            f"kvquant_b200 CUDA library not loadable from {library_path()}: {_load_error}. "
            "Build it with `python kvquant-paper-repro_b200/build_lib.py`.")
    return ops


def cuda_available() -> bool:
    """True when the library is loaded and a CUDA device is present."""
    return torch.cuda.is_available() and _try_load() is not None


def load_error():
    return _load_error


def ceil_div(a: int, b: int) -> int:
    return -(-a // b)


def rsqrt_head_dim(d: int) -> float:
    return 1.0 / math.sqrt(d)
