"""ctypes wrapper around the C oracle ``oracle/gdn_oracle.c`` (test infrastructure).

The checker and the timed CPU baseline only; never imported by the product.
Same contract as ``oracle.gdn_ref`` (which restates
``solution/gdn_baseline_torch.py:12-91`` in torch), but a C loop parallel over
(sequence, v-head) chains, so parity tests and the CPU baseline can use larger
cases.  The library is built by ``oracle/Makefile`` into ``oracle/_build/``.
"""

from __future__ import annotations

import ctypes
import math
import os
import subprocess
from typing import Optional, Tuple

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libgdn_oracle.so")
_lib = None

_DTYPE_CODE = {torch.float32: 0, torch.bfloat16: 1}


def build() -> str:
    """Compile the C oracle with its Makefile (gcc + OpenMP)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        lib = ctypes.CDLL(_LIB_PATH)
        vp, i64, i32, f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
        lib.gdn_oracle_prefill.restype = i32
        lib.gdn_oracle_prefill.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64,
                                           i32, i32, i32, f32, i32, i32, vp, vp, i32, i32]
        lib.gdn_oracle_decode.restype = i32
        lib.gdn_oracle_decode.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, i64, i32, i32,
                                          i32, f32, i32, i32, vp, vp, i32, i32]
        _lib = lib
    return _lib


def _cpu(t: torch.Tensor, dtype=None) -> torch.Tensor:
    t = t.detach().cpu()
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    return t.contiguous()


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _threads(num_threads: Optional[int]) -> int:
    return num_threads or os.cpu_count() or 1


def prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale,
            num_threads: Optional[int] = None,
            qk_l2norm: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
    """Varlen prefill on the CPU; returns (output bf16 [T,Hv,D], new_state fp32 [N,Hv,D,D]).
    ``qk_l2norm`` applies the library's optional q/k L2 normalisation first."""
    lib = _load()
    q = _cpu(q, torch.bfloat16); k = _cpu(k, torch.bfloat16); v = _cpu(v, torch.bfloat16)
    if k.shape[1] != q.shape[1]:
        raise ValueError("the C oracle expects Hk == Hq")
    gdt = a.dtype if a.dtype in _DTYPE_CODE else torch.float32
    pdt = A_log.dtype if A_log.dtype in _DTYPE_CODE else torch.float32
    a = _cpu(a, gdt); b = _cpu(b, gdt)
    A_log = _cpu(A_log, pdt); dt_bias = _cpu(dt_bias, pdt)
    cu = _cpu(cu_seqlens, torch.int32)
    st = None if state is None else _cpu(state, torch.float32)
    T, Hq, D = q.shape
    Hv = v.shape[1]
    N = cu.numel() - 1
    if scale is None or scale == 0.0:
        scale = 1.0 / math.sqrt(D)
    out = torch.empty((T, Hv, D), dtype=torch.bfloat16)
    ns = torch.empty((N, Hv, D, D), dtype=torch.float32)
    rc = lib.gdn_oracle_prefill(_ptr(q), _ptr(k), _ptr(v), _ptr(st), _ptr(A_log), _ptr(a),
                                _ptr(dt_bias), _ptr(b), _ptr(cu), N, T, Hq, Hv, D, float(scale),
                                _DTYPE_CODE[gdt], _DTYPE_CODE[pdt], _ptr(out), _ptr(ns),
                                _threads(num_threads), int(qk_l2norm))
    if rc != 0:
        raise ValueError(f"gdn_oracle_prefill rejected its arguments (rc={rc})")
    return out, ns


def decode(q, k, v, state, A_log, a, dt_bias, b, scale,
           num_threads: Optional[int] = None,
           inplace: bool = False, qk_l2norm: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
    """Single-token decode on the CPU.  q,k [B,1,Hq,D], v [B,1,Hv,D], a,b [B,1,Hv].

    With ``inplace=True`` and an fp32 contiguous CPU ``state`` the update is
    written into ``state`` itself (the aliasing the product supports)."""
    lib = _load()
    B = q.shape[0]
    Hq, D = q.shape[-2], q.shape[-1]
    Hv = v.shape[-2]
    q = _cpu(q, torch.bfloat16).view(B, Hq, D)
    k = _cpu(k, torch.bfloat16).view(B, Hq, D)
    v = _cpu(v, torch.bfloat16).view(B, Hv, D)
    gdt = a.dtype if a.dtype in _DTYPE_CODE else torch.float32
    pdt = A_log.dtype if A_log.dtype in _DTYPE_CODE else torch.float32
    a = _cpu(a, gdt).view(B, Hv); b = _cpu(b, gdt).view(B, Hv)
    A_log = _cpu(A_log, pdt); dt_bias = _cpu(dt_bias, pdt)
    if scale is None or scale == 0.0:
        scale = 1.0 / math.sqrt(D)
    out = torch.empty((B, Hv, D), dtype=torch.bfloat16)
    if inplace:
        if state is None or state.device.type != "cpu" or state.dtype != torch.float32 \
                or not state.is_contiguous():
            raise ValueError("inplace decode needs a contiguous fp32 CPU state")
        st = ns = state
    else:
        st = None if state is None else _cpu(state, torch.float32)
        ns = torch.empty((B, Hv, D, D), dtype=torch.float32)
    rc = lib.gdn_oracle_decode(_ptr(q), _ptr(k), _ptr(v), _ptr(st), _ptr(A_log), _ptr(a),
                               _ptr(dt_bias), _ptr(b), B, Hq, Hv, D, float(scale),
                               _DTYPE_CODE[gdt], _DTYPE_CODE[pdt], _ptr(out), _ptr(ns),
                               _threads(num_threads), int(qk_l2norm))
    if rc != 0:
        raise ValueError(f"gdn_oracle_decode rejected its arguments (rc={rc})")
    return out.unsqueeze(1), ns
