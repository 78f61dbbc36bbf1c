"""TEST INFRASTRUCTURE ONLY — the oracle.

ctypes bindings for ``liboracle_attn.so`` (built from ``attn_ref.cpp``, a CPU
restatement of luisroayerdi/MLIR-FlashAttention lib/Attention/TilingPass.cpp:155-392)
plus the input quantisation the GPU path sees and an independent float64
two-pass softmax used to pin the restatement.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU legs import this
module; the product path never does.

Parity status: the reference has no numeric tests, golden vectors or runnable
CPU pipeline here (it needs MLIR/LLVM, absent), so the restatement is
"parity unpinned" against the reference itself; it is pinned against known
answers and the float64 softmax below (tests/test_oracle.py).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle_attn.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i64p = ctypes.POINTER(ctypes.c_int64)


def build(force: bool = False) -> str:
    """Compile liboracle_attn.so with the committed Makefile (g++ only)."""
    if force or not os.path.exists(_LIB_PATH) or (
        os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "attn_ref.cpp"))
    ):
        subprocess.run(["make", "-s", "-C", _HERE, "liboracle_attn.so"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.oracle_attn_fused_f32.restype = ctypes.c_int
        L.oracle_attn_fused_f32.argtypes = [
            _f32p, _f32p, _f32p, ctypes.c_float, _u8p, ctypes.c_int, _f32p, _f32p,
            ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
        ]
        L.oracle_attn_batched.restype = ctypes.c_int
        L.oracle_attn_batched.argtypes = [
            _f32p, _f32p, _f32p, _f32p, _f32p,
            ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
            ctypes.c_int64, ctypes.c_float, ctypes.c_int, _u8p, ctypes.c_int64, ctypes.c_int,
            _i64p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
        ]
        L.oracle_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(t) if a is not None else None


def attn_fused_f32(Q, K, V, scale, mask=None, causal=False, T=128):
    """The reference op on one slice: Q [Nq,D], K/V [Nk,D] float32.

    ``mask`` is a bool/uint8 [Nq,Nk] array (True = masked), as the op's i1
    operand.  Returns (O [Nq,D] float32, lse [Nq] float32).
    """
    Q = np.ascontiguousarray(Q, np.float32)
    K = np.ascontiguousarray(K, np.float32)
    V = np.ascontiguousarray(V, np.float32)
    Nq, D = Q.shape
    Nk = K.shape[0]
    O = np.empty((Nq, D), np.float32)
    lse = np.empty((Nq,), np.float32)
    m = None if mask is None else np.ascontiguousarray(mask, np.uint8)
    rc = lib().oracle_attn_fused_f32(
        _p(Q, _f32p), _p(K, _f32p), _p(V, _f32p), float(scale), _p(m, _u8p), int(bool(causal)),
        _p(O, _f32p), _p(lse, _f32p), Nq, Nk, D, T)
    if rc != 0:
        raise ValueError("oracle rejected the arguments")
    return O, lse


def attn_batched(Q, K, V, scale, causal=False, mask=None, T=128, nthreads=0, slices=None,
                 tile_offset=0, tile_stride=1, out=None, lse_out=None):
    """[B,Hq,Nq,D] / [B,Hkv,Nk,D] float32 arrays; grouped-query heads.

    ``mask`` (optional) is [B,Hq,Nq,Nk] uint8.  ``slices`` restricts the
    computation to the listed flat (b*Hq+h) slices and ``tile_offset`` /
    ``tile_stride`` to a subset of Q tiles (a bounded timing sample); rows not
    computed are left as they were in ``out``.
    """
    Q = np.ascontiguousarray(Q, np.float32)
    K = np.ascontiguousarray(K, np.float32)
    V = np.ascontiguousarray(V, np.float32)
    B, Hq, Nq, D = Q.shape
    Hkv, Nk = K.shape[1], K.shape[2]
    O = out if out is not None else np.zeros((B, Hq, Nq, D), np.float32)
    lse = lse_out if lse_out is not None else np.zeros((B, Hq, Nq), np.float32)
    m = None if mask is None else np.ascontiguousarray(mask, np.uint8)
    sl = None if slices is None else np.ascontiguousarray(slices, np.int64)
    rc = lib().oracle_attn_batched(
        _p(Q, _f32p), _p(K, _f32p), _p(V, _f32p), _p(O, _f32p), _p(lse, _f32p),
        B, Hq, Hkv, Nq, Nk, D, float(scale), int(bool(causal)), _p(m, _u8p), T, int(nthreads),
        _p(sl, _i64p), 0 if sl is None else len(sl), int(tile_offset), int(tile_stride))
    if rc != 0:
        raise ValueError("oracle rejected the arguments")
    return O, lse


def max_threads() -> int:
    return int(lib().oracle_max_threads())


# --------------------------------------------------------------------------
# Independent float64 two-pass softmax (pins the restatement; not a port).
# --------------------------------------------------------------------------
def naive_f64(Q, K, V, scale, mask=None, causal=False):
    Q = np.asarray(Q, np.float64)
    K = np.asarray(K, np.float64)
    V = np.asarray(V, np.float64)
    S = (Q @ K.T) * scale
    Nq, Nk = S.shape
    if causal:
        S = np.where(np.arange(Nk)[None, :] > np.arange(Nq)[:, None], -np.inf, S)
    if mask is not None:
        S = np.where(np.asarray(mask, bool), -np.inf, S)
    m = S.max(axis=1, keepdims=True)
    P = np.exp(S - m)
    l = P.sum(axis=1, keepdims=True)
    return P @ V / l, (m + np.log(l))[:, 0]


# --------------------------------------------------------------------------
# Input quantisation: the values the GPU kernels actually see.
# --------------------------------------------------------------------------
def round_bf16(x):
    """float32 -> nearest bfloat16 (ties to even) -> float32, as torch casts."""
    x = np.ascontiguousarray(x, np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = rounded.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), x, out).astype(np.float32)


def quant_e4m3(x):
    """Per-tensor scale amax/448, cast to float8-e4m3fn (RNE, saturating).

    Returns (codes uint8, descale float32, dequantised float32).
    """
    import ml_dtypes  # noqa: PLC0415

    x = np.asarray(x, np.float32)
    amax = float(np.max(np.abs(x))) if x.size else 0.0
    descale = np.float32(amax / 448.0 if amax > 0 else 1.0)
    y = np.clip(x / descale, -448.0, 448.0).astype(ml_dtypes.float8_e4m3fn)
    deq = y.astype(np.float32) * descale
    return y.view(np.uint8), descale, deq.astype(np.float32)
