"""Host-side mirror of the reference's ``attention.fused`` op on B200.

The reference (luisroayerdi/MLIR-FlashAttention) exposes one operation,

    attention.fused ins(%Q, %K, %V) scale(%s) [mask(%m)] outs(%O)

(include/Attention/AttentionOps.td:20-54): ``O = softmax(Q·Kᵀ·scale, masked ->
-inf)·V`` written in place into ``O``.  :func:`fused` takes the same operands,
in the same order and with the same meaning, as torch tensors on a CUDA device
and runs them through ``libattnrt.so`` (``include/attn_rt.h``), whose sm_100a
kernels replace the reference's CPU lowering (lib/Attention/TilingPass.cpp).
Shape errors raise :class:`VerifyError` with the reference verifier's messages
(lib/Attention/AttentionOps.cpp:39-56).  There is no CPU fallback: if the
library is missing or no sm_100 device is present, calls raise.
"""
from __future__ import annotations

import ctypes
import os

__all__ = [
    "AttentionError", "VerifyError", "fused", "classify_mask", "lib", "launch_count",
    "check_status", "AttnDesc", "AttnMemRef2D", "AttnMemRef4D", "memref", "shard_slices",
    "ATTN_F32", "ATTN_BF16", "ATTN_E4M3", "ATTN_F16", "MASK_NONE", "MASK_CAUSAL", "MASK_DENSE",
]

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libattnrt.so")

ATTN_F32, ATTN_BF16, ATTN_E4M3, ATTN_F16 = 0, 1, 2, 3
MASK_NONE, MASK_CAUSAL, MASK_DENSE = 0, 1, 2

STATUS = {
    0: "ok", -1: "invalid argument", -2: "shape mismatch", -3: "unsupported stride",
    -4: "unsupported dtype", -5: "misaligned pointer or stride", -6: "CUDA error",
    -7: "device wait timed out", -8: "unsupported variant", -9: "no sm_100 device",
}


class AttentionError(RuntimeError):
    """A non-zero status from the runtime (``ATTN_ERR_*``)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"attention.fused: {message} [{STATUS.get(code, code)}]")
        self.code = code


class VerifyError(ValueError):
    """The op's verifier rejected the operands (AttentionOps.cpp:33-59)."""


class AttnDesc(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int32), ("out_dtype", ctypes.c_int32),
        ("mask_kind", ctypes.c_int32), ("flags", ctypes.c_int32),
        ("B", ctypes.c_int64), ("Hq", ctypes.c_int64), ("Hkv", ctypes.c_int64),
        ("Nq", ctypes.c_int64), ("Nk", ctypes.c_int64), ("D", ctypes.c_int64),
        ("q_stride", ctypes.c_int64 * 3), ("k_stride", ctypes.c_int64 * 3),
        ("v_stride", ctypes.c_int64 * 3), ("o_stride", ctypes.c_int64 * 3),
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
        ("o", ctypes.c_void_p), ("lse", ctypes.c_void_p), ("mask", ctypes.c_void_p),
        ("mask_stride", ctypes.c_int64 * 3),
        ("scale", ctypes.c_float), ("q_descale", ctypes.c_float),
        ("k_descale", ctypes.c_float), ("v_descale", ctypes.c_float),
        ("status", ctypes.c_void_p),
        ("q_descale_blocks", ctypes.c_void_p), ("k_descale_blocks", ctypes.c_void_p),
        ("v_descale_heads", ctypes.c_void_p),
    ]


class AttnMemRef2D(ctypes.Structure):
    _fields_ = [("allocated", ctypes.c_void_p), ("aligned", ctypes.c_void_p),
                ("offset", ctypes.c_int64), ("sizes", ctypes.c_int64 * 2),
                ("strides", ctypes.c_int64 * 2)]


class AttnMemRef4D(ctypes.Structure):
    _fields_ = [("allocated", ctypes.c_void_p), ("aligned", ctypes.c_void_p),
                ("offset", ctypes.c_int64), ("sizes", ctypes.c_int64 * 4),
                ("strides", ctypes.c_int64 * 4)]


_lib = None


def lib():
    """Load libattnrt.so (raises if it was not built — there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"libattnrt.so not found at {LIB_PATH}; build it with __graft_entry__.build()")
        L = ctypes.CDLL(LIB_PATH)
        L.attn_fwd.restype = ctypes.c_int
        L.attn_fwd.argtypes = [ctypes.POINTER(AttnDesc), ctypes.c_void_p]
        L.attn_rt_init.restype = ctypes.c_int
        L.attn_rt_init.argtypes = [ctypes.c_int]
        L.attn_rt_causal_split.restype = ctypes.c_int
        L.attn_rt_causal_split.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                           ctypes.c_int]
        L.attn_rt_check_status.restype = ctypes.c_int
        L.attn_rt_check_status.argtypes = [ctypes.c_int, ctypes.c_void_p]
        L.attn_rt_status_string.restype = ctypes.c_char_p
        L.attn_rt_status_string.argtypes = [ctypes.c_int]
        L.attn_rt_last_error.restype = ctypes.c_char_p
        L.attn_rt_last_error.argtypes = []
        L.attn_rt_version.restype = ctypes.c_int
        L.attn_rt_launch_count.restype = ctypes.c_int64
        L.attn_rt_probe_timeout.restype = ctypes.c_int
        L.attn_rt_probe_timeout.argtypes = [ctypes.c_int64]
        L.attn_rt_alloc.restype = ctypes.c_int
        L.attn_rt_alloc.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_size_t]
        L.attn_rt_free.restype = ctypes.c_int
        L.attn_rt_free.argtypes = [ctypes.c_void_p]
        L.attn_rt_copy.restype = ctypes.c_int
        L.attn_rt_copy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                   ctypes.c_void_p]
        m2, m4 = ctypes.POINTER(AttnMemRef2D), ctypes.POINTER(AttnMemRef4D)
        f = ctypes.c_float
        for name in ("nomask", "causal"):
            fn = getattr(L, f"_mlir_ciface_attn_fused_f32_{name}")
            fn.restype, fn.argtypes = ctypes.c_int32, [m2, m2, m2, f, m2]
            fn = getattr(L, f"_mlir_ciface_attn_fused_f32_{name}_4d")
            fn.restype, fn.argtypes = ctypes.c_int32, [m4, m4, m4, f, m4]
            fn = getattr(L, f"_mlir_ciface_attn_fused_bf16_{name}_4d")
            fn.restype, fn.argtypes = ctypes.c_int32, [m4, m4, m4, f, m4, m4]
            fn = getattr(L, f"_mlir_ciface_attn_fused_f16_{name}_4d")
            fn.restype, fn.argtypes = ctypes.c_int32, [m4, m4, m4, f, m4, m4]
            fn = getattr(L, f"_mlir_ciface_attn_fused_e4m3_{name}_4d")
            fn.restype, fn.argtypes = ctypes.c_int32, [m4, m4, m4, f, f, f, f, m4, m4]
        L._mlir_ciface_attn_fused_bf16_mask_4d.restype = ctypes.c_int32
        L._mlir_ciface_attn_fused_bf16_mask_4d.argtypes = [m4, m4, m4, f, m4, m4, m4]
        L._mlir_ciface_attn_fused_bf16_mask2d_4d.restype = ctypes.c_int32
        L._mlir_ciface_attn_fused_bf16_mask2d_4d.argtypes = [m4, m4, m4, f, m2, m4, m4]
        L._mlir_ciface_attn_fused_f32_mask.restype = ctypes.c_int32
        L._mlir_ciface_attn_fused_f32_mask.argtypes = [m2, m2, m2, f, m2, m2]
        _lib = L
    return _lib


def last_error() -> str:
    return lib().attn_rt_last_error().decode()


def launch_count() -> int:
    return int(lib().attn_rt_launch_count())


def _raise(code: int):
    if code != 0:
        raise AttentionError(code, last_error() or STATUS.get(code, "error"))


def check_status(device: int = 0, stream=None):
    """Synchronise and raise if a kernel recorded an error (e.g. a timeout)."""
    _raise(lib().attn_rt_check_status(device, _stream_ptr(stream)))


def _stream_ptr(stream):
    if stream is None:
        import torch  # noqa: PLC0415
        return torch.cuda.current_stream().cuda_stream
    return getattr(stream, "cuda_stream", stream)


def _dtype_code(t):
    import torch  # noqa: PLC0415
    if t.dtype == torch.float32:
        return ATTN_F32
    if t.dtype == torch.bfloat16:
        return ATTN_BF16
    if t.dtype == torch.float16:
        return ATTN_F16
    if t.dtype in (torch.float8_e4m3fn, torch.uint8):
        return ATTN_E4M3
    raise VerifyError(f"unsupported element type {t.dtype}")


def _as4(t, name, seq, dim):
    if t.dim() == 2:
        return t.unsqueeze(0).unsqueeze(0)
    if t.dim() == 4:
        return t
    raise VerifyError(f"{name} must be rank-2 [{seq}, {dim}] or rank-4 [batch, heads, {seq}, {dim}]")


def classify_mask(mask) -> int:
    """Classify an i1 [.., Nq, Nk] mask the way the lowering pass does.

    Returns MASK_NONE if nothing is masked, MASK_CAUSAL if it is exactly
    ``j > i`` for every slice, else MASK_DENSE.
    """
    import torch  # noqa: PLC0415
    m = mask.bool()
    if not bool(m.any()):
        return MASK_NONE
    nq, nk = m.shape[-2], m.shape[-1]
    causal = torch.ones(nq, nk, dtype=torch.bool, device=m.device).triu_(1)
    if bool((m == causal).all()):
        return MASK_CAUSAL
    return MASK_DENSE


def fused(Q, K, V, scale, mask=None, output=None, *, causal=False, lse=None,
          q_descale=1.0, k_descale=1.0, v_descale=1.0, stream=None, sync_check=False,
          classify=True):
    """Run ``attention.fused ins(Q, K, V) scale(scale) [mask(mask)] outs(output)``.

    Q: [Nq, D] or [B, Hq, Nq, D]; K, V: [Nk, D] or [B, Hkv, Nk, D] (Hq a
    multiple of Hkv: grouped-query heads).  f32 / bf16 / float8_e4m3fn inputs,
    head_dim unit-stride.  ``mask`` is an i1 (bool) tensor [Nq, Nk] (or
    broadcastable [B, Hq, Nq, Nk]) with True = masked; it is classified as
    none / causal / dense like the lowering pass does.  ``causal=True`` selects
    the causal specialisation without a mask tensor.  ``output`` is written in
    place and returned (allocated if None: f32 for f32 inputs, else bf16).
    ``lse`` (optional, f32 [B, Hq, Nq] or [Nq]) receives the natural-log
    log-sum-exp of each row.  The launch is asynchronous on ``stream``.

    e4m3 dequantisation factors are per tensor (Python floats) or per block
    (f32 CUDA tensors): ``q_descale`` [B, Hq, ceil(Nq/128)] (one per 128-row
    block of Q), ``k_descale`` [B, Hkv, ceil(Nk/128)], ``v_descale`` [B, Hkv].
    ``classify=False`` runs a given mask on the dense-mask kernel as it is
    (no check for the causal or empty pattern).
    """
    import torch  # noqa: PLC0415
    q4 = _as4(Q, "Q", "seq_q", "head_dim")
    k4 = _as4(K, "K", "seq_k", "head_dim")
    v4 = _as4(V, "V", "seq_k", "head_dim")
    B, Hq, Nq, D = q4.shape
    if k4.shape[3] != D:
        raise VerifyError("K head_dim must equal Q head_dim")
    if v4.shape[2] != k4.shape[2]:
        raise VerifyError("V seq_len must equal K seq_len")
    if v4.shape[3] != D:
        raise VerifyError("V head_dim must equal Q head_dim")
    if k4.shape[0] != B or v4.shape[0] != B or v4.shape[1] != k4.shape[1]:
        raise VerifyError("batch/head extents of K and V must match Q")
    dt = _dtype_code(Q)
    if _dtype_code(K) != dt or _dtype_code(V) != dt:
        raise VerifyError("Q, K and V must share one element type")
    if output is None:
        odt = {ATTN_F32: torch.float32, ATTN_F16: torch.float16}.get(dt, torch.bfloat16)
        output = torch.empty(Q.shape, dtype=odt, device=Q.device)
    o4 = _as4(output, "output", "seq_q", "head_dim")
    if o4.shape[2] != Nq:
        raise VerifyError("output seq_q must equal Q seq_q")
    if o4.shape[3] != D:
        raise VerifyError("output head_dim must equal Q head_dim")
    if o4.shape[0] != B or o4.shape[1] != Hq:
        raise VerifyError("output batch/head extents must equal Q")
    mask_kind = MASK_CAUSAL if causal else MASK_NONE
    m4 = None
    if mask is not None:
        if mask.shape[-2:] != (Nq, k4.shape[2]):
            raise VerifyError("mask must be [seq_q, seq_k]")
        kind = classify_mask(mask) if classify else MASK_DENSE
        if causal and kind not in (MASK_NONE, MASK_CAUSAL):
            mask_kind = MASK_DENSE
        elif not causal:
            mask_kind = kind
        if mask_kind == MASK_DENSE:
            m4 = mask.to(torch.uint8).expand(B, Hq, Nq, k4.shape[2])
    for t, n in ((q4, "Q"), (k4, "K"), (v4, "V"), (o4, "output")):
        if t.stride(3) != 1:
            raise VerifyError(f"{n} head_dim must be unit-stride")
        if not t.is_cuda:
            raise VerifyError(f"{n} must be a CUDA tensor")
    d = AttnDesc()
    d.dtype = dt
    d.out_dtype = {torch.float32: ATTN_F32, torch.float16: ATTN_F16}.get(output.dtype, ATTN_BF16)
    d.mask_kind = mask_kind
    d.B, d.Hq, d.Hkv, d.Nq, d.Nk, d.D = B, Hq, k4.shape[1], Nq, k4.shape[2], D
    for dst, t in ((d.q_stride, q4), (d.k_stride, k4), (d.v_stride, v4), (d.o_stride, o4)):
        dst[0], dst[1], dst[2] = t.stride(0), t.stride(1), t.stride(2)
    d.q, d.k, d.v, d.o = q4.data_ptr(), k4.data_ptr(), v4.data_ptr(), o4.data_ptr()
    if lse is not None:
        if lse.dtype != torch.float32 or not lse.is_contiguous() or lse.numel() != B * Hq * Nq:
            raise VerifyError("lse must be a contiguous f32 tensor of B*Hq*Nq elements")
        d.lse = lse.data_ptr()
    if m4 is not None:
        d.mask = m4.data_ptr()
        d.mask_stride[0], d.mask_stride[1], d.mask_stride[2] = m4.stride(0), m4.stride(1), m4.stride(2)
    d.scale = float(scale)
    Hkv, Nk = k4.shape[1], k4.shape[2]
    shapes = {"q_descale": (B, Hq, -(-Nq // 128)), "k_descale": (B, Hkv, -(-Nk // 128)),
              "v_descale": (B, Hkv)}
    for name, val, field in (("q_descale", q_descale, "q_descale_blocks"),
                             ("k_descale", k_descale, "k_descale_blocks"),
                             ("v_descale", v_descale, "v_descale_heads")):
        if isinstance(val, torch.Tensor):
            if dt != ATTN_E4M3:
                raise VerifyError(f"per-block {name} applies to float8_e4m3fn inputs")
            want = shapes[name]
            if Q.dim() == 2:
                want = want[2:] if name != "v_descale" else ()
            if (val.dtype != torch.float32 or not val.is_cuda or not val.is_contiguous()
                    or tuple(val.shape) != tuple(want)):
                raise VerifyError(f"per-block {name} must be a contiguous f32 CUDA tensor of "
                                  f"shape {list(want)}")
            setattr(d, field, val.data_ptr())
            setattr(d, name, 1.0)
        else:
            setattr(d, name, float(val))
    with torch.cuda.device(Q.device):
        _raise(lib().attn_fwd(ctypes.byref(d), _stream_ptr(stream)))
        if sync_check:
            check_status(Q.device.index or 0, stream)
    return output


def memref(t, rank=None):
    """MLIR memref descriptor (rank 2 or 4) viewing tensor ``t`` (host or device)."""
    r = t.dim() if rank is None else rank
    cls = AttnMemRef2D if r == 2 else AttnMemRef4D
    m = cls()
    m.allocated = m.aligned = t.data_ptr()
    m.offset = 0
    for i in range(r):
        m.sizes[i] = t.shape[i]
        m.strides[i] = t.stride(i)
    return m


def shard_slices(n_slices: int, world: int, rank: int):
    """Contiguous block of flat (batch, head) slices owned by ``rank``."""
    base, extra = divmod(n_slices, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)
