"""attn_fwd_host_noalloc: the entry point that allocates no device memory.

It serves callers that cannot call cudaMalloc (host programs whose process
has its device memory reserved by another allocator, or that must avoid the
implicit synchronisation of cudaMalloc/cudaFree).  Its device scratch is a
static array of ATTN_NOALLOC_SCRATCH_BYTES inside libattnrt.so.  These tests
call it through the C ABI, twice in a row, and compare each result with the
existing host-memref entry point; an oversized call must be rejected.  The
file is named to be collected last.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 64 << 20  # ATTN_NOALLOC_SCRATCH_BYTES in include/attn_rt.h


def _host_desc(pkg, q, k, v, o, lse, causal, scale):
    d = pkg.AttnDesc()
    d.dtype, d.out_dtype = pkg.ATTN_BF16, pkg.ATTN_BF16
    d.mask_kind = pkg.MASK_CAUSAL if causal else pkg.MASK_NONE
    d.B, d.Hq, d.Nq, d.D = q.shape
    d.Hkv, d.Nk = k.shape[1], k.shape[2]
    for dst, t in ((d.q_stride, q), (d.k_stride, k), (d.v_stride, v), (d.o_stride, o)):
        dst[0], dst[1], dst[2] = t.stride(0), t.stride(1), t.stride(2)
    d.q, d.k, d.v, d.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr()
    d.lse = lse.data_ptr() if lse is not None else None
    d.scale = scale
    d.q_descale = d.k_descale = d.v_descale = 1.0
    return d


def _inputs(B, Hq, Hkv, N, D, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((B, Hq, N, D), generator=g).to(torch.bfloat16).pin_memory()
    k = torch.randn((B, Hkv, N, D), generator=g).to(torch.bfloat16).pin_memory()
    v = torch.randn((B, Hkv, N, D), generator=g).to(torch.bfloat16).pin_memory()
    return q, k, v


def _existing_entry(pkg, q, k, v, causal, scale):
    o = torch.empty(q.shape, dtype=torch.bfloat16).pin_memory()
    lse = torch.empty(q.shape[:3] + (1,), dtype=torch.float32).pin_memory()
    fn = (pkg.lib()._mlir_ciface_attn_fused_bf16_causal_4d if causal
          else pkg.lib()._mlir_ciface_attn_fused_bf16_nomask_4d)
    rc = fn(pkg.memref(q), pkg.memref(k), pkg.memref(v), scale, pkg.memref(o), pkg.memref(lse))
    assert rc == 0, pkg.last_error()
    return o, lse[..., 0]


def _noalloc(pkg, q, k, v, causal, scale):
    o = torch.full(q.shape, 7.0, dtype=torch.bfloat16)
    lse = torch.zeros(q.shape[:3], dtype=torch.float32)
    d = _host_desc(pkg, q, k, v, o, lse, causal, scale)
    L = pkg.lib()
    L.attn_fwd_host_noalloc.restype = ctypes.c_int
    L.attn_fwd_host_noalloc.argtypes = [ctypes.POINTER(pkg.AttnDesc), ctypes.c_void_p]
    stream = torch.cuda.current_stream().cuda_stream
    rc = L.attn_fwd_host_noalloc(ctypes.byref(d), stream)
    return rc, o, lse


def _rel(a, b):
    a, b = a.float().numpy(), b.float().numpy()
    return float(np.abs(a - b).max() / np.abs(b).max())


def test_two_calls_match_existing_entry(pkg):
    torch.cuda.init()
    # First call: one chunk.  Second call: 16 groups of ~4 MiB, more than one
    # chunk of the 64 MiB scratch, different data and the non-causal variant.
    cases = [(1, 4, 2, 1000, 128, True, 11), (2, 8, 8, 4096, 128, False, 12)]
    for B, Hq, Hkv, N, D, causal, seed in cases:
        q, k, v = _inputs(B, Hq, Hkv, N, D, seed)
        scale = 1.0 / D ** 0.5
        ref_o, ref_lse = _existing_entry(pkg, q, k, v, causal, scale)
        rc, o, lse = _noalloc(pkg, q, k, v, causal, scale)
        assert rc == 0, pkg.last_error()
        assert _rel(o, ref_o) <= 2e-2
        assert float((lse - ref_lse).abs().max()) <= 1e-3


def test_oversized_group_is_rejected(pkg):
    # One (batch, kv-head) group of N=65536, d=128 bf16 needs 4 x 16 MiB plus
    # LSE: more than the static scratch holds.
    N, D = 65536, 128
    q = torch.zeros((1, 1, N, D), dtype=torch.bfloat16)
    rc, _, _ = _noalloc(pkg, q, q, q, True, 0.1)
    assert rc == -2
    msg = pkg.last_error()
    assert "static scratch holds" in msg and str(SCRATCH_BYTES - 256) in msg
