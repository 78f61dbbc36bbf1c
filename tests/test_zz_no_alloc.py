"""attn_fwd_host_noalloc: the entry point that allocates no device memory.

It serves callers that cannot call cudaMalloc (host programs whose process
has its device memory reserved by another allocator, or that must avoid the
implicit synchronisation of cudaMalloc/cudaFree).  Its device scratch is a
static array of ATTN_NOALLOC_SCRATCH_BYTES inside libattnrt.so.  These tests
call it through the C ABI, twice in a row, and compare each result bit for
bit with the existing host-memref entry points (both run the same kernel on
the same values); they also check that a call leaves free device memory
unchanged, and that oversized calls and device pointers are refused.  The
file is named to be collected last.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 64 << 20  # ATTN_NOALLOC_SCRATCH_BYTES in include/attn_rt.h


def _desc(pkg, q, k, v, o, lse, causal, scale, dtype, out_dtype, descales=(1.0, 1.0, 1.0)):
    d = pkg.AttnDesc()
    d.dtype, d.out_dtype = dtype, out_dtype
    d.mask_kind = pkg.MASK_CAUSAL if causal else pkg.MASK_NONE
    d.B, d.Hq, d.Nq, d.D = q.shape
    d.Hkv, d.Nk = k.shape[1], k.shape[2]
    for dst, t in ((d.q_stride, q), (d.k_stride, k), (d.v_stride, v), (d.o_stride, o)):
        dst[0], dst[1], dst[2] = t.stride(0), t.stride(1), t.stride(2)
    d.q, d.k, d.v, d.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr()
    d.lse = lse.data_ptr() if lse is not None else None
    d.scale = scale
    d.q_descale, d.k_descale, d.v_descale = descales
    return d


def _call_noalloc(pkg, d):
    L = pkg.lib()
    L.attn_fwd_host_noalloc.restype = ctypes.c_int
    L.attn_fwd_host_noalloc.argtypes = [ctypes.POINTER(pkg.AttnDesc), ctypes.c_void_p]
    return L.attn_fwd_host_noalloc(ctypes.byref(d), torch.cuda.current_stream().cuda_stream)


def _bf16_inputs(B, Hq, Hkv, N, D, seed, pinned=True):
    g = torch.Generator().manual_seed(seed)
    ts = [torch.randn((B, h, N, D), generator=g).to(torch.bfloat16) for h in (Hq, Hkv, Hkv)]
    return [t.pin_memory() for t in ts] if pinned else ts


def _bf16_memref(pkg, q, k, v, causal, scale):
    o = torch.empty(q.shape, dtype=torch.bfloat16).pin_memory()
    lse = torch.empty(q.shape[:3] + (1,), dtype=torch.float32).pin_memory()
    fn = (pkg.lib()._mlir_ciface_attn_fused_bf16_causal_4d if causal
          else pkg.lib()._mlir_ciface_attn_fused_bf16_nomask_4d)
    rc = fn(pkg.memref(q), pkg.memref(k), pkg.memref(v), scale, pkg.memref(o), pkg.memref(lse))
    assert rc == 0, pkg.last_error()
    return o, lse[..., 0]


def _bf16_noalloc(pkg, q, k, v, causal, scale, pinned_out=False):
    o = torch.full(q.shape, 7.0, dtype=torch.bfloat16)
    lse = torch.zeros(q.shape[:3], dtype=torch.float32)
    if pinned_out:
        o, lse = o.pin_memory(), lse.pin_memory()
    d = _desc(pkg, q, k, v, o, lse, causal, scale, pkg.ATTN_BF16, pkg.ATTN_BF16)
    return _call_noalloc(pkg, d), o, lse


def test_two_calls_bitwise_equal_to_memref_entry(pkg):
    torch.cuda.init()
    # First call: one chunk.  Second call: 16 groups of ~4 MiB, more than one
    # chunk of the 64 MiB scratch, different data and the non-causal variant.
    cases = [(1, 4, 2, 1000, 128, True, 11), (2, 8, 8, 4096, 128, False, 12)]
    for B, Hq, Hkv, N, D, causal, seed in cases:
        q, k, v = _bf16_inputs(B, Hq, Hkv, N, D, seed)
        scale = 1.0 / D ** 0.5
        ref_o, ref_lse = _bf16_memref(pkg, q, k, v, causal, scale)
        rc, o, lse = _bf16_noalloc(pkg, q, k, v, causal, scale)
        assert rc == 0, pkg.last_error()
        assert torch.equal(o, ref_o)
        assert torch.equal(lse, ref_lse)


def test_second_call_allocates_no_device_memory(pkg):
    """Free device memory is the same before and after a call (the call after
    the first one, which may load kernel code lazily)."""
    q, k, v = _bf16_inputs(2, 4, 4, 2048, 128, 21)
    rc, o1, _ = _bf16_noalloc(pkg, q, k, v, True, 0.09, pinned_out=True)
    assert rc == 0, pkg.last_error()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    rc, o2, _ = _bf16_noalloc(pkg, q, k, v, True, 0.09, pinned_out=True)
    assert rc == 0, pkg.last_error()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert torch.equal(o1, o2)


def test_pageable_buffers_and_odd_host_offset(pkg):
    """Pageable (unpinned) host buffers, and operands viewed at an element
    offset that is not 16-byte aligned: the call stages every chunk into its
    own aligned regions, so neither matters."""
    q, k, v = _bf16_inputs(1, 2, 2, 640, 64, 31, pinned=False)
    ref_o, ref_lse = _bf16_memref(pkg, q.pin_memory(), k.pin_memory(), v.pin_memory(), True, 0.125)
    for _ in range(2):
        rc, o, lse = _bf16_noalloc(pkg, q, k, v, True, 0.125)
        assert rc == 0, pkg.last_error()
        assert torch.equal(o, ref_o) and torch.equal(lse, ref_lse)
    # Q, K, V each one element past the start of a larger buffer (2 bytes:
    # not 16-byte aligned), with a padded row stride.
    def shifted(t):
        buf = torch.zeros(t.numel() + t.shape[0] * t.shape[1] * t.shape[2] * 8 + 1,
                          dtype=t.dtype)
        B, H, N, D = t.shape
        view = buf[1:1 + B * H * N * (D + 8)].view(B, H, N, D + 8)[..., :D]
        view.copy_(t)
        return view
    qs, ks, vs = shifted(q), shifted(k), shifted(v)
    assert qs.data_ptr() % 16 != 0
    rc, o, lse = _bf16_noalloc(pkg, qs, ks, vs, True, 0.125)
    assert rc == 0, pkg.last_error()
    assert torch.equal(o, ref_o) and torch.equal(lse, ref_lse)


def test_f32_two_calls_equal_memref_entry(pkg):
    g = torch.Generator().manual_seed(41)
    q, k, v = (torch.randn((2, 2, 300, 64), generator=g) for _ in range(3))
    ref = torch.empty_like(q)
    rc = pkg.lib()._mlir_ciface_attn_fused_f32_causal_4d(
        pkg.memref(q), pkg.memref(k), pkg.memref(v), 0.125, pkg.memref(ref))
    assert rc == 0, pkg.last_error()
    for _ in range(2):
        o = torch.full_like(q, 3.0)
        d = _desc(pkg, q, k, v, o, None, True, 0.125, pkg.ATTN_F32, pkg.ATTN_F32)
        assert _call_noalloc(pkg, d) == 0, pkg.last_error()
        assert torch.equal(o, ref)


def test_e4m3_without_lse_two_calls_equal_memref_entry(pkg, wl):
    w = wl.WORKLOADS["c5"]
    inp = wl.make_inputs(w, B=2, Hq=8, N=384)
    q, k, v = (torch.from_numpy(a) for a in (inp.q, inp.k, inp.v))  # uint8 e4m3 codes
    qd, kd, vd = inp.descale
    ref = torch.empty(q.shape, dtype=torch.bfloat16)
    no_lse = torch.empty((0, 0, 0, 1), dtype=torch.float32)
    rc = pkg.lib()._mlir_ciface_attn_fused_e4m3_causal_4d(
        pkg.memref(q), pkg.memref(k), pkg.memref(v), w.scale, qd, kd, vd, pkg.memref(ref),
        pkg.memref(no_lse))
    assert rc == 0, pkg.last_error()
    for _ in range(2):
        o = torch.full(q.shape, 5.0, dtype=torch.bfloat16)
        d = _desc(pkg, q, k, v, o, None, True, w.scale, pkg.ATTN_E4M3, pkg.ATTN_BF16,
                  (qd, kd, vd))
        assert _call_noalloc(pkg, d) == 0, pkg.last_error()
        assert torch.equal(o, ref)


def test_no_keys_gives_nan_rows_and_minus_inf_lse(pkg):
    q = torch.randn((1, 2, 5, 64)).to(torch.bfloat16)
    kv = torch.zeros((1, 2, 0, 64), dtype=torch.bfloat16)
    for _ in range(2):
        o = torch.zeros(q.shape, dtype=torch.bfloat16)
        lse = torch.zeros(q.shape[:3], dtype=torch.float32)
        d = _desc(pkg, q, kv, kv, o, lse, False, 0.1, pkg.ATTN_BF16, pkg.ATTN_BF16)
        assert _call_noalloc(pkg, d) == 0, pkg.last_error()
        assert torch.isnan(o.float()).all()
        assert torch.isneginf(lse).all()


def test_device_pointers_are_refused(pkg):
    q = torch.zeros((1, 1, 128, 128), dtype=torch.bfloat16, device="cuda")
    o = torch.zeros((1, 1, 128, 128), dtype=torch.bfloat16)
    d = _desc(pkg, q, q, q, o, None, True, 0.1, pkg.ATTN_BF16, pkg.ATTN_BF16)
    assert _call_noalloc(pkg, d) == -1
    assert "attn_fwd" in pkg.last_error()


def test_oversized_group_is_rejected(pkg):
    # One (batch, kv-head) group of N=65536, d=128 bf16 needs 4 x 16 MiB plus
    # LSE: more than the static scratch holds.
    N, D = 65536, 128
    q = torch.zeros((1, 1, N, D), dtype=torch.bfloat16)
    rc, _, _ = _bf16_noalloc(pkg, q, q, q, True, 0.1)
    assert rc == -2
    msg = pkg.last_error()
    assert "static scratch holds" in msg and str(SCRATCH_BYTES - 256) in msg
