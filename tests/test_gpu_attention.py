"""GPU parity tests: the sm_100a kernels (through the C ABI) against the oracle.

Tolerances: max|O - O_oracle| / max|O_oracle| <= 1e-4 (f32), 2e-2 (bf16),
6e-2 (e4m3); LSE max abs difference <= 1e-3 (1e-5 for f32).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _rel(got, ref):
    return float(np.abs(got - ref).max() / np.abs(ref).max())


def _run_pkg(pkg, wl, w, inp, causal, lse=True, out_f32=False):
    q, k, v = wl.to_device(inp, w)
    B, Hq, N, D = inp.q.shape
    out = None
    if out_f32:
        out = torch.empty((B, Hq, N, D), dtype=torch.float32, device="cuda")
    L = torch.empty((B, Hq, N), dtype=torch.float32, device="cuda") if lse else None
    qd, kd, vd = inp.descale
    out = pkg.fused(q, k, v, w.scale, output=out, causal=causal, lse=L,
                    q_descale=qd, k_descale=kd, v_descale=vd)
    pkg.check_status(0)
    return out.float().cpu().numpy(), (L.cpu().numpy() if lse else None)


def _ref(oracle, inp, w, causal, **kw):
    return oracle.attn_batched(inp.qf, inp.kf, inp.vf, w.scale, causal=causal, **kw)


def test_f32_reference_config(pkg, wl, oracle):
    """c1: the reference op's own form, f32 causal 128x64, scale 1/8."""
    w = wl.WORKLOADS["c1"]
    inp = wl.make_inputs(w)
    got, lse = _run_pkg(pkg, wl, w, inp, causal=True)
    ref, ref_lse = _ref(oracle, inp, w, True)
    assert _rel(got, ref) <= 1e-4
    assert np.abs(lse - ref_lse).max() <= 1e-5


def test_f32_dense_mask_rank2_memref(pkg, wl, oracle):
    """The rank-2 f32 memref entry with an explicit i1 mask, host buffers."""
    rng = np.random.default_rng(11)
    Nq, Nk, D = 96, 160, 32
    Q, K, V = (rng.standard_normal((n, D)).astype(np.float32) for n in (Nq, Nk, Nk))
    M = rng.random((Nq, Nk)) < 0.3
    M[:, 0] = False
    M[[3, 40], :128] = True  # masked over the whole first KV tile, visible later
    M[60, :] = True          # masked everywhere
    ref, _ = oracle.attn_fused_f32(Q, K, V, 0.2, mask=M)
    tq, tk, tv = (torch.from_numpy(a) for a in (Q, K, V))
    tm = torch.from_numpy(M.astype(np.uint8))
    to = torch.zeros((Nq, D), dtype=torch.float32)
    L = pkg.lib()
    rc = L._mlir_ciface_attn_fused_f32_mask(pkg.memref(tq), pkg.memref(tk), pkg.memref(tv), 0.2,
                                            pkg.memref(tm), pkg.memref(to))
    assert rc == 0, pkg.last_error()
    got = to.numpy()
    # The reference's loop yields NaN for rows masked over their first KV tile.
    nan_rows = np.isnan(ref).all(axis=1)
    assert nan_rows.tolist() == [r in (3, 40, 60) for r in range(Nq)]
    assert (np.isnan(got) == np.isnan(ref)).all()
    assert _rel(got[~nan_rows], ref[~nan_rows]) <= 1e-4


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("N", [128, 256, 384, 1000])
def test_bf16_parity(pkg, wl, oracle, D, causal, N):
    base = wl.WORKLOADS["c2"] if D == 64 else wl.WORKLOADS["c3"]
    w = wl.Workload("t", "bf16", 2, 3, 3, N, D, causal, seed=100 + N + D)
    inp = wl.make_inputs(w)
    got, lse = _run_pkg(pkg, wl, w, inp, causal)
    ref, ref_lse = _ref(oracle, inp, w, causal)
    assert np.isfinite(got).all()
    assert _rel(got, ref) <= base.tol
    assert np.abs(lse - ref_lse).max() <= 1e-3


def test_bf16_gqa_f32_output(pkg, wl, oracle):
    w = wl.Workload("t", "bf16", 1, 8, 2, 512, 128, True, seed=7)
    inp = wl.make_inputs(w)
    got, _ = _run_pkg(pkg, wl, w, inp, True, out_f32=True)
    ref, _ = _ref(oracle, inp, w, True)
    assert _rel(got, ref) <= 2e-2


def test_c2_full_config(pkg, wl, oracle):
    """bf16 causal B=8 H=16 N=1024 D=64 over every slice."""
    w = wl.WORKLOADS["c2"]
    inp = wl.make_inputs(w)
    got, lse = _run_pkg(pkg, wl, w, inp, True)
    ref, ref_lse = _ref(oracle, inp, w, True)
    assert _rel(got, ref) <= w.tol
    assert np.abs(lse - ref_lse).max() <= 1e-3


def test_e4m3_gqa_parity(pkg, wl, oracle):
    """c5 shape family: e4m3 causal GQA (group 4), reduced to B=2, Hq=8, N=512."""
    w = wl.WORKLOADS["c5"]
    inp = wl.make_inputs(w, B=2, Hq=8, N=512)
    got, lse = _run_pkg(pkg, wl, w, inp, True)
    ref, ref_lse = _ref(oracle, inp, w, True)
    assert _rel(got, ref) <= w.tol
    assert np.abs(lse - ref_lse).max() <= 1e-2


@pytest.mark.parametrize("causal,nq,nk", [(True, 512, 512), (False, 300, 520), (True, 640, 384)])
def test_e4m3_block_descales(pkg, wl, oracle, causal, nq, nk):
    """e4m3 GQA with per-block Q/K and per-head V dequantisation factors.

    Block magnitudes spread over two decades, so a factor applied to the wrong
    block or head shows up as a large error; checked per (batch, head) slice.
    """
    rng = np.random.default_rng(11)
    B, Hq, Hkv, D = 2, 8, 2, 128

    def spread(n, H):
        f = 10.0 ** rng.uniform(-1.0, 1.0, size=(B, H, -(-n // 128)))
        return np.repeat(f, 128, axis=2)[:, :, :n, None].astype(np.float32)

    q = rng.standard_normal((B, Hq, nq, D)).astype(np.float32) * spread(nq, Hq)
    k = rng.standard_normal((B, Hkv, nk, D)).astype(np.float32) * spread(nk, Hkv)
    v = rng.standard_normal((B, Hkv, nk, D)).astype(np.float32) * (
        10.0 ** rng.uniform(-1.0, 1.0, size=(B, Hkv, 1, 1))).astype(np.float32)
    q8, qd, qf = wl.quant_e4m3_blocks(q)
    k8, kd, kf = wl.quant_e4m3_blocks(k)
    v8, vd, vf = wl.quant_e4m3_heads(v)
    scale = 1.0 / np.sqrt(D)
    dev = [torch.from_numpy(a).cuda() for a in (q8, k8, v8, qd, kd, vd)]
    L = torch.empty((B, Hq, nq), dtype=torch.float32, device="cuda")
    out = pkg.fused(dev[0], dev[1], dev[2], scale, causal=causal, lse=L,
                    q_descale=dev[3], k_descale=dev[4], v_descale=dev[5])
    pkg.check_status(0)
    got = out.float().cpu().numpy()
    ref, ref_lse = oracle.attn_batched(qf, kf, vf, scale, causal=causal)
    for b in range(B):
        for h in range(Hq):
            assert _rel(got[b, h], ref[b, h]) <= 6e-2, (b, h)
    lse = L.cpu().numpy()
    assert (np.abs(lse - ref_lse) <= 1e-2 + 1e-4 * np.abs(ref_lse)).all()
    with pytest.raises(pkg.VerifyError):
        bf = torch.zeros((1, 1, 128, 128), dtype=torch.bfloat16, device="cuda")
        pkg.fused(bf, bf, bf, 0.1, q_descale=torch.ones((1, 1, 1), device="cuda"))


@pytest.mark.parametrize("dtype,D", [("bf16", 128), ("bf16", 64), ("e4m3", 128)])
@pytest.mark.parametrize("causal", [True, False])
def test_running_max_rescales(pkg, wl, oracle, dtype, D, causal):
    """Scores that grow along the keys (each KV tile's row max 15-35 log2
    units above the previous one), so the running max moves past the rescale
    threshold at nearly every step: O is rescaled in TMEM again and again
    (the e4m3 kernel waits for the previous P·V GEMM only then)."""
    rng = np.random.default_rng(80 + D + (dtype == "e4m3"))
    B, H, N = 1, 2, 640
    u = rng.standard_normal(D).astype(np.float32)
    u /= np.linalg.norm(u)
    ramp = np.linspace(0.0, 4.0, N, dtype=np.float32)
    q = (200.0 * u + rng.standard_normal((B, H, N, D))).astype(np.float32)
    k = (ramp[:, None] * u + 0.3 * rng.standard_normal((B, H, N, D))).astype(np.float32)
    v = rng.standard_normal((B, H, N, D)).astype(np.float32)
    scale = 1.0 / np.sqrt(D)
    L = torch.empty((B, H, N), dtype=torch.float32, device="cuda")
    if dtype == "e4m3":
        (q8, qd, qf), (k8, kd, kf), (v8, vd, vf) = (wl.quant_e4m3(a) for a in (q, k, v))
        dev = [torch.from_numpy(a).view(torch.float8_e4m3fn).cuda() for a in (q8, k8, v8)]
        out = pkg.fused(*dev, scale, causal=causal, lse=L, q_descale=qd, k_descale=kd,
                        v_descale=vd)
        tol, ltol = 6e-2, 1e-2
    else:
        qf, kf, vf = (wl.round_bf16(a) for a in (q, k, v))
        dev = [torch.from_numpy(a).to(torch.bfloat16).cuda() for a in (qf, kf, vf)]
        out = pkg.fused(*dev, scale, causal=causal, lse=L)
        tol, ltol = 2e-2, 1e-3
    pkg.check_status(0)
    ref, ref_lse = oracle.attn_batched(qf, kf, vf, scale, causal=causal)
    got = out.float().cpu().numpy()
    for h in range(H):
        assert _rel(got[0, h], ref[0, h]) <= tol, h
    lse = L.cpu().numpy()
    assert (np.abs(lse - ref_lse) <= ltol + 1e-4 * np.abs(ref_lse)).all()
    # The scores really do climb by more than the threshold across KV tiles.
    s = (qf[0, 0] @ kf[0, 0].T) * scale * np.log2(np.e)
    tile_max = s[-1].reshape(-1, 128).max(axis=1)
    assert (np.diff(tile_max) > 8.0).all()


def test_strided_operands_match_contiguous(pkg, wl):
    """A [B, N, H, D] buffer viewed as [B, H, N, D] (non-contiguous heads)."""
    w = wl.Workload("t", "bf16", 2, 4, 4, 256, 128, True, seed=5)
    inp = wl.make_inputs(w)
    q, k, v = wl.to_device(inp, w)
    qs, ks, vs = (t.transpose(1, 2).contiguous().transpose(1, 2) for t in (q, k, v))
    assert not qs.is_contiguous()
    a = pkg.fused(q, k, v, w.scale, causal=True)
    b = pkg.fused(qs, ks, vs, w.scale, causal=True)
    pkg.check_status(0)
    assert torch.equal(a, b)


def test_host_memref_pipeline_equals_device(pkg, wl):
    """The memref entry with pinned HOST buffers (staged, overlapped copies)
    gives bit-identical results to the device-resident call.  Host-buffer
    entries never split KV ranges, so the shape is one whose device call
    does not split either (296 slices x 2 pairs: enough work per SM)."""
    w = wl.Workload("t", "bf16", 2, 148, 148, 512, 128, True, seed=9)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert pkg.lib().attn_rt_causal_split(2 * 148, 512, 512, sms) == 0
    inp = wl.make_inputs(w)
    q, k, v = wl.to_device(inp, w)
    L_dev = torch.empty((2, 148, 512), dtype=torch.float32, device="cuda")
    ref = pkg.fused(q, k, v, w.scale, causal=True, lse=L_dev)
    pkg.check_status(0)
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    ho = torch.empty_like(hq).pin_memory()
    hl = torch.empty((2, 148, 512, 1), dtype=torch.float32).pin_memory()
    L = pkg.lib()
    rc = L._mlir_ciface_attn_fused_bf16_causal_4d(
        pkg.memref(hq), pkg.memref(hk), pkg.memref(hv), w.scale, pkg.memref(ho), pkg.memref(hl))
    assert rc == 0, pkg.last_error()
    assert torch.equal(ho, ref.cpu())
    assert torch.equal(hl[..., 0], L_dev.cpu())


def test_unsupported_variants_raise(pkg):
    q = torch.zeros((1, 1, 128, 96), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(pkg.AttentionError) as e:
        pkg.fused(q, q, q, 0.1)
    assert e.value.code == -8
    q = torch.zeros((1, 1, 128, 64), dtype=torch.bfloat16, device="cuda")
    o = torch.zeros((1, 1, 128, 68), dtype=torch.bfloat16, device="cuda")[..., :64]
    with pytest.raises(pkg.AttentionError) as e:
        pkg.fused(q, q, q, 0.1, output=o)
    assert e.value.code == -5


@pytest.mark.parametrize("D", [64, 128])
def test_bf16_dense_mask_parity(pkg, wl, oracle, D):
    """The op's general i1 mask on the tensor-core path (per-slice masks)."""
    w = wl.Workload("t", "bf16", 2, 3, 3, 1000, D, False, seed=40 + D)
    inp = wl.make_inputs(w)
    rng = np.random.default_rng(D)
    M = rng.random((2, 3, 1000, 1000)) < 0.35
    M[..., 0] = False
    # Rows masked over their whole first KV tile (keys 0-127) are NaN in the
    # reference (exp(-inf - -inf) in its loop), whatever later keys allow.
    M[0, 1, [5, 131, 700], :128] = True
    M[1, 2, 999, :] = True
    q, k, v = wl.to_device(inp, w)
    L = torch.empty((2, 3, 1000), dtype=torch.float32, device="cuda")
    out = pkg.fused(q, k, v, w.scale, mask=torch.from_numpy(M).cuda(), lse=L)
    pkg.check_status(0)
    ref, ref_lse = oracle.attn_batched(inp.qf, inp.kf, inp.vf, w.scale, mask=M)
    got, lse = out.float().cpu().numpy(), L.cpu().numpy()
    nan_rows = np.isnan(ref).all(axis=-1)
    assert nan_rows.sum() == 4 and nan_rows[0, 1, [5, 131, 700]].all() and nan_rows[1, 2, 999]
    assert (np.isnan(got) == np.isnan(ref)).all()
    assert (np.isnan(lse) == np.isnan(ref_lse)).all()
    assert _rel(got[~nan_rows], ref[~nan_rows]) <= 2e-2
    assert np.abs(lse[~nan_rows] - ref_lse[~nan_rows]).max() <= 1e-3


@pytest.mark.parametrize("D,broadcast", [(128, False), (64, False), (128, True)])
def test_bf16_dense_block_sparse_mask(pkg, wl, oracle, D, broadcast):
    """Block-structured masks: 128 x 128 blocks fully visible, fully masked
    (skipped by the kernel) or mixed, with ragged Nq / Nk and Q tiles whose
    first KV tile is fully masked (NaN rows, as in the reference)."""
    B, H, Nq, Nk = 2, 3, 700, 900
    w = wl.Workload("t", "bf16", B, H, H, Nq, D, False, seed=60 + D)
    inp = wl.make_inputs(w)
    rng = np.random.default_rng(D + broadcast)
    k_in = rng.standard_normal((B, H, Nk, D)).astype(np.float32)
    v_in = rng.standard_normal((B, H, Nk, D)).astype(np.float32)
    kf, vf = wl.round_bf16(k_in), wl.round_bf16(v_in)
    nqt, nkt = -(-Nq // 128), -(-Nk // 128)
    shape = (1, 1) if broadcast else (B, H)
    kind = rng.choice(3, size=shape + (nqt, nkt), p=[0.4, 0.35, 0.25])  # full, empty, mixed
    kind[..., 2, 0] = 1                      # a Q tile whose first KV tile is masked: NaN rows
    kind[..., 3, :] = 1                      # a Q tile masked everywhere
    kind[..., 4, 0] = 0
    M = np.zeros(shape + (nqt * 128, nkt * 128), bool)
    for idx in np.ndindex(*kind.shape):
        r0, c0 = idx[-2] * 128, idx[-1] * 128
        blk = M[idx[:-2]][r0:r0 + 128, c0:c0 + 128]
        if kind[idx] == 1:
            blk[:] = True
        elif kind[idx] == 2:
            blk[:] = rng.random((128, 128)) < 0.4
    M = M[..., :Nq, :Nk]
    q = torch.from_numpy(inp.qf).to(torch.bfloat16).cuda()
    k = torch.from_numpy(kf).to(torch.bfloat16).cuda()
    v = torch.from_numpy(vf).to(torch.bfloat16).cuda()
    tm = torch.from_numpy(np.ascontiguousarray(M)).cuda()
    if broadcast:
        tm = tm.reshape(Nq, Nk)
    L = torch.empty((B, H, Nq), dtype=torch.float32, device="cuda")
    out = pkg.fused(q, k, v, w.scale, mask=tm, lse=L)
    pkg.check_status(0)
    Mb = np.broadcast_to(M, (B, H, Nq, Nk))
    ref, ref_lse = oracle.attn_batched(inp.qf, kf, vf, w.scale, mask=Mb)
    got, lse = out.float().cpu().numpy(), L.cpu().numpy()
    nan_rows = np.isnan(ref).all(axis=-1)
    assert nan_rows[..., 256:512].all()       # the two Q tiles above
    assert (np.isnan(got) == np.isnan(ref)).all()
    assert (np.isnan(lse) == np.isnan(ref_lse)).all()
    assert _rel(got[~nan_rows], ref[~nan_rows]) <= 2e-2
    assert np.abs(lse[~nan_rows] - ref_lse[~nan_rows]).max() <= 1e-3


@pytest.mark.parametrize("D", [64, 128])
def test_dense_causal_mask_equals_causal_variant(pkg, wl, D):
    """A causal pattern given as an explicit i1 mask and run on the dense-mask
    path (every KV tile visited) gives the same bits as the causal
    specialisation, which skips the fully masked tiles: those tiles only add
    exact zeros."""
    import ctypes

    H = 200  # enough pairs per SM that the causal call runs no KV split
    w = wl.Workload("t", "bf16", 1, H, H, 640, D, True, seed=8)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert pkg.lib().attn_rt_causal_split(H, 640, 640, sms) == 0
    inp = wl.make_inputs(w)
    q, k, v = wl.to_device(inp, w)
    a = pkg.fused(q, k, v, w.scale, causal=True)
    m8 = torch.ones(640, 640, dtype=torch.uint8, device="cuda").triu(1).expand(1, H, 640, 640)
    out = torch.empty_like(a)
    d = pkg.AttnDesc()
    d.dtype, d.out_dtype, d.mask_kind = pkg.ATTN_BF16, pkg.ATTN_BF16, pkg.MASK_DENSE
    d.B, d.Hq, d.Hkv, d.Nq, d.Nk, d.D = 1, H, H, 640, 640, D
    for dst, t in ((d.q_stride, q), (d.k_stride, k), (d.v_stride, v), (d.o_stride, out)):
        dst[0], dst[1], dst[2] = t.stride(0), t.stride(1), t.stride(2)
    d.q, d.k, d.v, d.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr()
    d.mask = m8.data_ptr()
    d.mask_stride[0], d.mask_stride[1], d.mask_stride[2] = m8.stride(0), m8.stride(1), m8.stride(2)
    d.scale = w.scale
    d.q_descale = d.k_descale = d.v_descale = 1.0
    rc = pkg.lib().attn_fwd(ctypes.byref(d), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, pkg.last_error()
    pkg.check_status(0)
    assert torch.equal(out, a)


def test_d64_block_sparse_mask_many_pairs_per_cta(pkg, wl, oracle):
    """d = 64 runs the S GEMM of the next KV tile as soon as the softmax has
    read S (P in TMEM columns of its own).  Per-slice block-sparse masks over
    640 work items (several per persistent CTA), so the two Q tiles of a pair
    skip different KV tiles and the per-tile barrier phases carry across
    pairs; a sample of slices is checked against the oracle."""
    B, H, N, D = 4, 40, 1024, 64
    w = wl.Workload("t", "bf16", B, H, H, N, D, False, seed=77)
    inp = wl.make_inputs(w)
    rng = np.random.default_rng(77)
    nt = N // 128
    kind = rng.choice(3, size=(B, H, nt, nt), p=[0.4, 0.35, 0.25])  # full, empty, mixed
    kind[..., 0] = np.where(kind[..., 0] == 1, 0, kind[..., 0])
    kind[1, 7, 3, 0] = 1                      # a Q tile whose first KV tile is masked: NaN rows
    M = np.repeat(np.repeat(kind == 1, 128, axis=-2), 128, axis=-1)
    mixed = np.repeat(np.repeat(kind == 2, 128, axis=-2), 128, axis=-1)
    M |= mixed & (rng.integers(0, 5, size=(B, H, N, N), dtype=np.uint8) < 2)
    q, k, v = wl.to_device(inp, w)
    L = torch.empty((B, H, N), dtype=torch.float32, device="cuda")
    out = pkg.fused(q, k, v, w.scale, mask=torch.from_numpy(M).cuda(), lse=L)
    pkg.check_status(0)
    slices = [0, 1 * H + 7, 63, 101, 2 * H + 39, B * H - 1]
    ref, ref_lse = oracle.attn_batched(inp.qf, inp.kf, inp.vf, w.scale, mask=M, slices=slices)
    got = out.float().cpu().numpy().reshape(B * H, N, D)[slices]
    lse = L.cpu().numpy().reshape(B * H, N)[slices]
    ref = ref.reshape(B * H, N, D)[slices]
    ref_lse = ref_lse.reshape(B * H, N)[slices]
    nan_rows = np.isnan(ref).all(axis=-1)
    assert nan_rows[1, 384:512].all()
    assert (np.isnan(got) == np.isnan(ref)).all()
    assert (np.isnan(lse) == np.isnan(ref_lse)).all()
    assert _rel(got[~nan_rows], ref[~nan_rows]) <= 2e-2
    assert np.abs(lse[~nan_rows] - ref_lse[~nan_rows]).max() <= 1e-3


def test_bf16_mask_memref_with_host_buffers(pkg, wl, oracle):
    """_mlir_ciface_attn_fused_bf16_mask_4d on host memrefs, broadcast mask."""
    w = wl.Workload("t", "bf16", 1, 2, 2, 300, 64, False, seed=12)
    inp = wl.make_inputs(w)
    rng = np.random.default_rng(3)
    M = rng.random((300, 300)) < 0.5
    M[:, 0] = False
    q, k, v = (t.cpu() for t in wl.to_device(inp, w))
    o = torch.empty_like(q)
    m = torch.from_numpy(M.astype(np.uint8)).reshape(1, 1, 300, 300)
    lse = torch.empty((0, 0, 0, 1), dtype=torch.float32)
    rc = pkg.lib()._mlir_ciface_attn_fused_bf16_mask_4d(
        pkg.memref(q), pkg.memref(k), pkg.memref(v), w.scale, pkg.memref(m), pkg.memref(o),
        pkg.memref(lse))
    assert rc == 0, pkg.last_error()
    ref, _ = oracle.attn_batched(inp.qf, inp.kf, inp.vf, w.scale,
                                 mask=np.broadcast_to(M, (1, 2, 300, 300)))
    assert _rel(o.float().numpy(), ref) <= 2e-2


def test_rank2_mask_on_rank4_operands_as_the_pass_calls_it(pkg, wl, oracle):
    """The lowering pass's call for the op's own rank-2 mask [seq_q, seq_k]
    on rank-4 bf16 operands: _mlir_ciface_attn_fused_bf16_mask2d_4d with a
    2-D mask descriptor (host memrefs), equal bit for bit to the rank-4 mask
    entry given the same mask as [1, 1, seq_q, seq_k], and to the oracle."""
    w = wl.Workload("t", "bf16", 2, 2, 2, 300, 64, False, seed=13)
    inp = wl.make_inputs(w)
    rng = np.random.default_rng(5)
    M = rng.random((300, 300)) < 0.4
    M[:, 0] = False
    q, k, v = (t.cpu() for t in wl.to_device(inp, w))
    m2 = torch.from_numpy(M.astype(np.uint8))
    o2, o4 = torch.empty_like(q), torch.empty_like(q)
    l2 = torch.empty((2, 2, 300, 1), dtype=torch.float32)
    l4 = torch.empty_like(l2)
    L = pkg.lib()
    rc = L._mlir_ciface_attn_fused_bf16_mask2d_4d(
        pkg.memref(q), pkg.memref(k), pkg.memref(v), w.scale, pkg.memref(m2), pkg.memref(o2),
        pkg.memref(l2))
    assert rc == 0, pkg.last_error()
    rc = L._mlir_ciface_attn_fused_bf16_mask_4d(
        pkg.memref(q), pkg.memref(k), pkg.memref(v), w.scale, pkg.memref(m2.reshape(1, 1, 300, 300)),
        pkg.memref(o4), pkg.memref(l4))
    assert rc == 0, pkg.last_error()
    assert torch.equal(o2, o4) and torch.equal(l2, l4)
    ref, ref_lse = oracle.attn_batched(inp.qf, inp.kf, inp.vf, w.scale,
                                       mask=np.broadcast_to(M, (2, 2, 300, 300)))
    assert _rel(o2.float().numpy(), ref) <= 2e-2
    assert np.abs(l2[..., 0].numpy() - ref_lse).max() <= 1e-3
    # A mask whose extents do not match the operands is refused, not misread.
    bad = torch.zeros((300, 299), dtype=torch.uint8)
    rc = L._mlir_ciface_attn_fused_bf16_mask2d_4d(
        pkg.memref(q), pkg.memref(k), pkg.memref(v), w.scale, pkg.memref(bad), pkg.memref(o2),
        pkg.memref(l2))
    assert rc == -2


def test_bounded_wait_times_out_and_device_stays_usable(pkg, wl, oracle):
    """A wait on a barrier nothing arrives on gives up after its limit with
    ATTN_ERR_TIMEOUT (no trap, no hang), and the next attention call is
    correct."""
    import time

    t0 = time.perf_counter()
    rc = pkg.lib().attn_rt_probe_timeout(20_000_000)  # 20 ms
    assert rc == -7, pkg.last_error()
    assert time.perf_counter() - t0 < 5.0
    w = wl.Workload("t", "bf16", 1, 2, 2, 256, 128, True, seed=1)
    inp = wl.make_inputs(w)
    got, _ = _run_pkg(pkg, wl, w, inp, True)
    ref, _ = _ref(oracle, inp, w, True)
    assert _rel(got, ref) <= 2e-2


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("Nq,Nk,causal", [(300, 700, False), (300, 700, True), (700, 300, True),
                                          (128, 1024, False), (1000, 129, False), (300, 5, False),
                                          (5, 300, True)])
def test_unequal_query_and_key_lengths(pkg, wl, oracle, Nq, Nk, causal, D):
    """Cross-attention shapes (Nq != Nk), ragged tiles on both sides; causal
    is the op's mask[i][j] = j > i (top-left aligned).  d = 64 runs the early-S
    schedule, d = 128 the S-behind-P·V one."""
    rng = np.random.Generator(np.random.PCG64(Nq * 7 + Nk))
    B, H = 2, 2
    qf = wl.round_bf16(rng.standard_normal((B, H, Nq, D), dtype=np.float32))
    kf = wl.round_bf16(rng.standard_normal((B, H, Nk, D), dtype=np.float32))
    vf = wl.round_bf16(rng.standard_normal((B, H, Nk, D), dtype=np.float32))
    q, k, v = (torch.from_numpy(a).cuda().to(torch.bfloat16) for a in (qf, kf, vf))
    L = torch.empty((B, H, Nq), dtype=torch.float32, device="cuda")
    out = pkg.fused(q, k, v, D ** -0.5, causal=causal, lse=L)
    pkg.check_status(0)
    ref, ref_lse = oracle.attn_batched(qf, kf, vf, D ** -0.5, causal=causal)
    assert _rel(out.float().cpu().numpy(), ref) <= 2e-2
    assert np.abs(L.cpu().numpy() - ref_lse).max() <= 1e-3


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [True, False])
def test_f16_parity(pkg, oracle, D, causal):
    """f16 inputs on the same tensor-core kernels (f16 operand format, P in
    f16, f16 output), against the oracle on the f16-rounded values."""
    rng = np.random.Generator(np.random.PCG64(D + 17 * causal))
    B, H, N = 2, 2, 700
    arrs = [rng.standard_normal((B, H, N, D), dtype=np.float32).astype(np.float16)
            for _ in range(3)]
    q, k, v = (torch.from_numpy(a).cuda() for a in arrs)
    L = torch.empty((B, H, N), dtype=torch.float32, device="cuda")
    out = pkg.fused(q, k, v, D ** -0.5, causal=causal, lse=L)
    pkg.check_status(0)
    assert out.dtype == torch.float16
    ref, ref_lse = oracle.attn_batched(*(a.astype(np.float32) for a in arrs), D ** -0.5,
                                       causal=causal)
    assert _rel(out.float().cpu().numpy(), ref) <= 1e-2
    assert np.abs(L.cpu().numpy() - ref_lse).max() <= 1e-3


def test_host_memref_pipeline_strided_equals_device(pkg, wl):
    """Host memrefs whose heads are not packed ([B, N, H, D] storage viewed as
    [B, H, N, D]) take the per-slice staging copies; same bits as the device
    call on the same views."""
    w = wl.Workload("t", "bf16", 2, 4, 4, 384, 64, False, seed=19)
    inp = wl.make_inputs(w)
    q, k, v = (t.transpose(1, 2).contiguous().transpose(1, 2) for t in wl.to_device(inp, w))
    assert not q.is_contiguous()
    L_dev = torch.empty((2, 4, 384), dtype=torch.float32, device="cuda")
    ref = pkg.fused(q, k, v, w.scale, lse=L_dev)
    pkg.check_status(0)
    hq, hk, hv = (t.cpu().transpose(1, 2).contiguous().pin_memory().transpose(1, 2)
                  for t in (q, k, v))
    ho = torch.empty((2, 384, 4, 64), dtype=torch.bfloat16).pin_memory().transpose(1, 2)
    hl = torch.empty((2, 4, 384, 1), dtype=torch.float32).pin_memory()
    rc = pkg.lib()._mlir_ciface_attn_fused_bf16_nomask_4d(
        pkg.memref(hq), pkg.memref(hk), pkg.memref(hv), w.scale, pkg.memref(ho), pkg.memref(hl))
    assert rc == 0, pkg.last_error()
    assert torch.equal(ho, ref.cpu())
    assert torch.equal(hl[..., 0], L_dev.cpu())


def _block_mask(rng, shape, nq, nk):
    """Random 128 x 128 block structure (visible / masked / mixed blocks)."""
    nqt, nkt = -(-nq // 128), -(-nk // 128)
    kind = rng.choice(3, size=shape + (nqt, nkt), p=[0.4, 0.3, 0.3])
    kind[..., 0] = 2  # first KV tile mixed: no NaN rows
    M = np.zeros(shape + (nqt * 128, nkt * 128), bool)
    for idx in np.ndindex(*kind.shape):
        r0, c0 = idx[-2] * 128, idx[-1] * 128
        blk = M[idx[:-2]][r0:r0 + 128, c0:c0 + 128]
        if kind[idx] == 1:
            blk[:] = True
        elif kind[idx] == 2:
            blk[:] = rng.random((128, 128)) < 0.4
            blk[:, 0] = False
    return np.ascontiguousarray(M[..., :nq, :nk])


@pytest.mark.parametrize("dtype", ["f16", "e4m3"])
def test_dense_block_mask_gqa_other_types(pkg, wl, oracle, dtype):
    """Dense block masks with grouped-query heads on f16 inputs and on e4m3
    inputs with per-block factors (mask per query head, blocks skipped)."""
    rng = np.random.default_rng(5 if dtype == "f16" else 6)
    B, Hq, Hkv, Nq, Nk, D = 2, 4, 2, 520, 700, 128
    M = _block_mask(rng, (B, Hq), Nq, Nk)
    q = rng.standard_normal((B, Hq, Nq, D)).astype(np.float32)
    k = rng.standard_normal((B, Hkv, Nk, D)).astype(np.float32)
    v = rng.standard_normal((B, Hkv, Nk, D)).astype(np.float32)
    if dtype == "f16":
        qf, kf, vf = (a.astype(np.float16).astype(np.float32) for a in (q, k, v))
        dev = [torch.from_numpy(a.astype(np.float16)).cuda() for a in (q, k, v)]
        kw, tol = {}, 1e-2
    else:
        (q8, qd, qf), (k8, kd, kf), (v8, vd, vf) = (
            wl.quant_e4m3_blocks(q), wl.quant_e4m3_blocks(k), wl.quant_e4m3_heads(v))
        dev = [torch.from_numpy(a).cuda() for a in (q8, k8, v8)]
        kw = dict(q_descale=torch.from_numpy(qd).cuda(), k_descale=torch.from_numpy(kd).cuda(),
                  v_descale=torch.from_numpy(vd).cuda())
        tol = 6e-2
    L = torch.empty((B, Hq, Nq), dtype=torch.float32, device="cuda")
    out = pkg.fused(*dev, D ** -0.5, mask=torch.from_numpy(M).cuda(), lse=L, **kw)
    pkg.check_status(0)
    ref, ref_lse = oracle.attn_batched(qf, kf, vf, D ** -0.5, mask=M)
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all() and np.isfinite(ref).all()
    for b in range(B):
        for h in range(Hq):
            assert _rel(got[b, h], ref[b, h]) <= tol, (b, h)
    assert np.abs(L.cpu().numpy() - ref_lse).max() <= 1e-2


def test_dense_block_mask_f32_output(pkg, wl, oracle):
    """bf16 inputs, f32 output, dense block mask broadcast over heads."""
    rng = np.random.default_rng(8)
    w = wl.Workload("t", "bf16", 1, 3, 3, 900, 128, False, seed=21)
    inp = wl.make_inputs(w)
    M = _block_mask(rng, (), 900, 900)
    q, k, v = wl.to_device(inp, w)
    out = torch.empty((1, 3, 900, 128), dtype=torch.float32, device="cuda")
    pkg.fused(q, k, v, w.scale, mask=torch.from_numpy(M).cuda(), output=out)
    pkg.check_status(0)
    ref, _ = oracle.attn_batched(inp.qf, inp.kf, inp.vf, w.scale,
                                 mask=np.broadcast_to(M, (1, 3, 900, 900)))
    assert _rel(out.cpu().numpy(), ref) <= 2e-2


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_empty_extents_match_the_reference_loop(pkg, oracle, dtype):
    """No key: every output row NaN and LSE -inf (the reference's loop never
    runs a KV step, O = 0/0); no query row: a no-op.  Device tensors and host
    memrefs."""
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    q = torch.randn((2, 3, 200, 64), device="cuda").to(tdt)
    none = torch.empty((2, 3, 0, 64), device="cuda", dtype=tdt)
    L = torch.zeros((2, 3, 200), dtype=torch.float32, device="cuda")
    out = pkg.fused(q, none, none, 0.125, lse=L)
    pkg.check_status(0)
    ref, ref_lse = oracle.attn_batched(q.float().cpu().numpy(), none.float().cpu().numpy(),
                                       none.float().cpu().numpy(), 0.125)
    assert torch.isnan(out).all() and np.isnan(ref).all()
    assert torch.isneginf(L).all() and np.isneginf(ref_lse).all()
    # no query row: the output is left untouched
    q0 = torch.empty((2, 3, 0, 64), device="cuda", dtype=tdt)
    k = torch.randn((2, 3, 50, 64), device="cuda").to(tdt)
    o0 = pkg.fused(q0, k, k, 0.125)
    pkg.check_status(0)
    assert o0.shape == (2, 3, 0, 64)
    # host memrefs, rank-2 f32 form of the op
    hq = torch.randn((40, 64))
    hk = torch.empty((0, 64))
    ho = torch.zeros((40, 64))
    rc = pkg.lib()._mlir_ciface_attn_fused_f32_nomask(pkg.memref(hq), pkg.memref(hk),
                                                      pkg.memref(hk), 0.125, pkg.memref(ho))
    assert rc == 0, pkg.last_error()
    assert torch.isnan(ho).all()


def test_long_key_sequence_single_query_row(pkg, oracle):
    """One query row against 262144 keys (2048 KV tiles in one online-softmax
    chain, Nq far below a tile), bf16 with LSE."""
    g = torch.Generator(device="cuda").manual_seed(31)
    Nk, D = 262144, 128
    q = torch.randn((1, 1, 1, D), generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn((1, 1, Nk, D), generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn((1, 1, Nk, D), generator=g, device="cuda").to(torch.bfloat16)
    L = torch.empty((1, 1, 1), dtype=torch.float32, device="cuda")
    out = pkg.fused(q, k, v, D ** -0.5, lse=L)
    pkg.check_status(0)
    ref, ref_lse = oracle.attn_batched(*(t.float().cpu().numpy() for t in (q, k, v)), D ** -0.5)
    assert _rel(out.float().cpu().numpy(), ref) <= 2e-2
    assert abs(float(L.item()) - float(ref_lse.ravel()[0])) <= 1e-3


def test_long_causal_sequence_sampled_tiles(pkg, oracle):
    """N = 65536 causal, one head: the first, a middle and the last Q tile
    against the oracle (256 KV tiles on the longest rows)."""
    g = torch.Generator(device="cuda").manual_seed(32)
    N, D = 65536, 128
    q, k, v = (torch.randn((1, 1, N, D), generator=g, device="cuda").to(torch.bfloat16)
               for _ in range(3))
    L = torch.empty((1, 1, N), dtype=torch.float32, device="cuda")
    out = pkg.fused(q, k, v, D ** -0.5, causal=True, lse=L)
    pkg.check_status(0)
    got, lse = out.float().cpu().numpy(), L.cpu().numpy()
    assert np.isfinite(got).all()
    qf, kf, vf = (t.float().cpu().numpy() for t in (q, k, v))
    ref = np.zeros_like(qf)
    ref_lse = np.zeros((1, 1, N), np.float32)
    oracle.attn_batched(qf, kf, vf, D ** -0.5, causal=True, tile_offset=0, tile_stride=255,
                        out=ref, lse_out=ref_lse)
    for t in (0, 255, 510):
        rows = slice(t * 128, t * 128 + 128)
        assert _rel(got[0, 0, rows], ref[0, 0, rows]) <= 2e-2, t
        assert np.abs(lse[0, 0, rows] - ref_lse[0, 0, rows]).max() <= 1e-3, t


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("kind", ["none", "causal", "dense"])
def test_f32_tiled_parity(pkg, oracle, D, kind):
    """fp32 with head_dim 64 / 128 (the register-tiled CUDA-core kernel):
    ragged Nq / Nk, grouped heads, at the reference op's 1e-4 tolerance; dense
    masks include rows masked over keys [0, 128) only (NaN in the reference)."""
    rng = np.random.default_rng(D + len(kind))
    B, Hq, Hkv, Nq, Nk = 2, 4, 2, 333, 517
    if kind == "causal":
        Nk = Nq
    q = rng.standard_normal((B, Hq, Nq, D)).astype(np.float32)
    k = rng.standard_normal((B, Hkv, Nk, D)).astype(np.float32)
    v = rng.standard_normal((B, Hkv, Nk, D)).astype(np.float32)
    M = None
    if kind == "dense":
        M = rng.random((B, Hq, Nq, Nk)) < 0.3
        M[..., 0] = False
        M[0, 1, [7, 100], :128] = True
        M[1, 3, 200, :] = True
    L = torch.empty((B, Hq, Nq), dtype=torch.float32, device="cuda")
    out = pkg.fused(*(torch.from_numpy(a).cuda() for a in (q, k, v)), D ** -0.5,
                    causal=kind == "causal", lse=L,
                    mask=None if M is None else torch.from_numpy(M).cuda())
    pkg.check_status(0)
    ref, ref_lse = oracle.attn_batched(q, k, v, D ** -0.5, causal=kind == "causal", mask=M)
    got, lse = out.cpu().numpy(), L.cpu().numpy()
    assert (np.isnan(got) == np.isnan(ref)).all() and (np.isnan(lse) == np.isnan(ref_lse)).all()
    ok = ~np.isnan(ref)
    assert np.abs(got[ok] - ref[ok]).max() / np.abs(ref[ok]).max() <= 1e-4
    okl = ~np.isnan(ref_lse)
    assert np.abs(lse[okl] - ref_lse[okl]).max() <= 1e-4
    if kind == "dense":
        assert np.isnan(ref[0, 1, [7, 100]]).all() and np.isnan(ref[1, 3, 200]).all()


def test_device_resident_memrefs_via_runtime_helpers(pkg, wl):
    """A lowered program that keeps its operands on the GPU: attn_rt_alloc +
    attn_rt_copy, then the memref entry on device memrefs, gives the same bits
    as the host-memref call."""
    import ctypes

    w = wl.Workload("t", "bf16", 1, 4, 4, 300, 128, False, seed=23)
    inp = wl.make_inputs(w)
    q, k, v = (t.cpu().contiguous() for t in wl.to_device(inp, w))
    ho = torch.empty_like(q)
    L = pkg.lib()
    lse0 = torch.empty((0, 0, 0, 1), dtype=torch.float32)
    rc = L._mlir_ciface_attn_fused_bf16_nomask_4d(pkg.memref(q), pkg.memref(k), pkg.memref(v),
                                                  w.scale, pkg.memref(ho), pkg.memref(lse0))
    assert rc == 0, pkg.last_error()
    nbytes = q.numel() * 2
    ptrs = []
    for t in (q, k, v, ho):
        p = ctypes.c_void_p()
        assert L.attn_rt_alloc(ctypes.byref(p), nbytes) == 0, pkg.last_error()
        ptrs.append(p.value)
    for src, dst in zip((q, k, v), ptrs):
        assert L.attn_rt_copy(dst, src.data_ptr(), nbytes, None) == 0

    def dev_memref(ptr, like):
        m = pkg.memref(like)
        m.allocated = m.aligned = ptr
        return m

    rc = L._mlir_ciface_attn_fused_bf16_nomask_4d(
        dev_memref(ptrs[0], q), dev_memref(ptrs[1], k), dev_memref(ptrs[2], v), w.scale,
        dev_memref(ptrs[3], ho), pkg.memref(lse0))
    assert rc == 0, pkg.last_error()
    back = torch.empty_like(ho)
    assert L.attn_rt_copy(back.data_ptr(), ptrs[3], nbytes, None) == 0
    for p in ptrs:
        assert L.attn_rt_free(p) == 0
    assert torch.equal(back, ho)


def test_attn_fwd_rejects_host_pointers(pkg, wl):
    """The descriptor entry takes device pointers: a host buffer is refused
    before any launch (no fault), and the next call runs normally."""
    import ctypes

    w = wl.Workload("t", "bf16", 1, 2, 2, 256, 128, False, seed=3)
    inp = wl.make_inputs(w)
    q, k, v = wl.to_device(inp, w)
    out = torch.empty_like(q)
    host_k = k.cpu()
    d = pkg.AttnDesc()
    d.dtype, d.out_dtype, d.mask_kind = pkg.ATTN_BF16, pkg.ATTN_BF16, pkg.MASK_NONE
    d.B, d.Hq, d.Hkv, d.Nq, d.Nk, d.D = 1, 2, 2, 256, 256, 128
    for dst, t in ((d.q_stride, q), (d.k_stride, k), (d.v_stride, v), (d.o_stride, out)):
        dst[0], dst[1], dst[2] = t.stride(0), t.stride(1), t.stride(2)
    d.q, d.k, d.v, d.o = q.data_ptr(), host_k.data_ptr(), v.data_ptr(), out.data_ptr()
    d.scale = w.scale
    d.q_descale = d.k_descale = d.v_descale = 1.0
    rc = pkg.lib().attn_fwd(ctypes.byref(d), torch.cuda.current_stream().cuda_stream)
    assert rc == -1 and "device pointers" in pkg.last_error()
    ref = pkg.fused(q, k, v, w.scale)
    pkg.check_status(0)
    assert torch.isfinite(ref.float()).all()


@pytest.mark.parametrize("in_dt", ["bf16", "f16"])
@pytest.mark.parametrize("out_dt", ["bf16", "f16", "f32"])
def test_input_output_type_matrix(pkg, oracle, in_dt, out_dt):
    """Every input / output element type pair of the tensor-core kernel
    (causal, grouped heads, ragged N)."""
    tin = {"bf16": torch.bfloat16, "f16": torch.float16}[in_dt]
    tout = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[out_dt]
    g = torch.Generator(device="cuda").manual_seed(40 + len(in_dt) + len(out_dt))
    B, Hq, Hkv, N, D = 1, 4, 2, 300, 128
    q = torch.randn((B, Hq, N, D), generator=g, device="cuda").to(tin)
    k = torch.randn((B, Hkv, N, D), generator=g, device="cuda").to(tin)
    v = torch.randn((B, Hkv, N, D), generator=g, device="cuda").to(tin)
    out = torch.empty((B, Hq, N, D), dtype=tout, device="cuda")
    pkg.fused(q, k, v, D ** -0.5, output=out, causal=True)
    pkg.check_status(0)
    ref, _ = oracle.attn_batched(*(t.float().cpu().numpy() for t in (q, k, v)), D ** -0.5,
                                 causal=True)
    assert _rel(out.float().cpu().numpy(), ref) <= 2e-2


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("scale", [-0.09, 0.0])
@pytest.mark.parametrize("kind", ["causal", "dense"])
def test_negative_and_zero_scale(pkg, oracle, scale, kind, D):
    """The op's scale is any f32: a negative scale flips which score is the
    row maximum (the kernel reduces with min then), zero gives uniform weights
    over the visible keys."""
    g = torch.Generator(device="cuda").manual_seed(50)
    B, H, N = 1, 2, 400
    q, k, v = (torch.randn((B, H, N, D), generator=g, device="cuda").to(torch.bfloat16)
               for _ in range(3))
    M = None
    if kind == "dense":
        M = torch.rand((N, N), generator=g, device="cuda") < 0.3
        M[:, 0] = False
    L = torch.empty((B, H, N), dtype=torch.float32, device="cuda")
    out = pkg.fused(q, k, v, scale, causal=kind == "causal", mask=M, lse=L, classify=False)
    pkg.check_status(0)
    ref, ref_lse = oracle.attn_batched(*(t.float().cpu().numpy() for t in (q, k, v)), scale,
                                       causal=kind == "causal",
                                       mask=None if M is None else np.broadcast_to(
                                           M.cpu().numpy(), (B, H, N, N)))
    assert _rel(out.float().cpu().numpy(), ref) <= 2e-2
    assert np.abs(L.cpu().numpy() - ref_lse).max() <= 1e-3


@pytest.mark.parametrize("dtype,D,tol", [("bf16", 64, 2e-2), ("bf16", 128, 2e-2),
                                         ("f32", 64, 1e-4)])
@pytest.mark.parametrize("where", ["q", "k", "k_causal", "v"])
def test_nan_inputs_propagate_like_the_reference(pkg, wl, oracle, dtype, D, tol, where):
    """A NaN operand reaches exactly the outputs it reaches in the reference's
    loop (arith.maximumf propagates NaN): a NaN in Q row r makes O row r and
    its LSE NaN; a NaN key makes every row that sees it NaN (every row
    without a mask; with the causal mask only rows at or after the key, the
    mask select replacing the NaN score by -inf before it); a NaN in V
    element (s, c) makes column c NaN in every row (0 x NaN included)."""
    causal = where == "k_causal"
    w = wl.Workload("t", dtype, 1, 2, 2, 384, D, causal, seed=61)
    inp = wl.make_inputs(w)
    if where == "q":
        inp.q[0, 1, 5, 3] = np.nan
    elif where in ("k", "k_causal"):
        inp.k[0, 0, 300, 7] = np.nan
    else:
        inp.v[0, 1, 200, 9] = np.nan
    for a, b in ((inp.qf, inp.q), (inp.kf, inp.k), (inp.vf, inp.v)):
        assert a is b  # bf16 / f32 inputs: the oracle reads the same arrays
    got, lse = _run_pkg(pkg, wl, w, inp, causal=causal)
    ref, ref_lse = _ref(oracle, inp, w, causal)
    nan = np.isnan(ref)
    expect = np.zeros_like(nan)
    if where == "q":
        expect[0, 1, 5, :] = True
    elif where == "k":
        expect[0, 0] = True
    elif where == "k_causal":
        expect[0, 0, 300:] = True
    else:
        expect[0, 1, :, 9] = True
    assert (nan == expect).all()
    assert (np.isnan(got) == nan).all()
    assert (np.isnan(lse) == np.isnan(ref_lse)).all()
    assert _rel(got[~nan], ref[~nan]) <= tol
    ok = ~np.isnan(ref_lse)
    assert np.abs(lse[ok] - ref_lse[ok]).max() <= (1e-5 if dtype == "f32" else 1e-3)


def test_concurrent_streams_match_serial(pkg, wl):
    """Calls on two streams at once (causal and dense-mask calls on one, a
    no-mask call on the other; the dense call's scratch is stream-ordered)
    give the same bits as the same calls run one after another."""
    w = wl.Workload("t", "bf16", 2, 8, 8, 2048, 128, True, seed=91)
    inp = wl.make_inputs(w)
    q, k, v = wl.to_device(inp, w)
    q2, k2, v2 = (t.flip(2).contiguous() for t in (q, k, v))
    m = torch.rand(2048, 2048, device="cuda") < 0.3
    ref1 = pkg.fused(q, k, v, w.scale, causal=True)
    ref2 = pkg.fused(q2, k2, v2, w.scale)
    ref3 = pkg.fused(q2, k, v2, w.scale, mask=m, classify=False)
    torch.cuda.synchronize()
    pkg.check_status(0)
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    outs = []
    for _ in range(4):
        with torch.cuda.stream(s1):
            a = pkg.fused(q, k, v, w.scale, causal=True)
            c = pkg.fused(q2, k, v2, w.scale, mask=m, classify=False)
        with torch.cuda.stream(s2):
            b = pkg.fused(q2, k2, v2, w.scale)
        outs.append((a, b, c))
    torch.cuda.synchronize()
    pkg.check_status(0)
    for a, b, c in outs:
        assert torch.equal(a, ref1) and torch.equal(b, ref2) and torch.equal(c, ref3)


def test_cuda_graph_capture_replays(pkg, wl):
    """One causal call and one dense-mask call (classifier, ordering kernel,
    stream-ordered scratch, attention kernel) captured into a CUDA graph:
    replays on new inputs copied into the captured buffers give the same bits
    as eager calls on those inputs."""
    w = wl.Workload("t", "bf16", 1, 8, 8, 1024, 128, True, seed=93)
    inp = wl.make_inputs(w)
    q, k, v = wl.to_device(inp, w)
    m = torch.rand(1024, 1024, device="cuda") < 0.25
    o1, o2 = torch.empty_like(q), torch.empty_like(q)
    L = torch.empty((1, 8, 1024), dtype=torch.float32, device="cuda")

    def calls():
        pkg.fused(q, k, v, w.scale, output=o1, causal=True, lse=L)
        pkg.fused(q, k, v, w.scale, mask=m, output=o2, classify=False)

    calls()  # first-call setup (kernel attributes, device state) outside capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            calls()
    torch.cuda.synchronize()
    for seed in (1, 2):
        gen = torch.Generator(device="cuda")
        gen.manual_seed(seed)
        for t in (q, k, v):
            t.copy_(torch.randn(t.shape, generator=gen, device="cuda").to(t.dtype))
        g.replay()
        torch.cuda.synchronize()
        pkg.check_status(0)
        L_e = torch.empty_like(L)
        e1 = pkg.fused(q, k, v, w.scale, causal=True, lse=L_e)
        e2 = pkg.fused(q, k, v, w.scale, mask=m, classify=False)
        torch.cuda.synchronize()
        assert torch.equal(o1, e1) and torch.equal(L, L_e) and torch.equal(o2, e2)
    del g
