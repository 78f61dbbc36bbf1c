"""Causal KV split of the heaviest Q-tile pairs (few pairs per SM).

A causal launch with few pairs per SM (for instance 4 heads of N = 16384,
one GPU's share when c4's 32 heads are split over eight GPUs) is bounded by
its heaviest pairs.  The runtime then runs the heaviest pair indices as two
work items over the two halves of their KV tiles and merges them in the
kernel (attn_rt_causal_split gives the plan).  These tests run shapes whose
plan splits, on every kernel path that can split (d = 128 and the d = 64
early-S schedule, bf16 / f16 / e4m3 inputs, bf16 / f16 / f32 outputs, ragged
Nq != Nk), against the oracle on whole slices, and check that the merge is
deterministic.  Tolerances as in the other parity tests.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _sms():
    return torch.cuda.get_device_properties(0).multi_processor_count


def _rel(got, ref):
    return float(np.abs(got - ref).max() / np.abs(ref).max())


def _bf16(rng, shape):
    from mlir_flashattention_b200 import workloads as wl  # noqa: PLC0415
    return wl.round_bf16(rng.standard_normal(shape, dtype=np.float32))


@pytest.mark.parametrize("D", [128, 64])
def test_long_causal_few_heads(pkg, oracle, D):
    """bf16 causal N = 16384 with 4 (d = 128) or 2 (d = 64) heads: the
    heaviest pairs are split; two whole slices against the oracle, LSE
    included."""
    H, N = (4, 16384) if D == 128 else (2, 16384)
    S = pkg.lib().attn_rt_causal_split(H, N, N, _sms())
    assert S > 0
    rng = np.random.Generator(np.random.PCG64(500 + D))
    q, k, v = (_bf16(rng, (1, H, N, D)) for _ in range(3))
    tq, tk, tv = (torch.from_numpy(a).cuda().to(torch.bfloat16) for a in (q, k, v))
    L = torch.empty((1, H, N), dtype=torch.float32, device="cuda")
    out = pkg.fused(tq, tk, tv, D ** -0.5, causal=True, lse=L)
    pkg.check_status(0)
    again = pkg.fused(tq, tk, tv, D ** -0.5, causal=True)
    pkg.check_status(0)
    assert torch.equal(out, again)  # the merge order is fixed
    got = out.float().cpu().numpy()
    lse = L.cpu().numpy()
    slices = [0, H - 1]
    ref = np.zeros_like(q)
    ref_lse = np.zeros(q.shape[:3], np.float32)
    oracle.attn_batched(q, k, v, D ** -0.5, causal=True, slices=slices, out=ref, lse_out=ref_lse)
    for h in slices:
        assert _rel(got[0, h], ref[0, h]) <= 2e-2, h
        assert np.abs(lse[0, h] - ref_lse[0, h]).max() <= 1e-3, h


def test_e4m3_gqa_split(pkg, wl, oracle):
    """e4m3 causal GQA (4 q-heads on one kv head), N = 8192, bf16 output."""
    B, Hq, N = 1, 4, 8192
    assert pkg.lib().attn_rt_causal_split(B * Hq, N, N, _sms()) > 0
    w = wl.WORKLOADS["c5"]
    inp = wl.make_inputs(w, B=B, Hq=Hq, N=N, seed=77)
    q, k, v = wl.to_device(inp, w)
    L = torch.empty((B, Hq, N), dtype=torch.float32, device="cuda")
    qd, kd, vd = inp.descale
    out = pkg.fused(q, k, v, w.scale, causal=True, lse=L, q_descale=qd, k_descale=kd,
                    v_descale=vd)
    pkg.check_status(0)
    ref, ref_lse = oracle.attn_batched(inp.qf, inp.kf, inp.vf, w.scale, causal=True)
    got, lse = out.float().cpu().numpy(), L.cpu().numpy()
    for h in range(Hq):
        assert _rel(got[0, h], ref[0, h]) <= 6e-2, h
    assert np.abs(lse - ref_lse).max() <= 1e-2


@pytest.mark.parametrize("H,Nq,Nk,dt", [(4, 5000, 7000, "f32out"), (2, 7000, 3000, "f16")])
def test_ragged_cross_attention_split(pkg, oracle, H, Nq, Nk, dt):
    """Causal mask[i][j] = j > i with Nq != Nk and ragged tiles; rows of a
    second half may see no key at all (weight 0 in the merge).  bf16 in / f32
    out, and f16 in / f16 out."""
    B, D = 1, 128
    assert pkg.lib().attn_rt_causal_split(B * H, Nq, Nk, _sms()) > 0
    rng = np.random.Generator(np.random.PCG64(Nq + Nk))
    if dt == "f16":
        arrs = [rng.standard_normal(s, dtype=np.float32).astype(np.float16)
                for s in ((B, H, Nq, D), (B, H, Nk, D), (B, H, Nk, D))]
        tq, tk, tv = (torch.from_numpy(a).cuda() for a in arrs)
        qf, kf, vf = (a.astype(np.float32) for a in arrs)
        out = None
        tol = 1e-2
    else:
        qf, kf, vf = (_bf16(rng, s) for s in ((B, H, Nq, D), (B, H, Nk, D), (B, H, Nk, D)))
        tq, tk, tv = (torch.from_numpy(a).cuda().to(torch.bfloat16) for a in (qf, kf, vf))
        out = torch.empty((B, H, Nq, D), dtype=torch.float32, device="cuda")
        tol = 2e-2
    L = torch.empty((B, H, Nq), dtype=torch.float32, device="cuda")
    out = pkg.fused(tq, tk, tv, D ** -0.5, causal=True, output=out, lse=L)
    pkg.check_status(0)
    ref, ref_lse = oracle.attn_batched(qf, kf, vf, D ** -0.5, causal=True)
    assert _rel(out.float().cpu().numpy(), ref) <= tol
    assert np.abs(L.cpu().numpy() - ref_lse).max() <= 1e-3


def test_e4m3_per_block_descales_with_split(pkg, wl, oracle):
    """Per-block Q/K and per-head V e4m3 factors on a split launch: the second
    half of a pair starts at its own KV block's factor, so a wrong start block
    shows up as a large error (block magnitudes spread over two decades)."""
    B, Hq, Hkv, N, D = 1, 2, 1, 4096, 128
    assert pkg.lib().attn_rt_causal_split(B * Hq, N, N, _sms()) > 0
    rng = np.random.default_rng(23)

    def spread(H):
        f = 10.0 ** rng.uniform(-1.0, 1.0, size=(B, H, N // 128))
        return np.repeat(f, 128, axis=2)[:, :, :, None].astype(np.float32)

    q = rng.standard_normal((B, Hq, N, D)).astype(np.float32) * spread(Hq)
    k = rng.standard_normal((B, Hkv, N, D)).astype(np.float32) * spread(Hkv)
    v = rng.standard_normal((B, Hkv, N, D)).astype(np.float32)
    q8, qd, qf = wl.quant_e4m3_blocks(q)
    k8, kd, kf = wl.quant_e4m3_blocks(k)
    v8, vd, vf = wl.quant_e4m3_heads(v)
    scale = 1.0 / np.sqrt(D)
    dev = [torch.from_numpy(a).cuda() for a in (q8, k8, v8, qd, kd, vd)]
    L = torch.empty((B, Hq, N), dtype=torch.float32, device="cuda")
    out = pkg.fused(dev[0], dev[1], dev[2], scale, causal=True, lse=L, q_descale=dev[3],
                    k_descale=dev[4], v_descale=dev[5])
    pkg.check_status(0)
    got = out.float().cpu().numpy()
    ref, ref_lse = oracle.attn_batched(qf, kf, vf, scale, causal=True)
    for h in range(Hq):
        assert _rel(got[0, h], ref[0, h]) <= 6e-2, h
    assert (np.abs(L.cpu().numpy() - ref_lse) <= 1e-2 + 1e-4 * np.abs(ref_lse)).all()
