"""Parity at the benchmark configurations' own shapes (not reduced members).

Each test runs the full workload through ``fused`` (the C ABI) and compares
seeded samples of (batch, head) slices, every Q tile of each, with the oracle
(the CPU restatement of lib/Attention/TilingPass.cpp:188-386, which computes
every slice with the same loop nest).  The samples always hold head 0, the
last head and the last kv-head group, so a persistent-schedule or head-index
error at the real slice and pair counts shows up:

  c3  bf16 non-causal B=4 H=32 N=4096 d=128 (128 slices x 16 pairs), fp32 LSE
  c4  bf16 causal B=1 H=32 N=16384 d=128 (32 slices x 64 pairs)
  c5  e4m3 causal GQA B=16 Hq=32 Hkv=8 N=2048 d=128 (512 slices x 8 pairs),
      per-tensor amax/448 descales, bf16 output

Tolerances: max|O - O_oracle| / max|O_oracle| per slice <= 2e-2 (bf16) and
6e-2 (e4m3); LSE max abs difference <= 1e-3 (bf16) and 1e-2 (e4m3).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _sample(w, n, seed):
    """``n`` flat slice indices (b * Hq + h): head 0 and the last head of the
    first and last batch, the first head of the last kv-head group of the last
    batch, and seeded picks for the rest."""
    group = w.Hq // w.Hkv
    last_b = w.B - 1
    fixed = {0, w.Hq - 1, last_b * w.Hq, last_b * w.Hq + w.Hq - 1,
             last_b * w.Hq + (w.Hkv - 1) * group}
    rng = np.random.default_rng(seed)
    while len(fixed) < n:
        fixed.add(int(rng.integers(0, w.B * w.Hq)))
    return sorted(fixed)


def _check(pkg, wl, oracle, name, lse_tol, n=6):
    w = wl.WORKLOADS[name]
    inp = wl.make_inputs(w)
    q, k, v = wl.to_device(inp, w)
    L = torch.empty((w.B, w.Hq, w.N), dtype=torch.float32, device="cuda")
    qd, kd, vd = inp.descale
    out = pkg.fused(q, k, v, w.scale, causal=w.causal, lse=L, q_descale=qd, k_descale=kd,
                    v_descale=vd)
    pkg.check_status(0)
    got = out.float().cpu().numpy().reshape(w.B * w.Hq, w.N, w.D)
    lse = L.cpu().numpy().reshape(w.B * w.Hq, w.N)
    assert np.isfinite(got).all() and np.isfinite(lse).all()
    slices = _sample(w, n, seed=w.seed)
    assert len(slices) == n
    ref = np.zeros_like(inp.qf)
    ref_lse = np.zeros(inp.qf.shape[:3], np.float32)
    oracle.attn_batched(inp.qf, inp.kf, inp.vf, w.scale, causal=w.causal, slices=slices,
                        out=ref, lse_out=ref_lse)
    ref = ref.reshape(w.B * w.Hq, w.N, w.D)
    ref_lse = ref_lse.reshape(w.B * w.Hq, w.N)
    for s in slices:
        err = float(np.abs(got[s] - ref[s]).max() / np.abs(ref[s]).max())
        assert err <= w.tol, (name, s, err)
        lerr = float(np.abs(lse[s] - ref_lse[s]).max())
        assert lerr <= lse_tol, (name, s, lerr)
    return slices


def test_c3_full_config(pkg, wl, oracle):
    """bf16 non-causal B=4 H=32 N=4096 d=128, inputs N(0,1)/sqrt(2), fp32 LSE."""
    slices = _check(pkg, wl, oracle, "c3", 1e-3)
    assert {0, 31, 96, 127} <= set(slices)


def test_c4_full_config_whole_slices(pkg, wl, oracle):
    """bf16 causal B=1 H=32 N=16384 d=128: six whole slices (all 128 Q tiles
    of each, 64 pairs of very different weight) against the oracle."""
    slices = _check(pkg, wl, oracle, "c4", 1e-3)
    assert {0, 31} <= set(slices)


def test_c5_full_config(pkg, wl, oracle):
    """e4m3 causal GQA B=16 Hq=32 Hkv=8 N=2048 d=128, bf16 output."""
    slices = _check(pkg, wl, oracle, "c5", 1e-2, n=8)
    # Head 0, the last head and the last kv-head group (heads 28-31) of the
    # last batch are always among the checked slices.
    assert {0, 31, 15 * 32, 15 * 32 + 28, 15 * 32 + 31} <= set(slices)
