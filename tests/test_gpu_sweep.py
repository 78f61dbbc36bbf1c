"""Seeded random sweep over the tensor-core kernel's shape space against the
oracle: batch and head counts, grouped-query ratios, ragged and unequal
Nq / Nk (including lengths below one tile), head_dim 64 / 128, no mask /
causal, bf16 / f16 / e4m3 inputs and bf16 / f16 / f32 outputs.  Each case is
small enough for the oracle to finish in well under a second; the seed fixes
the cases.  Tolerances as in the other parity tests (bf16 2e-2, f16 1e-2,
e4m3 6e-2 of max|O|; LSE 1e-3, e4m3 1e-2).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _cases(n=24, seed=2024):
    rng = np.random.default_rng(seed)
    out = []
    for i in range(n):
        dt = ["bf16", "f16", "e4m3"][i % 3]
        D = 128 if dt == "e4m3" else int(rng.choice([64, 128]))
        Hkv = int(rng.integers(1, 4))
        group = int(rng.choice([1, 2, 4]))
        B = int(rng.integers(1, 3))
        Nq = int(rng.choice([int(rng.integers(1, 128)), int(rng.integers(128, 1200))]))
        Nk = Nq if rng.random() < 0.5 else int(rng.integers(1, 1200))
        causal = bool(rng.random() < 0.5)
        out_kind = ["same", "f32"][int(rng.random() < 0.3)]
        padded = bool(rng.random() < 0.3)
        out.append((i, dt, B, Hkv * group, Hkv, Nq, Nk, D, causal, out_kind, padded))
    return out


@pytest.mark.parametrize("case", _cases(), ids=lambda c: (f"{c[0]}-{c[1]}-B{c[2]}H{c[3]}kv{c[4]}-{c[5]}x{c[6]}-d{c[7]}-"
                                   f"{'causal' if c[8] else 'nomask'}-{c[9]}{'-padded' if c[10] else ''}"))
def test_random_shape(pkg, wl, oracle, case):
    i, dt, B, Hq, Hkv, Nq, Nk, D, causal, out_kind, padded = case
    rng = np.random.Generator(np.random.PCG64(1000 + i))
    q = rng.standard_normal((B, Hq, Nq, D), dtype=np.float32)
    k = rng.standard_normal((B, Hkv, Nk, D), dtype=np.float32)
    v = rng.standard_normal((B, Hkv, Nk, D), dtype=np.float32)
    descale = (1.0, 1.0, 1.0)

    def place(t):
        # Padded rows (64 extra elements, a 16-byte multiple for every type):
        # the operand is a strided view, not a contiguous tensor.
        if not padded:
            return t
        big = torch.zeros(t.shape[:-1] + (t.shape[-1] + 64,), dtype=t.dtype, device=t.device)
        big[..., :t.shape[-1]] = t
        return big[..., :t.shape[-1]]

    if dt == "bf16":
        qf, kf, vf = (wl.round_bf16(a) for a in (q, k, v))
        tq, tk, tv = (place(torch.from_numpy(a).cuda().to(torch.bfloat16)) for a in (qf, kf, vf))
        tol, ltol = 2e-2, 1e-3
    elif dt == "f16":
        qf, kf, vf = (a.astype(np.float16).astype(np.float32) for a in (q, k, v))
        tq, tk, tv = (place(torch.from_numpy(a).cuda().to(torch.float16)) for a in (qf, kf, vf))
        tol, ltol = 1e-2, 1e-3
    else:
        (q8, qd, qf), (k8, kd, kf), (v8, vd, vf) = (wl.quant_e4m3(a) for a in (q, k, v))
        tq, tk, tv = (place(torch.from_numpy(a).cuda()).view(torch.float8_e4m3fn) for a in (q8, k8, v8))
        descale = (qd, kd, vd)
        tol, ltol = 6e-2, 1e-2
    out = None
    if out_kind == "f32":
        out = place(torch.empty((B, Hq, Nq, D), dtype=torch.float32, device="cuda"))
    L = torch.empty((B, Hq, Nq), dtype=torch.float32, device="cuda")
    scale = D ** -0.5
    o = pkg.fused(tq, tk, tv, scale, output=out, causal=causal, lse=L, q_descale=descale[0],
                  k_descale=descale[1], v_descale=descale[2])
    pkg.check_status(0)
    ref, ref_lse = oracle.attn_batched(qf, kf, vf, scale, causal=causal)
    got = o.float().cpu().numpy()
    lse = L.cpu().numpy()
    # Causal rows past the last key (Nq > Nk) see keys [0, Nk); rows with no
    # key at all do not occur here (Nk >= 1 and key 0 is always visible).
    assert np.isfinite(got).all() and np.isfinite(lse).all()
    err = float(np.abs(got - ref).max() / np.abs(ref).max())
    assert err <= tol, err
    assert (np.abs(lse - ref_lse) <= ltol + 1e-4 * np.abs(ref_lse)).all()
