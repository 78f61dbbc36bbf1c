"""The oracle (CPU restatement of the reference's TilingPass lowering) pinned
against the committed golden fixtures, known answers and a float64 softmax."""
import glob
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "*.npz"))),
                         ids=lambda p: os.path.basename(p))
def test_golden_fixture_bitwise(oracle, path):
    g = np.load(path)
    mask = g["mask"] if "mask" in g.files else None
    O, lse = oracle.attn_fused_f32(g["Q"], g["K"], g["V"], float(g["scale"]), mask=mask,
                                   causal=bool(g["causal"]), T=int(g["T"]))
    assert np.array_equal(O, g["O"])
    assert np.array_equal(lse, g["lse"])


def test_golden_c1_matches_workload_inputs(oracle, wl):
    g = np.load(os.path.join(GOLDEN, "c1_f32_causal_128x64.npz"))
    inp = wl.make_inputs(wl.WORKLOADS["c1"])
    assert np.array_equal(inp.q[0, 0], g["Q"]) and np.array_equal(inp.v[0, 0], g["V"])


def test_uniform_v_gives_v_row(oracle):
    rng = np.random.default_rng(1)
    Q = rng.standard_normal((128, 64)).astype(np.float32)
    K = rng.standard_normal((256, 64)).astype(np.float32)
    V = np.tile(rng.standard_normal((1, 64)).astype(np.float32), (256, 1))
    O, _ = oracle.attn_fused_f32(Q, K, V, 0.125, causal=True)
    assert np.abs(O - V[:1]).max() < 1e-5


def test_one_hot_scores_select_value_row(oracle):
    D = 32
    K = np.eye(64, D, dtype=np.float32) * 30.0  # key j is a large basis vector
    Q = np.eye(64, D, dtype=np.float32)[[3, 7, 11]]
    V = np.arange(64 * D, dtype=np.float32).reshape(64, D)
    O, _ = oracle.attn_fused_f32(Q, K, V, 1.0)
    for i, j in enumerate([3, 7, 11]):
        assert np.abs(O[i] - V[j]).max() < 1e-3 * np.abs(V[j]).max()


def test_single_tile_equals_two_pass_softmax(oracle):
    rng = np.random.default_rng(2)
    Q, K, V = (rng.standard_normal((128, 64)).astype(np.float32) for _ in range(3))
    O, lse = oracle.attn_fused_f32(Q, K, V, 0.125)
    R, rl = oracle.naive_f64(Q, K, V, 0.125)
    assert np.abs(O - R).max() < 1e-6 and np.abs(lse - rl).max() < 1e-6


def test_causal_equals_explicit_i1_mask(oracle):
    rng = np.random.default_rng(3)
    Q, K, V = (rng.standard_normal((256, 64)).astype(np.float32) for _ in range(3))
    M = np.triu(np.ones((256, 256), bool), 1)
    a, la = oracle.attn_fused_f32(Q, K, V, 0.125, causal=True)
    b, lb = oracle.attn_fused_f32(Q, K, V, 0.125, mask=M)
    assert np.array_equal(a, b) and np.array_equal(la, lb)


def test_fully_masked_row_is_nan_like_reference(oracle):
    """The reference computes exp(-inf - -inf) = NaN for a row masked over all
    keys (TilingPass.cpp:299-305); the restatement keeps that behaviour."""
    rng = np.random.default_rng(4)
    Q, K, V = (rng.standard_normal((64, 32)).astype(np.float32) for _ in range(3))
    M = np.zeros((64, 64), bool)
    M[5] = True
    O, _ = oracle.attn_fused_f32(Q, K, V, 0.2, mask=M, T=32)
    assert np.isnan(O[5]).all() and np.isfinite(np.delete(O, 5, 0)).all()


@pytest.mark.parametrize("causal", [False, True])
def test_batched_gqa_matches_per_slice(oracle, causal):
    rng = np.random.default_rng(5)
    Q = rng.standard_normal((2, 4, 200, 64)).astype(np.float32)
    K = rng.standard_normal((2, 2, 200, 64)).astype(np.float32)
    V = rng.standard_normal((2, 2, 200, 64)).astype(np.float32)
    O, lse = oracle.attn_batched(Q, K, V, 0.125, causal=causal, nthreads=2)
    for b in range(2):
        for h in range(4):
            r, rl = oracle.attn_fused_f32(Q[b, h], K[b, h // 2], V[b, h // 2], 0.125,
                                          causal=causal)
            assert np.array_equal(O[b, h], r) and np.array_equal(lse[b, h], rl)


def test_tile_sample_covers_exactly_listed_tiles(oracle):
    rng = np.random.default_rng(6)
    Q = rng.standard_normal((1, 2, 512, 32)).astype(np.float32)
    K = rng.standard_normal((1, 2, 512, 32)).astype(np.float32)
    full, _ = oracle.attn_batched(Q, K, K, 0.2, causal=True)
    part = np.full_like(full, 7.0)
    oracle.attn_batched(Q, K, K, 0.2, causal=True, slices=[1], tile_offset=1, tile_stride=2,
                        out=part)
    assert np.array_equal(part[0, 1, 128:256], full[0, 1, 128:256])
    assert np.array_equal(part[0, 1, 384:512], full[0, 1, 384:512])
    assert (part[0, 0] == 7.0).all() and (part[0, 1, :128] == 7.0).all()


def test_quantisation_helpers(wl):
    x = np.array([1.0, 1.00390625, 1.01171875, -3.3e38], np.float32)
    r = wl.round_bf16(x)
    assert r[0] == 1.0 and r[1] == 1.0 and r[2] == 1.015625
    codes, descale, deq = wl.quant_e4m3(np.array([0.5, -2.0, 4.0], np.float32))
    assert abs(descale - 4.0 / 448) < 1e-9 and abs(deq[2] - 4.0) < 1e-6


def test_empty_extents_follow_the_loop_nest(oracle):
    """No key: the KV loop never runs, O_acc = 0 and l = 0, so O = 0/0 = NaN and
    LSE = -inf; no query row: nothing is computed."""
    rng = np.random.default_rng(3)
    q = rng.standard_normal((1, 2, 5, 64)).astype(np.float32)
    none = np.zeros((1, 2, 0, 64), np.float32)
    o, lse = oracle.attn_batched(q, none, none, 0.125)
    assert np.isnan(o).all() and np.isneginf(lse).all()
    o2, l2 = oracle.attn_fused_f32(q[0, 0], none[0, 0], none[0, 0], 0.125)
    assert np.isnan(o2).all() and np.isneginf(l2).all()
    k = rng.standard_normal((1, 2, 7, 64)).astype(np.float32)
    o3, l3 = oracle.attn_batched(none, k, k, 0.125)
    assert o3.shape == (1, 2, 0, 64) and l3.shape == (1, 2, 0)
