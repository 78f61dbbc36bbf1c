"""Generates tests/golden/*.npz from the oracle (run from the repo root:
``python tests/golden/make_golden.py``).

The reference ships no numeric golden vectors (its lit tests only check IR
structure, test/Attention/fusion.mlir and tiling.mlir), so these fixtures are
produced by the oracle's restatement of lib/Attention/TilingPass.cpp on
seeded inputs, each one cross-checked here against an independent float64
two-pass softmax before it is written.  Shapes follow the reference's own
test inputs: 128x64 with a 128x128 i1 mask (fusion.mlir:11-16) and 64x32 at
tile-size 32 with and without a 64x64 mask (tiling.mlir:12-50), plus the c1
configuration (f32 causal 128x64, scale 1/8, PCG64 seed 0).
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle  # noqa: E402


def case(name, Nq, Nk, D, scale, seed, T=128, mask=None, causal=False):
    rng = np.random.Generator(np.random.PCG64(seed))
    Q = rng.standard_normal((Nq, D), dtype=np.float32)
    K = rng.standard_normal((Nk, D), dtype=np.float32)
    V = rng.standard_normal((Nk, D), dtype=np.float32)
    M = None
    if mask == "random":
        M = rng.random((Nq, Nk)) < 0.25
        M[:, 0] = False
    O, lse = oracle.attn_fused_f32(Q, K, V, scale, mask=M, causal=causal, T=T)
    R, rl = oracle.naive_f64(Q, K, V, scale, mask=M, causal=causal)
    assert np.abs(O - R).max() < 1e-5 and np.abs(lse - rl).max() < 1e-5, name
    out = dict(Q=Q, K=K, V=V, O=O, lse=lse, scale=np.float32(scale), T=np.int64(T),
               causal=np.bool_(causal))
    if M is not None:
        out["mask"] = M
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)


if __name__ == "__main__":
    oracle.build()
    case("c1_f32_causal_128x64", 128, 128, 64, 1 / 8, 0, causal=True)
    case("fusion_masked_128x64", 128, 128, 64, 1 / 8, 20, mask="random")
    case("tiling_t32_64x32", 64, 64, 32, 1 / np.sqrt(32), 21, T=32)
    case("tiling_t32_masked_64x32", 64, 64, 32, 1 / np.sqrt(32), 22, T=32, mask="random")
    case("ragged_200x333x64", 200, 333, 64, 0.125, 23, causal=True)
    print("golden fixtures written")
