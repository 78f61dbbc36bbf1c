"""Named attention workloads and their seeded synthetic inputs.

Each workload is one call of the fused attention op over B x Hq (batch, head)
slices.  Inputs are i.i.d. normal draws from numpy's PCG64 generator (seeded
per workload, Q then K then V), quantised exactly as the GPU path consumes
them: bf16 by round-to-nearest-even, e4m3 with a per-tensor scale amax/448.
No public dataset is involved; these stand in for the prefill shapes named.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class Workload:
    name: str
    dtype: str          # "f32" | "bf16" | "e4m3"
    B: int
    Hq: int
    Hkv: int
    N: int
    D: int
    causal: bool
    seed: int
    std: float = 1.0
    tol: float = 2e-2   # max|O - O_ref| / max|O_ref|

    @property
    def scale(self) -> float:
        return 1.0 / math.sqrt(self.D)

    @property
    def slices(self) -> int:
        return self.B * self.Hq

    def flops(self, slices: int | None = None) -> float:
        """Causal-adjusted attention FLOPs: 4·N²·D per slice, halved if causal."""
        s = self.slices if slices is None else slices
        f = 4.0 * s * self.N * self.N * self.D
        return f / 2 if self.causal else f

    def bytes(self) -> int:
        """Algorithmic HBM bytes: Q, K, V read once, O (+ fp32 LSE) written once."""
        eb = {"f32": 4, "bf16": 2, "e4m3": 1}[self.dtype]
        ob = 4 if self.dtype == "f32" else 2
        q = self.B * self.Hq * self.N * self.D * eb
        kv = 2 * self.B * self.Hkv * self.N * self.D * eb
        o = self.B * self.Hq * self.N * self.D * ob
        lse = self.B * self.Hq * self.N * 4
        return q + kv + o + lse


WORKLOADS = {
    # f32 single-head causal, the reference op's own form (rank-2 f32).
    "c1": Workload("c1_f32_causal_b1h1n128d64", "f32", 1, 1, 1, 128, 64, True, 0, tol=1e-4),
    # bf16 causal multi-head, GPT-2-small-like.
    "c2": Workload("c2_bf16_causal_b8h16n1024d64", "bf16", 8, 16, 16, 1024, 64, True, 1),
    # bf16 non-causal 7B-prefill-like, inputs N(0,1)/sqrt(2).
    "c3": Workload("c3_bf16_nomask_b4h32n4096d128", "bf16", 4, 32, 32, 4096, 128, False, 2,
                   std=1 / math.sqrt(2)),
    # bf16 causal long sequence.
    "c4": Workload("c4_bf16_causal_b1h32n16384d128", "bf16", 1, 32, 32, 16384, 128, True, 3),
    # fp8-e4m3 causal grouped-query attention, bf16 output.
    "c5": Workload("c5_e4m3_causal_gqa_b16hq32hkv8n2048d128", "e4m3", 16, 32, 8, 2048, 128, True,
                   4, tol=6e-2),
}


def round_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 (ties to even) -> float32."""
    x = np.ascontiguousarray(x, np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32)
    return r.view(np.float32)


def quant_e4m3(x: np.ndarray):
    """Per-tensor scale amax/448 and e4m3 codes (RNE, saturating).

    Returns (codes uint8, descale float, dequantised float32).
    """
    import ml_dtypes  # noqa: PLC0415

    x = np.asarray(x, np.float32)
    amax = float(np.max(np.abs(x))) if x.size else 0.0
    descale = np.float32(amax / 448.0 if amax > 0 else 1.0)
    y = np.clip(x / descale, -448.0, 448.0).astype(ml_dtypes.float8_e4m3fn)
    return y.view(np.uint8), float(descale), (y.astype(np.float32) * descale).astype(np.float32)


def quant_e4m3_blocks(x: np.ndarray, block: int = 128):
    """Per-block e4m3 quantisation of [B, H, N, D] along N (blocks of ``block``
    rows, each scaled by its own amax/448).

    Returns (codes uint8 [B,H,N,D], descales float32 [B,H,ceil(N/block)],
    dequantised float32 [B,H,N,D]).
    """
    import ml_dtypes  # noqa: PLC0415

    x = np.asarray(x, np.float32)
    B, H, N, D = x.shape
    nb = -(-N // block)
    pad = np.zeros((B, H, nb * block, D), np.float32)
    pad[:, :, :N] = x
    blocks = pad.reshape(B, H, nb, block, D)
    amax = np.abs(blocks).max(axis=(3, 4))
    descale = np.where(amax > 0, amax / 448.0, 1.0).astype(np.float32)
    y = np.clip(blocks / descale[..., None, None], -448.0, 448.0).astype(ml_dtypes.float8_e4m3fn)
    deq = (y.astype(np.float32) * descale[..., None, None]).reshape(B, H, nb * block, D)[:, :, :N]
    codes = y.view(np.uint8).reshape(B, H, nb * block, D)[:, :, :N]
    return np.ascontiguousarray(codes), descale, np.ascontiguousarray(deq)


def quant_e4m3_heads(x: np.ndarray):
    """Per-(batch, head) e4m3 quantisation of [B, H, N, D].

    Returns (codes uint8, descales float32 [B,H], dequantised float32).
    """
    codes, descale, deq = quant_e4m3_blocks(x, block=x.shape[2])
    return codes, np.ascontiguousarray(descale[:, :, 0]), deq


@dataclass
class Inputs:
    """Host arrays for one workload.

    ``q/k/v`` are what the device receives (float32, bf16-valued float32, or
    e4m3 codes); ``qf/kf/vf`` are the float32 values the oracle consumes.
    """
    q: np.ndarray
    k: np.ndarray
    v: np.ndarray
    qf: np.ndarray
    kf: np.ndarray
    vf: np.ndarray
    descale: tuple = (1.0, 1.0, 1.0)


def make_inputs(w: Workload, B: int | None = None, Hq: int | None = None,
                N: int | None = None, seed: int | None = None) -> Inputs:
    """Seeded inputs for ``w`` (optionally with B / Hq / N overridden for a
    reduced parity case; Hkv shrinks with Hq to keep the group size)."""
    B = w.B if B is None else B
    Hq = w.Hq if Hq is None else Hq
    N = w.N if N is None else N
    Hkv = max(1, Hq * w.Hkv // w.Hq)
    rng = np.random.Generator(np.random.PCG64(w.seed if seed is None else seed))
    shp_q, shp_kv = (B, Hq, N, w.D), (B, Hkv, N, w.D)
    q = (rng.standard_normal(shp_q, dtype=np.float32) * np.float32(w.std)).astype(np.float32)
    k = (rng.standard_normal(shp_kv, dtype=np.float32) * np.float32(w.std)).astype(np.float32)
    v = (rng.standard_normal(shp_kv, dtype=np.float32) * np.float32(w.std)).astype(np.float32)
    if w.dtype == "f32":
        return Inputs(q, k, v, q, k, v)
    if w.dtype == "bf16":
        q, k, v = round_bf16(q), round_bf16(k), round_bf16(v)
        return Inputs(q, k, v, q, k, v)
    (qc, qd, qf), (kc, kd, kf), (vc, vd, vf) = quant_e4m3(q), quant_e4m3(k), quant_e4m3(v)
    return Inputs(qc, kc, vc, qf, kf, vf, (qd, kd, vd))


def to_device(inp: Inputs, w: Workload, device="cuda"):
    """Torch tensors of the device operands."""
    import torch  # noqa: PLC0415

    if w.dtype == "f32":
        cvt = lambda a: torch.from_numpy(a).to(device)  # noqa: E731
    elif w.dtype == "bf16":
        cvt = lambda a: torch.from_numpy(a).to(device).to(torch.bfloat16)  # noqa: E731
    else:
        cvt = lambda a: torch.from_numpy(a).to(device).view(torch.float8_e4m3fn)  # noqa: E731
    return cvt(inp.q), cvt(inp.k), cvt(inp.v)
