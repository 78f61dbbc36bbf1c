"""The fusion pass on torch.fx graphs (FuseAttentionPattern,
lib/Attention/FusionPass.cpp:95-168): which chains it rewrites into one
attention.fused call, which it leaves alone, and (on a B200) that the
rewritten graph computes what the unfused one did."""
import math

import numpy as np
import pytest
import torch


@pytest.fixture(scope="module")
def fusion(pkg):
    from mlir_flashattention_b200 import fusion as f

    return f


def _calls(gm, target):
    return [n for n in gm.graph.nodes if n.op == "call_function" and n.target is target]


def _ops(gm):
    return [(n.op, n.target) for n in gm.graph.nodes if n.op in ("call_function", "call_method")]


def unfused_masked(q, k, v, mask):
    # The reference's lit input (test/Attention/fusion.mlir): QKᵀ, scale,
    # mask select, softmax, P·V.
    s = q @ k.transpose(-2, -1)
    s = s * 0.125
    s = s.masked_fill(mask, float("-inf"))
    p = torch.softmax(s, dim=-1)
    return p @ v


def unfused_div(q, k, v):
    s = torch.matmul(q, k.transpose(-1, -2)) / math.sqrt(64)
    return torch.nn.functional.softmax(s, dim=-1) @ v


def unfused_where_keep(q, k, v, keep):
    s = 0.5 * (q @ k.mT)
    s = torch.where(keep, s, -3.4028234663852886e38)  # -FLT_MAX, the reference test's "-inf"
    return s.softmax(-1).matmul(v)


def test_masked_chain_becomes_one_fused_call(fusion):
    gm = torch.fx.symbolic_trace(unfused_masked)
    assert fusion.fuse_attention(gm) == 1
    calls = _calls(gm, fusion.attention_fused)
    assert len(calls) == 1
    q, k, v, scale, mask = calls[0].args
    assert [a.target for a in (q, k, v, mask)] == ["q", "k", "v", "mask"]
    assert scale == 0.125
    # Nothing of the chain is left: no matmul, transpose, scale, select or softmax.
    assert _ops(gm) == [("call_function", fusion.attention_fused)]


def test_division_scale_and_functional_softmax(fusion):
    gm = torch.fx.symbolic_trace(unfused_div)
    assert fusion.fuse_attention(gm) == 1
    (call,) = _calls(gm, fusion.attention_fused)
    assert call.args[3] == pytest.approx(1 / 8) and call.args[4] is None


def test_keep_mask_is_negated(fusion):
    """where(keep, s, -FLT_MAX) masks the entries where keep is False."""
    gm = torch.fx.symbolic_trace(unfused_where_keep)
    assert fusion.fuse_attention(gm) == 1
    (call,) = _calls(gm, fusion.attention_fused)
    mask = call.args[4]
    assert mask.target is torch.logical_not and mask.args[0].target == "keep"
    assert call.args[3] == 0.5


def test_two_chains_and_rank_two_operands(fusion):
    def two(q, k, v):
        a = torch.softmax((q @ k.t()) * 0.25, dim=-1) @ v
        b = torch.softmax((k @ q.t()) * 0.5, dim=-1) @ v
        return a + b

    gm = torch.fx.symbolic_trace(two)
    assert fusion.fuse_attention(gm) == 2
    assert len(_calls(gm, fusion.attention_fused)) == 2


@pytest.mark.parametrize("fn", [
    # softmax over another dim
    lambda q, k, v: torch.softmax(q @ k.transpose(-2, -1) * 0.1, dim=0) @ v,
    # no scale op (the reference pattern needs one)
    lambda q, k, v: torch.softmax(q @ k.transpose(-2, -1), dim=-1) @ v,
    # K not transposed
    lambda q, k, v: torch.softmax(q @ k * 0.1, dim=-1) @ v,
    # scale is a tensor, not a constant
    lambda q, k, v: torch.softmax(q @ k.transpose(-2, -1) * q.sum(), dim=-1) @ v,
    # masked with a finite value other than -FLT_MAX
    lambda q, k, v: torch.softmax((q @ k.transpose(-2, -1) * 0.1).masked_fill(q > 0, -1e4),
                                  dim=-1) @ v,
    # softmax with a dtype conversion
    lambda q, k, v: torch.softmax(q @ k.transpose(-2, -1) * 0.1, dim=-1,
                                  dtype=torch.float64) @ v,
])
def test_non_attention_chains_are_left_alone(fusion, fn):
    gm = torch.fx.symbolic_trace(fn)
    before = _ops(gm)
    assert fusion.fuse_attention(gm) == 0
    assert _ops(gm) == before


def test_intermediate_with_another_user_is_not_fused(fusion):
    """The probabilities are returned as well: erasing the softmax would lose
    them, so the chain stays (the reference erases regardless)."""
    def also_probs(q, k, v):
        p = torch.softmax(q @ k.transpose(-2, -1) * 0.1, dim=-1)
        return p @ v, p

    gm = torch.fx.symbolic_trace(also_probs)
    assert fusion.fuse_attention(gm) == 0


def test_shared_transpose_is_kept(fusion):
    """Kᵀ read elsewhere survives the rewrite; the rest of the chain goes."""
    def shared(q, k, v):
        kt = k.transpose(-2, -1)
        return torch.softmax(q @ kt * 0.1, dim=-1) @ v, kt

    gm = torch.fx.symbolic_trace(shared)
    assert fusion.fuse_attention(gm) == 1
    targets = [t for _, t in _ops(gm)]
    assert "transpose" in targets and torch.softmax not in targets


def test_leading_dims_flattened_for_the_op(fusion, monkeypatch):
    """Ranks other than 2 and 4 reach the op as [1, H, N, D] (leading dims
    flattened into heads) and come back in q's shape; mismatched leading
    dims are a VerifyError."""
    import mlir_flashattention_b200 as pkg_mod

    seen = {}

    def fake_fused(q, k, v, scale, mask=None):
        seen.update(q=tuple(q.shape), k=tuple(k.shape), mask=None if mask is None else tuple(mask.shape))
        return torch.zeros(q.shape)

    monkeypatch.setattr(pkg_mod, "fused", fake_fused)
    q = torch.zeros(3, 5, 40, 64)[0]          # rank 3: [5, 40, 64]
    k = v = torch.zeros(5, 48, 64)
    out = fusion.attention_fused(q, k, v, 0.1, torch.zeros(5, 40, 48, dtype=torch.bool))
    assert seen == {"q": (1, 5, 40, 64), "k": (1, 5, 48, 64), "mask": (1, 5, 40, 48)}
    assert tuple(out.shape) == (5, 40, 64)
    q5 = torch.zeros(2, 3, 4, 40, 64)         # rank 5, 2-D mask kept
    out = fusion.attention_fused(q5, torch.zeros(2, 3, 4, 48, 64), torch.zeros(2, 3, 4, 48, 64),
                                 0.1, torch.zeros(40, 48, dtype=torch.bool))
    assert seen["q"] == (1, 24, 40, 64) and seen["mask"] == (40, 48)
    assert tuple(out.shape) == (2, 3, 4, 40, 64)
    with pytest.raises(pkg_mod.VerifyError):
        fusion.attention_fused(q, torch.zeros(4, 48, 64), torch.zeros(4, 48, 64), 0.1)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,tol", [(torch.bfloat16, 2e-2), (torch.float32, 1e-4)])
def test_fused_graph_matches_unfused_graph(pkg, fusion, dtype, tol):
    """The rewritten graph runs the B200 kernel (launch counter moves) and
    gives the unfused graph's result: causal mask as a dense i1 mask
    (classified and run on the causal kernel), rank-4 operands."""
    g = torch.Generator(device="cuda").manual_seed(70)
    B, H, N, D = 2, 4, 384, 64
    q, k, v = (torch.randn((B, H, N, D), generator=g, device="cuda").to(dtype) for _ in range(3))
    mask = torch.triu(torch.ones(N, N, dtype=torch.bool, device="cuda"), diagonal=1)
    ref = unfused_masked(q.float(), k.float(), v.float(), mask)
    gm = torch.fx.symbolic_trace(unfused_masked)
    assert fusion.fuse_attention(gm) == 1
    before = pkg.launch_count()
    out = gm(q, k, v, mask)
    torch.cuda.synchronize()
    pkg.check_status(0)
    assert pkg.launch_count() > before
    assert out.dtype == dtype and out.shape == ref.shape
    err = (out.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err <= tol


@pytest.mark.gpu
def test_fused_graph_random_mask_and_keep_form(pkg, fusion):
    """A random dense mask (the dense-mask kernel) given in the keep form
    (where(keep, s, -FLT_MAX)), rank-2 operands with a ragged N."""
    g = torch.Generator(device="cuda").manual_seed(71)
    N, D = 300, 128
    q, k, v = (torch.randn((N, D), generator=g, device="cuda").to(torch.bfloat16) for _ in range(3))
    keep = torch.rand((N, N), generator=g, device="cuda") < 0.7
    keep[:, 0] = True  # every row keeps its first key (no all-masked first tile)
    ref = unfused_where_keep(q.float(), k.float(), v.float(), keep)
    gm = torch.fx.symbolic_trace(unfused_where_keep)
    assert fusion.fuse_attention(gm) == 1
    out = gm(q, k, v, keep)
    torch.cuda.synchronize()
    pkg.check_status(0)
    err = (out.float() - ref).abs().max().item() / ref.abs().max().item()
    assert np.isfinite(err) and err <= 2e-2


@pytest.mark.gpu
def test_fused_graph_rank3_operands(pkg, fusion):
    """[H, N, D] operands (no batch dim) through the fused graph."""
    g = torch.Generator(device="cuda").manual_seed(72)
    H, N, D = 6, 256, 64
    q, k, v = (torch.randn((H, N, D), generator=g, device="cuda").to(torch.bfloat16) for _ in range(3))
    ref = unfused_div(q.float(), k.float(), v.float())
    gm = torch.fx.symbolic_trace(unfused_div)
    assert fusion.fuse_attention(gm) == 1
    out = gm(q, k, v)
    torch.cuda.synchronize()
    pkg.check_status(0)
    assert out.shape == (H, N, D)
    assert (out.float() - ref).abs().max().item() / ref.abs().max().item() <= 2e-2
