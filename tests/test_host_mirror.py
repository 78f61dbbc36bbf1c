"""Host-side mirror of attention.fused: verifier messages, mask
classification and slice sharding (CPU only)."""
import pytest

torch = pytest.importorskip("torch")


def test_verifier_messages_match_reference(pkg):
    # AttentionOps.cpp:48-56 wording; shapes are checked before any device use.
    q = torch.zeros(128, 64)
    with pytest.raises(pkg.VerifyError, match="K head_dim must equal Q head_dim"):
        pkg.fused(q, torch.zeros(128, 32), torch.zeros(128, 64), 0.1)
    with pytest.raises(pkg.VerifyError, match="V seq_len must equal K seq_len"):
        pkg.fused(q, torch.zeros(128, 64), torch.zeros(64, 64), 0.1)
    with pytest.raises(pkg.VerifyError, match="output seq_q must equal Q seq_q"):
        pkg.fused(q, q, q, 0.1, output=torch.zeros(64, 64))
    with pytest.raises(pkg.VerifyError, match="output head_dim must equal Q head_dim"):
        pkg.fused(q, q, q, 0.1, output=torch.zeros(128, 32))
    with pytest.raises(pkg.VerifyError, match="Q must be rank-2"):
        pkg.fused(torch.zeros(2, 128, 64), q, q, 0.1)


def test_host_tensors_are_rejected_not_computed(pkg):
    q = torch.zeros(128, 64)
    with pytest.raises(pkg.VerifyError, match="CUDA tensor"):
        pkg.fused(q, q, q, 0.1)


def test_classify_mask(pkg):
    n = 64
    causal = torch.ones(n, n, dtype=torch.bool).triu(1)
    assert pkg.classify_mask(torch.zeros(n, n, dtype=torch.bool)) == pkg.MASK_NONE
    assert pkg.classify_mask(causal) == pkg.MASK_CAUSAL
    dense = causal.clone()
    dense[3, 1] = True
    assert pkg.classify_mask(dense) == pkg.MASK_DENSE


@pytest.mark.parametrize("n,world", [(32, 8), (33, 8), (7, 2), (1, 4)])
def test_shards_cover_all_slices_once(pkg, n, world):
    seen = []
    for r in range(world):
        a, b = pkg.shard_slices(n, world, r)
        seen.extend(range(a, b))
    assert seen == list(range(n))
