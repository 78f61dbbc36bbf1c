"""The causal KV-split plan (CPU: attn_rt_causal_split needs no GPU).

The runtime replays its persistent work order on the host and splits the
heaviest Q-tile pairs of causal calls only when there are too few pairs per
SM for the snake order to balance.  Pinned here on the benchmark shapes for a
148-SM B200.
"""


def test_split_only_where_pairs_per_sm_are_few(pkg):
    f = pkg.lib().attn_rt_causal_split
    # c4 on one GPU (32 heads) and its share on 2 and 4 GPUs: no split.
    assert f(32, 16384, 16384, 148) == 0
    assert f(16, 16384, 16384, 148) == 0
    assert f(8, 16384, 16384, 148) == 0
    # Its share on 8 GPUs (4 heads, 256 pairs on 148 SMs): at most the few
    # heaviest pair indices split (each half costs more than it saves).
    assert 0 <= f(4, 16384, 16384, 148) <= 4
    # One head of N = 16384 (64 pairs on 148 SMs): about half the pairs split.
    assert 16 <= f(1, 16384, 16384, 148) <= 48
    # c2 and c5 on one GPU: enough pairs.
    assert f(128, 1024, 1024, 148) == 0
    assert f(512, 2048, 2048, 148) == 0
    # One slice of N = 32768: most pairs split.
    assert f(1, 32768, 32768, 148) > 64


def test_split_plan_rejects_bad_shapes(pkg):
    f = pkg.lib().attn_rt_causal_split
    assert f(0, 1024, 1024, 148) == 0
    assert f(4, 0, 1024, 148) == 0
    assert f(4, 1024, 1024, 0) == 0
    assert f(4, 128, 128, 148) == 0  # one pair per slice: nothing to split
