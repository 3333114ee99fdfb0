"""Shard arithmetic: the exact ranges the reference's layouts produce (`tests/test_sharding.py:29-130` of the
reference holds the same expectations), plus the generalised split{a}{m} layouts."""
import pytest

from multi_modal_parallelism_b200.config import MODES, preset
from multi_modal_parallelism_b200.sharding import (
    all_norm_groups, attn_shard, build_mup_vector, k_grid, kv_replication_map, mlp_shard, parse_split, plan_for,
    ssm_shard, swing_width,
)

D7 = preset("falcon_h1_7b")
D34 = preset("falcon_h1_34b")


def partitions(ranges, total):
    got = sorted(i for r in ranges for i in r)
    assert got == list(range(total))


def test_yaml_dims_match_reference_7b():
    assert D7.in_proj_rows == 2 * 3072 + 2 * 256 + 24 == 6680
    assert D7.conv_rows == 3584
    assert D7.ssm_mults == (0.3535533, 0.25, 0.1767766, 0.5, 0.3535533)


def test_tp4_attention():
    sh = [attn_shard(D7, r, 4) for r in range(4)]
    partitions([s.q_heads for s in sh], 12)
    assert kv_replication_map(D7, 4) == {0: (0, 1), 1: (2, 3)}
    assert {s.kv_replicas for s in sh} == {2}
    assert sh[1].q_rows == slice(384, 768)
    assert sh[1].k_rows == slice(0, 128)
    assert sh[3].o_cols == slice(1152, 1536)


def test_uneven_query_heads_3b():
    d3 = preset("falcon_h1_3b")
    sh = [attn_shard(d3, r, 4) for r in range(4)]
    partitions([s.q_heads for s in sh], 10)
    assert [len(s.q_heads) for s in sh] == [3, 2, 3, 2]
    assert kv_replication_map(d3, 4) == {0: (0, 1), 1: (2, 3)}
    assert [attn_shard(d3, r, 2).q_heads for r in range(2)] == [range(0, 5), range(5, 10)]


def test_two_rank_attention_has_no_replication():
    sh = [attn_shard(D7, r, 2) for r in range(2)]
    partitions([s.q_heads for s in sh], 12)
    assert kv_replication_map(D7, 2) == {0: (0,), 1: (1,)}
    assert sh[1].q_rows == slice(768, 1536) and sh[1].k_rows == slice(128, 256)


def test_tp4_ssm_rows_and_replicated_group():
    sh = [ssm_shard(D7, r, 4, (0, 1, 2, 3)) for r in range(4)]
    partitions([s.heads for s in sh], 24)
    for s in sh:
        assert s.b_rows == slice(6144, 6400) and s.c_rows == slice(6400, 6656)
        assert s.norm_ranks == (0, 1, 2, 3)
        assert s.local_in_rows == (768, 768, 256, 256, 6)
    assert sh[2].z_rows == slice(1536, 2304)
    assert sh[2].x_rows == slice(3072 + 1536, 3072 + 2304)
    assert sh[2].dt_rows == slice(6656 + 12, 6656 + 18)
    assert sh[2].conv_rows == (slice(1536, 2304), slice(3072, 3328), slice(3328, 3584))


def test_two_rank_ssm_norm_pair():
    sh = [ssm_shard(D7, r, 2, (2, 3)) for r in range(2)]
    partitions([s.heads for s in sh], 24)
    assert sh[0].norm_ranks == (2, 3) == sh[1].norm_ranks
    assert sh[1].local_in_rows == (1536, 1536, 256, 256, 12)
    assert sh[1].out_cols == slice(1536, 3072)


def test_34b_group_aware_tp4():
    sh = [ssm_shard(D34, r, 4, (0, 1, 2, 3)) for r in range(4)]
    partitions([s.heads for s in sh], 32)
    assert [list(s.groups) for s in sh] == [[0], [0], [1], [1]]
    assert sh[0].norm_ranks == (0, 1) and sh[3].norm_ranks == (2, 3)
    assert sh[2].b_rows == slice(2 * 4096 + 256, 2 * 4096 + 512)
    assert sh[2].c_rows == slice(2 * 4096 + 2 * 256 + 256, 2 * 4096 + 2 * 256 + 512)
    assert kv_replication_map(D34, 4) == {0: (0,), 1: (1,), 2: (2,), 3: (3,)}
    assert attn_shard(D34, 0, 4).q_heads == range(0, 5)


def test_mup_vector_blocks():
    for G in (1, 2, 4):
        s = ssm_shard(D7, 0, G, tuple(range(G)))
        v = build_mup_vector(D7, s)
        d = 3072 // G
        assert tuple(v.shape) == (1, 2 * d + 2 * 256 + 24 // G)
        assert float(v[0, 0]) == pytest.approx(0.3535533)
        assert float(v[0, d]) == pytest.approx(0.25)
        assert float(v[0, 2 * d]) == pytest.approx(0.1767766)
        assert float(v[0, 2 * d + 256]) == pytest.approx(0.5)
        assert float(v[0, -1]) == pytest.approx(0.3535533)


def test_swing_pool():
    assert (swing_width(0.1, 3072), swing_width(0.4, 3072), swing_width(1.0, 3072)) == (320, 1216, 3072)
    w = 640
    a = mlp_shard(D7, 0, 4, 0.2, None, "attn", 2)
    s = mlp_shard(D7, 2, 4, 0.2, None, "ssm", 0)
    assert (a.w, a.k, s.k) == (w, w, w)
    assert len(a.col_order) == 3072 - w + 2 * w == len(s.col_order)
    assert sorted(a.active_global_cols()) == list(range(0, 3072))
    assert sorted(s.active_global_cols()) == list(range(2 * 3072, 3 * 3072))
    pair = set(range(0, 3072)) | set(range(2 * 3072, 3 * 3072))
    for k in k_grid(w, 128):
        a = mlp_shard(D7, 0, 4, 0.2, k, "attn", 2)
        s = mlp_shard(D7, 2, 4, 0.2, k, "ssm", 0)
        assert a.active_rows + s.active_rows == 2 * 3072
        got = list(a.active_global_cols()) + list(s.active_global_cols())
        assert len(got) == len(set(got)) and set(got) == pair
    assert k_grid(w, 128)[-1] == 2 * w
    t = mlp_shard(D7, 1, 4, 0.0, None)
    assert t.w == 0 and t.active_rows == 3072 and list(t.col_order) == list(range(3072, 6144))


def test_plan_modes():
    p = plan_for("tp1", 0, 1, D7)
    assert p.combine == "none" and p.ssm.norm_ranks == (0,)
    for r in range(4):
        p = plan_for("tp4", r, 4, D7)
        assert p.combine == "allreduce_each" and p.has_attn and p.has_ssm
        p = plan_for("split22", r, 4, D7, swing=0.3)
        assert p.combine == "sum_then_allreduce"
        assert p.has_attn == (r < 2) and p.has_ssm == (r >= 2)
        assert p.mlp.role == ("attn" if r < 2 else "ssm")
        assert p.mlp.partner == (r + 2 if r < 2 else r - 2)
    with pytest.raises(ValueError):
        plan_for("tp4", 0, 4, D7, swing=0.2)


@pytest.mark.parametrize("mode,world", [("split11", 2), ("split13", 4), ("split44", 8), ("split26", 8), ("split22", 4)])
def test_generalised_split_covers_every_head(mode, world):
    a, m = parse_split(mode)
    plans = [plan_for(mode, r, world, D7) for r in range(world)]
    partitions([p.attn.q_heads for p in plans if p.attn is not None], 12)
    partitions([p.ssm.heads for p in plans if p.ssm is not None], 24)
    assert sum(p.has_attn for p in plans) == a and sum(p.has_ssm for p in plans) == m
    # G = 1: one gated-norm group spanning all SSM ranks
    assert all_norm_groups(mode, world, D7) == ([tuple(range(a, world))] if m > 1 else [])
    # uneven splits have no swing pool; every rank computes its plain TP slice of the MLP
    if a != m:
        assert all(p.mlp.w == 0 and p.mlp.role == "tp" for p in plans)


def test_split_rejects_bad_layouts():
    with pytest.raises(ValueError):
        plan_for("split22", 0, 2, D7)  # world mismatch
    with pytest.raises(ValueError):
        plan_for("split31", 0, 4, D7)  # 2 KV heads do not spread over 3 ranks
    with pytest.raises(ValueError):
        plan_for("splitxy", 0, 2, D7)


def test_modes_listed():
    assert {"tp1", "tp4", "tp4_fused", "tp4_streams", "split22", "split11", "split13", "split44"} <= set(MODES)


def test_intermediate_zero_is_mixer_only():
    d = preset("falcon_h1_7b_like")
    assert d.intermediate == 0 and not d.has_mlp
    p = plan_for("tp1", 0, 1, d)
    assert p.mlp.active_rows == 0
