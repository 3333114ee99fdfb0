"""Host side of the measurement rows: the algorithmic HBM bytes of a decode step (the roofline column of run.py /
sweep.py rows) reproduce the per-step figure of the 7B-like layer at batch 64, context 2048 (weights 82.0 MB,
KV 134.3 MB, fp32 SSM state 402.7 MB, conv 2.75 MB), and a layout that splits the heads over ranks moves that
total plus only what it replicates (the B/C group on every SSM rank)."""
import pytest

from multi_modal_parallelism_b200.config import preset
from multi_modal_parallelism_b200.measure import step_hbm_bytes
from multi_modal_parallelism_b200.sharding import plan_for


def test_step_bytes_of_the_bench_layer():
    d = preset("falcon_h1_7b_like")
    assert step_hbm_bytes(plan_for("tp1", 0, 1, d), d, 64, 2048) == 621_625_344


@pytest.mark.parametrize("mode,world,ssm_ranks", [("split11", 2, 1), ("split13", 4, 3), ("split22", 4, 2)])
def test_branch_splits_add_only_the_replicated_group_rows(mode, world, ssm_ranks):
    """Each SSM rank beyond the first holds the one B/C group again (its in-projection rows and conv lines)."""
    d = preset("falcon_h1_7b_like")
    B, c = 64, 2048
    one = step_hbm_bytes(plan_for("tp1", 0, 1, d), d, B, c)
    gn = d.n_groups * d.d_state
    per_extra_rank = 2 * gn * d.hidden * 2 + 2 * B * (d.d_conv - 1) * 2 * gn * 2
    total = sum(step_hbm_bytes(plan_for(mode, r, world, d), d, B, c) for r in range(world))
    assert total - one == (ssm_ranks - 1) * per_extra_rank


@pytest.mark.parametrize("world,expected", [(2, "split11"), (4, "split13"), (8, "split26")])
def test_split_by_bytes_puts_the_state_heavy_branch_on_more_ranks(world, expected):
    """At batch 64, context 2048 the fp32 SSM state (402.7 MB) outweighs keys and values (134.3 MB), so the split
    with the lightest busiest rank gives the Mamba-2 branch more ranks; it is the minimum over every split the
    dimensions divide."""
    from multi_modal_parallelism_b200.measure import split_by_bytes

    d = preset("falcon_h1_7b_like")
    pick = split_by_bytes(d, world, 64, 2048)
    assert pick == expected
    worst = {}
    for a in range(1, world):
        mode = f"split{a}{world - a}"
        try:
            worst[mode] = max(step_hbm_bytes(plan_for(mode, r, world, d), d, 64, 2048) for r in range(world))
        except ValueError:
            pass
    assert worst[pick] == min(worst.values())


def test_split_by_bytes_follows_the_keys_when_context_is_long():
    """At context 32768 the keys and values (about 2.1 GB at batch 64) outweigh the state: the pick moves toward
    more attention ranks."""
    from multi_modal_parallelism_b200.measure import split_by_bytes

    d = preset("falcon_h1_7b_like")
    short, long = split_by_bytes(d, 8, 64, 2048), split_by_bytes(d, 8, 64, 32768)
    assert int(long[5]) > int(short[5])  # attention ranks: split{a}{m}


def test_bench_layout_candidates_are_valid_and_rank_independent():
    """bench.py's recipe lists: tp1 in both schedules at N=1; at N>1 the even split, the byte-model split when it
    differs, tp4_fused in both schedules (one with a pushed out-projection); every layout plans on every rank (a
    layout that fails on one rank would leave the others waiting in a collective)."""
    import importlib.util
    from pathlib import Path

    spec = importlib.util.spec_from_file_location("bench_mod", Path(__file__).resolve().parents[1] / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    d = preset("falcon_h1_7b_like")
    assert bench.layout_candidates(d, 1, 64, 2048) == ["tp1", "tp1_chains"]
    assert bench.layout_candidates(d, 4, 64, 2048) == ["split22", "split22_dn", "split13", "split13_dn", "tp4_fused",
                                                       "tp4_fused_chains"]
    assert bench.layout_candidates(d, 2, 64, 2048) == ["split11", "mix8", "mix8_dn", "mix6", "mix6_dn",
                                                       "mix8_chains", "mix8_dn_chains", "mix6_chains",
                                                       "mix6_dn_chains", "tp4_fused", "tp4_fused_chains"]
    assert bench.parse_recipe("mix8_dn_chains") == ("mix8", True, True)
    assert bench.layout_candidates(d, 4, 64, 2048, "p2p_fused") == ["split22", "split13", "tp4_fused"]
    assert bench.parse_recipe("tp4_fused_chains") == ("tp4_fused", True, False)
    assert bench.parse_recipe("split26") == ("split26", False, False)
    assert bench.parse_recipe("mix8_dn") == ("mix8", False, True)
    for world in (1, 2, 4, 8):
        labels = bench.layout_candidates(d, world, 64, 2048)
        assert len(set(labels)) == len(labels)
        for label in labels:
            mode, _, _ = bench.parse_recipe(label)
            for r in range(world):
                plan_for(mode, r, world, d)


def test_mix_by_bytes_balances_the_two_ranks():
    """7B-like layer, batch 64, context 2048: attention (156 MB) plus 8 Mamba-2 heads on rank 0, 16 heads on rank 1:
    314 / 311 MB, against split11's 156 / 465 MB."""
    from multi_modal_parallelism_b200.measure import mix_by_bytes

    d = preset("falcon_h1_7b_like")
    assert mix_by_bytes(d, 64, 2048) == 8
    per = [step_hbm_bytes(plan_for("mix8", r, 2, d), d, 64, 2048) for r in range(2)]
    assert abs(per[0] - per[1]) < 0.01 * sum(per)
    assert sum(per) - step_hbm_bytes(plan_for("tp1", 0, 1, d), d, 64, 2048) < 0.01 * sum(per)  # only B/C replicated
    assert mix_by_bytes(d.replace(n_groups=24), 64, 2048) is not None
