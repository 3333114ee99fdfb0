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
