"""Every parallel layout on 2 (and, where visible, 4) GPUs through the harness entry point
(`run.py --check`): one process per GPU over NCCL, rank outputs bitwise identical across ranks and within
tolerance of the fp32 layer on the full weights and states. Skipped when fewer GPUs are visible."""
import os
import re
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def ngpu() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_check(world, mode, tmp_path, extra=()):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           "-m", "multi_modal_parallelism_b200.run", "--mode", mode, "--dims-yaml", "falcon_h1_7b_like",
           "--batch", "16", "--ctx", "512", "--variant", "graph", "--n-warm", "3", "--n-iter", "10", "--check",
           "--out", str(tmp_path / "runs.csv"), "--correctness-out", str(tmp_path / "corr.csv"), *extra]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "600", *cmd], cwd=ROOT, env=env, capture_output=True, text=True)
    out = r.stdout + r.stderr
    m = re.search(r"\[check\].*pass=(True|False)", out)
    assert r.returncode == 0 and m and m.group(1) == "True", out[-3000:]
    return out


@pytest.mark.skipif(ngpu() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["split11", "tp4", "tp4_fused", "tp4_streams"])
def test_two_gpu_layouts(mode, tmp_path):
    run_check(2, mode, tmp_path)


@pytest.mark.skipif(ngpu() < 2, reason="needs 2 GPUs")
def test_two_gpu_full_layer_with_mlp(tmp_path):
    run_check(2, "split11", tmp_path, ("--dims-yaml", "falcon_h1_7b", "--swing", "0.2"))


@pytest.mark.skipif(ngpu() < 4, reason="needs 4 GPUs")
@pytest.mark.parametrize("mode", ["split22", "split13", "tp4", "tp4_fused"])
def test_four_gpu_layouts(mode, tmp_path):
    run_check(4, mode, tmp_path)


@pytest.mark.skipif(ngpu() < 8, reason="needs 8 GPUs")
@pytest.mark.parametrize("mode", ["split44", "split26", "tp4_fused"])
def test_eight_gpu_layouts(mode, tmp_path):
    run_check(8, mode, tmp_path)


def run_prefill_check(world, mode):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           str(ROOT / "tests" / "_prefill_ranks.py"), "--mode", mode]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "600", *cmd], cwd=ROOT, env=env, capture_output=True, text=True)
    out = r.stdout + r.stderr
    m = re.search(r"\[prefill-check\].*pass=(True|False)", out)
    assert r.returncode == 0 and m and m.group(1) == "True", out[-3000:]


@pytest.mark.skipif(ngpu() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["split11", "tp4", "tp4_fused"])
def test_two_gpu_prefill(mode):
    """Prefill (and the decode step after it) in each layout equals the single-rank prefill."""
    run_prefill_check(2, mode)


@pytest.mark.skipif(ngpu() < 4, reason="needs 4 GPUs")
@pytest.mark.parametrize("mode", ["split22", "tp4_fused"])
def test_four_gpu_prefill(mode):
    run_prefill_check(4, mode)


@pytest.mark.skipif(ngpu() < 8, reason="needs 8 GPUs")
@pytest.mark.parametrize("mode", ["split44", "tp4_fused"])
def test_eight_gpu_prefill(mode):
    run_prefill_check(8, mode)


def run_script_check(world, script, tag, mode):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()), str(ROOT / "tests" / script), "--mode", mode]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "600", *cmd], cwd=ROOT, env=env, capture_output=True, text=True)
    out = r.stdout + r.stderr
    m = re.search(rf"\[{tag}\].*pass=(True|False)", out)
    assert r.returncode == 0 and m and m.group(1) == "True", out[-3000:]


@pytest.mark.run_last
@pytest.mark.skipif(ngpu() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("world,mode", [(2, "tp"), (2, "attn_dp"), (4, "attn_dp"), (8, "tp"), (8, "attn_dp")])
def test_gdn_stack_layouts(world, mode):
    """The Gated DeltaNet stack at N ranks: ranks bitwise equal, within tolerance of one rank."""
    if ngpu() < world:
        pytest.skip(f"needs {world} GPUs")
    run_script_check(world, "_qwen35_ranks.py", "qwen35-check", mode)


@pytest.mark.run_last
@pytest.mark.skipif(ngpu() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("world,mode", [(2, "sg11"), (2, "tp"), (4, "sg22"), (8, "sg44")])
def test_mamba2_continuous_batching_layouts(world, mode):
    """The pure Mamba-2 layer under continuous batching at N ranks (SSM/gate split and tp)."""
    if ngpu() < world:
        pytest.skip(f"needs {world} GPUs")
    run_script_check(world, "_mamba2_ranks.py", "mamba2-check", mode)


@pytest.mark.run_last
@pytest.mark.skipif(ngpu() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_allreduce(world):
    """The peer-memory all-reduce fused with residual and norm: bit-exact sums, graph replays equal eager."""
    if ngpu() < world:
        pytest.skip(f"needs {world} GPUs")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()), str(ROOT / "tests" / "_p2p_ranks.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "300", *cmd], cwd=ROOT, env=env, capture_output=True, text=True)
    out = r.stdout + r.stderr
    m = re.search(r"\[p2p-check\].*pass=(True|False)", out)
    assert r.returncode == 0 and m and m.group(1) == "True", out[-3000:]


@pytest.mark.run_last
@pytest.mark.skipif(ngpu() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("impl", ["p2p", "p2p_fused"])
@pytest.mark.parametrize("world,mode", [(2, "split11"), (2, "tp4_fused"), (4, "split22"), (8, "split44")])
def test_layouts_with_peer_allreduce(world, mode, impl, tmp_path):
    """Every rank of the layer with the peer-memory all-reduce (and with the GEMMs pushing their tiles): bitwise
    equal across ranks, within tolerance of fp32."""
    if ngpu() < world:
        pytest.skip(f"needs {world} GPUs")
    run_check(world, mode, tmp_path, ("--ar-impl", impl, "--dims-yaml", "falcon_h1_7b", "--swing", "0.2")
              if mode.startswith("split") else ("--ar-impl", impl))


@pytest.mark.run_last
@pytest.mark.skipif(ngpu() < 1, reason="needs a GPU")
@pytest.mark.parametrize("world,mode,extra", [(1, "tp1", ()), (2, "tp4_fused", ()), (2, "tp4_fused", ("--ar-impl", "p2p")),
                                              (4, "tp4_fused", ())])
def test_branch_chains_schedule(world, mode, extra, tmp_path):
    """The branch-chains decode schedule (the attention chain on a side stream, the Mamba-2 out-projection adding
    its partial) through run.py --check: within tolerance of the fp32 layer, ranks bitwise equal."""
    if ngpu() < world:
        pytest.skip(f"needs {world} GPUs")
    run_check(world, mode, tmp_path, ("--branch-chains", *extra))


@pytest.mark.run_last
@pytest.mark.skipif(ngpu() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("extra", [(), ("--ar-impl", "p2p"), ("--ar-impl", "p2p_fused"), ("--branch-chains",),
                                   ("--branch-chains", "--defer-norm")])
def test_two_gpu_mix_layout(extra, tmp_path):
    """mix8: rank 0 the attention branch and 8 Mamba-2 heads (fused projections), rank 1 the other 16 heads."""
    run_check(2, "mix8", tmp_path, extra)


@pytest.mark.run_last
@pytest.mark.skipif(ngpu() < 2, reason="needs 2 GPUs")
def test_two_gpu_mix_prefill():
    """Prefill (and the decode step after it) in mix8 equals the single-rank prefill."""
    run_prefill_check(2, "mix8")


@pytest.mark.run_last
@pytest.mark.skipif(ngpu() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("world,mode", [(2, "mix8"), (4, "split13"), (4, "split22"), (8, "split26")])
def test_deferred_norm_statistic(world, mode, tmp_path):
    """Mamba-2-only ranks overlap the gated norm's row-statistic all-reduce with their out-projection."""
    if ngpu() < world:
        pytest.skip(f"needs {world} GPUs")
    run_check(world, mode, tmp_path, ("--defer-norm",))
