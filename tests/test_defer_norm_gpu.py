"""The deferred gated RMSNorm on a B200: mmp_gated_rmsnorm's deferred mode (partial sums of squares plus the
gated, weighted values unnormalised) followed by mmp_scale_rows equals the one-pass norm over the whole row, for a
row split in two column blocks as two ranks would hold it (the sums of both blocks added, each block projected and
scaled), within the suite's bf16 tolerance. Also the scaling of a projected product, as the layer uses it."""
import numpy as np
import pytest
import torch

from multi_modal_parallelism_b200 import kernels as K

pytestmark = [pytest.mark.gpu, pytest.mark.run_last]
DEV = torch.device("cuda", 0)
BF = torch.bfloat16


def close(got, ref, tol_abs=2e-2, tol_rel=1e-2):
    got, ref = got.float().cpu().numpy().astype(np.float64), ref.float().cpu().numpy().astype(np.float64)
    scale = max(1.0, float(np.abs(ref).max()))
    assert float(np.abs(got - ref).max()) <= tol_abs * scale
    assert float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)) <= tol_rel


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    K.check_device_errors(DEV)


@pytest.mark.parametrize("rows,D,cut", [(64, 3072, 1024), (3, 384, 128), (17, 2048, 1024)])
def test_deferred_norm_equals_one_pass_norm(rows, D, cut):
    g = torch.Generator().manual_seed(rows + D)
    y = (torch.randn(rows, D, generator=g) * 3).to(BF).to(DEV)
    z = torch.randn(rows, D, generator=g).to(BF).to(DEV)
    w = (torch.rand(D, generator=g) + 0.5).to(BF).to(DEV)
    ref = K.gated_rmsnorm(y, z, w, 1e-5, None, out=torch.empty(rows, D, dtype=BF, device=DEV))
    W = (torch.randn(256, D, generator=g) * 0.05).to(BF).to(DEV)
    parts, sums = [], []
    for lo, hi in ((0, cut), (cut, D)):  # two ranks' column blocks of the same rows
        out = torch.empty(rows, hi - lo, dtype=BF, device=DEV)
        s = torch.empty(rows, 1, dtype=torch.float32, device=DEV)
        K.gated_rmsnorm_deferred(y[:, lo:hi].contiguous(), z[:, lo:hi].contiguous(), w[lo:hi].contiguous(), out, s)
        parts.append(out)
        sums.append(s)
    total = sums[0] + sums[1]  # the all-reduce of the row statistic
    normed = torch.cat([K.scale_rows(p.clone(), total, D, 1e-5) for p in parts], 1)
    close(normed, ref)
    # the layer's use: project the unnormalised values, then scale the projected rows
    proj = sum(K.gemm(p, W[:, lo:hi].contiguous()) for p, (lo, hi) in zip(parts, ((0, cut), (cut, D))))
    close(K.scale_rows(proj.contiguous(), total, D, 1e-5), K.gemm(ref, W))
