"""Empty batches through the C library, on a machine without a GPU: every entry point the layers use returns
success for zero rows, sequences or tokens before it touches the device (the reference's kernels accept empty
batches too; a serving step may have no decode rows or no prefill). The wrappers run with CPU tensors and only
their CUDA-device assertions relaxed; a call that reached a CUDA launch would fail here, so passing means the
library returned early."""
import pytest
import torch

from multi_modal_parallelism_b200 import _lib
from multi_modal_parallelism_b200 import kernels as K
from multi_modal_parallelism_b200.state import alloc_kv

BF = torch.bfloat16
F32 = torch.float32


@pytest.fixture
def cpu_wrappers(monkeypatch):
    statuses = []

    def call(name, *args, kernels=1):
        rc = getattr(_lib.lib(), name)(*args)
        statuses.append((name, rc))
        assert rc == _lib.MMP_OK, f"{name}: {rc} {_lib.lib().mmp_last_error().decode(errors='replace')}"

    monkeypatch.setattr(K, "_cuda", lambda *a, **k: None)
    monkeypatch.setattr(K, "_stream", lambda t: None)
    monkeypatch.setattr(K, "error_word", lambda dev: torch.zeros(1, dtype=torch.int32))
    monkeypatch.setattr(_lib, "call", call)
    return statuses


def test_empty_decode_batch(cpu_wrappers):
    H, hd, nq, nkv, nh, p, N, rows = 256, 128, 4, 2, 4, 64, 64, 3 * 64 + 2 * 64
    x = torch.zeros(0, H, dtype=BF)
    w = torch.zeros(H, dtype=BF)
    K.rms_norm(x, w, 1e-5, torch.zeros(0, H, dtype=BF))
    K.gemm(x, torch.zeros(512, H, dtype=BF), out=torch.zeros(0, 512, dtype=BF))
    K.add(x, x, torch.zeros(0, H, dtype=BF))
    K.silu_mul(torch.zeros(0, 512, dtype=BF), torch.zeros(0, 512, dtype=BF), torch.zeros(0, 512, dtype=BF))
    K.gated_rmsnorm(torch.zeros(0, nh * p, dtype=BF), torch.zeros(0, nh * p, dtype=BF), torch.zeros(nh * p, dtype=BF),
                    1e-5, None, out=torch.zeros(0, nh * p, dtype=BF))
    conv = torch.zeros(3, 3, rows, dtype=BF).transpose(-1, -2)  # [lines, rows, d_conv-1] view
    K.conv_update(torch.zeros(0, rows, dtype=BF), conv, torch.zeros(rows, 4, dtype=BF), None,
                  torch.zeros(0, dtype=torch.int32))
    state = torch.zeros(3, nh, p, N, dtype=F32)
    K.ssm_update(state, torch.zeros(0, nh, p, dtype=BF), torch.zeros(0, nh, dtype=BF), torch.zeros(nh, dtype=F32),
                 torch.zeros(0, 1, N, dtype=BF), torch.zeros(0, 1, N, dtype=BF), None, None,
                 torch.zeros(0, dtype=torch.int32), torch.zeros(0, nh, p, dtype=BF))
    _, kc, vc, _ = alloc_kv(4, 16, nkv, hd, torch.device("cpu"))
    K.attn_decode(torch.zeros(0, nq, hd, dtype=BF), kc, vc, torch.zeros(1, dtype=torch.int32),
                  torch.zeros(0, dtype=torch.int32), 16, torch.zeros(0, 2, dtype=torch.int32),
                  torch.zeros(0, nq, hd, dtype=BF), workspace=torch.zeros(1, dtype=F32), splits=1)
    names = {n for n, _ in cpu_wrappers}
    assert {"mmp_rmsnorm", "mmp_add", "mmp_gated_rmsnorm", "mmp_conv1d_update", "mmp_ssu_decode",
            "mmp_paged_attn_decode"} <= names


def test_empty_prefill(cpu_wrappers):
    nh, p, N, nq, nkv, hd, rows = 4, 128, 64, 4, 2, 128, 128 + 2 * 64
    cu = torch.zeros(1, dtype=torch.int32)
    none = torch.zeros(0, dtype=torch.int32)
    conv = torch.zeros(2, 3, rows, dtype=BF).transpose(-1, -2)  # [lines, rows, d_conv-1] view
    K.conv_prefill(torch.zeros(0, rows, dtype=BF), conv, torch.zeros(rows, 4, dtype=BF), None, cu, none, none,
                   torch.zeros(0, rows, dtype=BF))
    K.ssd_prefill(torch.zeros(0, nh, p, dtype=BF), torch.zeros(0, nh, dtype=BF), torch.zeros(nh, dtype=F32),
                  torch.zeros(0, 1, N, dtype=BF), torch.zeros(0, 1, N, dtype=BF), None, None,
                  torch.zeros(2, nh, p, N, dtype=F32), cu, none, none, torch.zeros(0, nh, p, dtype=BF))
    _, kc, vc, _ = alloc_kv(4, 16, nkv, hd, torch.device("cpu"))
    K.attn_prefill(torch.zeros(0, nq, hd, dtype=BF), kc, vc, torch.zeros(0, 2, dtype=torch.int32), cu, none, 0,
                   torch.zeros(0, nq, hd, dtype=BF))
    names = {n for n, _ in cpu_wrappers}
    assert {"mmp_conv1d_prefill", "mmp_ssd_prefill", "mmp_paged_attn_prefill"} <= names
