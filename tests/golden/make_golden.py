"""Generate the golden fixtures that pin the CPU oracle to the reference's own code.

Run once in a container that has the reference checkout (it is not needed afterwards):

    python tests/golden/make_golden.py --reference /root/reference

It imports the reference's pure-PyTorch layer (`harness/reference.py:decode_step`), its seeded weight
initialiser (`harness/weights.py:random_layer`) and its seeded state generators (`harness/state.py:46-73`,
with a stand-in for the vLLM-bound `harness.kernels` module that `harness/state.py` imports but these
generators never call), runs them on the CPU and writes:

  golden_<case>.npz    input hidden, reference output and intermediates (float32)
  golden_hashes.json   SHA-256 of every seeded tensor (weights and initial states) per case

The tests regenerate the same tensors with this package's own code, require identical hashes, run the
oracle, and compare with the stored reference results.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

# (case, dims overrides, B, ctx, seed). Dims fields follow harness/config.py:FalconH1Dims.
SMALL = dict(hidden=1024, intermediate=0, n_q=8, n_kv=2, head_dim=128, n_mamba_heads=16, mamba_head_dim=64,
             d_ssm=1024, d_state=128, n_groups=1, d_conv=4, chunk=256, rms_eps=1e-5, rope_theta=1e4, max_pos=8192,
             attn_in=1.0, attn_out=1.0, key_mult=1.0, ssm_in=1.0, ssm_out=1.0, ssm_mults=(1.0,) * 5, mlp_mults=(1.0, 1.0))
MULTS7B = dict(attn_in=1.0, attn_out=0.1041666, key_mult=0.0307, ssm_in=0.4166666, ssm_out=0.1178511,
               ssm_mults=(0.3535533, 0.25, 0.1767766, 0.5, 0.3535533), mlp_mults=(0.2946278, 0.032552))
TINY_MLP_G2 = dict(hidden=256, intermediate=512, n_q=4, n_kv=2, head_dim=64, n_mamba_heads=8, mamba_head_dim=32,
                   d_ssm=256, d_state=32, n_groups=2, d_conv=4, chunk=64, rms_eps=1e-5, rope_theta=1e4, max_pos=4096,
                   **MULTS7B)
LIKE7B = dict(hidden=3072, intermediate=0, n_q=12, n_kv=2, head_dim=128, n_mamba_heads=24, mamba_head_dim=128,
              d_ssm=3072, d_state=256, n_groups=1, d_conv=4, chunk=256, rms_eps=1e-5, rope_theta=1e11, max_pos=262144,
              **MULTS7B)
CASES = [
    ("small", SMALL, 2, 24, 0),
    ("mlp_g2", TINY_MLP_G2, 3, 20, 1),
    ("like7b", LIKE7B, 2, 40, 0),
]


def sha(t: torch.Tensor) -> str:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def import_reference(root: Path):
    sys.path.insert(0, str(root))
    # harness/state.py imports harness.kernels (vLLM GPU ops) at module level; the generators used here do not
    # touch it, so a placeholder module is enough to import them on the CPU.
    stub = types.ModuleType("harness.kernels")
    stub.alloc_kv = None
    sys.modules["harness.kernels"] = stub
    import harness.config as rc  # noqa: E402
    import harness.reference as rr  # noqa: E402
    import harness.state as rs  # noqa: E402
    import harness.weights as rw  # noqa: E402
    return rc, rr, rs, rw


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    args = ap.parse_args()
    rc, rr, rs, rw = import_reference(Path(args.reference))
    torch.manual_seed(0)
    cpu = torch.device("cpu")
    hashes: dict = {}
    for name, dd, B, c, seed in CASES:
        dims = rc.FalconH1Dims(**dd)
        full = rw.random_layer(dims, seed)
        h = rs.input_hidden(seed, B, dims.hidden, cpu)
        kc, vc, conv, ssm = rs.full_states_for_reference(dims, B, c, seed, cpu)
        inter: dict = {}
        out = rr.decode_step(full, dims, h, kc, vc, conv, ssm, c, intermediates=inter)
        hashes[name] = {
            "dims": {k: (list(v) if isinstance(v, tuple) else v) for k, v in dd.items()},
            "B": B, "ctx": c, "seed": seed,
            "weights": {k: sha(v) for k, v in full.items()},
            "input_hidden": sha(h),
            "k_cache": sha(kc), "v_cache": sha(vc), "conv_state": sha(conv), "ssm_state": sha(ssm),
        }
        arrays = {"h": h.float().numpy(), "out": out.float().numpy()}
        for k, v in inter.items():
            arrays["inter_" + k] = v.float().numpy()
        np.savez_compressed(HERE / f"golden_{name}.npz", **arrays)
        print(f"{name}: out {tuple(out.shape)} max|out| {out.abs().max().item():.4g}; {len(arrays)} arrays")
    (HERE / "golden_hashes.json").write_text(json.dumps(hashes, indent=1, sort_keys=True) + "\n")


if __name__ == "__main__":
    main()
