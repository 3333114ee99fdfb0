"""Generate the golden fixture that pins the Gated DeltaNet oracle's mixer (oracle/gdn_layer.py:gdn_mixer_prefill) to
an independent public implementation of the same layer type: Hugging Face transformers' Qwen3-Next Gated DeltaNet
module (`transformers.models.qwen3_next.modeling_qwen3_next.Qwen3NextGatedDeltaNet`, transformers 5.5, in this
image; its PyTorch chunked delta rule, causal conv, L2-normalised q/k, decay -exp(A_log) softplus(a + dt_bias),
norm-before-gate RMSNorm). The reference harness has no implementation of these layers.

    python tests/golden/make_qwen3next_golden.py

The weights are one delta-rule layer of this package's `qwen35.random_stack` (conv bias zero, as the module has
none) plus seeded A_log / dt_bias, laid out into the module's interleaved projections ([q, k, v-group, z-group] and
[b-group, a-group] per key head); the input is a seeded, already normalised sequence. `qwen3next_golden.npz`
stores A_log, dt_bias and the module's output; `DIMS`, `L`, the seeds and `layer_weights` rebuild the rest.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

L, WSEED, XSEED = 150, 7, 8


def dims():
    from multi_modal_parallelism_b200.qwen35 import Qwen35Dims

    return Qwen35Dims(hidden=256, n_k=2, n_v=4, dk=32, dv=32, intermediate=64, layout="G", chunk=64)


def layer_weights(d) -> dict:
    """One delta-rule layer's weights (torch, CPU): the package's seeded draw, conv bias zero, seeded A_log / dt_bias."""
    from multi_modal_parallelism_b200.qwen35 import random_stack

    w = random_stack(d, WSEED)[0]
    w["conv1d.bias"] = torch.zeros_like(w["conv1d.bias"])
    g = torch.Generator().manual_seed(WSEED + 1)
    w["A_log"] = torch.log(torch.rand(d.n_v, generator=g) * 15 + 1)
    w["dt_bias"] = torch.randn(d.n_v, generator=g) * 0.5
    return w


def layer_input(d) -> torch.Tensor:
    return torch.randn(L, d.hidden, generator=torch.Generator().manual_seed(XSEED))


def main() -> None:
    from transformers.models.qwen3_next import configuration_qwen3_next as C
    from transformers.models.qwen3_next import modeling_qwen3_next as M

    d = dims()
    w = {k: v.float() for k, v in layer_weights(d).items()}
    cfg = C.Qwen3NextConfig(hidden_size=d.hidden, linear_num_value_heads=d.n_v, linear_num_key_heads=d.n_k,
                            linear_key_head_dim=d.dk, linear_value_head_dim=d.dv, linear_conv_kernel_dim=d.d_conv,
                            rms_norm_eps=d.rms_eps, hidden_act="silu", num_hidden_layers=1)
    mod = M.Qwen3NextGatedDeltaNet(cfg, layer_idx=0).float().eval()
    rep, kd, vd = d.n_v // d.n_k, d.n_k * d.dk, d.n_v * d.dv
    Wqkv, Wz = w["in_proj_qkv.weight"], w["in_proj_z.weight"]
    qkvz, ba = [], []
    for kh in range(d.n_k):
        vs = slice(kh * rep * d.dv, (kh + 1) * rep * d.dv)
        qkvz += [Wqkv[kh * d.dk:(kh + 1) * d.dk], Wqkv[kd + kh * d.dk:kd + (kh + 1) * d.dk],
                 Wqkv[2 * kd:][vs], Wz[vs]]
        hs = slice(kh * rep, (kh + 1) * rep)
        ba += [w["in_proj_b.weight"][hs], w["in_proj_a.weight"][hs]]
    sd = {"in_proj_qkvz.weight": torch.cat(qkvz), "in_proj_ba.weight": torch.cat(ba),
          "conv1d.weight": w["conv1d.weight"][:, None, :], "dt_bias": w["dt_bias"], "A_log": w["A_log"],
          "norm.weight": w["norm.weight"], "out_proj.weight": w["out_proj.weight"]}
    mod.load_state_dict(sd)
    with torch.no_grad():
        out = mod(layer_input(d)[None])[0]
    np.savez_compressed(HERE / "qwen3next_golden.npz", out=out.numpy())
    print("wrote qwen3next_golden.npz", tuple(out.shape), vd)


if __name__ == "__main__":
    main()
