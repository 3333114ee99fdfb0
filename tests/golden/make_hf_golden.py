"""Generate the golden fixture that pins the oracle's prefill (oracle/hybrid_layer.py:prefill_sequential) to an
independent public implementation of the same layer: Hugging Face transformers' Falcon-H1 decoder layer
(`transformers.models.falcon_h1.modeling_falcon_h1.FalconH1DecoderLayer`, transformers 5.5, in this image), whose
Mamba-2 mixer runs the chunked SSD scan in PyTorch (its `torch_forward`) and whose attention runs the eager
causal path. The reference harness has no prefill (its fp32 layer is one decode step), so this anchors the
prefill rows; the decode step is pinned to the reference itself by make_golden.py.

    python tests/golden/make_hf_golden.py

For each case the layer gets this package's seeded weights (`weights.random_layer`, whose tensors equal the
reference's by the hashes in golden_hashes.json), a seeded input sequence at positions 0..L-1, and returns the layer
output; `hf_prefill_golden.npz` stores the output per case (dims, lengths and seeds in CASES below; the input
is regenerated from its seed by `case_input`).
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

# (case, preset, dims overrides, L, weight seed, input seed)
MULTS7B = dict(attn_out=0.1041666, key_mult=0.0307, ssm_in=0.4166666, ssm_out=0.1178511,
               ssm_mults=(0.3535533, 0.25, 0.1767766, 0.5, 0.3535533), mlp_mults=(0.2946278, 0.032552))
CASES = [
    ("g2_mlp", "hybrid_small", dict(hidden=256, intermediate=512, n_q=4, n_kv=2, head_dim=64, n_mamba_heads=8,
                                    mamba_head_dim=32, d_ssm=256, d_state=32, n_groups=2, chunk=64, **MULTS7B), 150, 3, 1),
    ("g1_mixer", "hybrid_small", dict(hidden=256, intermediate=0, n_q=2, n_kv=1, head_dim=128, n_mamba_heads=4,
                                      mamba_head_dim=64, d_ssm=256, d_state=64, n_groups=1, chunk=32), 97, 4, 2),
]


def hf_layer(dims):
    from transformers.models.falcon_h1 import configuration_falcon_h1 as C
    from transformers.models.falcon_h1 import modeling_falcon_h1 as M

    cfg = C.FalconH1Config(
        hidden_size=dims.hidden, intermediate_size=max(dims.intermediate, 8), num_hidden_layers=1,
        num_attention_heads=dims.n_q, num_key_value_heads=dims.n_kv, head_dim=dims.head_dim, rms_norm_eps=dims.rms_eps,
        mamba_d_ssm=dims.d_ssm, mamba_n_heads=dims.n_mamba_heads, mamba_d_head=dims.mamba_head_dim,
        mamba_n_groups=dims.n_groups, mamba_d_state=dims.d_state, mamba_d_conv=dims.d_conv, mamba_chunk_size=dims.chunk,
        mamba_conv_bias=True, mamba_proj_bias=False, mamba_norm_before_gate=False, mamba_rms_norm=True,
        time_step_limit=(0.0, float("inf")), rope_parameters={"rope_type": "default", "rope_theta": dims.rope_theta},
        key_multiplier=dims.key_mult, attention_out_multiplier=dims.attn_out, attention_in_multiplier=dims.attn_in,
        ssm_multipliers=list(dims.ssm_mults), ssm_in_multiplier=dims.ssm_in, ssm_out_multiplier=dims.ssm_out,
        mlp_multipliers=list(dims.mlp_mults), attention_bias=False, mlp_bias=False, projectors_bias=False,
        max_position_embeddings=4096)
    cfg._attn_implementation = "eager"
    layer = M.FalconH1DecoderLayer(cfg, layer_idx=0).float().eval()
    layer.mamba.register_buffer("mup_vector", M.compute_mup_vector(cfg).clone(), persistent=False)
    return cfg, layer, M


def case_input(dims, L: int, hseed: int) -> torch.Tensor:
    """The seeded input sequence of a case ([L, hidden] fp32; torch's CPU generator, identical on every host)."""
    return torch.randn(1, L, dims.hidden, generator=torch.Generator().manual_seed(hseed))[0]


def case_dims(preset_name, over):
    from multi_modal_parallelism_b200.config import preset

    return preset(preset_name).replace(**over)


def run_case(name, preset_name, over, L, wseed, hseed):
    from multi_modal_parallelism_b200.weights import random_layer

    dims = case_dims(preset_name, over)
    cfg, layer, M = hf_layer(dims)
    full = random_layer(dims, wseed)
    sd = layer.state_dict()
    for k in sd:
        if k.startswith("feed_forward.") and dims.intermediate == 0:
            sd[k] = torch.zeros_like(sd[k])  # a mixer-only layer: the MLP adds exact zeros
        elif k in full:
            sd[k] = full[k].float()
        else:
            raise KeyError(k)
    layer.load_state_dict(sd)
    h = case_input(dims, L, hseed)[None]
    pos = torch.arange(L)[None]
    pe = M.FalconH1RotaryEmbedding(cfg)(h, pos)
    mask = torch.full((L, L), float("-inf")).triu(1)[None, None]
    with torch.no_grad():
        out = layer(h, attention_mask=mask, mamba_attention_mask=None, position_ids=pos, position_embeddings=pe)[0][0]
    return out.numpy()


def main() -> None:
    arrays = {}
    for name, pre, over, L, ws, hs in CASES:
        arrays[f"{name}_out"] = run_case(name, pre, over, L, ws, hs)
    np.savez_compressed(HERE / "hf_prefill_golden.npz", **arrays)
    print("wrote hf_prefill_golden.npz")


if __name__ == "__main__":
    main()
