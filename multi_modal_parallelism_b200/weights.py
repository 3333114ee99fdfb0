"""Layer weights: seeded random init or a safetensors checkpoint, and per-rank slicing onto the device.

API-compatible with the reference's `harness/weights.py` (`random_layer` :43-70, `RankWeights` :73-108,
`shard_to_device` :111-147, `layer_bytes` :150-156). `random_layer` draws from one CPU generator in the
same tensor order and with the same distributions as the reference, so a given seed yields the same
weights bit for bit (that equality is pinned by the golden fixtures under tests/golden):
linear N(0, 0.02) in bf16, conv weight U[-0.5, 0.5), conv bias U[0, 0.1), A_log = log(1 + 15 U),
D = 1, dt_bias = log(expm1(1e-3 + 0.099 U)), norm weights 1.

`shard_to_device` lays weights out for the C-ABI kernels: every projection is a row-major [out, in] bf16
matrix (the K-major operand of the GEMM), the muP multipliers of the in_proj output are an fp32 column
scale applied in the GEMM epilogue, and A = -exp(A_log), D and dt_bias are fp32 per-head vectors.
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

import torch

from .config import FalconH1Dims
from .sharding import RankPlan, build_mup_vector

KEYS = (
    "self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight", "self_attn.o_proj.weight",
    "mamba.in_proj.weight", "mamba.conv1d.weight", "mamba.conv1d.bias", "mamba.A_log", "mamba.D", "mamba.dt_bias",
    "mamba.norm.weight", "mamba.out_proj.weight",
    "feed_forward.gate_proj.weight", "feed_forward.up_proj.weight", "feed_forward.down_proj.weight",
    "input_layernorm.weight", "pre_ff_layernorm.weight",
)


def load_layer_from_safetensors(model_dir: str | Path, layer_idx: int) -> dict[str, torch.Tensor]:
    from safetensors import safe_open

    model_dir = Path(model_dir)
    index = json.loads((model_dir / "model.safetensors.index.json").read_text())["weight_map"]
    prefix = f"model.layers.{layer_idx}."
    per_file: dict[str, list[str]] = {}
    for key in KEYS:
        full = prefix + key
        if full not in index:
            raise KeyError(f"{full} not in checkpoint index")
        per_file.setdefault(index[full], []).append(key)
    out: dict[str, torch.Tensor] = {}
    for fname, keys in per_file.items():
        with safe_open(str(model_dir / fname), framework="pt", device="cpu") as f:
            for key in keys:
                out[key] = f.get_tensor(prefix + key)
    return out


def random_layer(dims: FalconH1Dims, seed: int = 0) -> dict[str, torch.Tensor]:
    """Seeded random layer on the CPU (draw order is part of the contract: see the module docstring)."""
    gen = torch.Generator().manual_seed(seed)
    H, I, hd, nh = dims.hidden, dims.intermediate, dims.head_dim, dims.n_mamba_heads

    def normal_bf16(rows: int, cols: int) -> torch.Tensor:
        return (torch.randn(rows, cols, generator=gen) * 0.02).to(torch.bfloat16)

    def uniform(*shape: int) -> torch.Tensor:
        return torch.rand(*shape, generator=gen)

    w: dict[str, torch.Tensor] = {}
    w["self_attn.q_proj.weight"] = normal_bf16(dims.n_q * hd, H)
    w["self_attn.k_proj.weight"] = normal_bf16(dims.n_kv * hd, H)
    w["self_attn.v_proj.weight"] = normal_bf16(dims.n_kv * hd, H)
    w["self_attn.o_proj.weight"] = normal_bf16(H, dims.n_q * hd)
    w["mamba.in_proj.weight"] = normal_bf16(dims.in_proj_rows, H)
    w["mamba.conv1d.weight"] = (uniform(dims.conv_rows, 1, dims.d_conv) - 0.5).to(torch.bfloat16)
    w["mamba.conv1d.bias"] = (uniform(dims.conv_rows) * 0.1).to(torch.bfloat16)
    w["mamba.A_log"] = torch.log(1 + 15 * uniform(nh))
    w["mamba.D"] = torch.ones(nh)
    w["mamba.dt_bias"] = torch.log(torch.expm1(1e-3 + 0.099 * uniform(nh)))
    w["mamba.norm.weight"] = torch.ones(dims.d_ssm, dtype=torch.bfloat16)
    w["mamba.out_proj.weight"] = normal_bf16(H, dims.d_ssm)
    w["feed_forward.gate_proj.weight"] = normal_bf16(I, H)
    w["feed_forward.up_proj.weight"] = normal_bf16(I, H)
    w["feed_forward.down_proj.weight"] = normal_bf16(H, I)
    w["input_layernorm.weight"] = torch.ones(H, dtype=torch.bfloat16)
    w["pre_ff_layernorm.weight"] = torch.ones(H, dtype=torch.bfloat16)
    return w


@dataclass
class RankWeights:
    # attention (None on SSM-only ranks)
    wqkv: torch.Tensor | None  # [q+k+v rows, H] bf16
    wo: torch.Tensor | None  # [H, q cols] bf16
    q_rows: int = 0
    kv_rows: int = 0
    # mamba-2 (None on attention-only ranks)
    win: torch.Tensor | None = None  # [z+x+B+C+dt rows, H] bf16
    conv_w: torch.Tensor | None = None  # [conv rows, d_conv] bf16
    conv_b: torch.Tensor | None = None  # [conv rows] bf16
    A: torch.Tensor | None = None  # [nhr] fp32, -exp(A_log)
    D: torch.Tensor | None = None  # [nhr] fp32
    dt_bias: torch.Tensor | None = None  # [nhr] fp32
    norm_w: torch.Tensor | None = None  # [nhr*p] bf16
    wout: torch.Tensor | None = None  # [H, nhr*p] bf16
    mup: torch.Tensor | None = None  # [1, in rows] fp32 per-column muP scale of the in_proj output
    # mlp pool: row r of gate/up (column r of down) is global intermediate column col_order[r]
    mlp_gate: torch.Tensor | None = None  # [n_pool, H] bf16
    mlp_up: torch.Tensor | None = None  # [n_pool, H] bf16
    mlp_down: torch.Tensor | None = None  # [H, n_pool] bf16 (down_proj columns of the pool)
    n_fixed: int = 0
    n_pool: int = 0
    # norms
    in_norm: torch.Tensor | None = None
    ff_norm: torch.Tensor | None = None
    # both branches on one rank: the projections that share an input or an output, concatenated (wqkv/win
    # and wo/wout are views into these)
    w_in_cat: torch.Tensor | None = None  # [q+k+v rows + in rows, H]
    in_colscale: torch.Tensor | None = None  # [q+k+v rows + in rows] fp32: attn_in, then ssm_in * muP
    w_out_cat: torch.Tensor | None = None  # [H, q cols + d_ssm local]

    @property
    def mlp_downT(self) -> torch.Tensor | None:
        """[n_pool, H] view of the pool's down_proj columns (the reference's storage orientation)."""
        return None if self.mlp_down is None else self.mlp_down.t()

    def resident_bytes(self) -> dict[str, int]:
        def nb(t: torch.Tensor | None) -> int:
            return 0 if t is None else t.numel() * t.element_size()

        return {
            "attn": nb(self.wqkv) + nb(self.wo),
            "mamba": nb(self.win) + nb(self.conv_w) + nb(self.conv_b) + nb(self.wout) + nb(self.norm_w),
            "mlp_pool": nb(self.mlp_gate) + nb(self.mlp_up) + nb(self.mlp_down),
        }


def shard_to_device(full: dict[str, torch.Tensor], plan: RankPlan, dims: FalconH1Dims, device: torch.device) -> RankWeights:
    bf = torch.bfloat16

    def put(t: torch.Tensor, dtype=bf) -> torch.Tensor:
        return t.to(device=device, dtype=dtype).contiguous()

    rw = RankWeights(wqkv=None, wo=None)
    a = plan.attn
    if a is not None:
        q = full["self_attn.q_proj.weight"][a.q_rows]
        k = full["self_attn.k_proj.weight"][a.k_rows]
        v = full["self_attn.v_proj.weight"][a.v_rows]
        rw.wqkv = put(torch.cat([q, k, v], 0))
        rw.wo = put(full["self_attn.o_proj.weight"][:, a.o_cols])
        rw.q_rows, rw.kv_rows = q.shape[0], k.shape[0]
    s = plan.ssm
    if s is not None:
        ip = full["mamba.in_proj.weight"]
        rw.win = put(torch.cat([ip[s.z_rows], ip[s.x_rows], ip[s.b_rows], ip[s.c_rows], ip[s.dt_rows]], 0))
        cw, cb = full["mamba.conv1d.weight"][:, 0, :], full["mamba.conv1d.bias"]
        rw.conv_w = put(torch.cat([cw[r] for r in s.conv_rows], 0))
        rw.conv_b = put(torch.cat([cb[r] for r in s.conv_rows], 0))
        rw.A = put(-torch.exp(full["mamba.A_log"][s.heads].float()), torch.float32)
        rw.D = put(full["mamba.D"][s.heads].float(), torch.float32)
        rw.dt_bias = put(full["mamba.dt_bias"][s.heads].float(), torch.float32)
        rw.norm_w = put(full["mamba.norm.weight"][s.norm_cols])
        rw.wout = put(full["mamba.out_proj.weight"][:, s.out_cols])
        rw.mup = put(build_mup_vector(dims, s), torch.float32)
    if a is not None and s is not None:
        nqkv, nin = rw.wqkv.shape[0], rw.win.shape[0]
        rw.w_in_cat = torch.cat([rw.wqkv, rw.win], 0).contiguous()
        rw.wqkv, rw.win = rw.w_in_cat[:nqkv], rw.w_in_cat[nqkv:]
        rw.in_colscale = torch.cat([torch.full((nqkv,), float(dims.attn_in), device=device),
                                    rw.mup.reshape(-1) * float(dims.ssm_in)]).contiguous()
        qc = rw.wo.shape[1]
        rw.w_out_cat = torch.cat([rw.wo, rw.wout], 1).contiguous()
        rw.wo, rw.wout = rw.w_out_cat[:, :qc], rw.w_out_cat[:, qc:]
    m = plan.mlp
    cols = torch.tensor(m.col_order, dtype=torch.long)
    rw.mlp_gate = put(full["feed_forward.gate_proj.weight"][cols])
    rw.mlp_up = put(full["feed_forward.up_proj.weight"][cols])
    rw.mlp_down = put(full["feed_forward.down_proj.weight"][:, cols])
    rw.n_fixed, rw.n_pool = m.n_fixed, len(m.col_order)
    rw.in_norm = put(full["input_layernorm.weight"])
    rw.ff_norm = put(full["pre_ff_layernorm.weight"])
    return rw


def layer_bytes(dims: FalconH1Dims) -> dict[str, int]:
    """Full-layer bf16 weight bytes by component."""
    H, I, hd = dims.hidden, dims.intermediate, dims.head_dim
    attn = 2 * (dims.n_q * hd * H + 2 * dims.n_kv * hd * H + H * dims.n_q * hd)
    mamba = 2 * (dims.in_proj_rows * H + H * dims.d_ssm + dims.conv_rows * dims.d_conv + dims.conv_rows + dims.d_ssm)
    mlp = 2 * 3 * I * H
    return {"attn": attn, "mamba": mamba, "mlp": mlp, "total": attn + mamba + mlp}
