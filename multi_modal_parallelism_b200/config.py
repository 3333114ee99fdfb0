"""Layer dimensions and run specifications.

API-compatible with the reference harness's `harness/config.py` (`FalconH1Dims` at :13-85, `RunSpec` at
:88-105): same field names, same derived sizes, same HF/YAML constructors. Two extensions:

* ``intermediate == 0`` describes a mixer-only layer (attention ∥ Mamba-2, summed, residual) with no MLP.
  The reference's fp32 layer already degenerates to that case (its MLP contributes exact zeros when the
  intermediate size is 0, `harness/reference.py:112-119`).
* ``MODES`` lists every branch-split layout ``split{a}{m}`` with ``a + m <= 8``; the reference's layer only
  accepts the literal ``split22`` (`harness/layer.py:209-216`).
"""
from __future__ import annotations

import json
from dataclasses import dataclass, fields
from pathlib import Path
from typing import Literal

_SPLITS = tuple(f"split{a}{m}" for a in range(1, 8) for m in range(1, 8) if a + m <= 8)
MODES: tuple[str, ...] = ("tp1", "tp4", "tp4_fused", "tp4_streams") + _SPLITS
Mode = str

CONFIG_DIR = Path(__file__).resolve().parent / "configs"


@dataclass(frozen=True)
class FalconH1Dims:
    hidden: int
    intermediate: int
    n_q: int
    n_kv: int
    head_dim: int
    n_mamba_heads: int
    mamba_head_dim: int
    d_ssm: int
    d_state: int
    n_groups: int
    d_conv: int
    chunk: int
    rms_eps: float
    rope_theta: float
    max_pos: int
    attn_in: float
    attn_out: float
    key_mult: float
    ssm_in: float
    ssm_out: float
    ssm_mults: tuple[float, float, float, float, float]
    mlp_mults: tuple[float, float]

    # ------------------------------------------------------------------ derived sizes
    @property
    def in_proj_rows(self) -> int:
        """Rows of Mamba-2 in_proj: [z | x | B | C | dt]."""
        gn = self.n_groups * self.d_state
        return self.d_ssm + self.d_ssm + gn + gn + self.n_mamba_heads

    @property
    def conv_rows(self) -> int:
        """Channels of the depthwise conv: [x | B | C]."""
        return self.d_ssm + 2 * self.n_groups * self.d_state

    @property
    def has_mlp(self) -> bool:
        return self.intermediate > 0

    # ------------------------------------------------------------------ constructors
    @classmethod
    def from_hf(cls, model_dir: str | Path) -> "FalconH1Dims":
        """Read a Hugging Face Falcon-H1 ``config.json`` (same keys and defaults as the reference)."""
        cfg = json.loads((Path(model_dir) / "config.json").read_text())
        hidden = int(cfg["hidden_size"])
        nh = int(cfg["mamba_n_heads"])
        d_ssm = cfg.get("mamba_d_ssm") or int(cfg.get("mamba_expand", 2) * hidden)
        n_q = int(cfg["num_attention_heads"])

        def get(key, default):
            v = cfg.get(key)
            return default if v is None else v

        return cls(
            hidden=hidden,
            intermediate=int(cfg["intermediate_size"]),
            n_q=n_q,
            n_kv=int(cfg["num_key_value_heads"]),
            head_dim=int(cfg.get("head_dim") or hidden // n_q),
            n_mamba_heads=nh,
            mamba_head_dim=int(cfg.get("mamba_d_head") or d_ssm // nh),
            d_ssm=int(d_ssm),
            d_state=int(cfg["mamba_d_state"]),
            n_groups=int(get("mamba_n_groups", 1)),
            d_conv=int(get("mamba_d_conv", 4)),
            chunk=int(get("mamba_chunk_size", 256)),
            rms_eps=float(get("rms_norm_eps", 1e-5)),
            rope_theta=float(get("rope_theta", 1e4)),
            max_pos=int(get("max_position_embeddings", 8192)),
            attn_in=float(get("attention_in_multiplier", 1.0)),
            attn_out=float(get("attention_out_multiplier", 1.0)),
            key_mult=float(get("key_multiplier", 1.0)),
            ssm_in=float(get("ssm_in_multiplier", 1.0)),
            ssm_out=float(get("ssm_out_multiplier", 1.0)),
            ssm_mults=tuple(float(v) for v in get("ssm_multipliers", [1.0] * 5)),
            mlp_mults=tuple(float(v) for v in get("mlp_multipliers", [1.0, 1.0])),
        )

    @classmethod
    def from_yaml(cls, path: str | Path) -> "FalconH1Dims":
        """Load a dims YAML. A bare name (``falcon_h1_7b``) resolves to the bundled ``configs/`` folder.
        Keys that are not dims fields (``name``, ``layers``) are ignored, as the reference's YAMLs carry them."""
        import yaml

        p = Path(path)
        if not p.exists():
            cand = CONFIG_DIR / (p.name if p.suffix else p.name + ".yaml")
            if cand.exists():
                p = cand
        d = yaml.safe_load(p.read_text())
        names = {f.name for f in fields(cls)}
        kw = {k: v for k, v in d.items() if k in names}
        kw["ssm_mults"] = tuple(float(v) for v in kw["ssm_mults"])
        kw["mlp_mults"] = tuple(float(v) for v in kw["mlp_mults"])
        for k in ("rms_eps", "rope_theta", "attn_in", "attn_out", "key_mult", "ssm_in", "ssm_out"):
            kw[k] = float(kw[k])
        return cls(**kw)

    def replace(self, **kw) -> "FalconH1Dims":
        d = {f.name: getattr(self, f.name) for f in fields(self)}
        d.update(kw)
        return FalconH1Dims(**d)


def preset(name: str) -> FalconH1Dims:
    """Bundled layer shapes: ``hybrid_small`` (1024-wide layer), ``falcon_h1_7b_like`` (mixer-only
    7B-like layer), ``falcon_h1_34b_like`` (34B-like layer with a 20480-wide SwiGLU MLP) and the reference's
    own ``falcon_h1_7b`` / ``falcon_h1_34b`` / ``falcon_h1_3b`` dims."""
    return FalconH1Dims.from_yaml(CONFIG_DIR / f"{name}.yaml")


@dataclass(frozen=True)
class RunSpec:
    mode: str
    swing: float = 0.0
    k: int | None = None  # swing split point in [0, 2w]; None -> resolved from cuts_src
    cuts_src: str = "neutral"  # neutral | model | grid | manual
    batch: int = 1
    ctx: int = 512
    variant: Literal["eager", "graph", "both"] = "eager"
    kv_block: int = 16
    n_warm: int = 20
    n_iter: int = 100
    repeats: int = 3
    repeat_offset: int = 0
    collectives: bool = True  # False = diagnostic: per-rank compute only (outputs are wrong)
    layer_idx: int = 0
    seed: int = 0
    tag: str = ""
