"""Output checks against the fp32 layer and across ranks (same API as the reference's
`harness/correctness.py`: `compare` :8-19, `passes` :22-24, `cross_rank_max_abs` :27-34), plus the
tolerance this implementation is held to (max-abs <= 2e-2 of the reference's scale, rel-L2 <= 1e-2)."""
from __future__ import annotations

import json
import os

import torch
import torch.distributed as dist

ABS_MAX = 2e-2  # the absolute max-abs bound, reported beside the scaled rule that within_tolerance applies


def compare(out: torch.Tensor, ref: torch.Tensor) -> dict[str, float]:
    o, r = out.float().cpu(), ref.float().cpu()
    diff = (o - r).abs()
    m = {
        "max_abs": diff.max().item(),
        "max_rel": (diff / r.abs().clamp_min(1e-6)).max().item(),
        "mean_rel": (diff.sum() / r.abs().sum()).item(),
        "rel_l2": (torch.linalg.vector_norm(o - r) / torch.linalg.vector_norm(r).clamp_min(1e-30)).item(),
        "cos": torch.nn.functional.cosine_similarity(o.flatten(), r.flatten(), dim=0).item(),
        "ref_max_abs": r.abs().max().item(),
    }
    _log(m)
    return m


def _log(m: dict[str, float]) -> None:
    """With MMP_PARITY_LOG set to a file path, append every comparison (and the test that made it) as one JSON
    line: the record of absolute max-abs errors behind the parity claims."""
    path = os.environ.get("MMP_PARITY_LOG")
    if not path:
        return
    rec = {"test": os.environ.get("PYTEST_CURRENT_TEST", "").split(" ")[0], **m,
           "abs_ok": m["max_abs"] <= ABS_MAX, "scaled_ok": within_tolerance(m)}
    with open(path, "a") as f:
        f.write(json.dumps(rec) + "\n")


def describe(m: dict[str, float]) -> str:
    """The comparison with both max-abs rules side by side, for assertion messages."""
    lim = 2e-2 * max(1.0, m["ref_max_abs"])
    return (f"max_abs={m['max_abs']:.4g} (absolute bound {ABS_MAX:g}: {'met' if m['max_abs'] <= ABS_MAX else 'over'}; "
            f"scaled bound {lim:.4g}: {'met' if m['max_abs'] <= lim else 'over'}), rel_l2={m['rel_l2']:.3g} "
            f"(bound 1e-2), max|ref|={m['ref_max_abs']:.3g}")


def passes(m: dict[str, float], mean_rel: float = 1.5e-2, max_abs_frac: float = 2e-2, cos: float = 0.9999) -> bool:
    """The reference's bf16 end-to-end gate."""
    return m["mean_rel"] <= mean_rel and m["max_abs"] <= max_abs_frac * m["ref_max_abs"] and m["cos"] >= cos


def within_tolerance(m: dict[str, float], max_abs_frac: float = 2e-2, rel_l2: float = 1e-2) -> bool:
    """max-abs <= 2e-2 * max(1, max|ref|) and rel-L2 <= 1e-2."""
    return m["max_abs"] <= max_abs_frac * max(1.0, m["ref_max_abs"]) and m["rel_l2"] <= rel_l2


def cross_rank_max_abs(out: torch.Tensor, world: int) -> float:
    """All ranks must hold identical outputs after the final all-reduce."""
    if world == 1:
        return 0.0
    gathered = [torch.empty_like(out) for _ in range(world)]
    dist.all_gather(gathered, out.contiguous())
    base = gathered[0].float()
    return max((g.float() - base).abs().max().item() for g in gathered[1:])
