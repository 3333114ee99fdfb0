"""Stage-by-stage comparison of the kernel path against the fp32 layer (one rank), the counterpart of the reference's
`harness/debug.py:1-181`: each stage runs on the kernels from the same states and inputs as the fp32 layer, and its
result is compared with the fp32 layer's intermediate of the same name.

  python -m multi_modal_parallelism_b200.debug --batch 2 --ctx 64 [--dims-yaml falcon_h1_7b] [--ssm-substages]

Stages: input norm; attention branch (o before the o-projection, the branch output); Mamba-2 in-projection,
conv, state update and gated norm (with --ssm-substages: each from the kernel's own inputs, as the reference's
`ssm_substages`); the branch output; h1 = h + attention + Mamba-2; the MLP; the whole step. Prints one line per
stage and a final `[debug] pass=...` line (every stage within max-abs 2e-2 * max(1, max|ref|), rel-L2 1e-2).
"""
from __future__ import annotations

import argparse
import os

import torch
import torch.nn.functional as F

from . import kernels as K
from .config import FalconH1Dims
from .correctness import compare, within_tolerance
from .dist import destroy, init_groups
from .layer import ParallelHybridLayer
from .reference import decode_step
from .sharding import plan_for
from .state import alloc_and_fill, full_states_for_reference, input_hidden, make_decode_ctx
from .timing import NULL
from .weights import load_layer_from_safetensors, random_layer, shard_to_device


class Report:
    def __init__(self):
        self.ok = True

    def __call__(self, name: str, got: torch.Tensor, ref: torch.Tensor) -> None:
        m = compare(got.float().cpu(), ref.float().cpu())
        good = within_tolerance(m)
        self.ok &= good
        print(f"  {name:20s} max_abs={m['max_abs']:.4g} ref_max={m['ref_max_abs']:.4g} rel_l2={m['rel_l2']:.3e} "
              f"cos={m['cos']:.6f} {'ok' if good else 'MISMATCH'}", flush=True)


def _rows16(rows: int, cols: int, dev) -> torch.Tensor:
    """[rows, cols] bf16 view whose rows start 16 bytes apart, so every column slice is a valid kernel operand."""
    return torch.empty(rows, (cols + 7) // 8 * 8, device=dev, dtype=torch.bfloat16)[:, :cols]


def _fresh(layer, plan, dims, ctx, dev) -> None:
    st = alloc_and_fill(plan, dims, ctx, 0, dev)
    for n in ("kv", "conv_state", "ssm_state"):
        dst, src = getattr(layer.st, n), getattr(st, n)
        if dst is not None and src is not None:
            dst.copy_(src)


def ssm_substages(layer, rw, dims, ctx, plan, dev, x, rep: Report) -> None:
    """Conv, state update and gated norm, each from the kernel path's own inputs against fp32 math."""
    s, B = layer.ssm, ctx.B
    _fresh(layer, plan, dims, ctx, dev)
    st0 = alloc_and_fill(plan, dims, ctx, 0, dev)
    zx = K.gemm(x, rw.win, out=_rows16(B, rw.win.shape[0], dev), alpha=dims.ssm_in, colscale=rw.mup)
    z = zx[:, :s.sizes[0]]
    xBC = zx[:, s.sizes[0]:s.sizes[0] + s.sizes[1]].contiguous()
    dt = zx[:, s.sizes[0] + s.sizes[1]:]
    lines = ctx.state_idx.long()
    window = torch.cat([st0.conv_state[lines].float(), xBC.float()[:, None, :]], 1)
    conv_ref = F.silu((window * rw.conv_w.float().T[None]).sum(1) + rw.conv_b.float())
    conv_k = K.conv_update(xBC.clone(), s.conv_state_T, rw.conv_w, rw.conv_b, ctx.state_idx)
    rep("conv", conv_k, conv_ref)
    xk, Bk, Ck = torch.split(conv_k, list(s.xbc_sizes), dim=-1)
    nhr, p, N, ng = s.nhr, s.p, s.N, s.ng
    dtr = F.softplus(dt.float() + rw.dt_bias[None])
    dA = torch.exp(dtr * rw.A[None])
    gidx = torch.arange(nhr, device=dev) // (nhr // ng)
    xm = xk.float().view(B, nhr, p)
    Bm, Cm = Bk.float().view(B, ng, N)[:, gidx], Ck.float().view(B, ng, N)[:, gidx]
    state1 = st0.ssm_state[lines].float() * dA[:, :, None, None] + (dtr[:, :, None] * xm)[..., None] * Bm[:, :, None, :]
    y_ref = (state1 * Cm[:, :, None, :]).sum(-1) + rw.D[None, :, None] * xm
    K.ssm_update(s.st.ssm_state, xk.view(B, nhr, p), dt, rw.A, Bk.view(B, ng, N), Ck.view(B, ng, N), rw.D, rw.dt_bias,
                 ctx.state_idx, s.y)
    rep("ssu_y", s.y, y_ref)
    rep("ssu_state", s.st.ssm_state[lines], state1)
    yg = y_ref.reshape(B, nhr * p) * F.silu(z.float())
    gs = (nhr * p) // ng
    yg = yg.view(B, ng, gs)
    yg = (yg * torch.rsqrt(yg.pow(2).mean(-1, keepdim=True) + dims.rms_eps)).view(B, nhr * p) * rw.norm_w.float()
    out = torch.empty(B, nhr * p, device=dev, dtype=torch.bfloat16)
    K.gated_rmsnorm(y_ref.to(torch.bfloat16).reshape(B, nhr * p), z, rw.norm_w, dims.rms_eps, None,
                    gs if ng > 1 else None, out=out)
    rep("gated_norm", out, yg)


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model-dir", default=os.environ.get("MMP_MODEL_DIR", ""))
    ap.add_argument("--dims-yaml", default="falcon_h1_7b")
    ap.add_argument("--batch", type=int, default=2)
    ap.add_argument("--ctx", type=int, default=64)
    ap.add_argument("--random-weights", action="store_true")
    ap.add_argument("--ssm-substages", action="store_true")
    args = ap.parse_args(argv)
    g = init_groups()
    dev = g.device
    dims = FalconH1Dims.from_hf(args.model_dir) if args.model_dir else FalconH1Dims.from_yaml(args.dims_yaml)
    full = random_layer(dims, 0) if (args.random_weights or not args.model_dir) else \
        load_layer_from_safetensors(args.model_dir, 0)
    plan = plan_for("tp4", 0, 1, dims)  # one rank, branches unfused: every stage has its own output
    rw = shard_to_device(full, plan, dims, dev)
    ctx = make_decode_ctx(args.batch, args.ctx, 16, dev)
    st = alloc_and_fill(plan, dims, ctx, 0, dev)
    h = input_hidden(0, args.batch, dims.hidden, dev)
    layer = ParallelHybridLayer(plan, rw, dims, g, st, ctx, dev)
    inter: dict = {}
    kc, vc, conv, ssm = full_states_for_reference(dims, args.batch, args.ctx, 0, dev)
    ref_out = decode_step(full, dims, h, kc, vc, conv, ssm, args.ctx, intermediates=inter)
    rep = Report()
    print(f"dims: hidden={dims.hidden} rope_theta={dims.rope_theta} key_mult={dims.key_mult} "
          f"attn_in/out={dims.attn_in}/{dims.attn_out} ssm_in/out={dims.ssm_in}/{dims.ssm_out}", flush=True)
    x = K.rms_norm(h, rw.in_norm, dims.rms_eps, torch.empty_like(h))
    rep("norm_in", x, inter["x"])
    if args.ssm_substages:
        ssm_substages(layer, rw, dims, ctx, plan, dev, x, rep)
    else:
        attn_k = layer.attn.decode(x, NULL, out=torch.empty_like(h), x_scale=dims.attn_in)
        rep("attn_o", layer.attn.out2d, inter["o"])
        rep("attn_out", attn_k, inter["attn"])
        zx = K.gemm(x, rw.win, out=_rows16(args.batch, rw.win.shape[0], dev), alpha=dims.ssm_in, colscale=rw.mup)
        rep("zxbcdt", zx, inter["zxbcdt"])
        _fresh(layer, plan, dims, ctx, dev)
        ssm_k = layer.ssm.decode(x, NULL, out=torch.empty_like(h), x_scale=dims.ssm_in)
        rep("ssm_conv_state", layer.st.conv_state[ctx.state_idx.long()], inter["conv_state"])
        rep("ssm_state", layer.st.ssm_state[ctx.state_idx.long()], inter["ssm_state"])
        rep("y_ssm(gated norm)", layer.ssm.yn, inter["y_ssm"])
        rep("ssm_out", ssm_k, inter["ssm"])
        h1 = K.add(h, attn_k, torch.empty_like(h), c=ssm_k)
        rep("h1", h1, inter["h1"])
        if dims.intermediate > 0:
            y2 = K.rms_norm(h1, rw.ff_norm, dims.rms_eps, torch.empty_like(h1))
            mlp_k = layer.mlp.forward(y2, NULL, out=torch.empty_like(h1))
            rep("mlp", mlp_k, inter["out"] - inter["h1"])
        _fresh(layer, plan, dims, ctx, dev)
        out = layer.step(h, NULL)
        rep("final", out, ref_out)
    torch.cuda.synchronize()
    K.check_device_errors(dev)
    print(f"[debug] pass={rep.ok}", flush=True)
    destroy()
    return 0 if rep.ok else 1


if __name__ == "__main__":
    raise SystemExit(main())
