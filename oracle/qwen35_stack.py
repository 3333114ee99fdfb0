"""numpy fp32 restatement of the Gated DeltaNet hybrid block stack (delta-rule and GQA attention layers, each
followed by a SwiGLU MLP): test infrastructure only.

The reference has no implementation of this model family (its config, `configs/qwen35_35b_a3b.yaml:1-22`, is
a description, and `harness/synth.py:114-160` a byte model): parity unpinned. Delta-rule layers are
`gdn_layer.gdn_layer_prefill` / `gdn_layer_decode`; the attention layer restated here is the attention branch
of the reference's fp32 layer (`harness/reference.py:52-68`: QKV projection, NeoX RoPE at the token's position,
causal GQA softmax attention over the sequence's keys, o-projection) without Falcon's multipliers, plus the
residual and the SwiGLU MLP of `harness/reference.py:112-119`. Weights are the package's `random_stack` dicts
converted with `to_numpy`; dims need the fields of `Qwen35Dims`.

State per layer and sequence: delta-rule layers (conv window [d_conv - 1, q|k|v rows], delta-rule state
[n_v, dv, dk]); attention layers (keys, values [positions, n_kv, hd], keys after RoPE).
"""
from __future__ import annotations

import math

import numpy as np

from .gdn_layer import gdn_layer_decode, gdn_layer_prefill
from .hybrid_layer import F32, apply_rope_neox, gemm, rmsnorm, rope_cos_sin, silu


def _mlp(w: dict, d, h1: np.ndarray) -> np.ndarray:
    y = rmsnorm(h1, w["post_attention_layernorm.weight"], d.rms_eps)
    g = silu(gemm(y, w["mlp.gate_proj.weight"])) * gemm(y, w["mlp.up_proj.weight"])
    return h1 + gemm(g, w["mlp.down_proj.weight"])


def attn_layer(w: dict, d, h: np.ndarray, K: np.ndarray | None, V: np.ndarray | None):
    """New tokens h [L, H] of one sequence, after the cached keys/values K, V [P, n_kv, hd] (None: P = 0).
    Token i sits at position P + i and attends to positions 0 .. P + i. Returns (out [L, H], K', V')."""
    h = h.astype(F32)
    L, hd = h.shape[0], d.head_dim
    P = 0 if K is None else K.shape[0]
    x = rmsnorm(h, w["input_layernorm.weight"], d.rms_eps)
    q = gemm(x, w["self_attn.q_proj.weight"]).reshape(L, d.n_q, hd)
    k = gemm(x, w["self_attn.k_proj.weight"]).reshape(L, d.n_kv, hd)
    v = gemm(x, w["self_attn.v_proj.weight"]).reshape(L, d.n_kv, hd)
    cos, sin = rope_cos_sin(np.arange(P, P + L), hd, d.rope_theta)
    q, k = apply_rope_neox(q, cos, sin), apply_rope_neox(k, cos, sin)
    K2 = k if K is None else np.concatenate([K, k], 0)
    V2 = v if V is None else np.concatenate([V, v], 0)
    rep = d.n_q // d.n_kv
    o = np.zeros((L, d.n_q, hd), F32)
    allowed = np.arange(P + L)[None, :] <= (P + np.arange(L))[:, None]  # [L, P + L]
    for hh in range(d.n_q):
        s = (q[:, hh] @ K2[:, hh // rep].T) * F32(1.0 / math.sqrt(hd))
        s = np.where(allowed, s, -np.inf)
        s = s - s.max(-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(-1, keepdims=True)
        o[:, hh] = p @ V2[:, hh // rep]
    h1 = h + gemm(o.reshape(L, -1), w["self_attn.o_proj.weight"])
    return _mlp(w, d, h1), K2, V2


def stack_prefill(ws: list[dict], d, hs: list[np.ndarray], state: list | None = None):
    """Prefill of sequences hs[i] [L_i, H] through every layer, each sequence from its state in `state`
    (per layer: a list over sequences of (conv, S) or (K, V) tuples, entries None = fresh) or fresh.
    Returns (outputs per sequence, new state)."""
    n = len(hs)
    state = [[None] * n for _ in ws] if state is None else state
    new_state = []
    for li, (kind, w) in enumerate(zip(d.layout, ws)):
        outs, st = [], []
        for i, h in enumerate(hs):
            s0 = state[li][i]
            if kind == "G":
                o, conv, S = gdn_layer_prefill(w, d, h, None if s0 is None else s0[0], None if s0 is None else s0[1])
                st.append((conv, S))
            else:
                o, K, V = attn_layer(w, d, h, None if s0 is None else s0[0], None if s0 is None else s0[1])
                st.append((K, V))
            outs.append(o)
        hs = outs
        new_state.append(st)
    return hs, new_state


def stack_decode(ws: list[dict], d, h: np.ndarray, state: list):
    """One token per sequence (h [B, H], sequence b = row b) through every layer from `state` (as returned by
    stack_prefill, one entry per row). Returns (out [B, H], new state)."""
    B = h.shape[0]
    new_state = []
    for li, (kind, w) in enumerate(zip(d.layout, ws)):
        st = state[li]
        if kind == "G":
            conv = np.stack([s[0] for s in st])
            S = np.stack([s[1] for s in st])
            h, conv, S = gdn_layer_decode(w, d, h, conv, S)
            new_state.append([(conv[b], S[b]) for b in range(B)])
        else:
            outs, ns = [], []
            for b in range(B):
                o, K, V = attn_layer(w, d, h[b:b + 1], st[b][0], st[b][1])
                outs.append(o)
                ns.append((K, V))
            h = np.concatenate(outs, 0)
            new_state.append(ns)
    return h, new_state
