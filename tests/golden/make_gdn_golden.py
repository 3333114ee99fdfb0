"""Generate the golden fixture that cross-checks the Gated DeltaNet oracle (oracle/gdn_layer.py) against an
independent published implementation of the gated delta rule: flash-linear-attention's (fla 0.5.1, third-party,
installed in this image) pure-PyTorch reference functions `fla.ops.gated_delta_rule.naive.
naive_recurrent_gated_delta_rule` and `naive_chunk_gated_delta_rule`. The reference harness has no implementation
of these layers (its config is a description), so this pins the oracle's conventions (log-space decay, the beta
write strength, the state's orientation, q scaling) to the algorithm's public implementation.

    python tests/golden/make_gdn_golden.py

Writes gdn_fla_golden.npz: q, k (L2-normalised), v, g, beta, an initial state, and FLA's outputs and final states
(recurrent and chunk-64 forms) for one sequence of 2 heads.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def main() -> None:
    from fla.ops.gated_delta_rule.naive import naive_chunk_gated_delta_rule, naive_recurrent_gated_delta_rule

    g = torch.Generator().manual_seed(0)
    T, H, K, V = 150, 2, 32, 32
    q = torch.nn.functional.normalize(torch.randn(1, T, H, K, generator=g), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(1, T, H, K, generator=g), dim=-1)
    v = torch.randn(1, T, H, V, generator=g)
    gl = -torch.nn.functional.softplus(torch.randn(1, T, H, generator=g))  # log decay
    beta = torch.sigmoid(torch.randn(1, T, H, generator=g))
    s0 = torch.randn(1, H, K, V, generator=g) * 0.3
    scale = K ** -0.5
    o_r, s_r = naive_recurrent_gated_delta_rule(q, k, v, beta, gl, scale=scale, initial_state=s0,
                                                output_final_state=True)
    o_c, s_c = naive_chunk_gated_delta_rule(q, k, v, gl, beta, chunk_size=64, scale=scale, initial_state=s0,
                                            output_final_state=True)
    f = lambda t: t.detach().float().numpy()  # noqa: E731
    np.savez_compressed(HERE / "gdn_fla_golden.npz", q=f(q[0]), k=f(k[0]), v=f(v[0]), g=f(gl[0]), beta=f(beta[0]),
                        s0=f(s0[0]), scale=np.float32(scale), o_recurrent=f(o_r[0]), s_recurrent=f(s_r[0]),
                        o_chunk=f(o_c[0]), s_chunk=f(s_c[0]))
    print("wrote gdn_fla_golden.npz")


if __name__ == "__main__":
    main()
