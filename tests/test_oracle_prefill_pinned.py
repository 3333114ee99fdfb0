"""The oracle's prefill (one fp32 decode step per position, oracle/hybrid_layer.py:prefill_sequential) against an
independent public implementation of the same layer: Hugging Face transformers' Falcon-H1 decoder layer (chunked
SSD scan in PyTorch, eager causal GQA attention, the same muP multipliers), through the golden fixture made by
tests/golden/make_hf_golden.py. Two cases: two B/C groups with the SwiGLU MLP and the 7B multipliers over 150
positions (chunk 64), and a one-group mixer-only layer over 97 positions (chunk 32). The reference harness has no
prefill; this anchors the prefill rows (the GPU prefill is tested against this oracle)."""
from pathlib import Path

import numpy as np
import pytest

import oracle
from multi_modal_parallelism_b200.weights import random_layer
from tests.golden.make_hf_golden import CASES, case_dims, case_input

G = np.load(Path(__file__).resolve().parent / "golden" / "hf_prefill_golden.npz")


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_oracle_prefill_matches_public_falcon_h1_layer(case):
    name, pre, over, L, wseed, hseed = case
    dims = case_dims(pre, over)
    full = {k: oracle.to_numpy(v) for k, v in random_layer(dims, wseed).items()}
    h = case_input(dims, L, hseed).numpy()
    outs = oracle.prefill_sequential(full, dims, [h])[0]
    ref = G[f"{name}_out"]
    assert float(np.linalg.norm(outs[0] - ref) / np.linalg.norm(ref)) < 1e-5
