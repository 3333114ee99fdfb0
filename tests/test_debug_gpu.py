"""The stage-by-stage diagnostic (python -m multi_modal_parallelism_b200.debug) on a B200: every stage of the kernel
path within tolerance of the fp32 layer's intermediate, for the full 7B layer (with MLP) and the 1024-wide layer's
Mamba-2 substages."""
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.run_last]
ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("args", [["--dims-yaml", "falcon_h1_7b", "--batch", "2", "--ctx", "64"],
                                  ["--dims-yaml", "hybrid_small", "--batch", "4", "--ctx", "100", "--ssm-substages"]])
def test_debug_stages_pass(args):
    r = subprocess.run(["timeout", "-k", "30", "600", sys.executable, "-m", "multi_modal_parallelism_b200.debug", *args],
                       cwd=ROOT, capture_output=True, text=True)
    out = r.stdout + r.stderr
    assert r.returncode == 0 and "[debug] pass=True" in out, out[-3000:]
