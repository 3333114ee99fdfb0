"""The C-ABI library loads on a machine without a GPU and exports every function the header declares,
and the Python signature table agrees with the header."""
import ctypes
import re
from pathlib import Path

import pytest

from multi_modal_parallelism_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared() -> list[str]:
    names = []
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(mmp_\w+)\s*\(", text, flags=re.M)
    return names


def test_header_declares_functions():
    names = declared()
    assert "mmp_ssu_decode" in names and "mmp_gemm_bf16" in names and len(names) == len(set(names))


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_signature_table_covers_header():
    assert set(declared()) == set(_lib.SIGNATURES), set(declared()) ^ set(_lib.SIGNATURES)


def test_argument_counts_match_header():
    text = "\n".join(re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S) for h in HEADERS)
    for name, (_, args) in _lib.SIGNATURES.items():
        m = re.search(rf"\b{name}\s*\((.*?)\)\s*;", text, flags=re.S)
        assert m, name
        params = [p for p in m.group(1).split(",") if p.strip() and p.strip() != "void"]
        assert len(params) == len(args), f"{name}: header {len(params)} args, table {len(args)}"


def test_version_and_error_calls_need_no_gpu():
    lib = _lib.lib()
    assert lib.mmp_version() >= 100
    assert lib.mmp_last_error() is not None


def test_invalid_arguments_rejected_without_gpu():
    # validation happens before any CUDA call, so it runs here
    with pytest.raises(ValueError):
        _lib.call("mmp_gemm_bf16", 16, 8, 16, 8, 16, 8, 4, 4, 7, 1.0, None, None, 0, None)  # K % 8 != 0
    # every pointer NULL, every size 1: rejected as a null-pointer request
    args = [None if t is _lib.P else 1 for t in _lib.SIGNATURES["mmp_ssu_decode"][1]]
    with pytest.raises(ValueError):
        _lib.call("mmp_ssu_decode", *args)
