"""Loader for libmmp_b200.so (the C ABI declared in include/mmp_b200.h).

The library is built in-tree by `multi_modal_parallelism_b200.build`. There is no fallback: if the
library is missing or a call fails, this module raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(os.environ.get("MMP_B200_LIB", Path(__file__).resolve().parent / "libmmp_b200.so"))

MMP_OK, MMP_ERR_INVALID, MMP_ERR_CUDA, MMP_ERR_UNSUPPORTED, MMP_ERR_TIMEOUT = 0, 1, 2, 3, 4
MMP_F32, MMP_BF16 = 0, 1
DEVERR = {1: "index out of range", 2: "position out of range", 4: "bounded wait timed out"}

P, I64, I32, F32, SZ = C.c_void_p, C.c_int64, C.c_int, C.c_float, C.c_size_t

# name -> (restype, argtypes); mirrors include/mmp_b200.h
SIGNATURES: dict[str, tuple] = {
    "mmp_version": (I32, []),
    "mmp_last_error": (C.c_char_p, []),
    "mmp_set_pdl": (I32, [I32]),
    "mmp_set_attn_prefill_tc": (I32, [I32]),
    "mmp_set_ssd_prefill_tc": (I32, [I32]),
    "mmp_set_gemm_decode_split": (I32, [I32]),
    "mmp_set_gemm_decode_stages": (I32, [I32]),
    "mmp_scale_rows": (I32, [P, I64, P, I32, I32, F32, F32, P]),
    "mmp_ssu_decode": (I32, [P, I32, I64, I64, I64, P, I64, I64, P, I64, I64, P, P, P, P, I64, I64, P, I64, I64,
                             P, I64, I64, P, P, I32, P, I64, I64, I32, I32, I32, I32, I32, I32, I32, P, P]),
    "mmp_conv1d_update": (I32, [P, I64, P, I64, P, I64, I64, I64, P, P, P, I32, I32, I32, I32, I32, I32, P, P]),
    "mmp_rmsnorm": (I32, [P, I64, P, I64, P, I64, P, P, I64, I32, I32, F32, P]),
    "mmp_gated_rmsnorm": (I32, [P, I64, P, I64, P, P, I64, P, I32, I32, I32, I32, F32, F32, P]),
    "mmp_rope_kv_write": (I32, [P, I64, P, I64, P, I64, I32, I32, I32, P, P, I32, P, F32, P, I64, P, I64,
                                P, P, I64, I64, I64, I32, I32, P, I32, P, P]),
    "mmp_silu_mul": (I32, [P, I64, P, I64, P, I64, I32, I32, F32, P]),
    "mmp_paged_attn_workspace_size": (SZ, [I32, I32, I32, I32]),
    "mmp_paged_attn_decode": (I32, [P, I64, I64, P, P, I64, I64, I64, P, I64, P, P, I64, I64, I32, I32, I32, I32, I32,
                                    I32, I32, F32, I32, P, SZ, P, P]),
    "mmp_paged_attn_default_splits": (I32, [I32, I32, I32]),
    "mmp_paged_attn_decode_noalloc": (I32, [P, I64, I64, P, P, I64, I64, I64, P, I64, P, P, I64, I64, I32, I32, I32,
                                            I32, I32, I32, I32, F32, I32, P, P]),
    "mmp_gemm_bf16": (I32, [P, I64, P, I64, P, I64, I32, I32, I32, F32, P, P, I64, P]),
    "mmp_gemm_bf16_tc": (I32, [P, I64, P, I64, P, I64, I32, I32, I32, F32, P, P, I64, P, P]),
    "mmp_gemm_bf16_seg": (I32, [P, I64, P, I64, P, I64, I32, I32, I32, F32, I32, F32, P, P, I64, P, P]),
    "mmp_conv1d_prefill": (I32, [P, I64, P, I64, P, I64, I64, P, P, P, P, P, I32, I32, I32, I32, I32, I32, P, P]),
    "mmp_ssd_prefill": (I32, [P, I64, I64, P, I64, I64, P, P, P, P, I64, I64, P, I64, I64, P, I32, I64, I64, I64,
                              P, P, P, P, I64, I64, I32, I32, I32, I32, I32, I32, I32, P, P]),
    "mmp_ssd_prefill_seg": (I32, [P, I64, I64, P, I64, I64, P, P, P, P, I64, I64, P, I64, I64, P, I32, I64, I64, I64,
                                  P, P, P, I64, I64, P, P, P, P, P, I32, I32, I32, I32, I32, I32, I32, I32, I32, P, P]),
    "mmp_paged_attn_prefill": (I32, [P, I64, I64, P, P, I64, I64, I64, P, I64, P, P, P, I64, I64, I32, I32, I32, I32,
                                     I32, I32, I32, F32, P, P]),
    "mmp_add": (I32, [P, I64, P, I64, P, I64, P, I64, I32, I32, P]),
    "mmp_ar_buffer_bytes": (SZ, [I32, I32, I32]),
    "mmp_ipc_export": (I32, [P, P]),
    "mmp_ipc_import": (I32, [P, P]),
    "mmp_ipc_release": (I32, [P]),
    "mmp_ar_join": (I32, [P, I32, I32, I32, I32, P, I64, P, I64, P, I64, P, F32, P, I64, I32, I32, P, P]),
    "mmp_gemm_bf16_push": (I32, [P, I64, P, I64, I32, I32, I32, F32, I32, F32, P, P, I32, I32, I32, P, P]),
    "mmp_gn_buffer_bytes": (SZ, [I32, I32]),
    "mmp_gated_rmsnorm_p2p": (I32, [P, I32, I32, I32, P, I64, P, I64, P, P, I64, I32, I32, F32, P, P]),
    "mmp_gdn_decode": (I32, [P, I64, I64, I64, P, I64, I64, P, I64, I64, P, I64, I64, P, I64, P, I64, P, P,
                             P, I64, I64, P, F32, P, I32, P, I64, I64, I32, I32, I32, I32, I32, I32, P, P]),
    "mmp_gdn_prefill": (I32, [P, I64, I64, P, I64, I64, P, I64, I64, P, I64, P, I64, P, P, P, I64, I64, P, F32,
                              P, I64, I64, I64, P, P, P, P, I64, I64, I32, I32, I32, I32, I32, I32, I32, P, P]),
    "mmp_gdn_prefill_workspace_size": (SZ, [I32, I32]),
    "mmp_gdn_prefill_tc": (I32, [P, I64, I64, P, I64, I64, P, I64, I64, P, I64, P, I64, P, P, P, I64, I64, P, F32,
                                 P, I64, I64, I64, P, P, P, P, I64, I64, I32, I32, I32, I32, I32, I32, I32, P, SZ, P,
                                 P]),
}

_lib: C.CDLL | None = None


class MmpError(RuntimeError):
    pass


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} not found: build it with `python -m multi_modal_parallelism_b200.build`")
        h = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(h, name)
            fn.restype, fn.argtypes = res, args
        _lib = h
    return _lib


def check(rc: int, what: str) -> None:
    if rc != MMP_OK:
        msg = lib().mmp_last_error().decode(errors="replace")
        if rc == MMP_ERR_INVALID:
            raise ValueError(f"{what}: {msg}")
        raise MmpError(f"{what}: status {rc}: {msg}")


LAUNCHES = [0]  # kernel launches issued through this module (a counter for launch accounting)


def call(name: str, *args, kernels: int = 1) -> None:
    check(getattr(lib(), name)(*args), name)
    LAUNCHES[0] += kernels
