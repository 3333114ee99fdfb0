"""Peer-memory all-reduce over NVLink for decode-sized [rows, H] partial sums (libmmp_b200's mmp_ar_join): a
one-shot all-reduce fused with the residual add and the next RMSNorm, replacing an NCCL all-reduce plus the
norm kernel after it (the reference's `ParallelHybridLayer._ar`, `harness/layer.py:175-181`, and the residual /
pre-MLP norm, `harness/layer.py:217-227`).

Setup is collective over the group: every rank allocates a zeroed buffer, exports it as a CUDA IPC blob, the blobs
are exchanged with `torch.distributed.all_gather_object`, and each rank maps the others'. Calls are then plain
kernel launches (graph-capturable); every rank must make the same sequence of calls. `gemm` + `join(None, ...)` is
the fused form: the producing decode GEMM writes its output tiles into every rank's buffer as they finish, so the
transfer overlaps the GEMM, and the join kernel only waits, sums and normalises.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .dist import Coordinator

BLOB_BYTES = 72


class _PeerBuffer:
    """A zeroed device buffer of `nbytes` on every rank of `group`, mapped into every rank (CUDA IPC). Collective
    over `group` (every member constructs it, in the same order as its other collectives)."""

    def __init__(self, group: Coordinator, global_rank: int, nbytes: int, device: torch.device):
        if not 1 <= group.world_size <= 8:
            raise ValueError(f"{type(self).__name__}: {group.world_size} ranks (1..8 on one node)")
        self.world, self.rank, self.device = group.world_size, group.ranks.index(global_rank), device
        self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        torch.cuda.synchronize(device)  # the zeros must be in place before any peer can write
        blob = ctypes.create_string_buffer(BLOB_BYTES)
        _lib.call("mmp_ipc_export", self.buf.data_ptr(), blob, kernels=0)
        blobs: list = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(blobs, blob.raw, group=group.pg)
        else:
            blobs = [blob.raw]
        self._imported: list[int] = []
        ptrs = []
        for q, b in enumerate(blobs):
            if q == self.rank:
                ptrs.append(self.buf.data_ptr())
                continue
            out = ctypes.c_void_p()
            _lib.call("mmp_ipc_import", ctypes.create_string_buffer(b, BLOB_BYTES), ctypes.byref(out), kernels=0)
            ptrs.append(int(out.value))
            self._imported.append(int(out.value))
        self.bufs = torch.tensor(ptrs, dtype=torch.int64, device=device)
        if self.world > 1:
            dist.barrier(group=group.pg)

    def close(self) -> None:
        """Unmap the peers' buffers (after the last call has finished on this rank)."""
        for ptr in self._imported:
            _lib.call("mmp_ipc_release", ptr, kernels=0)
        self._imported = []


class PeerAllReduce(_PeerBuffer):
    def __init__(self, group: Coordinator, global_rank: int, rows_max: int, hidden: int, device: torch.device):
        """Collective over `group` (every member calls it, in the same order as its other collectives)."""
        self.rows_max, self.hidden = rows_max, hidden
        nbytes = int(_lib.lib().mmp_ar_buffer_bytes(group.world_size, rows_max, hidden))
        super().__init__(group, global_rank, nbytes, device)
        self._pushed_rows = 0

    def gemm(self, x: torch.Tensor, w: torch.Tensor, alpha: float = 1.0, colscale: torch.Tensor | None = None,
             k_seg: int | None = None, alpha2: float | None = None) -> None:
        """This rank's partial alpha * colscale * (x @ w^T) (x: [rows <= 256, K] decode rows; w: [hidden, K]),
        written by the GEMM straight into every rank's buffer; complete it with join(None, ..., pushed rows)."""
        from .kernels import _cuda, _dtype, _rowmajor, _stream, error_word

        M, K = x.shape
        if w.shape[0] != self.hidden or w.shape[1] != K or M > self.rows_max:
            raise ValueError(f"PeerAllReduce.gemm: x {tuple(x.shape)} w {tuple(w.shape)} for [{self.rows_max}, "
                             f"{self.hidden}]")
        _cuda("PeerAllReduce.gemm", x, w, colscale)
        for t in (x, w):
            _dtype("PeerAllReduce.gemm", t, torch.bfloat16)
        if colscale is not None and (colscale.dtype != torch.float32 or colscale.numel() != self.hidden):
            raise ValueError("PeerAllReduce.gemm: colscale must be fp32 [hidden]")
        ks = K if k_seg is None else int(k_seg)
        a2 = float(alpha if alpha2 is None else alpha2)
        _lib.call("mmp_gemm_bf16_push", x.data_ptr(), _rowmajor("x", x), w.data_ptr(), _rowmajor("w", w), M,
                  self.hidden, K, float(alpha), ks, a2, None if colscale is None else colscale.data_ptr(),
                  self.bufs.data_ptr(), self.rank, self.world, self.rows_max, error_word(x.device).data_ptr(),
                  _stream(x))
        self._pushed_rows = M

    def join(self, part: torch.Tensor | None, resid: torch.Tensor | None, sum_out: torch.Tensor,
             norm_w: torch.Tensor | None = None, eps: float = 0.0, norm_out: torch.Tensor | None = None) -> torch.Tensor:
        """sum_out = resid + all-reduce(part) (bf16); with norm_w also norm_out = rmsnorm(sum_out) * norm_w.
        part None: the partial is the one the last gemm() pushed. Returns norm_out when given, else sum_out."""
        from .kernels import _cuda, _dtype, _rowmajor, _stream, error_word

        pushed = part is None
        rows, H = (self._pushed_rows, self.hidden) if pushed else part.shape
        if H != self.hidden or rows > self.rows_max:
            raise ValueError(f"PeerAllReduce.join: [{rows}, {H}] does not fit [{self.rows_max}, {self.hidden}]")
        _cuda("PeerAllReduce.join", part, resid, sum_out, norm_w, norm_out)
        for t in (part, resid, sum_out, norm_w, norm_out):
            _dtype("PeerAllReduce.join", t, torch.bfloat16)
        if (norm_w is None) != (norm_out is None):
            raise ValueError("PeerAllReduce.join: norm_w and norm_out go together")
        p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        ld = lambda n, t: 0 if t is None else _rowmajor(n, t)  # noqa: E731
        if sum_out.shape[0] != rows:
            raise ValueError(f"PeerAllReduce.join: sum_out has {sum_out.shape[0]} rows, the partial {rows}")
        _lib.call("mmp_ar_join", self.bufs.data_ptr(), self.rank, self.world, self.rows_max, 1 if pushed else 0,
                  p(part), ld("part", part), p(resid), ld("resid", resid), sum_out.data_ptr(),
                  ld("sum_out", sum_out), p(norm_w), float(eps), p(norm_out), ld("norm_out", norm_out),
                  rows, H, error_word(sum_out.device).data_ptr(), _stream(sum_out))
        return norm_out if norm_out is not None else sum_out


class PeerRowNorm(_PeerBuffer):
    """The Mamba-2 gated RMSNorm whose row statistic spans the ranks of a norm group (mmp_gated_rmsnorm_p2p): the
    partial sums of squares go straight to every rank's buffer, with no separate all-reduce launch."""

    def __init__(self, group: Coordinator, global_rank: int, rows_max: int, device: torch.device):
        self.rows_max = rows_max
        super().__init__(group, global_rank, int(_lib.lib().mmp_gn_buffer_bytes(group.world_size, rows_max)), device)

    def __call__(self, y: torch.Tensor, z: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor) -> torch.Tensor:
        from .kernels import _cuda, _dtype, _rowmajor, _stream, error_word

        rows, D = y.shape
        if rows > self.rows_max or z.shape != y.shape or out.shape != y.shape or w.numel() != D:
            raise ValueError(f"PeerRowNorm: y {tuple(y.shape)} z {tuple(z.shape)} out {tuple(out.shape)} w {w.numel()}")
        _cuda("PeerRowNorm", y, z, w, out)
        for t in (y, z, w, out):
            _dtype("PeerRowNorm", t, torch.bfloat16)
        _lib.call("mmp_gated_rmsnorm_p2p", self.bufs.data_ptr(), self.rank, self.world, self.rows_max, y.data_ptr(),
                  _rowmajor("y", y), z.data_ptr(), _rowmajor("z", z), w.data_ptr(), out.data_ptr(),
                  _rowmajor("out", out), rows, D, float(eps), error_word(y.device).data_ptr(), _stream(y))
        return out
