"""Process groups for the layer: one process per GPU over torch.distributed (NCCL on GPUs, gloo on CPU).

Same surface as the reference's `harness/dist.py` (`Groups` :16-34, `init_groups` :55-73,
`capture_context` :95-107, `barrier_sync` :110-113, `destroy` :116-120), without vLLM: a `Coordinator`
stands in for vLLM's GroupCoordinator (`all_reduce(t) -> t`, `world_size`, `ranks`). `group_for_ranks`
serves any rank set, so every split{a}{m} layout works: sets that are not pre-built (the world, the
consecutive pairs and quads the reference builds) are created collectively by `ensure`.
"""
from __future__ import annotations

import os
from contextlib import contextmanager
from dataclasses import dataclass, field
from datetime import timedelta
from typing import Iterator

import torch
import torch.distributed as dist


@dataclass
class Coordinator:
    ranks: tuple[int, ...]
    pg: object | None  # torch ProcessGroup (None: the default group, or a single process)

    @property
    def world_size(self) -> int:
        return len(self.ranks)

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        """In-place sum over the group's ranks; returns t."""
        if self.world_size > 1:
            dist.all_reduce(t, group=self.pg)
        return t

    def all_gather_rows(self, out: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
        """out [world * n, ...] <- every rank's t [n, ...] in rank order (contiguous tensors); returns out."""
        if self.world_size == 1:
            if out.data_ptr() != t.data_ptr():
                out.copy_(t)
            return out
        if out.is_cuda:
            dist.all_gather_into_tensor(out, t, group=self.pg)
        else:  # gloo: one output view per rank
            dist.all_gather(list(out.chunk(self.world_size)), t, group=self.pg)
        return out


@dataclass
class Groups:
    rank: int
    local_rank: int
    world_size: int
    tp: Coordinator
    pair: Coordinator | None
    device: torch.device
    quad: Coordinator | None = None
    extra: dict = field(default_factory=dict)
    prebuilt: frozenset = frozenset()  # every pre-built block set (all pairs / quads), the same on every rank
    created: set = field(default_factory=set)  # sets made by ensure(), the same on every rank

    def group_for_ranks(self, ranks: tuple[int, ...]) -> Coordinator | None:
        """The coordinator whose membership equals `ranks`, or None for a single rank."""
        ranks = tuple(ranks)
        if len(ranks) <= 1:
            return None
        if len(ranks) == self.world_size:
            return self.tp
        for g in (self.pair, self.quad, self.extra.get(ranks)):
            if g is not None and g.ranks == ranks and self.rank in ranks:
                return g
        raise ValueError(f"no communicator for ranks {ranks} (rank {self.rank})")

    def ensure(self, rank_sets: list[tuple[int, ...]]) -> None:
        """Collectively create communicators for `rank_sets` (every rank must call this with the same list).

        dist.new_group is collective over the whole world, so whether a set is skipped must not depend on the
        calling rank: sets that were pre-built (any rank's pair or quad) or created earlier are skipped on
        every rank alike."""
        for rs in rank_sets:
            rs = tuple(rs)
            if len(rs) <= 1 or len(rs) == self.world_size or rs in self.prebuilt or rs in self.created:
                continue
            pg = dist.new_group(list(rs))
            self.created.add(rs)
            if self.rank in rs:
                self.extra[rs] = Coordinator(rs, pg)


def _blocks(world: int, size: int, backend: str | None) -> list[tuple[tuple[int, ...], object]]:
    out = []
    for i in range(world // size):
        rs = tuple(range(i * size, (i + 1) * size))
        out.append((rs, dist.new_group(list(rs), backend=backend)))
    return out


def init_groups(backend: str | None = None, timeout_s: float = 300.0) -> Groups:
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", str(rank)))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    use_cuda = torch.cuda.is_available() and backend != "gloo"
    if use_cuda:
        torch.cuda.set_device(local_rank)
        device = torch.device("cuda", local_rank)
    else:
        device = torch.device("cpu")
    if world > 1 and not dist.is_initialized():
        be = backend or ("nccl" if use_cuda else "gloo")
        kw = {"device_id": device} if be == "nccl" else {}
        dist.init_process_group(be, rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s), **kw)
    tp = Coordinator(tuple(range(world)), None)
    pair = quad = None
    prebuilt = set()
    if world >= 4 and world % 2 == 0:
        for rs, pg in _blocks(world, 2, None):
            prebuilt.add(rs)
            if rank in rs:
                pair = Coordinator(rs, pg)
    if world >= 8 and world % 4 == 0:
        for rs, pg in _blocks(world, 4, None):
            prebuilt.add(rs)
            if rank in rs:
                quad = Coordinator(rs, pg)
    return Groups(rank=rank, local_rank=local_rank, world_size=world, tp=tp, pair=pair, device=device, quad=quad,
                  prebuilt=frozenset(prebuilt))


def describe_comm(g: Coordinator | None) -> dict:
    if g is None:
        return {"ranks": None}
    info = {"ranks": list(g.ranks), "world_size": g.world_size, "backend": None, "nccl_version": None}
    if dist.is_initialized():
        info["backend"] = str(dist.get_backend(g.pg))
        try:
            info["nccl_version"] = ".".join(map(str, torch.cuda.nccl.version()))
        except Exception:  # pragma: no cover
            pass
    return info


@dataclass
class _CaptureCtx:
    stream: torch.cuda.Stream


@contextmanager
def capture_context(groups: Groups) -> Iterator[_CaptureCtx]:
    """A side stream on which a whole step, collectives included, is warmed up and captured."""
    s = torch.cuda.Stream(device=groups.device)
    s.wait_stream(torch.cuda.current_stream(groups.device))
    yield _CaptureCtx(stream=s)
    torch.cuda.current_stream(groups.device).wait_stream(s)


def barrier_sync() -> None:
    if torch.cuda.is_available():
        torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier()


def destroy() -> None:
    if dist.is_initialized():
        dist.destroy_process_group()
