"""CUDA-event op timer and step timing, eager and CUDA-graph (same API as the reference's
`harness/timing.py`: `OpTimer` :12-42, `time_eager` :60-73, `time_graph` :76-104)."""
from __future__ import annotations

import statistics
import time

import torch

from .dist import Groups, barrier_sync, capture_context


class OpTimer:
    """Records a CUDA event pair per named op on the current stream."""

    def __init__(self, enabled: bool = True):
        self.enabled = enabled
        self._open: dict[str, torch.cuda.Event] = {}
        self.pairs: dict[str, list[tuple[torch.cuda.Event, torch.cuda.Event]]] = {}

    def _event(self) -> torch.cuda.Event:
        e = torch.cuda.Event(enable_timing=True)
        e.record(torch.cuda.current_stream())
        return e

    def begin(self, name: str) -> None:
        if self.enabled:
            self._open[name] = self._event()

    def end(self, name: str) -> None:
        if self.enabled:
            self.pairs.setdefault(name, []).append((self._open.pop(name), self._event()))

    def reset(self) -> None:
        self._open.clear()
        self.pairs.clear()

    def summarize(self) -> dict[str, dict[str, float]]:
        torch.cuda.synchronize()
        return {name: stats([s.elapsed_time(e) for s, e in pairs]) for name, pairs in self.pairs.items()}


NULL = OpTimer(enabled=False)


def stats(ms: list[float]) -> dict[str, float]:
    xs = sorted(ms)
    n = len(xs)
    return {
        "n": n,
        "median_ms": statistics.median(xs),
        "p10_ms": xs[max(0, int(0.1 * n) - 1)] if n > 1 else xs[0],
        "p90_ms": xs[min(n - 1, int(0.9 * n))],
        "mean_ms": statistics.fmean(xs),
    }


def time_eager(layer, h: torch.Tensor, n_warm: int, n_iter: int, groups: Groups) -> tuple[dict, float]:
    """(per-op stats including 'step', wall ms per step)."""
    for _ in range(n_warm):
        layer.step(h, NULL)
    barrier_sync()
    t = OpTimer(enabled=True)
    t0 = time.perf_counter()
    for _ in range(n_iter):
        t.begin("step")
        layer.step(h, t)
        t.end("step")
    torch.cuda.synchronize()
    wall = (time.perf_counter() - t0) * 1e3 / n_iter
    return t.summarize(), wall


def capture_step(layer, h: torch.Tensor, groups: Groups, warm: int = 2) -> torch.cuda.CUDAGraph:
    """Capture one whole layer step (collectives included) into a CUDA graph."""
    with capture_context(groups) as ctx:
        with torch.cuda.stream(ctx.stream):
            for _ in range(warm):
                layer.step(h, NULL)
        ctx.stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=ctx.stream):
            layer.step(h, NULL)
    torch.cuda.synchronize()
    return g


def time_graph(layer, h: torch.Tensor, n_warm: int, n_iter: int, groups: Groups) -> tuple[dict, float]:
    g = capture_step(layer, h, groups)
    for _ in range(n_warm):
        g.replay()
    barrier_sync()
    events = []
    t0 = time.perf_counter()
    for _ in range(n_iter):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        g.replay()
        e.record()
        events.append((s, e))
    torch.cuda.synchronize()
    wall = (time.perf_counter() - t0) * 1e3 / n_iter
    return {"step": stats([s.elapsed_time(e) for s, e in events])}, wall


class GraphedStep:
    """A layer decode step captured once and replayed: the serving call. `__call__(h_host, out_host)` copies
    the step's input from (pinned) host memory into the captured input buffer, replays the step, and copies
    the output back to host memory, all on the current stream."""

    def __init__(self, layer, groups: Groups, h_static: torch.Tensor):
        self.layer = layer
        self.h = h_static
        self.graph = capture_step(layer, h_static, groups)

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.layer.out

    def __call__(self, h_host: torch.Tensor | None = None, out_host: torch.Tensor | None = None) -> torch.Tensor:
        if h_host is not None:
            self.h.copy_(h_host, non_blocking=True)
        self.graph.replay()
        if out_host is None:
            return self.layer.out
        out_host.copy_(self.layer.out, non_blocking=True)
        return out_host

    def release(self) -> None:
        """Drop the graph (graphs holding NCCL calls must go before the process group is destroyed)."""
        self.graph = None
