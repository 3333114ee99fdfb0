"""Balanced walks for the prefill SSD scan (libmmp_b200's mmp_ssd_prefill_seg): where to cut each sequence.

The chunked scan runs one CTA per (head, sequence), walking the sequence's 64-token chunks in order, one CTA per
SM (its state lives in tensor memory). With nh x nseq walks slightly above a multiple of the SM count, the last
wave runs almost empty: 24 heads x 8 sequences = 192 walks of 32 chunks on 148 SMs take two full walk lengths.
Cutting each sequence into segments at chunk boundaries turns the walks into more, shorter ones that pack the
waves; the segments are joined afterwards (chained states, a correction of the later segments' outputs).

`plan_counts` chooses the cuts by simulating the block scheduler: walks dispatched in grid order (heads fastest,
then segments in token order) onto the SMs as they free up, each walk costing its chunks plus a fixed set-up, plus
the join's cost per corrected chunk; the segment length with the smallest estimate wins. Costs are in units of one
chunk step of the scan.
"""
from __future__ import annotations

import heapq
import math
from dataclasses import dataclass

import torch

CHUNK = 64


def _makespan(walks: list[float], slots: int) -> float:
    free = [0.0] * slots
    heapq.heapify(free)
    end = 0.0
    for w in walks:
        t = heapq.heappop(free) + w
        end = max(end, t)
        heapq.heappush(free, t)
    return end


def split_chunks(chunks: int, m: int) -> list[int]:
    """`chunks` chunks in `m` near-equal segments (longer ones first)."""
    q, r = divmod(chunks, m)
    return [q + 1] * r + [q] * (m - r)


def plan_counts(lens: list[int], nh: int, n_sm: int, max_segments: int = 8, walk_overhead: float = 0.5,
                join_per_chunk: float = 0.15, join_fixed: float = 1.0) -> list[int]:
    """Segments per sequence (1 = not cut) minimising the estimated scan + join time (the join, when anything is
    cut, costs `join_fixed` for its launches and state copies plus `join_per_chunk` per corrected chunk of the
    longest-corrected sequence)."""
    chunks = [math.ceil(L / CHUNK) for L in lens]
    if not chunks or max(chunks) <= 1:
        return [1] * len(lens)
    best = None
    for seg_len in sorted({math.ceil(max(chunks) / m) for m in range(1, max_segments + 1)}, reverse=True):
        counts = [max(1, min(max_segments, math.ceil(c / seg_len))) if c else 1 for c in chunks]
        walks = []
        for c, m in zip(chunks, counts):
            for s in split_chunks(c, m) if c else [0]:
                walks += [s + walk_overhead] * nh
        corrected = max((c - split_chunks(c, m)[0] for c, m in zip(chunks, counts) if c), default=0)
        cost = _makespan(walks, n_sm) + (corrected * join_per_chunk + join_fixed if any(m > 1 for m in counts) else 0.0)
        if best is None or cost < best[0] - 1e-9:
            best = (cost, counts)
    return best[1]


@dataclass
class SsdSegments:
    """A cut of the packed sequences into segments, as the device arrays mmp_ssd_prefill_seg reads, with the fp32
    scratch state lines of the segments."""
    counts: list[int]
    nvirt: int
    vcu: torch.Tensor      # [nvirt + 1] int32: token offsets of the segments (packed rows)
    vline: torch.Tensor    # [nvirt] int32: scratch line of each segment (its index)
    vinit: torch.Tensor    # [nvirt] int32: the segment starts from its scratch line (first segments of sequences
    #                        that continue from a state)
    seg0: torch.Tensor     # [nseq + 1] int32: sequence i owns segments [seg0[i], seg0[i + 1])
    scratch: torch.Tensor  # [nvirt, nh, p, N] fp32


def segment_bounds(lens: list[int], counts: list[int]) -> list[int]:
    """Token offsets (packed rows) of every segment boundary, cuts on chunk boundaries of each sequence."""
    vcu, base = [0], 0
    for L, m in zip(lens, counts):
        c = math.ceil(L / CHUNK)
        t = base
        for s in (split_chunks(c, m) if c else [0]):
            t = min(base + L, t + s * CHUNK)
            vcu.append(t)
        if m > 1 and vcu[-1] != base + L:
            raise AssertionError("segments must cover the sequence")
        base += L
    return vcu


def build_segments(lens: list[int], has_init: list[int], nh: int, p: int, N: int, device: torch.device,
                   n_sm: int | None = None, counts: list[int] | None = None) -> SsdSegments | None:
    """The plan for one prefill shape, or None when no sequence is worth cutting (or the head dim is not the
    join's 128): the plain scan then runs."""
    if p != 128 or N not in (64, 128, 256) or not lens:
        return None
    if counts is None:
        if n_sm is None:  # the device's SMs (a B200's 148 when planning off the GPU)
            n_sm = torch.cuda.get_device_properties(device).multi_processor_count if device.type == "cuda" else 148
        counts = plan_counts(lens, nh, n_sm)
    if len(counts) != len(lens) or all(m == 1 for m in counts):
        return None
    vcu = segment_bounds(lens, counts)
    nvirt = len(vcu) - 1
    seg0, vinit = [0], []
    for i, m in enumerate(counts):
        seg0.append(seg0[-1] + m)
        vinit += [int(has_init[i])] + [0] * (m - 1)
    i32 = lambda v: torch.tensor(v, dtype=torch.int32, device=device)  # noqa: E731
    return SsdSegments(counts=list(counts), nvirt=nvirt, vcu=i32(vcu), vline=i32(list(range(nvirt))), vinit=i32(vinit),
                       seg0=i32(seg0), scratch=torch.empty(nvirt, nh, p, N, dtype=torch.float32, device=device))
