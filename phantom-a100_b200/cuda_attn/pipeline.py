"""Attention over host-resident tensors: the GPU work is pipelined with the host link.

    o = cuda_attn.fused_tc_host(q, k, v)      # q, k, v: (B, H, N, d) pinned CPU tensors -> O on the host

Heads are independent, so the B*H heads are cut into chunks and streamed through three device slots on
three CUDA streams: while chunk i is attended on the compute stream, chunk i+1 is copied host->device and
chunk i-1 device->host. The host link (~55 GB/s per direction; ~50 for input copies while an output copy
and the kernel run) rather than the kernel then bounds the call,
and the two directions overlap each other. Three slots let the copy of chunk i+2 start while chunk i's
output is still in flight (the output copy shares the link with the input copies). The last full chunk is
cut into halves down to two heads (... per, per/2, ..., 2, 2), so that the work left after the last input
copy, the last chunk's attention and output copy, is small; back-to-back calls also overlap it with the
next call's first input copies (measured on config 4: 8.48 -> 8.13 ms per call). Chunks are also kept
large in bytes: a full chunk copies at least MIN_CHUNK_BYTES of each input tensor and the halving stops
at MIN_TAIL_BYTES, because small copies run far below the link rate (config 2's 2 MiB and 256 KiB copies
ran at ~30 GB/s: 1.59 ms per call in 11 chunks, 1.30-1.38 ms in two; config 3 8.41 -> 8.10 ms; config 4,
whose chunks were already 16 MiB, unchanged). Each chunk runs the same C-ABI entry point as
fused_tc, with the tail's K/V parts turned off (phantom_attn_set_kv_parts(0) on this thread for the
duration of the call): the call is bound by the host link, not by the kernel's last wave, and every query
block then runs over its whole K/V range, so the result equals a device-resident fused_tc call without
K/V parts bit for bit, however the heads are chunked.
"""
from __future__ import annotations

import math
import threading

import torch

from .capi import CAPI

_LOCAL = threading.local()
_PENDING_MAX = 8  # outputs of earlier calls on this thread whose copies may still be in flight


def _pending() -> list:
    p = getattr(_LOCAL, "pending", None)
    if p is None:
        p = _LOCAL.pending = []
    return p


def _span(t: torch.Tensor) -> tuple[int, int]:
    return t.data_ptr(), t.data_ptr() + t.numel() * t.element_size()


def _lib() -> CAPI:
    lib = getattr(_LOCAL, "lib", None)
    if lib is None:
        lib = _LOCAL.lib = CAPI()
    return lib


def _streams(device: torch.device):
    key = ("streams", device.index)
    s = getattr(_LOCAL, "streams", {})
    if key not in s:
        s[key] = tuple(torch.cuda.Stream(device=device) for _ in range(3))
        _LOCAL.streams = s
    return s[key]


MIN_TAIL_HEADS = 2  # a one-head chunk's three 4 MiB input copies ran at ~35 GB/s (config 4), two heads' at ~47
MIN_CHUNK_BYTES = 32 << 20  # per input tensor, full chunks
MIN_TAIL_BYTES = 8 << 20  # per input tensor, the halved tail chunks


def chunk_plan(bh: int, chunks: int, head_bytes: int = 0, min_chunk_bytes: int = 0,
               min_tail_bytes: int = 0) -> list[int]:
    """Head counts of the chunks: full chunks of ceil(bh / chunks) heads, then the last one cut into
    halves down to chunks of MIN_TAIL_HEADS (4 -> 2, 2; 8 -> 4, 2, 2), so the tail after the last input
    copy is small. With head_bytes (one head of one input tensor) given, a full chunk also holds at least
    min_chunk_bytes and the halving stops at min_tail_bytes per input tensor. chunks <= 1: one chunk of all
    heads (no pipelining)."""
    if chunks <= 1:
        return [bh]
    per = max(1, math.ceil(bh / chunks))
    tail_min = MIN_TAIL_HEADS
    if head_bytes > 0:
        per = max(per, math.ceil(min_chunk_bytes / head_bytes))
        tail_min = max(tail_min, math.ceil(min_tail_bytes / head_bytes))
    sizes = []
    left = bh
    while left > per:
        sizes.append(per)
        left -= per
    while left >= 2 * tail_min:
        half = left // 2
        sizes.append(left - half)
        left = half
    if left:
        sizes.append(left)
    return sizes


def fused_tc_host(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
                  out: torch.Tensor | None = None, chunks: int = 8, device: int | torch.device | None = None,
                  synchronize: bool = True, trace: list | None = None, min_chunk_bytes: int = MIN_CHUNK_BYTES,
                  min_tail_bytes: int = MIN_TAIL_BYTES) -> torch.Tensor:
    """fused_tc for (B, H, N, d) CPU tensors (pin them for overlap; pageable memory works but serialises
    the copies). Returns O as a CPU tensor of the input dtype (`out` if given, pinned otherwise). With
    synchronize=False the call returns once the work is queued; the current CUDA stream of `device` is
    ordered after the last copy, so synchronising it (or an event recorded on it) makes O valid.

    Ordering: the input copies start at once, so that back-to-back calls overlap (the next call's first
    input copies run during this call's last kernel and output copy). The host inputs must therefore hold
    their values when the call is made; the one exception it tracks is an output of an earlier call on
    this thread that is still being copied back, which the input copies wait for (chained calls, e.g.
    one call's O as the next call's Q). The output copies wait for the current stream, so GPU work queued
    on it before the call that still reads `out` is not overwritten.

    chunks: full chunks at most (heads are cut into ceil(B*H / chunks)-head chunks, each also holding at
    least min_chunk_bytes of each input tensor; the last is halved down to min_tail_bytes; pass 0 for both
    to chunk by head count alone).

    trace: if a list is given, one record per chunk is appended - {"heads", "h2d", "attend", "d2h"}, each
    a (start, end) pair of CUDA events (timing-enabled) on that stage's stream (cuda_attn.timeline)."""
    for t in (q, k, v):
        if t.is_cuda:
            raise RuntimeError("fused_tc_host: inputs must be CPU tensors (use fused_tc for device tensors)")
        if not t.is_contiguous():
            raise RuntimeError("fused_tc_host: inputs must be contiguous")
        if t.dim() != 4:
            raise RuntimeError("fused_tc_host: inputs must be shaped (B, H, N, d)")
        if t.dtype != q.dtype:
            raise RuntimeError("fused_tc_host: q, k, v must share a dtype")
    if q.shape != k.shape or q.shape != v.shape:
        raise RuntimeError("fused_tc_host: q, k, v must have the same shape")
    B, H, N, d = q.shape
    BH = B * H
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else torch.device(device).index or 0)
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    hq, hk, hv, ho = (x.view(BH, N, d) for x in (q, k, v, out))
    sizes = chunk_plan(BH, chunks, N * d * q.element_size(), min_chunk_bytes, min_tail_bytes)
    per = sizes[0]
    n_slots = min(3, len(sizes))
    lib = _lib()
    kv_parts = lib.get_kv_parts()
    lib.set_kv_parts(False)
    try:
        return _pipeline(lib, hq, hk, hv, ho, out, sizes, per, n_slots, N, d, q.dtype, causal, dev, synchronize,
                         trace)
    finally:
        lib.set_kv_parts(kv_parts)


def _pipeline(lib, hq, hk, hv, ho, out, sizes, per, n_slots, N, d, dtype, causal, dev, synchronize, trace=None):
    def mark(stream):
        if trace is None:
            return None
        e = torch.cuda.Event(enable_timing=True)
        e.record(stream)
        return e

    with torch.cuda.device(dev):
        h2d, comp, d2h = _streams(dev)
        cur = torch.cuda.current_stream(dev)
        slots = [[torch.empty((per, N, d), dtype=dtype, device=dev) for _ in range(4)] for _ in range(n_slots)]
        loaded = [torch.cuda.Event() for _ in range(n_slots)]
        computed = [torch.cuda.Event() for _ in range(n_slots)]
        freed = [torch.cuda.Event() for _ in range(n_slots)]
        pending = _pending()
        pending[:] = [(lo, hi, ev) for lo, hi, ev in pending if not ev.query()]
        for x in (hq, hk, hv):  # an input that an earlier call is still writing back
            lo, hi = _span(x)
            for plo, phi, ev in pending:
                if lo < phi and plo < hi:
                    h2d.wait_event(ev)
        d2h.wait_stream(cur)  # work queued on the caller's stream before this call may still read `out`
        b = 0
        for i, n in enumerate(sizes):
            s = i % n_slots
            a, b = b, b + n
            dq, dk, dv, do = (x[:n] for x in slots[s])
            if i >= n_slots:
                h2d.wait_event(freed[s])
            with torch.cuda.stream(h2d):
                t0 = mark(h2d)
                dq.copy_(hq[a:b], non_blocking=True)
                dk.copy_(hk[a:b], non_blocking=True)
                dv.copy_(hv[a:b], non_blocking=True)
                t1 = mark(h2d)
                loaded[s].record(h2d)
            comp.wait_event(loaded[s])
            t2 = mark(comp)
            lib.fused_tc(dq.unsqueeze(0), dk.unsqueeze(0), dv.unsqueeze(0), do.unsqueeze(0), causal=causal,
                         stream=comp)
            t3 = mark(comp)
            computed[s].record(comp)
            d2h.wait_event(computed[s])
            with torch.cuda.stream(d2h):
                t4 = mark(d2h)
                ho[a:b].copy_(do, non_blocking=True)
                t5 = mark(d2h)
                freed[s].record(d2h)
            if trace is not None:
                trace.append({"heads": n, "h2d": (t0, t1), "attend": (t2, t3), "d2h": (t4, t5)})
        cur.wait_stream(d2h)
        done = torch.cuda.Event()
        done.record(d2h)
        pending.append((*_span(ho), done))
        del pending[:-_PENDING_MAX]
        for t in (x for slot in slots for x in slot):
            t.record_stream(h2d)
            t.record_stream(comp)
            t.record_stream(d2h)
        if synchronize:
            cur.synchronize()
    return out
