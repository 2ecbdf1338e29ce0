"""Attention over host-resident tensors with copies and compute overlapped.

``flash_attn_fwd_host(q, k, v, causal, sm_scale)`` takes q/k/v [B, H, S, D] in
(pinned) host memory and returns o in pinned host memory. The (batch, head)
slices are independent, so the call splits them into chunks and runs three
CUDA streams: host->device copies of chunk c+1 and device->host copies of
chunk c-1 proceed while the tensor-core kernel works on chunk c. The two copy
directions use separate copy engines, so a call costs about the host->device
transfer of q, k and v plus one chunk's kernel and read-back, instead of the
sum of all three phases.

This is the path a caller whose tensors live in host memory uses (the
reference hands host buffers to its kernels the same way, driver.py:692+);
``flash_attn_fwd`` remains the device-tensor entry point.
"""
from __future__ import annotations

import math
import threading
from typing import Dict, Optional, Tuple

import torch

from . import ops

# Three side streams per (host thread, device): a thread's calls are ordered on
# its own streams, and two threads never share (and so never interleave) them.
_STREAMS: Dict[Tuple[int, int], Tuple[torch.cuda.Stream, torch.cuda.Stream, torch.cuda.Stream]] = {}
_STREAMS_LOCK = threading.Lock()


def _streams(dev: torch.device):
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    key = (threading.get_ident(), idx)
    with _STREAMS_LOCK:
        s = _STREAMS.get(key)
        if s is None:
            with torch.cuda.device(idx):
                s = (torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream())
            _STREAMS[key] = s
    return s


class _Slot:
    """Device staging for one call: q, k, v and o back to back, reused by later
    calls once the event recorded after the call's last read-back has passed."""

    def __init__(self):
        self.buf: Optional[torch.Tensor] = None
        self.done: Optional[torch.cuda.Event] = None


# Two staging slots per (host thread, device), used in turn, so a call's
# host->device copies can start while the previous call's read-back drains.
_STAGING: Dict[Tuple[int, int], list] = {}


def _slot(dev: torch.device, nbytes: int) -> _Slot:
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    key = (threading.get_ident(), idx)
    with _STREAMS_LOCK:
        st = _STAGING.get(key)
        if st is None:
            st = _STAGING[key] = [0, _Slot(), _Slot()]
    st[0] ^= 1
    slot = st[1 + st[0]]
    if slot.buf is None or slot.buf.numel() < nbytes:
        if slot.done is not None:
            slot.done.synchronize()  # the old buffer's last reader has finished
        slot.buf = None
        slot.buf = torch.empty((nbytes,), dtype=torch.uint8, device=dev)
    return slot


def release_staging() -> None:
    """Drop this thread's device staging buffers (they are kept between calls)."""
    me = threading.get_ident()
    with _STREAMS_LOCK:
        for key in [k for k in _STAGING if k[0] == me]:
            for slot in _STAGING[key][1:]:
                if slot.done is not None:
                    slot.done.synchronize()
            del _STAGING[key]


# Default chunk shares, largest first. When a call's uploads wait for the
# previous call's read-back, a call costs the upload of all inputs plus the
# kernel and read-back of what arrives last, so the last chunk is small; each
# further chunk adds per-copy cost. When they overlap (host_inputs_ready), the
# read-back hides behind the next call's uploads and fewer copies win.
# Measured on one B200 for [4, 16, 2048, 128] fp16 causal, ms per call back to
# back: waiting 10/5/1 2.13, four equal chunks 2.24, eight 2.38, 11/4/1 2.15,
# 9/5/2 2.15; overlapping 2/1 1.98, one chunk 1.99, 1/2 1.98, two equal 2.01,
# 10/5/1 2.06, four equal 2.10.
_DEFAULT_SHARES = (10, 5, 1)
_DEFAULT_SHARES_READY = (2, 1)


def _chunk_bounds(BH: int, chunks: Optional[int], ready: bool = False) -> list:
    """Start offsets of each (batch, head) chunk plus BH at the end, no empty chunk."""
    if chunks is None:
        shares = _DEFAULT_SHARES_READY if ready else _DEFAULT_SHARES
        tot = sum(shares)
        cum, b = 0, [0]
        for sh in shares:
            cum += sh
            b.append((BH * cum + tot - 1) // tot)
    else:
        n = max(1, min(int(chunks), BH))
        b = [(BH * c) // n for c in range(n + 1)]
    out = [0]
    for x in b[1:]:
        if x > out[-1]:
            out.append(x)
    return out


def flash_attn_fwd_host(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
                        sm_scale: Optional[float] = None, out: Optional[torch.Tensor] = None,
                        chunks: Optional[int] = None, device: Optional[torch.device] = None,
                        host_inputs_ready: bool = False) -> torch.Tensor:
    """o = softmax(sm_scale * q @ k^T [causal]) @ v for host tensors [B, H, S, D].

    q, k, v: CPU tensors of one shape and dtype, contiguous (pinned memory makes
    the copies asynchronous; pageable memory works but serialises them).
    out: optional contiguous CPU tensor like q (pinned), else one is allocated.
    chunks: number of equal (batch, head) groups pipelined through the GPU; by
    default 10/16, 5/16 and 1/16 of the slices, or 2/3 and 1/3 with
    host_inputs_ready (see ``_chunk_bounds``).
    host_inputs_ready: by default the uploads wait for all work already queued
    on the caller's current stream, which includes the previous call's
    read-back, so back-to-back calls run one after another. True declares that
    no GPU work still queued on that stream writes q, k or v (the usual case
    for inputs the CPU prepared); the uploads then wait only for this thread's
    staging slot, and a call's uploads overlap the previous call's read-back.
    The output's ordering is the same either way.
    The returned tensor is complete when the current CUDA stream of `device`
    reaches this point (synchronise it, or an event recorded on it, before
    reading).
    """
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.is_cuda:
            raise ValueError(f"flash_attn_fwd_host: {name} must be a host tensor "
                             "(use flash_attn_fwd for device tensors)")
        if not t.is_contiguous():
            raise ValueError(f"flash_attn_fwd_host: {name} must be contiguous")
    if q.dim() != 4 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError("flash_attn_fwd_host: q, k, v must all be [B, H, S, D] of one shape")
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError("flash_attn_fwd_host: q, k, v must share a dtype")
    B, H, S, D = q.shape
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    elif out.shape != q.shape or out.dtype != q.dtype or out.is_cuda or not out.is_contiguous():
        raise ValueError("flash_attn_fwd_host: out must be a contiguous host tensor like q")
    BH = B * H
    if BH == 0 or S == 0:
        return out
    qf, kf, vf, of = (t.view(BH, S, D) for t in (q, k, v, out))
    s_in, s_comp, s_out = _streams(dev)
    cur = torch.cuda.current_stream(dev)
    bounds = _chunk_bounds(BH, chunks, host_inputs_ready)
    n = len(bounds) - 1
    elems = BH * S * D
    with torch.cuda.device(dev):
        slot = _slot(dev, 4 * elems * q.element_size())
        dq, dk, dv, do = slot.buf[:4 * elems * q.element_size()].view(q.dtype).view(4, BH, S, D).unbind(0)
        # the copies may not start before earlier work on the caller's stream
        # (unless the caller declares the inputs ready), nor overwrite the slot
        # before its previous call's last read-back
        if not host_inputs_ready:
            s_in.wait_stream(cur)
        s_out.wait_stream(cur)
        if slot.done is not None:
            s_in.wait_event(slot.done)
        # All host->device copies are queued first, so the copy engine never waits
        # for the host to issue the next chunk's copies.
        ev_in = []
        with torch.cuda.stream(s_in):
            for c in range(n):
                h0, h1 = bounds[c], bounds[c + 1]
                for dst, src in ((dq, qf), (dk, kf), (dv, vf)):
                    dst[h0:h1].copy_(src[h0:h1], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(s_in)
                ev_in.append(ev)
        comp_handle = s_comp.cuda_stream
        for c in range(n):
            h0, h1 = bounds[c], bounds[c + 1]
            if h1 == h0:
                continue
            s_comp.wait_event(ev_in[c])
            ops._fa_into(dq[h0:h1].unsqueeze(0), dk[h0:h1].unsqueeze(0), dv[h0:h1].unsqueeze(0),
                         do[h0:h1].unsqueeze(0), causal, sm_scale, comp_handle)
            ev_c = torch.cuda.Event()
            ev_c.record(s_comp)
            s_out.wait_event(ev_c)
            with torch.cuda.stream(s_out):
                of[h0:h1].copy_(do[h0:h1], non_blocking=True)
        last = torch.cuda.Event()
        last.record(s_out)
        slot.done = last
        cur.wait_event(last)
    return out
