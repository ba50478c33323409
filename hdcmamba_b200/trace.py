"""Device-side tracing of a forward's launch sequence.

``trace(fn, device)`` wraps the layer's entry points -- the ``hdcmamba_b200.ops``
functions, torch's ``F.linear`` / ``torch.addmm`` (the cuBLAS projections) and the
peer-mailbox exchange -- with ``hdc_trace_stamp`` launches on the calling stream,
captures one call of ``fn`` in a CUDA graph, replays it and returns:

* ``ops``: per op name, the mean device time between its two stamps (stream order, so it
  includes the op's own queueing behind earlier work of that stream) and its count per
  replay;
* ``gaps``: per pair of consecutive ops on the capturing stream, the mean time from the end
  stamp of the first to the start stamp of the second (waits for other streams or ranks,
  launch gaps);
* ``total_us``: first to last stamp of the capturing stream;
* ``sequence``: the first stamps of the last replay in time order, each with its stream
  (how the side stream's ops overlap the main stream's).

The stamps add one one-thread kernel per boundary, so the figures attribute time between
ops; the benchmark figures come from untraced runs.
"""
import collections
import ctypes

import torch
import torch.nn.functional as F

from . import _lib, ops

OPS = ("ln_conv", "ssm_scan", "slot_scan_gate", "row_layernorm", "ssm_chunk_stats", "slot_state",
       "ssm_scan_out_blocked", "slot_scan_gate_carry", "layer_norm")


class _Stamps:
    def __init__(self, device, capacity=1 << 16):
        self.device = device
        self.buf = torch.zeros(capacity, dtype=torch.int64, device=device)
        self.labels = []  # (label, stream handle)

    def __call__(self, label):
        if len(self.labels) >= self.buf.numel():
            raise RuntimeError("trace: stamp buffer full")
        s = torch.cuda.current_stream(self.device).cuda_stream
        _lib.call("hdc_trace_stamp", ctypes.c_void_p(self.buf.data_ptr()), len(self.labels), ctypes.c_void_p(s))
        self.labels.append((label, s))


def _patch(stamps):
    """Wrap the entry points; returns the list of (owner, name, original) to restore."""
    saved = []

    def wrap(owner, name, label):
        fn = getattr(owner, name)

        def traced(*a, **k):
            stamps(label + ">")
            r = fn(*a, **k)
            stamps(label + "<")
            return r
        saved.append((owner, name, fn))
        setattr(owner, name, traced)

    for n in OPS:
        wrap(ops, n, n)
    wrap(F, "linear", "linear")
    wrap(torch, "addmm", "addmm")
    try:
        from .peer import PeerMailbox
        for n in ("put", "wait", "barrier", "next_generation"):
            wrap(PeerMailbox, n, "peer_" + n)
    except ImportError:
        pass
    return saved


def trace(fn, device, replays=5, before_replay=None, sequence_len=64):
    """Capture ``fn()`` with stamps in a CUDA graph (``fn`` must be capturable and already
    warmed up), replay it ``replays`` times (``before_replay()`` runs before each, e.g. a
    barrier across ranks) and summarise the stamps; ``sequence`` lists the first
    ``sequence_len`` stamps of the last replay in time order with their stream."""
    stamps = _Stamps(device)
    g = torch.cuda.CUDAGraph()
    saved = _patch(stamps)
    try:
        with torch.cuda.graph(g):
            main = torch.cuda.current_stream(device).cuda_stream
            stamps("begin")
            fn()
            stamps("end")
    finally:
        for owner, name, orig in reversed(saved):
            setattr(owner, name, orig)
    durations = collections.defaultdict(list)
    gaps = collections.defaultdict(list)
    totals = []
    n = len(stamps.labels)
    sequence = []
    for _ in range(replays):
        if before_replay is not None:
            before_replay()
        torch.cuda.synchronize(device)
        g.replay()
        torch.cuda.synchronize(device)
        t = stamps.buf[:n].cpu().tolist()
        stacks = collections.defaultdict(list)
        prev = None
        for (label, s), ti in zip(stamps.labels, t):
            if label.endswith(">"):
                stacks[s].append((label[:-1], ti))
            elif label.endswith("<"):
                name, t0 = stacks[s].pop()
                durations[name].append((ti - t0) / 1e3)
            if s == main:
                if prev is not None and prev[0].endswith("<") and label.endswith(">"):
                    gaps[f"{prev[0][:-1]} -> {label[:-1]}"].append((ti - prev[1]) / 1e3)
                prev = (label, ti)
        main_t = [ti for (label, s), ti in zip(stamps.labels, t) if s == main]
        totals.append((main_t[-1] - main_t[0]) / 1e3)
        # the last replay's stamps in time order (us from the first), main / side stream
        sequence = sorted(((ti - main_t[0]) / 1e3, label, "main" if s == main else "side")
                          for (label, s), ti in zip(stamps.labels, t))
    del g
    return {
        "total_us": sum(totals) / len(totals),
        "ops": {k: {"us": round(sum(v) / len(v), 2), "per_replay": len(v) // replays} for k, v in durations.items()},
        "gaps": {k: {"us": round(sum(v) / len(v), 2), "per_replay": len(v) // replays} for k, v in gaps.items()},
        "sequence": [(round(t, 2), label, stream) for t, label, stream in sequence[:sequence_len]],
    }
