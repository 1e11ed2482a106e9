"""Device timing of short launches with cold weights.

A decode GEMM runs for a few microseconds, shorter than the resolution of
CUDA events around one graph replay, and its weights must come from HBM, not
from the 126 MB L2 where the previous call left them.  rotating_graph_us
captures many calls back to back in one CUDA graph, each reading the next
of `copies` separate weight copies whose total size is well above L2, so
every call streams weights that the L2 has since evicted; the graph's event
time divided by the number of calls is the per-call device time, with no
host launch gaps and no flush in the timed region.
"""

import math

import torch

L2_BYTES = 126 << 20


def copies_for(weight_bytes: int, factor: float = 2.5) -> int:
    """Weight copies so that one pass over them is about factor x L2."""
    return max(2, math.ceil(factor * L2_BYTES / max(1, weight_bytes)))


def rotating_graph_stats(call, copies: int, calls: int = 64, replays: int = 7, warm_replays: int = 2) -> dict:
    """Per-call device microseconds of one graph of `calls` calls (cycling
    i over range(copies)), replayed `replays` times: median and
    interquartile range over the replays."""
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for i in range(copies):
            call(i)  # first launches outside capture (per-device setup)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for j in range(calls):
                call(j % copies)
    torch.cuda.current_stream().wait_stream(stream)
    for _ in range(warm_replays):
        graph.replay()
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(replays)]
    for start, end in events:
        start.record()
        graph.replay()
        end.record()
    torch.cuda.synchronize()
    us = sorted(s.elapsed_time(e) * 1e3 / calls for s, e in events)
    del graph

    def quantile(q):
        x = q * (len(us) - 1)
        lo = int(math.floor(x))
        hi = min(lo + 1, len(us) - 1)
        return us[lo] + (us[hi] - us[lo]) * (x - lo)

    return {"median": quantile(0.5), "q1": quantile(0.25), "q3": quantile(0.75), "replays": replays}


def rotating_graph_us(call, copies: int, calls: int = 64, warm_replays: int = 2) -> float:
    """Mean device microseconds per call(i) over one graph of `calls` calls,
    cycling i over range(copies)."""
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for i in range(copies):
            call(i)  # first launches outside capture (per-device setup)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for j in range(calls):
                call(j % copies)
    torch.cuda.current_stream().wait_stream(stream)
    for _ in range(warm_replays):
        graph.replay()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    graph.replay()
    end.record()
    torch.cuda.synchronize()
    us = start.elapsed_time(end) * 1e3 / calls
    del graph
    return us
