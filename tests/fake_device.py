"""A deterministic fake device API for timing-policy tests (no GPU, no torch.cuda).

The device clock advances only when submitted work executes: a direct
launch adds `kernel_ms`; a captured graph adds launches x kernel_ms per
replay.  Events record the clock; elapsed_time optionally quantizes to an
event resolution, which exercises the calibration and restart paths of the
timing policy.  The same fake drives both the reference suite's measure()
(when generating golden fixtures) and this package's runtime.measure().
"""

from __future__ import annotations

from contextlib import contextmanager
import math
from types import SimpleNamespace


class FakeDeviceAPI:
    def __init__(self, kernel_ms=0.25, event_resolution_ms=None, with_graph=True,
                 graph_kernel_ms=None):
        self.kernel_ms = kernel_ms
        self.graph_kernel_ms = graph_kernel_ms
        self.event_resolution_ms = event_resolution_ms
        self.now_ms = 0.0
        self.synchronized_ms = 0.0
        self.capturing = None
        self.replays = 0
        self.launches = 0
        if with_graph:
            api = self

            class CUDAGraph:
                def __init__(self):
                    self.count = 0

                def replay(self):
                    api.replays += 1
                    per = api.kernel_ms if api.graph_kernel_ms is None else api.graph_kernel_ms
                    api.now_ms += self.count * per

            self.CUDAGraph = CUDAGraph

    # -- device API surface used by the timing policy
    def synchronize(self, *args):
        self.synchronized_ms = self.now_ms

    def Event(self, enable_timing=False):
        if not enable_timing:
            raise AssertionError("timing events must be requested with enable_timing=True")
        api = self

        class Event:
            timestamp_ms = None

            def record(self, stream=None):
                self.timestamp_ms = api.now_ms

            def elapsed_time(self, end):
                if api.synchronized_ms < end.timestamp_ms:
                    raise AssertionError("elapsed time read before completion")
                elapsed = end.timestamp_ms - self.timestamp_ms
                if api.event_resolution_ms:
                    return math.floor(elapsed / api.event_resolution_ms) * api.event_resolution_ms
                return elapsed

        return Event()

    def Stream(self, *args, **kwargs):
        return SimpleNamespace()

    @contextmanager
    def stream(self, stream):
        yield stream

    @contextmanager
    def graph(self, graph, *args, **kwargs):
        if self.capturing is not None:
            raise AssertionError("nested capture")
        self.capturing = graph
        try:
            yield graph
        finally:
            self.capturing = None

    # -- the "kernel"
    def launch(self):
        self.launches += 1
        if self.capturing is not None:
            self.capturing.count += 1
        else:
            self.now_ms += self.kernel_ms


SCENARIOS = {
    "graph_default": dict(api=dict(kernel_ms=0.25), args=dict(timing="auto")),
    "graph_short_kernel": dict(api=dict(kernel_ms=0.003), args=dict(timing="auto")),
    "graph_long_kernel": dict(api=dict(kernel_ms=7.0), args=dict(timing="auto", rep=100.0)),
    "events_requested": dict(api=dict(kernel_ms=0.05), args=dict(timing="events")),
    "auto_fallback_no_graph": dict(api=dict(kernel_ms=0.1, with_graph=False),
                                   args=dict(timing="auto")),
    "coarse_timer": dict(api=dict(kernel_ms=0.004, event_resolution_ms=0.5),
                         args=dict(timing="auto")),
    "coarse_timer_resolved": dict(api=dict(kernel_ms=0.01, event_resolution_ms=0.1),
                                  args=dict(timing="auto")),
    "coarse_timer_events": dict(api=dict(kernel_ms=0.02, event_resolution_ms=0.25),
                                args=dict(timing="events", batch_ms=2.0, rounds=4)),
    "graph_faster_replay": dict(api=dict(kernel_ms=0.2, graph_kernel_ms=0.15),
                                args=dict(timing="graph", warmup=20.0, rep=50.0)),
}


def make_args(**overrides):
    base = dict(timing="auto", warmup=100.0, rep=200.0, batch_ms=10.0, rounds=10)
    base.update(overrides)
    return SimpleNamespace(**base)
