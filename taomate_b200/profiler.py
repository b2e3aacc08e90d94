"""Per-section CUDA-event timing for the streaming attention path.

The counterpart of the reference's ``_BlockProfiler``
(ltx_causal/transformer/kv_cache.py:160-315): sections are bracketed by CUDA
events on the current stream with no host synchronisation; ``summary()``
synchronises once and aggregates milliseconds per section name.  Section
names follow the reference's (``<profile_base>.rope_reshape``, ``.sdpa``,
``.a2a_seq2head``, ``.a2a_head2seq``, ``.cache_append``, ``.qkv_proj_norm``,
``.out_proj``; here ``qkv_proj_norm`` covers the projection GEMMs only, the
q/k norms being fused into ``rope_reshape``).  Disabled (the default) it costs
one attribute check per section.

A section opened while a CUDA graph is being captured records *external*
events, which become event-record nodes of the graph: every replay then
re-records them, and ``summary()`` reports the sections of the latest replay.
"""

from __future__ import annotations

import contextlib
from collections import defaultdict
from typing import Dict, List, Optional, Tuple

import torch


class SectionTimer:
    def __init__(self):
        self.enabled = False
        self._events: List[Tuple[str, torch.cuda.Event, torch.cuda.Event]] = []

    def start(self) -> None:
        self._events.clear()
        self.enabled = True

    def stop(self) -> None:
        self.enabled = False

    @contextlib.contextmanager
    def section(self, name: str):
        if not self.enabled:
            yield
            return
        ext = torch.cuda.is_current_stream_capturing()
        s = torch.cuda.Event(enable_timing=True, external=ext)
        e = torch.cuda.Event(enable_timing=True, external=ext)
        s.record()
        try:
            yield
        finally:
            e.record()
            self._events.append((name, s, e))

    def summary(self) -> Dict[str, Dict[str, float]]:
        """``{name: {"count": n, "total_ms": t, "mean_ms": t / n}}``."""
        if self._events:
            self._events[-1][2].synchronize()
        acc: Dict[str, List[float]] = defaultdict(list)
        for name, s, e in self._events:
            acc[name].append(s.elapsed_time(e))
        return {k: {"count": len(v), "total_ms": sum(v), "mean_ms": sum(v) / len(v)}
                for k, v in acc.items()}


TIMER = SectionTimer()


def section(name: Optional[str]):
    if name is None or not TIMER.enabled:
        return contextlib.nullcontext()
    return TIMER.section(name)
