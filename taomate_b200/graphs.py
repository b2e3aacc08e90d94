"""CUDA-graph replay of a streaming forward (the host-side executor).

A forward of the streaming model is a fixed sequence of launches per layer
(projection GEMMs, the fused norm+RoPE, the Ulysses exchanges, attention), but
issuing it from Python costs ~0.2-0.3 ms of host time per attention call,
more than the GPU work per call once the heads are split over several GPUs.
``AttentionGraph`` captures one forward into a CUDA graph (NCCL exchanges
included) and replays it.

What changes between the streaming blocks is where the cache rows sit in the
slot arena: every attention call of a captured forward therefore reads its key
tiles from one device table instead of its launch parameters, and
``replay(site_spans)`` rewrites that table from the new cache layout before the
replay (a small kernel reads the pinned staging buffer).  A block may replay the graph as long
as every attention call keeps the tile count it was captured with (the window
is full); anything else must recapture.  Inputs and outputs of a replay are the
tensors the captured forward read and returned (the graph's own memory).

Reference counterpart: none (the reference issues every forward eagerly from
Python, ltx_causal/transformer/kv_cache.py:2681-3365); the graph replays the
same calls.
"""

from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence, Tuple

import torch

from . import _lib

MAX_TILES = 384   # the kernel's key-tile capacity (24576 keys of 64)
_SITE_ALIGN = 2   # tiles; keeps every site's table 16-byte aligned

_RECORDER: Optional["AttentionGraph"] = None


def recorder() -> Optional["AttentionGraph"]:
    """The graph being captured on this process, if any."""
    return _RECORDER


class _Site:
    __slots__ = ("offset", "n_tiles", "cache_rows", "new_rows", "key")

    def __init__(self, offset, n_tiles, cache_rows, new_rows, key=None):
        self.offset, self.n_tiles = offset, n_tiles
        self.cache_rows, self.new_rows = cache_rows, new_rows
        self.key = key


class AttentionGraph:
    """Capture and replay one forward.

    ``capture(fn, *args)`` runs ``fn`` under ``torch.cuda.graph`` (run it once
    eagerly first, as for any captured torch code, so cuBLAS and NCCL are
    initialised); every ``flash_attention`` call inside becomes a *site* whose
    key-tile list lives in the device table.  ``replay(site_spans)`` takes, per
    site in call order, the span list ``[(source, row_start, rows), ...]`` of
    the new cache layout (``attention_spans`` builds it), or ``None`` to keep
    the current one.
    """

    def __init__(self, device: torch.device, max_sites: int = 512):
        self.device = torch.device(device)
        n = max_sites * MAX_TILES * 2
        self.table = torch.zeros(n, dtype=torch.int32, device=self.device)
        # two pinned staging buffers: one may still be in flight to the table
        self._stage = [torch.zeros(n, dtype=torch.int32).pin_memory() for _ in range(2)]
        self._events: List[Optional[torch.cuda.Event]] = [None, None]
        self._cur = 0
        self._dirty = False
        self.max_sites = max_sites
        self.sites: List[_Site] = []
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.launches = 0
        self._used = 0  # int32 entries of the table in use

    # -- capture -----------------------------------------------------------
    def capture(self, fn, *args, **kwargs):
        global _RECORDER
        if _RECORDER is not None:
            raise RuntimeError("another AttentionGraph is capturing")
        self.sites = []
        self._used = 0
        self.graph = torch.cuda.CUDAGraph()
        l0 = _lib.LAUNCHES
        _RECORDER = self
        try:
            with torch.cuda.graph(self.graph):
                out = fn(*args, **kwargs)
        finally:
            _RECORDER = None
        self.launches = _lib.LAUNCHES - l0
        self._dirty = True  # the capture-time tile lists are staged, not yet copied
        return out

    def _add_site(self, spans, n_spans: int, cache_rows: int, new_rows: int,
                  key: Optional[int] = None) -> int:
        """Called by flash_attention while capturing: stage this call's tile
        list and return the device address its kernel reads.  ``key`` names
        the site for ``replay`` (the cache source's base address)."""
        if len(self.sites) >= self.max_sites:
            raise RuntimeError(f"more than {self.max_sites} attention calls in one graph")
        offset = self._used
        n = self._write_tiles(self._stage[self._cur], offset, spans, n_spans, cache_rows,
                              new_rows)
        self.sites.append(_Site(offset, n, cache_rows, new_rows, key))
        step = (n + _SITE_ALIGN - 1) // _SITE_ALIGN * _SITE_ALIGN
        self._used = offset + 2 * max(step, _SITE_ALIGN)
        return self.table.data_ptr() + offset * 4

    @staticmethod
    def _write_tiles(buf: torch.Tensor, offset: int, spans, n_spans: int, cache_rows: int,
                     new_rows: int) -> int:
        n = ctypes.c_int(0)
        lib = _lib.load()
        _lib.check(lib.tm_attention_tiles(spans, n_spans, cache_rows, new_rows,
                                          buf.data_ptr() + offset * 4, MAX_TILES,
                                          ctypes.byref(n)), "attention tiles")
        return n.value

    # -- replay ------------------------------------------------------------
    def replay(self, site_spans=None):
        """Replay the graph.  ``site_spans``: None (keep the tables), a list
        with one span list per site in call order, or a dict from a site's key
        (its cache source's base address) to its span list; sites not in the
        dict keep their current table."""
        if self.graph is None:
            raise RuntimeError("nothing captured")
        stream = torch.cuda.current_stream(self.device)
        if site_spans is not None:
            nxt = 1 - self._cur
            ev = self._events[nxt]
            if ev is not None:
                ev.synchronize()  # its previous copy to the table has run
            buf = self._stage[nxt]
            if isinstance(site_spans, dict):
                buf[:self._used].copy_(self._stage[self._cur][:self._used])
                pairs = [(site, site_spans[site.key]) for site in self.sites
                         if site.key in site_spans]
                covered = {site.key for site, _ in pairs}
                if set(site_spans) - covered:
                    raise ValueError("span lists for keys no site was captured with")
            else:
                if len(site_spans) != len(self.sites):
                    raise ValueError(f"{len(site_spans)} span lists for {len(self.sites)} sites")
                pairs = list(zip(self.sites, site_spans))
            for site, spans in pairs:
                arr = (_lib.KVSpan * max(1, len(spans)))()
                for i, (src, s, r) in enumerate(spans):
                    arr[i].source, arr[i].row_start, arr[i].rows = int(src), int(s), int(r)
                n = self._write_tiles(buf, site.offset, arr, len(spans), site.cache_rows,
                                      site.new_rows)
                if n != site.n_tiles:
                    raise ValueError(f"attention site has {n} key tiles, captured with "
                                     f"{site.n_tiles}: recapture")
            self._cur = nxt
            self._dirty = True
        if self._dirty:
            with torch.cuda.stream(stream):
                # A kernel reads the pinned staging buffer (mapped into the GPU's
                # address space): a copy-engine transfer here would queue behind
                # bulk host transfers of other streams and stall the replay.
                nbytes = (self._used * 4 + 15) // 16 * 16
                copy_bytes(self.table.data_ptr(), self._stage[self._cur].data_ptr(), nbytes,
                           self.device)
                ev = torch.cuda.Event()
                ev.record(stream)
            self._events[self._cur] = ev
            self._dirty = False
        self.graph.replay()
        _lib.launched(self.launches)

    def reset(self) -> None:
        """Release the graph (before the process group that its NCCL calls
        use is destroyed)."""
        self.graph = None
        self.sites = []


def copy_bytes(dst: int, src: int, nbytes: int, device: torch.device) -> None:
    """Copy ``nbytes`` (a multiple of 16) with the row-copy kernel on the
    current stream; ``src`` may be pinned host memory."""
    span = (_lib.CopySpan * 1)()
    span[0].src, span[0].dst, span[0].rows = src, dst, 1
    span[0].src_row_stride = span[0].dst_row_stride = nbytes
    _lib.check(_lib.load().tm_copy_rows(span, 1, nbytes, _lib.stream_ptr(device)), "copy_bytes")
    _lib.launched()


def copy_into(dst: torch.Tensor, src: torch.Tensor) -> None:
    """``dst.copy_(src)`` for ``[1, H, R, W]`` tensors with contiguous rows,
    with the row-copy kernel (no copy engine; see ``AttentionGraph.replay``)."""
    if dst.shape != src.shape or dst.dtype != src.dtype or dst.dim() != 4 or dst.shape[0] != 1 \
            or dst.stride(3) != 1 or src.stride(3) != 1:
        raise ValueError("copy_into takes equal [1, H, R, W] tensors with unit column stride")
    H, R = int(dst.shape[1]), int(dst.shape[2])
    row = int(dst.shape[3]) * dst.element_size()
    if H > 64 or row % 16:
        raise ValueError("copy_into: at most 64 heads, rows a multiple of 16 bytes")
    spans = (_lib.CopySpan * H)()
    for h in range(H):
        spans[h].src, spans[h].dst, spans[h].rows = src[0, h].data_ptr(), dst[0, h].data_ptr(), R
        spans[h].src_row_stride = src.stride(2) * src.element_size()
        spans[h].dst_row_stride = dst.stride(2) * dst.element_size()
    _lib.check(_lib.load().tm_copy_rows(spans, H, row, _lib.stream_ptr(dst.device)), "copy_into")
    _lib.launched()


def attention_spans(cached_k, cached_v, new_rows: int) -> List[Tuple[int, int, int]]:
    """The span list ``flash_attention`` builds for a call over this cache and
    ``new_rows`` chunk rows (pending arena chunks are copied into their slots
    first, eagerly)."""
    from .attention import _cache_source
    _, _, rows = _cache_source(cached_k, cached_v)
    spans = [(0, int(s), int(n)) for (s, n) in rows if n > 0]
    if new_rows > 0:
        spans.append((1, 0, int(new_rows)))
    return spans
