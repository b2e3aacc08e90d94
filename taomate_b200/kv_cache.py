"""KV cache objects for the streaming path, backed by a per-layer slot arena.

``LayerKVCache`` / ``KVCache`` keep the field names and ``[B, L, H, D]``
semantics of ``ltx_causal/transformer/kv_cache.py:321-358``.  A field may hold
either a plain tensor (exactly as in the reference) or an :class:`ArenaKV`
view: an ordered list of row ranges inside a preallocated per-layer arena
(:class:`KVArena`).  With arena views

* the attention kernel reads the cached keys where they lie (no
  ``torch.cat`` per forward, kv_cache.py:1486-1492);
* appending a block (``_cat_cache``, kv_cache.py:394-398) records the new
  chunk and copies it into a free slot only when the cache is next read or
  retained, so the three denoising forwards of a block, whose caches the
  pipeline throws away (taomate/inference/model_runtime.py:847-895), move no
  bytes;
* eviction (``retain_streaming_context``, taomate/inference/cache.py:58-67)
  rewrites the row list and moves no bytes.

Views never change the rows they reference: new data only goes to slots no
live view references (slot reference counts), so an old ``LayerKVCache`` kept
as a snapshot stays valid after later appends and evictions, which the
denoise snapshot/restore relies on.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field, fields as dataclass_fields
from typing import List, Optional, Sequence, Tuple

import torch
from torch import Tensor

from . import _lib

FIELD_PAIRS = (("video_self_k", "video_self_v"), ("audio_self_k", "audio_self_v"),
               ("a2v_k", "a2v_v"), ("v2a_k", "v2a_v"))


class KVArena:
    """Slot arena for one K/V pair of one layer.

    ``k`` and ``v`` are ``[B, n_slots * slot_rows, H, D]`` tensors (zero
    initialised so rows outside any view are finite); slot ``i`` owns rows
    ``[i * slot_rows, (i + 1) * slot_rows)``.  Slots are handed out lowest
    index first and returned when the last view that references them dies.
    """

    def __init__(self, n_slots: int, slot_rows: int, batch: int, heads: int, dim_head: int,
                 dtype: torch.dtype = torch.bfloat16, device="cuda"):
        if n_slots < 1 or slot_rows < 1:
            raise ValueError("arena needs at least one slot of one row")
        self.n_slots = int(n_slots)
        self.slot_rows = int(slot_rows)
        self.batch, self.heads, self.dim_head = int(batch), int(heads), int(dim_head)
        shape = (self.batch, self.n_slots * self.slot_rows, self.heads, self.dim_head)
        self.k = torch.zeros(shape, dtype=dtype, device=device)
        self.v = torch.zeros(shape, dtype=dtype, device=device)
        self.refs = [0] * self.n_slots
        self.appends = 0  # slot writes so far (commit appends)

    @property
    def rows(self) -> int:
        return self.n_slots * self.slot_rows

    def free_slots(self) -> List[int]:
        return [i for i, r in enumerate(self.refs) if r == 0]

    def _take(self) -> int:
        for i, r in enumerate(self.refs):
            if r == 0:
                self.refs[i] = 1
                return i
        raise RuntimeError(f"KV arena full: all {self.n_slots} slots of {self.slot_rows} rows "
                           "are referenced by live cache views")

    def _ref(self, slot: int, delta: int) -> None:
        self.refs[slot] += delta
        if self.refs[slot] < 0:
            raise RuntimeError("KV arena slot reference count went negative")

    def write(self, k: Tensor, v: Tensor) -> List[Tuple[int, int, int]]:
        """Copy a ``[B, L, H, D]`` chunk into free slots (one launch of the
        span-copy kernel for K and V together); returns the row entries."""
        entries, spans, row_bytes = self.plan_write(k, v)
        _launch_copies(spans, row_bytes, k.device)
        self.appends += 1
        return entries

    def plan_write(self, k: Tensor, v: Tensor):
        """Take free slots for a ``[B, L, H, D]`` chunk; returns ``(entries,
        copy spans, row bytes)`` without launching (see :func:`flush_many`)."""
        if k.shape != v.shape or k.dim() != 4 or k.shape[0] != self.batch or \
                k.shape[2] != self.heads or k.shape[3] != self.dim_head:
            raise ValueError(f"chunk shape {tuple(k.shape)} does not fit arena "
                             f"[B={self.batch}, H={self.heads}, D={self.dim_head}]")
        if k.dtype != self.k.dtype:
            raise TypeError(f"chunk dtype {k.dtype} != arena dtype {self.k.dtype}")
        L = int(k.shape[1])
        entries: List[Tuple[int, int, int]] = []
        pieces = []
        off = 0
        while off < L:
            n = min(self.slot_rows, L - off)
            slot = self._take()
            entries.append((slot, slot * self.slot_rows, n))
            pieces.append((off, slot * self.slot_rows, n))
            off += n
        row_bytes = self.heads * self.dim_head * k.element_size()
        spans = []
        _lib.require_cuda(k, v, self.k)
        for src, dst in ((k, self.k), (v, self.v)):
            if src.stride(3) != 1 or src.stride(2) != self.dim_head:
                src = src.contiguous()
            for (soff, drow, n) in pieces:
                for b in range(self.batch):
                    spans.append((src[b, soff].data_ptr(), dst[b, drow].data_ptr(), n,
                                  src.stride(1) * src.element_size(),
                                  dst.stride(1) * dst.element_size(), src))
        return entries, spans, row_bytes


def _launch_copies(spans, row_bytes: int, device) -> None:
    """Row-span copies of one row size, 64 spans per launch of the span-copy
    kernel (current stream).  Each span is ``(src, dst, rows, src_stride,
    dst_stride, keep)``."""
    if not spans:
        return
    dev = torch.device(device)
    lib = _lib.load()
    with torch.cuda.device(dev):
        for i in range(0, len(spans), 64):
            part = spans[i:i + 64]
            arr = (_lib.CopySpan * len(part))()
            for j, (src, dst, n, ss, ds, _) in enumerate(part):
                arr[j].src, arr[j].dst, arr[j].rows = src, dst, n
                arr[j].src_row_stride, arr[j].dst_row_stride = ss, ds
            _lib.check(lib.tm_copy_rows(arr, len(part), row_bytes, _lib.stream_ptr(dev)),
                       "KV arena copy")
            _lib.launched()


def flush_many(views) -> None:
    """Copy the pending chunks of many arena views into free slots with as few
    launches as possible: the copies of every view are grouped by row size,
    64 spans per launch (a commit of 48 layers x 4 pairs takes a handful of
    launches instead of 192).  Same result as ``view.entries()`` on each."""
    groups = {}
    device = None
    for view in views:
        if not isinstance(view, ArenaKV):
            continue
        st = view._state
        while st.pending:
            k, v = st.pending[0]
            if v is None:
                raise RuntimeError("K chunk appended without its V chunk")
            entries, spans, row_bytes = st.arena.plan_write(k, v)
            st.arena.appends += 1
            st.pending.pop(0)
            st.entries.extend(entries)
            groups.setdefault(row_bytes, []).extend(spans)
            device = k.device
    for row_bytes, spans in groups.items():
        _launch_copies(spans, row_bytes, device)


class ArenaKV:
    """A K or V cache field as an ordered list of arena row ranges plus chunks
    appended but not yet copied in.  Behaves like a ``[B, L, H, D]`` tensor for
    ``shape`` / ``size`` / ``dtype`` / ``device``; ``materialize()`` returns
    the contiguous tensor.  ``kind`` is ``"k"`` or ``"v"``; the K and V views
    of a pair share their row entries and pending chunks (``_pair``)."""

    __slots__ = ("arena", "kind", "_state", "__weakref__")

    def __init__(self, arena: KVArena, kind: str, state: "_PairState"):
        self.arena = arena
        self.kind = kind
        self._state = state

    # --- tensor-like surface -------------------------------------------------
    @property
    def shape(self) -> torch.Size:
        return torch.Size((self.arena.batch, self._state.length(), self.arena.heads,
                           self.arena.dim_head))

    def size(self, dim: Optional[int] = None):
        return self.shape if dim is None else self.shape[dim]

    @property
    def dtype(self) -> torch.dtype:
        return self.arena.k.dtype

    @property
    def device(self) -> torch.device:
        return self.arena.k.device

    def dim(self) -> int:
        return 4

    def entries(self) -> List[Tuple[int, int, int]]:
        """Arena row entries ``(slot, first_row, rows)`` after flushing pending chunks."""
        self._state.flush()
        return list(self._state.entries)

    def materialize(self) -> Tensor:
        """Contiguous ``[B, L, H, D]`` copy (span-copy kernel)."""
        ents = self.entries()
        src = self.arena.k if self.kind == "k" else self.arena.v
        out = torch.empty(self.shape, dtype=self.dtype, device=self.device)
        if not ents:
            return out
        row_bytes = self.arena.heads * self.arena.dim_head * src.element_size()
        spans = (_lib.CopySpan * (len(ents) * self.arena.batch))()
        i = 0
        off = 0
        for (_, row, n) in ents:
            for b in range(self.arena.batch):
                sp = spans[i]
                sp.src = src[b, row].data_ptr()
                sp.dst = out[b, off].data_ptr()
                sp.rows = n
                sp.src_row_stride = src.stride(1) * src.element_size()
                sp.dst_row_stride = out.stride(1) * out.element_size()
                i += 1
            off += n
        dev = self.device
        with torch.cuda.device(dev):
            _lib.check(_lib.load().tm_copy_rows(spans, i, row_bytes, _lib.stream_ptr(dev)),
                       "ArenaKV.materialize")
            _lib.launched()
        return out

    def __repr__(self) -> str:
        return (f"ArenaKV({self.kind}, shape={tuple(self.shape)}, entries={self._state.entries}, "
                f"pending={[tuple(p[0].shape) for p in self._state.pending]})")


class _PairState:
    """Shared state of the K and V views of one cache field pair: committed
    arena entries ``(slot, first_row, rows)`` and pending ``[k, v]`` chunks.
    ``child`` links a state to the state produced by a K append that still
    waits for its V chunk (the reference appends K and V with two separate
    ``_cat_cache`` calls)."""

    __slots__ = ("arena", "entries", "pending", "child", "__weakref__")

    def __init__(self, arena: KVArena, entries: Sequence[Tuple[int, int, int]],
                 pending: Sequence[list] = ()):
        self.arena = arena
        self.entries = list(entries)
        self.pending = [list(p) for p in pending]
        self.child = None
        for (slot, _, _) in self.entries:
            arena._ref(slot, +1)

    def length(self) -> int:
        return sum(n for (_, _, n) in self.entries) + sum(int(p[0].shape[1]) for p in self.pending)

    def flush(self) -> None:
        while self.pending:
            k, v = self.pending[0]
            if v is None:
                raise RuntimeError("K chunk appended without its V chunk")
            new = self.arena.write(k, v)  # slots come back with refcount 1 (ours)
            self.pending.pop(0)
            self.entries.extend(new)

    def sliced(self, spans: Sequence[Tuple[int, int]]) -> "_PairState":
        """State holding token ranges ``[start, end)`` of this one, in order
        (no data moves)."""
        self.flush()
        out = []
        for (s, e) in spans:
            off = 0
            for (slot, row, n) in self.entries:
                lo, hi = max(s, off), min(e, off + n)
                if hi > lo:
                    out.append((slot, row + (lo - off), hi - lo))
                off += n
            if e > off or s < 0:
                raise IndexError(f"span [{s}, {e}) outside cache of {off} rows")
        return _PairState(self.arena, out)

    def __del__(self):
        try:
            for (slot, _, _) in self.entries:
                self.arena._ref(slot, -1)
        except Exception:
            pass


def arena_pair(arena: KVArena, entries=(), pending=()) -> Tuple[ArenaKV, ArenaKV]:
    st = _PairState(arena, entries, pending)
    return ArenaKV(arena, "k", st), ArenaKV(arena, "v", st)


def is_arena(x) -> bool:
    return isinstance(x, ArenaKV)


@dataclass
class LayerKVCache:
    """Per-layer KV cache for the 4 cached attention types (kv_cache.py:321-348).

    Shapes ``video_self_{k,v}: [B, Lv, Hv, Dv]``, ``audio_self_{k,v}: [B, La,
    Ha, Da]``, ``a2v_{k,v}: [B, La, Hc, Dc]``, ``v2a_{k,v}: [B, Lv, Hc, Dc]``;
    head-sharded (H/sp heads, full sequence) under Ulysses SP.  Each field is a
    tensor or an :class:`ArenaKV` view.
    """
    video_self_k: Optional[object] = None
    video_self_v: Optional[object] = None
    audio_self_k: Optional[object] = None
    audio_self_v: Optional[object] = None
    a2v_k: Optional[object] = None
    a2v_v: Optional[object] = None
    v2a_k: Optional[object] = None
    v2a_v: Optional[object] = None


@dataclass
class KVCache:
    """Full KV cache across layers (kv_cache.py:351-358)."""
    layers: List[LayerKVCache] = field(default_factory=list)
    layerwise_cpu_offload: bool = False


def _cat_cache(old, new: Tensor):
    """Append ``new`` K/V along the sequence (kv_cache.py:394-398).

    Plain tensors concatenate like the reference (span-copy kernel into a
    fresh tensor).  For an :class:`ArenaKV` the chunk is recorded as pending
    and copied into a free slot on first use; the result is a new view and
    ``old`` is unchanged.  As in ``block_forward_with_cache``
    (kv_cache.py:2642-2654) the K field of a pair is appended first, then
    the V field of the same pair.
    """
    if old is None:
        return new
    if isinstance(old, ArenaKV):
        st = old._state
        if old.kind == "k":
            ns = _PairState(st.arena, st.entries, st.pending + [[new, None]])
            st.child = ns
            return ArenaKV(st.arena, "k", ns)
        ns = st.child
        if ns is None or not ns.pending or ns.pending[-1][1] is not None:
            raise RuntimeError("append the K field of an arena pair before its V field")
        if tuple(ns.pending[-1][0].shape) != tuple(new.shape):
            raise ValueError(f"V chunk {tuple(new.shape)} does not match K chunk "
                             f"{tuple(ns.pending[-1][0].shape)}")
        ns.pending[-1][1] = new
        st.child = None
        return ArenaKV(st.arena, "v", ns)
    return cat_tensors(old, new)


def last_chunk(view_k: "ArenaKV") -> Tuple[Tensor, Tensor]:
    """The ``(k, v)`` chunk most recently appended to an arena view pair and
    not yet copied into a slot (a forward's new K/V, as ``_cat_cache``
    recorded it)."""
    if not isinstance(view_k, ArenaKV) or not view_k._state.pending:
        raise ValueError("no pending chunk on this cache view")
    k, v = view_k._state.pending[-1]
    if v is None:
        raise RuntimeError("K chunk appended without its V chunk")
    return k, v


def cat_cache_pair(old_k, old_v, new_k: Tensor, new_v: Tensor):
    """Append a K/V chunk to a pair of cache fields; returns ``(k, v)``."""
    return _cat_cache(old_k, new_k), _cat_cache(old_v, new_v)


def cat_tensors(a: Tensor, b: Tensor) -> Tensor:
    """``torch.cat([a, b], dim=1)`` for ``[B, L, H, D]`` CUDA tensors through
    the span-copy kernel."""
    dev = _lib.require_cuda(a, b)
    if a.shape[0] != b.shape[0] or a.shape[2:] != b.shape[2:] or a.dtype != b.dtype:
        raise ValueError(f"cannot concatenate {tuple(a.shape)} and {tuple(b.shape)}")
    a = a if a.is_contiguous() else a.contiguous()
    b = b if b.is_contiguous() else b.contiguous()
    B, La, Lb = int(a.shape[0]), int(a.shape[1]), int(b.shape[1])
    out = torch.empty((B, La + Lb) + tuple(a.shape[2:]), dtype=a.dtype, device=dev)
    row_bytes = a[0, 0].numel() * a.element_size() if La else b[0, 0].numel() * b.element_size()
    spans = (_lib.CopySpan * (2 * B))()
    i = 0
    for src, off, n in ((a, 0, La), (b, La, Lb)):
        if n == 0:
            continue
        for bi in range(B):
            sp = spans[i]
            sp.src = src[bi, 0].data_ptr()
            sp.dst = out[bi, off].data_ptr()
            sp.rows = n
            sp.src_row_stride = src.stride(1) * src.element_size()
            sp.dst_row_stride = out.stride(1) * out.element_size()
            i += 1
    if i:
        with torch.cuda.device(dev):
            _lib.check(_lib.load().tm_copy_rows(spans, i, row_bytes, _lib.stream_ptr(dev)),
                       "cat_tensors")
            _lib.launched()
    return out


@dataclass
class ArenaSpec:
    """Arena geometry for one field pair of every layer."""
    n_slots: int
    slot_rows: int
    heads: int
    dim_head: int


def init_arena_cache(num_layers: int, specs: dict, batch: int = 1,
                     dtype: torch.dtype = torch.bfloat16, device="cuda") -> KVCache:
    """A :class:`KVCache` whose fields are empty arena views.

    ``specs`` maps a pair name (``"video_self"``, ``"audio_self"``, ``"a2v"``,
    ``"v2a"``) to an :class:`ArenaSpec`; pairs not listed stay ``None``.  For
    the production schedule (sink block + 2 recent blocks, up to 5 blocks in
    the first window) 6 slots of the largest block size suffice.
    """
    layers = []
    for _ in range(num_layers):
        kw = {}
        for name, sp in specs.items():
            arena = KVArena(sp.n_slots, sp.slot_rows, batch, sp.heads, sp.dim_head, dtype, device)
            kw[name + "_k"], kw[name + "_v"] = arena_pair(arena)
        layers.append(LayerKVCache(**kw))
    return KVCache(layers=layers)


def cache_rows_view(x):
    """``(tensor, [(row_start, rows), ...])`` for the attention kernel's cache
    source: an arena (all entries, flushed) or a plain ``[B, L, H, D]`` tensor."""
    if isinstance(x, ArenaKV):
        ents = x.entries()
        t = x.arena.k if x.kind == "k" else x.arena.v
        return t, [(row, n) for (_, row, n) in ents]
    return x, [(0, int(x.shape[1]))]
