"""Streaming generation on one rank: the block loop of the causal pipeline.

Per block (taomate/inference/model.py:166-248, model_runtime.py:772-895):
three denoising forwards over the block's noisy latents against the cached
prefix (each followed by the Euler update of the latents), one sigma = 0
commit forward whose new K/V are appended to every cache field, a segment
record, then the streaming eviction (``retain_streaming_context``: sink
segment + two newest, taomate/inference/cache.py:58-67), from
``evict_from_block`` on.

Execution: the first block runs eagerly (it initialises cuBLAS, NCCL and the
text K/V cache).  Every later forward runs from a CUDA graph
(:class:`taomate_b200.graphs.AttentionGraph`) chosen by the forward's layout:
its chunk geometry and the row count of every cache span it attends.  A
layout seen for the first time is captured once, then replayed wherever it
recurs: the four forwards of a block, every steady-state block (sink + 2
window blocks), and the sigma = 0 re-prefill forwards of each conditioning
refresh, whose layouts are those of the first window's blocks 0-2.  Per
replay only the attention key-tile table (the new arena layout), the RoPE
tables, the conditioning rows and the latents change, and each is written
into the graph's own buffers by a kernel copy.  The text K/V of every layer
are projected once per block by a separate captured graph (the reference
projects them in every forward unless its text K/V cache is on, which keeps
them per prompt).
"""

from __future__ import annotations

import gc
import time
from collections import OrderedDict
from dataclasses import dataclass, fields
from typing import List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

from . import _lib
from . import parallel as P
from .cache import (attach_segments, cache_segments, replace_modal_fields,
                    retain_streaming_context)
from .graphs import AttentionGraph, attention_spans, copy_bytes
from .kv_cache import (FIELD_PAIRS, KVCache, LayerKVCache, arena_pair, cat_cache_pair,
                       flush_many, last_chunk)
from .model import (CausalModelWeights, Conditioning, StreamConfig, arena_cache, model_forward,
                    rope_tables)
from .rope import norm_rope

# denoising sigmas of one block (taomate/inference/model.py:11-19), then 0
SIGMAS = (1.0, 0.757, 0.522, 0.0)
COND_FIELDS = ("video_ts", "audio_ts", "video_cross_ss", "video_cross_gate", "audio_cross_ss",
               "audio_cross_gate", "video_emb2", "audio_emb2")


def block_geometry(k: int, cfg: StreamConfig, first_frames: int = 4, frames: int = 3,
                   audio_first: int = 26, audio: int = 25):
    """(video frames, audio tokens, video start frame, audio start token) of
    block ``k`` in the "4-3-3-3" layout (compute_av_blocks,
    ltx_causal/attention/mask_builder.py:96-140)."""
    if k == 0:
        return first_frames, audio_first, 0, 0
    return frames, audio, first_frames + frames * (k - 1), audio_first + audio * (k - 1)


def _empty_cache(cache: KVCache) -> KVCache:
    """A cache with every field empty, on the same arenas as ``cache``."""
    layers = []
    for lay in cache.layers:
        kw = {}
        for kf, vf in FIELD_PAIRS:
            kw[kf], kw[vf] = arena_pair(getattr(lay, kf).arena)
        layers.append(LayerKVCache(**kw))
    return attach_segments(KVCache(layers=layers), [])


class _Forward:
    """One captured forward: its graph, the fixed buffers it reads (RoPE
    tables, conditioning rows, latents) and writes (the denoised latents and
    this forward's K/V chunk of every cache field)."""

    def __init__(self, runner: "StreamRunner", k: int, v: torch.Tensor, a: torch.Tensor,
                 cond: Conditioning, cache: KVCache):
        pe, off = runner._pe(k)
        self.pe = [t for pair in pe for t in pair]  # fresh tensors: the graph's own
        self.cond = [getattr(cond, n).clone() for n in COND_FIELDS]
        self.v, self.a = v.clone(), a.clone()
        scond = Conditioning(**dict(zip(COND_FIELDS, self.cond)), video_ctx=runner.ctx[0],
                             audio_ctx=runner.ctx[1], pe=pe)
        self.graph = AttentionGraph(runner.dev, max_sites=6 * runner.cfg.layers)
        with torch.no_grad():
            self.out_v, self.out_a, new = self.graph.capture(
                model_forward, runner.model, self.v, self.a, scond, cache,
                video_token_offset=off, overlap_audio=runner.overlap_audio)
        # the chunk tensors only: views of ``new`` would keep capture-time slots referenced
        self.chunks = [[last_chunk(getattr(lay, kf)) for kf, _ in FIELD_PAIRS]
                       for lay in new.layers]

    def release(self) -> None:
        self.graph.reset()


class StreamRunner:
    """Runs blocks of one stream on this rank.  ``sp``/``rank``: the sequence
    parallel layout (video tokens split, audio replicated).  ``max_graphs``:
    captured forward layouts kept (least recently used dropped first).
    ``overlap_audio``: each block's audio chain on a second stream."""

    def __init__(self, model: CausalModelWeights, device, sp: int = 1, rank: int = 0,
                 graphed: bool = True, evict_from_block: int = 0, slots: int = 6,
                 max_graphs: int = 6, overlap_audio: bool = True):
        self.model, self.cfg, self.dev = model, model.cfg, torch.device(device)
        self.sp, self.rank, self.graphed = sp, rank, graphed
        self.overlap_audio = overlap_audio
        self.evict_from_block = evict_from_block
        cfg = self.cfg
        ff, fa, _, _ = block_geometry(0, cfg)
        self.cache = arena_cache(cfg, ff * cfg.frame_tokens, fa, sp, slots, device=self.dev)
        attach_segments(self.cache, [])
        self.block = 0
        self.graphs: "OrderedDict[tuple, _Forward]" = OrderedDict()
        self.max_graphs = max_graphs
        self.captures = 0
        self.text_graph: Optional[torch.cuda.CUDAGraph] = None
        self._warm = False  # an eager forward ran since the text K/V cache was last cleared
        self.ctx = None  # (video_ctx, audio_ctx) of the current prompt
        self.latents = {}  # block_idx -> committed clean latents of the retained blocks
        self.refreshes = 0
        self.host_ms = {}  # host time of the replayed blocks, by phase
        self.host_blocks = 0

    def reset(self) -> None:
        """Start a new stream on the same arenas: every cache field empty (all
        slots free), no retained latents, block 0.  The captured forwards and
        the text graph stay: they depend only on the cache layout, so a new
        stream replays them from its first block (a service captures them
        once, in a warm-up stream)."""
        arenas = [(i, kf, getattr(lay, kf).arena) for i, lay in enumerate(self.cache.layers)
                  for kf, _ in FIELD_PAIRS]
        self.cache = _empty_cache(self.cache)
        self.latents = {}
        self.block = 0
        gc.collect()  # views of the old stream that sit in reference cycles release their slots
        busy = [(i, kf, [s for s, r in enumerate(a.refs) if r]) for i, kf, a in arenas
                if any(a.refs)]
        if busy:
            raise RuntimeError(f"arena slots still referenced after reset (layer, field, "
                               f"slots): {busy[:4]}")

    @property
    def graph(self) -> Optional[AttentionGraph]:
        """The most recently used captured forward (None: nothing captured)."""
        if not self.graphs:
            return None
        return next(reversed(self.graphs.values())).graph

    # -- geometry -------------------------------------------------------------
    def local_tokens(self, frames: int) -> Tuple[int, int]:
        L = frames * self.cfg.frame_tokens
        if L % self.sp:
            raise ValueError(f"{L} video tokens do not split over {self.sp} ranks")
        n = L // self.sp
        return n, self.rank * n

    # -- one forward ------------------------------------------------------------
    def _cond(self, c: Conditioning, pe) -> Conditioning:
        vctx, actx = self.ctx
        return Conditioning(**{f.name: getattr(c, f.name) for f in fields(Conditioning)
                               if f.name not in ("pe", "video_ctx", "audio_ctx")},
                            video_ctx=vctx, audio_ctx=actx, pe=pe)

    def set_prompt(self, video_ctx: torch.Tensor, audio_ctx: torch.Tensor) -> None:
        """New text conditioning (projected contexts ``[1, 256, D]``).  Kept in
        fixed buffers so captured graphs read the current prompt."""
        if self.ctx is None:
            self.ctx = (video_ctx.clone(), audio_ctx.clone())
        else:
            self.ctx[0].copy_(video_ctx)
            self.ctx[1].copy_(audio_ctx)
        if self.text_graph is not None:
            self.text_graph.replay()  # re-project into the entries the forward graphs read
        else:
            # the text K/V cache is keyed by the context tensor's identity, which
            # stays: drop its entries so the next forward projects the new prompt
            for blk in self.model.transformer_blocks:
                for attn in (blk.attn2, blk.audio_attn2):
                    if hasattr(attn, "_ltx_text_cross_kv_cache"):
                        attn._ltx_text_cross_kv_cache.clear()
            self._warm = False  # the next forward projects them eagerly

    def _use_graphs(self) -> bool:
        return self.graphed and self._warm

    # -- the block ------------------------------------------------------------
    def run_block(self, video_latent: torch.Tensor, audio_latent: torch.Tensor,
                  conds: Sequence[Conditioning]) -> Tuple[torch.Tensor, torch.Tensor]:
        """Denoise the block's latents (``[1, Lv_local, C]``, ``[1, La, C]``)
        with ``conds[0..2]``, commit with ``conds[3]``; returns the denoised
        latents (fresh tensors)."""
        if self._use_graphs():
            return self._replay_block(video_latent, audio_latent, conds)
        return self._eager_block(video_latent, audio_latent, conds)

    def end_segment(self) -> None:
        """The streaming eviction at a window boundary (runtime.py:634)."""
        if len(cache_segments(self.cache)) > 3:
            self.cache = retain_streaming_context(self.cache)
        self._drop_latents()

    def refresh(self, conds: dict) -> None:
        """Re-prefill the prompt-sensitive K/V of the retained blocks with the
        current prompt (``_refresh_conditioning_cache``, taomate/inference/
        runtime.py:386-470): one sigma = 0 ``kv_cache_only`` forward per
        retained segment, in order, over that block's committed clean
        latents, each against the K/V rebuilt so far; then every field except
        the video self-attention K/V is taken from the rebuilt cache (no data
        moves).  The rebuilt rows go to free slots of the same arenas, so a
        captured forward keeps reading them.  ``conds[block_idx]``: the
        block's sigma = 0 conditioning rows.  The forwards replay the graphs
        of their layouts (those of the first window's blocks 0-2)."""
        segs = cache_segments(self.cache)
        if not segs:
            raise RuntimeError("The retained cache has no block metadata.")
        rebuilt = _empty_cache(self.cache)
        with torch.no_grad():
            for seg in segs:
                k = int(seg["block_idx"])
                v, a = self.latents[k]
                if self._use_graphs():
                    g, spans = self._graph_for(k, v, a, conds[k], rebuilt)
                    pe, _ = self._pe(k)
                    self._load(g.pe, [t for pair in pe for t in pair])
                    self._load([g.v, g.a] + g.cond,
                               [v, a] + [getattr(conds[k], n) for n in COND_FIELDS])
                    g.graph.replay(spans)
                    rebuilt = self._appended(rebuilt, g.chunks)
                else:
                    pe, off = self._pe(k)
                    _, _, rebuilt = model_forward(self.model, v, a, self._cond(conds[k], pe),
                                                  rebuilt, kv_cache_only=True,
                                                  video_token_offset=off,
                                                  overlap_audio=self.overlap_audio)
                    self._warm = True
                flush_many([getattr(lay, kf) for lay in rebuilt.layers for kf, _ in FIELD_PAIRS])
        self.cache = replace_modal_fields(self.cache, rebuilt)
        self.refreshes += 1

    def _drop_latents(self) -> None:
        keep = {int(s["block_idx"]) for s in cache_segments(self.cache)}
        for k in [k for k in self.latents if k not in keep]:
            del self.latents[k]

    def _pe(self, k: int):
        F_, La, vs, as_ = block_geometry(k, self.cfg)
        n, off = self.local_tokens(F_)
        return rope_tables(self.cfg, F_, La, vs, as_, self.dev, slice(off, off + n)), off

    def _commit(self, new_cache: KVCache, clean: Tuple[torch.Tensor, torch.Tensor]) -> None:
        self.latents[self.block] = clean
        F_, La, _, _ = block_geometry(self.block, self.cfg)
        segs = cache_segments(self.cache) + [{"block_idx": self.block,
                                              "video_tokens": F_ * self.cfg.frame_tokens,
                                              "audio_tokens": La}]
        attach_segments(new_cache, segs)
        # copy the pending chunks into their slots now, in a few batched launches
        flush_many([getattr(lay, kf) for lay in new_cache.layers for kf, _ in FIELD_PAIRS])
        if self.block >= self.evict_from_block and len(segs) > 3:
            new_cache = retain_streaming_context(new_cache)
        self.cache = new_cache
        self._drop_latents()
        self.block += 1

    def _eager_block(self, v, a, conds):
        pe, off = self._pe(self.block)
        x_v, x_a = v, a
        with torch.no_grad():
            for fwd in range(3):
                vo, ao, _ = model_forward(self.model, x_v, x_a, self._cond(conds[fwd], pe),
                                          self.cache, video_token_offset=off,
                                          overlap_audio=self.overlap_audio)
                dt = SIGMAS[fwd + 1] - SIGMAS[fwd]
                x_v = torch.add(x_v, vo, alpha=dt)  # the graph path's update, same rounding
                x_a = torch.add(x_a, ao, alpha=dt)
            _, _, new = model_forward(self.model, x_v, x_a, self._cond(conds[3], pe), self.cache,
                                      kv_cache_only=True, video_token_offset=off,
                                      overlap_audio=self.overlap_audio)
        self._warm = True
        self._commit(new, (x_v, x_a))
        return x_v, x_a

    # -- graph executor -------------------------------------------------------
    def _spans(self, cache: KVCache, k: int):
        """Key spans of every cached attention of a forward of block ``k``
        over ``cache``, keyed by the site's cache arena (the text
        cross-attention sites keep theirs)."""
        F_, La, _, _ = block_geometry(k, self.cfg)
        Lv = F_ * self.cfg.frame_tokens
        Lv_local, _ = self.local_tokens(F_)  # V2A keys: this rank's video tokens
        out = {}
        for lay in cache.layers:
            for (kf, vf), new_rows in zip(FIELD_PAIRS, (Lv, La, La, Lv_local)):
                kv, vv = getattr(lay, kf), getattr(lay, vf)
                out[kv.arena.k.data_ptr()] = attention_spans(kv, vv, new_rows)
        return out

    @staticmethod
    def _layout(spans: dict) -> tuple:
        """What a captured forward fixes: the row count of every key span of
        every site (the tile counts follow from it)."""
        return tuple((key, tuple((src, rows) for src, _, rows in sp))
                     for key, sp in sorted(spans.items()))

    def _graph_for(self, k: int, v, a, cond: Conditioning, cache: KVCache):
        """The captured forward of block ``k``'s geometry over ``cache``'s
        layout (captured now if this layout is new) and the spans to replay
        it with."""
        spans = self._spans(cache, k)  # also copies pending chunks into their slots
        F_, La, _, _ = block_geometry(k, self.cfg)
        sig = (F_, La, self._layout(spans))
        g = self.graphs.get(sig)
        if g is not None:
            self.graphs.move_to_end(sig)
            return g, spans
        while len(self.graphs) >= self.max_graphs:
            _, old = self.graphs.popitem(last=False)
            old.release()
        g = _Forward(self, k, v, a, cond, cache)
        self.graphs[sig] = g
        self.captures += 1
        if self.text_graph is None:
            self._capture_text()
        return g, spans

    def _capture_text(self):
        """A graph that re-projects the text K/V of every layer into the
        buffers the forward graphs read (the text K/V cache entries)."""
        jobs = []
        for blk in self.model.transformer_blocks:
            for attn, ctx in ((blk.attn2, self.ctx[0]), (blk.audio_attn2, self.ctx[1])):
                ent = [e for e in getattr(attn, "_ltx_text_cross_kv_cache", {}).values()
                       if e[0]() is ctx]
                if len(ent) != 1:
                    raise RuntimeError("text K/V cache entry missing before capture")
                jobs.append((attn, ctx, ent[0][1], ent[0][2]))
        self._text_jobs = jobs
        g = torch.cuda.CUDAGraph()
        with torch.no_grad(), torch.cuda.graph(g):
            self._project_text()
        self.text_graph = g

    def _project_text(self):
        for attn, ctx, k, v in self._text_jobs:
            H, D = int(attn.heads), int(attn.dim_head)
            kp = F.linear(ctx, attn.to_k.weight, attn.to_k.bias)
            (kn,) = norm_rope([kp], [attn.k_norm.weight], [None], H, D,
                              float(attn.k_norm.eps or 1e-6))
            k.copy_(kn)
            v.copy_(F.linear(ctx, attn.to_v.weight, attn.to_v.bias).view_as(v))

    def _load(self, dst: List[torch.Tensor], src: List[torch.Tensor]) -> None:
        for d, s in zip(dst, src):
            s = s if s.is_contiguous() else s.contiguous()
            copy_bytes(d.data_ptr(), s.data_ptr(), (d.numel() * d.element_size() + 15) // 16 * 16,
                       self.dev)

    @staticmethod
    def _appended(cache: KVCache, chunks) -> KVCache:
        """``cache`` with a captured forward's K/V chunk appended to every field."""
        layers = []
        for lay, lay_chunks in zip(cache.layers, chunks):
            kw = {}
            for (kf, vf), (nk, nv) in zip(FIELD_PAIRS, lay_chunks):
                kw[kf], kw[vf] = cat_cache_pair(getattr(lay, kf), getattr(lay, vf), nk, nv)
            layers.append(LayerKVCache(**kw))
        return KVCache(layers=layers)

    def _replay_block(self, v, a, conds):
        t0 = time.perf_counter()
        g, spans = self._graph_for(self.block, v, a, conds[0], self.cache)
        pe, _ = self._pe(self.block)
        self._load(g.pe, [t for pair in pe for t in pair])
        self._load([g.v, g.a], [v, a])
        self.text_graph.replay()
        t1 = time.perf_counter()
        for fwd in range(4):
            self._load(g.cond, [getattr(conds[fwd], n) for n in COND_FIELDS])
            g.graph.replay(spans if fwd == 0 else None)
            if fwd < 3:
                dt = SIGMAS[fwd + 1] - SIGMAS[fwd]
                g.v.add_(g.out_v, alpha=dt)
                g.a.add_(g.out_a, alpha=dt)
        t2 = time.perf_counter()
        # commit: this block's K/V (the fourth replay's) appended to the cache
        clean = (g.v.clone(), g.a.clone())
        self._commit(self._appended(self.cache, g.chunks), clean)
        t3 = time.perf_counter()
        for k, dt in (("prepare", t1 - t0), ("replays", t2 - t1), ("commit_evict", t3 - t2)):
            self.host_ms[k] = self.host_ms.get(k, 0.0) + dt * 1e3
        self.host_blocks += 1
        return clean

    def release(self):
        """Drop the captured graphs (before the process group goes away)."""
        for g in self.graphs.values():
            g.release()
        self.graphs.clear()
        self.text_graph = None
