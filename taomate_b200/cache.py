"""Cache segment metadata and streaming eviction (taomate/inference/cache.py).

Same functions and behaviour as the reference module: a segment is a dict
``{"block_idx", "video_tokens", "audio_tokens"}`` recorded after every clean
commit; ``retain_streaming_context`` keeps the sink segment (``block_idx ==
0``) and the two newest other segments, in chronological order.

For arena-backed caches (:class:`taomate_b200.kv_cache.ArenaKV` fields) the
slice is a rewrite of each view's row list: no bytes move and the evicted
slots return to the arena once no snapshot references them.  Plain-tensor
fields are sliced with the span-copy kernel into new tensors, as the
reference does with ``torch.cat``.
"""

from __future__ import annotations

from typing import Dict, List, Tuple

import torch

from . import _lib
from .kv_cache import ArenaKV, KVCache, LayerKVCache

VIDEO_FIELDS = ("video_self_k", "video_self_v", "v2a_k", "v2a_v")
AUDIO_FIELDS = ("audio_self_k", "audio_self_v", "a2v_k", "a2v_v")


def cache_segments(cache: KVCache) -> List[Dict[str, int]]:
    """Copy of the cache's segment list (cache.py:7-8)."""
    return [dict(item) for item in getattr(cache, "segments", [])]


def attach_segments(cache: KVCache, segments: List[Dict[str, int]]) -> KVCache:
    """Attach a copy of ``segments`` to ``cache`` (cache.py:10-12)."""
    cache.segments = [dict(item) for item in segments]
    return cache


def _segment_offsets(segments: List[Dict[str, int]]) -> List[Tuple[int, int, int, int]]:
    """Cumulative ``(video_start, video_end, audio_start, audio_end)`` token
    offsets per segment (cache.py:14-26)."""
    video_offset = 0
    audio_offset = 0
    offsets = []
    for segment in segments:
        video_end = video_offset + int(segment["video_tokens"])
        audio_end = audio_offset + int(segment["audio_tokens"])
        offsets.append((video_offset, video_end, audio_offset, audio_end))
        video_offset = video_end
        audio_offset = audio_end
    return offsets


def retain_indices(segments: List[Dict[str, int]], recent_blocks: int = 2) -> List[int]:
    """Segment indices kept by the streaming policy (cache.py:58-66)."""
    if not segments:
        raise RuntimeError("Cached inference did not attach block metadata.")
    sink = next(index for index, item in enumerate(segments) if int(item["block_idx"]) == 0)
    non_sink = [index for index in range(len(segments)) if index != sink]
    recent = non_sink[-recent_blocks:] if recent_blocks > 0 else []
    return sorted([sink, *recent])


def _slice_tensor(tensor: torch.Tensor, spans: List[Tuple[int, int]]) -> torch.Tensor:
    """Concatenation of ``tensor[:, s:e]`` over ``spans`` (cache.py:28-32),
    through the span-copy kernel."""
    pieces = [(s, e) for s, e in spans if e > s]
    if len(pieces) == 1:
        s, e = pieces[0]
        return tensor[:, s:e]
    dev = _lib.require_cuda(tensor)
    t = tensor if tensor.stride(-1) == 1 and tensor[0, 0].is_contiguous() else tensor.contiguous()
    B = int(t.shape[0])
    total = sum(e - s for s, e in pieces)
    out = torch.empty((B, total) + tuple(t.shape[2:]), dtype=t.dtype, device=dev)
    if total == 0:
        return out
    row_bytes = t[0, 0].numel() * t.element_size()
    spans_c = (_lib.CopySpan * (len(pieces) * B))()
    i = off = 0
    for s, e in pieces:
        for b in range(B):
            sp = spans_c[i]
            sp.src = t[b, s].data_ptr()
            sp.dst = out[b, off].data_ptr()
            sp.rows = e - s
            sp.src_row_stride = t.stride(1) * t.element_size()
            sp.dst_row_stride = out.stride(1) * out.element_size()
            i += 1
        off += e - s
    with torch.cuda.device(dev):
        _lib.check(_lib.load().tm_copy_rows(spans_c, i, row_bytes, _lib.stream_ptr(dev)),
                   "_slice_tensor")
        _lib.launched()
    return out


def _slice_pair(k, v, spans: List[Tuple[int, int]]):
    if k is None:
        return None, None
    if isinstance(k, ArenaKV):
        if not isinstance(v, ArenaKV) or v._state is not k._state:
            raise ValueError("K and V arena views of a pair must share their state")
        st = k._state.sliced(spans)
        return ArenaKV(st.arena, "k", st), ArenaKV(st.arena, "v", st)
    return _slice_tensor(k, spans), _slice_tensor(v, spans)


def _field_spans(spans: List[Tuple[int, int]], tokens: int, field) -> List[Tuple[int, int]]:
    """Token spans as row spans of a cache field that holds every token
    (rows == tokens) or one rank's equal share of each segment's tokens
    (tokens / rows rows per token: the split-key V2A cache under sequence
    parallelism)."""
    if field is None:
        return spans
    rows = int(field.shape[1])
    if rows == tokens:
        return spans
    if rows == 0 or tokens % rows:
        raise ValueError(f"a cache field of {rows} rows does not hold shares of {tokens} tokens")
    f = tokens // rows
    if any(s % f or e % f for s, e in spans):
        raise ValueError(f"segment boundaries do not split over {f} ranks")
    return [(s // f, e // f) for s, e in spans]


def _slice_cache(cache: KVCache, indices: List[int]) -> KVCache:
    """Keep the segments ``indices`` of every layer field (cache.py:34-56):
    video spans slice ``video_self_*`` and ``v2a_*``, audio spans slice
    ``audio_self_*`` and ``a2v_*`` (a V2A cache holding one rank's share of
    the video tokens is sliced by the same share of each span)."""
    segments = cache_segments(cache)
    offsets = _segment_offsets(segments)
    video_spans = [(offsets[i][0], offsets[i][1]) for i in indices]
    audio_spans = [(offsets[i][2], offsets[i][3]) for i in indices]
    video_tokens = offsets[-1][1] if offsets else 0
    layers = []
    for layer in cache.layers:
        vk, vv = _slice_pair(layer.video_self_k, layer.video_self_v, video_spans)
        ak, av = _slice_pair(layer.audio_self_k, layer.audio_self_v, audio_spans)
        a2k, a2v = _slice_pair(layer.a2v_k, layer.a2v_v, audio_spans)
        v2k, v2v = _slice_pair(layer.v2a_k, layer.v2a_v,
                               _field_spans(video_spans, video_tokens, layer.v2a_k))
        layers.append(LayerKVCache(video_self_k=vk, video_self_v=vv, audio_self_k=ak,
                                   audio_self_v=av, a2v_k=a2k, a2v_v=a2v, v2a_k=v2k, v2a_v=v2v))
    return attach_segments(KVCache(layers=layers), [segments[i] for i in indices])


def retain_streaming_context(cache: KVCache) -> KVCache:
    """Keep the sink block and the two newest blocks (cache.py:58-67)."""
    segments = cache_segments(cache)
    keep = retain_indices(segments)
    return cache if keep == list(range(len(segments))) else _slice_cache(cache, keep)


def retain_window(cache: KVCache, anchor_tokens: int, window_tokens: int,
                  field_names=("video_self",)) -> KVCache:
    """Token-granular retention for arena caches: the first ``anchor_tokens``
    rows plus the newest ``window_tokens`` rows of each listed pair (the
    "1 anchor frame + 8 window frames" layout of the benchmark config).  No
    data moves; segments are not tracked."""
    layers = []
    for layer in cache.layers:
        kw = {f.name: getattr(layer, f.name) for f in LayerKVCache.__dataclass_fields__.values()}
        for name in field_names:
            k, v = kw[name + "_k"], kw[name + "_v"]
            if k is None:
                continue
            L = int(k.shape[1])
            if L <= anchor_tokens + window_tokens:
                continue
            spans = [(0, anchor_tokens), (L - window_tokens, L)]
            kw[name + "_k"], kw[name + "_v"] = _slice_pair(k, v, spans)
        layers.append(LayerKVCache(**kw))
    return KVCache(layers=layers)


# ---------------------------------------------------------------------------
# Conditioning refresh (taomate/inference/runtime.py:386-470,
# taomate/inference/streaming_runtime.py:1003-1200)
# ---------------------------------------------------------------------------
AUDIO_FRAMES_PER_BLOCK = 25    # ltx_causal/attention/mask_builder.py:97
AUDIO_FRAMES_FIRST_BLOCK = 26  # mask_builder.py:99


def compute_av_blocks(total_video_latent_frames: int, num_frame_per_block: int = 3,
                      num_frame_per_block_first: int = 0) -> List[Tuple[int, int, int, int, int]]:
    """``(block_idx, video_start, video_end, audio_start, audio_end)`` of the
    streaming blocks (mask_builder.py:102-186): an optional longer first block
    (26 audio frames), then blocks of ``num_frame_per_block`` video frames with
    25 audio frames each (a short last block gets the proportional share)."""
    if num_frame_per_block_first > 0:
        if total_video_latent_frames < num_frame_per_block_first:
            raise AssertionError(f"{total_video_latent_frames} frames < first block "
                                 f"{num_frame_per_block_first}")
        out = [(0, 0, num_frame_per_block_first, 0, AUDIO_FRAMES_FIRST_BLOCK)]
    else:
        if total_video_latent_frames < 1:
            raise AssertionError("need at least one video frame")
        out = [(0, 0, 1, 0, 1)]
    b, v, a = 1, out[0][2], out[0][4]
    while v < total_video_latent_frames:
        ve = min(v + num_frame_per_block, total_video_latent_frames)
        n = ve - v
        ae = a + (AUDIO_FRAMES_PER_BLOCK if n == num_frame_per_block
                  else AUDIO_FRAMES_PER_BLOCK * n // num_frame_per_block)
        out.append((b, v, ve, a, ae))
        b, v, a = b + 1, ve, ae
    return out


def refresh_blocks(segments: List[Dict[str, int]], prefix_frames: int, next_frames: int,
                   num_frame_per_block: int = 3, num_frame_per_block_first: int = 4):
    """The retained prefix blocks whose K/V a prompt change re-prefills, one
    per retained segment in order (streaming_runtime.py:1037-1075,
    runtime.py:398-419): the local sink block when the cache keeps the sink,
    then the newest warm blocks of the retained latent prefix."""
    if not segments:
        raise RuntimeError("Selective KV rebuild requires committed segment metadata")
    blocks = compute_av_blocks(prefix_frames + next_frames, num_frame_per_block,
                               num_frame_per_block_first)
    prefix = [blk for blk in blocks if blk[2] <= prefix_frames]
    if not prefix:
        raise RuntimeError("Selective KV rebuild received an empty latent prefix")
    has_sink = int(segments[0].get("block_idx", -1)) == 0
    warm = len(segments) - (1 if has_sink else 0)
    candidates = prefix[1:] if has_sink else prefix
    if warm > len(candidates):
        raise ValueError(f"Selective KV rebuild does not have enough retained prefix latents: "
                         f"segments={len(segments)}, warm_needed={warm}, "
                         f"warm_available={len(candidates)}")
    picked = ([prefix[0]] if has_sink else []) + (candidates[-warm:] if warm > 0 else [])
    if len(picked) != len(segments):
        raise RuntimeError("Selective KV latent/segment layout mismatch")
    return picked


def replace_modal_fields(cache: KVCache, rebuilt: KVCache,
                         keep: Tuple[str, ...] = ("video_self",)) -> KVCache:
    """Every cache field except ``keep`` taken from ``rebuilt`` (the
    re-prefilled prompt-sensitive K/V), video self-attention K/V kept
    (runtime.py:458-466): a field swap per layer, no data moves; the segment
    metadata stays attached."""
    if rebuilt is None or len(rebuilt.layers) != len(cache.layers):
        raise RuntimeError("Conditioning cache refresh failed.")
    segments = cache_segments(cache)
    kept = {f + s for f in keep for s in ("_k", "_v")}
    for layer, new in zip(cache.layers, rebuilt.layers):
        for f in LayerKVCache.__dataclass_fields__:
            if f not in kept:
                setattr(layer, f, getattr(new, f))
    return attach_segments(cache, segments)
