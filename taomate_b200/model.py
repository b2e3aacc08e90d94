"""The streaming model forward: patchify, 48 blocks with KV cache, output.

Follows ``model_forward_inference`` (ltx_causal/transformer/kv_cache.py:
2681-3365) for the parts that run per forward:
  * patchify linears (:2772-2779);
  * the RoPE tables (:2906-3000): video 3-D, audio 1-D, the two 1-D cross
    tables, the video cross table expanded per frame token by the table kernel;
  * the 48 ``block_forward_with_cache`` calls (:3220-3300);
  * ``kv_cache_only`` returns after the blocks (:3302-3309);
  * the output LayerNorm + modulation + ``proj_out`` (``_process_output``,
    causal_model.py:568-598).

The conditioning the blocks read (AdaLN rows, text contexts) comes from the
model's timestep embedders and caption projections (:2784-2904), which run
once per forward or once per prompt on a few rows; :class:`Conditioning`
holds them as tensors, per video frame and per audio token (the blocks map
tokens to frames in their kernels).  ``synthetic_conditioning`` makes seeded
random ones of the right shapes.

Sequence parallelism (one process per GPU): the video stream is split by
tokens (each rank holds 1152 / G of a 3-frame chunk and 32 / G heads of the
video self-attention cache, as the reference lays it out, kv_cache.py:
331-339); the 25-token audio stream is replicated (``audio_replicated`` of
``block_forward_with_cache``), so per layer only the video self-attention's
two exchanges and the gather of V2A's partial results (~0.2 MB per rank)
cross NVLink; each rank's V2A cache holds its own video tokens.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Optional, Tuple

import torch
import torch.nn.functional as F
from torch import Tensor

from . import parallel as P
from .block import BlockWeights, block_forward_with_cache, fuse_block_weights, residual_norm
from .block import AdaParams
from .kv_cache import ArenaSpec, KVCache, init_arena_cache
from .profiler import section
from .rope import causal_precompute_freqs_cis


@dataclass
class StreamConfig:
    """Model and stream geometry (LTX-2 19B defaults, ltx_causal/config.py:85-95,
    causal_model.py:100-120; 512x768 video -> 16 x 24 latent tokens per frame,
    25 audio latent tokens per second)."""
    layers: int = 48
    video_dim: int = 4096
    video_heads: int = 32
    video_dim_head: int = 128
    audio_dim: int = 2048
    audio_heads: int = 32
    audio_dim_head: int = 64
    in_channels: int = 128
    frame_h: int = 16
    frame_w: int = 24
    text_tokens: int = 256
    norm_eps: float = 1e-6

    @property
    def frame_tokens(self) -> int:
        return self.frame_h * self.frame_w


class CausalModelWeights(torch.nn.Module):
    """The streaming model's weights under the reference's attribute names
    (CausalLTXModel, ltx_causal/transformer/causal_model.py:230-395):
    ``transformer_blocks``, ``patchify_proj``, ``audio_patchify_proj``,
    ``scale_shift_table`` / ``audio_scale_shift_table`` (2 x D, output
    modulation), ``proj_out`` / ``audio_proj_out``; random N(0, std)."""

    def __init__(self, cfg: StreamConfig, device=None, std: float = 0.02, fuse_qkv: bool = True):
        super().__init__()
        kw = dict(device=device, dtype=torch.bfloat16)
        self.cfg = cfg
        self.transformer_blocks = torch.nn.ModuleList([
            BlockWeights(cfg.video_dim, cfg.video_heads, cfg.video_dim_head, cfg.audio_dim,
                         cfg.audio_heads, cfg.audio_dim_head, norm_eps=cfg.norm_eps,
                         device=device, std=std) for _ in range(cfg.layers)])
        if fuse_qkv:
            for b in self.transformer_blocks:
                fuse_block_weights(b)
        self.patchify_proj = torch.nn.Linear(cfg.in_channels, cfg.video_dim, **kw)
        self.audio_patchify_proj = torch.nn.Linear(cfg.in_channels, cfg.audio_dim, **kw)
        self.proj_out = torch.nn.Linear(cfg.video_dim, cfg.in_channels, **kw)
        self.audio_proj_out = torch.nn.Linear(cfg.audio_dim, cfg.in_channels, **kw)
        self.scale_shift_table = torch.nn.Parameter(torch.empty(2, cfg.video_dim, **kw))
        self.audio_scale_shift_table = torch.nn.Parameter(torch.empty(2, cfg.audio_dim, **kw))
        with torch.no_grad():
            for m in (self.patchify_proj, self.audio_patchify_proj, self.proj_out,
                      self.audio_proj_out):
                m.weight.normal_(0.0, std)
                m.bias.normal_(0.0, std)
            self.scale_shift_table.normal_(0.0, std)
            self.audio_scale_shift_table.normal_(0.0, std)
        for p in self.parameters():
            p.requires_grad_(False)


@dataclass
class Conditioning:
    """Per-forward inputs of the blocks besides the latents.  AdaLN rows per
    video frame ``[1, F, n * Dv]`` and per audio token ``[1, La, n * Da]``;
    ``*_emb2`` are the output modulation rows (the embedded timestep twice,
    shift and scale read the same row, causal_model.py:590-594); contexts are
    the projected text ``[1, 256, D]``; ``pe`` holds the four RoPE tables of
    this rank's tokens."""
    video_ts: Tensor
    audio_ts: Tensor
    video_cross_ss: Tensor
    video_cross_gate: Tensor
    audio_cross_ss: Tensor
    audio_cross_gate: Tensor
    video_emb2: Tensor
    audio_emb2: Tensor
    video_ctx: Tensor
    audio_ctx: Tensor
    pe: Tuple = ()
    video_mask: Optional[Tensor] = None
    audio_mask: Optional[Tensor] = None


def synthetic_conditioning(cfg: StreamConfig, frames: int, audio_tokens: int, device,
                           generator: torch.Generator, scale: float = 0.1) -> Conditioning:
    """Seeded random conditioning of the right shapes: AdaLN rows ~ N(0,
    scale^2), text contexts ~ N(0, 1) (the prompt embeddings after the caption
    projection)."""
    Dv, Da = cfg.video_dim, cfg.audio_dim
    r = lambda *s, sc=scale: (torch.randn(*s, device=device, generator=generator) * sc).to(
        torch.bfloat16)
    ve, ae = r(1, frames, Dv), r(1, audio_tokens, Da)
    return Conditioning(
        video_ts=r(1, frames, 6 * Dv), audio_ts=r(1, audio_tokens, 6 * Da),
        video_cross_ss=r(1, frames, 4 * Dv), video_cross_gate=r(1, frames, Dv),
        audio_cross_ss=r(1, audio_tokens, 4 * Da), audio_cross_gate=r(1, audio_tokens, Da),
        video_emb2=torch.cat([ve, ve], -1), audio_emb2=torch.cat([ae, ae], -1),
        video_ctx=r(1, cfg.text_tokens, Dv, sc=1.0), audio_ctx=r(1, cfg.text_tokens, Da, sc=1.0))


def rope_tables(cfg: StreamConfig, frames: int, audio_tokens: int, video_start: int,
                audio_start: int, device, token_slice: Optional[slice] = None):
    """``(video_pe, audio_pe, video_cross_pe, audio_cross_pe)`` as
    model_forward_inference builds them (kv_cache.py:2906-3000), bf16; the video
    tables restricted to ``token_slice`` (this rank's tokens)."""
    kw = dict(device=device, dtype=torch.bfloat16)
    ia = cfg.audio_heads * cfg.audio_dim_head
    vpe = causal_precompute_freqs_cis(torch.tensor([[frames, cfg.frame_h, cfg.frame_w]]),
                                      cfg.video_heads * cfg.video_dim_head,
                                      start_frame=video_start,
                                      num_attention_heads=cfg.video_heads, **kw)
    ape = causal_precompute_freqs_cis(torch.tensor([[audio_tokens]]), ia, max_pos=[20],
                                      start_frame=audio_start, is_audio=True,
                                      num_attention_heads=cfg.audio_heads, **kw)
    vcpe = causal_precompute_freqs_cis(torch.tensor([[frames]]), ia, max_pos=[20],
                                       start_frame=video_start, num_attention_heads=cfg.audio_heads,
                                       repeat_per_frame=cfg.frame_tokens, **kw)
    acpe = ape  # the audio cross table is the audio self table at audio_cross_attention_dim
    if token_slice is not None:
        cut = lambda t: tuple(x[:, :, token_slice].contiguous() for x in t)
        vpe, vcpe = cut(vpe), cut(vcpe)
    return vpe, ape, vcpe, acpe


def arena_cache(cfg: StreamConfig, video_rows: int, audio_rows: int, sp: int = 1,
                slots: int = 6, device=None) -> KVCache:
    """Empty per-layer slot arenas for the four cache pairs: video self-attention
    head-sharded over the ``sp`` ranks (reference layout), audio self-attention
    and A2V (audio keys) with all heads (the audio stream is replicated), V2A
    (video keys) with all heads for this rank's 1 / ``sp`` of the video
    tokens (the split-key V2A)."""
    if video_rows % sp:
        raise ValueError(f"{video_rows} video rows do not split over {sp} ranks")
    specs = {
        "video_self": ArenaSpec(slots, video_rows, cfg.video_heads // sp, cfg.video_dim_head),
        "audio_self": ArenaSpec(slots, audio_rows, cfg.audio_heads, cfg.audio_dim_head),
        "a2v": ArenaSpec(slots, audio_rows, cfg.audio_heads, cfg.audio_dim_head),
        "v2a": ArenaSpec(slots, video_rows // sp, cfg.audio_heads, cfg.audio_dim_head),
    }
    return init_arena_cache(cfg.layers, specs, device=device)


def _output(x: Tensor, table: Tensor, emb2: Tensor, proj: torch.nn.Linear, frame_seqlen: int,
            offset: int, eps: float) -> Tensor:
    """LayerNorm (no affine) * (1 + scale) + shift, then ``proj_out``
    (causal_model.py:590-598)."""
    B, L, D = (int(v) for v in x.shape)
    prm = AdaParams(table, emb2, L, 2, D, frame_seqlen, offset)
    h = torch.empty_like(x)
    residual_norm(x, outs=[(h, prm, 1, 0)], norm="layer", eps=eps)
    return F.linear(h, proj.weight, proj.bias)


def model_forward(model: CausalModelWeights, video_tokens: Tensor, audio_tokens: Tensor,
                  cond: Conditioning, cache: KVCache, kv_cache_only: bool = False,
                  video_token_offset: int = 0, overlap_audio: bool = True):
    """One forward over a chunk: ``video_tokens [1, Lv_local, C]`` (this rank's
    tokens of the chunk's patchified latents), ``audio_tokens [1, La, C]``
    (all of them).  Returns ``(video_out, audio_out, new_cache)`` with
    ``new_cache`` holding the chunk's K/V appended to every field (the denoise
    forwards drop it, the commit forward keeps it: model_runtime.py:847-895,
    model.py:88-129); with ``kv_cache_only`` the outputs are None.
    ``overlap_audio``: run each block's audio chain on a second stream."""
    cfg = model.cfg
    fs = cfg.frame_tokens
    vpe, ape, vcpe, acpe = cond.pe
    sp = P.is_sp_enabled()
    with section("model.patchify"):
        vx = F.linear(video_tokens, model.patchify_proj.weight, model.patchify_proj.bias)
        ax = F.linear(audio_tokens, model.audio_patchify_proj.weight,
                      model.audio_patchify_proj.bias)
    layers = []
    for i, blk in enumerate(model.transformer_blocks):
        vx, ax, lc = block_forward_with_cache(
            blk, vx, ax, cond.video_ts, cond.audio_ts, vpe, ape, vcpe, acpe, cond.video_ctx,
            cond.audio_ctx, cond.video_mask, cond.audio_mask, cond.video_cross_ss,
            cond.video_cross_gate, cond.audio_cross_ss, cond.audio_cross_gate, None, None,
            None, None, cache.layers[i], layer_idx=i, video_frame_seqlen=fs,
            audio_frame_seqlen=1, video_token_offset=video_token_offset,
            audio_replicated=sp, overlap_audio=overlap_audio)
        layers.append(lc)
    new_cache = KVCache(layers=layers)
    if hasattr(cache, "segments"):
        new_cache.segments = [dict(s) for s in cache.segments]
    if kv_cache_only:
        return None, None, new_cache
    with section("model.output"):
        v_out = _output(vx, model.scale_shift_table, cond.video_emb2, model.proj_out, fs,
                        video_token_offset, cfg.norm_eps)
        a_out = _output(ax, model.audio_scale_shift_table, cond.audio_emb2,
                        model.audio_proj_out, 1, 0, cfg.norm_eps)
    return v_out, a_out, new_cache
