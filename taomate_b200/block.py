"""One transformer block of the causal LTX audio-video model with KV cache.

``block_forward_with_cache`` has the signature and return contract of
``ltx_causal/transformer/kv_cache.py:2145-2654``: video self-attention, video
text cross-attention, audio self-attention, audio text cross-attention, the
A2V / V2A cross-modal pair, the video and audio FFNs, each behind its AdaLN
modulation and gated residual, then the cache update.  ``block`` is the
reference's ``CausalAVTransformerBlock`` or :class:`BlockWeights` (same
attribute names).

What runs where:
  * attentions: :func:`taomate_b200.attention.attention_with_cache` /
    ``text_cross_attention_with_kv_cache`` (tcgen05 attention kernel, fused
    q/k norm + RoPE, slot-arena caches);
  * every norm, modulation and gated residual: ``tm_residual_norm``, one pass
    per token row that adds the previous sublayer's gated output into the
    residual stream and writes the next sublayer's modulated input (up to two
    of them: the cross-modal pair reads two modulations of one norm);
  * FFN: the two linears through cuBLAS (torch), the tanh GELU in the
    first one's epilogue (``tm_gelu_tanh`` in place when it has no bias).

AdaLN parameters come as the reference passes them (per token, ``[B, L, n *
D]``) or per frame (``[B, F, n * D]`` with ``video_frame_seqlen`` /
``audio_frame_seqlen`` tokens per frame, and ``video_token_offset`` /
``audio_token_offset`` giving the first local token's index under sequence
parallelism): the kernel maps each token to its frame's row, so the per-token
expansion (kv_cache.py:2970, 56 MB per forward at C2) is never built.

Out of scope (raise ``NotImplementedError``): pyramid KV selection and the
learned-memory adapters, which no shipped inference config enables.
"""

from __future__ import annotations

import contextlib
from typing import Optional, Tuple

import torch
import torch.nn.functional as F
from torch import Tensor

from . import _lib
from . import parallel as P
from .attention import (AttentionWeights, _cache_source, _norm_eps, attention_with_cache,
                        cross_attention_local, flash_attention, kv_projection,
                        text_cross_attention_with_kv_cache)
from .kv_cache import LayerKVCache, _cat_cache
from .profiler import section
from .rope import norm_rope

# get_ada_values slices (causal_block.py:434-452): (shift, scale, gate) per sublayer
_MSA = (0, 1, 2)
_MLP = (3, 4, 5)
_TEXT_Q = (6, 7, 8)  # cross_attention_adaln only


class AdaParams:
    """AdaLN parameter source ``table[p] + ts[row(t), p]`` for the kernel:
    ``ts`` is ``[B, T, n * D]`` with one row per token (T = L), per frame
    (``div`` tokens per row, first local token ``offset``) or one row for
    all tokens."""

    __slots__ = ("table", "ts", "div", "offset", "keep")

    def __init__(self, table: Optional[Tensor], ts: Optional[Tensor], L: int, n: int, D: int,
                 frame_seqlen: Optional[int] = None, offset: int = 0):
        keep = []
        if table is not None:
            if table.dim() != 2 or table.shape[1] != D or table.shape[0] < n:
                raise ValueError(f"AdaLN table {tuple(table.shape)} does not hold {n} x {D}")
            table = table.detach()
            if table.dtype != torch.bfloat16 or not table.is_contiguous():
                table = table.to(torch.bfloat16).contiguous()
            keep.append(table)
        if ts is not None:
            if ts.dim() == 2:
                ts = ts[:, None]
            if ts.dim() != 3 or ts.shape[2] != n * D:
                raise ValueError(f"AdaLN timestep {tuple(ts.shape)} is not [B, T, {n} * {D}]")
            if ts.dtype != torch.bfloat16 or ts.stride(2) != 1 or ts.stride(1) % 8 or \
                    (ts.shape[0] > 1 and ts.stride(0) % 8) or ts.data_ptr() % 16:
                ts = ts.to(torch.bfloat16).contiguous()
            keep.append(ts)
            T = int(ts.shape[1])
            if T == L and offset == 0:
                div = 1
            elif T == 1:
                div, offset = max(L + offset, 1), 0
            else:
                if not frame_seqlen:
                    raise ValueError(f"{T} AdaLN rows for {L} tokens need the tokens per frame")
                div = int(frame_seqlen)
                if (L + offset + div - 1) // div > T:
                    raise ValueError(f"{T} AdaLN rows do not cover tokens {offset}..{offset + L}")
        else:
            div = 1
        self.table, self.ts, self.div, self.offset, self.keep = table, ts, div, int(offset), keep

    def source(self) -> "_lib.AdaSource":
        s = _lib.AdaSource()
        if self.table is not None:
            s.table = self.table.data_ptr()
        if self.ts is not None:
            s.ts = self.ts.data_ptr()
            s.ts_batch_stride = self.ts.stride(0) if self.ts.shape[0] > 1 else 0
            s.ts_row_stride = self.ts.stride(1)
        s.ts_row_div, s.ts_row_offset = self.div, self.offset
        return s


def residual_norm(x: Tensor, y: Optional[Tensor] = None, gate: Optional[AdaParams] = None,
                  gate_index: int = -1, x_out: Optional[Tensor] = None,
                  outs=(), norm: str = "rms", eps: float = 1e-6) -> None:
    """One launch of ``tm_residual_norm`` over ``[B, L, D]`` bf16 rows:
    ``r = x + y * gate[gate_index]`` (stored to ``x_out``), then for each
    ``(out, params, scale_index, shift_index)`` of ``outs``:
    ``out = norm(r) * (1 + scale) + shift`` (``params`` None: ``norm(r)``)."""
    dev = _lib.require_cuda(x, y, x_out)
    B, L, D = (int(v) for v in x.shape)
    for t in (x, y, x_out):
        if t is not None and (t.dtype != torch.bfloat16 or t.stride(2) != 1 or
                              tuple(t.shape) != (B, L, D)):
            raise ValueError(f"residual_norm: expected [{B}, {L}, {D}] bf16 rows, got "
                             f"{tuple(t.shape)} {t.dtype}")
    arr = (_lib.NormOutput * 2)()
    for k, (o, prm, si, hi) in enumerate(outs):
        if o.dtype != torch.bfloat16 or tuple(o.shape) != (B, L, D) or o.stride(2) != 1:
            raise ValueError("residual_norm: outputs must be [B, L, D] bf16 rows")
        arr[k].out = o.data_ptr()
        arr[k].batch_stride, arr[k].row_stride = o.stride(0), o.stride(1)
        if prm is not None:
            arr[k].mod = prm.source()
            arr[k].scale_index, arr[k].shift_index = int(si), int(hi)
        else:
            arr[k].scale_index = arr[k].shift_index = -1
    gsrc = gate.source() if gate is not None else None
    st = lambda t: (t.stride(0), t.stride(1)) if t is not None else (0, 0)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().tm_residual_norm(
            x.data_ptr(), *st(x), y.data_ptr() if y is not None else None, *st(y),
            gsrc if gsrc is not None else None, int(gate_index) if gate is not None else -1,
            x_out.data_ptr() if x_out is not None else None, *st(x_out), arr, len(outs),
            1 if norm == "layer" else 0, B, L, D, float(eps), _lib.stream_ptr(dev)),
            "residual_norm")
        _lib.launched()


def gelu_tanh_(x: Tensor) -> Tensor:
    """In-place tanh GELU (``tm_gelu_tanh``) of a contiguous bf16 tensor."""
    dev = _lib.require_cuda(x)
    if x.dtype != torch.bfloat16 or not x.is_contiguous():
        raise ValueError("gelu_tanh_ takes a contiguous bf16 tensor")
    with torch.cuda.device(dev):
        _lib.check(_lib.load().tm_gelu_tanh(x.data_ptr(), x.numel(), _lib.stream_ptr(dev)),
                   "gelu_tanh")
        _lib.launched()
    return x


_ADDMM_GELU = getattr(torch, "_addmm_activation", None)


def feed_forward(ff, x: Tensor) -> Tensor:
    """``FeedForward`` (ltx_causal/transformer/compat.py:47-70): Linear ->
    tanh GELU -> Linear, both linears through cuBLAS.  With a bias the GELU
    runs in the first GEMM's epilogue (cuBLASLt GELU_BIAS, the tanh form, on
    the fp32 accumulator: one bf16 rounding instead of two, and the hidden
    rows are written once instead of written, read and written again);
    without one, ``tm_gelu_tanh`` in place."""
    proj = ff.net[0].proj
    x2 = x.reshape(-1, x.shape[-1])
    # torch._addmm_activation is torch's own (private) entry to the epilogue;
    # a torch without it takes the unfused path
    if _ADDMM_GELU is not None and proj.bias is not None and x2.is_contiguous() and \
            x2.shape[0] > 1 and proj.bias.dtype == x.dtype == proj.weight.dtype:
        h = _ADDMM_GELU(proj.bias, x2, proj.weight.t(), use_gelu=True)
        h = h.view(*x.shape[:-1], h.shape[-1])
    else:
        h = F.linear(x, proj.weight, proj.bias)
        gelu_tanh_(h)
    out = ff.net[2]
    return F.linear(h, out.weight, out.bias)


_V2A_MAX_PARTS = 8


def v2a_gather_bytes(audio_tokens: int, heads: int, dim_head: int, sp: int) -> int:
    """Bytes of one gather buffer of the split-key V2A for up to
    ``audio_tokens`` audio queries on ``sp`` ranks (for
    ``parallel.init_peer_exchange(gather_bytes=)``)."""
    from .attention import partial_bytes
    splits = max(1, _V2A_MAX_PARTS // sp)
    return sp * partial_bytes(1, audio_tokens, heads, dim_head, splits)


def video_to_audio_split_keys(attn, ax_v2a: Tensor, vx_v2a: Tensor, audio_cross_pe,
                              video_cross_pe, cached_k, cached_v,
                              video_real_len: Optional[int] = None,
                              layer_idx: Optional[int] = None, kv=None):
    """V2A attention (audio queries over video keys) when the audio stream is
    replicated on every rank and the video stream is split by sequence.

    The reference moves Q, K and V seq->head and the output head->seq
    (kv_cache.py:1432-1462, 1535-1538) over audio tokens padded to the rank
    count, so every rank attends its heads over all video keys.  Here the
    keys stay where they were made: each rank projects its own video tokens'
    K/V (norm + cross RoPE fused) and attends the 25 audio queries, all heads,
    over its own cached and new video keys, exporting per key range the
    normalised fp32 output and its (max, sum) (tm_attention_fwd_ext with
    parts, ~0.2 MB); one all-gather of those parts, and every rank merges all
    ranks' parts in the same order (tm_attention_combine, the per-head gate
    fused), so the output is the same softmax over all keys and the same bits
    on every rank.  The all-gather is a copy into every peer's buffer over
    NVLink plus a bounded flag handshake when the peer exchange holds gather
    buffers (the buffer alternates with ``layer_idx``), NCCL otherwise.  The
    V2A cache of each rank holds its own video tokens (all heads); this call
    returns those new K/V.  ``kv``: this rank's K/V already projected
    (:func:`taomate_b200.attention.kv_projection`); ``vx_v2a`` is then unused."""
    import torch.distributed as dist
    from .attention import combine_partials, partial_bytes, partial_splits
    G, grp, r = P.get_sp_world_size(), P.get_sp_group(), P.get_sp_rank()
    H, D = int(attn.heads), int(attn.dim_head)
    src = kv[0] if kv is not None else vx_v2a
    B, Lloc, La = int(src.shape[0]), int(src.shape[1]), int(ax_v2a.shape[1])
    if B != 1:
        raise NotImplementedError("the split-key V2A path takes batch 1")
    eps = _norm_eps(attn.q_norm)
    with section("video_to_audio.qkv_proj_norm"):
        q = F.linear(ax_v2a, attn.to_q.weight, attn.to_q.bias)
        if kv is None:
            k, v = kv_projection(attn, vx_v2a, video_cross_pe, eps)
        else:
            k, v = kv
    with section("video_to_audio.rope_reshape"):
        (q,) = norm_rope([q], [attn.q_norm.weight], [audio_cross_pe], H, D, eps)
    n = Lloc  # this rank's real video rows of the chunk
    if video_real_len is not None:
        n = max(0, min(Lloc, int(video_real_len) - r * Lloc))
    k, v = k[:, :n], v[:, :n]
    ck, cv, spans = _cache_source(cached_k, cached_v)
    cached = sum(int(rows) for _, rows in spans)
    # the same number of key ranges on every rank (ranks hold equal cache rows)
    # at most 8 parts in all: past that, moving the parts costs more than the
    # key-range split saves
    splits = min(partial_splits(B, La, H, D, cached + Lloc), max(1, _V2A_MAX_PARTS // G))
    pb = partial_bytes(B, La, H, D, splits)
    peer = P.get_peer_exchange()
    gathered = peer.gather_buffer(layer_idx or 0, pb) if peer is not None else None
    if gathered is None:
        peer = None
        gathered = torch.empty(G * pb, dtype=torch.uint8, device=q.device)
    own = gathered[r * pb:(r + 1) * pb]
    with section("video_to_audio.sdpa"):
        if cached + n == 0:
            # no keys on this rank: a part of weight zero, (max, sum) = (-inf, 0)
            rows = splits * B * La * H
            off = (rows * D * 4 + 255) // 256 * 256
            own.zero_()
            ml = own[off:off + rows * 8].view(torch.float32).view(rows, 2)
            ml[:, 0] = float("-inf")
        else:
            flash_attention(q, ck, cv, spans, k, v, n, parts=own, part_splits=splits)
    with section("video_to_audio.all_gather"):
        if peer is not None:
            peer.all_gather_parts(gathered, pb)  # NVLink copies + a bounded handshake
        else:
            dist.all_gather_into_tensor(gathered, own, group=grp)
    with section("video_to_audio.combine"):
        glog = None
        if getattr(attn, "to_gate_logits", None) is not None:
            glog = attn.to_gate_logits(ax_v2a)
        out = combine_partials(gathered, G, pb, splits, B, La, H, D, gate_logits=glog)
    with section("video_to_audio.out_proj"):
        out = attn.to_out(out.view(B, La, H * D))
    return out, k, v


_AUDIO_STREAMS = {}


def _audio_stream(dev: torch.device) -> torch.cuda.Stream:
    st = _AUDIO_STREAMS.get(dev.index)
    if st is None:
        st = _AUDIO_STREAMS[dev.index] = torch.cuda.Stream(dev)
    return st


def _ada(table, ts, L, n, D, frame_seqlen, offset):
    return AdaParams(table, ts, L, n, D, frame_seqlen, offset)


def _text_input(block, x: Tensor, src: AdaParams, eps: float) -> Tensor:
    """Query input of the text cross-attention: ``rms_norm(x)``, modulated by
    the (shift, scale) of slice 6:9 under ``cross_attention_adaln``
    (kv_cache.py:874-901)."""
    out = torch.empty_like(x)
    if block.cross_attention_adaln:
        residual_norm(x, outs=[(out, src, _TEXT_Q[1], _TEXT_Q[0])], eps=eps)
    else:
        residual_norm(x, outs=[(out, None, -1, -1)], eps=eps)
    return out


def _text_context(block, context: Tensor, prompt_table, prompt_ts) -> Tensor:
    """``context * (1 + scale_kv) + shift_kv`` under ``cross_attention_adaln``
    (kv_cache.py:888-899); the context itself otherwise."""
    if not block.cross_attention_adaln:
        return context
    B = context.shape[0]
    sv = (prompt_table[None, None].to(device=context.device, dtype=context.dtype)
          + prompt_ts.reshape(B, prompt_ts.shape[1], 2, -1))
    shift_kv, scale_kv = sv.unbind(dim=2)
    return context * (1 + scale_kv) + shift_kv


def block_forward_with_cache(
    block,
    video_x: Tensor,
    audio_x: Tensor,
    video_timestep_6d: Tensor,
    audio_timestep_6d: Tensor,
    video_pe: Tuple[Tensor, Tensor],
    audio_pe: Tuple[Tensor, Tensor],
    video_cross_pe: Tuple[Tensor, Tensor],
    audio_cross_pe: Tuple[Tensor, Tensor],
    video_ctx: Tensor,
    audio_ctx: Tensor,
    video_context_mask: Optional[Tensor],
    audio_context_mask: Optional[Tensor],
    video_cross_ss: Tensor,
    video_cross_gate: Tensor,
    audio_cross_ss: Tensor,
    audio_cross_gate: Tensor,
    video_prompt_ts: Optional[Tensor],
    audio_prompt_ts: Optional[Tensor],
    video_prompt_cache_key=None,
    audio_prompt_cache_key=None,
    layer_cache: Optional[LayerKVCache] = None,
    video_memory: Optional[Tensor] = None,
    audio_memory: Optional[Tensor] = None,
    color_memory: Optional[Tensor] = None,
    pyramid_policy=None,
    layer_idx: Optional[int] = None,
    video_frame_seqlen: Optional[int] = None,
    audio_frame_seqlen: Optional[int] = None,
    video_real_len: Optional[int] = None,
    audio_real_len: Optional[int] = None,
    *,
    video_token_offset: int = 0,
    audio_token_offset: int = 0,
    audio_replicated: bool = False,
    overlap_audio: bool = True,
) -> Tuple[Tensor, Tensor, LayerKVCache]:
    """One block forward with KV cache (kv_cache.py:2145-2654); returns
    ``(video_x, audio_x, updated_layer_cache)``.  The inputs are not
    modified.

    Under sequence parallelism the video stream is this rank's token shard
    (``video_token_offset`` = its first token).  The audio stream is split
    the same way (the reference's layout) unless ``audio_replicated``: then
    every rank holds all audio tokens, the audio sublayers and A2V run
    locally with all heads, V2A attends over each rank's own video keys and
    merges the ranks' partial results (:func:`video_to_audio_split_keys`);
    the audio and A2V caches hold all heads, the V2A cache this rank's video
    tokens with all heads.  ``overlap_audio`` runs the audio chain on a second stream
    beside the video chain (same kernels, same results)."""
    if pyramid_policy is not None:
        raise NotImplementedError("pyramid KV selection is disabled in every shipped config")
    if getattr(block, "learned_memory_mode", None) is not None:
        raise NotImplementedError("learned-memory adapters are not on this path")
    if layer_cache is None:
        layer_cache = LayerKVCache()
    eps = float(block.norm_eps)
    B, Lv, Dv = (int(v) for v in video_x.shape)
    La, Da = int(audio_x.shape[1]), int(audio_x.shape[2])
    n_ada = int(block.scale_shift_table.shape[0])
    vsrc = _ada(block.scale_shift_table, video_timestep_6d, Lv, n_ada, Dv, video_frame_seqlen,
                video_token_offset)
    asrc = _ada(block.audio_scale_shift_table, audio_timestep_6d, La, n_ada, Da,
                audio_frame_seqlen, audio_token_offset)

    # Two chains meet only at the cross-modal norms: the video chain (self,
    # text, A2V, FFN) runs on the current stream, the audio chain (self, text,
    # V2A, FFN: 25-token kernels bound by latency and weight reads) on a side
    # stream beside it, inside a captured graph too.  Every tensor either
    # chain touches stays referenced until the streams join at the end.
    main = torch.cuda.current_stream(video_x.device)
    side = _audio_stream(video_x.device) if overlap_audio else main
    side.wait_stream(main)
    audio_local = audio_replicated and P.is_sp_enabled()
    local = P.sp_local if audio_local else contextlib.nullcontext

    # ── audio self-attention (kv_cache.py:2464-2490) + audio text cross (:2493-2510)
    with torch.cuda.stream(side):
        with section("block.audio_norm"):
            norm_ax = torch.empty_like(audio_x)
            residual_norm(audio_x, outs=[(norm_ax, asrc, _MSA[1], _MSA[0])], eps=eps)
        with local():
            ax_attn, new_as_k, new_as_v = attention_with_cache(
                block.audio_attn1, norm_ax, None, audio_pe, None, layer_cache.audio_self_k,
                layer_cache.audio_self_v, layer_idx=layer_idx, modality="audio",
                frame_seqlen=audio_frame_seqlen, new_kv_real_len=audio_real_len,
                profile_name="audio_self")
        ax = torch.empty_like(audio_x)
        atin = torch.empty_like(audio_x)
        with section("block.audio_norm"):
            if block.cross_attention_adaln:
                residual_norm(audio_x, ax_attn, asrc, _MSA[2], ax,
                              [(atin, asrc, _TEXT_Q[1], _TEXT_Q[0])], eps=eps)
            else:
                residual_norm(audio_x, ax_attn, asrc, _MSA[2], ax, [(atin, None, -1, -1)],
                              eps=eps)
        a_ctx = _text_context(block, audio_ctx,
                              getattr(block, "audio_prompt_scale_shift_table", None),
                              audio_prompt_ts)
        a_text = text_cross_attention_with_kv_cache(
            block.audio_attn2, atin, a_ctx, mask=audio_context_mask, base_context=audio_ctx,
            prompt_cache_key=audio_prompt_cache_key, cache_name="audio_text_cross",
            layer_idx=layer_idx)

    # ── video self-attention (kv_cache.py:2197-2218)
    with section("block.video_norm"):
        norm_vx = torch.empty_like(video_x)
        residual_norm(video_x, outs=[(norm_vx, vsrc, _MSA[1], _MSA[0])], eps=eps)
    vx_attn, new_vs_k, new_vs_v = attention_with_cache(
        block.attn1, norm_vx, None, video_pe, None, layer_cache.video_self_k,
        layer_cache.video_self_v, layer_idx=layer_idx, modality="video",
        frame_seqlen=video_frame_seqlen, new_kv_real_len=video_real_len,
        profile_name="video_self")
    # residual (gate of 0:3) + the text cross-attention's query input
    vx = torch.empty_like(video_x)
    tin = torch.empty_like(video_x)
    with section("block.video_norm"):
        if block.cross_attention_adaln:
            residual_norm(video_x, vx_attn, vsrc, _MSA[2], vx,
                          [(tin, vsrc, _TEXT_Q[1], _TEXT_Q[0])], eps=eps)
        else:
            residual_norm(video_x, vx_attn, vsrc, _MSA[2], vx, [(tin, None, -1, -1)], eps=eps)
    # ── video text cross-attention (kv_cache.py:2441-2460, 1090-1139)
    v_ctx = _text_context(block, video_ctx, getattr(block, "prompt_scale_shift_table", None),
                          video_prompt_ts)
    v_text = text_cross_attention_with_kv_cache(
        block.attn2, tin, v_ctx, mask=video_context_mask, base_context=video_ctx,
        prompt_cache_key=video_prompt_cache_key, cache_name="video_text_cross",
        layer_idx=layer_idx)

    # the text cross residuals (gate 6:9 under cross_attention_adaln, none
    # otherwise), fused with the norms that follow
    tgate_v = vsrc if block.cross_attention_adaln else None
    tgate_a = asrc if block.cross_attention_adaln else None
    new_a2v_k = new_a2v_v = new_v2a_k = new_v2a_v = None
    ffin_v = torch.empty_like(video_x)
    ffin_a = torch.empty_like(audio_x)
    cross = not getattr(block, "skip_cross_modal_attention", False)
    # one GPU, or replicated audio under sequence parallelism: the pair runs
    # without exchanges inside it except V2A's gather of partial results
    split_chains = audio_local or not P.is_sp_enabled()
    if cross:
        # ── A2V / V2A (kv_cache.py:2512-2598): norm3 of both streams and the
        # four modulated inputs, from get_av_ca_ada_values (causal_block.py:454-478):
        # table[:4] + cross_ss -> (scale_a2v, shift_a2v, scale_v2a, shift_v2a),
        # table[4:] + cross_gate -> gate
        vca = _ada(block.scale_shift_table_a2v_ca_video[:4], video_cross_ss, Lv, 4, Dv,
                   video_frame_seqlen, video_token_offset)
        aca = _ada(block.scale_shift_table_a2v_ca_audio[:4], audio_cross_ss, La, 4, Da,
                   audio_frame_seqlen, audio_token_offset)
        vg = _ada(block.scale_shift_table_a2v_ca_video[4:], video_cross_gate, Lv, 1, Dv,
                  video_frame_seqlen, video_token_offset)
        ag = _ada(block.scale_shift_table_a2v_ca_audio[4:], audio_cross_gate, La, 1, Da,
                  audio_frame_seqlen, audio_token_offset)
        vx_a2v, vx_v2a = torch.empty_like(video_x), torch.empty_like(video_x)
        ax_a2v, ax_v2a = torch.empty_like(audio_x), torch.empty_like(audio_x)
    if cross and split_chains:
        # Each chain normalises its own stream and projects the keys and values
        # that the other chain's attention reads (V2A's from the video tokens on
        # the video chain, A2V's from the audio tokens on the audio chain); a
        # chain waits for the other only where that attention starts.
        a2v, v2a = block.audio_to_video_attn, block.video_to_audio_attn
        with section("block.video_norm"):
            residual_norm(vx, v_text, tgate_v, _TEXT_Q[2], vx,
                          [(vx_a2v, vca, 0, 1), (vx_v2a, vca, 2, 3)], eps=eps)
        with section("video_to_audio.kv_proj_norm"):
            v2a_kv = kv_projection(v2a, vx_v2a, video_cross_pe, _norm_eps(v2a.q_norm))
        v2a_ready = torch.cuda.Event()
        v2a_ready.record(main)
        with torch.cuda.stream(side):
            with section("block.audio_norm"):
                residual_norm(ax, a_text, tgate_a, _TEXT_Q[2], ax,
                              [(ax_a2v, aca, 0, 1), (ax_v2a, aca, 2, 3)], eps=eps)
            with section("audio_to_video.kv_proj_norm"):
                a2v_kv = kv_projection(a2v, ax_a2v, audio_cross_pe, _norm_eps(a2v.q_norm))
            a2v_ready = torch.cuda.Event()
            a2v_ready.record(side)
            # audio chain: V2A, gated residual + FFN input (slice 3:6)
            side.wait_event(v2a_ready)
            if audio_local:
                v2a_out, new_v2a_k, new_v2a_v = video_to_audio_split_keys(
                    v2a, ax_v2a, vx_v2a, audio_cross_pe, video_cross_pe, layer_cache.v2a_k,
                    layer_cache.v2a_v, video_real_len, layer_idx, kv=v2a_kv)
            else:
                v2a_out, new_v2a_k, new_v2a_v = cross_attention_local(
                    v2a, ax_v2a, audio_cross_pe, *v2a_kv, layer_cache.v2a_k, layer_cache.v2a_v,
                    video_real_len, "video_to_audio")
            with section("block.audio_norm"):
                residual_norm(ax, v2a_out, ag, 0, ax, [(ffin_a, asrc, _MLP[1], _MLP[0])],
                              eps=eps)
        # video chain: A2V (this rank's video queries over all audio keys), gated
        # residual + FFN input
        main.wait_event(a2v_ready)
        a2v_out, new_a2v_k, new_a2v_v = cross_attention_local(
            a2v, vx_a2v, video_cross_pe, *a2v_kv, layer_cache.a2v_k, layer_cache.a2v_v,
            audio_real_len, "audio_to_video")
        with section("block.video_norm"):
            residual_norm(vx, a2v_out, vg, 0, vx, [(ffin_v, vsrc, _MLP[1], _MLP[0])], eps=eps)
    elif cross:
        # the reference's layout under sequence parallelism (audio split too):
        # both attentions exchange through the group, one after the other
        main.wait_stream(side)
        with section("block.video_norm"):
            residual_norm(vx, v_text, tgate_v, _TEXT_Q[2], vx,
                          [(vx_a2v, vca, 0, 1), (vx_v2a, vca, 2, 3)], eps=eps)
        with section("block.audio_norm"):
            residual_norm(ax, a_text, tgate_a, _TEXT_Q[2], ax,
                          [(ax_a2v, aca, 0, 1), (ax_v2a, aca, 2, 3)], eps=eps)
        v2a_out, new_v2a_k, new_v2a_v = attention_with_cache(
            block.video_to_audio_attn, ax_v2a, vx_v2a, audio_cross_pe, video_cross_pe,
            layer_cache.v2a_k, layer_cache.v2a_v, new_kv_real_len=video_real_len,
            profile_name="video_to_audio")
        with section("block.audio_norm"):
            residual_norm(ax, v2a_out, ag, 0, ax, [(ffin_a, asrc, _MLP[1], _MLP[0])], eps=eps)
        a2v_out, new_a2v_k, new_a2v_v = attention_with_cache(
            block.audio_to_video_attn, vx_a2v, ax_a2v, video_cross_pe, audio_cross_pe,
            layer_cache.a2v_k, layer_cache.a2v_v, new_kv_real_len=audio_real_len,
            profile_name="audio_to_video")
        with section("block.video_norm"):
            residual_norm(vx, a2v_out, vg, 0, vx, [(ffin_v, vsrc, _MLP[1], _MLP[0])], eps=eps)
        side.wait_stream(main)
    else:
        with section("block.video_norm"):
            residual_norm(vx, v_text, tgate_v, _TEXT_Q[2], vx,
                          [(ffin_v, vsrc, _MLP[1], _MLP[0])], eps=eps)
        with torch.cuda.stream(side):
            with section("block.audio_norm"):
                residual_norm(ax, a_text, tgate_a, _TEXT_Q[2], ax,
                              [(ffin_a, asrc, _MLP[1], _MLP[0])], eps=eps)

    # ── FFNs (kv_cache.py:2600-2640)
    with torch.cuda.stream(side):
        with section("block.audio_ff"):
            a_ff = feed_forward(block.audio_ff, ffin_a)
            residual_norm(ax, a_ff, asrc, _MLP[2], ax, eps=eps)
    with section("block.video_ff"):
        v_ff = feed_forward(block.ff, ffin_v)
        residual_norm(vx, v_ff, vsrc, _MLP[2], vx, eps=eps)
    main.wait_stream(side)

    # ── cache update (kv_cache.py:2642-2654)
    keep = lambda old, new: _cat_cache(old, new) if new is not None else old
    updated = LayerKVCache(
        video_self_k=_cat_cache(layer_cache.video_self_k, new_vs_k),
        video_self_v=_cat_cache(layer_cache.video_self_v, new_vs_v),
        audio_self_k=_cat_cache(layer_cache.audio_self_k, new_as_k),
        audio_self_v=_cat_cache(layer_cache.audio_self_v, new_as_v),
        a2v_k=keep(layer_cache.a2v_k, new_a2v_k), a2v_v=keep(layer_cache.a2v_v, new_a2v_v),
        v2a_k=keep(layer_cache.v2a_k, new_v2a_k), v2a_v=keep(layer_cache.v2a_v, new_v2a_v),
    )
    return vx, ax, updated


class _GELUProj(torch.nn.Module):
    def __init__(self, dim_in: int, dim_out: int, **kw):
        super().__init__()
        self.proj = torch.nn.Linear(dim_in, dim_out, bias=True, **kw)


class FeedForwardWeights(torch.nn.Module):
    """``FeedForward`` weights with the reference's state-dict layout
    (``net.0.proj``, ``net.2``; ltx_causal/transformer/compat.py:47-70)."""

    def __init__(self, dim: int, mult: int = 4, **kw):
        super().__init__()
        inner = int(dim * mult)
        self.net = torch.nn.Sequential(_GELUProj(dim, inner, **kw), torch.nn.Identity(),
                                       torch.nn.Linear(inner, dim, bias=True, **kw))


class BlockWeights(torch.nn.Module):
    """Weights of one ``CausalAVTransformerBlock``
    (ltx_causal/transformer/causal_block.py:211-380) under the reference's
    attribute names, random-initialised N(0, std) (no checkpoints here).
    ``cross_attention_adaln`` adds the 9-row tables and the prompt tables."""

    def __init__(self, video_dim: int = 4096, video_heads: int = 32, video_dim_head: int = 128,
                 audio_dim: int = 2048, audio_heads: int = 32, audio_dim_head: int = 64,
                 video_context_dim: Optional[int] = None, audio_context_dim: Optional[int] = None,
                 norm_eps: float = 1e-6, cross_attention_adaln: bool = False, gated: bool = False,
                 device=None, dtype: torch.dtype = torch.bfloat16, std: Optional[float] = 0.02):
        super().__init__()
        kw = dict(device=device, dtype=dtype)
        vctx = video_dim if video_context_dim is None else video_context_dim
        actx = audio_dim if audio_context_dim is None else audio_context_dim
        self.norm_eps = norm_eps
        self.cross_attention_adaln = cross_attention_adaln
        self.skip_cross_modal_attention = False
        self.learned_memory_mode = None
        n_ada = 9 if cross_attention_adaln else 6
        A = lambda q, h, d, c=None, g=gated: AttentionWeights(q, h, d, context_dim=c, gated=g,
                                                              device=device, dtype=dtype, std=std)
        self.attn1 = A(video_dim, video_heads, video_dim_head)
        self.attn2 = A(video_dim, video_heads, video_dim_head, vctx)
        self.ff = FeedForwardWeights(video_dim, **kw)
        self.scale_shift_table = torch.nn.Parameter(torch.empty(n_ada, video_dim, **kw))
        self.audio_attn1 = A(audio_dim, audio_heads, audio_dim_head)
        self.audio_attn2 = A(audio_dim, audio_heads, audio_dim_head, actx)
        self.audio_ff = FeedForwardWeights(audio_dim, **kw)
        self.audio_scale_shift_table = torch.nn.Parameter(torch.empty(n_ada, audio_dim, **kw))
        if cross_attention_adaln:
            self.prompt_scale_shift_table = torch.nn.Parameter(torch.empty(2, video_dim, **kw))
            self.audio_prompt_scale_shift_table = torch.nn.Parameter(
                torch.empty(2, audio_dim, **kw))
        # A2V: queries from video, keys from audio; V2A the reverse (audio head config)
        self.audio_to_video_attn = A(video_dim, audio_heads, audio_dim_head, audio_dim)
        self.video_to_audio_attn = A(audio_dim, audio_heads, audio_dim_head, video_dim)
        self.scale_shift_table_a2v_ca_audio = torch.nn.Parameter(torch.empty(5, audio_dim, **kw))
        self.scale_shift_table_a2v_ca_video = torch.nn.Parameter(torch.empty(5, video_dim, **kw))
        if std is not None:
            with torch.no_grad():
                for m in (self.ff, self.audio_ff):
                    for lin in m.modules():
                        if isinstance(lin, torch.nn.Linear):
                            lin.weight.normal_(0.0, std)
                            lin.bias.normal_(0.0, std)
                for n, p in self.named_parameters(recurse=False):
                    p.normal_(0.0, std)
        for p in self.parameters():
            p.requires_grad_(False)


def fuse_block_weights(block) -> int:
    """``fuse_qkv_weights`` on the block's self-attention modules (one
    projection GEMM per self-attention call) and ``fuse_kv_weights`` on the
    A2V / V2A modules (one GEMM for the keys and values of each); returns how
    many modules were fused."""
    from .attention import fuse_kv_weights, fuse_qkv_weights
    n = sum(bool(fuse_qkv_weights(a)) for a in (block.attn1, block.audio_attn1))
    return n + sum(bool(fuse_kv_weights(a))
                   for a in (block.audio_to_video_attn, block.video_to_audio_attn))
