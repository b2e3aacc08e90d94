"""Streaming attention with KV cache on the sm_100a kernels.

``attention_with_cache`` has the signature and return contract of
``ltx_causal/transformer/kv_cache.py:1148-1547``; ``standard_attention_forward``
that of ``ltx_causal/attention/flex_attention_utils.py:225-276``.

Per call (video self-attention, C2 shapes):
  1. projections ``to_q/to_k/to_v`` (cuBLAS GEMMs through torch; one GEMM
     for a module prepared by ``fuse_qkv_weights``);
  2. ONE fused kernel: q/k RMSNorm over the inner dim + split RoPE (+ the V
     layout copy), storing straight into the Ulysses send buffer when SP is on;
  3. under SP, ONE NCCL all-to-all for Q, K and V together;
  4. ONE attention kernel over [cached spans..., new chunk] read in place
     (slot arena or plain cache tensor; no concatenation);
  5. under SP, the head->seq all-to-all and its unpack;
  6. optional per-head gate and ``to_out`` (torch / cuBLAS).
"""

from __future__ import annotations

import ctypes
from typing import Optional, Sequence, Tuple

import torch
import torch.nn.functional as F
from torch import Tensor

from . import _lib
from . import graphs as _graphs
from . import parallel as P
from .kv_cache import ArenaKV, cache_rows_view
from .profiler import section
from .rope import norm_rope


def _row_strides(t: Tensor, H: int, D: int) -> Tuple[int, int]:
    """(batch, row) element strides of a ``[B, L, H, D]`` tensor with
    contiguous heads."""
    if t.dim() != 4 or t.shape[2] != H or t.shape[3] != D or t.stride(3) != 1 or t.stride(2) != D:
        raise ValueError(f"expected [B, L, {H}, {D}] with contiguous heads, got shape "
                         f"{tuple(t.shape)} strides {t.stride()}")
    return (t.stride(0) if t.shape[0] > 1 else 0), t.stride(1)


def flash_attention(q: Tensor, cache_k: Optional[Tensor], cache_v: Optional[Tensor],
                    cache_spans: Sequence[Tuple[int, int]], new_k: Optional[Tensor],
                    new_v: Optional[Tensor], new_rows: int, scale: Optional[float] = None,
                    out: Optional[Tensor] = None, peer=None,
                    gate_logits: Optional[Tensor] = None, parts: Optional[Tensor] = None,
                    part_splits: int = 1) -> Tensor:
    """``softmax(q K^T * scale) V`` with the keys of ``cache_spans`` (row ranges
    of ``cache_k/v``) followed by the first ``new_rows`` rows of ``new_k/v``.
    All tensors ``[B, L, H, D]`` bf16 with contiguous heads.

    With ``peer`` (a :class:`taomate_b200.parallel.PeerExchange`) the kernel
    stores each output row in its owner rank's ``peer.out`` (the fused
    head->seq exchange); the caller then runs ``peer.exchange(1)`` and reads
    ``peer.out``, which is also what this returns.  ``gate_logits``
    (``[B, Lq, H]`` bf16) multiplies each output row of head h by
    ``2 * sigmoid(logit)`` in the kernel's epilogue.

    With ``parts`` (a uint8 tensor of :func:`partial_bytes`) the call
    stores no output: the keys are divided into ``part_splits`` ranges and
    each range's normalised fp32 output and (max, sum) go to ``parts``, for
    :func:`combine_partials` to merge with other GPUs' parts; returns
    ``parts``."""
    dev = _lib.require_cuda(q, cache_k, new_k)
    B, Lq, H, D = (int(v) for v in q.shape)
    if q.dtype != torch.bfloat16:
        raise TypeError(f"expected bfloat16, got {q.dtype}")
    qbs, qrs = _row_strides(q, H, D)
    ext = _lib.AttentionExt()
    if parts is not None:
        if peer is not None or gate_logits is not None or out is not None:
            raise ValueError("an export of partial results takes no output, peer or gate")
        need = partial_bytes(B, Lq, H, D, part_splits)
        if parts.dtype != torch.uint8 or parts.numel() < need or not parts.is_contiguous():
            raise ValueError(f"parts must be a contiguous uint8 tensor of {need} bytes")
        ext.parts, ext.parts_bytes, ext.part_splits = parts.data_ptr(), parts.numel(), part_splits
        out = parts
        obs, ors = 0, H * D
    elif peer is not None:
        if Lq != peer.sp * peer.S_loc or H != peer.Hl or D != peer.D or B != peer.B:
            raise ValueError("attention output does not match the peer exchange's shapes")
        out = peer.out
        obs, ors = (out.stride(0) if B > 1 else 0), out.stride(1)
        ext.rows_per_rank, ext.head_base = peer.S_loc, peer.rank * peer.Hl
        for i in range(8):
            ext.out_delta[i] = peer.delta["out"][i]
    else:
        if out is None:
            out = torch.empty(B, Lq, H, D, device=dev, dtype=torch.bfloat16)
        obs, ors = _row_strides(out, H, D)
    if gate_logits is not None:
        if gate_logits.dtype != torch.bfloat16 or gate_logits.shape != (B, Lq, H) or \
                gate_logits.stride(2) != 1:
            raise ValueError(f"gate logits must be [B, Lq, H] bf16 with unit head stride")
        ext.gate_logits = gate_logits.data_ptr()
        ext.gate_batch_stride, ext.gate_row_stride = gate_logits.stride(0), gate_logits.stride(1)
    spans = [(0, int(s), int(n)) for (s, n) in cache_spans if n > 0]
    if new_k is not None and new_rows > 0:
        spans.append((1, 0, int(new_rows)))
    arr = (_lib.KVSpan * max(1, len(spans)))()
    for i, (src, s, n) in enumerate(spans):
        arr[i].source, arr[i].row_start, arr[i].rows = src, s, n
    cbs = crs = crows = 0
    if cache_k is not None:
        if cache_k.dtype != torch.bfloat16 or cache_v.dtype != torch.bfloat16:
            raise TypeError("cache must be bfloat16")
        cbs, crs = _row_strides(cache_k, H, D)
        if _row_strides(cache_v, H, D) != (cbs, crs):
            raise ValueError("cached K and V must share strides")
        crows = int(cache_k.shape[1])
    nbs = nrs = nrows = 0
    if new_k is not None:
        if new_k.dtype != torch.bfloat16 or new_v.dtype != torch.bfloat16:
            raise TypeError("new K/V must be bfloat16")
        nbs, nrs = _row_strides(new_k, H, D)
        if _row_strides(new_v, H, D) != (nbs, nrs):
            raise ValueError("new K and V must share strides")
        nrows = int(new_k.shape[1])
    lib = _lib.load()
    keys = sum(n for (_, _, n) in spans)
    ws_bytes = 0 if parts is not None else _workspace_bytes(lib, dev, B, Lq, H, D, keys)
    # the key-range split's partial outputs live in a torch-owned workspace
    if ws_bytes:
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        ext.workspace, ext.workspace_bytes = ws.data_ptr(), ws_bytes
    rec = _graphs.recorder()
    if rec is not None:
        # captured into a graph: the key-tile list goes to the graph's device table
        ext.device_tiles = rec._add_site(arr, len(spans), crows, nrows,
                                         cache_k.data_ptr() if cache_k is not None else None)
    with torch.cuda.device(dev):
        _lib.check(lib.tm_attention_fwd_ext(
            q.data_ptr(), qbs, qrs,
            cache_k.data_ptr() if cache_k is not None else None,
            cache_v.data_ptr() if cache_v is not None else None, cbs, crs, crows,
            new_k.data_ptr() if new_k is not None else None,
            new_v.data_ptr() if new_v is not None else None, nbs, nrs, nrows,
            arr, len(spans), out.data_ptr(), obs, ors, B, Lq, H, D,
            float(scale) if scale is not None else 0.0, ctypes.byref(ext),
            _lib.stream_ptr(dev)), "attention")
        _lib.launched(2 if ws_bytes else 1)  # + the merge kernel of a key-range split
    return out


def partial_bytes(B: int, Lq: int, H: int, D: int, splits: int) -> int:
    """Bytes of one export of partial results (``flash_attention(parts=)``)
    with ``splits`` key ranges, a multiple of 16."""
    n = int(_lib.load().tm_attention_partial_bytes(B, Lq, H, D, splits))
    if n <= 0:
        raise ValueError(f"no partial layout for B={B} Lq={Lq} H={H} D={D} splits={splits}")
    return (n + 15) // 16 * 16


def partial_splits(B: int, Lq: int, H: int, D: int, keys: int) -> int:
    """Key ranges per query tile that keep the SMs busy for an export over
    ``keys`` keys (the kernel's work-partition cost model)."""
    return int(_lib.load().tm_attention_partial_splits(B, Lq, H, D, keys))


_PLAN_MODES = {0: "pair", 1: "split", 2: "pair+cross-head"}


def attention_plan(B: int, Lq: int, H: int, D: int, keys: int,
                   workspace_bytes: Optional[int] = None) -> dict:
    """The work partition the attention entry points choose for ``B x Lq``
    queries and ``H`` heads of dim ``D`` over ``keys`` keys in one span with
    ``workspace_bytes`` of workspace (None: as much as the plan wants):
    ``{"mode": "pair" | "split" | "pair+cross-head", "kv_splits": s,
    "ctas": n}`` (``tm_attention_plan``; host arithmetic, no GPU needed)."""
    mode, splits, ctas = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    ws = (1 << 62) if workspace_bytes is None else int(workspace_bytes)
    _lib.check(_lib.load().tm_attention_plan(B, Lq, H, D, int(keys), ws, ctypes.byref(mode),
                                            ctypes.byref(splits), ctypes.byref(ctas)),
               "attention_plan")
    return {"mode": _PLAN_MODES[mode.value], "kv_splits": splits.value, "ctas": ctas.value}


def combine_partials(parts: Tensor, n_groups: int, group_bytes: int, splits: int, B: int,
                     Lq: int, H: int, D: int, out: Optional[Tensor] = None,
                     gate_logits: Optional[Tensor] = None) -> Tensor:
    """Merge ``n_groups`` exports of ``splits`` key ranges each (group g at
    byte ``g * group_bytes`` of ``parts``: one group per GPU after an
    all-gather) into ``out [B, Lq, H, D]`` bf16, one softmax over all their
    keys; ``gate_logits`` as in :func:`flash_attention`.  The merge order is
    fixed, so every GPU merging the same bytes gets the same bits."""
    dev = _lib.require_cuda(parts)
    if parts.dtype != torch.uint8 or not parts.is_contiguous() or \
            parts.numel() < (n_groups - 1) * group_bytes + partial_bytes(B, Lq, H, D, splits):
        raise ValueError("parts: a contiguous uint8 tensor holding every group")
    if out is None:
        out = torch.empty(B, Lq, H, D, device=dev, dtype=torch.bfloat16)
    obs, ors = _row_strides(out, H, D)
    gp, gbs, grs = None, 0, 0
    if gate_logits is not None:
        if gate_logits.dtype != torch.bfloat16 or gate_logits.shape != (B, Lq, H) or \
                gate_logits.stride(2) != 1:
            raise ValueError("gate logits must be [B, Lq, H] bf16 with unit head stride")
        gp, gbs, grs = gate_logits.data_ptr(), gate_logits.stride(0), gate_logits.stride(1)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().tm_attention_combine(
            parts.data_ptr(), n_groups, group_bytes, splits, B, Lq, H, D, out.data_ptr(), obs,
            ors, gp, gbs, grs, _lib.stream_ptr(dev)), "attention combine")
        _lib.launched()
    return out


_WS_CACHE = {}


def _workspace_bytes(lib, dev, B, Lq, H, D, keys) -> int:
    """Bytes of partial outputs the kernel's work partition needs for this
    shape on this device (0 when it keeps every key range in one CTA)."""
    key = (dev.index, B, Lq, H, D, keys)
    n = _WS_CACHE.get(key)
    if n is None:
        with torch.cuda.device(dev):
            n = int(lib.tm_attention_workspace_bytes(B, Lq, H, D, keys))
        _WS_CACHE[key] = n
    return n


def standard_attention_forward(q: Tensor, k: Tensor, v: Tensor, mask: Optional[Tensor] = None,
                               scale: Optional[float] = None) -> Tensor:
    """SDPA on ``[B, L, H, D]`` tensors (flex_attention_utils.py:225-276).

    ``mask`` may be a key-padding mask (see :func:`key_padding_runs`): the
    visible keys become the kernel's key spans.  Other masks (per-query
    patterns, non-binary biases) raise ``NotImplementedError``."""
    if mask is None:
        return flash_attention(q, None, None, (), k, v, int(k.shape[1]), scale)
    B, Lk = int(q.shape[0]), int(k.shape[1])
    return _masked_attention(q, k, v, key_padding_runs(mask, B, Lk), scale)


_RUNS_CACHE: "OrderedDict" = None


def key_padding_runs(mask: Tensor, batch: int, kv_len: int):
    """Per batch element, the runs ``[(start, rows), ...]`` of visible keys of
    a key-padding mask: boolean / integer ``[B, Lk]`` or ``[B, 1, 1, Lk]``
    (True / 1 = visible, as SDPA's boolean masks), or the additive float mask
    of ``_prepare_attention_mask`` (ltx_causal/transformer/causal_model.py:
    551-562: 0 visible, ``-finfo.max`` padding; ``[B, 1, 1, Lk]``, or
    ``[B, 1, Lq, Lk]`` with equal rows).  One device-to-host read per mask
    tensor (cached by identity and version)."""
    global _RUNS_CACHE
    from collections import OrderedDict
    if _RUNS_CACHE is None:
        _RUNS_CACHE = OrderedDict()
    key = (mask.data_ptr(), mask._version, tuple(mask.shape), str(mask.dtype), batch, kv_len)
    hit = _RUNS_CACHE.get(key)
    if hit is not None:
        _RUNS_CACHE.move_to_end(key)
        return hit
    m = mask.detach()
    if m.dim() == 2:
        m = m[:, None, None, :]
    elif m.dim() == 3:
        m = m[:, None]
    if m.dim() != 4 or m.shape[-1] != kv_len or m.shape[1] != 1 or m.shape[0] not in (1, batch):
        raise NotImplementedError(f"only key-padding masks are supported, got {tuple(mask.shape)}")
    m = m.to("cpu")
    if m.dtype == torch.bool:
        vis = m
    elif not torch.is_floating_point(m):
        vis = m != 0
    else:
        big = torch.finfo(m.dtype).max
        vis = m == 0
        if not bool(((m == 0) | (m <= -big * 0.5) | torch.isinf(m)).all()):
            raise NotImplementedError("additive masks other than 0 / -max are not supported")
    if vis.shape[2] > 1 and not bool((vis == vis[:, :, :1]).all()):
        raise NotImplementedError("per-query masks are not supported (key padding only)")
    vis = vis[:, 0, 0].expand(batch, kv_len)
    runs = []
    for b in range(batch):
        row = vis[b].tolist()
        r, i = [], 0
        while i < kv_len:
            if row[i]:
                j = i
                while j < kv_len and row[j]:
                    j += 1
                r.append((i, j - i))
                i = j
            else:
                i += 1
        runs.append(r)
    _RUNS_CACHE[key] = runs
    while len(_RUNS_CACHE) > 64:
        _RUNS_CACHE.popitem(last=False)
    return runs


def _masked_attention(q: Tensor, k: Tensor, v: Tensor, runs, scale: Optional[float] = None,
                      out: Optional[Tensor] = None) -> Tensor:
    """Attention of ``q`` over the key runs of each batch element (one launch
    when every element has the same runs).  An element without visible keys
    gets the mean of V over all keys — what the additive ``-finfo.max`` mask
    gives once every score saturates to the same value."""
    B, Lq, H, D = (int(t) for t in q.shape)
    if out is None:
        out = torch.empty(B, Lq, H, D, device=q.device, dtype=q.dtype)
    if all(r == runs[0] for r in runs) and runs[0]:
        return flash_attention(q, k, v, runs[0], None, None, 0, scale, out=out)
    for b in range(B):
        if runs[b]:
            flash_attention(q[b:b + 1], k[b:b + 1], v[b:b + 1], runs[b], None, None, 0, scale,
                            out=out[b:b + 1])
        else:
            out[b] = v[b].float().mean(dim=0, keepdim=True).to(out.dtype).expand(Lq, H, D)
    return out


def _text_kv(attn, context: Tensor, base_context: Tensor, prompt_cache_key, cache_name: str,
             sp_size: int) -> Tuple[Tensor, Tensor]:
    """k_norm(to_k(context)) and to_v(context) as ``[B, Lk, H(/sp), D]``, with
    the reference's exact inference LRU (kv_cache.py:676-761): keyed by the
    module, the identity / pointer / shape of ``base_context``, the prompt key
    and the SP rank; 4 entries per module; an entry is valid only while
    ``base_context`` is the same live object."""
    import weakref
    from collections import OrderedDict
    H, D = int(attn.heads), int(attn.dim_head)
    B = int(context.shape[0])
    key = None
    try:
        weakref.ref(base_context)
        rank = P.get_sp_rank() if sp_size > 1 else 0
        key = (cache_name, id(attn), id(base_context), int(base_context.data_ptr()),
               tuple(base_context.shape), tuple(base_context.stride()), str(base_context.dtype),
               str(base_context.device), prompt_cache_key, tuple(context.shape),
               str(context.dtype), str(context.device), int(sp_size), int(rank))
    except TypeError:
        key = None
    cache = getattr(attn, "_ltx_text_cross_kv_cache", None)
    if key is not None:
        if cache is None:
            cache = OrderedDict()
            setattr(attn, "_ltx_text_cross_kv_cache", cache)
        hit = cache.get(key)
        if hit is not None:
            ref, k, v = hit
            if ref() is base_context:
                cache.move_to_end(key)
                return k, v
            cache.pop(key, None)
    # all heads: every rank holds the whole text context, so under sequence
    # parallelism it attends its own query tokens over all heads locally
    k = F.linear(context, attn.to_k.weight, attn.to_k.bias)
    (k,) = norm_rope([k], [attn.k_norm.weight], [None], H, D, _norm_eps(attn.k_norm))
    v = F.linear(context, attn.to_v.weight, attn.to_v.bias).view(B, -1, H, D)
    if key is not None:
        cache[key] = (weakref.ref(base_context), k, v)
        cache.move_to_end(key)
        while len(cache) > 4:
            cache.popitem(last=False)
    return k, v


def text_cross_attention_with_kv_cache(attn, x: Tensor, context: Tensor, *,
                                       mask: Optional[Tensor], base_context: Tensor,
                                       prompt_cache_key=None, cache_name: str = "text",
                                       layer_idx: Optional[int] = None) -> Tensor:
    """Text cross-attention with cached K/V projections
    (``_text_cross_attention_with_kv_cache``, kv_cache.py:764-827): video
    queries against a prompt's text tokens; the padding mask becomes the
    kernel's key spans (no mask tensor is built), K/V projections are cached
    per prompt as the reference does, then gate and out projection.

    Under sequence parallelism the reference moves Q seq->head, attends one
    head group against head-narrowed K/V and moves the output head->seq
    (kv_cache.py:797-817).  Every rank already holds the whole text context,
    so here each rank attends its own query tokens over all heads: the same
    values per (token, head), no exchange."""
    B = int(x.shape[0])
    H, D = int(attn.heads), int(attn.dim_head)
    sp_size = P.get_sp_world_size() if P.is_sp_enabled() else 1
    with section(f"{cache_name}.text_q_project"):
        q = F.linear(x, attn.to_q.weight, attn.to_q.bias)
        (q,) = norm_rope([q], [attn.q_norm.weight], [None], H, D, _norm_eps(attn.q_norm))
    k, v = _text_kv(attn, context, base_context, prompt_cache_key, cache_name, sp_size)
    runs = [[(0, int(k.shape[1]))]] * B if mask is None else key_padding_runs(mask, B,
                                                                            int(k.shape[1]))
    with section(f"{cache_name}.text_sdpa"):
        out = _masked_attention(q, k, v, runs)
    out = out.reshape(B, -1, H * D)
    if getattr(attn, "to_gate_logits", None) is not None:
        gates = 2.0 * torch.sigmoid(attn.to_gate_logits(x))
        out = (out.view(B, -1, H, D) * gates.unsqueeze(-1)).view(B, -1, H * D)
    return attn.to_out(out)


def _norm_eps(norm) -> float:
    eps = getattr(norm, "eps", None)
    return 1e-6 if eps is None else float(eps)


def _cache_source(cached_k, cached_v):
    """Cache tensors and row spans for the kernel (arena views read in place)."""
    if cached_k is None:
        return None, None, []
    if isinstance(cached_k, ArenaKV):
        if not isinstance(cached_v, ArenaKV) or cached_v._state is not cached_k._state:
            raise ValueError("cached K and V arena views must belong to one pair")
        kt, rows = cache_rows_view(cached_k)
        return kt, cached_k.arena.v, rows
    return cached_k, cached_v, [(0, int(cached_k.shape[1]))]


def _fuse_linears(attn, names: Tuple[str, ...], tag: str) -> bool:
    """Lay the linears ``names`` of ``attn`` out as one ``[n * out, in]``
    weight buffer (and one bias buffer): the parameters become row blocks of
    it, values unchanged.  False (nothing changed) when they differ in shape,
    dtype, device or bias."""
    lins = [getattr(attn, n) for n in names]
    ws = [l.weight for l in lins]
    bs = [l.bias for l in lins]
    w0 = ws[0]
    if any(w.shape != w0.shape or w.dtype != w0.dtype or w.device != w0.device for w in ws):
        return False
    if any((b is None) != (bs[0] is None) for b in bs):
        return False
    if bs[0] is not None and any(b.shape != bs[0].shape or b.dtype != bs[0].dtype for b in bs):
        return False
    n = int(w0.shape[0])
    with torch.no_grad():
        W = torch.cat([w.detach() for w in ws]).contiguous()
        Bv = torch.cat([b.detach() for b in bs]).contiguous() if bs[0] is not None else None
        for i, l in enumerate(lins):
            l.weight.data = W[i * n:(i + 1) * n]
            if Bv is not None:
                l.bias.data = Bv[i * n:(i + 1) * n]
    setattr(attn, tag, (W, Bv))
    return True


def _fused(attn, names: Tuple[str, ...], tag: str):
    """The fused buffers of :func:`_fuse_linears` while the module's
    parameters still point into them, else None."""
    f = getattr(attn, tag, None)
    if f is None:
        return None
    W, Bv = f
    n = W.shape[0] // len(names)
    for i, name in enumerate(names):
        l = getattr(attn, name)
        if l.weight.data_ptr() != W[i * n].data_ptr() or l.weight.shape[0] != n:
            return None
        if Bv is not None and (l.bias is None or l.bias.data_ptr() != Bv[i * n:].data_ptr()):
            return None
    return f


def fuse_qkv_weights(attn) -> bool:
    """Lay ``to_q``, ``to_k`` and ``to_v`` of a self-attention module out as one
    ``[3 * inner, in]`` weight buffer (and one bias buffer): the three
    parameters become row blocks of it, with their values unchanged, so
    ``attention_with_cache`` runs the three projections of a self-attention
    call as ONE GEMM.  At the short chunks of a streaming step (1152 rows, or
    1152 / G per GPU under sequence parallelism) one GEMM with three times the
    columns fills the SMs better than three.  Returns False (and changes
    nothing) when the three linears differ in shape, dtype, device or bias.

    Reference counterpart: none (the reference runs the three linears,
    ltx_causal/transformer/kv_cache.py:1380-1410); a loader calls this once
    per module after loading weights.  Weights later loaded in place
    (``load_state_dict``, ``copy_``) land in the shared buffer; a parameter
    that is replaced by a new tensor ends the fusion for that module.
    """
    return _fuse_linears(attn, ("to_q", "to_k", "to_v"), "_tm_qkv")


def fuse_kv_weights(attn) -> bool:
    """``fuse_qkv_weights`` for the key and value projections of a
    cross-attention module (``to_k``, ``to_v`` read the same context): one
    ``[2 * inner, in]`` GEMM computes both (the A2V / V2A pair,
    kv_cache.py:2011-2022)."""
    return _fuse_linears(attn, ("to_k", "to_v"), "_tm_kv")


def _fused_qkv(attn):
    return _fused(attn, ("to_q", "to_k", "to_v"), "_tm_qkv")


def _fused_kv(attn):
    return _fused(attn, ("to_k", "to_v"), "_tm_kv")


def kv_projection(attn, ctx: Tensor, pe, eps: float) -> Tuple[Tensor, Tensor]:
    """Keys and values of a cross-attention call on one GPU: ``to_k`` /
    ``to_v`` of ``ctx`` (one GEMM after :func:`fuse_kv_weights`), K
    RMS-normalised and rotated by ``pe`` (None: no rotation) in one fused
    launch; returns ``[B, L, H, D]`` views that share one row stride
    (kv_cache.py:1380-1410 for the K/V side)."""
    H, D = int(attn.heads), int(attn.dim_head)
    B, L = int(ctx.shape[0]), int(ctx.shape[1])
    f = _fused_kv(attn)
    if f is not None:
        k, v = F.linear(ctx, f[0], f[1]).split(f[0].shape[0] // 2, dim=-1)
        (k,) = norm_rope([k], [attn.k_norm.weight], [pe], H, D, eps, inplace=True)
        return k, v.unflatten(-1, (H, D))
    k = F.linear(ctx, attn.to_k.weight, attn.to_k.bias)
    v = F.linear(ctx, attn.to_v.weight, attn.to_v.bias)
    (k,) = norm_rope([k], [attn.k_norm.weight], [pe], H, D, eps)
    return k, v.view(B, L, H, D)


def cross_attention_local(attn, x: Tensor, pe, k: Tensor, v: Tensor, cached_k, cached_v,
                          new_kv_real_len: Optional[int] = None,
                          profile_name: str = "cross") -> Tuple[Tensor, Tensor, Tensor]:
    """``attention_with_cache`` on one GPU (or under ``sp_local``) for a
    cross-attention whose keys and values were projected beforehand
    (:func:`kv_projection`, e.g. on another stream): the query projection,
    its norm + RoPE, attention over the cache spans and the new rows (the
    per-head gate fused), ``to_out``.  Returns ``(out, new_k, new_v)`` as
    ``attention_with_cache`` does (kv_cache.py:1148-1547)."""
    H, D = int(attn.heads), int(attn.dim_head)
    B = int(x.shape[0])
    eps = _norm_eps(attn.q_norm)
    with section(profile_name + ".qkv_proj_norm"):
        q = F.linear(x, attn.to_q.weight, attn.to_q.bias)
    with section(profile_name + ".rope_reshape"):
        (q,) = norm_rope([q], [attn.q_norm.weight], [pe], H, D, eps)
    n = int(k.shape[1])
    if new_kv_real_len is not None and new_kv_real_len < n:
        n = int(new_kv_real_len)
        k, v = k[:, :n], v[:, :n]
    ck, cv, spans = _cache_source(cached_k, cached_v)
    glog = attn.to_gate_logits(x) if getattr(attn, "to_gate_logits", None) is not None else None
    with section(profile_name + ".sdpa"):
        out = flash_attention(q, ck, cv, spans, k, v, n, gate_logits=glog)
    with section(profile_name + ".out_proj"):
        out = attn.to_out(out.reshape(B, -1, H * D))
    return out, k, v


def _projections(attn, x: Tensor, ctx: Tensor):
    """q, k, v projections (cuBLAS through torch).  For self-attention over a
    module prepared by ``fuse_qkv_weights`` one GEMM computes all three, and
    q, k, v are column slices of its ``[B, L, 3 * inner]`` output."""
    f = _fused_qkv(attn) if ctx is x else None
    if f is not None:
        qkv = F.linear(x, f[0], f[1])
        return qkv.split(f[0].shape[0] // 3, dim=-1)
    return (F.linear(x, attn.to_q.weight, attn.to_q.bias),
            F.linear(ctx, attn.to_k.weight, attn.to_k.bias),
            F.linear(ctx, attn.to_v.weight, attn.to_v.bias))


_SIDE_STREAMS = {}


def _side_stream(dev: torch.device) -> torch.cuda.Stream:
    st = _SIDE_STREAMS.get(dev.index)
    if st is None:
        st = _SIDE_STREAMS[dev.index] = torch.cuda.Stream(dev)
    return st


def _copy_kv(k: Tensor, v: Tensor, outs: Tuple[Tensor, Tensor]) -> Tuple[Tensor, Tensor]:
    """Contiguous copies of two ``[1, L, H, D]`` row-strided views into
    ``outs`` in one launch of the row-copy kernel (current stream)."""
    dev = k.device
    row = int(k.shape[2]) * int(k.shape[3]) * k.element_size()
    spans = (_lib.CopySpan * 2)()
    for i, (src, dst) in enumerate(((k, outs[0]), (v, outs[1]))):
        spans[i].src, spans[i].dst, spans[i].rows = src.data_ptr(), dst.data_ptr(), int(src.shape[1])
        spans[i].src_row_stride = src.stride(1) * src.element_size()
        spans[i].dst_row_stride = row
    with torch.cuda.device(dev):
        _lib.check(_lib.load().tm_copy_rows(spans, 2, row, _lib.stream_ptr(dev)), "new K/V copy")
        _lib.launched()
    return outs


def attention_with_cache(
    attn,
    x: Tensor,
    context: Optional[Tensor],
    pe: Optional[Tuple[Tensor, Tensor]],
    k_pe: Optional[Tuple[Tensor, Tensor]],
    cached_k,
    cached_v,
    logit_log_scale: Optional[Tensor] = None,
    pyramid_policy=None,
    layer_idx: Optional[int] = None,
    modality: Optional[str] = None,
    frame_seqlen: Optional[int] = None,
    sp_context_sharded: bool = True,
    new_kv_real_len: Optional[int] = None,
    profile_name: Optional[str] = None,
):
    """One attention op with KV cache (kv_cache.py:1148-1547).

    ``attn`` is the reference ``CausalLTXAttention`` module (or any object
    with ``to_q/to_k/to_v/to_out[0]`` linears, ``q_norm/k_norm`` RMSNorms,
    ``heads``, ``dim_head`` and optional ``to_gate_logits``).  ``cached_k/v``
    are ``[B, L, H(/sp), D]`` tensors or arena views.  Returns ``(out, new_k,
    new_v)`` with ``new_k/v`` in the cache layout (head-sharded under SP).
    """
    if pyramid_policy is not None:
        raise NotImplementedError("pyramid KV selection is disabled in every shipped config")
    B, L, _ = x.shape
    ctx = x if context is None else context
    H, D = int(attn.heads), int(attn.dim_head)
    sp_size = P.get_sp_world_size() if P.is_sp_enabled() else 1
    if sp_size > 1 and not sp_context_sharded:
        # The context is replicated on every rank (text cross-attention): the
        # reference narrows K/V to this rank's heads after a seq->head move of
        # Q (kv_cache.py:1446-1451).  Attending this rank's query tokens over
        # all heads gives the same values per (token, head) with no exchange;
        # cached and returned K/V then hold all heads.
        with P.sp_local():
            return attention_with_cache(attn, x, context, pe, k_pe, cached_k, cached_v,
                                        logit_log_scale, pyramid_policy, layer_idx, modality,
                                        frame_seqlen, True, new_kv_real_len, profile_name)

    base = profile_name or ("self" if context is None else "cross")
    # 1. projections (library GEMMs)
    with section(base + ".qkv_proj_norm"):
        q, k, v = _projections(attn, x, ctx)
    q_pe = pe
    kk_pe = k_pe if k_pe is not None else pe
    eps_q, eps_k = _norm_eps(attn.q_norm), _norm_eps(attn.k_norm)
    if abs(eps_q - eps_k) > 0:
        raise NotImplementedError("q_norm and k_norm with different eps")

    # 2-3. fused norm + RoPE (+ send layout) and the seq->head exchange
    if sp_size == 1:
        # fused QKV: q and k are normalised in place, so the new K and V the
        # kernel reads (and this call returns) share one row stride
        inplace = not v.is_contiguous() and k.stride() == v.stride()
        with section(base + ".rope_reshape"):
            q, k = norm_rope([q, k], [attn.q_norm.weight, attn.k_norm.weight], [q_pe, kk_pe], H,
                             D, eps_q, inplace=inplace)
        v = v.view(B, -1, H, D)
        if logit_log_scale is not None:
            s = logit_log_scale.to(q.dtype)
            q = q * (s.unsqueeze(-1) if s.dim() == 3 else s.view(B, -1, 1, 1))
    else:
        same = (q.shape == k.shape == v.shape)
        peer = P.get_peer_exchange()
        if peer is not None and not (same and B == 1 and peer.fits(B, L, H, D)):
            peer = None
        if peer is not None:
            # fused exchanges: the kernels store into the owner rank's buffers over NVLink
            with section(base + ".rope_reshape"):
                norm_rope([q, k, v], [attn.q_norm.weight, attn.k_norm.weight, None],
                          [q_pe, kk_pe, None], H, D, eps_q, sp_size=sp_size, packed=True,
                          peer=peer)
            with section(base + ".a2a_seq2head"):
                peer.exchange(0)
            flat = peer.recv.view(sp_size * L, 3, H // sp_size, D)
            q, k, v = (flat[:, i].unsqueeze(0) for i in range(3))
        elif same:
            with section(base + ".rope_reshape"):
                send = norm_rope([q, k, v], [attn.q_norm.weight, attn.k_norm.weight, None],
                                 [q_pe, kk_pe, None], H, D, eps_q, sp_size=sp_size, packed=True)
            with section(base + ".a2a_seq2head"):
                q, k, v = P.seq_all_to_all_head_packed(send, P.get_sp_group(), sp_size)
        else:
            sq, sk, sv = norm_rope([q, k, v], [attn.q_norm.weight, attn.k_norm.weight, None],
                                   [q_pe, kk_pe, None], H, D, eps_q, sp_size=sp_size)
            grp = P.get_sp_group()
            q = P._recv_to_head_layout(P._a2a(sq, grp)[0])
            k = P._recv_to_head_layout(P._a2a(sk, grp)[0])
            v = P._recv_to_head_layout(P._a2a(sv, grp)[0])
        if logit_log_scale is not None:
            s = logit_log_scale.to(q.dtype)
            s = s.unsqueeze(-1) if s.dim() == 3 else (s if s.dim() == 4 else s.view(1, -1, 1, 1))
            q = q * s

    # real-length strip (kv_cache.py:1474-1478): the kernel reads only the real rows
    nk_rows = int(k.shape[1])
    if new_kv_real_len is not None and new_kv_real_len < nk_rows:
        nk_rows = int(new_kv_real_len)
        k = k[:, :nk_rows]
        v = v[:, :nk_rows]

    # 4. attention over [cache spans..., new chunk]
    ck, cv, spans = _cache_source(cached_k, cached_v)
    if q.stride(3) != 1 or q.stride(2) != D:
        q = q.contiguous()
    peer = P.get_peer_exchange() if sp_size > 1 else None
    if peer is not None and not (q.data_ptr() >= peer.recv.data_ptr() and
                                 q.data_ptr() < peer.recv.data_ptr() + peer.recv.nbytes):
        peer = None  # this call's exchange went through NCCL
    # the per-head gate (kv_cache.py:1691-1697) rides in the kernel's epilogue
    # when the output rows stay on this rank
    fuse_gate = sp_size == 1 and getattr(attn, "to_gate_logits", None) is not None
    glog = attn.to_gate_logits(x) if fuse_gate else None
    if peer is not None:
        # The returned cache K/V must outlive the receive buffer, where the
        # peers store the next call's rows once this rank has signalled the
        # head->seq exchange.  They are copied out on a side stream, next to
        # the attention kernel (which leaves a few SMs idle under sequence
        # parallelism), and joined before the signal.
        main, side = torch.cuda.current_stream(q.device), _side_stream(q.device)
        kv_out = (torch.empty(k.shape, dtype=k.dtype, device=q.device),
                  torch.empty(v.shape, dtype=v.dtype, device=q.device))
        side.wait_stream(main)
        with torch.cuda.stream(side):
            _copy_kv(k, v, kv_out)
    with section(base + ".sdpa"):
        out = flash_attention(q, ck, cv, spans, k, v, nk_rows, peer=peer, gate_logits=glog)

    # 5. head -> seq
    if peer is not None:
        main.wait_stream(side)
        k, v = kv_out
        with section(base + ".a2a_head2seq"):
            peer.exchange(1)
        out = peer.out
    elif sp_size > 1:
        with section(base + ".a2a_head2seq"):
            out = P.head_all_to_all_seq(out, P.get_sp_group(), sp_size)

    # 6. gate + out projection (kv_cache.py:1680-1700)
    with section(base + ".out_proj"):
        out = out.reshape(B, -1, H * D)
        if getattr(attn, "to_gate_logits", None) is not None and not fuse_gate:
            gates = 2.0 * torch.sigmoid(attn.to_gate_logits(x))
            out = (out.view(B, -1, H, D) * gates.unsqueeze(-1)).view(B, -1, H * D)
        out = attn.to_out(out)
    return out, k, v


def cross_modal_pair_attention_with_cache(
    audio_to_video_attn,
    video_to_audio_attn,
    vx_a2v: Tensor,
    ax_a2v: Tensor,
    ax_v2a: Tensor,
    vx_v2a: Tensor,
    video_cross_pe: Optional[Tuple[Tensor, Tensor]],
    audio_cross_pe: Optional[Tuple[Tensor, Tensor]],
    layer_cache,
    *,
    video_real_len: Optional[int],
    audio_real_len: Optional[int],
    layer_idx: Optional[int],
):
    """Paired A2V / V2A attention with cache (kv_cache.py:1967-2138).

    A2V: queries from video (``vx_a2v``, video cross RoPE), keys and values
    from audio (``ax_a2v``, audio cross RoPE), cached in
    ``layer_cache.a2v_k/v``; ``audio_real_len`` new rows are kept.  V2A is
    the reverse, cached in ``layer_cache.v2a_k/v``, keeping ``video_real_len``
    rows.  The two attentions are independent until the caller's residual
    updates.  The reference pairs them only to pack their same-shaped
    all-to-alls.  Here each one is an ``attention_with_cache`` call with a
    context: the same kernels, with each call's Q, K and V packed into its
    own exchange.  Returns ``(a2v_out, new_a2v_k, new_a2v_v, v2a_out,
    new_v2a_k, new_v2a_v)``.
    """
    a2v = attention_with_cache(audio_to_video_attn, vx_a2v, ax_a2v, video_cross_pe,
                               audio_cross_pe, layer_cache.a2v_k, layer_cache.a2v_v,
                               layer_idx=layer_idx, new_kv_real_len=audio_real_len,
                               profile_name="attn.audio_to_video")
    v2a = attention_with_cache(video_to_audio_attn, ax_v2a, vx_v2a, audio_cross_pe,
                               video_cross_pe, layer_cache.v2a_k, layer_cache.v2a_v,
                               layer_idx=layer_idx, new_kv_real_len=video_real_len,
                               profile_name="attn.video_to_audio")
    return a2v + v2a


_cross_modal_pair_attention_with_cache = cross_modal_pair_attention_with_cache


class AttentionWeights(torch.nn.Module):
    """Weight container with the attribute names of the reference's
    ``CausalLTXAttention`` (ltx_causal/attention/causal_attention.py:55-118):
    ``to_q/to_k/to_v`` (bias), ``q_norm/k_norm`` (RMSNorm over heads*dim_head),
    ``to_out[0]`` and optional ``to_gate_logits``.  For benchmarks and tests
    on machines without the reference package; ``attention_with_cache`` takes
    either."""

    def __init__(self, query_dim: int, heads: int, dim_head: int, context_dim: Optional[int] = None,
                 norm_eps: float = 1e-6, gated: bool = False, device=None,
                 dtype: torch.dtype = torch.bfloat16, std: Optional[float] = 0.02):
        super().__init__()
        inner = heads * dim_head
        ctx = query_dim if context_dim is None else context_dim
        kw = dict(device=device, dtype=dtype)
        self.heads, self.dim_head, self.inner_dim = heads, dim_head, inner
        self.to_q = torch.nn.Linear(query_dim, inner, bias=True, **kw)
        self.to_k = torch.nn.Linear(ctx, inner, bias=True, **kw)
        self.to_v = torch.nn.Linear(ctx, inner, bias=True, **kw)
        self.q_norm = torch.nn.RMSNorm(inner, eps=norm_eps, **kw)
        self.k_norm = torch.nn.RMSNorm(inner, eps=norm_eps, **kw)
        self.to_gate_logits = torch.nn.Linear(query_dim, heads, bias=True, **kw) if gated else None
        self.to_out = torch.nn.Sequential(torch.nn.Linear(inner, query_dim, bias=True, **kw),
                                          torch.nn.Identity())
        if std is not None:
            with torch.no_grad():
                for m in self.modules():
                    if isinstance(m, torch.nn.Linear):
                        m.weight.normal_(0.0, std)
                        m.bias.normal_(0.0, std)
