"""CPU oracle for the causal-LTX streaming attention hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this module:
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
``--impl reference`` leg use it, always as the checker or the timed CPU
reference, never as a code path of the library.

This is a numpy restatement (float64 by default) of the reference algorithm.
Each function cites the reference file:line it restates (paths relative to the
TaoLiveAIGC/TaoMate source tree).  The arithmetic of the reference lives in
PyTorch (``F.scaled_dot_product_attention``, ``nn.RMSNorm``, elementwise ops)
and einops (``rearrange``); this module restates the published math of those
ops.  Parity is pinned against golden vectors produced by running the
reference itself on CPU (``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

# Physical-coordinate constants, ltx_causal/rope/causal_rope.py:32-37.
VIDEO_TEMPORAL_SCALE = 8
VIDEO_SPATIAL_SCALE = 32
VIDEO_FPS = 24
AUDIO_DOWNSAMPLE_FACTOR = 4
AUDIO_HOP_LENGTH = 160
AUDIO_SAMPLE_RATE = 16000

# Block layout constants, ltx_causal/attention/mask_builder.py:96-99.
AUDIO_FRAMES_PER_BLOCK = 25
AUDIO_FRAMES_FIRST_BLOCK = 26


# ----------------------------------------------------------------------------
# A1: RoPE frequency tables (ltx_causal/rope/causal_rope.py)
# ----------------------------------------------------------------------------
def linspace_f32(start: float, end: float, steps: int) -> np.ndarray:
    """fp32 linspace with the symmetric two-sided formula torch uses (the first
    half counts up from ``start``, the second half down from ``end``), each
    element formed with one rounding (fused multiply-add) from an fp32 step."""
    if steps == 1:
        return np.array([start], np.float32)
    f = np.float32
    step = np.float64(f((f(end) - f(start)) / f(steps - 1)))
    i = np.arange(steps, dtype=np.float64)
    half = steps // 2
    lo = (np.float64(f(start)) + step * i[:half]).astype(np.float32)
    hi = (np.float64(f(end)) - step * (steps - 1 - i[half:])).astype(np.float32)
    return np.concatenate([lo, hi])


def generate_freq_grid(theta: float, max_pos_count: int, inner_dim: int,
                       precision: str = "f64") -> np.ndarray:
    """``theta ** linspace(0, 1, inner_dim // (2 n)) * pi / 2``.

    Restates ``generate_freq_grid`` (causal_rope.py:45-80): the linspace runs
    from log_theta(1)=0 to log_theta(theta)=1.  ``precision="f32"`` repeats
    the reference's fp32 op sequence (fp32 linspace, pow rounded to fp32,
    multiply by fp32(pi), divide by 2); ``"f64"`` is the exact math.
    """
    n = inner_dim // (2 * max_pos_count)
    if precision == "f32":
        lin = linspace_f32(0.0, 1.0, n)
        base = np.float64(np.float32(theta))  # the scalar base is applied in fp32
        ind = np.power(base, lin.astype(np.float64)).astype(np.float32)
        return (ind * np.float32(math.pi)).astype(np.float32) / np.float32(2)
    lin = np.linspace(0.0, 1.0, n, dtype=np.float64)
    return np.power(float(theta), lin) * (math.pi / 2)


def ntk_theta(theta: float, dim: int, start_frame: int, max_latent_f: int,
              is_audio: bool, train_max_seconds: float) -> float:
    """NTK-aware theta scaling, causal_rope.py:199-246."""
    max_latent_abs = int(start_frame) + int(max_latent_f)
    if max_latent_abs <= 0:
        return float(theta)
    if is_audio:
        mel_end = max(0.0, max_latent_abs * AUDIO_DOWNSAMPLE_FACTOR + 1 - AUDIO_DOWNSAMPLE_FACTOR)
        t_max = mel_end * AUDIO_HOP_LENGTH / AUDIO_SAMPLE_RATE
    else:
        pixel_end = max(0.0, max_latent_abs * VIDEO_TEMPORAL_SCALE + 1 - VIDEO_TEMPORAL_SCALE)
        t_max = pixel_end / VIDEO_FPS
    ratio = max(1.0, t_max / max(float(train_max_seconds), 1e-6))
    if ratio > 1.0:
        return float(theta) * ratio ** (float(dim) / max(float(dim - 2), 1.0))
    return float(theta)


def temporal_seconds(start_frame: int, frames: int, is_audio: bool,
                     dtype=np.float64) -> np.ndarray:
    """Latent frame -> physical midpoint in seconds with the causal fix.

    Video: causal_rope.py:262-265 (pixel frames [8t-7, 8t+1] clamped at 0, /24).
    Audio: causal_rope.py:296-300 (mel frames [4t-3, 4t+1] clamped, *160/16000).
    Integer steps are exact in either precision; the divisions round in ``dtype``.
    """
    t = np.arange(start_frame, start_frame + frames).astype(dtype)
    c = lambda v: dtype(v)
    if is_audio:
        s = np.maximum(t * c(AUDIO_DOWNSAMPLE_FACTOR) + c(1 - AUDIO_DOWNSAMPLE_FACTOR), c(0))
        e = np.maximum((t + c(1)) * c(AUDIO_DOWNSAMPLE_FACTOR) + c(1 - AUDIO_DOWNSAMPLE_FACTOR), c(0))
        return ((s + e) / c(2.0) * c(AUDIO_HOP_LENGTH) / c(AUDIO_SAMPLE_RATE)).astype(dtype)
    s = np.maximum(t * c(VIDEO_TEMPORAL_SCALE) + c(1 - VIDEO_TEMPORAL_SCALE), c(0))
    e = np.maximum((t + c(1)) * c(VIDEO_TEMPORAL_SCALE) + c(1 - VIDEO_TEMPORAL_SCALE), c(0))
    return ((s + e) / c(2.0) / c(VIDEO_FPS)).astype(dtype)


def fractional_positions(grid: Sequence[int], start_frame: int, max_pos: Sequence[float],
                         is_audio: bool, dtype=np.float64) -> np.ndarray:
    """[T, n_pos] fractional positions (causal_rope.py:253-308).

    3-D video grid (F, H, W): time as above, space at pixel midpoints
    ``32 i + 16``; each axis divided by ``max_pos``; tokens ordered (f, h, w)
    row-major (meshgrid 'ij').
    """
    c = lambda v: dtype(v)
    if len(grid) == 3:
        f, h, w = (int(v) for v in grid)
        t_frac = temporal_seconds(start_frame, f, False, dtype) / c(max_pos[0])
        h_frac = (np.arange(h).astype(dtype) * c(VIDEO_SPATIAL_SCALE) + c(VIDEO_SPATIAL_SCALE / 2.0)) / c(max_pos[1])
        w_frac = (np.arange(w).astype(dtype) * c(VIDEO_SPATIAL_SCALE) + c(VIDEO_SPATIAL_SCALE / 2.0)) / c(max_pos[2])
        gt, gh, gw = np.meshgrid(t_frac, h_frac, w_frac, indexing="ij")
        return np.stack([gt, gh, gw], axis=-1).reshape(f * h * w, 3).astype(dtype)
    if len(grid) == 1:
        f = int(grid[0])
        return (temporal_seconds(start_frame, f, is_audio, dtype) / c(max_pos[0])).reshape(f, 1).astype(dtype)
    raise ValueError(f"Unsupported num_pos_dims: {len(grid)}")


def precompute_freqs_cis_split(grid: Sequence[int], dim: int, theta: float = 10000.0,
                               max_pos: Optional[Sequence[float]] = None, start_frame: int = 0,
                               is_audio: bool = False, num_heads: int = 32,
                               rope_extrapolation: str = "off",
                               rope_train_max_seconds: float = 8.0,
                               precision: str = "f64") -> Tuple[np.ndarray, np.ndarray]:
    """SPLIT-mode cos/sin tables ``[H, T, dim // 2 // H]`` (batch dim dropped).

    Restates ``causal_precompute_freqs_cis`` (causal_rope.py:139-357) for
    ``rope_type=SPLIT``: per-token frequencies ``indices * (2 frac - 1)`` laid
    out axis-interleaved ``[f0_t, f0_h, f0_w, f1_t, ...]`` (:287-288), padded at
    the FRONT with identity entries (cos 1, sin 0) up to ``dim // 2``
    (:323-336), then split per head (:340-341).  ``precision="f32"`` forms
    the rotation angle with the reference's fp32 operations; cos/sin are then
    evaluated exactly (float64) on that fp32 angle.
    """
    if max_pos is None:
        max_pos = [20, 2048, 2048]
    n_pos = len(grid)
    if rope_extrapolation == "ntk":
        theta = ntk_theta(theta, dim, start_frame, int(grid[0]), is_audio, rope_train_max_seconds)
    elif rope_extrapolation != "off":
        raise ValueError(f"rope_extrapolation must be 'off' or 'ntk', got {rope_extrapolation!r}")
    dt = np.float32 if precision == "f32" else np.float64
    indices = generate_freq_grid(theta, n_pos, dim, precision)            # [n_freq]
    frac = fractional_positions(grid, start_frame, max_pos, is_audio, dt)  # [T, n_pos]
    freqs = indices[None, None, :] * (frac[:, :, None] * dt(2.0) - dt(1.0))  # [T, n_pos, n_freq]
    freqs = np.swapaxes(freqs, 1, 2).reshape(frac.shape[0], -1).astype(np.float64)
    half = dim // 2
    pad = half - freqs.shape[-1]
    cos = np.cos(freqs)
    sin = np.sin(freqs)
    if pad > 0:
        cos = np.concatenate([np.ones((cos.shape[0], pad)), cos], axis=-1)
        sin = np.concatenate([np.zeros((sin.shape[0], pad)), sin], axis=-1)
    T = cos.shape[0]
    cos = cos.reshape(T, num_heads, -1).transpose(1, 0, 2)
    sin = sin.reshape(T, num_heads, -1).transpose(1, 0, 2)
    return cos, sin


def expand_per_frame(table: np.ndarray, frame_seqlen: int) -> np.ndarray:
    """``[H, F, d] -> [H, F * frame_seqlen, d]`` (ltx_causal/transformer/kv_cache.py:2973-2983)."""
    return np.repeat(table, frame_seqlen, axis=1)


# ----------------------------------------------------------------------------
# A2 / A3: RMSNorm + split rotary
# ----------------------------------------------------------------------------
def rms_norm(x: np.ndarray, weight: Optional[np.ndarray], eps: float = 1e-6) -> np.ndarray:
    """``x / sqrt(mean(x^2) + eps) * w`` over the last dim (torch.nn.RMSNorm,
    used as q_norm/k_norm at ltx_causal/attention/causal_attention.py:105-106)."""
    dt = np.float32 if isinstance(x, np.ndarray) and x.dtype == np.float32 else np.float64
    x = np.asarray(x, dtype=dt)
    r = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + dt(eps))
    y = x * r
    if weight is not None:
        y = y * np.asarray(weight, dtype=dt)
    return y


def apply_split_rotary_emb(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Rotate-half RoPE per head (causal_rope.py:102-132).

    ``x``: ``[T, H * D]``; ``cos``/``sin``: ``[H, T, D // 2]``.  With x1/x2 the
    first/second half of each head: ``out1 = x1 cos - x2 sin``,
    ``out2 = x2 cos + x1 sin``.
    """
    x = np.asarray(x, dtype=x.dtype if isinstance(x, np.ndarray) and x.dtype == np.float32
                   else np.float64)
    H, T, half = cos.shape
    xh = x.reshape(T, H, 2, half).transpose(1, 0, 2, 3)  # [H, T, 2, half]
    x1, x2 = xh[:, :, 0], xh[:, :, 1]
    o1 = x1 * cos - x2 * sin
    o2 = x2 * cos + x1 * sin
    out = np.stack([o1, o2], axis=2).transpose(1, 0, 2, 3).reshape(T, H * 2 * half)
    return out


# ----------------------------------------------------------------------------
# A7: attention core
# ----------------------------------------------------------------------------
def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: Optional[float] = None,
              mask: Optional[np.ndarray] = None, dtype=np.float64) -> np.ndarray:
    """``softmax(q k^T * scale [+ mask]) v`` per head, layout ``[L, H, D]``.

    Restates ``standard_attention_forward`` (ltx_causal/attention/
    flex_attention_utils.py:225-276), i.e. ``F.scaled_dot_product_attention``
    with ``is_causal=False`` and default scale ``D ** -0.5``.  ``mask`` is a
    boolean ``[Lq, Lk]`` (True = visible) or additive float mask.
    """
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    D = q.shape[-1]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if mask is None and dtype != np.float64:
        # head-by-head BLAS products (the fp32 path times the CPU baseline)
        out = np.empty_like(q)
        for h in range(q.shape[1]):
            s = (q[:, h] @ k[:, h].T) * dtype(scale)
            s -= s.max(axis=-1, keepdims=True)
            np.exp(s, out=s)
            s /= s.sum(axis=-1, keepdims=True)
            out[:, h] = s @ v[:, h]
        return out
    s = np.einsum("qhd,khd->hqk", q, k) * scale
    if mask is not None:
        if mask.dtype == bool:
            s = np.where(mask[None], s, -np.inf)
        else:
            s = s + mask[None]
    m = np.max(s, axis=-1, keepdims=True)
    p = np.exp(s - m)
    p /= np.sum(p, axis=-1, keepdims=True)
    return np.einsum("hqk,khd->qhd", p, v)


def attention_with_cache(x: np.ndarray, params: Dict[str, np.ndarray], heads: int, dim_head: int,
                         pe: Optional[Tuple[np.ndarray, np.ndarray]],
                         cached_k: Optional[np.ndarray], cached_v: Optional[np.ndarray],
                         context: Optional[np.ndarray] = None,
                         k_pe: Optional[Tuple[np.ndarray, np.ndarray]] = None,
                         new_kv_real_len: Optional[int] = None,
                         eps: float = 1e-6, dtype=np.float64):
    """Single-rank ``attention_with_cache`` (ltx_causal/transformer/kv_cache.py:1148-1547).

    ``x``: ``[L, Dq]`` (batch 1); ``params``: ``to_q/to_k/to_v/to_out`` weight
    (``*_w``, torch ``[out, in]``) and bias (``*_b``), ``q_norm_w``,
    ``k_norm_w`` and optionally ``to_gate_logits_w/_b``.  Returns
    ``(out [L, Dq], new_k [Lk, H, D], new_v [Lk, H, D])``.
    Steps: projections + q/k RMSNorm (:1404-1408), RoPE (:1411-1417),
    reshape (:1426-1428), real-length strip (:1474-1478), cache concat
    (:1486-1492), SDPA without mask (:1531), gate + out projection (:1680-1700).
    """
    ctx = x if context is None else context
    f64 = lambda a: np.asarray(a, dtype=dtype)
    q = f64(x) @ f64(params["to_q_w"]).T + f64(params["to_q_b"])
    k = f64(ctx) @ f64(params["to_k_w"]).T + f64(params["to_k_b"])
    v = f64(ctx) @ f64(params["to_v_w"]).T + f64(params["to_v_b"])
    q = rms_norm(q, params["q_norm_w"], eps)
    k = rms_norm(k, params["k_norm_w"], eps)
    if pe is not None:
        q = apply_split_rotary_emb(q, pe[0], pe[1])
        kp = k_pe if k_pe is not None else pe
        k = apply_split_rotary_emb(k, kp[0], kp[1])
    q = q.reshape(q.shape[0], heads, dim_head)
    k = k.reshape(k.shape[0], heads, dim_head)
    v = v.reshape(v.shape[0], heads, dim_head)
    if new_kv_real_len is not None and new_kv_real_len < k.shape[0]:
        k = k[:new_kv_real_len]
        v = v[:new_kv_real_len]
    full_k = k if cached_k is None else np.concatenate([f64(cached_k), k], axis=0)
    full_v = v if cached_v is None else np.concatenate([f64(cached_v), v], axis=0)
    out = attention(q, full_k, full_v, dtype=dtype)
    out = out.reshape(out.shape[0], heads * dim_head)
    if "to_gate_logits_w" in params:
        g = f64(x) @ f64(params["to_gate_logits_w"]).T + f64(params["to_gate_logits_b"])
        gates = 2.0 / (1.0 + np.exp(-g))
        out = (out.reshape(-1, heads, dim_head) * gates[:, :, None]).reshape(out.shape)
    out = out @ f64(params["to_out_w"]).T + f64(params["to_out_b"])
    return out, k, v


def text_cross_attention(x: np.ndarray, context: np.ndarray, params: Dict[str, np.ndarray],
                         heads: int, dim_head: int, mask: Optional[np.ndarray] = None,
                         eps: float = 1e-6, dtype=np.float64) -> np.ndarray:
    """Text cross-attention with cached K/V projections
    (``_text_cross_attention_with_kv_cache``, ltx_causal/transformer/kv_cache.py:764-827;
    the cache only skips recomputing K/V).

    ``x``: ``[B, Lq, Dq]``, ``context``: ``[B, Lk, Dc]``, ``mask``: ``[B, Lk]``
    0/1 (1 = real token) turned into the additive ``(mask - 1) * float32 max``
    of ``_prepare_attention_mask`` (ltx_causal/transformer/causal_model.py:551-562).
    Steps: q = q_norm(to_q(x)) (:796), k = k_norm(to_k(context)), v = to_v(context)
    (:744-747), SDPA with the mask (:811, flex_attention_utils.py:245-276), gate
    2·sigmoid(to_gate_logits(x)) (:821-825), to_out (:826).  No RoPE.
    """
    f = lambda a: np.asarray(a, dtype=dtype)
    B = x.shape[0]
    outs = []
    for b in range(B):
        q = rms_norm(f(x[b]) @ f(params["to_q_w"]).T + f(params["to_q_b"]), params["q_norm_w"], eps)
        k = rms_norm(f(context[b]) @ f(params["to_k_w"]).T + f(params["to_k_b"]),
                     params["k_norm_w"], eps)
        v = f(context[b]) @ f(params["to_v_w"]).T + f(params["to_v_b"])
        q = q.reshape(q.shape[0], heads, dim_head)
        k = k.reshape(k.shape[0], heads, dim_head)
        v = v.reshape(v.shape[0], heads, dim_head)
        add = None
        if mask is not None:
            row = (f(mask[b]) - 1.0) * float(np.finfo(np.float32).max)
            add = np.broadcast_to(row[None, :], (q.shape[0], k.shape[0]))
        o = attention(q, k, v, mask=add, dtype=dtype).reshape(q.shape[0], heads * dim_head)
        if "to_gate_logits_w" in params:
            g = f(x[b]) @ f(params["to_gate_logits_w"]).T + f(params["to_gate_logits_b"])
            gates = 2.0 / (1.0 + np.exp(-g))
            o = (o.reshape(-1, heads, dim_head) * gates[:, :, None]).reshape(o.shape)
        outs.append(o @ f(params["to_out_w"]).T + f(params["to_out_b"]))
    return np.stack(outs)


def cross_modal_pair_attention(a2v_params: Dict[str, np.ndarray], v2a_params: Dict[str, np.ndarray],
                               heads: int, dim_head: int, vx_a2v: np.ndarray, ax_a2v: np.ndarray,
                               ax_v2a: np.ndarray, vx_v2a: np.ndarray,
                               video_cross_pe: Tuple[np.ndarray, np.ndarray],
                               audio_cross_pe: Tuple[np.ndarray, np.ndarray],
                               a2v_cache=None, v2a_cache=None,
                               video_real_len: Optional[int] = None,
                               audio_real_len: Optional[int] = None, eps: float = 1e-6,
                               dtype=np.float64):
    """Paired A2V / V2A attention on one rank
    (``_cross_modal_pair_attention_with_cache``,
    ltx_causal/transformer/kv_cache.py:1967-2138).  The pairing only packs the
    two attentions' all-to-alls; each is the cached attention of
    ``attention_with_cache`` with a context: A2V takes queries from video
    (video cross RoPE) and keys from audio (audio cross RoPE) against the
    ``a2v`` cache, keeping ``audio_real_len`` new keys; V2A the reverse
    against the ``v2a`` cache (``_project_qkv_local_for_cross_pair`` :1550-1597,
    ``_finish_attention_from_head_layout`` :1600-1651).  Caches are
    ``(k, v)`` pairs of ``[L, H, D]`` or None.  Returns
    ``(a2v_out, a2v_k, a2v_v, v2a_out, v2a_k, v2a_v)``.
    """
    ck = lambda c, i: None if c is None else c[i]
    a2v = attention_with_cache(vx_a2v, a2v_params, heads, dim_head, video_cross_pe,
                               ck(a2v_cache, 0), ck(a2v_cache, 1), context=ax_a2v,
                               k_pe=audio_cross_pe, new_kv_real_len=audio_real_len, eps=eps,
                               dtype=dtype)
    v2a = attention_with_cache(ax_v2a, v2a_params, heads, dim_head, audio_cross_pe,
                               ck(v2a_cache, 0), ck(v2a_cache, 1), context=vx_v2a,
                               k_pe=video_cross_pe, new_kv_real_len=video_real_len, eps=eps,
                               dtype=dtype)
    return a2v + v2a


# ----------------------------------------------------------------------------
# A4 / A8 / A13: Ulysses layout permutations (global view over all ranks)
# ----------------------------------------------------------------------------
# ----------------------------------------------------------------------------
# f4: the transformer block around the attention
# ----------------------------------------------------------------------------
def attn_params(sd: Dict[str, np.ndarray], name: str) -> Dict[str, np.ndarray]:
    """The ``to_q_w`` / ``q_norm_w`` ... parameter dict of attention module
    ``name`` from a block state dict (``name.to_q.weight`` ...)."""
    p = {}
    for lin, key in (("to_q", "to_q"), ("to_k", "to_k"), ("to_v", "to_v"), ("to_out.0", "to_out"),
                     ("to_gate_logits", "to_gate_logits")):
        if f"{name}.{lin}.weight" in sd:
            p[key + "_w"] = sd[f"{name}.{lin}.weight"]
            p[key + "_b"] = sd[f"{name}.{lin}.bias"]
    p["q_norm_w"] = sd[f"{name}.q_norm.weight"]
    p["k_norm_w"] = sd[f"{name}.k_norm.weight"]
    return p


def ada_values(table: np.ndarray, ts: np.ndarray, idx: Sequence[int], dtype=np.float64):
    """``table[i] + timestep[:, i]`` for i in ``idx`` (CausalAVTransformerBlock.
    get_ada_values, ltx_causal/transformer/causal_block.py:434-452); ``ts`` is
    ``[L, n * D]`` (one row per token) or ``[1, n * D]``."""
    n, D = table.shape
    t = np.asarray(ts, dtype=dtype).reshape(ts.shape[0], n, D)
    return [np.asarray(table[i], dtype=dtype)[None] + t[:, i] for i in idx]


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    """GELU, tanh approximation (GELUApprox, ltx_causal/transformer/compat.py:40)."""
    return 0.5 * x * (1.0 + np.tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * x ** 3)))


def feed_forward(sd: Dict[str, np.ndarray], name: str, x: np.ndarray, dtype=np.float64):
    """FeedForward (compat.py:47-70): Linear -> tanh GELU -> Linear."""
    f = lambda a: np.asarray(a, dtype=dtype)
    h = f(x) @ f(sd[f"{name}.net.0.proj.weight"]).T + f(sd[f"{name}.net.0.proj.bias"])
    return gelu_tanh(h) @ f(sd[f"{name}.net.2.weight"]).T + f(sd[f"{name}.net.2.bias"])


def block_forward_with_cache(sd: Dict[str, np.ndarray], cfg: Dict[str, int], vx: np.ndarray,
                             ax: np.ndarray, video_ts: np.ndarray, audio_ts: np.ndarray,
                             video_pe, audio_pe, video_cross_pe, audio_cross_pe,
                             video_ctx: np.ndarray, audio_ctx: np.ndarray,
                             video_mask: Optional[np.ndarray], audio_mask: Optional[np.ndarray],
                             video_cross_ss: np.ndarray, video_cross_gate: np.ndarray,
                             audio_cross_ss: np.ndarray, audio_cross_gate: np.ndarray,
                             caches: Dict[str, Tuple[Optional[np.ndarray], Optional[np.ndarray]]],
                             video_real_len: Optional[int] = None,
                             audio_real_len: Optional[int] = None, eps: float = 1e-6,
                             dtype=np.float64):
    """One block with KV cache (block_forward_with_cache,
    ltx_causal/transformer/kv_cache.py:2145-2654, the default path:
    cross_attention_adaln off, no learned memory, A2V/V2A as two calls).

    ``sd``: block state dict (reference names); ``cfg``: ``video_heads``,
    ``video_dim_head``, ``audio_heads``, ``audio_dim_head``.  Activations
    ``[L, D]``; AdaLN rows per token (``video_ts [Lv, 6 Dv]``, ``*_cross_ss
    [L, 4 D]``, ``*_cross_gate [L, D]``); masks ``[Lk]`` 0/1 or None; ``caches``
    maps ``video_self`` / ``audio_self`` / ``a2v`` / ``v2a`` to ``(k, v)``
    ``[L, H, D]`` or ``(None, None)``.  Returns ``(vx, ax, new)`` with ``new``
    the same map holding this call's new K/V rows.
    Order (kv_cache.py:2197-2640): video self (:2197-2218), video text cross
    (:2441-2460), audio self (:2464-2490), audio text cross (:2493-2510),
    norm3 + A2V + V2A (:2512-2598, get_av_ca_ada_values causal_block.py:454-478),
    video FFN (:2600-2618), audio FFN (:2620-2640).
    """
    f = lambda a: np.asarray(a, dtype=dtype)
    Hv, dv = cfg["video_heads"], cfg["video_dim_head"]
    Ha, da = cfg["audio_heads"], cfg["audio_dim_head"]
    rms = lambda x: rms_norm(x, None, eps)
    vx, ax = f(vx), f(ax)
    new = {}
    tab = lambda k: f(sd[k])
    sh, sc, g = ada_values(tab("scale_shift_table"), video_ts, (0, 1, 2), dtype)
    out, k, v = attention_with_cache(rms(vx) * (1 + sc) + sh, attn_params(sd, "attn1"), Hv, dv,
                                     video_pe, *caches["video_self"],
                                     new_kv_real_len=video_real_len, eps=eps, dtype=dtype)
    new["video_self"] = (k, v)
    vx = vx + out * g
    vm = None if video_mask is None else video_mask[None]
    vx = vx + text_cross_attention(rms(vx)[None], f(video_ctx)[None], attn_params(sd, "attn2"),
                                   Hv, dv, mask=vm, eps=eps, dtype=dtype)[0]
    sh, sc, g = ada_values(tab("audio_scale_shift_table"), audio_ts, (0, 1, 2), dtype)
    out, k, v = attention_with_cache(rms(ax) * (1 + sc) + sh, attn_params(sd, "audio_attn1"), Ha,
                                     da, audio_pe, *caches["audio_self"],
                                     new_kv_real_len=audio_real_len, eps=eps, dtype=dtype)
    new["audio_self"] = (k, v)
    ax = ax + out * g
    am = None if audio_mask is None else audio_mask[None]
    ax = ax + text_cross_attention(rms(ax)[None], f(audio_ctx)[None],
                                   attn_params(sd, "audio_attn2"), Ha, da, mask=am, eps=eps,
                                   dtype=dtype)[0]
    vn, an = rms(vx), rms(ax)
    tv, ta = tab("scale_shift_table_a2v_ca_video"), tab("scale_shift_table_a2v_ca_audio")
    sc_va, sh_va, sc_vv, sh_vv = ada_values(tv[:4], video_cross_ss, (0, 1, 2, 3), dtype)
    (g_a2v,) = ada_values(tv[4:], video_cross_gate, (0,), dtype)
    sc_aa, sh_aa, sc_av, sh_av = ada_values(ta[:4], audio_cross_ss, (0, 1, 2, 3), dtype)
    (g_v2a,) = ada_values(ta[4:], audio_cross_gate, (0,), dtype)
    a2v, k, v = attention_with_cache(vn * (1 + sc_va) + sh_va, attn_params(sd, "audio_to_video_attn"),
                                     Ha, da, video_cross_pe, *caches["a2v"],
                                     context=an * (1 + sc_aa) + sh_aa, k_pe=audio_cross_pe,
                                     new_kv_real_len=audio_real_len, eps=eps, dtype=dtype)
    new["a2v"] = (k, v)
    v2a, k, v = attention_with_cache(an * (1 + sc_av) + sh_av, attn_params(sd, "video_to_audio_attn"),
                                     Ha, da, audio_cross_pe, *caches["v2a"],
                                     context=vn * (1 + sc_vv) + sh_vv, k_pe=video_cross_pe,
                                     new_kv_real_len=video_real_len, eps=eps, dtype=dtype)
    new["v2a"] = (k, v)
    vx = vx + a2v * g_a2v
    ax = ax + v2a * g_v2a
    sh, sc, g = ada_values(tab("scale_shift_table"), video_ts, (3, 4, 5), dtype)
    vx = vx + feed_forward(sd, "ff", rms(vx) * (1 + sc) + sh, dtype) * g
    sh, sc, g = ada_values(tab("audio_scale_shift_table"), audio_ts, (3, 4, 5), dtype)
    ax = ax + feed_forward(sd, "audio_ff", rms(ax) * (1 + sc) + sh, dtype) * g
    return vx, ax, new


def seq_to_head(shards: List[np.ndarray]) -> List[np.ndarray]:
    """Seq-sharded ``[B, S/G, H, D]`` per rank -> head-sharded ``[B, S, H/G, D]``.

    Restates ``_seq_to_head`` (taomate/runtime_support/parallel/all_to_all.py:
    125-151) as the permutation it computes over all ranks: rank r receives
    head group r of every rank's sequence shard, concatenated in rank order.
    """
    G = len(shards)
    B, S_loc, H, D = shards[0].shape
    if H % G:
        raise AssertionError(f"H ({H}) must be divisible by sp_size ({G})")
    Hl = H // G
    return [np.concatenate([s[:, :, r * Hl:(r + 1) * Hl] for s in shards], axis=1) for r in range(G)]


def head_to_seq(shards: List[np.ndarray]) -> List[np.ndarray]:
    """Inverse of :func:`seq_to_head` (all_to_all.py:154-173)."""
    G = len(shards)
    B, S, Hl, D = shards[0].shape
    if S % G:
        raise AssertionError(f"S ({S}) must be divisible by sp_size ({G})")
    Sl = S // G
    return [np.concatenate([s[:, r * Sl:(r + 1) * Sl] for s in shards], axis=2) for r in range(G)]


def split_sequence(x: np.ndarray, sp_rank: int, sp_size: int, dim: int = 1) -> np.ndarray:
    """Right-pad to a multiple of ``sp_size`` with zeros and take shard
    ``sp_rank`` (taomate/runtime_support/parallel/sp_utils.py:25-55)."""
    if sp_size <= 1:
        return x
    S = x.shape[dim]
    if S % sp_size:
        pad = sp_size - S % sp_size
        shape = list(x.shape)
        shape[dim] = pad
        x = np.concatenate([x, np.zeros(shape, dtype=x.dtype)], axis=dim)
    chunk = x.shape[dim] // sp_size
    return np.take(x, np.arange(sp_rank * chunk, (sp_rank + 1) * chunk), axis=dim)


# ----------------------------------------------------------------------------
# A11: cache segments and streaming eviction (taomate/inference/cache.py)
# ----------------------------------------------------------------------------
def segment_offsets(segments: List[Dict[str, int]]) -> List[Tuple[int, int, int, int]]:
    """Cumulative ``(video_start, video_end, audio_start, audio_end)`` per
    segment (cache.py:14-26)."""
    vo = ao = 0
    out = []
    for s in segments:
        ve = vo + int(s["video_tokens"])
        ae = ao + int(s["audio_tokens"])
        out.append((vo, ve, ao, ae))
        vo, ao = ve, ae
    return out


def retain_indices(segments: List[Dict[str, int]], recent_blocks: int = 2) -> List[int]:
    """Indices kept by ``retain_streaming_context`` (cache.py:58-67): the
    segment with ``block_idx == 0`` plus the last ``recent_blocks`` others, in
    chronological order.  Raises like the reference when empty or sink-less."""
    if not segments:
        raise RuntimeError("Cached inference did not attach block metadata.")
    sink = next(i for i, s in enumerate(segments) if int(s["block_idx"]) == 0)
    non_sink = [i for i in range(len(segments)) if i != sink]
    return sorted([sink, *non_sink[-recent_blocks:]]) if recent_blocks > 0 else [sink]


def slice_spans(segments: List[Dict[str, int]], keep: List[int]):
    """Video / audio token spans of the kept segments (cache.py:34-41)."""
    offs = segment_offsets(segments)
    return ([(offs[i][0], offs[i][1]) for i in keep], [(offs[i][2], offs[i][3]) for i in keep])


def slice_tensor(t: np.ndarray, spans: List[Tuple[int, int]], axis: int = 1) -> np.ndarray:
    """Concatenate the spans of ``t`` along the sequence axis (cache.py:28-32)."""
    pieces = [np.take(t, np.arange(s, e), axis=axis) for s, e in spans if e > s]
    return pieces[0] if len(pieces) == 1 else np.concatenate(pieces, axis=axis)


def compute_av_blocks(total_video_latent_frames: int, num_frame_per_block: int = 3,
                      num_frame_per_block_first: int = 0) -> List[Tuple[int, int, int, int, int]]:
    """``(block_idx, video_start, video_end, audio_start, audio_end)`` per block
    (ltx_causal/attention/mask_builder.py:102-186)."""
    blocks = []
    if num_frame_per_block_first > 0:
        if total_video_latent_frames < num_frame_per_block_first:
            raise AssertionError("not enough frames")
        blocks.append((0, 0, num_frame_per_block_first, 0, AUDIO_FRAMES_FIRST_BLOCK))
        v, a, b = num_frame_per_block_first, AUDIO_FRAMES_FIRST_BLOCK, 1
    else:
        if total_video_latent_frames < 1:
            raise AssertionError("need at least 1 frame")
        blocks.append((0, 0, 1, 0, 1))
        v, a, b = 1, 1, 1
    while v < total_video_latent_frames:
        ve = min(v + num_frame_per_block, total_video_latent_frames)
        n = ve - v
        ae = a + (AUDIO_FRAMES_PER_BLOCK if n == num_frame_per_block
                  else (AUDIO_FRAMES_PER_BLOCK * n) // num_frame_per_block)
        blocks.append((b, v, ve, a, ae))
        v, a, b = ve, ae, b + 1
    return blocks


def streaming_schedule(num_windows: int = 12, blocks_per_window: int = 5, frames_first: int = 4,
                       frames_per_block: int = 3, frame_tokens: int = 384,
                       evict_in_first_window: bool = False) -> List[List[int]]:
    """Replay the batch runtime's commit/evict schedule and return the kept
    ``block_idx`` list after every committed block.

    Window 0 commits blocks 0..4 without eviction and evicts once at the end
    (taomate/inference/runtime.py:634); later windows evict after every commit
    (taomate/inference/model.py:225-243).
    """
    total_frames = frames_first + (num_windows * blocks_per_window - 1) * frames_per_block
    blocks = compute_av_blocks(total_frames, frames_per_block, frames_first)
    segments: List[Dict[str, int]] = []
    history = []
    for bi, (idx, vs, ve, as_, ae) in enumerate(blocks[: num_windows * blocks_per_window]):
        segments.append({"block_idx": idx, "video_tokens": (ve - vs) * frame_tokens,
                         "audio_tokens": ae - as_})
        window = bi // blocks_per_window
        if window > 0 or evict_in_first_window:
            segments = [segments[i] for i in retain_indices(segments)]
        elif bi == blocks_per_window - 1:
            history.append([s["block_idx"] for s in segments])
            segments = [segments[i] for i in retain_indices(segments)]
            history.append([s["block_idx"] for s in segments])
            continue
        history.append([s["block_idx"] for s in segments])
    return history
