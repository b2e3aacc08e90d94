"""RoPE for the causal-LTX streaming path, on the sm_100a kernels.

Same call signatures as ``ltx_causal/rope/causal_rope.py``:
``causal_precompute_freqs_cis`` (:139) builds the SPLIT cos/sin tables on the
device (one kernel per batch row instead of a Python loop of ~20 small torch
ops) and ``apply_split_rotary_emb`` (:102) rotates ``[B, T, H*D]`` activations
in one fused pass.
"""

from __future__ import annotations

import ctypes
import math
from enum import Enum
from typing import List, Optional, Tuple, Union

import torch

from . import _lib

# Physical-coordinate constants, ltx_causal/rope/causal_rope.py:32-37.
_VIDEO_TEMPORAL_SCALE = 8
_VIDEO_FPS = 24
_AUDIO_DOWNSAMPLE_FACTOR = 4
_AUDIO_HOP_LENGTH = 160
_AUDIO_SAMPLE_RATE = 16000


class CausalRopeType(Enum):
    """RoPE layout (causal_rope.py:20-23).  Only SPLIT, the layout the shipped
    loader selects (taomate/inference/model.py:38), is built."""
    INTERLEAVED = "interleaved"
    SPLIT = "split"


def ntk_theta(theta: float, dim: int, start_frame: int, max_latent_f: int, is_audio: bool,
              rope_train_max_seconds: float) -> float:
    """NTK-aware effective theta, same host arithmetic as causal_rope.py:199-246."""
    theta_eff = float(theta)
    max_latent_abs = int(start_frame) + int(max_latent_f)
    if max_latent_abs > 0:
        if is_audio:
            mel_end = max(0.0, max_latent_abs * _AUDIO_DOWNSAMPLE_FACTOR + 1 - _AUDIO_DOWNSAMPLE_FACTOR)
            t_max_seconds = mel_end * _AUDIO_HOP_LENGTH / _AUDIO_SAMPLE_RATE
        else:
            pixel_end = max(0.0, max_latent_abs * _VIDEO_TEMPORAL_SCALE + 1 - _VIDEO_TEMPORAL_SCALE)
            t_max_seconds = pixel_end / _VIDEO_FPS
        train_max = max(float(rope_train_max_seconds), 1e-6)
        ratio = max(1.0, t_max_seconds / train_max)
        if ratio > 1.0:
            exponent = float(dim) / max(float(dim - 2), 1.0)
            theta_eff = float(theta) * (ratio ** exponent)
    return theta_eff


def causal_precompute_freqs_cis(
    grid_sizes: torch.Tensor,
    dim: int,
    theta: float = 10000.0,
    max_pos: Optional[List[int]] = None,
    start_frame: int = 0,
    rope_type: CausalRopeType = CausalRopeType.SPLIT,
    device: Union[torch.device, str] = "cuda",
    dtype: torch.dtype = torch.float32,
    is_audio: bool = False,
    rope_extrapolation: str = "off",
    rope_train_max_seconds: float = 8.0,
    num_attention_heads: int = 32,
    repeat_per_frame: int = 1,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """SPLIT cos/sin tables ``[B, H, T, dim // 2 // H]`` (causal_rope.py:139-357).

    ``repeat_per_frame > 1`` additionally expands each temporal position to
    that many tokens, which is what the model forward does for the
    cross-modal PE (ltx_causal/transformer/kv_cache.py:2973-2983), without
    materialising the un-expanded table first.
    """
    if max_pos is None:
        max_pos = [20, 2048, 2048]
    if rope_type != CausalRopeType.SPLIT:
        raise NotImplementedError("only SPLIT RoPE tables are built on the device")
    if rope_extrapolation not in ("off", "ntk"):
        raise ValueError(f"rope_extrapolation must be 'off' or 'ntk', got {rope_extrapolation!r}")
    if dtype not in (torch.bfloat16, torch.float32):
        raise NotImplementedError(f"table dtype {dtype}")
    device = torch.device(device)
    if device.type != "cuda":
        raise RuntimeError("causal_precompute_freqs_cis runs on a CUDA device")
    if grid_sizes.ndim == 3:
        grid_sizes = (grid_sizes[..., 0] + grid_sizes[..., 1]) / 2.0
    grid = grid_sizes.detach().to("cpu")
    B, n_pos = int(grid.shape[0]), int(grid.shape[1])
    if n_pos not in (1, 3):
        raise ValueError(f"Unsupported num_pos_dims: {n_pos}")
    theta_eff = float(theta)
    if rope_extrapolation == "ntk":
        try:
            max_latent_f_local = int(grid[:, 0].max().item())
        except RuntimeError:
            max_latent_f_local = 0
        theta_eff = ntk_theta(theta, dim, start_frame, max_latent_f_local, is_audio,
                              rope_train_max_seconds)
    rows = [[int(v) for v in grid[b].tolist()] for b in range(B)]
    T = math.prod(rows[0]) * int(repeat_per_frame)
    if any(math.prod(r) * int(repeat_per_frame) != T for r in rows):
        raise ValueError("all batch rows must describe the same number of tokens")
    hp = dim // 2 // num_attention_heads
    cos = torch.empty(B, num_attention_heads, T, hp, device=device, dtype=dtype)
    sin = torch.empty_like(cos)
    lib = _lib.load()
    mp = (ctypes.c_double * 3)(*[float(v) for v in list(max_pos)[:n_pos]] + [0.0] * (3 - n_pos))
    out_dt = _lib.TM_DTYPE_BF16 if dtype == torch.bfloat16 else _lib.TM_DTYPE_F32
    with torch.cuda.device(device):
        stream = _lib.stream_ptr(device)
        for b in range(B):
            g = (ctypes.c_int64 * 3)(*rows[b] + [0] * (3 - n_pos))
            _lib.check(lib.tm_rope_tables_split(cos[b].data_ptr(), sin[b].data_ptr(), out_dt, n_pos,
                                                g, int(dim), int(num_attention_heads), theta_eff,
                                                mp, int(start_frame), int(bool(is_audio)),
                                                int(repeat_per_frame), stream),
                       "causal_precompute_freqs_cis")
            _lib.launched()
    return cos, sin


def _pe_strides(cos: torch.Tensor) -> Tuple[int, int, int]:
    """Element strides (batch, head, token) of a [B, H, T, D/2] table."""
    if cos.stride(-1) != 1:
        raise ValueError("cos/sin tables must be contiguous in the last dim")
    return cos.stride(0) if cos.shape[0] > 1 else 0, cos.stride(1), cos.stride(2)


def norm_rope(xs, weights, pes, heads: int, dim_head: int, eps: float, sp_size: int = 1,
              packed: bool = False, peer=None, inplace: bool = False):
    """Fused RMSNorm + split RoPE over up to four ``[B, L, H*D]`` bf16 tensors
    in one launch (weight ``None`` skips the norm, pe ``None`` skips the
    rotation, both ``None`` is a layout copy).

    ``sp_size == 1``: returns one ``[B, L, H, D]`` tensor per input.
    ``sp_size > 1``: the store writes the Ulysses seq->head send layout.  With
    ``packed=True`` all jobs share one buffer ``[sp, B, L, n, H/sp, D]`` (job
    ``j`` at index ``j`` of dim 3), which is returned alone; otherwise each job
    gets its own ``[sp, B, L, H/sp, D]`` buffer.  With ``peer`` (a
    :class:`taomate_b200.parallel.PeerExchange`, packed jobs only) the kernel
    stores head group g straight into rank g's receive buffer, at this rank's
    slot; the caller then runs ``peer.exchange(0)`` and reads ``peer.recv``.

    ``inplace=True`` (``sp_size == 1`` only) writes each result over its input
    rows and returns ``[B, L, H, D]`` views of the inputs: every thread of the
    kernel stores exactly the 16-byte chunks it loaded, after loading them, so
    rows with any row stride (e.g. column slices of a fused QKV projection)
    are safe to overwrite.
    """
    dev = _lib.require_cuda(*xs)
    B = int(xs[0].shape[0])
    n = len(xs)
    Hl = heads // sp_size
    L0 = int(xs[0].shape[1])
    if peer is not None:
        if not packed or n != 3 or not peer.fits(B, L0, heads, dim_head) or sp_size != peer.sp:
            raise ValueError("peer stores need the exchange's packed Q/K/V shapes")
        buf = peer.recv
    elif packed:
        if any(int(x.shape[1]) != L0 for x in xs):
            raise ValueError("packed send buffer needs equal lengths")
        buf = torch.empty(sp_size, B, L0, n, Hl, dim_head, device=dev, dtype=torch.bfloat16)
    if inplace and (sp_size != 1 or packed or peer is not None):
        raise ValueError("in-place norm_rope is for the unsharded layout only")
    jobs = (_lib.NormRopeJob * n)()
    keep = []
    outs = []
    for i, x in enumerate(xs):
        if x.dtype != torch.bfloat16:
            raise TypeError(f"expected bfloat16 activations, got {x.dtype}")
        if x.dim() != 3 or x.shape[-1] != heads * dim_head or x.stride(-1) != 1:
            raise ValueError(f"expected [B, L, {heads * dim_head}] rows, got {tuple(x.shape)}")
        L = int(x.shape[1])
        j = jobs[i]
        if peer is not None:
            o = buf[peer.rank, :, :, i]  # this rank's slot; group g adds rank g's offset
            j.out = o.data_ptr()
            j.out_group_stride, j.out_batch_stride, j.out_row_stride = 0, buf.stride(1), buf.stride(2)
        elif packed:
            o = buf[:, :, :, i]
            j.out = o.data_ptr()
            j.out_group_stride, j.out_batch_stride, j.out_row_stride = buf.stride(0), buf.stride(1), buf.stride(2)
        elif sp_size > 1:
            o = torch.empty(sp_size, B, L, Hl, dim_head, device=dev, dtype=torch.bfloat16)
            outs.append(o)
            j.out = o.data_ptr()
            j.out_group_stride, j.out_batch_stride, j.out_row_stride = o.stride(0), o.stride(1), o.stride(2)
        elif inplace:
            o = x.view(B, L, heads, dim_head)
            outs.append(o)
            j.out = o.data_ptr()
            j.out_group_stride, j.out_batch_stride, j.out_row_stride = 0, x.stride(0), x.stride(1)
        else:
            o = torch.empty(B, L, heads, dim_head, device=dev, dtype=torch.bfloat16)
            outs.append(o)
            j.out = o.data_ptr()
            j.out_group_stride, j.out_batch_stride, j.out_row_stride = 0, o.stride(0), o.stride(1)
        j.x = x.data_ptr()
        j.x_batch_stride = x.stride(0) if B > 1 else 0
        j.x_row_stride = x.stride(1)
        w = weights[i]
        if w is not None:
            w = w.to(torch.bfloat16).contiguous()
            j.norm_weight = w.data_ptr()
            keep.append(w)
        pe = pes[i]
        if pe is not None:
            c, s = pe
            if c.dtype != torch.bfloat16:
                c, s = c.to(torch.bfloat16), s.to(torch.bfloat16)
            if c.dim() != 4 or c.shape[1] != heads or c.shape[2] != L or c.shape[3] * 2 != dim_head:
                raise ValueError(f"cos/sin must be [B, {heads}, {L}, {dim_head // 2}], "
                                 f"got {tuple(c.shape)}")
            if s.stride() != c.stride():
                s = s.contiguous()
                c = c.contiguous()
            j.cos, j.sin = c.data_ptr(), s.data_ptr()
            j.pe_batch_stride, j.pe_head_stride, j.pe_row_stride = _pe_strides(c)
            keep.append((c, s))
        j.L = L
    lib = _lib.load()
    with torch.cuda.device(dev):
        if peer is not None:
            _lib.check(lib.tm_norm_rope_peer(jobs, n, B, int(heads), int(dim_head), float(eps),
                                             int(sp_size), peer.delta["recv"],
                                             _lib.stream_ptr(dev)), "norm_rope")
        else:
            _lib.check(lib.tm_norm_rope(jobs, n, B, int(heads), int(dim_head), float(eps),
                                        int(sp_size), _lib.stream_ptr(dev)), "norm_rope")
        _lib.launched()
    return buf if packed else outs


def apply_split_rotary_emb(input_tensor: torch.Tensor, cos_freqs: torch.Tensor,
                           sin_freqs: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE (causal_rope.py:102-132) for ``[B, T, H*D]`` input
    with ``[B, H, T, D/2]`` tables; returns ``[B, T, H*D]``."""
    if input_tensor.ndim != 3 or cos_freqs.ndim != 4:
        raise NotImplementedError("the fused kernel takes [B, T, H*D] input with [B, H, T, D/2] "
                                  "tables (the layout attention_with_cache uses)")
    b, h, t, half = cos_freqs.shape
    out = norm_rope([input_tensor], [None], [(cos_freqs, sin_freqs)], h, 2 * half, 0.0)[0]
    return out.view(input_tensor.shape[0], t, h * 2 * half)
