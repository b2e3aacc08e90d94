"""Deterministic inputs shared by the golden generator and the tests.

Every golden case is rebuilt from a numpy ``default_rng`` seed, so the
fixtures only hold the reference's outputs.  ``make_golden.py`` feeds these
exact arrays to the reference; the tests feed them to the oracle and to the
CUDA path.
"""

from __future__ import annotations

import math
from typing import Dict

import numpy as np

# name: hidden, heads, dim_head, q_len, cache_len, rope grid, start_frame,
#       gated, init, audio rope, new_kv_real_len, compute dtypes
ATTN_CASES: Dict[str, dict] = {
    # Config 1 (CPU fp32): hidden 256, 4 x 64, one 8x12 query frame, six cached frames.
    "c1": dict(hidden=256, heads=4, dim_head=64, lq=96, lcache=576, grid=(1, 8, 12), start=6,
               gated=False, init="xavier", audio=False, real_len=None, seed=0),
    # Head dim 128 with ragged lengths (query 160, cache 300).
    "d128": dict(hidden=512, heads=4, dim_head=128, lq=160, lcache=300, grid=(1, 10, 16), start=5,
                 gated=False, init="normal", audio=False, real_len=None, seed=1),
    # Per-head gated attention, empty cache (first block).
    "gated": dict(hidden=256, heads=4, dim_head=64, lq=96, lcache=0, grid=(1, 8, 12), start=0,
                  gated=True, init="normal", audio=False, real_len=None, seed=2),
    # Audio-like: 28 padded query rows, real K/V length 25, 101 cached, 1-D audio RoPE.
    "audio": dict(hidden=512, heads=8, dim_head=64, lq=28, lcache=101, grid=(28,), start=26,
                  gated=False, init="normal", audio=True, real_len=25, seed=3),
}


def _xavier(rng, out_f, in_f):
    a = math.sqrt(6.0 / (in_f + out_f))
    return rng.uniform(-a, a, size=(out_f, in_f)).astype(np.float32)


def attn_case_inputs(name: str) -> dict:
    """Seeded inputs for one golden attention case (float32 arrays, batch 1
    dropped).  Weights use torch's ``[out, in]`` layout."""
    c = ATTN_CASES[name]
    rng = np.random.default_rng(1000 + c["seed"])
    hid, inner = c["hidden"], c["heads"] * c["dim_head"]
    p = {}
    for nm, (o, i) in {"to_q": (inner, hid), "to_k": (inner, hid), "to_v": (inner, hid),
                       "to_out": (hid, inner)}.items():
        if c["init"] == "xavier":
            p[nm + "_w"] = _xavier(rng, o, i)
            p[nm + "_b"] = np.zeros(o, np.float32)
        else:
            p[nm + "_w"] = (rng.standard_normal((o, i)) * 0.02).astype(np.float32)
            p[nm + "_b"] = (rng.standard_normal(o) * 0.02).astype(np.float32)
    if c["gated"]:
        p["to_gate_logits_w"] = (rng.standard_normal((c["heads"], hid)) * 0.02).astype(np.float32)
        p["to_gate_logits_b"] = (rng.standard_normal(c["heads"]) * 0.02).astype(np.float32)
    p["q_norm_w"] = rng.uniform(0.5, 1.5, inner).astype(np.float32)
    p["k_norm_w"] = rng.uniform(0.5, 1.5, inner).astype(np.float32)
    x = rng.standard_normal((c["lq"], hid)).astype(np.float32)
    ck = cv = None
    if c["lcache"]:
        ck = rng.standard_normal((c["lcache"], c["heads"], c["dim_head"])).astype(np.float32)
        cv = rng.standard_normal((c["lcache"], c["heads"], c["dim_head"])).astype(np.float32)
    return dict(cfg=c, params=p, x=x, cached_k=ck, cached_v=cv)


# Text cross-attention (kv_cache.py:764-827): video queries against a padded
# text context; per-batch key-padding masks as _prepare_attention_mask builds them.
TEXT_CROSS_CASES: Dict[str, dict] = {
    "plain": dict(hidden=256, ctx_dim=384, heads=4, dim_head=64, lq=96, lk=48, batch=2,
                  valid=(40, 48), gated=False, seed=10),
    "gated": dict(hidden=256, ctx_dim=384, heads=4, dim_head=64, lq=96, lk=48, batch=1,
                  valid=(33,), gated=True, seed=11),
    "d128": dict(hidden=512, ctx_dim=256, heads=4, dim_head=128, lq=130, lk=70, batch=1,
                 valid=(70,), gated=False, seed=12),
}


def text_cross_inputs(name: str) -> dict:
    """Seeded inputs of a text cross-attention case: weights ([out, in]),
    x ``[B, lq, hidden]``, context ``[B, lk, ctx_dim]`` and the 0/1 key mask
    ``[B, lk]`` (valid keys first, then padding)."""
    c = TEXT_CROSS_CASES[name]
    rng = np.random.default_rng(2000 + c["seed"])
    hid, ctx, inner = c["hidden"], c["ctx_dim"], c["heads"] * c["dim_head"]
    p = {}
    for nm, (o, i) in {"to_q": (inner, hid), "to_k": (inner, ctx), "to_v": (inner, ctx),
                       "to_out": (hid, inner)}.items():
        p[nm + "_w"] = (rng.standard_normal((o, i)) * 0.02).astype(np.float32)
        p[nm + "_b"] = (rng.standard_normal(o) * 0.02).astype(np.float32)
    if c["gated"]:
        p["to_gate_logits_w"] = (rng.standard_normal((c["heads"], hid)) * 0.02).astype(np.float32)
        p["to_gate_logits_b"] = (rng.standard_normal(c["heads"]) * 0.02).astype(np.float32)
    p["q_norm_w"] = rng.uniform(0.5, 1.5, inner).astype(np.float32)
    p["k_norm_w"] = rng.uniform(0.5, 1.5, inner).astype(np.float32)
    B = c["batch"]
    x = rng.standard_normal((B, c["lq"], hid)).astype(np.float32)
    context = rng.standard_normal((B, c["lk"], ctx)).astype(np.float32)
    mask = np.zeros((B, c["lk"]), np.int64)
    for b, n in enumerate(c["valid"]):
        mask[b, :n] = 1
    return dict(cfg=c, params=p, x=x, context=context, mask=mask)


# Paired A2V / V2A cross-modal attention (kv_cache.py:1967-2138): video
# queries against audio keys and audio queries against video keys, both with
# 1-D temporal cross RoPE and their own caches.
PAIR_CASES: Dict[str, dict] = {
    # 2 video frames of 48 tokens, 25 audio tokens, both caches filled.
    "av": dict(v_hidden=384, a_hidden=256, heads=4, dim_head=64, v_frames=2, frame_seqlen=48,
               la=25, a2v_cache=50, v2a_cache=96, v_start=3, a_start=75, gated=(False, True),
               video_real_len=None, audio_real_len=None, seed=20),
    # Audio padded to 28 rows (as under sequence parallelism), real length 25;
    # empty caches (first block).
    "strip": dict(v_hidden=256, a_hidden=256, heads=4, dim_head=64, v_frames=1, frame_seqlen=96,
                  la=28, a2v_cache=0, v2a_cache=0, v_start=0, a_start=0, gated=(True, False),
                  video_real_len=None, audio_real_len=25, seed=21),
}


def _pair_attn_params(rng, q_dim, kv_dim, inner, heads, gated):
    p = {}
    for nm, (o, i) in {"to_q": (inner, q_dim), "to_k": (inner, kv_dim), "to_v": (inner, kv_dim),
                       "to_out": (q_dim, inner)}.items():
        p[nm + "_w"] = (rng.standard_normal((o, i)) * 0.02).astype(np.float32)
        p[nm + "_b"] = (rng.standard_normal(o) * 0.02).astype(np.float32)
    if gated:
        p["to_gate_logits_w"] = (rng.standard_normal((heads, q_dim)) * 0.02).astype(np.float32)
        p["to_gate_logits_b"] = (rng.standard_normal(heads) * 0.02).astype(np.float32)
    p["q_norm_w"] = rng.uniform(0.5, 1.5, inner).astype(np.float32)
    p["k_norm_w"] = rng.uniform(0.5, 1.5, inner).astype(np.float32)
    return p


def pair_case_inputs(name: str) -> dict:
    """Seeded inputs of a paired cross-modal case: the A2V module (queries
    from video, keys from audio) and the V2A module, the four normed inputs
    ``vx_a2v [Lv, Dv]``, ``ax_a2v [La, Da]``, ``ax_v2a``, ``vx_v2a`` and the
    caches (``a2v`` holds audio keys, ``v2a`` video keys; ``None`` when empty)."""
    c = PAIR_CASES[name]
    rng = np.random.default_rng(3000 + c["seed"])
    H, D = c["heads"], c["dim_head"]
    inner = H * D
    lv = c["v_frames"] * c["frame_seqlen"]
    a2v = _pair_attn_params(rng, c["v_hidden"], c["a_hidden"], inner, H, c["gated"][0])
    v2a = _pair_attn_params(rng, c["a_hidden"], c["v_hidden"], inner, H, c["gated"][1])
    x = {nm: rng.standard_normal((n, dim)).astype(np.float32)
         for nm, n, dim in (("vx_a2v", lv, c["v_hidden"]), ("ax_a2v", c["la"], c["a_hidden"]),
                            ("ax_v2a", c["la"], c["a_hidden"]), ("vx_v2a", lv, c["v_hidden"]))}
    caches = {}
    for nm in ("a2v", "v2a"):
        n = c[nm + "_cache"]
        caches[nm] = None if n == 0 else tuple(
            rng.standard_normal((n, H, D)).astype(np.float32) for _ in range(2))
    return dict(cfg=c, a2v=a2v, v2a=v2a, x=x, caches=caches, lv=lv)


def split_rope_inputs() -> np.ndarray:
    """x ``[96, 256]`` for the split-RoPE case (C1 shapes)."""
    return np.random.default_rng(77).standard_normal((96, 256)).astype(np.float32)


def a2a_inputs():
    """Full (unsharded) tensors for the all-to-all cases."""
    rng = np.random.default_rng(1234)
    full = rng.standard_normal((1, 24, 8, 4)).astype(np.float32)
    full2 = rng.standard_normal((1, 24, 8, 4)).astype(np.float32)
    raw = rng.standard_normal((1, 25, 6)).astype(np.float32)
    return full, full2, raw
