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


# Full-size cases at the benchmark's own shapes.  Their inputs and weights are
# rounded to bf16 before use, so the reference's fp32 run is the exact answer
# for the very inputs every bf16 path sees; fixtures keep sampled rows only
# (``full_rows``).
FULL_ATTN_CASES: Dict[str, dict] = {
    # hidden 4096 = 32 x 128, 3 frames of 16 x 24 = 1152 query tokens,
    # 1 anchor + 8 window frames = 3456 cached tokens (4608 keys per query).
    "c2": dict(hidden=4096, heads=32, dim_head=128, lq=1152, lcache=3456, grid=(3, 16, 24),
               start=9, gated=False, init="normal", audio=False, real_len=None, seed=30,
               bf16_inputs=True),
    # The reference's production layout: a 4-frame anchor block + two 3-frame window
    # blocks = 3840 cached tokens (4992 keys), read from three arena slots.
    "c2_prod": dict(hidden=4096, heads=32, dim_head=128, lq=1152, lcache=3840, grid=(3, 16, 24),
                    start=10, gated=False, init="normal", audio=False, real_len=None, seed=31,
                    bf16_inputs=True, cache_blocks=(1536, 1152, 1152)),
    # BASELINE config 3 audio self-attention: hidden 2048 = 32 x 64, 25 tokens over
    # 76 cached (101 keys), 1-D audio RoPE.
    "c3_audio": dict(hidden=2048, heads=32, dim_head=64, lq=25, lcache=76, grid=(25,), start=76,
                     gated=False, init="normal", audio=True, real_len=None, seed=32,
                     bf16_inputs=True),
}


def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), kept as
    float32."""
    b = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    b = (b + np.uint32(0x7FFF) + ((b >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return b.view(np.float32)


def _normal(rng, shape, scale, full):
    """N(0, scale^2) float32; the full-size cases draw float32 directly."""
    if full:
        z = rng.standard_normal(shape, dtype=np.float32)
        return z * np.float32(scale) if scale != 1.0 else z
    return (rng.standard_normal(shape) * scale).astype(np.float32)


def full_rows(n: int, step: int = 24) -> np.ndarray:
    """Row indices a full-size fixture keeps of an ``n``-row output."""
    return np.arange(0, n, step) if n > 2 * step else np.arange(n)


def _xavier(rng, out_f, in_f):
    a = math.sqrt(6.0 / (in_f + out_f))
    return rng.uniform(-a, a, size=(out_f, in_f)).astype(np.float32)


def attn_case_inputs(name: str) -> dict:
    """Seeded inputs for one golden attention case (float32 arrays, batch 1
    dropped).  Weights use torch's ``[out, in]`` layout."""
    c = ATTN_CASES[name] if name in ATTN_CASES else FULL_ATTN_CASES[name]
    full = bool(c.get("bf16_inputs"))
    rng = np.random.default_rng(1000 + c["seed"])
    hid, inner = c["hidden"], c["heads"] * c["dim_head"]
    p = {}
    for nm, (o, i) in {"to_q": (inner, hid), "to_k": (inner, hid), "to_v": (inner, hid),
                       "to_out": (hid, inner)}.items():
        if c["init"] == "xavier":
            p[nm + "_w"] = _xavier(rng, o, i)
            p[nm + "_b"] = np.zeros(o, np.float32)
        else:
            p[nm + "_w"] = _normal(rng, (o, i), 0.02, full)
            p[nm + "_b"] = _normal(rng, (o,), 0.02, full)
    if c["gated"]:
        p["to_gate_logits_w"] = _normal(rng, (c["heads"], hid), 0.02, full)
        p["to_gate_logits_b"] = _normal(rng, (c["heads"],), 0.02, full)
    p["q_norm_w"] = rng.uniform(0.5, 1.5, inner).astype(np.float32)
    p["k_norm_w"] = rng.uniform(0.5, 1.5, inner).astype(np.float32)
    x = _normal(rng, (c["lq"], hid), 1.0, full)
    ck = cv = None
    if c["lcache"]:
        ck = _normal(rng, (c["lcache"], c["heads"], c["dim_head"]), 1.0, full)
        cv = _normal(rng, (c["lcache"], c["heads"], c["dim_head"]), 1.0, full)
    if c.get("bf16_inputs"):
        p = {k: bf16_round(v) for k, v in p.items()}
        x = bf16_round(x)
        ck = None if ck is None else bf16_round(ck)
        cv = None if cv is None else bf16_round(cv)
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


# BASELINE config 3's cross-modal pair: A2V = 1152 video queries (hidden 4096)
# over 76 cached + 25 new audio keys; V2A = 25 audio queries (hidden 2048) over
# 3456 cached + 1152 new video keys (4608); 32 heads x 64, 1-D temporal RoPE.
FULL_PAIR_CASES: Dict[str, dict] = {
    "c3": dict(v_hidden=4096, a_hidden=2048, heads=32, dim_head=64, v_frames=3,
               frame_seqlen=384, la=25, a2v_cache=76, v2a_cache=3456, v_start=9, a_start=76,
               gated=(False, False), video_real_len=None, audio_real_len=None, seed=40,
               bf16_inputs=True),
}


def _pair_attn_params(rng, q_dim, kv_dim, inner, heads, gated, full=False):
    p = {}
    for nm, (o, i) in {"to_q": (inner, q_dim), "to_k": (inner, kv_dim), "to_v": (inner, kv_dim),
                       "to_out": (q_dim, inner)}.items():
        p[nm + "_w"] = _normal(rng, (o, i), 0.02, full)
        p[nm + "_b"] = _normal(rng, (o,), 0.02, full)
    if gated:
        p["to_gate_logits_w"] = _normal(rng, (heads, q_dim), 0.02, full)
        p["to_gate_logits_b"] = _normal(rng, (heads,), 0.02, full)
    p["q_norm_w"] = rng.uniform(0.5, 1.5, inner).astype(np.float32)
    p["k_norm_w"] = rng.uniform(0.5, 1.5, inner).astype(np.float32)
    return p


def pair_case_inputs(name: str) -> dict:
    """Seeded inputs of a paired cross-modal case: the A2V module (queries
    from video, keys from audio) and the V2A module, the four normed inputs
    ``vx_a2v [Lv, Dv]``, ``ax_a2v [La, Da]``, ``ax_v2a``, ``vx_v2a`` and the
    caches (``a2v`` holds audio keys, ``v2a`` video keys; ``None`` when empty)."""
    c = PAIR_CASES[name] if name in PAIR_CASES else FULL_PAIR_CASES[name]
    rng = np.random.default_rng(3000 + c["seed"])
    H, D = c["heads"], c["dim_head"]
    inner = H * D
    lv = c["v_frames"] * c["frame_seqlen"]
    full = bool(c.get("bf16_inputs"))
    a2v = _pair_attn_params(rng, c["v_hidden"], c["a_hidden"], inner, H, c["gated"][0], full)
    v2a = _pair_attn_params(rng, c["a_hidden"], c["v_hidden"], inner, H, c["gated"][1], full)
    x = {nm: _normal(rng, (n, dim), 1.0, full)
         for nm, n, dim in (("vx_a2v", lv, c["v_hidden"]), ("ax_a2v", c["la"], c["a_hidden"]),
                            ("ax_v2a", c["la"], c["a_hidden"]), ("vx_v2a", lv, c["v_hidden"]))}
    caches = {}
    for nm in ("a2v", "v2a"):
        n = c[nm + "_cache"]
        caches[nm] = None if n == 0 else tuple(
            _normal(rng, (n, H, D), 1.0, full) for _ in range(2))
    if c.get("bf16_inputs"):
        a2v = {k: bf16_round(v) for k, v in a2v.items()}
        v2a = {k: bf16_round(v) for k, v in v2a.items()}
        x = {k: bf16_round(v) for k, v in x.items()}
        caches = {k: None if kv is None else tuple(bf16_round(t) for t in kv)
                  for k, kv in caches.items()}
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


# One whole transformer block (block_forward_with_cache, kv_cache.py:2145-2654)
# at small shapes: video 4 heads x 128, audio 4 heads x 64, FFN x4, filled caches,
# a padded text context.  AdaLN parameters per video frame / per audio token.
BLOCK_CASES: Dict[str, dict] = {
    "small": dict(video_dim=512, video_heads=4, video_dim_head=128, audio_dim=256,
                  audio_heads=4, audio_dim_head=64, v_frames=2, fh=8, fw=12, la=16, ctx_len=24,
                  ctx_valid=20, v_cache=288, a_cache=32, v_start=3, a_start=26, seed=50),
}


def block_param_shapes(c: dict) -> Dict[str, tuple]:
    """Parameter names and shapes of one block, in the state-dict layout of the
    reference's CausalAVTransformerBlock (and of taomate_b200.block.BlockWeights)."""
    Dv, Da = c["video_dim"], c["audio_dim"]
    iv = c["video_heads"] * c["video_dim_head"]
    ia = c["audio_heads"] * c["audio_dim_head"]
    shapes: Dict[str, tuple] = {}

    def attn(name, q_dim, kv_dim, inner):
        for lin, (o, i) in (("to_q", (inner, q_dim)), ("to_k", (inner, kv_dim)),
                            ("to_v", (inner, kv_dim)), ("to_out.0", (q_dim, inner))):
            shapes[f"{name}.{lin}.weight"] = (o, i)
            shapes[f"{name}.{lin}.bias"] = (o,)
        shapes[f"{name}.q_norm.weight"] = (inner,)
        shapes[f"{name}.k_norm.weight"] = (inner,)

    def ff(name, dim):
        shapes[f"{name}.net.0.proj.weight"] = (4 * dim, dim)
        shapes[f"{name}.net.0.proj.bias"] = (4 * dim,)
        shapes[f"{name}.net.2.weight"] = (dim, 4 * dim)
        shapes[f"{name}.net.2.bias"] = (dim,)

    attn("attn1", Dv, Dv, iv)
    attn("attn2", Dv, Dv, iv)
    ff("ff", Dv)
    shapes["scale_shift_table"] = (6, Dv)
    attn("audio_attn1", Da, Da, ia)
    attn("audio_attn2", Da, Da, ia)
    ff("audio_ff", Da)
    shapes["audio_scale_shift_table"] = (6, Da)
    attn("audio_to_video_attn", Dv, Da, ia)
    attn("video_to_audio_attn", Da, Dv, ia)
    shapes["scale_shift_table_a2v_ca_audio"] = (5, Da)
    shapes["scale_shift_table_a2v_ca_video"] = (5, Dv)
    return shapes


def block_case_inputs(name: str) -> dict:
    """Seeded inputs of a block case, all rounded to bf16: ``params`` (state
    dict), activations ``video_x [Lv, Dv]`` / ``audio_x [La, Da]``, AdaLN rows
    (video per frame, audio per token), text contexts and key mask, caches."""
    c = BLOCK_CASES[name]
    rng = np.random.default_rng(5000 + c["seed"])
    p = {}
    for nm, shp in block_param_shapes(c).items():
        if nm.endswith("norm.weight"):
            p[nm] = rng.uniform(0.5, 1.5, shp).astype(np.float32)
        elif "scale_shift_table" in nm:
            p[nm] = (rng.standard_normal(shp) * 0.1).astype(np.float32)
        else:
            p[nm] = (rng.standard_normal(shp) * 0.02).astype(np.float32)
    Dv, Da = c["video_dim"], c["audio_dim"]
    F, fs, La = c["v_frames"], c["fh"] * c["fw"], c["la"]
    Lv = F * fs
    g = lambda *s: rng.standard_normal(s).astype(np.float32)
    d = dict(
        video_x=g(Lv, Dv), audio_x=g(La, Da),
        video_ts=g(F, 6 * Dv) * 0.1, audio_ts=g(La, 6 * Da) * 0.1,
        video_cross_ss=g(F, 4 * Dv) * 0.1, video_cross_gate=g(F, Dv) * 0.1,
        audio_cross_ss=g(La, 4 * Da) * 0.1, audio_cross_gate=g(La, Da) * 0.1,
        video_ctx=g(c["ctx_len"], Dv), audio_ctx=g(c["ctx_len"], Da))
    Hv, dv, Ha, da = c["video_heads"], c["video_dim_head"], c["audio_heads"], c["audio_dim_head"]
    caches = {"video_self": (g(c["v_cache"], Hv, dv), g(c["v_cache"], Hv, dv)),
              "audio_self": (g(c["a_cache"], Ha, da), g(c["a_cache"], Ha, da)),
              "a2v": (g(c["a_cache"], Ha, da), g(c["a_cache"], Ha, da)),
              "v2a": (g(c["v_cache"], Ha, da), g(c["v_cache"], Ha, da))}
    mask = np.zeros(c["ctx_len"], np.int64)
    mask[:c["ctx_valid"]] = 1
    r = bf16_round
    return dict(cfg=c, params={k: r(v) for k, v in p.items()},
                x={k: r(v) for k, v in d.items()},
                caches={k: (r(a), r(b)) for k, (a, b) in caches.items()}, mask=mask,
                Lv=Lv, frame_seqlen=fs)
