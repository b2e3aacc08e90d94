"""Generate golden vectors by running the TaoMate reference itself on CPU.

Run once in a container where the reference source tree is available:

    TAOMATE_REFERENCE=/path/to/TaoMate python tests/golden/make_golden.py [group ...]

The reference is pure PyTorch; this script imports it, feeds it seeded inputs
and stores the outputs as small ``.npz``/``.json`` files next to this script
(the inputs are rebuilt from numpy seeds by ``inputs.py``).
The tests compare the numpy oracle and the CUDA path against these files; the
reference itself is never needed at test time.  Torch / numpy versions are
recorded in ``versions.json``.
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("TAOMATE_REFERENCE")
sys.path.insert(0, HERE)
import inputs  # noqa: E402


def _import_reference():
    if not REF:
        raise SystemExit("set TAOMATE_REFERENCE to the TaoMate source tree (the directory that "
                         "holds ltx_causal/ and taomate/)")
    if not os.path.isdir(REF):
        raise SystemExit(f"reference tree not found at TAOMATE_REFERENCE={REF}")
    sys.path.insert(0, REF)
    import torch  # noqa: F401
    from ltx_causal.rope import causal_rope
    from ltx_causal.attention.causal_attention import CausalLTXAttention
    from ltx_causal.transformer import kv_cache
    from taomate.inference import cache as tcache
    from ltx_causal.attention.mask_builder import compute_av_blocks
    return causal_rope, CausalLTXAttention, kv_cache, tcache, compute_av_blocks


def f32(t):
    return t.detach().to("cpu").float().numpy()


def gen_rope(causal_rope, torch):
    out = {}
    cases = {
        # name: (grid, dim, heads, start, is_audio, max_pos, extrapolation)
        "c1_video": ((1, 8, 12), 256, 4, 6, False, [20, 2048, 2048], "off"),
        "c2_video": ((3, 16, 24), 4096, 32, 13, False, [20, 2048, 2048], "off"),
        "c2_video_first": ((4, 16, 24), 4096, 32, 0, False, [20, 2048, 2048], "off"),
        "audio": ((25,), 2048, 32, 26, True, [20], "off"),
        "video_cross": ((3,), 2048, 32, 13, False, [20], "off"),
        "c2_video_ntk": ((3, 16, 24), 4096, 32, 200, False, [20, 2048, 2048], "ntk"),
    }
    for name, (grid, dim, heads, start, is_audio, max_pos, ext) in cases.items():
        g = torch.tensor([list(grid)])
        kw = dict(dim=dim, theta=10000.0, max_pos=max_pos, start_frame=start,
                  rope_type=causal_rope.CausalRopeType.SPLIT, device="cpu",
                  is_audio=is_audio, rope_extrapolation=ext, rope_train_max_seconds=8.0,
                  num_attention_heads=heads)
        cos32, sin32 = causal_rope.causal_precompute_freqs_cis(g, dtype=torch.float32, **kw)
        cosbf, sinbf = causal_rope.causal_precompute_freqs_cis(g, dtype=torch.bfloat16, **kw)
        T = cos32.shape[2]
        rows = np.arange(T) if T <= 128 else np.arange(0, T, 17)
        out[f"{name}__rows"] = rows
        out[f"{name}__cos_f32"] = f32(cos32[0])[:, rows]
        out[f"{name}__sin_f32"] = f32(sin32[0])[:, rows]
        out[f"{name}__cos_bf16"] = f32(cosbf[0])[:, rows]
        out[f"{name}__sin_bf16"] = f32(sinbf[0])[:, rows]
        out[f"{name}__meta"] = np.array([*grid, *([0] * (3 - len(grid))), len(grid), dim, heads,
                                         start, int(is_audio), int(ext == "ntk")] + list(max_pos)
                                        + [0] * (3 - len(max_pos)), dtype=np.float64)
    np.savez_compressed(os.path.join(HERE, "rope_tables.npz"), **out)


def gen_split_rope(causal_rope, torch):
    g = torch.tensor([[1, 8, 12]])
    cos, sin = causal_rope.causal_precompute_freqs_cis(g, 256, start_frame=6, device="cpu",
                                                       num_attention_heads=4)
    x = torch.from_numpy(inputs.split_rope_inputs())[None]
    y32 = causal_rope.apply_split_rotary_emb(x, cos, sin)
    ybf = causal_rope.apply_split_rotary_emb(x.bfloat16(), cos.bfloat16(), sin.bfloat16())
    np.savez_compressed(os.path.join(HERE, "split_rope.npz"), y_f32=f32(y32[0]),
                        y_bf16=f32(ybf[0]))


def _attn_case(causal_rope, CausalLTXAttention, kv_cache, torch, name):
    d = inputs.attn_case_inputs(name)
    c, prm = d["cfg"], d["params"]
    heads, dh, hid = c["heads"], c["dim_head"], c["hidden"]
    attn = CausalLTXAttention(hid, None, heads=heads, dim_head=dh,
                              apply_gated_attention=c["gated"])
    with torch.no_grad():
        mods = {"to_q": attn.to_q, "to_k": attn.to_k, "to_v": attn.to_v,
                "to_out": attn.to_out[0]}
        if c["gated"]:
            mods["to_gate_logits"] = attn.to_gate_logits
        for nm, m in mods.items():
            m.weight.copy_(torch.from_numpy(prm[nm + "_w"]))
            m.bias.copy_(torch.from_numpy(prm[nm + "_b"]))
        attn.q_norm.weight.copy_(torch.from_numpy(prm["q_norm_w"]))
        attn.k_norm.weight.copy_(torch.from_numpy(prm["k_norm_w"]))
    x = torch.from_numpy(d["x"])[None]
    ck = None if d["cached_k"] is None else torch.from_numpy(d["cached_k"])[None]
    cv = None if d["cached_v"] is None else torch.from_numpy(d["cached_v"])[None]
    g = torch.tensor([list(c["grid"])])
    cos, sin = causal_rope.causal_precompute_freqs_cis(
        g, heads * dh, start_frame=c["start"], device="cpu", num_attention_heads=heads,
        is_audio=c["audio"], max_pos=[20] if len(c["grid"]) == 1 else None)
    rec = {"cos_f32": f32(cos[0]), "sin_f32": f32(sin[0])}
    for tag, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
        a = attn.to(dt)
        with torch.no_grad():
            out, nk, nv = kv_cache.attention_with_cache(
                a, x.to(dt), None, (cos.to(dt), sin.to(dt)), None,
                None if ck is None else ck.to(dt), None if cv is None else cv.to(dt),
                new_kv_real_len=c["real_len"])
        rec[f"out_{tag}"] = f32(out[0])
        rec[f"new_k_{tag}"] = f32(nk[0])
        rec[f"new_v_{tag}"] = f32(nv[0])
    np.savez_compressed(os.path.join(HERE, f"attn_{name}.npz"), **rec)


def gen_text_cross(CausalLTXAttention, kv_cache, torch):
    """_text_cross_attention_with_kv_cache (kv_cache.py:764-827) with the
    K/V cache switched on, the mask prepared as causal_model.py:551-562 does,
    called twice (miss, then cache hit) in fp32 and bf16."""
    kv_cache._CACHE_TEXT_CROSS_KV = True
    for name in inputs.TEXT_CROSS_CASES:
        d = inputs.text_cross_inputs(name)
        c, prm = d["cfg"], d["params"]
        attn = CausalLTXAttention(c["hidden"], c["ctx_dim"], heads=c["heads"],
                                  dim_head=c["dim_head"], apply_gated_attention=c["gated"])
        attn.eval()
        with torch.no_grad():
            mods = {"to_q": attn.to_q, "to_k": attn.to_k, "to_v": attn.to_v,
                    "to_out": attn.to_out[0]}
            if c["gated"]:
                mods["to_gate_logits"] = attn.to_gate_logits
            for nm, m in mods.items():
                m.weight.copy_(torch.from_numpy(prm[nm + "_w"]))
                m.bias.copy_(torch.from_numpy(prm[nm + "_b"]))
            attn.q_norm.weight.copy_(torch.from_numpy(prm["q_norm_w"]))
            attn.k_norm.weight.copy_(torch.from_numpy(prm["k_norm_w"]))
        rec = {}
        for tag, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
            a = attn.to(dt)
            x = torch.from_numpy(d["x"]).to(dt)
            ctx = torch.from_numpy(d["context"]).to(dt)
            m = torch.from_numpy(d["mask"])
            mask = (m - 1).to(dt).reshape(m.shape[0], 1, -1, m.shape[-1]) * torch.finfo(dt).max
            with torch.no_grad():
                outs = [kv_cache._text_cross_attention_with_kv_cache(
                    a, x, ctx, mask=mask, base_context=ctx, prompt_cache_key=None,
                    cache_name="text", layer_idx=0) for _ in range(2)]
            assert torch.equal(outs[0], outs[1])
            rec[f"out_{tag}"] = f32(outs[0])
        np.savez_compressed(os.path.join(HERE, f"text_cross_{name}.npz"), **rec)


def _load_module(attn, prm, torch):
    with torch.no_grad():
        mods = {"to_q": attn.to_q, "to_k": attn.to_k, "to_v": attn.to_v,
                "to_out": attn.to_out[0]}
        if attn.to_gate_logits is not None:
            mods["to_gate_logits"] = attn.to_gate_logits
        for nm, m in mods.items():
            m.weight.copy_(torch.from_numpy(prm[nm + "_w"]))
            m.bias.copy_(torch.from_numpy(prm[nm + "_b"]))
        attn.q_norm.weight.copy_(torch.from_numpy(prm["q_norm_w"]))
        attn.k_norm.weight.copy_(torch.from_numpy(prm["k_norm_w"]))


def gen_pair(causal_rope, CausalLTXAttention, kv_cache, torch):
    """_cross_modal_pair_attention_with_cache (kv_cache.py:1967-2138) on one
    rank, fp32 and bf16, with the cross RoPE tables built as
    kv_cache.py:2955-2990 builds them (1-D temporal tables, the video one
    repeated per frame token)."""
    for name in inputs.PAIR_CASES:
        d = inputs.pair_case_inputs(name)
        c = d["cfg"]
        H, D = c["heads"], c["dim_head"]
        inner = H * D
        a2v = CausalLTXAttention(c["v_hidden"], c["a_hidden"], heads=H, dim_head=D,
                                 apply_gated_attention=c["gated"][0])
        v2a = CausalLTXAttention(c["a_hidden"], c["v_hidden"], heads=H, dim_head=D,
                                 apply_gated_attention=c["gated"][1])
        _load_module(a2v, d["a2v"], torch)
        _load_module(v2a, d["v2a"], torch)
        vc, vs = causal_rope.causal_precompute_freqs_cis(
            torch.tensor([[c["v_frames"]]]), inner, max_pos=[20], start_frame=c["v_start"],
            device="cpu", is_audio=False, num_attention_heads=H)
        fs = c["frame_seqlen"]
        expand = lambda t: t.unsqueeze(3).expand(-1, -1, -1, fs, -1).reshape(
            t.shape[0], t.shape[1], t.shape[2] * fs, t.shape[3])
        vc, vs = expand(vc), expand(vs)
        ac, as_ = causal_rope.causal_precompute_freqs_cis(
            torch.tensor([[c["la"]]]), inner, max_pos=[20], start_frame=c["a_start"],
            device="cpu", is_audio=True, num_attention_heads=H)
        rec = {"vcos_f32": f32(vc[0]), "vsin_f32": f32(vs[0]), "acos_f32": f32(ac[0]),
               "asin_f32": f32(as_[0])}
        for tag, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
            t = lambda a: None if a is None else torch.from_numpy(a)[None].to(dt)
            cache = kv_cache.LayerKVCache()
            for nm in ("a2v", "v2a"):
                kv = d["caches"][nm]
                if kv is not None:
                    setattr(cache, nm + "_k", t(kv[0]))
                    setattr(cache, nm + "_v", t(kv[1]))
            with torch.no_grad():
                outs = kv_cache._cross_modal_pair_attention_with_cache(
                    a2v.to(dt), v2a.to(dt), t(d["x"]["vx_a2v"]), t(d["x"]["ax_a2v"]),
                    t(d["x"]["ax_v2a"]), t(d["x"]["vx_v2a"]), (vc.to(dt), vs.to(dt)),
                    (ac.to(dt), as_.to(dt)), cache, video_real_len=c["video_real_len"],
                    audio_real_len=c["audio_real_len"], layer_idx=0)
            for key, o in zip(("a2v_out", "a2v_k", "a2v_v", "v2a_out", "v2a_k", "v2a_v"), outs):
                rec[f"{key}_{tag}"] = f32(o[0])
        np.savez_compressed(os.path.join(HERE, f"pair_{name}.npz"), **rec)


def _bf16_bits(t):
    """bf16 tensor -> its raw 16-bit patterns (exact, half the bytes of f32)."""
    return t.detach().to("cpu").contiguous().view(torch_int16()).numpy().view(np.uint16)


def torch_int16():
    import torch
    return torch.int16


def _sampled(rec, key, t, rows):
    """Store rows ``rows`` of a [1, L, ...] output: fp32 as float32, bf16 as bits."""
    import torch
    r = torch.from_numpy(rows)
    sub = t[0].index_select(0, r)
    if t.dtype == torch.bfloat16:
        rec[key] = _bf16_bits(sub)
    else:
        rec[key] = f32(sub)


def gen_full(causal_rope, CausalLTXAttention, kv_cache, torch):
    """The full-size cases (BASELINE configs 2 and 3): attention_with_cache
    and the paired cross-modal attention at their real shapes, on inputs
    already rounded to bf16, in fp32 (the exact answer for those inputs) and
    in bf16 (the reference's deployed precision).  Sampled rows only."""
    for name in inputs.FULL_ATTN_CASES:
        d = inputs.attn_case_inputs(name)
        c, prm = d["cfg"], d["params"]
        heads, dh, hid = c["heads"], c["dim_head"], c["hidden"]
        attn = CausalLTXAttention(hid, None, heads=heads, dim_head=dh,
                                  apply_gated_attention=c["gated"])
        _load_module(attn, prm, torch)
        x = torch.from_numpy(d["x"])[None]
        ck = torch.from_numpy(d["cached_k"])[None]
        cv = torch.from_numpy(d["cached_v"])[None]
        g = torch.tensor([list(c["grid"])])
        cos, sin = causal_rope.causal_precompute_freqs_cis(
            g, heads * dh, start_frame=c["start"], device="cpu", num_attention_heads=heads,
            is_audio=c["audio"], max_pos=[20] if len(c["grid"]) == 1 else None)
        rows_out = inputs.full_rows(c["lq"])
        rows_kv = inputs.full_rows(c["lq"], 48)
        rec = {"rows_out": rows_out, "rows_kv": rows_kv}
        for tag, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
            a = attn.to(dt)
            with torch.no_grad():
                out, nk, nv = kv_cache.attention_with_cache(
                    a, x.to(dt), None, (cos.to(dt), sin.to(dt)), None, ck.to(dt), cv.to(dt),
                    new_kv_real_len=c["real_len"])
            _sampled(rec, f"out_{tag}", out, rows_out)
            _sampled(rec, f"new_k_{tag}", nk, rows_kv)
            _sampled(rec, f"new_v_{tag}", nv, rows_kv)
        np.savez_compressed(os.path.join(HERE, f"full_attn_{name}.npz"), **rec)
        print("full", name, flush=True)
    for name in inputs.FULL_PAIR_CASES:
        d = inputs.pair_case_inputs(name)
        c = d["cfg"]
        H, D = c["heads"], c["dim_head"]
        inner = H * D
        a2v = CausalLTXAttention(c["v_hidden"], c["a_hidden"], heads=H, dim_head=D,
                                 apply_gated_attention=c["gated"][0])
        v2a = CausalLTXAttention(c["a_hidden"], c["v_hidden"], heads=H, dim_head=D,
                                 apply_gated_attention=c["gated"][1])
        _load_module(a2v, d["a2v"], torch)
        _load_module(v2a, d["v2a"], torch)
        vc, vs = causal_rope.causal_precompute_freqs_cis(
            torch.tensor([[c["v_frames"]]]), inner, max_pos=[20], start_frame=c["v_start"],
            device="cpu", is_audio=False, num_attention_heads=H)
        fs = c["frame_seqlen"]
        expand = lambda t: t.unsqueeze(3).expand(-1, -1, -1, fs, -1).reshape(
            t.shape[0], t.shape[1], t.shape[2] * fs, t.shape[3])
        vc, vs = expand(vc), expand(vs)
        ac, as_ = causal_rope.causal_precompute_freqs_cis(
            torch.tensor([[c["la"]]]), inner, max_pos=[20], start_frame=c["a_start"],
            device="cpu", is_audio=True, num_attention_heads=H)
        lv = d["lv"]
        rows = {"a2v_out": inputs.full_rows(lv), "a2v_k": inputs.full_rows(c["la"]),
                "a2v_v": inputs.full_rows(c["la"]), "v2a_out": inputs.full_rows(c["la"]),
                "v2a_k": inputs.full_rows(lv, 48), "v2a_v": inputs.full_rows(lv, 48)}
        rec = {f"rows_{k}": v for k, v in rows.items()}
        for tag, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
            t = lambda a: None if a is None else torch.from_numpy(a)[None].to(dt)
            cache = kv_cache.LayerKVCache()
            for nm in ("a2v", "v2a"):
                kv = d["caches"][nm]
                if kv is not None:
                    setattr(cache, nm + "_k", t(kv[0]))
                    setattr(cache, nm + "_v", t(kv[1]))
            with torch.no_grad():
                outs = kv_cache._cross_modal_pair_attention_with_cache(
                    a2v.to(dt), v2a.to(dt), t(d["x"]["vx_a2v"]), t(d["x"]["ax_a2v"]),
                    t(d["x"]["ax_v2a"]), t(d["x"]["vx_v2a"]), (vc.to(dt), vs.to(dt)),
                    (ac.to(dt), as_.to(dt)), cache, video_real_len=c["video_real_len"],
                    audio_real_len=c["audio_real_len"], layer_idx=0)
            for key, o in zip(("a2v_out", "a2v_k", "a2v_v", "v2a_out", "v2a_k", "v2a_v"), outs):
                _sampled(rec, f"{key}_{tag}", o, rows[key])
        np.savez_compressed(os.path.join(HERE, f"full_pair_{name}.npz"), **rec)
        print("full pair", name, flush=True)


def gen_block(causal_rope, kv_cache, torch):
    """block_forward_with_cache (kv_cache.py:2145-2654) of a real reference
    CausalAVTransformerBlock loaded with the seeded weights (strict state
    dict), fp32 and bf16, with the text K/V cache off (the reference default)
    and the PE tables / per-token AdaLN rows built as model_forward_inference
    builds them (kv_cache.py:2906-3000, 2960-2970)."""
    from ltx_causal.transformer.causal_block import CausalAVTransformerBlock, TransformerConfig
    kv_cache._CACHE_TEXT_CROSS_KV = False
    for name in inputs.BLOCK_CASES:
        d = inputs.block_case_inputs(name)
        c = d["cfg"]
        Dv, Da = c["video_dim"], c["audio_dim"]
        Hv, dv, Ha, da = c["video_heads"], c["video_dim_head"], c["audio_heads"], c["audio_dim_head"]
        blk = CausalAVTransformerBlock(
            0, video=TransformerConfig(dim=Dv, heads=Hv, d_head=dv, context_dim=Dv),
            audio=TransformerConfig(dim=Da, heads=Ha, d_head=da, context_dim=Da))
        blk.load_state_dict({k: torch.from_numpy(v) for k, v in d["params"].items()}, strict=True)
        blk.eval()
        F, fs, La, Lv = c["v_frames"], c["fh"] * c["fw"], c["la"], d["Lv"]
        vpe = causal_rope.causal_precompute_freqs_cis(
            torch.tensor([[F, c["fh"], c["fw"]]]), Hv * dv, start_frame=c["v_start"],
            device="cpu", num_attention_heads=Hv)
        ape = causal_rope.causal_precompute_freqs_cis(
            torch.tensor([[La]]), Ha * da, max_pos=[20], start_frame=c["a_start"], device="cpu",
            is_audio=True, num_attention_heads=Ha)
        vc, vs = causal_rope.causal_precompute_freqs_cis(
            torch.tensor([[F]]), Ha * da, max_pos=[20], start_frame=c["v_start"], device="cpu",
            is_audio=False, num_attention_heads=Ha)
        expand = lambda t: t.unsqueeze(3).expand(-1, -1, -1, fs, -1).reshape(
            t.shape[0], t.shape[1], t.shape[2] * fs, t.shape[3])
        vcpe = (expand(vc), expand(vs))
        acpe = causal_rope.causal_precompute_freqs_cis(
            torch.tensor([[La]]), Ha * da, max_pos=[20], start_frame=c["a_start"], device="cpu",
            is_audio=True, num_attention_heads=Ha)
        x = {k: torch.from_numpy(v)[None] for k, v in d["x"].items()}
        per_tok = lambda t: t.repeat_interleave(fs, dim=1)  # per-frame rows -> per token
        rec = {}
        for tag, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
            b = blk.to(dt)
            cv = lambda t: t.to(dt)
            m = torch.from_numpy(d["mask"])[None]
            mask = (m - 1).to(dt).reshape(1, 1, 1, -1) * torch.finfo(dt).max
            lc = kv_cache.LayerKVCache(**{
                f"{nm}_{kv}": torch.from_numpy(arr)[None].to(dt)
                for nm, pair in d["caches"].items() for kv, arr in zip("kv", pair)})
            with torch.no_grad():
                vx, ax, new = kv_cache.block_forward_with_cache(
                    b, cv(x["video_x"]), cv(x["audio_x"]), cv(per_tok(x["video_ts"])),
                    cv(x["audio_ts"]), tuple(map(cv, vpe)), tuple(map(cv, ape)),
                    tuple(map(cv, vcpe)), tuple(map(cv, acpe)), cv(x["video_ctx"]),
                    cv(x["audio_ctx"]), mask, mask, cv(per_tok(x["video_cross_ss"])),
                    cv(per_tok(x["video_cross_gate"])), cv(x["audio_cross_ss"]),
                    cv(x["audio_cross_gate"]), None, None, None, None, lc, layer_idx=0,
                    video_frame_seqlen=fs, audio_frame_seqlen=1)
            rec[f"video_x_{tag}"] = f32(vx[0])
            rec[f"audio_x_{tag}"] = f32(ax[0])
            for fld, n_new in (("video_self_k", Lv), ("video_self_v", Lv), ("audio_self_k", La),
                               ("audio_self_v", La), ("a2v_k", La), ("a2v_v", La),
                               ("v2a_k", Lv), ("v2a_v", Lv)):
                t = getattr(new, fld)
                rec[f"{fld}_{tag}"] = f32(t[0, -n_new:])
        np.savez_compressed(os.path.join(HERE, f"block_{name}.npz"), **rec)
        print("block", name, flush=True)


def gen_attention(causal_rope, CausalLTXAttention, kv_cache, torch):
    for name in inputs.ATTN_CASES:
        _attn_case(causal_rope, CausalLTXAttention, kv_cache, torch, name)


def gen_cache(kv_cache, tcache, torch, compute_av_blocks):
    """Replay the batch runtime's commit/evict schedule through the reference
    ``retain_streaming_context`` with token-index payloads."""
    blocks = compute_av_blocks(4 + (60 - 1) * 3, num_frame_per_block_first=4)[:60]
    frame_tokens = 6  # small stand-in for 384 tokens per frame; ratios preserved
    segments = []
    layer = kv_cache.LayerKVCache()
    v_next = a_next = 0
    kept, vtok, atok = [], [], []
    for bi, b in enumerate(blocks):
        nv = (b.video_end - b.video_start) * frame_tokens
        na = b.audio_end - b.audio_start
        vid = torch.arange(v_next, v_next + nv, dtype=torch.float32).view(1, nv, 1, 1)
        aud = torch.arange(a_next, a_next + na, dtype=torch.float32).view(1, na, 1, 1)
        v_next += nv
        a_next += na
        cat = kv_cache._cat_cache
        layer = kv_cache.LayerKVCache(
            video_self_k=cat(layer.video_self_k, vid), video_self_v=cat(layer.video_self_v, -vid),
            audio_self_k=cat(layer.audio_self_k, aud), audio_self_v=cat(layer.audio_self_v, -aud),
            a2v_k=cat(layer.a2v_k, aud + 0.5), a2v_v=cat(layer.a2v_v, -aud - 0.5),
            v2a_k=cat(layer.v2a_k, vid + 0.5), v2a_v=cat(layer.v2a_v, -vid - 0.5))
        segments.append({"block_idx": int(b.block_idx), "video_tokens": nv, "audio_tokens": na})
        cache = tcache.attach_segments(kv_cache.KVCache(layers=[layer]), segments)
        window = bi // 5
        if window > 0 or bi == 4:
            if bi == 4:
                kept.append([s["block_idx"] for s in segments])
                vtok.append(cache.layers[0].video_self_k.flatten().tolist())
                atok.append(cache.layers[0].audio_self_k.flatten().tolist())
            cache = tcache.retain_streaming_context(cache)
        layer = cache.layers[0]
        segments = tcache.cache_segments(cache)
        kept.append([s["block_idx"] for s in segments])
        vtok.append(layer.video_self_k.flatten().tolist())
        atok.append(layer.audio_self_k.flatten().tolist())
        for f in ("video_self_v", "v2a_k", "v2a_v"):
            ref = {"video_self_v": -layer.video_self_k, "v2a_k": layer.video_self_k + 0.5,
                   "v2a_v": -layer.video_self_k - 0.5}[f]
            assert torch.equal(getattr(layer, f), ref)
    with open(os.path.join(HERE, "cache_schedule.json"), "w") as fh:
        json.dump({"frame_tokens": frame_tokens, "kept_block_idx": kept,
                   "video_token_ids": vtok, "audio_token_ids": atok,
                   "blocks": [[b.block_idx, b.video_start, b.video_end, b.audio_start, b.audio_end]
                              for b in blocks]}, fh)
    # compute_av_blocks known answers (mask_builder.py:129-140 docstring examples)
    kab = {
        "first4_16": [[b.block_idx, b.video_start, b.video_end, b.audio_start, b.audio_end]
                      for b in compute_av_blocks(16, num_frame_per_block_first=4)],
        "legacy_16": [[b.block_idx, b.video_start, b.video_end, b.audio_start, b.audio_end]
                      for b in compute_av_blocks(16)],
        "first4_partial_18": [[b.block_idx, b.video_start, b.video_end, b.audio_start, b.audio_end]
                              for b in compute_av_blocks(18, num_frame_per_block_first=4)],
    }
    with open(os.path.join(HERE, "av_blocks.json"), "w") as fh:
        json.dump(kab, fh)


def _a2a_worker(rank, world, port, outdir):
    import torch
    import torch.distributed as dist
    sys.path.insert(0, REF)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from taomate.runtime_support.parallel import all_to_all as a2a
    from taomate.runtime_support.parallel import sp_utils
    full_np, full2_np, raw_np = inputs.a2a_inputs()
    full, full2 = torch.from_numpy(full_np), torch.from_numpy(full2_np)
    S = full.shape[1]
    Sl = S // world
    shard = full[:, rank * Sl:(rank + 1) * Sl].contiguous()
    shard2 = full2[:, rank * Sl:(rank + 1) * Sl].contiguous()
    grp = dist.group.WORLD
    s2h = a2a._seq_to_head(shard, world, grp)
    h2s = a2a._head_to_seq(s2h, world, grp)
    with torch.no_grad():
        many = a2a.seq_all_to_all_head_many((shard, shard2), grp, world)
    raw = torch.from_numpy(raw_np)  # odd length -> padded split
    split = sp_utils.split_sequence(raw, dim=1, sp_rank=rank, sp_size=world)
    gathered = sp_utils.gather_sequence(split, dim=1, group=grp, sp_size=world, sp_rank=rank)
    np.savez_compressed(os.path.join(outdir, f"a2a_g{world}_r{rank}.npz"), s2h=s2h.numpy(),
                        h2s=h2s.numpy(), many0=many[0].numpy(), many1=many[1].numpy(),
                        split=split.numpy(), gathered=gathered.numpy())
    dist.barrier()
    dist.destroy_process_group()


def gen_a2a():
    import torch.multiprocessing as mp
    for world, port in ((2, 29611), (4, 29612)):
        mp.spawn(_a2a_worker, args=(world, port, HERE), nprocs=world, join=True)
    merged = {}
    for world in (2, 4):
        for r in range(world):
            p = os.path.join(HERE, f"a2a_g{world}_r{r}.npz")
            with np.load(p) as z:
                for k in z.files:
                    merged[f"g{world}_r{r}__{k}"] = z[k]
            os.remove(p)
    np.savez_compressed(os.path.join(HERE, "a2a.npz"), **merged)


def main():
    causal_rope, CausalLTXAttention, kv_cache, tcache, compute_av_blocks = _import_reference()
    import torch
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    groups = {
        "rope": lambda: gen_rope(causal_rope, torch),
        "split_rope": lambda: gen_split_rope(causal_rope, torch),
        "attention": lambda: gen_attention(causal_rope, CausalLTXAttention, kv_cache, torch),
        "text_cross": lambda: gen_text_cross(CausalLTXAttention, kv_cache, torch),
        "pair": lambda: gen_pair(causal_rope, CausalLTXAttention, kv_cache, torch),
        "cache": lambda: gen_cache(kv_cache, tcache, torch, compute_av_blocks),
        "a2a": gen_a2a,
        "full": lambda: gen_full(causal_rope, CausalLTXAttention, kv_cache, torch),
        "block": lambda: gen_block(causal_rope, kv_cache, torch),
    }
    for name in (sys.argv[1:] or list(groups)):  # e.g. `make_golden.py pair`
        groups[name]()
    import einops
    with open(os.path.join(HERE, "versions.json"), "w") as fh:
        json.dump({"torch": torch.__version__, "numpy": np.__version__,
                   "einops": einops.__version__, "python": sys.version.split()[0]}, fh)


if __name__ == "__main__":
    main()
