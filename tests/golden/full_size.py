"""Full-size parity of the CUDA path against the reference's own outputs.

Test infrastructure: the GPU tests and ``__graft_entry__.smoke()`` call
these.  The fixtures (``full_attn_*.npz``, ``full_pair_*.npz``) are made by
``make_golden.py full``, which runs the TaoMate reference on CPU at the
benchmark's own shapes (BASELINE configs 2 and 3) on inputs already rounded
to bf16, twice: in fp32 (the exact answer for those inputs, "gold") and in
bf16 (the reference's deployed precision).  Sampled rows only; bf16 outputs
are stored as their 16-bit patterns.

Each run returns, per output, three relative L2 figures over the sampled rows:
  ours  - this library's bf16 output against gold;
  ref   - the reference's bf16 output against gold (the reference's own error);
  cross - this library's output against the reference's bf16 output.
"""

from __future__ import annotations

import os
from typing import Dict

import numpy as np
import torch

import inputs

HERE = os.path.dirname(os.path.abspath(__file__))


def bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


class _Lin(torch.nn.Module):
    def __init__(self, w, b, dev):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.from_numpy(w).to(dev, torch.bfloat16),
                                         requires_grad=False)
        self.bias = torch.nn.Parameter(torch.from_numpy(b).to(dev, torch.bfloat16),
                                       requires_grad=False)

    def forward(self, x):
        return torch.nn.functional.linear(x, self.weight, self.bias)


def make_module(p: dict, heads: int, dim_head: int, gated: bool, dev) -> torch.nn.Module:
    """An object with the attribute names of the reference's
    ``CausalLTXAttention`` holding the case's weights in bf16 on ``dev``."""
    attn = torch.nn.Module()
    attn.heads, attn.dim_head = heads, dim_head
    attn.to_q = _Lin(p["to_q_w"], p["to_q_b"], dev)
    attn.to_k = _Lin(p["to_k_w"], p["to_k_b"], dev)
    attn.to_v = _Lin(p["to_v_w"], p["to_v_b"], dev)
    attn.to_out = torch.nn.Sequential(_Lin(p["to_out_w"], p["to_out_b"], dev))
    inner = heads * dim_head
    attn.q_norm = torch.nn.RMSNorm(inner, eps=1e-6).to(dev, torch.bfloat16)
    attn.k_norm = torch.nn.RMSNorm(inner, eps=1e-6).to(dev, torch.bfloat16)
    with torch.no_grad():
        attn.q_norm.weight.copy_(torch.from_numpy(p["q_norm_w"]))
        attn.k_norm.weight.copy_(torch.from_numpy(p["k_norm_w"]))
    attn.to_gate_logits = (_Lin(p["to_gate_logits_w"], p["to_gate_logits_b"], dev)
                           if gated else None)
    return attn


def _figures(z, key: str, ours: torch.Tensor, rows: np.ndarray) -> Dict[str, float]:
    got = ours[0].index_select(0, torch.from_numpy(rows).to(ours.device)).float().cpu().numpy()
    gold = z[f"{key}_f32"]
    ref = bits_to_f32(z[f"{key}_bf16"])
    return {"ours": rel_l2(got, gold), "ref": rel_l2(ref, gold), "cross": rel_l2(got, ref)}


def arena_cache(ck: torch.Tensor, cv: torch.Tensor, blocks, dev):
    """The cached rows as an arena view: one slot per block, written in an
    order that leaves the blocks out of order and apart in the arena (the
    anchor block lands after the window blocks, with unused rows between)."""
    from taomate_b200.kv_cache import KVArena, arena_pair
    H, D = int(ck.shape[2]), int(ck.shape[3])
    arena = KVArena(len(blocks) + 1, max(blocks), 1, H, D, device=dev)
    starts = np.cumsum([0] + list(blocks))[:-1]
    ents = {}
    for i in list(range(1, len(blocks))) + [0]:
        s, n = int(starts[i]), int(blocks[i])
        ents[i] = arena.write(ck[:, s:s + n].contiguous(), cv[:, s:s + n].contiguous())
    entries = [e for i in range(len(blocks)) for e in ents[i]]
    k, v = arena_pair(arena, entries)
    for i in range(len(blocks)):  # the views hold the slots now
        for (slot, _, _) in ents[i]:
            arena._ref(slot, -1)
    return k, v


def run_attention_case(name: str, dev, fused: bool = True) -> Dict[str, Dict[str, float]]:
    """``attention_with_cache`` at a full-size case through the public API."""
    import taomate_b200 as tm
    d = inputs.attn_case_inputs(name)
    c = d["cfg"]
    z = np.load(os.path.join(HERE, f"full_attn_{name}.npz"))
    H, D = c["heads"], c["dim_head"]
    attn = make_module(d["params"], H, D, c["gated"], dev)
    if fused:
        assert tm.fuse_qkv_weights(attn)
    bf = lambda a: torch.from_numpy(a).to(dev, torch.bfloat16)
    x = bf(d["x"])[None]
    grid = torch.tensor([list(c["grid"])])
    cos, sin = tm.causal_precompute_freqs_cis(
        grid, H * D, start_frame=c["start"], device=dev, dtype=torch.bfloat16,
        num_attention_heads=H, is_audio=c["audio"],
        max_pos=[20] if len(c["grid"]) == 1 else None)
    ck, cv = bf(d["cached_k"])[None], bf(d["cached_v"])[None]
    if c.get("cache_blocks"):
        ck, cv = arena_cache(ck, cv, c["cache_blocks"], dev)
    with torch.no_grad():
        out, nk, nv = tm.attention_with_cache(attn, x, None, (cos, sin), None, ck, cv,
                                              new_kv_real_len=c["real_len"])
    torch.cuda.synchronize(dev)
    assert tuple(out.shape) == (1, c["lq"], c["hidden"])
    return {"out": _figures(z, "out", out, z["rows_out"]),
            "new_k": _figures(z, "new_k", nk, z["rows_kv"]),
            "new_v": _figures(z, "new_v", nv, z["rows_kv"])}


def run_pair_case(name: str, dev) -> Dict[str, Dict[str, float]]:
    """The paired A2V / V2A attention at a full-size case."""
    import taomate_b200 as tm
    from taomate_b200.kv_cache import LayerKVCache
    d = inputs.pair_case_inputs(name)
    c = d["cfg"]
    z = np.load(os.path.join(HERE, f"full_pair_{name}.npz"))
    H, D = c["heads"], c["dim_head"]
    a2v = make_module(d["a2v"], H, D, c["gated"][0], dev)
    v2a = make_module(d["v2a"], H, D, c["gated"][1], dev)
    bf = lambda a: torch.from_numpy(a).to(dev, torch.bfloat16)
    cache = LayerKVCache()
    for nm in ("a2v", "v2a"):
        kv = d["caches"][nm]
        if kv is not None:
            setattr(cache, nm + "_k", bf(kv[0])[None])
            setattr(cache, nm + "_v", bf(kv[1])[None])
    inner = H * D
    vpe = tm.causal_precompute_freqs_cis(
        torch.tensor([[c["v_frames"]]]), inner, max_pos=[20], start_frame=c["v_start"],
        device=dev, dtype=torch.bfloat16, num_attention_heads=H,
        repeat_per_frame=c["frame_seqlen"])
    ape = tm.causal_precompute_freqs_cis(
        torch.tensor([[c["la"]]]), inner, max_pos=[20], start_frame=c["a_start"], device=dev,
        dtype=torch.bfloat16, is_audio=True, num_attention_heads=H)
    x = {k: bf(v)[None] for k, v in d["x"].items()}
    with torch.no_grad():
        outs = tm.cross_modal_pair_attention_with_cache(
            a2v, v2a, x["vx_a2v"], x["ax_a2v"], x["ax_v2a"], x["vx_v2a"], vpe, ape, cache,
            video_real_len=c["video_real_len"], audio_real_len=c["audio_real_len"], layer_idx=0)
    torch.cuda.synchronize(dev)
    keys = ("a2v_out", "a2v_k", "a2v_v", "v2a_out", "v2a_k", "v2a_v")
    return {k: _figures(z, k, o, z[f"rows_{k}"]) for k, o in zip(keys, outs)}


def format_figures(case: str, figs: Dict[str, Dict[str, float]]) -> str:
    parts = [f"{k} {v['ours']:.2e} (ref bf16 {v['ref']:.2e}, vs ref {v['cross']:.2e})"
             for k, v in figs.items()]
    return f"{case}: rel_l2 vs exact: " + "; ".join(parts)
