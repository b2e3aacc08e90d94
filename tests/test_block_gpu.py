"""The whole transformer block (block_forward_with_cache, kv_cache.py:2145-2654)
on the GPU against a real reference block run on CPU.

The golden case loads the same seeded weights into the reference's
``CausalAVTransformerBlock`` by state-dict name and runs its
``block_forward_with_cache`` in fp32 and bf16 on bf16-rounded inputs (video 4
heads x 128, audio 4 heads x 64, filled caches, a padded text context).

Bars:
* video / audio outputs and every new K/V row: relative L2 to the reference's
  fp32 result at most 1.01x the reference's own bf16 run's (outputs that are
  one rounding of a projection tie with it at the bf16 rounding floor);
* AdaLN rows given per frame (the kernel maps tokens to frames) and given per
  token (as the reference passes them) give identical bits;
* cache views in the slot arena give identical bits to plain cache tensors.
"""

import os

import numpy as np
import pytest
import torch

import inputs
import full_size as FS

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0") if torch.cuda.is_available() else None
NEW = (("video_self_k", "video_self_v"), ("audio_self_k", "audio_self_v"), ("a2v_k", "a2v_v"),
       ("v2a_k", "v2a_v"))


@pytest.fixture(scope="module", autouse=True)
def _device():
    if DEV is None:
        pytest.skip("no CUDA device")
    torch.cuda.set_device(DEV)
    yield
    from taomate_b200 import _lib
    assert _lib.device_error() == 0, "a kernel set the device error flag"


def _setup(d, arena=False, fused=False):
    import taomate_b200 as tm
    from taomate_b200.block import BlockWeights, fuse_block_weights
    from taomate_b200.kv_cache import LayerKVCache
    c = d["cfg"]
    blk = BlockWeights(c["video_dim"], c["video_heads"], c["video_dim_head"], c["audio_dim"],
                       c["audio_heads"], c["audio_dim_head"], device=DEV, std=None)
    blk.load_state_dict({k: torch.from_numpy(v) for k, v in d["params"].items()}, strict=True)
    if fused:
        # QKV of the two self-attentions, K/V of A2V and V2A
        assert tm.block.fuse_block_weights(blk) == 4
    bf = lambda a: torch.from_numpy(a).to(DEV, torch.bfloat16)[None]
    x = {k: bf(v) for k, v in d["x"].items()}
    Hv, dv, Ha, da = c["video_heads"], c["video_dim_head"], c["audio_heads"], c["audio_dim_head"]
    F, fs, La = c["v_frames"], d["frame_seqlen"], c["la"]
    kw = dict(device=DEV, dtype=torch.bfloat16)
    vpe = tm.causal_precompute_freqs_cis(torch.tensor([[F, c["fh"], c["fw"]]]), Hv * dv,
                                         start_frame=c["v_start"], num_attention_heads=Hv, **kw)
    ape = tm.causal_precompute_freqs_cis(torch.tensor([[La]]), Ha * da, max_pos=[20],
                                         start_frame=c["a_start"], is_audio=True,
                                         num_attention_heads=Ha, **kw)
    vcpe = tm.causal_precompute_freqs_cis(torch.tensor([[F]]), Ha * da, max_pos=[20],
                                          start_frame=c["v_start"], num_attention_heads=Ha,
                                          repeat_per_frame=fs, **kw)
    m = torch.from_numpy(d["mask"]).to(DEV)
    mask = ((m - 1).to(torch.bfloat16) * torch.finfo(torch.bfloat16).max).view(1, 1, 1, -1)
    lc = LayerKVCache()
    for nm, (k, v) in d["caches"].items():
        kt, vt = bf(k), bf(v)
        if arena:
            kt, vt = FS.arena_cache(kt, vt, (int(kt.shape[1]),), DEV)
        setattr(lc, nm + "_k", kt)
        setattr(lc, nm + "_v", vt)
    return blk, x, (vpe, ape, vcpe, ape), mask, lc


def _run(blk, x, pes, mask, lc, fs, per_token=False):
    from taomate_b200.block import block_forward_with_cache
    tok = (lambda t: t.repeat_interleave(fs, dim=1)) if per_token else (lambda t: t)
    vpe, ape, vcpe, acpe = pes
    with torch.no_grad():
        vx, ax, new = block_forward_with_cache(
            blk, x["video_x"], x["audio_x"], tok(x["video_ts"]), x["audio_ts"], vpe, ape, vcpe,
            acpe, x["video_ctx"], x["audio_ctx"], mask, mask, tok(x["video_cross_ss"]),
            tok(x["video_cross_gate"]), x["audio_cross_ss"], x["audio_cross_gate"], None, None,
            None, None, lc, layer_idx=0, video_frame_seqlen=fs, audio_frame_seqlen=1)
    torch.cuda.synchronize()
    return vx, ax, new


def _new_rows(new, d):
    c = d["cfg"]
    n = {"video_self": d["Lv"], "audio_self": c["la"], "a2v": c["la"], "v2a": d["Lv"]}
    out = {}
    for kk, vk in NEW:
        nm = kk[:-2]
        for key in (kk, vk):
            t = getattr(new, key)
            t = t.materialize() if hasattr(t, "materialize") else t
            out[key] = t[0, -n[nm]:]
    return out


@pytest.mark.parametrize("fused", [False, True], ids=["qkv3", "qkv_fused"])
def test_block_forward_vs_reference(golden_dir, parity_report, fused):
    z = np.load(os.path.join(golden_dir, "block_small.npz"))
    d = inputs.block_case_inputs("small")
    blk, x, pes, mask, lc = _setup(d, fused=fused)
    vx, ax, new = _run(blk, x, pes, mask, lc, d["frame_seqlen"])
    got = {"video_x": vx[0], "audio_x": ax[0], **_new_rows(new, d)}
    figs = {}
    for key, t in got.items():
        a = t.float().cpu().numpy()
        ours, ref = FS.rel_l2(a, z[f"{key}_f32"]), FS.rel_l2(z[f"{key}_bf16"], z[f"{key}_f32"])
        figs[key] = {"ours": ours, "ref": ref, "cross": FS.rel_l2(a, z[f"{key}_bf16"])}
    parity_report.append(FS.format_figures(f"block small ({'fused' if fused else 'qkv3'})",
                                           {k: figs[k] for k in ("video_x", "audio_x",
                                                                 "video_self_k", "v2a_v")}))
    for key, f in figs.items():
        assert f["ours"] <= 1.01 * f["ref"], (key, f)
    # inputs untouched (the reference returns new tensors)
    assert torch.equal(x["video_x"], torch.from_numpy(d["x"]["video_x"]).to(DEV, torch.bfloat16)[None])


def test_block_adaln_rows_per_frame_equal_per_token():
    d = inputs.block_case_inputs("small")
    blk, x, pes, mask, lc = _setup(d)
    a = _run(blk, x, pes, mask, lc, d["frame_seqlen"], per_token=False)
    b = _run(blk, x, pes, mask, lc, d["frame_seqlen"], per_token=True)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_block_audio_stream_overlap_same_bits():
    """The audio chain on its own stream (the default) gives the bits of the
    one-stream schedule."""
    from taomate_b200.block import block_forward_with_cache
    d = inputs.block_case_inputs("small")
    blk, x, pes, mask, lc = _setup(d)
    a = _run(blk, x, pes, mask, lc, d["frame_seqlen"])
    fs = d["frame_seqlen"]
    vpe, ape, vcpe, acpe = pes
    with torch.no_grad():
        b = block_forward_with_cache(
            blk, x["video_x"], x["audio_x"], x["video_ts"], x["audio_ts"], vpe, ape, vcpe, acpe,
            x["video_ctx"], x["audio_ctx"], mask, mask, x["video_cross_ss"],
            x["video_cross_gate"], x["audio_cross_ss"], x["audio_cross_gate"], None, None, None,
            None, lc, layer_idx=0, video_frame_seqlen=fs, audio_frame_seqlen=1,
            overlap_audio=False)
    torch.cuda.synchronize()
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_block_arena_caches_equal_plain_caches():
    d = inputs.block_case_inputs("small")
    blk, x, pes, mask, lc = _setup(d)
    a = _run(blk, x, pes, mask, lc, d["frame_seqlen"])
    blk2, x2, pes2, mask2, lc2 = _setup(d, arena=True)
    b = _run(blk2, x2, pes2, mask2, lc2, d["frame_seqlen"])
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    ra, rb = _new_rows(a[2], d), _new_rows(b[2], d)
    for key in ra:
        assert torch.equal(ra[key], rb[key]), key
