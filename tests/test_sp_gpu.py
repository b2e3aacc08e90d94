"""Ulysses sequence parallelism on 2, 4 and 8 GPUs (each skipped with fewer).

Each rank holds its shard of the chunk's tokens and a head shard of the KV
cache over the whole sequence, as the reference lays them out
(ltx_causal/transformer/kv_cache.py:331-339, 1432-1462, 1535-1538).
``attention_with_cache`` with the packed seq->head exchange and the head->seq
exchange must reproduce the single-GPU call on the same inputs: the output rows
of the rank's token shard and the new K/V of the rank's heads.  The only
difference allowed is the projection GEMMs' bf16 rounding on a different
number of rows.
"""

import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, outdir):
    sys.path.insert(0, os.path.dirname(HERE))
    import ctypes

    import taomate_b200 as tm
    from taomate_b200 import _lib, parallel as P
    from taomate_b200.attention import AttentionWeights

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        heads, dim_head, frames, fh, fw = 8, 128, 2, 8, 12
        hidden, lq, lc = heads * dim_head, frames * fh * fw, 320
        torch.manual_seed(0)  # identical weights on both ranks
        attn = AttentionWeights(hidden, heads, dim_head, gated=True, device=dev)
        g = torch.Generator(device=dev).manual_seed(1)
        x = torch.randn(1, lq, hidden, device=dev, generator=g).to(torch.bfloat16)
        ck = torch.randn(1, lc, heads, dim_head, device=dev, generator=g).to(torch.bfloat16)
        cv = torch.randn(1, lc, heads, dim_head, device=dev, generator=g).to(torch.bfloat16)
        cos, sin = tm.causal_precompute_freqs_cis(torch.tensor([[frames, fh, fw]]), hidden,
                                                  start_frame=3, device=dev,
                                                  dtype=torch.bfloat16,
                                                  num_attention_heads=heads)
        with torch.no_grad():
            ref_out, ref_k, ref_v = tm.attention_with_cache(attn, x, None, (cos, sin), None,
                                                            ck, cv)
        P.init_sp_mesh(world, world)
        sl, hl = lq // world, heads // world
        ts = slice(rank * sl, (rank + 1) * sl)
        hs = slice(rank * hl, (rank + 1) * hl)
        with torch.no_grad():
            out, nk, nv = tm.attention_with_cache(
                attn, x[:, ts].contiguous(), None, (cos[:, :, ts], sin[:, :, ts]), None,
                ck[:, :, hs].contiguous(), cv[:, :, hs].contiguous())
        # the same calls with the exchanges fused into the kernels' NVLink stores,
        # twice in a row (the second on other inputs: buffers and flag epochs reused)
        from taomate_b200.block import v2a_gather_bytes
        P.init_peer_exchange(1, sl, heads, dim_head,
                             gather_bytes=v2a_gather_bytes(16, 4, 64, world))
        x2 = torch.randn(1, lq, hidden, device=dev, generator=g).to(torch.bfloat16)
        with torch.no_grad():
            out_p, nk_p, nv_p = tm.attention_with_cache(
                attn, x[:, ts].contiguous(), None, (cos[:, :, ts], sin[:, :, ts]), None,
                ck[:, :, hs].contiguous(), cv[:, :, hs].contiguous())
            out_p = out_p.clone()
            out_p2, _, _ = tm.attention_with_cache(
                attn, x2[:, ts].contiguous(), None, (cos[:, :, ts], sin[:, :, ts]), None,
                ck[:, :, hs].contiguous(), cv[:, :, hs].contiguous())
            out_p2 = out_p2.clone()
            # one fused QKV GEMM: the kernel reads q/k/v as column slices
            assert tm.fuse_qkv_weights(attn)
            out_f, nk_f, nv_f = tm.attention_with_cache(
                attn, x[:, ts].contiguous(), None, (cos[:, :, ts], sin[:, :, ts]), None,
                ck[:, :, hs].contiguous(), cv[:, :, hs].contiguous())
        # the whole block (small shapes): video split by tokens, audio replicated,
        # text cross-attention over all heads locally, V2A over each rank's own
        # video keys with the ranks' partial results merged
        from taomate_b200.block import BlockWeights
        from taomate_b200.kv_cache import LayerKVCache
        from taomate_b200.model import StreamConfig, rope_tables, synthetic_conditioning
        cfg = StreamConfig(layers=1, video_dim=hidden, video_heads=heads, video_dim_head=dim_head,
                           audio_dim=256, audio_heads=4, audio_dim_head=64, frame_h=fh,
                           frame_w=fw, text_tokens=24)
        torch.manual_seed(4)
        blk = BlockWeights(hidden, heads, dim_head, 256, 4, 64, device=dev, std=0.05)
        cond = synthetic_conditioning(cfg, frames, 16, dev, g)
        vx = torch.randn(1, lq, hidden, device=dev, generator=g).to(torch.bfloat16)
        ax = torch.randn(1, 16, 256, device=dev, generator=g).to(torch.bfloat16)
        rnd = lambda *s_: torch.randn(*s_, device=dev, generator=g).to(torch.bfloat16)
        caches = {"video_self": (rnd(1, lc, heads, dim_head), rnd(1, lc, heads, dim_head)),
                  "audio_self": (rnd(1, 32, 4, 64), rnd(1, 32, 4, 64)),
                  "a2v": (rnd(1, 32, 4, 64), rnd(1, 32, 4, 64)),
                  "v2a": (rnd(1, lc, 4, 64), rnd(1, lc, 4, 64))}

        def lcache(shard):
            kw = {}
            for nm, (k_, v_) in caches.items():
                if shard and nm == "video_self":
                    k_, v_ = k_[:, :, hs].contiguous(), v_[:, :, hs].contiguous()
                if shard and nm == "v2a":  # this rank's share of the cached video tokens
                    cs = slice(rank * (lc // world), (rank + 1) * (lc // world))
                    k_, v_ = k_[:, cs].contiguous(), v_[:, cs].contiguous()
                kw[nm + "_k"], kw[nm + "_v"] = k_, v_
            return LayerKVCache(**kw)

        def bargs(pe, off, rep, shard):
            return dict(video_timestep_6d=cond.video_ts, audio_timestep_6d=cond.audio_ts,
                        video_pe=pe[0], audio_pe=pe[1], video_cross_pe=pe[2],
                        audio_cross_pe=pe[3], video_ctx=cond.video_ctx, audio_ctx=cond.audio_ctx,
                        video_context_mask=None, audio_context_mask=None,
                        video_cross_ss=cond.video_cross_ss,
                        video_cross_gate=cond.video_cross_gate,
                        audio_cross_ss=cond.audio_cross_ss,
                        audio_cross_gate=cond.audio_cross_gate, video_prompt_ts=None,
                        audio_prompt_ts=None, layer_cache=lcache(shard),
                        video_frame_seqlen=fh * fw, audio_frame_seqlen=1,
                        video_token_offset=off, audio_replicated=rep)

        with torch.no_grad():
            with P.sp_local():
                rv, ra, rc = tm.block_forward_with_cache(
                    blk, vx, ax, **bargs(rope_tables(cfg, frames, 16, 3, 26, dev), 0, False,
                                         False))
            bv, ba, bc = tm.block_forward_with_cache(
                blk, vx[:, ts].contiguous(), ax,
                **bargs(rope_tables(cfg, frames, 16, 3, 26, dev, ts), rank * sl, True, True))
            # V2A parts gathered over NVLink above; the same block with every
            # exchange through NCCL
            P.close_peer_exchange()
            nv_, na_, _ = tm.block_forward_with_cache(
                blk, vx[:, ts].contiguous(), ax,
                **bargs(rope_tables(cfg, frames, 16, 3, 26, dev, ts), rank * sl, True, True))
        torch.cuda.synchronize()
        code = ctypes.c_int(0)
        assert _lib.load().tm_device_error(ctypes.byref(code)) == 0 and code.value == 0
        f = lambda t: t.float().cpu().numpy()
        np.savez(os.path.join(outdir, f"b{rank}.npz"), vx=f(bv), ref_vx=f(rv[:, ts]), ax=f(ba),
                 ref_ax=f(ra), vs_k=f(bc.video_self_k[:, lc:]), ref_vs_k=f(rc.video_self_k[:, lc:, hs]),
                 v2a_k=f(bc.v2a_k[:, lc // world:]), ref_v2a_k=f(rc.v2a_k[:, lc:][:, ts]),
                 a2v_k=f(bc.a2v_k[:, 32:]), ref_a2v_k=f(rc.a2v_k[:, 32:]),
                 vx_nccl=f(nv_), ax_nccl=f(na_))
        f = lambda t: t.float().cpu().numpy()
        np.savez(os.path.join(outdir, f"r{rank}.npz"), out=f(out), ref_out=f(ref_out[:, ts]),
                 k=f(nk), ref_k=f(ref_k[:, :, hs]), v=f(nv), ref_v=f(ref_v[:, :, hs]),
                 out_p=f(out_p), k_p=f(nk_p), v_p=f(nv_p), out_p2=f(out_p2), out_f=f(out_f),
                 k_f=f(nk_f), v_f=f(nv_f))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _rel_l2(a, b):
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_ulysses_sp_matches_single_gpu(tmp_path, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        z = np.load(tmp_path / f"r{r}.npz")
        assert z["out"].shape == z["ref_out"].shape
        assert z["k"].shape == z["ref_k"].shape
        # bf16 rounding of the projections on half the rows; everything after
        # them (norm, RoPE, exchange, attention) is the same arithmetic
        assert _rel_l2(z["k"], z["ref_k"]) < 5e-3
        assert _rel_l2(z["v"], z["ref_v"]) < 5e-3
        assert _rel_l2(z["out"], z["ref_out"]) < 1e-2
        # fused NVLink exchanges: the same kernels and data as the NCCL path
        assert _rel_l2(z["out_p"], z["out"]) < 1e-3
        assert _rel_l2(z["k_p"], z["k"]) < 1e-3 and _rel_l2(z["v_p"], z["v"]) < 1e-3
        assert _rel_l2(z["out_p2"], z["out_p"]) > 1e-1  # the second call saw new inputs
        # fused QKV projection: another GEMM kernel, the same arithmetic after it
        assert _rel_l2(z["out_f"], z["out_p"]) < 1e-2
        assert _rel_l2(z["k_f"], z["k_p"]) < 5e-3 and _rel_l2(z["v_f"], z["v_p"]) < 5e-3
        # the block: same bar as the attention call (projection rounding on 1/G of the rows)
        b = np.load(tmp_path / f"b{r}.npz")
        assert b["vx"].shape == b["ref_vx"].shape and b["ax"].shape == b["ref_ax"].shape
        assert _rel_l2(b["vx"], b["ref_vx"]) < 1e-2
        assert _rel_l2(b["ax"], b["ref_ax"]) < 1e-2  # replicated audio: every rank's full output
        assert _rel_l2(b["vs_k"], b["ref_vs_k"]) < 5e-3
        # V2A cache: this rank's video tokens, all heads
        assert _rel_l2(b["v2a_k"], b["ref_v2a_k"]) < 5e-3
        assert _rel_l2(b["a2v_k"], b["ref_a2v_k"]) < 5e-3
        # NVLink exchanges and gathers against NCCL: the same arithmetic
        assert _rel_l2(b["vx"], b["vx_nccl"]) < 1e-3 and _rel_l2(b["ax"], b["ax_nccl"]) < 1e-3
