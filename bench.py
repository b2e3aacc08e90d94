#!/usr/bin/env python
"""Benchmark of the causal-LTX streaming step on B200.

Headline: one streaming block of the 48-block joint
audio-video model, as the pipeline runs it (taomate/inference/model.py:
166-248): the text K/V projection of every layer, 3 denoising forwards and
the sigma = 0 commit forward over a 3-latent-frame chunk (512x768 -> 16 x 24 =
384 tokens per frame, 1152 video tokens; 25 audio tokens), then the commit
append and the eviction, at the cache's steady state (sink block of 4 frames
+ the 2 newest blocks: 3840 video / 76 audio cached tokens).  Each forward:
patchify, 48 x block_forward_with_cache (video self-attention, video text
cross-attention, audio self-attention, audio text cross-attention, A2V, V2A,
video and audio FFN, all behind AdaLN), output projection.  Hidden 4096 =
32 x 128 (video), 2048 = 32 x 64 (audio); weights random N(0, 0.02) (about
38 GB in bf16), latents and text N(0, 1), AdaLN rows N(0, 0.1).

  value  latent frames/s (3 per block) with all inputs resident in HBM
         (device time, CUDA events, max over ranks);
  e2e    the same with each block's latents and conditioning rows copied from
         pinned host memory and the denoised latents read back, inside the
         timed region.

With --gpus N: Ulysses sequence parallelism, one process per GPU; video tokens
split over the ranks (1152 / N each, 32 / N heads of the video self-attention
cache), audio replicated; total work per block fixed, so scaling is "strong".
The line also carries ``attention_step`` (the video self-attention step alone,
BASELINE config 2 shapes) and, at N > 1, ``parity_rel_l2`` (the sequence
parallel calls against the same calls on one GPU, on the same box).

``--impl reference`` times the reference algorithm's CPU restatement
(oracle/ltx_oracle.py, numpy fp32, all host threads) on one layer-forward per
step and reports the same metric.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

FRAME_TOKENS = 16 * 24
Q_FRAMES = 3
ANCHOR_FRAMES = 1
WINDOW_FRAMES = 8
HIDDEN, HEADS, DIM_HEAD = 4096, 32, 128
FORWARDS_PER_STEP = 4  # 3 denoising + 1 commit


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--nccl-exchange", action="store_true",
                    help="N>1: the Ulysses exchanges through NCCL all_to_all_single instead of "
                         "the kernels' NVLink peer stores")
    ap.add_argument("--eager", action="store_true",
                    help="issue every forward from Python instead of replaying a CUDA graph")
    ap.add_argument("--serial-audio", action="store_true",
                    help="run each block's audio chain on the main stream (no second stream)")
    ap.add_argument("--qkv3", action="store_true",
                    help="three projection GEMMs per call instead of one over the fused weights")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--segments", type=int, default=12, help="--workload c5: 5-block segments")
    ap.add_argument("--workload", choices=["c4", "attention", "both", "c5"], default="both",
                    help="c4: the 48-block audio-video step (headline); attention: the video "
                         "self-attention step alone; both: c4 headline + attention as an extra key")
    ap.add_argument("--kernel-case", choices=["attention", "norm_rope", "kv_append",
                                              "residual_norm", "linear"], default=None,
                    help="time one kernel in isolation at C2 shapes (profiling target)")
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--rows", type=int, default=144,
                    help="--kernel-case linear: token rows (1152 / G video, 25 audio)")
    ap.add_argument("--heads", type=int, default=None,
                    help="--kernel-case attention: heads per GPU (32 / sequence-parallel ranks)")
    ap.add_argument("--cached", type=int, default=None,
                    help="--kernel-case attention: cached keys (3456: config 2; 3840: the "
                         "production layout of the C4 step)")
    return ap.parse_args()


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.path = tempfile.mktemp(suffix=".csv")
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.fh,
                stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        sm, smax, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as fh:
            for line in fh:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax = float(parts[2])
                    power.append(float(parts[3]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "power_w_max": max(power) if power else None, "samples": len(sm),
                "reasons": sorted(reasons)}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as fh:
            d = json.load(fh)
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def profiled_traffic(kernel: str, heads: int, keys: int = 4608):
    """DRAM bytes per launch of ``kernel`` at ``heads`` heads per GPU and
    ``keys`` keys per query from the committed ncu capture table
    (profiles/traffic.json), or None when that launch shape was not captured."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as fh:
        table = json.load(fh).get(kernel, {})
    for ent in table.values():
        if int(ent.get("heads", -1)) == heads and int(ent.get("keys", -1)) == keys:
            return float(ent["dram_bytes_per_launch"])
    return None


# --------------------------------------------------------------------------- CPU
def cpu_sample_time(reps: int, warm: int):
    """Seconds per video self-attention layer-forward (C2 shapes) of the numpy
    fp32 restatement, min over ``reps`` after ``warm`` untimed runs."""
    import numpy as np
    from oracle import ltx_oracle as O
    rng = np.random.default_rng(0)
    f32 = np.float32
    prm = {n: (rng.standard_normal((HIDDEN, HIDDEN)) * 0.02).astype(f32)
           for n in ("to_q_w", "to_k_w", "to_v_w", "to_out_w")}
    for n in ("to_q_b", "to_k_b", "to_v_b", "to_out_b"):
        prm[n] = (rng.standard_normal(HIDDEN) * 0.02).astype(f32)
    prm["q_norm_w"] = np.ones(HIDDEN, f32)
    prm["k_norm_w"] = np.ones(HIDDEN, f32)
    Lq = Q_FRAMES * FRAME_TOKENS
    Lc = (ANCHOR_FRAMES + WINDOW_FRAMES) * FRAME_TOKENS
    x = rng.standard_normal((Lq, HIDDEN)).astype(f32)
    ck = rng.standard_normal((Lc, HEADS, DIM_HEAD)).astype(f32)
    cv = rng.standard_normal((Lc, HEADS, DIM_HEAD)).astype(f32)
    cos, sin = O.precompute_freqs_cis_split((Q_FRAMES, 16, 24), HIDDEN, start_frame=9,
                                            num_heads=HEADS, precision="f32")
    cos, sin = cos.astype(f32), sin.astype(f32)
    times = []
    for i in range(warm + reps):
        t0 = time.perf_counter()
        O.attention_with_cache(x, prm, HEADS, DIM_HEAD, (cos, sin), ck, cv, dtype=f32)
        dt = time.perf_counter() - t0
        if i >= warm:
            times.append(dt)
    return times


def cpu_c4_layer_times(reps: int, warm: int):
    """Seconds per layer-forward of the whole block at C4 shapes (numpy fp32
    restatement of block_forward_with_cache: video 1152 tokens over 3840
    cached, audio 25 over 76, text 256, all host BLAS threads), min/mean over
    ``reps`` after ``warm`` untimed runs; plus the per-block text K/V
    projection of one layer."""
    import numpy as np
    from oracle import ltx_oracle as O
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import inputs
    rng = np.random.default_rng(0)
    f32 = np.float32
    Dv, Da, Hv, dv, Ha, da = 4096, 2048, 32, 128, 32, 64
    c = dict(video_dim=Dv, video_heads=Hv, video_dim_head=dv, audio_dim=Da, audio_heads=Ha,
             audio_dim_head=da)
    sd = {}
    for nm, shp in inputs.block_param_shapes(c).items():
        if nm.endswith("norm.weight"):
            sd[nm] = np.ones(shp, f32)
        else:
            sd[nm] = rng.standard_normal(shp, dtype=f32) * f32(0.02)
    cfg = {"video_heads": Hv, "video_dim_head": dv, "audio_heads": Ha, "audio_dim_head": da}
    Lv, La, T, fs = 1152, 25, 256, 384
    g = lambda *sh, sc=1.0: rng.standard_normal(sh, dtype=f32) * f32(sc)
    vpe = O.precompute_freqs_cis_split((3, 16, 24), Dv, start_frame=10, num_heads=Hv,
                                       precision="f32")
    ape = O.precompute_freqs_cis_split((La,), Ha * da, start_frame=76, is_audio=True,
                                       num_heads=Ha, precision="f32", max_pos=[20])
    vc, vs = O.precompute_freqs_cis_split((3,), Ha * da, start_frame=10, num_heads=Ha,
                                          precision="f32", max_pos=[20])
    tabs = [tuple(t.astype(f32) for t in p) for p in
            (vpe, ape, (np.repeat(vc, fs, 1), np.repeat(vs, fs, 1)), ape)]
    caches = {"video_self": (g(3840, Hv, dv), g(3840, Hv, dv)),
              "audio_self": (g(76, Ha, da), g(76, Ha, da)), "a2v": (g(76, Ha, da), g(76, Ha, da)),
              "v2a": (g(3840, Ha, da), g(3840, Ha, da))}
    tok = lambda a: np.repeat(a, fs, axis=0)
    argv = (g(Lv, Dv), g(La, Da), tok(g(3, 6 * Dv, sc=0.1)), g(La, 6 * Da, sc=0.1), *tabs,
            g(T, Dv), g(T, Da), None, None, tok(g(3, 4 * Dv, sc=0.1)), tok(g(3, Dv, sc=0.1)),
            g(La, 4 * Da, sc=0.1), g(La, Da, sc=0.1))
    times = []
    for i in range(warm + reps):
        t0 = time.perf_counter()
        O.block_forward_with_cache(sd, cfg, *argv, caches=caches, dtype=f32)
        dt = time.perf_counter() - t0
        if i >= warm:
            times.append(dt)
    return times


def cpu_c4_sample(layers: int, reps: int = 2, warm: int = 0):
    times = cpu_c4_layer_times(reps, warm)
    t = min(times)
    return {"value": 3.0 / (t * layers * FORWARDS_PER_STEP), "unit": "latent frames/s",
            "cores": cpu_threads(), "kind": "port",
            "sample": f"{len(times)} C4 layer-forwards of the numpy fp32 restatement of "
                      f"block_forward_with_cache (min {t:.3f} s), x{layers * FORWARDS_PER_STEP} "
                      f"per block; text K/V projection not counted"}


def cpu_threads():
    try:
        from threadpoolctl import threadpool_info
        n = max((int(i.get("num_threads", 1)) for i in threadpool_info()), default=1)
        return n
    except Exception:
        return os.cpu_count() or 1


def cpu_breakdown():
    """The CPU timings BASELINE lists beside the step, on the oracle port
    (numpy fp32, all host BLAS threads), one warm-up then the minimum of 3:
    attention_with_cache at C1 and C2 (projections included), the C2 RoPE
    tables + split rotation of q and k, and one retain_streaming_context of a
    48-layer cache at the production layout (every video and audio field)."""
    import numpy as np
    from oracle import ltx_oracle as O
    f32 = np.float32
    rng = np.random.default_rng(3)
    out = {}

    def best(fn):
        fn()
        ts = []
        for _ in range(3):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return min(ts) * 1e3

    def attn_case(hid, H, D, lq, lc, grid, start):
        prm = {n: rng.standard_normal((hid, hid), dtype=f32) * f32(0.02)
               for n in ("to_q_w", "to_k_w", "to_v_w", "to_out_w")}
        for n in ("to_q_b", "to_k_b", "to_v_b", "to_out_b"):
            prm[n] = rng.standard_normal(hid, dtype=f32) * f32(0.02)
        prm["q_norm_w"] = prm["k_norm_w"] = np.ones(hid, f32)
        x = rng.standard_normal((lq, hid), dtype=f32)
        ck = rng.standard_normal((lc, H, D), dtype=f32)
        cv = rng.standard_normal((lc, H, D), dtype=f32)
        cos, sin = O.precompute_freqs_cis_split(grid, hid, start_frame=start, num_heads=H,
                                                precision="f32")
        pe = (cos.astype(f32), sin.astype(f32))
        return lambda: O.attention_with_cache(x, prm, H, D, pe, ck, cv, dtype=f32)

    out["attention_with_cache_c1_f32_ms"] = best(attn_case(256, 4, 64, 96, 576, (1, 8, 12), 6))
    out["attention_with_cache_c2_f32_ms"] = best(
        attn_case(HIDDEN, HEADS, DIM_HEAD, 1152, 3456, (3, 16, 24), 9))
    xq = rng.standard_normal((1152, HIDDEN), dtype=f32)

    def rope():
        c, s_ = O.precompute_freqs_cis_split((3, 16, 24), HIDDEN, start_frame=9, num_heads=HEADS,
                                             precision="f32")
        c, s_ = c.astype(f32), s_.astype(f32)
        O.apply_split_rotary_emb(xq, c, s_)
        O.apply_split_rotary_emb(xq, c, s_)
    out["rope_tables_and_rotate_qk_c2_ms"] = best(rope)
    segs = [{"block_idx": 0, "video_tokens": 1536, "audio_tokens": 26}] + \
        [{"block_idx": i, "video_tokens": 1152, "audio_tokens": 25} for i in (1, 2, 3)]
    layer = {"video": rng.standard_normal((4992, 32, 128), dtype=f32).astype(np.float16),
             "v2a": rng.standard_normal((4992, 32, 64), dtype=f32).astype(np.float16),
             "audio": rng.standard_normal((101, 32, 64), dtype=f32).astype(np.float16)}

    def retain():
        keep = O.retain_indices(segs)
        vs, as_ = O.slice_spans(segs, keep)
        for _ in range(48):
            for _kv in range(2):  # K and V of each pair
                O.slice_tensor(layer["video"], vs, axis=0)
                O.slice_tensor(layer["v2a"], vs, axis=0)
                O.slice_tensor(layer["audio"], as_, axis=0)
                O.slice_tensor(layer["audio"], as_, axis=0)
    out["retain_streaming_context_48_layers_ms"] = best(retain)
    out["note"] = ("numpy restatement; the reference's own bf16 CPU path is not timed (numpy has "
                   "no bf16; 16-bit storage is used for the retained cache rows)")
    return out


def run_reference(args):
    """The reference's CPU arm: the numpy restatement of the reference block
    (the reference itself is pure PyTorch and its source tree does not travel
    to the GPU box), one C4 layer-forward per timed step, all host threads,
    rank 0 only.  ``value`` extrapolates to the 48-layer x 4-forward block;
    ``ms_per_step`` is the time of what each timed step ran."""
    rank, world, _ = env_rank()
    if rank != 0:
        return
    times = cpu_c4_layer_times(max(1, args.steps), max(0, args.warmup))
    t = statistics.mean(times)
    per_block = t * args.layers * FORWARDS_PER_STEP
    value = 3.0 / per_block
    line = {
        "metric": METRIC_C4, "value": value, "unit": "latent frames/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "impl": "reference",
        "config": C4_CONFIG | {"sample": "one C4 layer-forward per timed step; value = 3 latent "
                                         f"frames / ({args.layers} x 4 layer-forwards)",
                               "extrapolated_ms_per_block": per_block * 1e3},
        "cpu_baseline": {"value": value, "unit": "latent frames/s", "cores": cpu_threads(),
                         "kind": "port",
                         "sample": f"{len(times)} C4 layer-forwards of the numpy fp32 "
                                   f"restatement of block_forward_with_cache, mean {t:.3f} s"},
        "e2e": {"value": value, "unit": "latent frames/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "cpu_breakdown": cpu_breakdown(),
        # what this box holds of the reference itself: an offline install of its
        # tree into baseline/_ref is refused (no setup.py / pyproject.toml)
        "reference_installed": os.path.isdir(os.path.join(ROOT, "baseline", "_ref")),
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- GPU
def attention_step(args, dev, rank, world, local):
    """The video self-attention step alone (BASELINE config 2 shapes): 48
    layers x 4 forwards of ``attention_with_cache`` per 3-frame block, cache 1
    anchor + 8 window frames.  Returns the measurements as a dict."""
    import torch
    import torch.distributed as dist
    import taomate_b200 as tm
    from taomate_b200 import _lib, parallel as P
    from taomate_b200.attention import AttentionWeights
    from taomate_b200.cache import retain_window
    from taomate_b200.graphs import AttentionGraph, attention_spans, copy_bytes, copy_into
    from taomate_b200.kv_cache import ArenaSpec, KVCache, LayerKVCache, init_arena_cache
    from taomate_b200.profiler import TIMER

    sp = world
    L = args.layers
    Lq = Q_FRAMES * FRAME_TOKENS
    if Lq % sp or HEADS % sp:
        raise SystemExit(f"{sp} ranks do not divide {Lq} tokens / {HEADS} heads")
    S_loc, H_loc = Lq // sp, HEADS // sp
    anchor, window = ANCHOR_FRAMES * FRAME_TOKENS, WINDOW_FRAMES * FRAME_TOKENS

    torch.manual_seed(0)  # identical weights on every rank
    attn = [AttentionWeights(HIDDEN, HEADS, DIM_HEAD, device=dev) for _ in range(L)]
    if not args.qkv3:
        for a in attn:  # one projection GEMM per call (weights laid out as one buffer)
            tm.fuse_qkv_weights(a)
    gen = torch.Generator(device=dev).manual_seed(1)
    xs = [torch.randn(1, Lq, HIDDEN, device=dev, generator=gen).to(torch.bfloat16)
          [:, rank * S_loc:(rank + 1) * S_loc].contiguous() for _ in range(L)]

    def fresh_cache():
        return init_arena_cache(L, {"video_self": ArenaSpec(6, Lq, H_loc, DIM_HEAD)}, device=dev)

    grid = torch.tensor([[Q_FRAMES, 16, 24]])

    def step(cache, block, x_in=None, outs=None):
        start = block * Q_FRAMES
        for fwd in range(FORWARDS_PER_STEP):
            cos, sin = tm.causal_precompute_freqs_cis(grid, HIDDEN, start_frame=start, device=dev,
                                                      dtype=torch.bfloat16,
                                                      num_attention_heads=HEADS)
            pe = (cos[:, :, rank * S_loc:(rank + 1) * S_loc],
                  sin[:, :, rank * S_loc:(rank + 1) * S_loc])
            commit = fwd == FORWARDS_PER_STEP - 1
            new_layers = []
            out = None
            for li in range(L):
                lay = cache.layers[li]
                x = xs[li] if x_in is None else x_in[li]
                out, nk, nv = tm.attention_with_cache(attn[li], x, None, pe, None,
                                                      lay.video_self_k, lay.video_self_v,
                                                      profile_name="video_self")
                if commit:
                    k2, v2 = tm.cat_cache_pair(lay.video_self_k, lay.video_self_v, nk, nv)
                    new_layers.append(LayerKVCache(video_self_k=k2, video_self_v=v2))
            if outs is not None:
                outs[fwd].copy_(out, non_blocking=True)
            if commit:
                cache = retain_window(KVCache(layers=new_layers), anchor, window)
        return cache

    def tables(block):
        cos, sin = tm.causal_precompute_freqs_cis(grid, HIDDEN, start_frame=block * Q_FRAMES,
                                                  device=dev, dtype=torch.bfloat16,
                                                  num_attention_heads=HEADS)
        return (cos[:, :, rank * S_loc:(rank + 1) * S_loc],
                sin[:, :, rank * S_loc:(rank + 1) * S_loc])

    read_stream = torch.cuda.Stream(dev)  # output read-back of the graph runners

    class GraphRunner:
        """One captured 48-layer forward (all four forwards of a block are the
        same computation over the same cache: the commit forward only keeps its
        new K/V).  Captured at the steady state, where every call sees the same
        number of key tiles; per block only the tile table, the RoPE tables and
        the inputs change."""

        def __init__(self, cache, block, inputs):
            self.inputs = inputs  # the per-layer inputs the captured forward reads
            c, s = tables(block)
            self.pe = (c.contiguous(), s.contiguous())
            for lay in cache.layers:  # pending chunks go to their slots before capture
                attention_spans(lay.video_self_k, lay.video_self_v, Lq)
            self.graph = AttentionGraph(dev, max_sites=L)

            def forward():
                kv, out = [], None
                for li in range(L):
                    lay = cache.layers[li]
                    out, nk, nv = tm.attention_with_cache(attn[li], inputs[li], None, self.pe,
                                                          None, lay.video_self_k,
                                                          lay.video_self_v,
                                                          profile_name="video_self")
                    kv.append((nk, nv))
                return out, kv

            self.out, self.kv = self.graph.capture(forward)
            # read-back: a kernel copy into one of two device buffers on the
            # compute stream, then the device-to-host copy on the read-back
            # stream, so that the next forward does not wait for PCIe
            self.stage = [torch.empty_like(self.out) for _ in range(2)]
            self.read_done = [None, None]

        def read_back(self, fwd, host):
            i = fwd % 2
            main = torch.cuda.current_stream(dev)
            if self.read_done[i] is not None:
                main.wait_event(self.read_done[i])  # that buffer's previous copy has left
            copy_bytes(self.stage[i].data_ptr(), self.out.data_ptr(),
                       self.out.numel() * self.out.element_size(), dev)
            ready = torch.cuda.Event()
            ready.record(main)
            read_stream.wait_event(ready)
            with torch.cuda.stream(read_stream):
                host.copy_(self.stage[i], non_blocking=True)
                done = torch.cuda.Event()
                done.record(read_stream)
            self.read_done[i] = done

        def step(self, cache, block, outs=None):
            c, s = tables(block)  # once per block: the four forwards share the start frame
            copy_into(self.pe[0], c)  # kernel copies: nothing queues behind the input upload
            copy_into(self.pe[1], s)
            spans = [attention_spans(lay.video_self_k, lay.video_self_v, Lq)
                     for lay in cache.layers]
            for fwd in range(FORWARDS_PER_STEP):
                self.graph.replay(spans if fwd == 0 else None)
                if outs is not None:
                    self.read_back(fwd, outs[fwd])
            new_layers = []
            for li, lay in enumerate(cache.layers):
                nk, nv = self.kv[li]
                k2, v2 = tm.cat_cache_pair(lay.video_self_k, lay.video_self_v, nk, nv)
                k2.entries()  # into its slot now: the next replay rewrites nk / nv
                new_layers.append(LayerKVCache(video_self_k=k2, video_self_v=v2))
            return retain_window(KVCache(layers=new_layers), anchor, window)

    def timed(n_steps, n_warm, host_io, graphed=False, sections=False):
        cache = fresh_cache()
        x_host = outs = None
        if host_io:
            x_host = [x.cpu().pin_memory() for x in xs]
            x_dev = [torch.empty_like(x) for x in xs]
            outs = [torch.empty(1, S_loc, HIDDEN, dtype=torch.bfloat16).pin_memory()
                    for _ in range(FORWARDS_PER_STEP)]
        block = 0
        runners = []
        with torch.no_grad():
            for _ in range(n_warm):
                cache = step(cache, block)
                block += 1
            if graphed:
                if sections:
                    TIMER.start()  # the sections become event nodes of the captured graph
                runners.append(GraphRunner(cache, block, xs))
                TIMER.stop()
                if host_io:
                    # a second captured forward with its own inputs: the next step's
                    # host-to-device copy overlaps this step's forwards
                    runners.append(GraphRunner(cache, block, [torch.empty_like(x) for x in xs]))
        runner = runners[0] if runners else None
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        l0 = _lib.LAUNCHES
        if sections and not graphed:
            TIMER.start()
        sampler = ClockSampler(local)
        sampler.start()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        with torch.no_grad():
            if runner is not None and host_io:
                main = torch.cuda.current_stream(dev)
                cs = torch.cuda.Stream(dev)
                ready = [torch.cuda.Event(), torch.cuda.Event()]
                done = [None, None]

                def upload(r):
                    with torch.cuda.stream(cs):
                        if done[r] is not None:
                            cs.wait_event(done[r])  # its previous forwards have read it
                        for li in range(L):
                            runners[r].inputs[li].copy_(x_host[li], non_blocking=True)
                        ready[r].record(cs)

                cs.wait_stream(main)
                upload(0)
            for i in range(n_steps):
                if runner is not None and host_io:
                    r = i % 2
                    main.wait_event(ready[r])
                    if i + 1 < n_steps:
                        upload(1 - r)
                    cache = runners[r].step(cache, block, outs)
                    done[r] = torch.cuda.Event()
                    done[r].record(main)
                elif runner is not None:
                    cache = runner.step(cache, block, outs)
                elif host_io:
                    for li in range(L):
                        x_dev[li].copy_(x_host[li], non_blocking=True)
                    cache = step(cache, block, x_dev, outs)
                else:
                    cache = step(cache, block)
                block += 1
            # the timed region ends once the last read-back has reached the host
            torch.cuda.current_stream(dev).wait_stream(read_stream)
        e1.record()
        torch.cuda.synchronize()
        clocks = sampler.stop()
        TIMER.stop()
        launches = _lib.LAUNCHES - l0
        ms = e0.elapsed_time(e1)
        # a bounded device wait that ran out (a lost peer, a stuck pipeline)
        # would leave stale rows behind: read the flag after every pass
        derr = _lib.device_error()
        if world > 1:
            t = torch.tensor([ms, float(derr)], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms, derr = float(t[0].item()), int(t[1].item())
            dist.barrier()
        DEVICE_ERRORS.append(derr)
        h2d = sum(x.numel() * x.element_size() for x in xs) if host_io else 0
        d2h = FORWARDS_PER_STEP * S_loc * HIDDEN * 2 if host_io else 0
        for r in runners:
            r.graph.reset()  # before the process group its exchanges use goes away
        runners.clear()
        runner = None
        return ms, launches, clocks, h2d, d2h

    DEVICE_ERRORS = []
    graphed = not args.eager
    ms, launches, clocks, _, _ = timed(args.steps, args.warmup, host_io=False, graphed=graphed)
    value = Q_FRAMES * args.steps / (ms / 1e3)
    # Per-section times (the attention launch among them) come from a second
    # pass of the same steps whose captured forward also holds event nodes
    # around each section; the headline pass above has none.
    timed(args.steps, args.warmup, host_io=False, graphed=graphed, sections=True)
    sections = TIMER.summary()

    e2e = None
    if not args.no_e2e and args.workload == "attention":
        ems, _, _, h2d, d2h = timed(args.steps, args.warmup, host_io=True, graphed=graphed)
        e2e = {"value": Q_FRAMES * args.steps / (ems / 1e3), "unit": "latent frames/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "ms_per_step": ems / args.steps}

    peaks, peak_kind = measured_peaks()
    sd = sections.get("video_self.sdpa")
    Lkv = anchor + window + Lq
    flops = 4.0 * Lq * Lkv * H_loc * DIM_HEAD
    roof = None
    if sd:
        achieved = flops / (sd["mean_ms"] * 1e-3) / 1e12
        peak = float(peaks["bf16_tflops_sustained"])
        traffic = profiled_traffic("attn_fwd_kernel<128>", H_loc)
        roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "traffic": traffic,
                "kernel": "tm attention (tcgen05)", "launch_ms": sd["mean_ms"],
                "flops_per_launch": flops,
                "peak_source": f"{peak_kind} bf16_tflops_sustained (kernel timed inside a long step)"}

    del attn, xs
    return {"value": value, "ms_per_step": ms / args.steps, "e2e": e2e, "roofline": roof,
            "gpu_launches": launches, "clocks": clocks, "device_error": max(DEVICE_ERRORS),
            "sections_ms_per_call": {k: v["mean_ms"] for k, v in sections.items()},
            "config": {"workload": "C2 video self-attention, 48 layers x (3 denoise + 1 commit) "
                                   "forwards per 3-frame block",
                       "q_tokens": Lq, "cached_tokens": anchor + window, "keys_per_query": Lkv,
                       "heads": HEADS, "dim_head": DIM_HEAD,
                       "cache": "1 anchor + 8 window frames"}}


# --------------------------------------------------------------------------- C4
def c4_flops(cfg, Lv, La, cached_v, cached_a, text):
    """Algorithmic FLOPs of one layer-forward of the block (2 per MAC for the
    linears, 4 * Lq * Lk * inner for each attention) and of the per-block text
    K/V projection of one layer."""
    Dv, Da = cfg.video_dim, cfg.audio_dim
    iv, ia = cfg.video_heads * cfg.video_dim_head, cfg.audio_heads * cfg.audio_dim_head
    lin = lambda m, k, n: 2.0 * m * k * n
    att = lambda q, k, inner: 4.0 * q * k * inner
    f = 0.0
    f += lin(Lv, Dv, 3 * iv) + att(Lv, cached_v + Lv, iv) + lin(Lv, iv, Dv)      # video self
    f += lin(Lv, Dv, iv) + att(Lv, text, iv) + lin(Lv, iv, Dv)                    # video text
    f += lin(La, Da, 3 * ia) + att(La, cached_a + La, ia) + lin(La, ia, Da)      # audio self
    f += lin(La, Da, ia) + att(La, text, ia) + lin(La, ia, Da)                    # audio text
    f += lin(Lv, Dv, ia) + 2 * lin(La, Da, ia) + att(Lv, cached_a + La, ia) + lin(Lv, ia, Dv)  # A2V
    f += lin(La, Da, ia) + 2 * lin(Lv, Dv, ia) + att(La, cached_v + Lv, ia) + lin(La, ia, Da)  # V2A
    f += 2 * lin(Lv, Dv, 4 * Dv) + 2 * lin(La, Da, 4 * Da)                        # FFNs
    text_kv = 2 * lin(text, Dv, iv) + 2 * lin(text, Da, ia)
    return f, text_kv


def c4_step(args, dev, rank, world, local, read_stream):
    """The headline workload: one streaming block of the
    48-layer joint audio-video model = text K/V projection + 3 denoising
    forwards + 1 commit forward + eviction, at the steady-state cache (sink
    block of 4 frames + 2 window blocks of 3 frames: 3840 video / 76 audio
    cached tokens, 4992 / 101 keys)."""
    import torch
    import torch.distributed as dist
    from taomate_b200 import _lib
    from taomate_b200.model import CausalModelWeights, StreamConfig, synthetic_conditioning
    from taomate_b200.profiler import TIMER
    from taomate_b200.stream import StreamRunner, block_geometry

    cfg = StreamConfig(layers=args.layers)
    torch.manual_seed(0)  # identical weights on every rank
    model = CausalModelWeights(cfg, device=dev)
    gen = torch.Generator(device=dev).manual_seed(7)
    C = cfg.in_channels

    def block_inputs(k):
        F_, La, _, _ = block_geometry(k, cfg)
        Lv = F_ * cfg.frame_tokens
        n = Lv // world
        v = torch.randn(1, Lv, C, device=dev, generator=gen).to(torch.bfloat16)
        v = v[:, rank * n:(rank + 1) * n].contiguous()
        a = torch.randn(1, La, C, device=dev, generator=gen).to(torch.bfloat16)
        conds = [synthetic_conditioning(cfg, F_, La, dev, gen) for _ in range(4)]
        return v, a, conds

    prompt = synthetic_conditioning(cfg, 3, 25, dev, gen)

    def timed(n_steps, n_warm, host_io=False, sections=False):
        runner = StreamRunner(model, dev, sp=world, rank=rank, graphed=not args.eager,
                              overlap_audio=not args.serial_audio)
        runner.set_prompt(prompt.video_ctx, prompt.audio_ctx)
        for k in range(n_warm):  # eager blocks until the steady state, then capture
            runner.run_block(*block_inputs(k))
        if sections:
            TIMER.start()
        steady = [block_inputs(n_warm + i) for i in range(n_steps)]
        runner.run_block(*steady[0])  # capture (if not yet) + one replay, untimed
        TIMER.stop()
        runner.host_ms, runner.host_blocks = {}, 0  # host time of the timed blocks only
        host = None
        if host_io:
            flat = lambda v, a, conds: [v, a] + [getattr(c, nm) for c in conds
                                                 for nm in COND_NAMES]
            host = [[t.cpu().pin_memory() for t in flat(*b)] for b in steady]
            dev_in = [[torch.empty_like(t) for t in flat(*steady[0])] for _ in range(2)]
            outs = [(torch.empty(steady[0][0].shape, dtype=torch.bfloat16).pin_memory(),
                     torch.empty(steady[0][1].shape, dtype=torch.bfloat16).pin_memory())
                    for _ in range(n_steps)]
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        l0 = _lib.LAUNCHES
        sampler = ClockSampler(local)
        sampler.start()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        main = torch.cuda.current_stream(dev)
        e0.record()
        with torch.no_grad():
            if host_io:
                cs = torch.cuda.Stream(dev)
                ready = [torch.cuda.Event(), torch.cuda.Event()]
                done = [None, None]

                def upload(i):
                    r = i % 2
                    with torch.cuda.stream(cs):
                        if done[r] is not None:
                            cs.wait_event(done[r])
                        for d, h in zip(dev_in[r], host[i]):
                            d.copy_(h, non_blocking=True)
                        ready[r].record(cs)

                cs.wait_stream(main)
                upload(0)
            for i in range(n_steps):
                if host_io:
                    r = i % 2
                    main.wait_event(ready[r])
                    if i + 1 < n_steps:
                        upload(i + 1)
                    t = dev_in[r]
                    nc = len(COND_NAMES)
                    conds = [Cond(**dict(zip(COND_NAMES, t[2 + j * nc:2 + (j + 1) * nc])))
                             for j in range(4)]
                    vo, ao = runner.run_block(t[0], t[1], conds)
                    done[r] = torch.cuda.Event()
                    done[r].record(main)
                    read_stream.wait_stream(main)
                    with torch.cuda.stream(read_stream):
                        outs[i][0].copy_(vo, non_blocking=True)
                        outs[i][1].copy_(ao, non_blocking=True)
                        vo.record_stream(read_stream)
                        ao.record_stream(read_stream)
                else:
                    runner.run_block(*steady[i])
            main.wait_stream(read_stream)
        e1.record()
        torch.cuda.synchronize()
        clocks = sampler.stop()
        launches = _lib.LAUNCHES - l0
        ms = e0.elapsed_time(e1)
        derr = _lib.device_error()
        if world > 1:
            t = torch.tensor([ms, float(derr)], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms, derr = float(t[0].item()), int(t[1].item())
            dist.barrier()
        DEVICE_ERRORS.append(derr)
        h2d = d2h = 0
        if host_io:
            h2d = sum(x.numel() * x.element_size() for x in host[0])
            d2h = sum(x.numel() * x.element_size() for x in outs[0])
        cache_bytes = live_cache_bytes(runner.cache)
        HOST_MS.clear()
        if runner.host_blocks:
            HOST_MS.update({k: v / runner.host_blocks for k, v in runner.host_ms.items()})
        runner.release()
        return ms, launches, clocks, h2d, d2h, cache_bytes

    DEVICE_ERRORS = []
    HOST_MS = {}
    warm = max(args.warmup, 3)
    ms, launches, clocks, _, _, cache_bytes = timed(args.steps, warm)
    host_ms = dict(HOST_MS)  # host time per replayed block of the headline pass, by phase
    value = 3.0 * args.steps / (ms / 1e3)
    # 3 warm-up blocks: the steady-state layout is then captured with the timer on
    timed(max(2, min(args.steps, 5)), 3, sections=True)
    sections = TIMER.summary()
    e2e = None
    if not args.no_e2e:
        ems, _, _, h2d, d2h, _ = timed(args.steps, warm, host_io=True)
        e2e = {"value": 3.0 * args.steps / (ems / 1e3), "unit": "latent frames/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "ms_per_step": ems / args.steps}

    Lv, La = 3 * cfg.frame_tokens, 25
    per_layer, text_kv = c4_flops(cfg, Lv, La, 3840, 76, cfg.text_tokens)
    step_flops = cfg.layers * (4 * per_layer + text_kv)
    peaks, peak_kind = measured_peaks()
    sd = sections.get("video_self.sdpa")
    H_loc = cfg.video_heads // world
    flops = 4.0 * Lv * (3840 + Lv) * H_loc * cfg.video_dim_head
    roof = None
    if sd:
        achieved = flops / (sd["mean_ms"] * 1e-3) / 1e12
        peak = float(peaks["bf16_tflops_sustained"])
        roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak,
                "traffic": profiled_traffic("attn_fwd_kernel<128>", H_loc, keys=3840 + Lv),
                "kernel": "tm attention (tcgen05), video self-attention",
                "launch_ms": sd["mean_ms"], "flops_per_launch": flops,
                "peak_source": f"{peak_kind} bf16_tflops_sustained (kernel timed inside a long "
                               "step)"}
    del model
    torch.cuda.empty_cache()
    step_s = ms / args.steps / 1e3
    return {"value": value, "ms_per_step": ms / args.steps, "e2e": e2e, "roofline": roof,
            "gpu_launches": launches, "clocks": clocks, "device_error": max(DEVICE_ERRORS),
            "sections_ms_per_call": {k: v["mean_ms"] for k, v in sections.items()},
            "step_flops": step_flops, "host_ms_per_block": host_ms,
            "step_tflops": step_flops / world / step_s / 1e12,
            "kv_cache_bytes_per_gpu": cache_bytes,
            # real time = 3 latent frames/s (24 fps video, 8x temporal compression)
            "realtime_factor": value / 3.0}


def c5_longform(args, dev, rank, world, local):
    """a 60 s stream = 12 segments x 5 blocks (4-3-3-3-3
    latent frames in the first window, then 3 per block; 181 latent frames),
    as taomate/inference/runtime.py:569-634 drives it: a new prompt every
    segment, whose K/V refresh re-prefills the retained blocks (sigma = 0
    kv_cache_only forwards, runtime.py:386-470) from segment 1 on; no eviction
    inside the first window, then sink + 2 newest after every block, and at
    every window end.  Timed as a whole on the device (max over ranks): every
    block and every refresh of the 60 s stream.  Before it, a warm-up stream
    (the first window, one refresh, one block) captures the CUDA graphs of
    every cache layout the stream meets, as a service does once at start;
    the runner is then reset (same arenas, empty cache) and the timed stream
    replays them from its first block (``graph_captures_timed`` counts any
    capture inside the timed region)."""
    import torch
    import torch.distributed as dist
    from taomate_b200 import _lib
    from taomate_b200.model import CausalModelWeights, StreamConfig, synthetic_conditioning
    from taomate_b200.stream import StreamRunner, block_geometry

    cfg = StreamConfig(layers=args.layers)
    torch.manual_seed(0)
    model = CausalModelWeights(cfg, device=dev)
    gen = torch.Generator(device=dev).manual_seed(9)
    C = cfg.in_channels
    segs, per = args.segments, 5
    prompts = [synthetic_conditioning(cfg, 3, 25, dev, gen) for _ in range(segs)]
    zero = {4: synthetic_conditioning(cfg, 4, 26, dev, gen),
            3: synthetic_conditioning(cfg, 3, 25, dev, gen)}  # sigma = 0 rows by block size

    def block_inputs(k):
        F_, La, _, _ = block_geometry(k, cfg)
        n = F_ * cfg.frame_tokens // world
        v = torch.randn(1, n, C, device=dev, generator=gen).to(torch.bfloat16)
        a = torch.randn(1, La, C, device=dev, generator=gen).to(torch.bfloat16)
        return v, a, [synthetic_conditioning(cfg, F_, La, dev, gen) for _ in range(4)]

    runner = StreamRunner(model, dev, sp=world, rank=rank, graphed=not args.eager,
                          evict_from_block=per, overlap_audio=not args.serial_audio)
    # warm-up stream: window 0, a prompt change with its refresh, one block of window 1
    warm_in = [block_inputs(k) for k in range(per + 1)]
    runner.set_prompt(prompts[0].video_ctx, prompts[0].audio_ctx)
    for k in range(per):
        runner.run_block(*warm_in[k])
    runner.end_segment()
    runner.set_prompt(prompts[1 % segs].video_ctx, prompts[1 % segs].audio_ctx)
    runner.refresh({int(sg["block_idx"]): zero[block_geometry(int(sg["block_idx"]), cfg)[0]]
                    for sg in runner.cache.segments})
    runner.run_block(*warm_in[per])
    del warm_in
    runner.reset()
    captures0 = runner.captures
    inputs = [block_inputs(k) for k in range(segs * per)]
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    frames = 0
    peak_cache = 0
    for sgi in range(segs):
        runner.set_prompt(prompts[sgi].video_ctx, prompts[sgi].audio_ctx)
        if sgi > 0:
            conds = {int(sg["block_idx"]): zero[block_geometry(int(sg["block_idx"]), cfg)[0]]
                     for sg in runner.cache.segments}
            runner.refresh(conds)
        for b in range(per):
            k = sgi * per + b
            runner.run_block(*inputs[k])
            frames += block_geometry(k, cfg)[0]
            peak_cache = max(peak_cache, live_cache_bytes(runner.cache))
        runner.end_segment()
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    derr = _lib.device_error()
    live = live_cache_bytes(runner.cache)
    arena = sum(getattr(lay, f).arena.k.numel() * 2 * 2 for lay in runner.cache.layers
                for f in ("video_self_k", "audio_self_k", "a2v_k", "v2a_k"))
    if world > 1:
        t = torch.tensor([ms, float(derr)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, derr = float(t[0].item()), int(t[1].item())
    captured = runner.graph is not None
    captures = runner.captures - captures0
    runner.release()
    del model
    torch.cuda.empty_cache()
    video_s = (1 + 8 * (frames - 1)) / 24.0  # pixel frames at 24 fps (8x temporal compression)
    return {"metric": "sustained latent frames/s over a 60 s stream (12 segments x 5 blocks)",
            "value": frames / (ms / 1e3), "unit": "latent frames/s", "n_gpus": world,
            "blocks": segs * per, "latent_frames": frames, "video_seconds": video_s,
            "wall_ms": ms, "realtime_factor": video_s / (ms / 1e3),
            "refreshes": runner.refreshes, "graph_captured": captured,
            "graph_captures_timed": captures,
            "kv_cache_bytes_per_gpu": live, "kv_cache_peak_bytes_per_gpu": peak_cache,
            "kv_arena_bytes_per_gpu": arena, "clocks": clocks, "device_error": derr,
            "config": {"workload": "C5: 60 s long-form stream", "segments": segs,
                       "blocks_per_segment": per, "layers": args.layers,
                       "prompt": "new 256-token text conditioning every segment (N(0, 1)), "
                                 "K/V refresh of the retained blocks",
                       "parallelism": f"ulysses sp{world} (video split, audio replicated)"
                                      if world > 1 else "single gpu"}}


COND_NAMES = ("video_ts", "audio_ts", "video_cross_ss", "video_cross_gate", "audio_cross_ss",
              "audio_cross_gate", "video_emb2", "audio_emb2")


def Cond(**kw):
    """Per-forward conditioning rows (the text contexts and RoPE tables are the
    runner's own)."""
    import torch
    from taomate_b200.model import Conditioning
    z = torch.empty(0)
    return Conditioning(video_ctx=z, audio_ctx=z, **kw)


def live_cache_bytes(cache):
    """Bytes of K/V rows the cache's views reference (every layer and field)."""
    total = 0
    for lay in cache.layers:
        for f in ("video_self_k", "video_self_v", "audio_self_k", "audio_self_v", "a2v_k",
                  "a2v_v", "v2a_k", "v2a_v"):
            t = getattr(lay, f)
            if t is None:
                continue
            total += int(t.shape[1]) * int(t.shape[2]) * int(t.shape[3]) * 2
    return total


def sp_parity(dev, rank, world):
    """Sequence-parallel results against the same call on one GPU, on this box:
    one C2 ``attention_with_cache`` call (fused NVLink exchanges) and one
    48-layer-model block forward at C4 shapes (replicated audio, split-key
    V2A).  Each rank runs the single-GPU call itself (all tokens, all heads)
    and compares its own output rows / heads.  Max over ranks."""
    import torch
    import torch.distributed as dist
    import taomate_b200 as tm
    from taomate_b200 import parallel as P
    from taomate_b200.attention import AttentionWeights
    from taomate_b200.model import StreamConfig, rope_tables, synthetic_conditioning
    from taomate_b200.block import BlockWeights, fuse_block_weights
    from taomate_b200.kv_cache import LayerKVCache

    rel = lambda a, b: float(torch.linalg.norm((a.float() - b.float()).double())
                             / torch.linalg.norm(b.float().double()))
    g = torch.Generator(device=dev).manual_seed(11)
    Lq, S = Q_FRAMES * FRAME_TOKENS, Q_FRAMES * FRAME_TOKENS // world
    Hl = HEADS // world
    ts, hs = slice(rank * S, (rank + 1) * S), slice(rank * Hl, (rank + 1) * Hl)
    torch.manual_seed(5)
    attn = AttentionWeights(HIDDEN, HEADS, DIM_HEAD, device=dev)
    tm.fuse_qkv_weights(attn)
    x = torch.randn(1, Lq, HIDDEN, device=dev, generator=g).to(torch.bfloat16)
    ck = torch.randn(1, 3456, HEADS, DIM_HEAD, device=dev, generator=g).to(torch.bfloat16)
    cv = torch.randn(1, 3456, HEADS, DIM_HEAD, device=dev, generator=g).to(torch.bfloat16)
    cos, sin = tm.causal_precompute_freqs_cis(torch.tensor([[Q_FRAMES, 16, 24]]), HIDDEN,
                                              start_frame=9, device=dev, dtype=torch.bfloat16,
                                              num_attention_heads=HEADS)
    out = {}
    with torch.no_grad():
        with P.sp_local():
            r_out, r_k, r_v = tm.attention_with_cache(attn, x, None, (cos, sin), None, ck, cv)
        s_out, s_k, s_v = tm.attention_with_cache(
            attn, x[:, ts].contiguous(), None, (cos[:, :, ts], sin[:, :, ts]), None,
            ck[:, :, hs].contiguous(), cv[:, :, hs].contiguous())
        out["attention_with_cache_c2"] = {"out": rel(s_out, r_out[:, ts]),
                                          "new_k": rel(s_k, r_k[:, :, hs]),
                                          "new_v": rel(s_v, r_v[:, :, hs])}
        del attn
        cfg = StreamConfig(layers=1)
        torch.manual_seed(6)
        blk = BlockWeights(device=dev)
        fuse_block_weights(blk)
        cond = synthetic_conditioning(cfg, 3, 25, dev, g)
        vx = torch.randn(1, Lq, cfg.video_dim, device=dev, generator=g).to(torch.bfloat16)
        ax = torch.randn(1, 25, cfg.audio_dim, device=dev, generator=g).to(torch.bfloat16)
        args = lambda pe, vx_, off, rep: dict(
            video_timestep_6d=cond.video_ts, audio_timestep_6d=cond.audio_ts, video_pe=pe[0],
            audio_pe=pe[1], video_cross_pe=pe[2], audio_cross_pe=pe[3], video_ctx=cond.video_ctx,
            audio_ctx=cond.audio_ctx, video_context_mask=None, audio_context_mask=None,
            video_cross_ss=cond.video_cross_ss, video_cross_gate=cond.video_cross_gate,
            audio_cross_ss=cond.audio_cross_ss, audio_cross_gate=cond.audio_cross_gate,
            video_prompt_ts=None, audio_prompt_ts=None, layer_cache=LayerKVCache(),
            video_frame_seqlen=cfg.frame_tokens, audio_frame_seqlen=1, video_token_offset=off,
            audio_replicated=rep)
        pe_full = rope_tables(cfg, 3, 25, 9, 76, dev)
        pe_loc = rope_tables(cfg, 3, 25, 9, 76, dev, ts)
        with P.sp_local():
            rv, ra, _ = tm.block_forward_with_cache(blk, vx, ax, **args(pe_full, vx, 0, False))
        sv, sa, _ = tm.block_forward_with_cache(blk, vx[:, ts].contiguous(), ax,
                                                **args(pe_loc, None, rank * S, True))
        out["block_c4"] = {"video_x": rel(sv, rv[:, ts]), "audio_x": rel(sa, ra)}
    t = torch.tensor([v for d in out.values() for v in d.values()], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    vals = iter(t.tolist())
    res = {k: {kk: next(vals) for kk in d} for k, d in out.items()}
    res["bar"] = 1e-2
    res["what"] = ("relative L2, sequence-parallel vs single-GPU call on the same inputs "
                   "(projection GEMMs round on 1152/G rows vs 1152), max over ranks")
    return res


def run_ours(args):
    import torch
    import torch.distributed as dist
    from taomate_b200 import parallel as P

    rank, world, local = env_rank()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        P.init_sp_mesh(world, world)
        if not args.nccl_exchange:
            from taomate_b200.block import v2a_gather_bytes
            P.init_peer_exchange(1, Q_FRAMES * FRAME_TOKENS // world, HEADS, DIM_HEAD,
                                 gather_bytes=v2a_gather_bytes(26, 32, 64, world))
    read_stream = torch.cuda.Stream(dev)
    if args.workload == "c5":
        line = c5_longform(args, dev, rank, world, local)
        if rank == 0:
            print(json.dumps(line), flush=True)
        if world > 1:
            dist.barrier()
            P.close_peer_exchange()
            dist.destroy_process_group()
        return
    parity = sp_parity(dev, rank, world) if world > 1 else None
    c4 = None if args.workload == "attention" else c4_step(args, dev, rank, world, local,
                                                           read_stream)
    att = None
    if args.workload in ("attention", "both"):
        att = attention_step(args, dev, rank, world, local)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_c4_sample(args.layers) if c4 is not None else None
    if rank == 0:
        head = c4 if c4 is not None else att
        line = {
            "metric": METRIC_C4 if c4 is not None else METRIC_ATT,
            "value": head["value"], "unit": "latent frames/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (random N(0, 0.02) weights, N(0, 1) latents and "
                                     "text, N(0, 0.1) AdaLN rows)",
            "config": (C4_CONFIG if c4 is not None else head["config"]) | {
                "parallelism": (f"ulysses sp{world} (video split by tokens, audio replicated), "
                                "video self-attention exchanges "
                                + ("nccl all_to_all" if args.nccl_exchange
                                   else "fused NVLink peer stores")
                                + ", split-key V2A (partial results gathered over "
                                + ("nccl)" if args.nccl_exchange else "NVLink)")
                                + (", audio chain on the main stream" if args.serial_audio
                                   else ", audio chain on a second stream"))
                               if world > 1 else "single gpu",
                "executor": "eager" if args.eager else "cuda graph per forward layout (block 0 "
                                                       "eager, one capture per cache layout)",
                "layers": args.layers,
                "l2": "inputs larger than L2 (48 layers of weights ~38 GB, caches, activations), "
                      "no flush"},
            "roofline": head["roofline"], "cpu_baseline": cpu, "e2e": head["e2e"],
            "gpu_launches": head["gpu_launches"], "clocks": head["clocks"],
            "device_error": max(x["device_error"] for x in (c4, att) if x is not None),
            "sections_ms_per_call": head["sections_ms_per_call"],
        }
        if c4 is not None:
            line.update({k: c4[k] for k in ("step_flops", "step_tflops", "kv_cache_bytes_per_gpu",
                                            "realtime_factor", "host_ms_per_block")})
            if att is not None:
                line["attention_step"] = {k: att[k] for k in ("value", "ms_per_step", "roofline",
                                                              "sections_ms_per_call", "config")}
                line["attention_step"]["metric"] = METRIC_ATT
        if parity is not None:
            line["parity_rel_l2"] = parity
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        P.close_peer_exchange()
        dist.destroy_process_group()


METRIC_C4 = "latent frames/s at 512x768 (48-block causal audio-video step)"
METRIC_ATT = "latent frames/s at 512x768 (48-layer video self-attention step)"
C4_CONFIG = {
    "workload": "C4: one streaming block of the 48-block joint audio-video model = text K/V "
                "projection + 3 denoising forwards + 1 commit forward + eviction",
    "video": "hidden 4096 = 32 x 128, 3 latent frames of 16 x 24 = 1152 tokens per block",
    "audio": "hidden 2048 = 32 x 64, 25 tokens per block",
    "text": "256 tokens (video context 4096, audio context 2048)",
    "cache": "steady state of the reference policy: sink block (4 frames, 26 audio) + 2 newest "
             "blocks = 3840 video / 76 audio cached tokens (4992 / 101 keys)",
    "ffn": "mult 4, tanh GELU", "adaln": "per-frame (video) / per-token (audio) rows",
}


def run_kernel_case(args):
    """One kernel at C2 shapes, ``--reps`` launches, CUDA-event time per launch."""
    import torch
    import taomate_b200 as tm
    from taomate_b200.rope import norm_rope
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    Lq = Q_FRAMES * FRAME_TOKENS
    Lc = args.cached or (ANCHOR_FRAMES + WINDOW_FRAMES) * FRAME_TOKENS
    rnd = lambda *s: torch.randn(*s, device=dev, generator=g).to(torch.bfloat16)
    if args.kernel_case == "linear":
        return run_linear_case(args, dev, rnd)
    if args.kernel_case == "attention":
        Hk = args.heads or HEADS
        q = rnd(1, Lq, Hk, DIM_HEAD)
        ck, cv = rnd(1, Lc, Hk, DIM_HEAD), rnd(1, Lc, Hk, DIM_HEAD)
        nk, nv = rnd(1, Lq, Hk, DIM_HEAD), rnd(1, Lq, Hk, DIM_HEAD)
        out = torch.empty_like(q)
        fn = lambda: tm.flash_attention(q, ck, cv, [(0, Lc)], nk, nv, Lq, out=out)
        work, unit = 4.0 * Lq * (Lc + Lq) * Hk * DIM_HEAD / 1e12, "TFLOP/s"
    elif args.kernel_case == "kv_append":
        # the commit append: one block's K and V [1152, 32, 128] into an arena slot
        from taomate_b200.kv_cache import KVArena
        arena = KVArena(2, Lq, 1, HEADS, DIM_HEAD, dtype=torch.bfloat16, device=dev)
        nk, nv = rnd(1, Lq, HEADS, DIM_HEAD), rnd(1, Lq, HEADS, DIM_HEAD)

        def fn():
            ents = arena.write(nk, nv)
            for (slot, _, _) in ents:  # give the slot back: the same copy every launch
                arena._ref(slot, -1)

        work, unit = 4.0 * Lq * HEADS * DIM_HEAD * 2 / 1e9, "GB/s"
    elif args.kernel_case == "residual_norm":
        # the cross-modal boundary of the C4 block: r = x + y * gate stored, then two
        # modulations of rms_norm(r) (A2V and V2A inputs); AdaLN rows per frame
        from taomate_b200.block import AdaParams, residual_norm
        x, y = rnd(1, Lq, HIDDEN), rnd(1, Lq, HIDDEN)
        o1, o2 = torch.empty_like(x), torch.empty_like(x)
        table = rnd(6, HIDDEN) * 0.1
        ts = rnd(1, Q_FRAMES, 6 * HIDDEN) * 0.1
        prm = AdaParams(table, ts, Lq, 6, HIDDEN, FRAME_TOKENS, 0)
        fn = lambda: residual_norm(x, y, prm, 2, x, [(o1, prm, 1, 0), (o2, prm, 4, 3)])
        work, unit = 5 * Lq * HIDDEN * 2 / 1e9, "GB/s"  # x, y read; x, o1, o2 written
    else:
        xq, xk = rnd(1, Lq, HIDDEN), rnd(1, Lq, HIDDEN)
        w = torch.ones(HIDDEN, device=dev, dtype=torch.bfloat16)
        cos, sin = tm.causal_precompute_freqs_cis(torch.tensor([[Q_FRAMES, 16, 24]]), HIDDEN,
                                                  device=dev, dtype=torch.bfloat16,
                                                  num_attention_heads=HEADS)
        fn = lambda: norm_rope([xq, xk], [w, w], [(cos, sin), (cos, sin)], HEADS, DIM_HEAD, 1e-6)
        work, unit = (4 * Lq * HIDDEN * 2 + 2 * cos.numel() * 2) / 1e9, "GB/s"
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    # replay a captured launch so the host-side wrapper cost stays out of the timing
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    graph.replay()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.reps)]
    for a, b in ev:
        a.record()
        graph.replay()
        b.record()
    torch.cuda.synchronize()
    ms = sorted(a.elapsed_time(b) for a, b in ev)
    med = ms[len(ms) // 2]
    print(json.dumps({"kernel_case": args.kernel_case, "heads": args.heads or HEADS,
                      "cached": Lc,
                      "median_ms": med, "min_ms": ms[0],
                      "achieved": work / (med * 1e-3), "unit": unit}), flush=True)


def run_linear_case(args, dev, rnd):
    """cuBLAS (torch F.linear, bias included) at the block's weight shapes and
    ``--rows`` token rows, as the captured step runs them: one CUDA graph of
    consecutive calls over rotating weight copies (more bytes than L2 holds),
    so launch gaps and L2 reuse match the step.  Prints one line per shape
    with the time per call and the weight-read floor at the measured HBM
    bandwidth."""
    import torch
    import torch.nn.functional as F
    peaks, kind = measured_peaks()
    hbm = float(peaks["hbm_gbs"]) * 1e9
    shapes = {"video_qkv": (4096, 12288), "video_out": (4096, 4096), "ff1": (4096, 16384),
              "ff2": (16384, 4096), "a2v_q": (4096, 2048), "v2a_kv": (4096, 4096),
              "audio_qkv": (2048, 6144), "audio_out": (2048, 2048), "audio_ff1": (2048, 8192),
              "audio_ff2": (8192, 2048)}
    M = args.rows
    for name, (K, N) in shapes.items():
        copies = min(16, max(2, int(4 * 134e6 // (K * N * 2)) + 1))
        ws = [rnd(N, K) * 0.02 for _ in range(copies)]
        b = rnd(N) * 0.1
        x = rnd(M, K)
        for i in range(copies):
            F.linear(x, ws[i], b)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(copies):
                F.linear(x, ws[i], b)
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (args.reps * copies)
        floor = K * N * 2 / hbm * 1e6
        print(json.dumps({"kernel_case": "linear", "shape": name, "rows": M, "K": K, "N": N,
                          "us_per_call": round(us, 2), "weight_floor_us": round(floor, 2),
                          "floor_source": f"{kind} hbm_gbs",
                          "tflops": round(2 * M * K * N / us / 1e6, 1)}), flush=True)
        del ws
        torch.cuda.empty_cache()


def main():
    args = parse()
    if args.kernel_case:
        run_kernel_case(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
