"""The streaming block loop (taomate_b200.stream.StreamRunner) on one GPU.

A 2-layer model at small shapes (video 4 heads x 128 over 8 x 12 tokens per
frame, audio 4 heads x 64, text 24 tokens) runs the pipeline's schedule:
block 0 of 4 frames, then blocks of 3 frames, each with 3 denoising forwards
and a commit forward, eviction to the sink block + the 2 newest blocks.

* The CUDA-graph executor (one capture per cache layout from block 1 on,
  replayed with a rewritten key-tile table, kernel-copied inputs, per-block
  text K/V graph) gives the same bits as issuing every forward eagerly; the
  refresh forwards replay the first window's layouts.
* The retained segments follow the reference policy ([0], [0,1], [0,1,2],
  [0,2,3], [0,3,4], ...) and the cache holds 3840-equivalent rows (sink + 2
  blocks) at the steady state.
* A prompt change reaches the captured graph (the outputs change and match
  the eager run with the same prompt change).
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0") if torch.cuda.is_available() else None


@pytest.fixture(scope="module", autouse=True)
def _device():
    if DEV is None:
        pytest.skip("no CUDA device")
    torch.cuda.set_device(DEV)
    yield
    from taomate_b200 import _lib
    assert _lib.device_error() == 0, "a kernel set the device error flag"


def _run(graphed, n_blocks=7, prompt_change_at=5):
    from taomate_b200.model import CausalModelWeights, StreamConfig, synthetic_conditioning
    from taomate_b200.stream import StreamRunner, block_geometry
    cfg = StreamConfig(layers=2, video_dim=512, video_heads=4, video_dim_head=128, audio_dim=256,
                       audio_heads=4, audio_dim_head=64, frame_h=8, frame_w=12, text_tokens=24)
    torch.manual_seed(0)
    model = CausalModelWeights(cfg, device=DEV, std=0.05)
    gen = torch.Generator(device=DEV).manual_seed(3)
    runner = StreamRunner(model, DEV, graphed=graphed)
    p0 = synthetic_conditioning(cfg, 3, 25, DEV, gen)
    p1 = synthetic_conditioning(cfg, 3, 25, DEV, gen)
    runner.set_prompt(p0.video_ctx, p0.audio_ctx)
    outs, kept = [], []
    for k in range(n_blocks):
        if k == prompt_change_at:
            runner.set_prompt(p1.video_ctx, p1.audio_ctx)
        F_, La, _, _ = block_geometry(k, cfg)
        v = torch.randn(1, F_ * cfg.frame_tokens, cfg.in_channels, device=DEV,
                        generator=gen).to(torch.bfloat16)
        a = torch.randn(1, La, cfg.in_channels, device=DEV, generator=gen).to(torch.bfloat16)
        conds = [synthetic_conditioning(cfg, F_, La, DEV, gen) for _ in range(4)]
        vo, ao = runner.run_block(v, a, conds)
        outs.append((vo.clone(), ao.clone()))
        kept.append([s["block_idx"] for s in runner.cache.segments])
    torch.cuda.synchronize()
    rows = int(runner.cache.layers[0].video_self_k.shape[1])
    captured = runner.graph is not None
    captures = runner.captures
    runner.release()
    return outs, kept, rows, captured, captures


def test_graph_executor_equals_eager():
    eo, ek, erows, ecap, _ = _run(graphed=False)
    go, gk, grows, gcap, gn = _run(graphed=True)
    assert not ecap and gcap
    # block 0 eager; layouts [4], [4, 3], then the steady [4, 3, 3] for blocks 3-6
    assert gn == 3
    assert ek == gk == [[0], [0, 1], [0, 1, 2], [0, 2, 3], [0, 3, 4], [0, 4, 5], [0, 5, 6]]
    assert erows == grows == (4 + 3 + 3) * 96
    for i, ((ev, ea), (gv, ga)) in enumerate(zip(eo, go)):
        assert torch.equal(ev, gv), f"video output of block {i}"
        assert torch.equal(ea, ga), f"audio output of block {i}"
    # the prompt change at block 5 is visible
    assert not torch.equal(go[5][0], go[4][0])


def _small():
    from taomate_b200.model import CausalModelWeights, StreamConfig
    cfg = StreamConfig(layers=2, video_dim=512, video_heads=4, video_dim_head=128, audio_dim=256,
                       audio_heads=4, audio_dim_head=64, frame_h=8, frame_w=12, text_tokens=24)
    torch.manual_seed(0)
    return cfg, CausalModelWeights(cfg, device=DEV, std=0.05)


def _longform(graphed, segments=3, check=None):
    """The runtime's schedule: 5-block windows, no eviction in the first, a
    prompt change + K/V refresh at every later window."""
    from taomate_b200.model import synthetic_conditioning
    from taomate_b200.stream import StreamRunner, block_geometry
    cfg, model = _small()
    gen = torch.Generator(device=DEV).manual_seed(5)
    runner = StreamRunner(model, DEV, graphed=graphed, evict_from_block=5)
    prompts = [synthetic_conditioning(cfg, 3, 25, DEV, gen) for _ in range(segments)]
    zero = {4: synthetic_conditioning(cfg, 4, 26, DEV, gen),
            3: synthetic_conditioning(cfg, 3, 25, DEV, gen)}
    outs, kept = [], []
    for s in range(segments):
        runner.set_prompt(prompts[s].video_ctx, prompts[s].audio_ctx)
        if s > 0:
            before = [lay.video_self_k.entries() for lay in runner.cache.layers]
            conds = {int(g["block_idx"]): zero[block_geometry(int(g["block_idx"]), cfg)[0]]
                     for g in runner.cache.segments}
            runner.refresh(conds)
            after = [lay.video_self_k.entries() for lay in runner.cache.layers]
            assert before == after  # video self-attention K/V kept where they lie
            if check is not None:
                check(runner, model, conds)
        for b in range(5):
            k = s * 5 + b
            F_, La, _, _ = block_geometry(k, cfg)
            v = torch.randn(1, F_ * cfg.frame_tokens, cfg.in_channels, device=DEV,
                            generator=gen).to(torch.bfloat16)
            a = torch.randn(1, La, cfg.in_channels, device=DEV, generator=gen).to(torch.bfloat16)
            conds4 = [synthetic_conditioning(cfg, F_, La, DEV, gen) for _ in range(4)]
            vo, ao = runner.run_block(v, a, conds4)
            outs.append((vo.clone(), ao.clone()))
            kept.append([g["block_idx"] for g in runner.cache.segments])
        runner.end_segment()
    torch.cuda.synchronize()
    captured = runner.graph is not None
    captures = runner.captures
    runner.release()
    return outs, kept, captured, captures


def _check_sink_rebuilt(runner, model, conds):
    """The sink block's rebuilt audio K (layer 0) equals a sigma = 0
    kv_cache_only forward of that block alone under the new prompt, which is
    what the reference's refresh computes for its first retained block."""
    from taomate_b200.kv_cache import last_chunk
    from taomate_b200.model import arena_cache, model_forward
    cfg = model.cfg
    v, a = runner.latents[0]
    pe, off = runner._pe(0)
    empty = arena_cache(cfg, 4 * cfg.frame_tokens, 26, device=DEV)
    with torch.no_grad():
        _, _, new = model_forward(model, v, a, runner._cond(conds[0], pe), empty,
                                  kv_cache_only=True)
    k_ref, _ = last_chunk(new.layers[0].audio_self_k)
    k_got = runner.cache.layers[0].audio_self_k.materialize()[:, :26]
    assert torch.equal(k_got, k_ref)


def test_longform_refresh_graph_equals_eager():
    eo, ek, ecap, _ = _longform(graphed=False, check=_check_sink_rebuilt)
    go, gk, gcap, gn = _longform(graphed=True, check=_check_sink_rebuilt)
    assert not ecap and gcap
    # window 0: blocks 1-4 ([4], [4,3], [4,3,3], [4,3,3,3]); the first refresh adds the
    # sink's empty-cache layout and replays blocks 1-2's; every later block is [4,3,3]
    assert gn == 5
    # window 0 keeps every block; the window end and every later block evict
    assert ek == gk
    assert ek[4] == [0, 1, 2, 3, 4] and ek[5] == [0, 4, 5] and ek[14] == [0, 13, 14]
    for i, ((ev, ea), (gv, ga)) in enumerate(zip(eo, go)):
        assert torch.equal(ev, gv), f"video output of block {i}"
        assert torch.equal(ea, ga), f"audio output of block {i}"


def test_reset_stream_replays_captured_layouts():
    """A second stream on the same runner (``reset``: same arenas, empty
    cache) replays the graphs the first stream captured from its first block
    on, captures nothing, and gives the first stream's bits for the same
    inputs."""
    from taomate_b200.model import synthetic_conditioning
    from taomate_b200.stream import StreamRunner, block_geometry
    cfg, model = _small()
    runner = StreamRunner(model, DEV, graphed=True, evict_from_block=5)

    def stream():
        gen = torch.Generator(device=DEV).manual_seed(8)
        prompts = [synthetic_conditioning(cfg, 3, 25, DEV, gen) for _ in range(2)]
        zero = {4: synthetic_conditioning(cfg, 4, 26, DEV, gen),
                3: synthetic_conditioning(cfg, 3, 25, DEV, gen)}
        outs = []
        for s in range(2):
            runner.set_prompt(prompts[s].video_ctx, prompts[s].audio_ctx)
            if s > 0:
                runner.refresh({int(g["block_idx"]): zero[block_geometry(int(g["block_idx"]),
                                                                         cfg)[0]]
                                for g in runner.cache.segments})
            for b in range(5 if s == 0 else 2):
                F_, La, _, _ = block_geometry(s * 5 + b, cfg)
                v = torch.randn(1, F_ * cfg.frame_tokens, cfg.in_channels, device=DEV,
                                generator=gen).to(torch.bfloat16)
                a = torch.randn(1, La, cfg.in_channels, device=DEV,
                                generator=gen).to(torch.bfloat16)
                conds = [synthetic_conditioning(cfg, F_, La, DEV, gen) for _ in range(4)]
                outs.append(tuple(t.clone() for t in runner.run_block(v, a, conds)))
            runner.end_segment()
        torch.cuda.synchronize()
        return outs

    first = stream()
    n = runner.captures
    assert n == 5
    runner.reset()
    second = stream()
    assert runner.captures == n
    for i, ((v1, a1), (v2, a2)) in enumerate(zip(first, second)):
        assert torch.equal(v1, v2), f"video output of block {i}"
        assert torch.equal(a1, a2), f"audio output of block {i}"
    runner.release()
