"""CUDA-graph replay of a streaming forward (taomate_b200.graphs) on one GPU.

Two identical streaming runs over a slot-arena cache: one issues every forward
eagerly, the other captures the forward once at the full window and replays it
for the following blocks, rewriting the attention kernels' device tile table as
the cache rows move between arena slots.  Outputs and committed K/V must match
the eager run (same kernels, same tiles), and a layout with a different tile
count must be refused instead of replayed.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0) if torch.cuda.is_available() else None


def _rel(a, b):
    a, b = a.double(), b.double()
    return float(torch.linalg.norm(a - b) / torch.linalg.norm(b))


def test_graph_replay_matches_eager_over_blocks():
    import taomate_b200 as tm
    from taomate_b200.attention import AttentionWeights
    from taomate_b200.cache import retain_window
    from taomate_b200.graphs import AttentionGraph, attention_spans
    from taomate_b200.kv_cache import ArenaSpec, KVCache, LayerKVCache, init_arena_cache

    torch.cuda.set_device(DEV)
    L, H, D, frames, fh, fw = 2, 4, 128, 2, 8, 12
    hidden, Lq = H * D, frames * fh * fw
    anchor, window = fh * fw, 2 * frames * fh * fw
    torch.manual_seed(0)
    attn = [AttentionWeights(hidden, H, D, device=DEV) for _ in range(L)]
    g = torch.Generator(device=DEV).manual_seed(3)
    xs = [torch.randn(1, Lq, hidden, device=DEV, generator=g).to(torch.bfloat16)
          for _ in range(L)]
    grid = torch.tensor([[frames, fh, fw]])

    def pe_of(block):
        return tm.causal_precompute_freqs_cis(grid, hidden, start_frame=block * frames,
                                              device=DEV, dtype=torch.bfloat16,
                                              num_attention_heads=H)

    def fresh():
        return init_arena_cache(L, {"video_self": ArenaSpec(6, Lq, H, D)}, device=DEV)

    def commit(cache, kv):
        layers = []
        for lay, (nk, nv) in zip(cache.layers, kv):
            k2, v2 = tm.cat_cache_pair(lay.video_self_k, lay.video_self_v, nk, nv)
            k2.entries()
            layers.append(LayerKVCache(video_self_k=k2, video_self_v=v2))
        return retain_window(KVCache(layers=layers), anchor, window)

    def eager_block(cache, block):
        pe = pe_of(block)
        kv, out = [], None
        for li in range(L):
            lay = cache.layers[li]
            out, nk, nv = tm.attention_with_cache(attn[li], xs[li], None, pe, None,
                                                  lay.video_self_k, lay.video_self_v)
            kv.append((nk, nv))
        return out, commit(cache, kv), kv

    with torch.no_grad():
        ce, cg = fresh(), fresh()
        for b in range(3):  # fill the window in both runs
            _, ce, _ = eager_block(ce, b)
            _, cg, _ = eager_block(cg, b)
        torch.cuda.synchronize()

        pe_static = tuple(t.contiguous() for t in pe_of(3))
        for lay in cg.layers:
            attention_spans(lay.video_self_k, lay.video_self_v, Lq)
        graph = AttentionGraph(DEV, max_sites=L)
        cap = {"cache": cg}

        def forward():
            kv, out = [], None
            for li in range(L):
                lay = cap["cache"].layers[li]
                out, nk, nv = tm.attention_with_cache(attn[li], xs[li], None, pe_static, None,
                                                      lay.video_self_k, lay.video_self_v)
                kv.append((nk, nv))
            return out, kv

        g_out, g_kv = graph.capture(forward)
        for b in range(3, 8):
            out_e, ce, kv_e = eager_block(ce, b)
            c, s = pe_of(b)
            pe_static[0].copy_(c)
            pe_static[1].copy_(s)
            spans = [attention_spans(l.video_self_k, l.video_self_v, Lq) for l in cg.layers]
            graph.replay(spans)
            torch.cuda.synchronize()
            assert _rel(g_out, out_e) < 1e-3, f"block {b}"
            for (gk, gv), (ek, ev) in zip(g_kv, kv_e):
                assert _rel(gk, ek) < 1e-3 and _rel(gv, ev) < 1e-3
            cg = commit(cg, g_kv)
        # a layout with another tile count is refused
        short = [s[:-1] + [(1, 0, Lq - 64)] for s in spans]
        with pytest.raises(ValueError, match="recapture"):
            graph.replay(short)
        graph.reset()
