"""Host-side cache logic without a GPU: slot reference counting, slicing of
arena views (no data movement), the retention policy and the reference's
error behaviour."""

import pytest
import torch

from taomate_b200 import cache as C
from taomate_b200.kv_cache import ArenaKV, KVArena, KVCache, LayerKVCache, _PairState, arena_pair


def _arena(n_slots=6, slot_rows=8):
    return KVArena(n_slots, slot_rows, 1, 2, 8, dtype=torch.bfloat16, device="meta")


def _pair_with(arena, lens):
    entries = []
    for n in lens:
        slot = arena._take()
        entries.append((slot, slot * arena.slot_rows, n))
    k, v = arena_pair(arena, entries)
    for (slot, _, _) in entries:  # arena_pair took its own references
        arena._ref(slot, -1)
    return k, v


def test_slot_refcounts_follow_views():
    a = _arena()
    k, v = _pair_with(a, [8, 6, 6])
    assert a.refs[:3] == [1, 1, 1] and a.free_slots() == [3, 4, 5]
    st = k._state.sliced([(0, 8), (14, 20)])  # keep segments 0 and 2
    k2, v2 = ArenaKV(a, "k", st), ArenaKV(a, "v", st)
    assert k2.shape == (1, 14, 2, 8)
    assert [e[0] for e in k2._state.entries] == [0, 2]
    assert a.refs[:3] == [2, 1, 2]
    del k, v
    assert a.refs[:3] == [1, 0, 1]
    assert a.free_slots() == [1, 3, 4, 5]
    del k2, v2, st
    assert a.free_slots() == [0, 1, 2, 3, 4, 5]


def test_slice_moves_no_rows_and_splits_entries():
    a = _arena(slot_rows=10)
    k, _ = _pair_with(a, [10, 9, 9])
    st = k._state.sliced([(2, 5), (12, 25)])
    assert st.entries == [(0, 2, 3), (1, 12, 7), (2, 20, 6)]
    with pytest.raises(IndexError):
        k._state.sliced([(20, 40)])


def test_retain_streaming_context_policy_on_views():
    a = _arena(n_slots=8, slot_rows=24)
    vk, vv = _pair_with(a, [24, 18, 18, 18, 18])
    layer = LayerKVCache(video_self_k=vk, video_self_v=vv)
    segs = [{"block_idx": i, "video_tokens": n, "audio_tokens": 0}
            for i, n in enumerate([24, 18, 18, 18, 18])]
    cache = C.attach_segments(KVCache(layers=[layer]), segs)
    out = C.retain_streaming_context(cache)
    assert [s["block_idx"] for s in C.cache_segments(out)] == [0, 3, 4]
    L = out.layers[0]
    assert L.video_self_k.shape[1] == 24 + 18 + 18
    assert [e[0] for e in L.video_self_k._state.entries] == [0, 3, 4]
    assert L.video_self_k._state is L.video_self_v._state
    # already minimal: same object back, like the reference
    assert C.retain_streaming_context(out) is out


def test_retain_without_segments_raises_like_reference():
    with pytest.raises(RuntimeError, match="block metadata"):
        C.retain_streaming_context(KVCache(layers=[]))


def test_segment_offsets_match_oracle():
    from oracle import ltx_oracle as O
    segs = [{"block_idx": 0, "video_tokens": 1536, "audio_tokens": 26},
            {"block_idx": 3, "video_tokens": 1152, "audio_tokens": 25},
            {"block_idx": 4, "video_tokens": 1152, "audio_tokens": 25}]
    assert C._segment_offsets(segs) == O.segment_offsets(segs)
    for n in range(1, 8):
        s = [{"block_idx": i, "video_tokens": 1, "audio_tokens": 1} for i in range(n)]
        assert C.retain_indices(s) == O.retain_indices(s)


def test_arena_full_raises():
    a = _arena(n_slots=2)
    _pair_with(a, [8, 8])  # views dropped immediately -> slots free again
    k, v = _pair_with(a, [8, 8])
    with pytest.raises(RuntimeError, match="arena full"):
        a._take()
    del k, v


def test_cat_cache_requires_k_before_v():
    from taomate_b200.kv_cache import _cat_cache
    a = _arena()
    k, v = _pair_with(a, [8])
    chunk = torch.zeros(1, 4, 2, 8, dtype=torch.bfloat16, device="meta")
    with pytest.raises(RuntimeError, match="K field"):
        _cat_cache(v, chunk)
    k2 = _cat_cache(k, chunk)
    v2 = _cat_cache(v, chunk)
    assert k2._state is v2._state and k2.shape == (1, 12, 2, 8)
    assert k.shape == (1, 8, 2, 8)  # the old view is unchanged


def test_key_padding_runs_from_reference_masks():
    """Key-padding masks in the forms the reference builds become runs of
    visible keys (host logic; CPU tensors)."""
    from taomate_b200.attention import key_padding_runs
    m01 = torch.tensor([[1, 1, 1, 0, 0], [1, 1, 1, 1, 1]])
    assert key_padding_runs(m01, 2, 5) == [[(0, 3)], [(0, 5)]]
    # _prepare_attention_mask: (mask - 1) * finfo.max, shape [B, 1, 1, Lk]
    add = ((m01 - 1).to(torch.bfloat16) * torch.finfo(torch.bfloat16).max).reshape(2, 1, -1, 5)
    assert key_padding_runs(add, 2, 5) == [[(0, 3)], [(0, 5)]]
    holes = torch.tensor([[True, False, True, True, False, True]])
    assert key_padding_runs(holes, 3, 6) == [[(0, 1), (2, 2), (5, 1)]] * 3  # batch broadcast
    assert key_padding_runs(torch.zeros(1, 4, dtype=torch.bool), 1, 4) == [[]]
    with pytest.raises(NotImplementedError):
        key_padding_runs(torch.tensor([[[0.0, -1.5, 0.0]]]), 1, 3)  # a real bias
    per_query = torch.tensor([[[[1, 0], [0, 1]]]], dtype=torch.bool)
    with pytest.raises(NotImplementedError):
        key_padding_runs(per_query, 1, 2)


def test_compute_av_blocks_matches_oracle():
    from oracle import ltx_oracle as O
    for total in (4, 5, 7, 16, 18, 31):
        for first in (0, 4):
            if first and total < first:
                continue
            assert C.compute_av_blocks(total, 3, first) == [tuple(b) for b in
                                                           O.compute_av_blocks(total, 3, first)]


def test_refresh_blocks_select_sink_and_newest_warm_blocks():
    # retained: sink block 0 plus the two newest warm blocks, prefix of 16 frames
    segs = [{"block_idx": 0, "video_tokens": 4, "audio_tokens": 26},
            {"block_idx": 7, "video_tokens": 3, "audio_tokens": 25},
            {"block_idx": 8, "video_tokens": 3, "audio_tokens": 25}]
    picked = C.refresh_blocks(segs, prefix_frames=16, next_frames=3)
    blocks = C.compute_av_blocks(19, 3, 4)
    prefix = [b for b in blocks if b[2] <= 16]
    assert picked == [prefix[0], prefix[-2], prefix[-1]]
    # no sink retained: the newest blocks only
    assert C.refresh_blocks(segs[1:], 16, 3) == prefix[-2:]
    with pytest.raises(ValueError, match="not have enough"):
        C.refresh_blocks(segs + [dict(block_idx=9, video_tokens=3, audio_tokens=25)] * 9, 7, 3)
    with pytest.raises(RuntimeError):
        C.refresh_blocks([], 16, 3)


def test_replace_modal_fields_keeps_video_self():
    segs = [{"block_idx": 0, "video_tokens": 8, "audio_tokens": 0}]
    a = _arena()
    vk, vv = _pair_with(a, [8])
    old = LayerKVCache(video_self_k=vk, video_self_v=vv, audio_self_k=torch.zeros(1),
                       audio_self_v=torch.zeros(1))
    new = LayerKVCache(video_self_k=torch.ones(2), video_self_v=torch.ones(2),
                       audio_self_k=torch.ones(3), audio_self_v=torch.ones(3),
                       a2v_k=torch.ones(4), a2v_v=torch.ones(4))
    cache = C.attach_segments(KVCache(layers=[old]), segs)
    out = C.replace_modal_fields(cache, KVCache(layers=[new]))
    lay = out.layers[0]
    assert lay.video_self_k is vk and lay.video_self_v is vv
    assert lay.audio_self_k is new.audio_self_k and lay.a2v_v is new.a2v_v
    assert C.cache_segments(out) == segs
    with pytest.raises(RuntimeError):
        C.replace_modal_fields(cache, KVCache(layers=[]))


def test_retention_slices_a_per_rank_v2a_cache_by_its_share():
    """Under sequence parallelism each rank's V2A cache holds its own 1/G of
    every segment's video tokens (the split-key V2A); retention keeps the
    same segments of it as of the full-sequence fields."""
    a = _arena(n_slots=8, slot_rows=24)
    b = _arena(n_slots=8, slot_rows=12)
    lens = [24, 18, 18, 18, 18]
    vk, vv = _pair_with(a, lens)
    sk, sv = _pair_with(b, [n // 2 for n in lens])  # G = 2
    layer = LayerKVCache(video_self_k=vk, video_self_v=vv, v2a_k=sk, v2a_v=sv)
    segs = [{"block_idx": i, "video_tokens": n, "audio_tokens": 0} for i, n in enumerate(lens)]
    out = C.retain_streaming_context(C.attach_segments(KVCache(layers=[layer]), segs))
    lay = out.layers[0]
    assert [e[0] for e in lay.video_self_k._state.entries] == [0, 3, 4]
    assert [e[0] for e in lay.v2a_k._state.entries] == [0, 3, 4]
    assert lay.v2a_k.shape[1] == (24 + 18 + 18) // 2 and lay.video_self_k.shape[1] == 60
    # a field whose rows are not a whole share of the tokens is refused
    ck, cv = _pair_with(_arena(n_slots=8, slot_rows=24), [7, 5, 5, 5, 5])
    bad = LayerKVCache(video_self_k=vk, video_self_v=vv, v2a_k=ck, v2a_v=cv)
    with pytest.raises(ValueError):
        C.retain_streaming_context(C.attach_segments(KVCache(layers=[bad]), segs))


def test_stream_block_geometry_follows_compute_av_blocks():
    """The streaming runner's per-block geometry (video frames, audio tokens,
    first video frame, first audio token) is the reference's 4-3-3-3 block
    layout (compute_av_blocks with a first block of 4 frames) for the 181
    latent frames of the 60 s stream."""
    from oracle import ltx_oracle as O
    from taomate_b200.model import StreamConfig
    from taomate_b200.stream import block_geometry
    cfg = StreamConfig(layers=1)
    blocks = O.compute_av_blocks(181, 3, 4)
    assert len(blocks) == 60  # 12 segments x 5 blocks: 4 + 59 x 3 frames
    for k, (b, vs, ve, as_, ae) in enumerate(blocks):
        assert b == k
        assert block_geometry(k, cfg) == (ve - vs, ae - as_, vs, as_)
