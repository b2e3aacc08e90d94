"""CPU tests of the attention work partition (tm_attention_plan): host
arithmetic only, so they run without a GPU (148 SMs assumed when no device
answers, the B200's count).

The cases are the launches of the C4 step and of its sequence-parallel
shards: 1152 query rows are 9 query tiles per head, so at 32 heads pair mode
would need 128 pair CTAs + 32 odd-tile CTAs, 12 more than one wave; the plan
puts the odd tiles of two heads in one CTA instead (144 CTAs).  At 16, 8 and
4 heads per GPU the split CTAs with 1, 2 and 4 key ranges fill one wave; the
V2A call (25 audio queries over 4992 video keys) splits its keys 4 ways.
"""

import pytest

from taomate_b200 import _lib
from taomate_b200.attention import attention_plan

BIG = None  # as much workspace as the plan wants


@pytest.mark.parametrize("B,Lq,H,D,keys,ws,mode,splits,ctas", [
    (1, 1152, 32, 128, 4992, BIG, "pair+cross-head", 1, 144),  # C4 video self-attention
    (1, 1152, 32, 128, 4608, BIG, "pair+cross-head", 1, 144),  # C2
    (1, 1152, 32, 128, 256, BIG, "pair+cross-head", 1, 144),   # video text cross
    (1, 1152, 32, 64, 101, BIG, "pair+cross-head", 1, 144),    # A2V
    (2, 1152, 16, 128, 256, BIG, "pair+cross-head", 1, 144),   # pairs never cross a batch
    (1, 1152, 31, 64, 256, BIG, "pair+cross-head", 1, 140),    # odd heads: last one split
    (1, 1152, 16, 128, 4992, BIG, "split", 1, 144),            # 2 GPUs
    (1, 1152, 8, 128, 4992, BIG, "split", 2, 144),             # 4 GPUs
    (1, 1152, 4, 128, 4992, BIG, "split", 4, 144),             # 8 GPUs
    (1, 1152, 4, 128, 4992, 0, "split", 1, 36),                # no workspace: no key ranges
    (1, 25, 32, 64, 4992, BIG, "split", 4, 128),               # V2A
    (1, 25, 32, 64, 101, BIG, "pair", 1, 32),                  # audio self: one tile per head
    (1, 576, 32, 128, 256, BIG, "pair", 1, 96),                # text cross at 2 GPUs: one wave
])
def test_plan_of_the_step_launches(B, Lq, H, D, keys, ws, mode, splits, ctas):
    plan = attention_plan(B, Lq, H, D, keys, ws)
    assert plan == {"mode": mode, "kv_splits": splits, "ctas": ctas}
    assert plan["ctas"] <= 148  # every step launch fits one wave


@pytest.mark.parametrize("B,Lq,H,D,keys", [
    (1, 1152, 32, 128, 4992), (1, 1152, 4, 128, 4992), (1, 25, 32, 64, 4992),
    (1, 144, 32, 128, 256), (3, 700, 5, 64, 1000)])
def test_workspace_query_agrees_with_plan(B, Lq, H, D, keys):
    """tm_attention_workspace_bytes is non-zero exactly when the plan splits
    the keys (its fp32 partial outputs and (max, sum) per key range)."""
    plan = attention_plan(B, Lq, H, D, keys)
    ws = int(_lib.load().tm_attention_workspace_bytes(B, Lq, H, D, keys))
    if plan["kv_splits"] > 1:
        assert ws >= plan["kv_splits"] * B * Lq * H * (D * 4 + 8)
        # with exactly that workspace the same plan is chosen
        assert attention_plan(B, Lq, H, D, keys, ws) == plan
    else:
        assert ws == 0


def test_plan_rejects_bad_shapes():
    with pytest.raises(NotImplementedError):
        attention_plan(1, 128, 4, 96, 100)
    with pytest.raises(ValueError):
        attention_plan(1, 128, 4, 64, 384 * 64 + 1)  # more keys than the tile table holds
    with pytest.raises(ValueError):
        attention_plan(0, 128, 4, 64, 100)
