"""Attention over keys split between GPUs: partial export + merge.

Under sequence parallelism the V2A attention (25 audio queries over the video
keys) keeps every rank's video keys where they were made: each rank attends
over its own keys and exports, per key range, the normalised fp32 output and
its (max, sum) (``flash_attention(parts=)``, tm_attention_fwd_ext); the parts
of all ranks are gathered and merged (``combine_partials``,
tm_attention_combine).  Here the ranks are emulated on one GPU: the keys of
one attention are divided into groups (cache spans and new rows mixed, groups
of unequal size), each group's call writes its part at its own offset of one
buffer, and the merge must give the softmax over all keys:

* against an fp32 reference, within the bf16 output rounding (the bar of the
  kernel's other tests), with and without the per-head gate;
* a group that holds no keys ((max, sum) = (-inf, 0)) changes no bit;
* two merges of the same bytes give the same bits (every rank merges the same
  gathered bytes, so the replicated audio stream stays identical);
* the call checks its key-range count and buffer size.
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


def _rel_l2(a, b):
    a, b = a.double(), b.double()
    return float(torch.linalg.norm(a - b) / torch.linalg.norm(b))


def _reference(q, k_all, v_all, glog=None):
    o = torch.nn.functional.scaled_dot_product_attention(
        q.transpose(1, 2).float(), k_all.transpose(1, 2).float(),
        v_all.transpose(1, 2).float()).transpose(1, 2)
    if glog is not None:
        o = o * (2.0 * torch.sigmoid(glog.float())).unsqueeze(-1)
    return o


def _parts(q, ck, cv, nk, nv, groups, splits, empty=()):
    """One buffer with every group's part at g * stride; ``groups`` are
    (cache rows [start, end), new rows [start, end)) per group."""
    from taomate_b200.attention import flash_attention, partial_bytes
    B, Lq, H, D = (int(v) for v in q.shape)
    pb = partial_bytes(B, Lq, H, D, splits)
    buf = torch.full((len(groups) * pb,), 0x7F, dtype=torch.uint8, device=DEV)
    for g, ((c0, c1), (n0, n1)) in enumerate(groups):
        own = buf[g * pb:(g + 1) * pb]
        if g in empty:
            rows = splits * B * Lq * H
            off = (rows * D * 4 + 255) // 256 * 256
            own.zero_()
            own[off:off + rows * 8].view(torch.float32).view(rows, 2)[:, 0] = float("-inf")
            continue
        spans = [(c0, c1 - c0)] if c1 > c0 else []
        k_new = nk[:, n0:n1].contiguous() if n1 > n0 else None
        v_new = nv[:, n0:n1].contiguous() if n1 > n0 else None
        flash_attention(q, ck if spans else None, cv if spans else None, spans, k_new, v_new,
                        n1 - n0, parts=own, part_splits=splits)
    return buf, pb


def _inputs(seed, Lq, H, D, Lc, Ln):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g).to(DEV, torch.bfloat16)
    return r(1, Lq, H, D), r(1, Lc, H, D), r(1, Lc, H, D), r(1, Ln, H, D), r(1, Ln, H, D)


CASES = [
    # (Lq, H, D, cached, new, groups, splits): V2A shapes (25 audio queries,
    # 32 heads of 64) with 4 unequal groups; 3 query tiles of 128-dim heads
    (25, 32, 64, 300, 160, [((0, 130), (0, 0)), ((130, 300), (0, 40)), ((0, 0), (40, 100)),
                            ((0, 0), (100, 160))], 1),
    (25, 32, 64, 600, 0, [((0, 300), (0, 0)), ((300, 600), (0, 0))], 2),
    (300, 4, 128, 256, 200, [((0, 256), (0, 72)), ((0, 0), (72, 200))], 1),
]


@pytest.mark.parametrize("Lq,H,D,Lc,Ln,groups,splits", CASES,
                         ids=["v2a-4groups", "v2a-2groups-split2", "d128-3qtiles"])
def test_merge_equals_attention_over_all_keys(Lq, H, D, Lc, Ln, groups, splits):
    from taomate_b200.attention import combine_partials, flash_attention
    q, ck, cv, nk, nv = _inputs(Lq + Lc, Lq, H, D, Lc, Ln)
    buf, pb = _parts(q, ck, cv, nk, nv, groups, splits)
    out = combine_partials(buf, len(groups), pb, splits, 1, Lq, H, D)
    # the keys of every group, in group order (softmax does not depend on the order)
    ks, vs = [], []
    for (c0, c1), (n0, n1) in groups:
        ks += [ck[:, c0:c1], nk[:, n0:n1]]
        vs += [cv[:, c0:c1], nv[:, n0:n1]]
    k_all, v_all = torch.cat(ks, 1), torch.cat(vs, 1)
    ref = _reference(q, k_all, v_all)
    assert _rel_l2(out, ref) < 4e-3
    # the one-call path over the same keys (one GPU): both round fp32 once to bf16
    one = flash_attention(q, None, None, (), k_all.contiguous(), v_all.contiguous(),
                          int(k_all.shape[1]))
    assert _rel_l2(out, one) < 4e-3
    # the same bytes merged again: the same bits
    assert torch.equal(out, combine_partials(buf, len(groups), pb, splits, 1, Lq, H, D))
    # the per-head gate in the merge
    glog = torch.randn(1, Lq, H, generator=torch.Generator().manual_seed(5)).to(DEV,
                                                                              torch.bfloat16)
    gated = combine_partials(buf, len(groups), pb, splits, 1, Lq, H, D, gate_logits=glog)
    assert _rel_l2(gated, _reference(q, k_all, v_all, glog)) < 4e-3


def test_group_without_keys_changes_nothing():
    from taomate_b200.attention import combine_partials
    Lq, H, D = 25, 32, 64
    q, ck, cv, nk, nv = _inputs(9, Lq, H, D, 200, 100)
    groups = [((0, 200), (0, 0)), ((0, 0), (0, 0)), ((0, 0), (0, 100))]
    buf, pb = _parts(q, ck, cv, nk, nv, groups, 1, empty=(1,))
    out3 = combine_partials(buf, 3, pb, 1, 1, Lq, H, D)
    two = torch.cat([buf[:pb], buf[2 * pb:3 * pb]])
    out2 = combine_partials(two, 2, pb, 1, 1, Lq, H, D)
    assert torch.equal(out3, out2)
    assert torch.isfinite(out3.float()).all()


def test_export_checks_its_arguments():
    from taomate_b200 import _lib
    from taomate_b200.attention import flash_attention, partial_bytes
    Lq, H, D = 25, 32, 64
    q, ck, cv, nk, nv = _inputs(3, Lq, H, D, 64, 64)
    small = torch.empty(partial_bytes(1, Lq, H, D, 2) - 16, dtype=torch.uint8, device=DEV)
    with pytest.raises(ValueError):
        flash_attention(q, None, None, (), nk, nv, 64, parts=small, part_splits=2)
    # 64 keys are one key tile: two key ranges cannot both hold keys
    ok = torch.empty(partial_bytes(1, Lq, H, D, 2), dtype=torch.uint8, device=DEV)
    with pytest.raises(ValueError, match="key ranges"):
        flash_attention(q, None, None, (), nk, nv, 64, parts=ok, part_splits=2)
    assert _lib.device_error() == 0
