"""fuse_qkv_weights on the host: the three projection parameters become row
blocks of one buffer with unchanged values, in-place loads land in the fused
buffer, and replacing a parameter ends the fusion for that module."""

import torch

from taomate_b200.attention import AttentionWeights, _fused_qkv, fuse_qkv_weights


def _module():
    torch.manual_seed(0)
    return AttentionWeights(64, 4, 16, device="cpu", dtype=torch.float32)


def test_fusion_keeps_values_and_shares_storage():
    m = _module()
    before = [l.weight.detach().clone() for l in (m.to_q, m.to_k, m.to_v)]
    bias = [l.bias.detach().clone() for l in (m.to_q, m.to_k, m.to_v)]
    assert fuse_qkv_weights(m)
    W, B = _fused_qkv(m)
    assert W.shape == (192, 64) and B.shape == (192,)
    for i, l in enumerate((m.to_q, m.to_k, m.to_v)):
        assert torch.equal(l.weight, before[i]) and torch.equal(l.bias, bias[i])
        assert torch.equal(W[64 * i:64 * (i + 1)], before[i])
    x = torch.randn(2, 5, 64)
    ref = [torch.nn.functional.linear(x, w, b) for w, b in zip(before, bias)]
    got = torch.nn.functional.linear(x, W, B).split(64, dim=-1)
    for r, g in zip(ref, got):
        torch.testing.assert_close(g, r)
    # a weight loaded in place lands in the fused buffer
    with torch.no_grad():
        m.to_k.weight.copy_(torch.ones(64, 64))
    assert torch.equal(W[64:128], torch.ones(64, 64))
    assert _fused_qkv(m) is not None


def test_replaced_parameter_ends_fusion():
    m = _module()
    assert fuse_qkv_weights(m)
    m.to_v.weight = torch.nn.Parameter(torch.zeros(64, 64))
    assert _fused_qkv(m) is None


def test_mismatched_linears_are_left_alone():
    m = _module()
    m.to_k = torch.nn.Linear(64, 64, bias=False)
    w = m.to_q.weight.data_ptr()
    assert not fuse_qkv_weights(m)
    assert m.to_q.weight.data_ptr() == w and _fused_qkv(m) is None
