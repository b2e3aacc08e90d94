"""``taomate_b200.install()`` against the reference's own modules (CPU).

Imports the TaoMate reference from the tree named by ``TAOMATE_REFERENCE``
(skipped when it is unset or absent), installs, and checks that every call
site of the drop-in boundary resolves to this library's function: the names
the reference bound at import (kv_cache.py:48-61, causal_attention.py:20-39,
taomate/inference/model.py:8, runtime.py:16-19), the block that
``CausalAVTransformerBlock.forward`` imports lazily (causal_block.py:530),
and the SP mesh queries, which then share this library's mesh.  Then
``uninstall()`` restores every original.
"""

import importlib
import os
import sys

import pytest

REF = os.environ.get("TAOMATE_REFERENCE")
pytestmark = pytest.mark.skipif(not REF or not os.path.isdir(REF),
                                reason="TAOMATE_REFERENCE does not name the reference tree")

MODULES = ("ltx_causal.transformer.kv_cache", "ltx_causal.attention.causal_attention",
           "ltx_causal.transformer.causal_block", "ltx_causal.transformer.causal_model",
           "taomate.inference.cache", "taomate.inference.model", "taomate.inference.runtime",
           "taomate.runtime_support.parallel")


def test_install_rebinds_every_call_site():
    if REF not in sys.path:
        sys.path.insert(0, REF)
    mods = {m: importlib.import_module(m) for m in MODULES}
    import taomate_b200 as tm
    from taomate_b200 import parallel as P
    kvc, ca = mods["ltx_causal.transformer.kv_cache"], mods["ltx_causal.attention.causal_attention"]
    cm, sp = mods["ltx_causal.transformer.causal_model"], mods["taomate.runtime_support.parallel"]
    orig_awc = kvc.attention_with_cache
    report = tm.install()
    try:
        assert all(report.values()), report
        # attention and the block (callers: kv_cache.py:2205-2590, causal_block.py:530)
        assert kvc.attention_with_cache is tm.attention_with_cache
        assert kvc._cross_modal_pair_attention_with_cache is tm._cross_modal_pair_attention_with_cache
        assert kvc._cat_cache is tm._cat_cache
        ns = {}
        exec("from ltx_causal.transformer.kv_cache import block_forward_with_cache", ns)
        assert ns["block_forward_with_cache"] is tm.block_forward_with_cache
        for m in (kvc, ca):
            assert m.standard_attention_forward is tm.standard_attention_forward
        # RoPE (causal_attention.py:326 via _apply_rope; kv_cache.py:592-647)
        assert ca.apply_split_rotary_emb is tm.apply_split_rotary_emb
        for m in (kvc, cm):
            assert m.causal_precompute_freqs_cis is tm.causal_precompute_freqs_cis
        # eviction (model.py:241, runtime.py:634)
        for m in ("taomate.inference.cache", "taomate.inference.model", "taomate.inference.runtime"):
            assert mods[m].retain_streaming_context is tm.retain_streaming_context
        # sequence parallelism: one mesh for both
        for m in (kvc, ca, cm):
            assert m._is_sp_enabled is P.is_sp_enabled
            assert m._get_sp_world_size is P.get_sp_world_size
        for name in ("_seq_all_to_all_head", "_seq_all_to_all_head_many", "_head_all_to_all_seq",
                     "_split_sequence", "_gather_sequence"):
            assert getattr(kvc, name) is getattr(P, name.lstrip("_")), name
        assert sp.init_sp_mesh is P.init_sp_mesh and sp.is_sp_enabled is P.is_sp_enabled
        assert sp.is_sp_enabled() is False  # this library's mesh is not set
    finally:
        tm.uninstall()
    assert kvc.attention_with_cache is orig_awc
    assert kvc._is_sp_enabled is not P.is_sp_enabled
