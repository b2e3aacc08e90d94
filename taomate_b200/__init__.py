"""taomate_b200: B200 (sm_100a) kernels for TaoMate's causal-LTX streaming
attention step, behind the reference's Python call signatures.

Modules mirror the reference's layout for this path:
  rope       -> ltx_causal/rope/causal_rope.py
  attention  -> ltx_causal/transformer/kv_cache.py (attention_with_cache)
                ltx_causal/attention/flex_attention_utils.py (standard_attention_forward)
  block      -> ltx_causal/transformer/kv_cache.py (block_forward_with_cache)
  kv_cache   -> LayerKVCache / KVCache / _cat_cache, plus the slot arena
  cache      -> taomate/inference/cache.py (segments, retain_streaming_context)
  parallel   -> taomate/runtime_support/parallel (Ulysses SP)
  install    -> rebinds the reference's hot-path names to these (the drop-in)
The compute runs in ``lib/libtaomate_b200.so`` (C ABI: include/taomate_b200.h).
"""

from .rope import CausalRopeType, apply_split_rotary_emb, causal_precompute_freqs_cis
from .attention import (_cross_modal_pair_attention_with_cache, attention_with_cache,
                        cross_modal_pair_attention_with_cache, flash_attention,
                        fuse_kv_weights, fuse_qkv_weights, key_padding_runs,
                        standard_attention_forward,
                        text_cross_attention_with_kv_cache)
from .kv_cache import (ArenaKV, ArenaSpec, KVArena, KVCache, LayerKVCache, _cat_cache,
                       cat_cache_pair, init_arena_cache)
from .cache import (attach_segments, cache_segments, retain_streaming_context, retain_window)
from . import block
from .block import BlockWeights, block_forward_with_cache, fuse_block_weights
from .install import install, uninstall

__all__ = [
    "CausalRopeType", "apply_split_rotary_emb", "causal_precompute_freqs_cis",
    "attention_with_cache", "flash_attention", "standard_attention_forward",
    "text_cross_attention_with_kv_cache", "key_padding_runs", "fuse_qkv_weights",
    "fuse_kv_weights",
    "cross_modal_pair_attention_with_cache", "_cross_modal_pair_attention_with_cache",
    "ArenaKV", "ArenaSpec", "KVArena", "KVCache", "LayerKVCache", "_cat_cache",
    "cat_cache_pair", "init_arena_cache",
    "attach_segments", "cache_segments", "retain_streaming_context", "retain_window",
    "block", "BlockWeights", "block_forward_with_cache", "fuse_block_weights",
    "install", "uninstall",
]
