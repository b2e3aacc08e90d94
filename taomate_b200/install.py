"""Drop-in installation into a running TaoMate process.

The reference binds most hot-path functions by name when its modules import:
``kv_cache.py`` takes ``_is_sp_enabled``, ``_seq_all_to_all_head_many``,
``_head_all_to_all_seq`` ... from ``taomate.runtime_support.parallel``
(kv_cache.py:48-61), ``causal_attention.py`` takes ``apply_split_rotary_emb``
and its own ``_seq_*`` aliases (causal_attention.py:20-39), ``model.py`` and
``runtime.py`` take ``retain_streaming_context`` (taomate/inference/model.py:8,
runtime.py:16-19).  Replacing the defining module's attribute alone would leave
those copies pointing at the old functions.

``install()`` therefore rebinds, in every loaded module of the reference
(``ltx_causal.*``, ``taomate.*``), every attribute that *is* one of the
replaced reference functions (identity, whatever alias it was imported under),
to this library's function of the same contract.  The SP mesh functions are
among them, so the reference's ``init_sp_mesh`` / ``is_sp_enabled`` and this
library's share one mesh: after ``install()`` a model whose code asks the
reference whether sequence parallelism is on gets this library's answer.

Call it after the reference modules are imported and before the model runs;
``uninstall()`` restores the originals.
"""

from __future__ import annotations

import importlib
import sys
from typing import Dict, List, Tuple

from . import attention as _attention
from . import block as _block
from . import cache as _cache
from . import kv_cache as _kv
from . import parallel as _parallel
from . import rope as _rope

# (reference module, function, replacement): the drop-in boundary of this path
REPLACEMENTS: Tuple[Tuple[str, str, object], ...] = (
    ("ltx_causal.transformer.kv_cache", "attention_with_cache", _attention.attention_with_cache),
    ("ltx_causal.transformer.kv_cache", "_cross_modal_pair_attention_with_cache",
     _attention._cross_modal_pair_attention_with_cache),
    ("ltx_causal.transformer.kv_cache", "_cat_cache", _kv._cat_cache),
    ("ltx_causal.transformer.kv_cache", "block_forward_with_cache",
     _block.block_forward_with_cache),
    ("ltx_causal.attention.flex_attention_utils", "standard_attention_forward",
     _attention.standard_attention_forward),
    ("ltx_causal.rope.causal_rope", "apply_split_rotary_emb", _rope.apply_split_rotary_emb),
    ("ltx_causal.rope.causal_rope", "causal_precompute_freqs_cis",
     _rope.causal_precompute_freqs_cis),
    ("taomate.inference.cache", "retain_streaming_context", _cache.retain_streaming_context),
    ("taomate.runtime_support.parallel.mesh", "init_sp_mesh", _parallel.init_sp_mesh),
    ("taomate.runtime_support.parallel.mesh", "get_device_mesh", _parallel.get_device_mesh),
    ("taomate.runtime_support.parallel.mesh", "is_sp_enabled", _parallel.is_sp_enabled),
    ("taomate.runtime_support.parallel.mesh", "get_sp_group", _parallel.get_sp_group),
    ("taomate.runtime_support.parallel.mesh", "get_sp_world_size", _parallel.get_sp_world_size),
    ("taomate.runtime_support.parallel.mesh", "get_sp_rank", _parallel.get_sp_rank),
    ("taomate.runtime_support.parallel.mesh", "get_dp_group", _parallel.get_dp_group),
    ("taomate.runtime_support.parallel.mesh", "get_dp_world_size", _parallel.get_dp_world_size),
    ("taomate.runtime_support.parallel.mesh", "get_dp_rank", _parallel.get_dp_rank),
    ("taomate.runtime_support.parallel.all_to_all", "seq_all_to_all_head",
     _parallel.seq_all_to_all_head),
    ("taomate.runtime_support.parallel.all_to_all", "seq_all_to_all_head_many",
     _parallel.seq_all_to_all_head_many),
    ("taomate.runtime_support.parallel.all_to_all", "seq_all_to_all_head_async",
     _parallel.seq_all_to_all_head_async),
    ("taomate.runtime_support.parallel.all_to_all", "seq_all_to_all_head_many_async",
     _parallel.seq_all_to_all_head_many_async),
    ("taomate.runtime_support.parallel.all_to_all", "head_all_to_all_seq",
     _parallel.head_all_to_all_seq),
    ("taomate.runtime_support.parallel.all_to_all", "head_all_to_all_seq_async",
     _parallel.head_all_to_all_seq_async),
    ("taomate.runtime_support.parallel.sp_utils", "split_sequence", _parallel.split_sequence),
    ("taomate.runtime_support.parallel.sp_utils", "gather_sequence", _parallel.gather_sequence),
    ("taomate.runtime_support.parallel.sp_utils", "pad_sequence_to_multiple",
     _parallel.pad_sequence_to_multiple),
    ("taomate.runtime_support.parallel.sp_utils", "unpad_sequence", _parallel.unpad_sequence),
)

_SCOPES = ("ltx_causal", "taomate")
_SAVED: List[Tuple[object, str, object]] = []


def _in_scope(name: str) -> bool:
    return any(name == s or name.startswith(s + ".") for s in _SCOPES)


def install() -> Dict[str, List[str]]:
    """Rebind the reference's hot-path functions to this library's in every
    loaded reference module; returns ``{"module.function": [rebound
    "module.attribute", ...]}``.  Raises ``ImportError`` if a defining module
    of the reference cannot be imported."""
    originals = []
    for modname, fname, repl in REPLACEMENTS:
        mod = importlib.import_module(modname)
        orig = getattr(mod, fname)
        if orig is not repl:
            originals.append((f"{modname}.{fname}", orig, repl))
    report: Dict[str, List[str]] = {key: [] for key, _, _ in originals}
    by_id = {id(orig): (key, orig, repl) for key, orig, repl in originals}
    for name, mod in list(sys.modules.items()):
        if mod is None or not _in_scope(name):
            continue
        for attr, val in list(vars(mod).items()):
            hit = by_id.get(id(val))
            if hit is None or hit[1] is not val:
                continue
            key, orig, repl = hit
            _SAVED.append((mod, attr, orig))
            setattr(mod, attr, repl)
            report[key].append(f"{name}.{attr}")
    return report


def uninstall() -> None:
    """Put back every attribute ``install()`` rebound."""
    while _SAVED:
        mod, attr, orig = _SAVED.pop()
        setattr(mod, attr, orig)
