"""CPU tests of the C ABI: the library builds, loads, exports every entry
point declared in include/*.h, and rejects bad arguments on the host before
touching a GPU."""

import ctypes
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        with open(h) as fh:
            txt = fh.read()
        names.update(re.findall(r"TM_API\s+[\w\s\*]+?\b(tm_\w+)\s*\(", txt))
    return names


def test_library_exports_every_declared_symbol():
    from taomate_b200 import _lib
    lib = _lib.load()
    decl = declared_symbols()
    assert decl, "no declarations found"
    for name in decl:
        assert hasattr(lib, name), f"{name} declared but not exported"
    assert set(_lib.EXPORTED) == decl
    assert lib.tm_abi_version() == 1


def test_library_is_sm100a_only():
    from taomate_b200 import build
    assert any("compute_100a" in a for a in build.ARCH)


def _status(fn, *args):
    from taomate_b200 import _lib
    return fn(*args)


def test_attention_rejects_before_launch():
    from taomate_b200 import _lib
    lib = _lib.load()
    span = (_lib.KVSpan * 1)()
    span[0].source, span[0].row_start, span[0].rows = 1, 0, 8
    # head dim 96 is not built
    st = lib.tm_attention_fwd(16, 0, 96, None, None, 0, 0, 0, 16, 16, 0, 96, 8, span, 1, 16, 0,
                              96, 1, 8, 1, 96, 0.0, None)
    assert st == _lib.TM_ERR_UNSUPPORTED
    assert b"head dim" in lib.tm_last_error()
    # misaligned q
    st = lib.tm_attention_fwd(8, 0, 64, None, None, 0, 0, 0, 16, 16, 0, 64, 8, span, 1, 16, 0,
                              64, 1, 8, 1, 64, 0.0, None)
    assert st == _lib.TM_ERR_ALIGNMENT
    # span outside its source
    span[0].rows = 9
    st = lib.tm_attention_fwd(16, 0, 64, None, None, 0, 0, 0, 16, 16, 0, 64, 8, span, 1, 16, 0,
                              64, 1, 8, 1, 64, 0.0, None)
    assert st == _lib.TM_ERR_INVALID_ARGUMENT
    # more visible keys than the kernel's tile table holds
    span[0].rows = 200 * 128
    st = lib.tm_attention_fwd(16, 0, 64, None, None, 0, 0, 0, 16, 16, 0, 64, 200 * 128, span, 1,
                              16, 0, 64, 1, 8, 1, 64, 0.0, None)
    assert st == _lib.TM_ERR_INVALID_ARGUMENT


def test_norm_rope_rejects_before_launch():
    from taomate_b200 import _lib
    lib = _lib.load()
    jobs = (_lib.NormRopeJob * 1)()
    jobs[0].x, jobs[0].out, jobs[0].L = 16, 32, 4
    assert lib.tm_norm_rope(jobs, 1, 1, 3, 128, 1e-6, 1, None) == _lib.TM_ERR_INVALID_ARGUMENT
    assert lib.tm_norm_rope(jobs, 1, 1, 32, 96, 1e-6, 1, None) == _lib.TM_ERR_UNSUPPORTED
    assert lib.tm_norm_rope(jobs, 1, 1, 32, 128, 1e-6, 3, None) == _lib.TM_ERR_INVALID_ARGUMENT
    assert lib.tm_norm_rope(jobs, 5, 1, 32, 128, 1e-6, 1, None) == _lib.TM_ERR_INVALID_ARGUMENT
    jobs[0].cos = 64  # cos without sin
    assert lib.tm_norm_rope(jobs, 1, 1, 32, 128, 1e-6, 1, None) == _lib.TM_ERR_INVALID_ARGUMENT


def test_copy_and_tables_reject_before_launch():
    from taomate_b200 import _lib
    lib = _lib.load()
    spans = (_lib.CopySpan * 1)()
    spans[0].src, spans[0].dst, spans[0].rows = 16, 32, 1
    assert lib.tm_copy_rows(spans, 1, 24, None) == _lib.TM_ERR_ALIGNMENT
    assert lib.tm_copy_rows(spans, 65, 32, None) == _lib.TM_ERR_INVALID_ARGUMENT
    g = (ctypes.c_int64 * 3)(1, 2, 3)
    mp = (ctypes.c_double * 3)(20, 2048, 2048)
    assert lib.tm_rope_tables_split(16, 16, 0, 2, g, 4096, 32, 1e4, mp, 0, 0, 1, None) \
        == _lib.TM_ERR_INVALID_ARGUMENT
    assert b"num_pos_dims" in lib.tm_last_error()
    sizes = (ctypes.c_int64 * 5)(1, 1, 1, 1, 3)
    st = (ctypes.c_int64 * 5)(0, 0, 0, 0, 1)
    assert lib.tm_strided_copy5(16, 32, sizes, st, st, 2, None) == _lib.TM_ERR_ALIGNMENT


def test_status_maps_to_reference_exception_types():
    from taomate_b200 import _lib
    lib = _lib.load()
    spans = (_lib.CopySpan * 1)()
    with pytest.raises(ValueError):
        _lib.check(lib.tm_copy_rows(spans, 0, 16, None), "copy")
    jobs = (_lib.NormRopeJob * 1)()
    jobs[0].x, jobs[0].out, jobs[0].L = 16, 32, 4
    with pytest.raises(NotImplementedError):
        _lib.check(lib.tm_norm_rope(jobs, 1, 1, 32, 96, 1e-6, 1, None), "norm_rope")


def test_product_path_refuses_cpu_tensors():
    import torch
    import taomate_b200 as tm
    q = torch.zeros(1, 8, 2, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        tm.flash_attention(q, None, None, [], q, q, 8)
    with pytest.raises(RuntimeError):
        tm.causal_precompute_freqs_cis(torch.tensor([[1, 2, 3]]), 256, device="cpu")


def test_every_entry_point_cites_the_reference_or_says_it_has_none():
    """Each declaration in include/*.h is documented by the comment right
    before it (or before its group) with the reference function it replaces
    (file.py:line) or with the words "no counterpart" and the reason."""
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        with open(h) as fh:
            txt = fh.read()
        comments = [(m.end(), m.group(0)) for m in re.finditer(r"/\*.*?\*/", txt, re.S)]
        for m in re.finditer(r"TM_API\s+[\w\s\*]+?\b(tm_\w+)\s*\(", txt):
            before = [c for end, c in comments if end <= m.start()]
            doc = before[-1] if before else ""
            assert re.search(r"\.py:\d+", doc) or re.search(r"no\s+counterpart", doc, re.I), \
                f"{m.group(1)}: no reference citation or 'no counterpart' note"
