"""The attention entry point that allocates nothing (tm_attention_fwd_noalloc).

Some programs that host this library cannot allocate device memory while it
runs: a runtime that reserves all of the GPU's memory up front and offers its
plugins no allocator, or a latency-critical path where cudaMalloc's implicit
device synchronisation is not allowed.  For them the key-range split keeps its
scratch in a fixed 16 MiB array inside the library instead of a workspace the
caller allocates.

Through the C ABI, two calls in a row (the second on different inputs, so
anything stale in the shared array would show) are checked against the
workspace entry point on the same inputs, at shapes whose work partition uses
the scratch.  Both entry points plan the same partition and launch the same
kernels, so their outputs must be identical bit for bit.  Two more cases: a
shape that needs no scratch (compared with tm_attention_fwd), and a shape whose
partition needs more than the fixed array, which must be refused before
anything is launched.  This file is collected last on purpose: if it fails, a
run that stops at the first failure has already run every other test.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0) if torch.cuda.is_available() else None
FIXED_BYTES = 16 << 20

SHAPES = [
    # (heads, dim_head, query rows, keys): 4 and 8 heads of the C2 chunk (the
    # per-GPU share under 8- and 4-way sequence parallelism) and V2A's 25
    # audio queries against the video keys
    (4, 128, 1152, 4608),
    (8, 128, 1152, 4608),
    (32, 64, 25, 4608),
]


def _rel_l2(a, b):
    a, b = a.double(), b.double()
    return float(torch.linalg.norm(a - b) / torch.linalg.norm(b))


def _args(lib_mod, q, k, v, out, H, D):
    Lq, Lk = int(q.shape[1]), int(k.shape[1])
    spans = (lib_mod.KVSpan * 1)()
    spans[0].source, spans[0].row_start, spans[0].rows = 1, 0, Lk
    head = (q.data_ptr(), 0, H * D, None, None, 0, 0, 0, k.data_ptr(), v.data_ptr(), 0, H * D,
            Lk, spans, 1, out.data_ptr(), 0, H * D, 1, Lq, H, D, 0.0)
    return head, spans


def _inputs(seed, H, D, Lq, Lk):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(1, Lq, H, D, generator=gen).to(DEV, torch.bfloat16)
    k = torch.randn(1, Lk, H, D, generator=gen).to(DEV, torch.bfloat16)
    v = torch.randn(1, Lk, H, D, generator=gen).to(DEV, torch.bfloat16)
    return q, k, v


def _device_error_clear(lib):
    code = ctypes.c_int(0)
    assert lib.tm_device_error(ctypes.byref(code)) == 0 and code.value == 0


@pytest.mark.parametrize("H,D,Lq,Lk", SHAPES)
def test_noalloc_matches_workspace_entry_on_two_calls(H, D, Lq, Lk):
    from taomate_b200 import _lib
    lib = _lib.load()
    torch.cuda.set_device(DEV)
    need = lib.tm_attention_workspace_bytes(1, Lq, H, D, Lk)
    assert 0 < need <= FIXED_BYTES, "the shape must use the scratch and fit the fixed array"
    stream = _lib.stream_ptr(DEV)
    for call in range(2):
        q, k, v = _inputs(1000 * call + H + D + Lq, H, D, Lq, Lk)
        out_na = torch.full_like(q, float("nan"))
        out_ws = torch.full_like(q, float("nan"))
        args, spans = _args(_lib, q, k, v, out_na, H, D)
        st = lib.tm_attention_fwd_noalloc(*args, stream)
        assert st == 0, lib.tm_last_error()
        ws = torch.empty(need, dtype=torch.uint8, device=DEV)
        args_ws, spans_ws = _args(_lib, q, k, v, out_ws, H, D)
        st = lib.tm_attention_fwd_ws(*args_ws, ws.data_ptr(), need, stream)
        assert st == 0, lib.tm_last_error()
        torch.cuda.synchronize()
        assert torch.isfinite(out_na).all()
        # same partition, same kernels: identical bits
        assert torch.equal(out_na, out_ws)
        # and against an fp32 reference, to the bf16 noise floor
        ref = torch.nn.functional.scaled_dot_product_attention(
            q.transpose(1, 2).float(), k.transpose(1, 2).float(),
            v.transpose(1, 2).float()).transpose(1, 2)
        assert _rel_l2(out_na, ref) < 4e-3
    _device_error_clear(lib)


def test_noalloc_without_split_equals_plain_entry():
    """C2's 32 heads fill the GPU without a key-range split: the fixed array
    goes unused and the result is the plain entry point's."""
    from taomate_b200 import _lib
    lib = _lib.load()
    torch.cuda.set_device(DEV)
    H, D, Lq, Lk = 32, 128, 1152, 4608
    assert lib.tm_attention_workspace_bytes(1, Lq, H, D, Lk) == 0
    stream = _lib.stream_ptr(DEV)
    q, k, v = _inputs(7, H, D, Lq, Lk)
    out_na = torch.full_like(q, float("nan"))
    out_plain = torch.full_like(q, float("nan"))
    args, spans = _args(_lib, q, k, v, out_na, H, D)
    assert lib.tm_attention_fwd_noalloc(*args, stream) == 0, lib.tm_last_error()
    args_p, spans_p = _args(_lib, q, k, v, out_plain, H, D)
    assert lib.tm_attention_fwd(*args_p, stream) == 0, lib.tm_last_error()
    torch.cuda.synchronize()
    assert torch.equal(out_na, out_plain)
    _device_error_clear(lib)


def test_noalloc_refuses_shapes_above_the_fixed_array():
    """13 heads of 832 queries over 4608 keys: the partition splits every
    query tile into 3 key ranges, 16.09 MiB of partial outputs.  The call is
    refused with TM_ERR_INVALID_ARGUMENT before any launch; out is untouched."""
    from taomate_b200 import _lib
    lib = _lib.load()
    torch.cuda.set_device(DEV)
    H, D, Lq, Lk = 13, 128, 832, 4608
    need = lib.tm_attention_workspace_bytes(1, Lq, H, D, Lk)
    assert need > FIXED_BYTES
    q, k, v = _inputs(11, H, D, Lq, Lk)
    out = torch.full_like(q, float("nan"))
    args, spans = _args(_lib, q, k, v, out, H, D)
    st = lib.tm_attention_fwd_noalloc(*args, _lib.stream_ptr(DEV))
    assert st == _lib.TM_ERR_INVALID_ARGUMENT
    msg = lib.tm_last_error().decode()
    assert "tm_attention_fwd_ws" in msg and str(need) in msg
    torch.cuda.synchronize()
    assert torch.isnan(out.float()).all()
    _device_error_clear(lib)
