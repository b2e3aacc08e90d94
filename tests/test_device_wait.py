"""Device-side failure path of the NVLink exchange: a bounded flag wait.

A lost peer must never hang the GPU.  Each wait of tm_peer_wait /
tm_peer_exchange spins on flags that the other ranks publish, bounded by a
wall-clock limit; when it runs out the kernel records device error 2 and
returns, and the host reads it with tm_device_error.  Here one GPU waits for a
second rank that does not exist: the flag arrays are local, zeroed, and nothing
ever signals them.  The limit is set short (50 ms) through the C ABI, so each
wait ends by itself; the test checks the status, that the epoch counter moved
on (the next wait waits for the following epoch), and that the context still
runs a normal kernel correctly afterwards.
"""

import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0) if torch.cuda.is_available() else None
LIMIT_NS = 50_000_000
SLOTS, MAX_RANKS = 4, 8


def _read_error(lib):
    code = ctypes.c_int(-1)
    assert lib.tm_device_error(ctypes.byref(code)) == 0, lib.tm_last_error()
    return code.value


def test_peer_wait_runs_out_and_context_survives():
    from taomate_b200 import _lib
    lib = _lib.load()
    torch.cuda.set_device(DEV)
    assert _read_error(lib) == 0
    nbytes = int(lib.tm_peer_flag_bytes())
    assert nbytes == 8 * (SLOTS * MAX_RANKS + 2 * SLOTS)
    own = torch.zeros(nbytes // 8, dtype=torch.int64, device=DEV)    # this rank's flags
    other = torch.zeros(nbytes // 8, dtype=torch.int64, device=DEV)  # "rank 1", never runs
    counters = own[SLOTS * MAX_RANKS:]
    stream = _lib.stream_ptr(DEV)
    old = lib.tm_peer_set_wait_limit(LIMIT_NS)
    try:
        # 1. a plain wait on slot 0 for two ranks: nobody signals
        t0 = time.perf_counter()
        assert lib.tm_peer_wait(own.data_ptr(), 2, counters.data_ptr(), 0, stream) == 0
        assert _read_error(lib) == 2
        first = time.perf_counter() - t0
        # the awaited epoch of slot 0 moved on; the next wait targets epoch 2
        assert int(counters[SLOTS + 0]) == 1
        assert lib.tm_peer_wait(own.data_ptr(), 2, counters.data_ptr(), 0, stream) == 0
        assert _read_error(lib) == 2
        assert int(counters[SLOTS + 0]) == 2
        # 2. signal + wait in one launch (slot 1): this rank's own flag is
        # published in both arrays, rank 1's never arrives
        peers = (ctypes.c_void_p * 2)(own.data_ptr(), other.data_ptr())
        assert lib.tm_peer_exchange(peers, 2, 0, own.data_ptr(), counters.data_ptr(), 1,
                                    stream) == 0
        assert _read_error(lib) == 2
        assert int(own[1 * MAX_RANKS + 0]) == 1 and int(other[1 * MAX_RANKS + 0]) == 1
        assert int(own[1 * MAX_RANKS + 1]) == 0
        assert int(counters[1]) == 1 and int(counters[SLOTS + 1]) == 1
        assert first < 5.0, f"a 50 ms wait took {first:.2f} s"
    finally:
        lib.tm_peer_set_wait_limit(old)
    assert lib.tm_peer_set_wait_limit(0) == old  # 0 restores the default
    # 3. the context is intact: an attention call still gives the right answer
    import taomate_b200 as tm
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(1, 256, 4, 128, generator=g).to(DEV, torch.bfloat16) for _ in range(3))
    out = tm.standard_attention_forward(q, k, v)
    ref = torch.nn.functional.scaled_dot_product_attention(
        q.transpose(1, 2).float(), k.transpose(1, 2).float(), v.transpose(1, 2).float()
    ).transpose(1, 2)
    rel = float(torch.linalg.norm((out.float() - ref).double()) / torch.linalg.norm(ref.double()))
    assert rel < 4e-3
    assert _read_error(lib) == 0
