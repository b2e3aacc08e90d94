"""Ulysses all-to-all host logic on CPU ranks (gloo, world size 2 and 4).

The library has no CPU permute kernel; these tests register a plain torch
permute for CPU tensors (test infrastructure) and check the exchange, the
packed Q/K/V layout and split/gather against the reference's outputs
(tests/golden/a2a.npz), bit-exact.  A rank that never joins must make its
peer's collective fail with a timeout instead of hanging.
"""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cpu_permute(x, perm):
    return x.permute(*perm).contiguous()


def _worker(rank, world, port, outdir):
    import sys
    sys.path.insert(0, os.path.dirname(HERE))
    sys.path.insert(0, os.path.join(HERE, "golden"))
    import inputs
    from taomate_b200 import parallel as P
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    P.register_layout_copy("cpu", _cpu_permute)
    try:
        P.init_sp_mesh(world, world, device_type="cpu")
        assert P.is_sp_enabled() and P.get_sp_world_size() == world
        assert P.get_sp_rank() == rank
        full_np, full2_np, raw_np = inputs.a2a_inputs()
        full, full2 = torch.from_numpy(full_np), torch.from_numpy(full2_np)
        S = full.shape[1]
        Sl = S // world
        shard = full[:, rank * Sl:(rank + 1) * Sl].contiguous()
        shard2 = full2[:, rank * Sl:(rank + 1) * Sl].contiguous()
        s2h = P.seq_all_to_all_head(shard)
        h2s = P.head_all_to_all_seq(s2h)
        with torch.no_grad():
            many = P.seq_all_to_all_head_many((shard, shard2))
            am = P.seq_all_to_all_head_many_async((shard, shard2)).wait()
        a1 = P.seq_all_to_all_head_async(shard).wait()
        a2 = P.head_all_to_all_seq_async(s2h).wait()
        raw = torch.from_numpy(raw_np)
        split = P.split_sequence(raw, dim=1)
        gathered = P.gather_sequence(split, dim=1)
        np.savez(os.path.join(outdir, f"r{rank}.npz"), s2h=s2h.numpy(), h2s=h2s.numpy(),
                 many0=many[0].contiguous().numpy(), many1=many[1].contiguous().numpy(),
                 am0=am[0].contiguous().numpy(), am1=am[1].contiguous().numpy(),
                 a1=a1.numpy(), a2=a2.numpy(), split=split.numpy(), gathered=gathered.numpy())
        dist.barrier()
    finally:
        P.register_layout_copy("cpu", None)
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_ulysses_a2a_matches_reference(tmp_path, golden_dir, world):
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    z = np.load(os.path.join(golden_dir, "a2a.npz"))
    for r in range(world):
        got = np.load(tmp_path / f"r{r}.npz")
        pre = f"g{world}_r{r}__"
        np.testing.assert_array_equal(got["s2h"], z[pre + "s2h"])
        np.testing.assert_array_equal(got["h2s"], z[pre + "h2s"])
        np.testing.assert_array_equal(got["many0"], z[pre + "many0"])
        np.testing.assert_array_equal(got["many1"], z[pre + "many1"])
        np.testing.assert_array_equal(got["am0"], z[pre + "many0"])
        np.testing.assert_array_equal(got["am1"], z[pre + "many1"])
        np.testing.assert_array_equal(got["a1"], z[pre + "s2h"])
        np.testing.assert_array_equal(got["a2"], z[pre + "h2s"])
        np.testing.assert_array_equal(got["split"], z[pre + "split"])
        np.testing.assert_array_equal(got["gathered"], z[pre + "gathered"])


def _absent_peer_worker(rank, world, port, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    import sys
    sys.path.insert(0, os.path.dirname(HERE))
    from taomate_b200 import parallel as P
    P.register_layout_copy("cpu", _cpu_permute)
    x = torch.zeros(1, 4, 4, 2)
    if rank == 1:
        # this rank leaves between steps without joining the collective
        open(os.path.join(outdir, "r1_left"), "w").close()
        return
    try:
        P.seq_all_to_all_head(x, dist.group.WORLD, world)
        open(os.path.join(outdir, "r0_no_error"), "w").close()
    except Exception as e:  # gloo raises on the process-group timeout
        with open(os.path.join(outdir, "r0_error"), "w") as fh:
            fh.write(type(e).__name__)


def test_absent_rank_times_out(tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_absent_peer_worker, args=(r, 2, port, str(tmp_path)))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert (tmp_path / "r1_left").exists()
    assert (tmp_path / "r0_error").exists(), "collective with an absent peer did not fail"
