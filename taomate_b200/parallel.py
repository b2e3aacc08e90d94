"""Ulysses sequence parallelism for the streaming attention path.

Same public API as ``taomate/runtime_support/parallel`` (mesh.py,
all_to_all.py, sp_utils.py): a ``(dp, sp)`` device mesh, seq<->head
all-to-all (sync, packed "many", async) and sequence split / gather.

B200 design:
* one process per GPU, NCCL ``all_to_all_single`` over NVLink / NVSwitch
  (every peer at full bandwidth, so a flat all-to-all needs no topology
  logic);
* the pack permute before the seq->head exchange is done by the producing
  kernel (the fused norm+RoPE store, see :func:`taomate_b200.rope.norm_rope`)
  or by the strided-copy kernel; for batch 1 the receive side of seq->head
  and the send side of head->seq are plain views (no copy);
* Q, K and V travel in ONE collective, interleaved per token, so that after
  the exchange Q/K/V are strided views with a uniform row stride that the
  attention kernel's TMA maps read directly.

With :func:`init_peer_exchange` the two exchanges of ``attention_with_cache``
skip NCCL: every rank maps its peers' receive buffers (CUDA IPC) and the
producing kernels store rows straight into the owner's buffer over NVLink,
followed by a bounded flag handshake (:class:`PeerExchange`).

Layout permutes run on CUDA tensors only.  A test may register a
permute implementation for another device type (e.g. CPU ranks on gloo)
with :func:`register_layout_copy`; the library registers none.
"""

from __future__ import annotations

import contextlib

import ctypes
from typing import Callable, Dict, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from . import _lib

try:  # pragma: no cover - depends on the torch build
    from torch.distributed.device_mesh import init_device_mesh, DeviceMesh
except ImportError:  # pragma: no cover
    init_device_mesh = None
    DeviceMesh = None

# ---------------------------------------------------------------------------
# Mesh (mesh.py:32-160)
# ---------------------------------------------------------------------------
_DEVICE_MESH = None
_SP_SIZE = 1
_DP_SIZE = 1
# Groups and ranks of the mesh, looked up once: slicing a DeviceMesh costs
# ~0.1 ms of host time, far more than the exchange it would precede.
_SP_GROUP = None
_SP_RANK = 0
_DP_GROUP = None
_DP_RANK = 0


def init_sp_mesh(world_size: int, sp_size: int, device_type: str = "cuda"):
    """Create and cache the 2-D ``(dp, sp)`` mesh; ``sp_size <= 1`` disables SP."""
    global _DEVICE_MESH, _SP_SIZE, _DP_SIZE, _SP_GROUP, _SP_RANK, _DP_GROUP, _DP_RANK
    if sp_size <= 1:
        _DEVICE_MESH, _SP_SIZE, _DP_SIZE = None, 1, max(world_size, 1)
        _SP_GROUP, _SP_RANK, _DP_GROUP, _DP_RANK = None, 0, None, 0
        return None, _DP_SIZE, 1
    if world_size % sp_size != 0:
        raise ValueError(f"world_size ({world_size}) must be divisible by sp_size ({sp_size}).")
    if init_device_mesh is None:
        raise RuntimeError("torch.distributed.device_mesh.init_device_mesh is unavailable")
    if not dist.is_available() or not dist.is_initialized():
        raise RuntimeError("init_sp_mesh requires torch.distributed to be initialized first.")
    dp_size = world_size // sp_size
    mesh = init_device_mesh(device_type, (dp_size, sp_size), mesh_dim_names=("dp", "sp"))
    _DEVICE_MESH, _SP_SIZE, _DP_SIZE = mesh, sp_size, dp_size
    _SP_GROUP, _SP_RANK = mesh["sp"].get_group(), int(mesh["sp"].get_local_rank())
    _DP_GROUP, _DP_RANK = mesh["dp"].get_group(), int(mesh["dp"].get_local_rank())
    return mesh, dp_size, sp_size


def get_device_mesh():
    return _DEVICE_MESH


_SP_LOCAL = 0  # > 0 inside sp_local(): calls run as if sequence parallelism were off


def is_sp_enabled() -> bool:
    return _DEVICE_MESH is not None and _SP_SIZE > 1 and _SP_LOCAL == 0


@contextlib.contextmanager
def sp_local():
    """Run the enclosed calls as single-GPU calls on this rank's tensors even
    though the SP mesh is set: for work every rank holds in full (the audio
    stream, which a block replicates instead of splitting its 25 tokens) and
    for attentions whose keys and values every rank already has.  Same role as
    the reference's ``cp_disabled`` (ltx_causal/parallel/cp_utils.py:169-188)."""
    global _SP_LOCAL
    _SP_LOCAL += 1
    try:
        yield
    finally:
        _SP_LOCAL -= 1


def get_sp_group():
    return None if _DEVICE_MESH is None else _SP_GROUP


def get_sp_world_size() -> int:
    return _SP_SIZE


def get_sp_rank() -> int:
    return 0 if _DEVICE_MESH is None else _SP_RANK


def get_dp_group():
    if _DEVICE_MESH is None:
        return dist.group.WORLD if dist.is_available() and dist.is_initialized() else None
    return _DP_GROUP


def get_dp_world_size() -> int:
    if _DEVICE_MESH is None:
        return dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1
    return _DP_SIZE


def get_dp_rank() -> int:
    if _DEVICE_MESH is None:
        return dist.get_rank() if dist.is_available() and dist.is_initialized() else 0
    return _DP_RANK


# ---------------------------------------------------------------------------
# Layout copies
# ---------------------------------------------------------------------------
_LAYOUT_COPY: Dict[str, Callable[[torch.Tensor, Sequence[int]], torch.Tensor]] = {}


def register_layout_copy(device_type: str, fn: Optional[Callable]) -> None:
    """Install (or remove with ``None``) the permute-copy used for tensors of
    ``device_type`` other than CUDA."""
    if fn is None:
        _LAYOUT_COPY.pop(device_type, None)
    else:
        _LAYOUT_COPY[device_type] = fn


def permute_copy(x: torch.Tensor, perm: Sequence[int]) -> torch.Tensor:
    """Contiguous ``x.permute(perm)`` for a rank-5 tensor whose last dim stays
    last and contiguous (one strided-copy kernel on CUDA)."""
    if x.dim() != 5 or perm[4] != 4:
        raise ValueError("permute_copy expects rank 5 with the innermost dim fixed")
    if not x.is_cuda:
        fn = _LAYOUT_COPY.get(x.device.type)
        if fn is None:
            raise RuntimeError(f"no layout-copy kernel for {x.device.type} tensors")
        return fn(x, perm)
    if x.stride(4) != 1:
        x = x.contiguous()
    xp = x.permute(*perm)
    out = torch.empty(xp.shape, dtype=x.dtype, device=x.device)
    if out.numel() == 0:
        return out
    sizes = (ctypes.c_int64 * 5)(*[int(v) for v in xp.shape])
    sst = (ctypes.c_int64 * 5)(*[int(v) for v in xp.stride()])
    dst = (ctypes.c_int64 * 5)(*[int(v) for v in out.stride()])
    with torch.cuda.device(x.device):
        _lib.check(_lib.load().tm_strided_copy5(xp.data_ptr(), out.data_ptr(), sizes, sst, dst,
                                                x.element_size(), _lib.stream_ptr(x.device)),
                   "permute_copy")
        _lib.launched()
    return out


def _a2a(send: torch.Tensor, group, async_op: bool = False):
    recv = torch.empty_like(send)
    work = dist.all_to_all_single(recv, send, group=group, async_op=async_op)
    return recv, work


def _recv_to_head_layout(recv: torch.Tensor) -> torch.Tensor:
    """``[sp, B, S_loc, H_l, D] -> [B, sp * S_loc, H_l, D]`` (a view when B == 1)."""
    sp, B, S_loc, Hl, D = recv.shape
    if B == 1:
        return recv.view(1, sp * S_loc, Hl, D)
    return permute_copy(recv, (1, 0, 2, 3, 4)).view(B, sp * S_loc, Hl, D)


def _seq_to_head_send(x: torch.Tensor, sp_size: int) -> torch.Tensor:
    B, S_loc, H, D = x.shape
    if H % sp_size != 0:
        raise AssertionError(f"H ({H}) must be divisible by sp_size ({sp_size})")
    return permute_copy(x.reshape(B, S_loc, sp_size, H // sp_size, D), (2, 0, 1, 3, 4))


def _head_to_seq_send(x: torch.Tensor, sp_size: int) -> torch.Tensor:
    B, S, Hl, D = x.shape
    if S % sp_size != 0:
        raise AssertionError(f"S ({S}) must be divisible by sp_size ({sp_size})")
    if B == 1 and x.is_contiguous():
        return x.view(sp_size, 1, S // sp_size, Hl, D)
    return permute_copy(x.reshape(B, sp_size, S // sp_size, Hl, D), (1, 0, 2, 3, 4))


def _recv_to_seq_layout(recv: torch.Tensor) -> torch.Tensor:
    """``[sp, B, S_loc, H_l, D] -> [B, S_loc, sp * H_l, D]``."""
    sp, B, S_loc, Hl, D = recv.shape
    return permute_copy(recv, (1, 2, 0, 3, 4)).view(B, S_loc, sp * Hl, D)


def _seq_to_head(x: torch.Tensor, sp_size: int, group) -> torch.Tensor:
    """``[B, S/sp, H, D] -> [B, S, H/sp, D]`` (all_to_all.py:125-151)."""
    recv, _ = _a2a(_seq_to_head_send(x, sp_size), group)
    return _recv_to_head_layout(recv)


def _head_to_seq(x: torch.Tensor, sp_size: int, group) -> torch.Tensor:
    """``[B, S, H/sp, D] -> [B, S/sp, H, D]`` (all_to_all.py:154-173)."""
    recv, _ = _a2a(_head_to_seq_send(x, sp_size), group)
    return _recv_to_seq_layout(recv)


# ---------------------------------------------------------------------------
# Public all-to-all API (all_to_all.py:267-432)
# ---------------------------------------------------------------------------
def _resolve(group, sp_size):
    if sp_size is None:
        sp_size = get_sp_world_size()
    if group is None and sp_size > 1:
        group = get_sp_group()
    return group, sp_size


def seq_all_to_all_head(x: torch.Tensor, group=None, sp_size: Optional[int] = None) -> torch.Tensor:
    """``[B, S/sp, H, D] -> [B, S, H/sp, D]``; identity when ``sp_size <= 1``."""
    group, sp_size = _resolve(group, sp_size)
    if sp_size <= 1:
        return x
    return _seq_to_head(x, sp_size, group)


def head_all_to_all_seq(x: torch.Tensor, group=None, sp_size: Optional[int] = None) -> torch.Tensor:
    """``[B, S, H/sp, D] -> [B, S/sp, H, D]``; identity when ``sp_size <= 1``."""
    group, sp_size = _resolve(group, sp_size)
    if sp_size <= 1:
        return x
    return _head_to_seq(x, sp_size, group)


def seq_all_to_all_head_packed(send: torch.Tensor, group=None, sp_size: Optional[int] = None):
    """Exchange a packed send buffer ``[sp, B, S_loc, n, H/sp, D]`` (as written
    by ``norm_rope(..., packed=True)``) and return the ``n`` head-sharded
    ``[B, S, H/sp, D]`` views (uniform row stride ``n * H/sp * D`` when B == 1)."""
    group, sp_size = _resolve(group, sp_size)
    sp, B, S_loc, n, Hl, D = send.shape
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    if B == 1:
        flat = recv.view(sp * S_loc, n, Hl, D)
        return tuple(flat[:, i].unsqueeze(0) for i in range(n))
    return tuple(_recv_to_head_layout(recv[:, :, :, i]) for i in range(n))


def seq_all_to_all_head_many(tensors, group=None, sp_size: Optional[int] = None):
    """Packed ``seq_all_to_all_head`` for same-shaped tensors: one collective
    (all_to_all.py:285-315)."""
    tensors = tuple(tensors)
    if not tensors:
        return tuple()
    group, sp_size = _resolve(group, sp_size)
    if sp_size <= 1 or len(tensors) == 1:
        return tensors if sp_size <= 1 else (seq_all_to_all_head(tensors[0], group, sp_size),)
    base = tuple(tensors[0].shape)
    if any(tuple(t.shape) != base for t in tensors):
        return tuple(seq_all_to_all_head(t, group=group, sp_size=sp_size) for t in tensors)
    B, S_loc, H, D = base
    if H % sp_size != 0:
        raise AssertionError(f"H ({H}) must be divisible by sp_size ({sp_size})")
    Hl = H // sp_size
    n = len(tensors)
    send = torch.empty(sp_size, B, S_loc, n, Hl, D, dtype=tensors[0].dtype,
                       device=tensors[0].device)
    for i, t in enumerate(tensors):
        send[:, :, :, i].copy_(_seq_to_head_send(t, sp_size))
    return seq_all_to_all_head_packed(send, group, sp_size)


class _AsyncAllToAll:
    """Handle of a non-blocking exchange; ``wait()`` returns the result."""

    def __init__(self, recv, work, finish):
        self._recv, self._work, self._finish = recv, work, finish

    def wait(self):
        if self._work is not None:
            self._work.wait()
            self._work = None
        return self._finish(self._recv)


class _Immediate:
    def __init__(self, value):
        self.value = value

    def wait(self):
        return self.value


def seq_all_to_all_head_async(x: torch.Tensor, group=None, sp_size: Optional[int] = None):
    group, sp_size = _resolve(group, sp_size)
    if sp_size <= 1:
        return _Immediate(x)
    recv, work = _a2a(_seq_to_head_send(x, sp_size), group, async_op=True)
    return _AsyncAllToAll(recv, work, _recv_to_head_layout)


def head_all_to_all_seq_async(x: torch.Tensor, group=None, sp_size: Optional[int] = None):
    group, sp_size = _resolve(group, sp_size)
    if sp_size <= 1:
        return _Immediate(x)
    recv, work = _a2a(_head_to_seq_send(x, sp_size), group, async_op=True)
    return _AsyncAllToAll(recv, work, _recv_to_seq_layout)


def seq_all_to_all_head_many_async(tensors, group=None, sp_size: Optional[int] = None):
    tensors = tuple(tensors)
    if not tensors:
        raise ValueError("seq_all_to_all_head_many_async requires at least one tensor")
    group, sp_size = _resolve(group, sp_size)
    if sp_size <= 1:
        return _Immediate(tensors)
    if len(tensors) == 1:
        return seq_all_to_all_head_async(tensors[0], group, sp_size)
    if torch.is_grad_enabled():
        raise RuntimeError("seq_all_to_all_head_many_async is inference-only")
    base = tuple(tensors[0].shape)
    if any(tuple(t.shape) != base for t in tensors):
        raise ValueError("seq_all_to_all_head_many_async requires same-shaped tensors")
    B, S_loc, H, D = base
    Hl = H // sp_size
    n = len(tensors)
    send = torch.empty(sp_size, B, S_loc, n, Hl, D, dtype=tensors[0].dtype,
                       device=tensors[0].device)
    for i, t in enumerate(tensors):
        send[:, :, :, i].copy_(_seq_to_head_send(t, sp_size))
    recv = torch.empty_like(send)
    work = dist.all_to_all_single(recv, send, group=group, async_op=True)

    def finish(r):
        if B == 1:
            flat = r.view(sp_size * S_loc, n, Hl, D)
            return tuple(flat[:, i].unsqueeze(0) for i in range(n))
        return tuple(_recv_to_head_layout(r[:, :, :, i]) for i in range(n))

    return _AsyncAllToAll(recv, work, finish)


# ---------------------------------------------------------------------------
# Sequence split / gather (sp_utils.py:25-144)
# ---------------------------------------------------------------------------
def pad_sequence_to_multiple(x: torch.Tensor, multiple: int, dim: int = 1,
                             pad_value: float = 0.0) -> Tuple[torch.Tensor, int, int]:
    S = x.shape[dim]
    if multiple <= 1 or S % multiple == 0:
        return x, S, S
    pad = multiple - (S % multiple)
    shape = list(x.shape)
    shape[dim] = S + pad
    out = torch.full(shape, pad_value, dtype=x.dtype, device=x.device)
    out.narrow(dim, 0, S).copy_(x)
    return out, S, S + pad


def unpad_sequence(x: torch.Tensor, original_length: int, dim: int = 1) -> torch.Tensor:
    if x.shape[dim] == original_length:
        return x
    return x.narrow(dim, 0, original_length).contiguous()


def split_sequence(x: torch.Tensor, dim: int = 1, sp_rank: Optional[int] = None,
                   sp_size: Optional[int] = None) -> torch.Tensor:
    """Local shard along ``dim`` after right-padding with zeros to a multiple
    of ``sp_size``."""
    if sp_size is None:
        sp_size = get_sp_world_size()
    if sp_size <= 1:
        return x
    if sp_rank is None:
        sp_rank = get_sp_rank()
    x, _, S = pad_sequence_to_multiple(x, sp_size, dim)
    chunk = S // sp_size
    return x.narrow(dim, sp_rank * chunk, chunk).contiguous()


def gather_sequence(x: torch.Tensor, dim: int = 1, group=None, sp_size: Optional[int] = None,
                    sp_rank: Optional[int] = None) -> torch.Tensor:
    """All-gather along ``dim`` over the SP group."""
    if sp_size is None:
        sp_size = get_sp_world_size()
    if sp_size <= 1:
        return x
    if group is None:
        group = get_sp_group()
    x = x.contiguous()
    parts = [torch.empty_like(x) for _ in range(sp_size)]
    dist.all_gather(parts, x, group=group)
    return torch.cat(parts, dim=dim)


# ---------------------------------------------------------------------------
# Fused exchanges over NVLink peer memory
# ---------------------------------------------------------------------------
class _DevBuffer:
    """A cudaMalloc'd buffer exposed to torch without a copy."""

    def __init__(self, ptr: int, nbytes: int, device: torch.device):
        self.__cuda_array_interface__ = {"shape": (nbytes // 2,), "typestr": "<u2",
                                         "data": (ptr, False), "version": 3, "strides": None}
        self.tensor = torch.as_tensor(self, device=device).view(torch.bfloat16)


class PeerExchange:
    """Receive buffers of the two Ulysses exchanges, mapped on every rank.

    * ``recv``: ``[sp, B, S_loc, 3, H/sp, D]`` — Q, K, V of the full chunk for
      this rank's heads; rank g's norm+RoPE kernel stores its tokens at
      ``recv[g]`` (all_to_all.py:125-151 layout).
    * ``out``: ``[B, S_loc, H, D]`` — this rank's tokens for all heads; rank
      g's attention kernel stores heads ``g * H/sp ...`` of them
      (all_to_all.py:154-173).
    * ``gather`` (optional, ``gather_bytes`` > 0): two buffers of
      ``gather_bytes`` for small all-gathers (the V2A partial results under
      sequence parallelism): rank g's part sits at ``g * part_bytes``; a rank
      copies its part into every peer's buffer and runs the handshake of
      slot 2 (:meth:`all_gather_parts`).  Consecutive layers use the two
      buffers in turn, so a rank that runs ahead never overwrites parts a
      slower peer is still merging.
    * flags and device epoch counters for the handshakes (slot 0: seq->head,
      slot 1: head->seq, slot 2: gather).

    The buffers are reused by every call: the returned Q/K/V/out are views
    that the next call overwrites (``attention_with_cache`` copies the new K/V
    it returns).  One exchange object per process; calls must come in the
    same order on every rank.
    """

    def __init__(self, group, sp_size: int, rank: int, batch: int, tokens_local: int,
                 heads: int, dim_head: int, device: torch.device, gather_bytes: int = 0):
        if sp_size < 2 or sp_size > 8 or heads % sp_size:
            raise ValueError(f"peer exchange needs 2..8 ranks dividing {heads} heads")
        lib = _lib.load()
        self.lib, self.group, self.sp, self.rank = lib, group, sp_size, rank
        self.B, self.S_loc, self.H, self.D = batch, tokens_local, heads, dim_head
        self.Hl = heads // sp_size
        self.device = torch.device(device)
        el = 2
        sizes = {
            "recv": sp_size * batch * tokens_local * 3 * self.Hl * dim_head * el,
            "out": batch * tokens_local * heads * dim_head * el,
            "flags": int(lib.tm_peer_flag_bytes()),
        }
        self.gather_bytes = (int(gather_bytes) + 255) // 256 * 256
        if self.gather_bytes > 0:
            sizes["gather"] = 2 * self.gather_bytes
        self._own: Dict[str, int] = {}
        self._opened = []
        handles = {}
        with torch.cuda.device(self.device):
            for name, n in sizes.items():
                ptr = ctypes.c_void_p()
                h = (ctypes.c_char * 64)()
                _lib.check(lib.tm_peer_alloc(n, ctypes.byref(ptr), ctypes.cast(h, ctypes.c_void_p)),
                           "peer_alloc")
                self._own[name] = int(ptr.value)
                handles[name] = bytes(h)
            gathered = [None] * sp_size
            dist.all_gather_object(gathered, handles, group=group)
            self.peers: Dict[str, list] = {name: [] for name in sizes}
            for g in range(sp_size):
                for name in sizes:
                    if g == rank:
                        self.peers[name].append(self._own[name])
                        continue
                    p = ctypes.c_void_p()
                    hb = (ctypes.c_char * 64).from_buffer_copy(gathered[g][name])
                    _lib.check(lib.tm_peer_open(ctypes.cast(hb, ctypes.c_void_p), ctypes.byref(p)),
                               "peer_open")
                    self.peers[name].append(int(p.value))
                    self._opened.append(int(p.value))
        self.delta = {name: (ctypes.c_int64 * 8)(*[v - self._own[name] for v in self.peers[name]])
                      for name in ("recv", "out")}
        self._flag_ptrs = (ctypes.c_void_p * 8)(*self.peers["flags"])
        self._counters = self._own["flags"] + sizes["flags"] - 64
        self.recv = _DevBuffer(self._own["recv"], sizes["recv"], self.device).tensor.view(
            sp_size, batch, tokens_local, 3, self.Hl, dim_head)
        self.out = _DevBuffer(self._own["out"], sizes["out"], self.device).tensor.view(
            batch, tokens_local, heads, dim_head)
        self.gather = None
        if self.gather_bytes:
            self.gather = _DevBuffer(self._own["gather"], sizes["gather"],
                                     self.device).tensor.view(torch.uint8)

    def gather_buffer(self, index: int, part_bytes: int) -> Optional[torch.Tensor]:
        """Gather buffer ``index % 2`` as a uint8 tensor of ``sp * part_bytes``
        bytes (None when the parts do not fit)."""
        n = self.sp * int(part_bytes)
        if self.gather is None or n > self.gather_bytes or part_bytes % 16:
            return None
        off = (index % 2) * self.gather_bytes
        return self.gather[off:off + n]

    def all_gather_parts(self, buf: torch.Tensor, part_bytes: int) -> None:
        """Copy this rank's part of ``buf`` (a :meth:`gather_buffer` view,
        already written) into the same place of every peer's buffer over
        NVLink, then the slot-2 handshake: afterwards ``buf`` holds every
        rank's part."""
        base = self._own["gather"]
        off = buf.data_ptr() - base + self.rank * part_bytes
        if off < 0 or off + part_bytes > 2 * self.gather_bytes:
            raise ValueError("not a view of this exchange's gather buffers")
        spans = (_lib.CopySpan * max(1, self.sp - 1))()
        i = 0
        for g in range(self.sp):
            if g == self.rank:
                continue
            spans[i].src, spans[i].dst, spans[i].rows = base + off, self.peers["gather"][g] + off, 1
            spans[i].src_row_stride = spans[i].dst_row_stride = part_bytes
            i += 1
        stream = _lib.stream_ptr(self.device)
        with torch.cuda.device(self.device):
            _lib.check(self.lib.tm_copy_rows(spans, i, part_bytes, stream), "gather copy")
            _lib.launched()
        self.exchange(2)

    def fits(self, B: int, L: int, H: int, D: int) -> bool:
        return (B, L, H, D) == (self.B, self.S_loc, self.H, self.D)

    def exchange(self, slot: int) -> None:
        """Publish this rank's stores of ``slot`` and wait for every rank's."""
        stream = _lib.stream_ptr(self.device)
        _lib.check(self.lib.tm_peer_exchange(self._flag_ptrs, self.sp, self.rank,
                                             self._own["flags"], self._counters, slot, stream),
                   "peer_exchange")
        _lib.launched()

    def close(self) -> None:
        if not self._own:
            return
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for p in self._opened:
                self.lib.tm_peer_close(ctypes.c_void_p(p))
            for p in self._own.values():
                self.lib.tm_peer_free(ctypes.c_void_p(p))
        self._opened, self._own = [], {}


_PEER: Optional[PeerExchange] = None


def init_peer_exchange(batch: int, tokens_local: int, heads: int, dim_head: int,
                       device=None, gather_bytes: int = 0) -> Optional[PeerExchange]:
    """Map NVLink receive buffers for ``attention_with_cache``'s exchanges on
    the SP group (collective over the group; call after :func:`init_sp_mesh`
    on every rank).  Calls whose shapes differ keep using NCCL.
    ``gather_bytes``: size of each of the two gather buffers of the split-key
    V2A (``taomate_b200.block.v2a_gather_bytes``); 0 keeps it on NCCL."""
    global _PEER
    if not is_sp_enabled():
        return None
    if _PEER is not None:
        _PEER.close()
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    _PEER = PeerExchange(_SP_GROUP, _SP_SIZE, _SP_RANK, batch, tokens_local, heads, dim_head,
                         dev, gather_bytes=gather_bytes)
    return _PEER


def get_peer_exchange() -> Optional[PeerExchange]:
    return _PEER


def close_peer_exchange() -> None:
    """Unmap and free the exchange buffers (before the process group goes)."""
    global _PEER
    if _PEER is not None:
        _PEER.close()
    _PEER = None
