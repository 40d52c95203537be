"""Multi-GPU sharding of the quantized-inference path (one process per GPU).

* DequantizeLinear -> MatMul: the weight [K, N] (with its scales / zero points)
  is split by columns into `world` contiguous slices; every rank computes its
  [M, N/world] output slice with the fused kernel and the slices are
  all-gathered (NCCL over NVLink on GPUs, gloo on CPU) into the full [M, N]
  output.  Activations are replicated.
* Attention: KV heads are split into `world` contiguous groups; each rank holds
  the KV cache of its heads and the matching query heads (GQA groups never
  straddle ranks), and the per-head outputs are all-gathered.

Three ways to produce the gathered output:
* `PeerGroup.matmul` (GPUs, int4 decode): the fused DequantizeLinear -> MatMul
  kernel stores its column slice straight into every rank's full output
  (b2_dequantize_matmul_peer) and publishes its completion; the next sharded
  call waits for it before reading -- no gather kernel at all;
* `PeerGroup.gather` (GPUs): b2_allgather_cols stores each rank's slice straight
  into the [M, N] output of every rank over NVLink (CUDA IPC peer buffers set
  up once) and waits on per-rank arrival flags -- one kernel, no staging
  buffer, graph-capturable;
* `gather_columns` (any backend, gloo on CPU): a collective all-gather into the
  rank-major buffer [world, M, N/world]; for M == 1 that is already the [M, N]
  layout, otherwise one transpose copy restores it.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Callable, Dict, Optional

import torch
import torch.distributed as dist


def shard_range(n: int, world: int, rank: int):
    """Contiguous [begin, end) of `n` items owned by `rank` (equal shards)."""
    if n % world:
        raise ValueError(f"{n} columns do not split evenly over {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


def column_slice(t: torch.Tensor, world: int, rank: int, axis: int = -1) -> torch.Tensor:
    b, e = shard_range(t.shape[axis], world, rank)
    return t.narrow(axis, b, e - b).contiguous()


def gather_columns(local: torch.Tensor, world: int, group=None,
                   out: Optional[torch.Tensor] = None,
                   staging: Optional[torch.Tensor] = None) -> torch.Tensor:
    """All-gathers [M, n_loc] slices into [M, world * n_loc] (rank order)."""
    M, n_loc = local.shape
    if staging is None:
        staging = torch.empty((world, M, n_loc), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(staging.view(-1), local.contiguous().view(-1), group=group)
    if out is None:
        out = torch.empty((M, world * n_loc), dtype=local.dtype, device=local.device)
    if M == 1:
        out.view(-1).copy_(staging.view(-1))
    else:
        out.copy_(staging.permute(1, 0, 2).reshape(M, world * n_loc))
    return out


@dataclass
class ShardedLinear:
    """A column-sharded weight-only quantized projection.

    `compute(a, w, scale, zp)` runs the local fused DequantizeLinear -> MatMul
    (the CUDA kernel on GPUs); `__call__` returns the gathered full output.
    """

    w: object
    scale: torch.Tensor
    zp: object
    n_total: int
    world: int
    compute: Callable
    group: object = None

    def __call__(self, a: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        local = self.compute(a, self.w, self.scale, self.zp)
        local = local.reshape(-1, local.shape[-1])
        full = gather_columns(local, self.world, self.group)
        shape = tuple(a.shape[:-1]) + (self.n_total,)
        if out is not None:
            out.view(-1, self.n_total).copy_(full)
            return out
        return full.reshape(shape)


def kv_head_range(kv_heads: int, q_heads: int, world: int, rank: int):
    """(kv_begin, kv_end, q_begin, q_end) of the heads a rank owns."""
    kb, ke = shard_range(kv_heads, world, rank)
    group = q_heads // kv_heads
    return kb, ke, kb * group, ke * group


def gather_heads(local_y: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """All-gathers rank-4 [B, Hq/world, S, D] head slices into [B, Hq, S, D]."""
    B, h, S, D = local_y.shape
    staging = torch.empty((world, B, h, S, D), dtype=local_y.dtype, device=local_y.device)
    dist.all_gather_into_tensor(staging.view(-1), local_y.contiguous().view(-1), group=group)
    return staging.permute(1, 0, 2, 3, 4).reshape(B, world * h, S, D)


class _CudaArray:
    """__cuda_array_interface__ view of a raw device allocation (for torch.as_tensor)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape),
                                         "typestr": typestr, "version": 3, "strides": None}


_TYPESTR = {torch.float16: "<f2", torch.bfloat16: "<u2", torch.float32: "<f4",
            torch.int32: "<i4", torch.uint8: "|u1"}


class PeerGroup:
    """Peer-memory all-gather buffers of one process group (one rank per GPU).

    `buffer(name, shape, dtype)` allocates a full output every rank can write
    (CUDA IPC, exchanged once through the process group); `gather(name,
    local)` runs b2_allgather_cols on the current stream: this rank's column
    slice lands in every rank's `buffer(name)`, and the call returns once all
    slices are in place here.  All ranks must create the same buffers and
    issue the same gathers in the same order.  Set-up allocates and talks to
    the process group; gathers do neither.
    """

    FLAGS = 8  # uint32 per flag array (b2_allgather_cols supports up to 8 ranks)

    def __init__(self, group=None):
        from . import _capi
        self._capi = _capi
        self.lib = _capi.lib()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > self.FLAGS:
            raise ValueError(f"b2_allgather_cols supports up to {self.FLAGS} ranks")
        self._own = []      # (ptr) allocations of this rank
        self._opened = []   # peer mappings
        self.bufs: Dict[str, tuple] = {}
        self._dirty = set()  # buffers a sharded call wrote since the last wait
        # flags: one array per rank; counters: local only
        flags_ptr, peers = self._shared(self.FLAGS * 4)
        self.flag_ptrs = (C.c_void_p * self.world)(*peers)
        ctr = C.c_void_p()
        handle = C.create_string_buffer(64)
        _capi.check(self.lib.b2_ipc_alloc(8, C.byref(ctr), handle))
        self._own.append(ctr.value)
        self.counters = ctr.value

    def _shared(self, nbytes: int):
        """Allocates nbytes here and maps every rank's allocation: (own, [per rank])."""
        ptr = C.c_void_p()
        handle = C.create_string_buffer(64)
        self._capi.check(self.lib.b2_ipc_alloc(nbytes, C.byref(ptr), handle))
        self._own.append(ptr.value)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=self.group)
        peers = []
        for r, h in enumerate(handles):
            if r == self.rank:
                peers.append(ptr.value)
                continue
            p = C.c_void_p()
            self._capi.check(self.lib.b2_ipc_open(C.create_string_buffer(h, 64), C.byref(p)))
            self._opened.append(p.value)
            peers.append(p.value)
        return ptr.value, peers

    def buffer(self, name: str, shape, dtype=torch.float16) -> torch.Tensor:
        if name not in self.bufs:
            nbytes = int(torch.tensor([], dtype=dtype).element_size())
            for d in shape:
                nbytes *= int(d)
            own, peers = self._shared(nbytes)
            t = torch.as_tensor(_CudaArray(own, shape, _TYPESTR[dtype]), device="cuda")
            if dtype == torch.bfloat16:
                t = t.view(torch.bfloat16)
            self.bufs[name] = (t, (C.c_void_p * self.world)(*peers), int(shape[-1]))
        return self.bufs[name][0]

    def _peer_out(self, name: str):
        full, peers, n_total = self.bufs[name]
        po = self._capi.B2PeerOut()
        for r in range(self.world):
            po.full[r] = peers[r]
            po.flags[r] = self.flag_ptrs[r]
        po.counters = self.counters
        po.world, po.rank, po.n_full = self.world, self.rank, n_total
        return po

    def matmul(self, name: str, a: torch.Tensor, w, scale: torch.Tensor, axis: int = 0,
               workspace_fn=None) -> torch.Tensor:
        """y = DequantizeLinear(w, scale) @ a on this rank's column slice, stored
        into every rank's `buffer(name)` by the kernel itself
        (b2_dequantize_matmul_peer); returns this rank's full buffer, complete
        for the next sharded call (which waits for it) or after `wait()`."""
        from . import kernels
        full, peers, n_total = self.bufs[name]
        n_loc = n_total // self.world
        lead = tuple(a.shape[:-1])
        po = self._peer_out(name)
        # wait for the other ranks only when the input is a peer output
        # written since the last wait (then every earlier call is complete)
        src = next((n for n, b in self.bufs.items() if b[0].data_ptr() == a.data_ptr()), None)
        po.wait_input = 1 if src in self._dirty else 0
        if po.wait_input:
            self._dirty.clear()
        self._dirty.add(name)
        ad = self._capi.Desc(a.data_ptr(), self._capi.TORCH_TO_ONNX[a.dtype], tuple(a.shape))
        wd = kernels._desc(w)
        sd = kernels._desc(scale)
        yd = self._capi.Desc(0, self._capi.TORCH_TO_ONNX[a.dtype], lead + (n_loc,))
        kernels._call_with_workspace(self.lib.b2_dequantize_matmul_peer,
                                     (ad.ref, wd.ref, sd.ref, None, int(axis), 0, yd.ref,
                                      C.byref(po)), (self._capi.stream_ptr(a.device),), a.device)
        return full

    def matmul_group(self, names, a: torch.Tensor, ws, scales, axis: int = 0):
        """matmul for projections that read the same `a` (q / k / v, gate /
        up), as one launch (b2_dequantize_matmul_group_peer); returns this
        rank's full buffers."""
        from . import kernels
        names = list(names)
        if len(names) == 1:
            return [self.matmul(names[0], a, ws[0], scales[0], axis)]
        lead = tuple(a.shape[:-1])
        pos = (self._capi.B2PeerOut * len(names))()
        for i, name in enumerate(names):
            pos[i] = self._peer_out(name)
        src = next((n for n, b in self.bufs.items() if b[0].data_ptr() == a.data_ptr()), None)
        pos[0].wait_input = 1 if src in self._dirty else 0
        if pos[0].wait_input:
            self._dirty.clear()
        self._dirty.update(names)
        ad = self._capi.Desc(a.data_ptr(), self._capi.TORCH_TO_ONNX[a.dtype], tuple(a.shape))
        wd = self._capi.DescArray([kernels._desc(w) for w in ws])
        sd = self._capi.DescArray([kernels._desc(sc) for sc in scales])
        yd = self._capi.DescArray([self._capi.Desc(0, self._capi.TORCH_TO_ONNX[a.dtype],
                                                   lead + (self.bufs[n][2] // self.world,))
                                   for n in names])
        kernels._call_with_workspace(self.lib.b2_dequantize_matmul_group_peer,
                                     (len(names), ad.ref, wd.ref, sd.ref, int(axis), yd.ref,
                                      C.cast(pos, C.POINTER(self._capi.B2PeerOut))),
                                     (self._capi.stream_ptr(a.device),), a.device)
        return [self.bufs[n][0] for n in names]

    def wait(self, device=None):
        """Makes this rank's stream wait until every rank finished the group's
        last sharded call or gather (so the full buffers may be read)."""
        po = self._capi.B2PeerOut()
        for r in range(self.world):
            po.flags[r] = self.flag_ptrs[r]
        po.counters = self.counters
        po.world, po.rank, po.n_full = self.world, self.rank, 0
        self._capi.check(self.lib.b2_peer_wait(C.byref(po), self._capi.stream_ptr(device)))
        self._dirty.clear()

    def gather(self, name: str, local: torch.Tensor) -> torch.Tensor:
        full, peers, n_total = self.bufs[name]
        self._dirty.clear()  # the gather waits for every rank's slice
        d = self._capi.Desc(local.data_ptr(), self._capi.TORCH_TO_ONNX[local.dtype],
                            tuple(local.shape))
        self._capi.check(self.lib.b2_allgather_cols(
            d.ref, peers, self.flag_ptrs, C.c_void_p(self.counters), self.world, self.rank,
            n_total, self._capi.stream_ptr(local.device)))
        return full

    def close(self):
        torch.cuda.synchronize()
        for p in self._opened:
            self.lib.b2_ipc_close(C.c_void_p(p))
        self._opened.clear()
        dist.barrier(group=self.group)  # peers have unmapped before the memory goes
        for p in self._own:
            self.lib.b2_ipc_free(C.c_void_p(p))
        self._own.clear()
        self.bufs.clear()

