"""KV-head sharding of the decode path across GPUs (one process per GPU).

GPU r of N owns KV heads [r*K/N, (r+1)*K/N) of every layer and the query
heads that attend to them (q head h uses KV head h // G, sf37_cuda.cu:2544),
i.e. the contiguous slice [r*Q/N, (r+1)*Q/N).  Each rank decodes its slice
with no data exchange; the per-head outputs are all-gathered once per step
for all layers.  The gathered tensor is [N][layers][Q/N][d]; the per-layer
[Q][d] order is its (1, 0, 2, 3) permutation.
"""
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class ShardPlan:
    world: int
    rank: int
    kv_heads: int = 8
    q_heads: int = 64
    head_dim: int = 128

    def __post_init__(self):
        if self.kv_heads % self.world or self.q_heads % self.kv_heads:
            raise ValueError(f"{self.world} ranks cannot split {self.kv_heads} KV heads evenly")

    @property
    def kv_local(self) -> int:
        return self.kv_heads // self.world

    @property
    def q_local(self) -> int:
        return self.q_heads // self.world

    @property
    def kv_range(self):
        return self.rank * self.kv_local, (self.rank + 1) * self.kv_local

    @property
    def q_range(self):
        return self.rank * self.q_local, (self.rank + 1) * self.q_local

    def slice_rows(self, rows: torch.Tensor) -> torch.Tensor:
        """This rank's head slice of full K/V rows [..., kv_heads*head_dim]."""
        a, b = self.kv_range
        return rows[..., a * self.head_dim:b * self.head_dim]

    def slice_q(self, q: torch.Tensor) -> torch.Tensor:
        """This rank's query heads of q [..., q_heads, head_dim]."""
        a, b = self.q_range
        return q[..., a:b, :]


def gather_outputs(out_local: torch.Tensor, plan: ShardPlan, group=None, gathered=None):
    """All-gathers [layers, Q/N, d] per rank into [layers, Q, d]."""
    if plan.world == 1:
        return out_local
    if gathered is None:
        gathered = torch.empty((plan.world,) + tuple(out_local.shape), dtype=out_local.dtype,
                               device=out_local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(gathered, out_local.contiguous(), group=group)
    else:
        dist.all_gather(list(gathered.unbind(0)), out_local.contiguous(), group=group)
    return gathered.permute(1, 0, 2, 3).reshape(out_local.shape[0], plan.q_heads, out_local.shape[-1])


class _CudaArray:
    """__cuda_array_interface__ wrapper so torch can view library memory."""

    def __init__(self, ptr, shape, typestr="<f4"):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 2}


class _PeerBuffer:
    """One zero-filled device buffer per rank (sf37kv_dev_alloc): `floats`
    f32 of payload, then the ranks' epoch flags and a done counter; mapped
    into every other rank by CUDA IPC.  `struct` is the sf37kv_peer_gather
    descriptor the library calls take."""

    def __init__(self, world, rank, floats, group=None):
        import ctypes
        from ._lib import PeerGather as PG, lib
        L = lib()
        self._lib = L
        self.world, self.rank = world, rank
        self.off_flags = (floats * 4 + 255) // 256 * 256
        self.off_done = self.off_flags + 256
        self.base = L.sf37kv_dev_alloc(self.off_done + 256)
        if not self.base:
            raise RuntimeError("sf37kv_dev_alloc failed")
        h = ctypes.create_string_buffer(64)
        if L.sf37kv_ipc_handle(self.base, h):
            raise RuntimeError("sf37kv_ipc_handle failed")
        torch.cuda.synchronize()
        handles = [None] * world
        dist.all_gather_object(handles, bytes(h.raw), group=group)
        self.peers = []
        st = PG()
        for p in range(world):
            if p == rank:
                ptr = self.base
            else:
                ptr = L.sf37kv_ipc_open(ctypes.create_string_buffer(handles[p], 64))
                if not ptr:
                    raise RuntimeError(f"sf37kv_ipc_open of rank {p} failed")
                self.peers.append(ptr)
            st.peer_buf[p] = ptr
            st.peer_flags[p] = ptr + self.off_flags
        st.my_flags = self.base + self.off_flags
        st.done_counter = self.base + self.off_done
        st.world, st.rank = world, rank
        self.struct = st
        self.epoch = 0
        dist.barrier(group=group)

    def view(self, shape):
        return torch.as_tensor(_CudaArray(self.base, shape), device="cuda")

    def close(self):
        for p in self.peers:
            self._lib.sf37kv_ipc_close(p)
        self.peers = []
        if self.base:
            self._lib.sf37kv_dev_free(self.base)
            self.base = None


class PeerGather(_PeerBuffer):
    """Output gather over peer memory for sf37kv_decode_gather (see
    include/sf37kv.h): [2][world][n_layers][q_local][head_dim] f32 outputs,
    the half selected by the step's epoch parity."""

    def __init__(self, plan: ShardPlan, n_layers: int, group=None):
        self.plan, self.n_layers = plan, n_layers
        super().__init__(plan.world, plan.rank, 2 * plan.world * n_layers * plan.q_local * plan.head_dim, group)
        self.gathered = self.view((2, plan.world, n_layers, plan.q_local, plan.head_dim))

    def heads(self) -> torch.Tensor:
        """[n_layers, q_heads, head_dim] outputs of the last completed step
        (valid on the stream after step(); a copy, since the half is reused
        two steps later)."""
        g = self.gathered[self.epoch & 1]
        return g.permute(1, 0, 2, 3).reshape(self.n_layers, self.plan.q_heads, self.plan.head_dim)

    def step(self, descs, dtype, stream=None):
        """Decode this rank's slice, store outputs into every rank, wait for all."""
        import ctypes
        from ._lib import check
        from .kv import decode_layers_desc
        if isinstance(descs, list):
            descs = decode_layers_desc(descs)
        if len(descs) != self.n_layers:
            raise ValueError(f"PeerGather was set up for {self.n_layers} layers, got {len(descs)}")
        self.epoch += 1
        sp = None if stream is None else ctypes.c_void_p(stream.cuda_stream)
        check(self._lib.sf37kv_decode_gather(descs, len(descs), self.plan.q_local, self.plan.kv_local,
                                             self.plan.head_dim, dtype, ctypes.byref(self.struct),
                                             self.epoch, sp), "sf37kv_decode_gather")
        check(self._lib.sf37kv_gather_wait(ctypes.byref(self.struct), self.epoch, sp), "sf37kv_gather_wait")


class PeerReduce(_PeerBuffer):
    """Row-parallel o_proj (sf37kv_oproj_q8_0_shard + sf37kv_oproj_reduce):
    each rank multiplies its heads' columns and the partial [n_layers][out_dim]
    vectors are summed across ranks over peer memory."""

    def __init__(self, world, rank, n_layers, out_dim, group=None):
        self.n_layers, self.out_dim = n_layers, out_dim
        super().__init__(world, rank, 2 * world * n_layers * out_dim, group)

    @staticmethod
    def weight_slice(w_rows: torch.Tensor, world: int, rank: int):
        """(pointer offset in bytes, row stride) of rank's column slice of
        Q8_0 rows w_rows [out_dim][in_dim/32*34]."""
        row_bytes = w_rows.shape[-1]
        return rank * row_bytes // world, row_bytes

    def step(self, layers, in_dim_local, row_stride, out, stream=None):
        """layers: ctypes OprojLayer array (x = this rank's heads, weights =
        its column slice); out: [n_layers][out_dim] f32, the summed result."""
        import ctypes
        from ._lib import check
        self.epoch += 1
        sp = None if stream is None else ctypes.c_void_p(stream.cuda_stream)
        check(self._lib.sf37kv_oproj_q8_0_shard(layers, len(layers), in_dim_local, self.out_dim, row_stride,
                                                ctypes.byref(self.struct), self.epoch, sp),
              "sf37kv_oproj_q8_0_shard")
        check(self._lib.sf37kv_oproj_reduce(ctypes.byref(self.struct), self.n_layers, self.out_dim, self.epoch,
                                            out.data_ptr(), sp), "sf37kv_oproj_reduce")
