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
