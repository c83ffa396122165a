"""Expert parallelism over token-sharded ranks: dispatch -> local experts -> combine.

Reference: the `--ep-size` mode of the reference's server (DeepEP dispatch/combine for V4.1 and GLM,
scripts/local/run-server.sh:89-100): every rank holds its own tokens and `E / world` routed experts;
each (token, expert) pair of a rank's routing is sent to the expert's owner, computed there, and the
result is sent back and summed with the routing weight.  Here the two exchanges are
`torch.distributed.all_to_all_single` (NCCL on GPUs, gloo on CPU ranks): the baseline against which a
fused dispatch / grouped-GEMM / combine kernel is measured.

Within one layer call:
  1. pairs sorted by owner rank (stable, so the order within a rank is the token order), per-owner
     counts exchanged;
  2. hidden rows + local expert ids -> owners (all-to-all);
  3. owner runs its experts on the rows it received (unweighted outputs);
  4. outputs (bf16 by default) -> back to the source ranks (all-to-all), weighted and summed in fp32 per
     token in routing order.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


class EPMoE:
    def __init__(self, num_experts: int, group=None, combine_dtype: torch.dtype = torch.bfloat16):
        """`combine_dtype`: type of the expert outputs sent back (bf16 halves the combine traffic; the
        weighted sum is accumulated in fp32 either way)."""
        self.combine_dtype = combine_dtype
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if num_experts % self.world:
            raise ValueError("routed experts must divide evenly over the EP ranks")
        self.num_experts = num_experts
        self.local_experts = num_experts // self.world
        self.expert_base = self.rank * self.local_experts
        self.last_counts: dict = {}

    def _exchange(self, x: torch.Tensor, out_rows: int, send: list[int], recv: list[int]) -> torch.Tensor:
        out = torch.empty((out_rows,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        if self.world == 1:
            out.copy_(x)
            return out
        dist.all_to_all_single(out, x.contiguous(), output_split_sizes=recv, input_split_sizes=send,
                               group=self.group)
        return out

    def forward(self, h: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor,
                local_fn: Callable[[torch.Tensor, torch.Tensor], torch.Tensor]) -> torch.Tensor:
        """h [T, H] (this rank's tokens), topk_ids / topk_w [T, k] over all experts ->
        fp32 [T, H] = sum_k w_k expert_k(h).  `local_fn(rows, local_expert_ids)` runs this rank's
        experts on received rows and returns their unweighted outputs [R, H]."""
        T, k = topk_ids.shape
        ids = topk_ids.reshape(-1).long()
        owner = ids // self.local_experts
        order = torch.sort(owner, stable=True).indices
        send_counts = torch.bincount(owner, minlength=self.world)
        recv_counts = self._exchange(send_counts, self.world, [1] * self.world, [1] * self.world)
        send, recv = send_counts.tolist(), recv_counts.tolist()
        rows = h[order // k]
        local_ids = ids[order] - owner[order] * self.local_experts
        r_rows = self._exchange(rows, sum(recv), send, recv)
        r_ids = self._exchange(local_ids, sum(recv), send, recv)
        y = local_fn(r_rows, r_ids).to(self.combine_dtype)
        back = self._exchange(y, T * k, recv, send)
        pairs = torch.empty(back.shape, dtype=torch.float32, device=back.device)
        pairs[order] = back.float()
        out = (pairs.view(T, k, -1) * topk_w.float()[..., None]).sum(1)
        self.last_counts = {"sent": send, "received": recv}
        return out


def local_expert_fn(lw: dict, expert_base: int, local_experts: int, expert_format: str,
                    precision: str = "default") -> Callable[[torch.Tensor, torch.Tensor], torch.Tensor]:
    """This rank's experts as `local_fn`: each received row goes through its one expert (weight 1),
    on the same expert kernels as the TP path (CPU: the BF16 reference)."""
    from ..ops import moe as moe_ops

    def run(rows: torch.Tensor, local_ids: torch.Tensor) -> torch.Tensor:
        if rows.shape[0] == 0:
            return torch.zeros(0, rows.shape[1], dtype=torch.float32, device=rows.device)
        ids = (local_ids + expert_base).to(torch.int32)[:, None].contiguous()
        w = torch.ones(rows.shape[0], 1, dtype=torch.float32, device=rows.device)
        return moe_ops.experts(rows.contiguous(), ids, w, lw, expert_base, local_experts, expert_format,
                               precision=precision)

    return run
