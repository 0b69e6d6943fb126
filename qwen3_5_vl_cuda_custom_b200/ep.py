"""Expert parallelism: token dispatch to the rank that owns each expert, and the
way back, over torch.distributed all-to-all (NCCL over NVLink on GPUs).

Rank r of an N-rank group owns experts [r * E/N, (r + 1) * E/N).  The
single-GPU MoE pipeline already sorts the routed (token, slot) pairs by
(expert, token) and gathers their rows in that order, so the rows bound for
each owner rank are contiguous: they are the send buffer as they stand.

dispatch():
  1. all_to_all of the per-expert row counts (int32, E/N per destination);
     the counts come to the host once to size the row exchange,
  2. all_to_all of the rows (bf16, H per row),
  3. received rows are source-major (rank s, then expert, then token); one row
     gather makes them expert-major (expert, then source rank, then token), the
     layout the grouped GEMM reads, with per-local-expert offsets.
combine():
  the inverse gather back to source-major, then the reverse all_to_all; the
  rows land in the sender's sorted order, where the single-GPU combine kernel
  (weights, residual) consumes them unchanged.

The row gathers are this library's gather kernel on CUDA tensors; the index
bookkeeping (a few small int tensors) is plain torch on the same device.  The
reference has no counterpart: it runs every expert on one GPU
(REF cuda_qwen3_vl/modules/moe.py:71-83).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist

from . import kernels as K
from .modules import CudaSparseMoE


@dataclass
class DispatchState:
    send_splits: list[int]          # rows sent to each rank
    recv_splits: list[int]          # rows received from each rank
    order: torch.Tensor             # expert-major row r <- source-major row order[r]
    inverse: torch.Tensor           # source-major row r <- expert-major row inverse[r]
    local_offsets: torch.Tensor     # int32 [E_local + 1] offsets of the expert-major rows
    local_counts: torch.Tensor      # int32 [E_local]


def _default_gather(src: torch.Tensor, rows: torch.Tensor) -> torch.Tensor:
    if src.is_cuda:
        return K.gather_rows(src, rows.to(torch.int32))
    return src.index_select(0, rows.long())


class ExpertParallelExchange:
    """All-to-all dispatch/combine of expert-sorted rows within ``group``."""

    def __init__(self, num_experts: int, group=None,
                 gather: Callable[[torch.Tensor, torch.Tensor], torch.Tensor] | None = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if num_experts % self.world != 0:
            raise ValueError(f"{num_experts} experts do not split over {self.world} ranks")
        self.E = num_experts
        self.E_local = num_experts // self.world
        self.gather = gather or _default_gather

    @property
    def expert_range(self) -> tuple[int, int]:
        return self.rank * self.E_local, (self.rank + 1) * self.E_local

    def dispatch(self, rows: torch.Tensor, expert_counts: torch.Tensor):
        """rows: [R, H] sorted by (expert, token); expert_counts: int [E] rows per
        expert.  Returns (expert-major received rows [R_recv, H], state)."""
        N, El = self.world, self.E_local
        dev = rows.device
        counts = expert_counts.to(torch.int32).reshape(N, El).contiguous()
        recv_counts = torch.empty_like(counts)
        dist.all_to_all_single(recv_counts, counts, group=self.group)
        both = torch.stack([counts.sum(1), recv_counts.sum(1)]).cpu()
        send_splits = both[0].tolist()
        recv_splits = both[1].tolist()
        recv = rows.new_empty(sum(recv_splits), rows.shape[1])
        dist.all_to_all_single(recv, rows.contiguous(), recv_splits, send_splits, group=self.group)

        # source-major (s, e) blocks -> expert-major (e, s) blocks
        c = recv_counts.to(torch.int64)                          # [N, El]
        src_start = (torch.cumsum(c.reshape(-1), 0) - c.reshape(-1)).reshape(N, El)
        sizes_em = c.t().reshape(-1)                             # (e, s) order
        total = int(sum(recv_splits))
        block_src = src_start.t().reshape(-1)
        dst_start = torch.cumsum(sizes_em, 0) - sizes_em
        ar = torch.arange(total, device=dev, dtype=torch.int64)
        order = (torch.repeat_interleave(block_src, sizes_em, output_size=total)
                 + ar - torch.repeat_interleave(dst_start, sizes_em, output_size=total))
        inverse = torch.empty_like(order)
        inverse[order] = ar
        local_counts = c.sum(0).to(torch.int32)
        local_offsets = torch.zeros(El + 1, device=dev, dtype=torch.int32)
        local_offsets[1:] = torch.cumsum(local_counts, 0)
        em_rows = self.gather(recv, order) if total else recv
        state = DispatchState(send_splits, recv_splits, order.to(torch.int32),
                              inverse.to(torch.int32), local_offsets, local_counts)
        return em_rows, state

    def combine(self, y_expert_major: torch.Tensor, state: DispatchState) -> torch.Tensor:
        """Expert outputs (expert-major, as dispatched) back to the sender's sorted rows."""
        src_major = (self.gather(y_expert_major, state.inverse) if y_expert_major.shape[0]
                     else y_expert_major)
        out = y_expert_major.new_empty(sum(state.send_splits), y_expert_major.shape[1])
        dist.all_to_all_single(out, src_major.contiguous(), state.send_splits, state.recv_splits,
                               group=self.group)
        return out


def _local_permutation(offsets: torch.Tensor, counts: torch.Tensor):
    """A kernels.Permutation over the expert-major received rows (the grouped
    GEMM reads offsets; the 128-row tile prefix is rebuilt for completeness)."""
    tiles = (counts.to(torch.int64) + 127) // 128
    tile_offsets = torch.zeros_like(offsets)
    tile_offsets[1:] = torch.cumsum(tiles, 0).to(torch.int32)
    return K.Permutation(counts, offsets, None, None, tile_offsets, counts.numel())


def make_expert_parallel_moe(hidden_size: int, moe_intermediate_size: int, num_experts: int,
                             top_k: int, norm_topk_prob: bool = True, group=None):
    """CudaSparseMoE whose experts are sharded over ``group`` (see
    ExpertParallelSparseMoE)."""
    return ExpertParallelSparseMoE(hidden_size, moe_intermediate_size, num_experts, top_k,
                                   norm_topk_prob, group=group)


class ExpertParallelSparseMoE(CudaSparseMoE):
    """CudaSparseMoE with its experts sharded over a process group.

    Same constructor arguments plus ``group``; same forward signature and
    outputs.  The router weight is replicated; ``gate_up_proj`` and
    ``down_proj`` hold only this rank's E/N experts ([E/N, 2I, H], [E/N, H, I]).
    ``load_state_dict`` accepts the full-size expert tensors of a reference
    state dict and keeps this rank's slice, so the reference's weight names and
    shapes still load unchanged.  Each rank routes its own tokens; the expert
    rows travel with ExpertParallelExchange.
    """

    def __init__(self, hidden_size: int, moe_intermediate_size: int, num_experts: int, top_k: int,
                 norm_topk_prob: bool = True, group=None):
        super().__init__(hidden_size, moe_intermediate_size, num_experts, top_k, norm_topk_prob)
        self.exchange = ExpertParallelExchange(num_experts, group)
        lo, hi = self.exchange.expert_range
        with torch.no_grad():
            self.gate_up_proj = torch.nn.Parameter(self.gate_up_proj[lo:hi].clone())
            self.down_proj = torch.nn.Parameter(self.down_proj[lo:hi].clone())

    def _load_from_state_dict(self, state_dict, prefix, *args, **kwargs):
        lo, hi = self.exchange.expert_range
        for name in ("gate_up_proj", "down_proj"):
            key = prefix + name
            t = state_dict.get(key)
            if t is not None and t.shape[0] == self.num_experts and hi - lo != self.num_experts:
                state_dict[key] = t[lo:hi]
        super()._load_from_state_dict(state_dict, prefix, *args, **kwargs)

    def experts(self, x2d: torch.Tensor, idx: torch.Tensor, weights: torch.Tensor,
                residual: torch.Tensor | None = None) -> torch.Tensor:
        T, H = x2d.shape
        perm = K.moe_permute(idx, self.num_experts)
        xs = K.gather_rows(x2d, perm.sorted_tok)
        em, st = self.exchange.dispatch(xs, perm.counts)
        local = _local_permutation(st.local_offsets, st.local_counts)
        act = K.grouped_gateup_swiglu(em, self.gate_up_proj, local)
        y_em = K.grouped_down(act, self.down_proj, local)
        y = self.exchange.combine(y_em, st)
        return K.moe_combine(y, weights, perm.slot_pos, residual, T, H)
