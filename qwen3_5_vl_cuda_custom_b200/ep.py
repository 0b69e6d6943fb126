"""Expert parallelism: token dispatch to the ranks that own a token's experts,
and the way back, over torch.distributed all-to-all (NCCL over NVLink on GPUs).

Rank r of an N-rank group owns experts [r * E/N, (r + 1) * E/N).  A token
whose top-k experts sit on several ranks is sent once to each of those ranks
(not once per expert) with a k-slot list of (local expert id, routing weight).
A token sends at most one row to a rank, so every send fits a fixed slab of T
rows per destination: the all-to-alls split evenly and need no host-side
sizes (no host synchronisation; the layer can be captured in a CUDA graph).

Sender:   q35_ep_scatter writes token t's row and slot list into slab d for
          each rank d it uses (slot id -1: not this rank's expert).
Receiver: the N*T received slot lists (-1 = empty slot, unused rows are all
          -1) go through the (expert, token) permutation; the gather, grouped
          gate_up/SwiGLU, grouped down and weighted combine kernels run on
          them unchanged, leaving one bf16 partial sum per received row.
Return:   the reverse all-to-all brings each rank's partial sums back; the
          combine kernel adds a token's partials (weight 1, ret_pos) and its
          residual.

Link traffic is (N-1) * T rows each way per rank whether a slab row is used
or not (at most ~1/(1-(1-1/N)^k) above the rows actually needed: 1.0x at
N = 2, 1.5x at N = 8 with k = 8).  The reference has no counterpart: it runs
every expert on one GPU (REF cuda_qwen3_vl/modules/moe.py:71-83).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import kernels as K
from .modules import CudaSparseMoE


class ExpertParallelExchange:
    """Even-split all-to-all between the ranks of ``group``."""

    def __init__(self, num_experts: int, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if num_experts % self.world != 0:
            raise ValueError(f"{num_experts} experts do not split over {self.world} ranks")
        self.E = num_experts
        self.E_local = num_experts // self.world

    @property
    def expert_range(self) -> tuple[int, int]:
        return self.rank * self.E_local, (self.rank + 1) * self.E_local

    def exchange(self, buf: torch.Tensor) -> torch.Tensor:
        """buf [N * rows, ...]: slab d goes to rank d; returns the N received slabs."""
        out = torch.empty_like(buf)
        dist.all_to_all_single(out, buf.contiguous(), group=self.group)
        return out


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
                residual: torch.Tensor | None = None, mark=None) -> torch.Tensor:
        """``mark(name)`` (optional) is called after each stage (benchmark timing)."""
        mark = mark or (lambda name: None)
        T, H = x2d.shape
        k = idx.shape[1]
        ex = self.exchange
        N, El = ex.world, ex.E_local
        dev = x2d.device
        # ---- sender: slab d holds the rows and slot lists for rank d
        send = torch.empty(N * T, H, device=dev, dtype=x2d.dtype)
        meta_idx = torch.empty(N * T, k, device=dev, dtype=torch.int32)
        meta_w = torch.empty(N * T, k, device=dev, dtype=torch.float32)
        ret_pos = torch.empty(T, N, device=dev, dtype=torch.int32)
        with torch.cuda.device(dev):
            K._lib.call("q35_ep_scatter", x2d.data_ptr(), idx.data_ptr(), weights.data_ptr(), T, k,
                        H, El, N, send.data_ptr(), meta_idx.data_ptr(), meta_w.data_ptr(),
                        ret_pos.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
        r_rows = ex.exchange(send)
        r_idx = ex.exchange(meta_idx)
        r_w = ex.exchange(meta_w)
        mark("ep_dispatch")
        # ---- receiver: local experts over the received slot lists
        R = r_rows.shape[0]
        lperm = K.moe_permute(r_idx, El)
        # only offsets[El] of the R*k slots hold an expert: gather that many
        xs = K.gather_rows(r_rows, lperm.sorted_tok, n_dev=lperm.offsets[El:])
        act = K.grouped_gateup_swiglu(xs, self.gate_up_proj, lperm)
        mark("gate_up_swiglu")
        y = K.grouped_down(act, self.down_proj, lperm)
        mark("down")
        partial = K.moe_combine(y, r_w, lperm.slot_pos, None, R, H)
        # ---- return: partial sums back to the senders, summed with the residual
        back = ex.exchange(partial)
        mark("ep_return")
        ones = torch.ones(T, N, device=dev, dtype=torch.float32)
        return K.moe_combine(back, ones, ret_pos, residual, T, H)
