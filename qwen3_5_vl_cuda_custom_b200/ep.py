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

    ep_chunks = 2  # token chunks whose exchange overlaps the other chunk's experts
    ep_sm_reserve = 32  # SMs left to the collectives while the expert GEMMs run

    def _chunk_send(self, x2d, idx, w):
        """Send slabs of one token chunk: rows [N*Tc, H] and slot lists packed as
        [N, 2, Tc, k] int32 (expert ids, then the weights' bits)."""
        Tc, H = x2d.shape
        k = idx.shape[1]
        N, El = self.exchange.world, self.exchange.E_local
        dev = x2d.device
        send = torch.empty(N * Tc, H, device=dev, dtype=x2d.dtype)
        meta = torch.empty(N, 2, Tc, k, device=dev, dtype=torch.int32)
        ret_pos = torch.empty(Tc, N, device=dev, dtype=torch.int32)
        with torch.cuda.device(dev):
            K._lib.call("q35_ep_scatter", x2d.data_ptr(), idx.data_ptr(), w.data_ptr(), Tc, k, H, El, N,
                        send.data_ptr(), meta.data_ptr(), meta[:, 1].data_ptr(), 2 * Tc * k,
                        ret_pos.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
        return send, meta, ret_pos

    def _chunk_experts(self, r_rows, r_meta):
        """Local experts over one chunk's received slot lists -> bf16 partial sums."""
        N, El = self.exchange.world, self.exchange.E_local
        R, H = r_rows.shape
        r_idx = r_meta[:, 0].reshape(R, -1).contiguous()
        r_w = r_meta[:, 1].reshape(R, -1).contiguous().view(torch.float32)
        lperm = K.moe_permute(r_idx, El)
        # only offsets[El] of the R*k slots hold an expert: gather that many
        xs = K.gather_rows(r_rows, lperm.sorted_tok, n_dev=lperm.offsets[El:])
        act = K.grouped_gateup_swiglu(xs, self.gate_up_proj, lperm)
        y = K.grouped_down(act, self.down_proj, lperm)
        return K.moe_combine(y, r_w, lperm.slot_pos, None, R, H)

    def _run_chunks(self, inflight, returns, grp, mark):
        for c, (r_rows, r_meta, w1, w2) in enumerate(inflight):
            w1.wait()
            w2.wait()
            if c == 0:
                mark("ep_dispatch")
            partial = self._chunk_experts(r_rows, r_meta)
            if c == 0:
                mark("experts_chunk0")
            back = torch.empty_like(partial)
            returns.append((back, dist.all_to_all_single(back, partial, group=grp, async_op=True)))

    def experts(self, x2d: torch.Tensor, idx: torch.Tensor, weights: torch.Tensor,
                residual: torch.Tensor | None = None, mark=None) -> torch.Tensor:
        """``mark(name)`` (optional) is called after each stage (benchmark timing).

        Tokens are processed in ``ep_chunks`` chunks: all dispatches are issued
        first (asynchronous all-to-alls on the communicator's stream), then each
        chunk's experts run as soon as its rows arrive and its return is issued
        right after, so chunk c+1's dispatch and chunk c's return overlap the
        expert GEMMs of the other chunk."""
        mark = mark or (lambda name: None)
        T, H = x2d.shape
        N = self.exchange.world
        grp = self.exchange.group
        # NCCL's copy kernels share SMs and HBM with the expert GEMMs: overlap
        # only pays where the exchange is large relative to the experts (N >= 4)
        chunks = self.ep_chunks if (T >= 256 * self.ep_chunks and N >= 4) else 1
        bounds = [T * c // chunks for c in range(chunks + 1)]
        sends = [self._chunk_send(x2d[a:b], idx[a:b].contiguous(), weights[a:b].contiguous())
                 for a, b in zip(bounds[:-1], bounds[1:])]
        inflight = []
        for send, meta, _ in sends:
            r_rows, r_meta = torch.empty_like(send), torch.empty_like(meta)
            w1 = dist.all_to_all_single(r_rows, send, group=grp, async_op=True)
            w2 = dist.all_to_all_single(r_meta, meta, group=grp, async_op=True)
            inflight.append((r_rows, r_meta, w1, w2))
        returns = []
        n_sms = torch.cuda.get_device_properties(x2d.device).multi_processor_count
        if chunks > 1 and self.ep_sm_reserve:
            K._lib.call("q35_set_sm_limit", max(2, n_sms - self.ep_sm_reserve))
        try:
            self._run_chunks(inflight, returns, grp, mark)
        finally:
            K._lib.call("q35_set_sm_limit", 0)
        out = torch.empty(T, H, device=x2d.device, dtype=torch.bfloat16)

        ones = torch.ones(max(bounds[1] - bounds[0], 1), N, device=x2d.device, dtype=torch.float32)
        for (a, b), (_, _, ret_pos), (back, work) in zip(zip(bounds[:-1], bounds[1:]), sends, returns):
            work.wait()
            res = None if residual is None else residual[a:b]
            K.moe_combine(back, ones[: b - a], ret_pos, res, b - a, H, out=out[a:b])
        mark("ep_return")
        return out
