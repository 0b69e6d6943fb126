"""Expert parallelism: token dispatch to the ranks that own a token's experts,
and the way back.

Rank r of an N-rank group owns experts [r * E/N, (r + 1) * E/N).  A token
whose top-k experts sit on several ranks is sent once to each of those ranks
(not once per expert) with a k-slot list of (local expert id, routing weight).

Two transports, same results:

* ``"p2p"`` (default on GPUs that can map each other's memory): every rank
  holds an exchange window in its own memory, mapped into all ranks with
  CUDA IPC.  ``q35_ep_dispatch`` stores each token row straight into the
  owner ranks' windows over NVLink (only the rows in use, compacted per
  source), ``q35_ep_return`` stores each received row's weighted partial sum
  straight back into the sender's window, and bounded flag waits order the
  two sides (csrc/ep_p2p.cu).  No collective library runs on the data path,
  so nothing competes with the expert GEMMs for SMs and no host
  synchronisation is needed: the layer is captured in a CUDA graph.
* ``"nccl"``: fixed slabs of T rows per destination exchanged with
  ``all_to_all_single`` (even splits, graph-capturable).  Used for the gloo
  CPU tests' host logic and wherever peer mapping is unavailable.

Receiver: the received slot lists (-1 = another rank's expert) go through the
(expert, token) permutation; the gather, grouped gate_up/SwiGLU, grouped down
kernels run on them unchanged, leaving one bf16 partial sum per received row.
The sender's combine kernel adds a token's partials (rank order) to its
residual.  The reference has no counterpart: it runs every expert on one GPU
(REF cuda_qwen3_vl/modules/moe.py:71-83).
"""
from __future__ import annotations

import ctypes
import os
import warnings

import torch
import torch.distributed as dist

from . import _lib
from . import kernels as K
from .modules import CudaSparseMoE

# bounded flag waits of the peer-memory exchange (a missing rank becomes a
# device error, never a hang)
WAIT_LIMIT_NS = int(float(os.environ.get("Q35_EP_WAIT_MS", "5000")) * 1e6)


class _DeviceArray:
    """A raw device allocation exposed through __cuda_array_interface__, so that
    torch.as_tensor views it without a copy."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3,
                                         "strides": None}


def _view(ptr: int, shape: tuple, dtype: torch.dtype, device) -> torch.Tensor:
    typestr = {torch.int32: "<i4", torch.float32: "<f4", torch.bfloat16: "<i2"}[dtype]
    t = torch.as_tensor(_DeviceArray(ptr, shape, typestr), device=device)
    return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t


class PeerWindow:
    """The exchange windows of one process group, mapped into this rank.

    Collective to create (every rank of ``group`` must construct it with the
    same N, Tcap, H, k).  Tensors returned by the accessors are views of the
    window and live as long as this object."""

    _OFFS = ("rows", "ret", "idx", "wts", "tok", "cnt", "flags", "ctrl", "peers", "total")

    def __init__(self, group, device, N: int, rank: int, Tcap: int, H: int, k: int):
        self.N, self.rank, self.Tcap, self.H, self.k = N, rank, Tcap, H, k
        self.device = device
        offs = (ctypes.c_int64 * 10)()
        _lib.call("q35_ep_window_offsets", N, Tcap, H, k, offs)
        self.off = dict(zip(self._OFFS, list(offs)))
        self.ptr = None
        self.opened: list[int] = []
        with torch.cuda.device(device):
            p = ctypes.c_void_p()
            _lib.call("q35_ep_window_alloc", N, Tcap, H, k, ctypes.byref(p))
            self.ptr = p.value
            h = (ctypes.c_uint8 * 64)()
            _lib.call("q35_ep_ipc_handle", self.ptr, h)
            mine = torch.tensor(list(h), dtype=torch.uint8, device=device)
            allh = torch.empty(N * 64, dtype=torch.uint8, device=device)
            dist.all_gather_into_tensor(allh, mine, group=group)
            allh = allh.cpu().reshape(N, 64)
            bases, failure = [], None
            for d in range(N):
                if d == rank:
                    bases.append(self.ptr)
                    continue
                hb = (ctypes.c_uint8 * 64)(*allh[d].tolist())
                q = ctypes.c_void_p()
                try:
                    _lib.call("q35_ep_ipc_open", hb, ctypes.byref(q))
                except RuntimeError as e:
                    failure = e
                    break
                self.opened.append(q.value)
                bases.append(q.value)
            # every rank must agree before any kernel stores into a peer
            ok = torch.tensor([0 if failure else 1], dtype=torch.int32, device=device)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
            if not bool(ok.item()):
                self.close()
                raise RuntimeError(f"ep_window: peer mapping failed on some rank ({failure})")
            arr = (ctypes.c_uint64 * N)(*bases)
            _lib.call("q35_ep_set_peers", self.ptr, N, Tcap, H, k, arr)
        dist.barrier(group=group)
        R = N * Tcap
        self.rows = _view(self.ptr + self.off["rows"], (R, H), torch.bfloat16, device)
        self.ret = _view(self.ptr + self.off["ret"], (R, H), torch.bfloat16, device)
        self.idx = _view(self.ptr + self.off["idx"], (R, k), torch.int32, device)
        self.cnt = _view(self.ptr + self.off["cnt"], (N,), torch.int32, device)

    def close(self):
        for q in self.opened:
            try:
                _lib.call("q35_ep_ipc_close", q)
            except RuntimeError:
                pass
        self.opened = []
        if self.ptr is not None:
            try:
                _lib.call("q35_ep_window_free", self.ptr)
            except RuntimeError:
                pass
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_WINDOWS: dict = {}


def _window_for(group, device, N, rank, T, H, k, max_tokens):
    """The shared PeerWindow of (group, device, H, k), created on first use with
    a capacity of ``max_tokens`` (or the largest T over the ranks, agreed with
    one all-reduce).  All MoE layers of a model share it: their calls are
    ordered on the stream."""
    key = (id(group), str(device), H, k)
    win = _WINDOWS.get(key)
    if win is not None:
        if T > win.Tcap:
            raise RuntimeError(f"expert-parallel window holds {win.Tcap} tokens per rank, "
                               f"got {T}: construct the layer with a larger ep_max_tokens")
        return win
    cap = max_tokens or T
    t = torch.tensor([cap], dtype=torch.int64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    win = PeerWindow(group, device, N, rank, int(t.item()), H, k)
    _WINDOWS[key] = win
    return win


def release_windows():
    """Unmaps and frees every exchange window of this process (call on all
    ranks together, after the last expert-parallel forward has finished)."""
    torch.cuda.synchronize()
    for w in list(_WINDOWS.values()):
        w.close()
    _WINDOWS.clear()


class ExpertParallelExchange:
    """Rank bookkeeping of the expert-parallel group and the even-split
    all-to-all of the ``nccl`` transport."""

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


def balanced_placement(counts, world: int) -> list[list[int]]:
    """Experts per rank with equal numbers of experts (E/N) and near-equal
    expected load: longest-processing-time assignment of the experts, heaviest
    first, each to the least-loaded rank that still has room (ties to the lower
    rank and expert id; deterministic).  ``counts`` [E]: tokens routed to each
    expert on a calibration batch (all ranks' tokens)."""
    c = [int(v) for v in (counts.tolist() if hasattr(counts, "tolist") else counts)]
    E = len(c)
    if E % world:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    cap = E // world
    order = sorted(range(E), key=lambda e: (-c[e], e))
    load = [0] * world
    out: list[list[int]] = [[] for _ in range(world)]
    for e in order:
        r = min((r for r in range(world) if len(out[r]) < cap), key=lambda r: (load[r], r))
        out[r].append(e)
        load[r] += c[e]
    return [sorted(x) for x in out]


def _default_transport(group) -> str:
    if dist.get_backend(group) != "nccl" or not torch.cuda.is_available():
        return "nccl"
    return os.environ.get("Q35_EP_TRANSPORT", "p2p")


class ExpertParallelSparseMoE(CudaSparseMoE):
    """CudaSparseMoE with its experts sharded over a process group.

    Same constructor arguments plus ``group``, ``transport`` ("p2p" or
    "nccl"; default p2p on NCCL groups, overridable with Q35_EP_TRANSPORT) and
    ``ep_max_tokens`` (tokens per rank the p2p window holds; default: the
    first call's largest T over the ranks) and ``expert_placement`` (None: rank
    r owns experts [r*E/N, (r+1)*E/N) as in a plain split; else N lists of E/N
    global expert ids per rank, e.g. from ``balanced_placement``, so that a
    skewed router does not load some ranks more than others; p2p transport).
    Same forward signature and outputs.  The router weight is replicated; ``gate_up_proj`` and
    ``down_proj`` hold only this rank's E/N experts ([E/N, 2I, H], [E/N, H, I]).
    ``load_state_dict`` accepts the full-size expert tensors of a reference
    state dict and keeps this rank's slice, so the reference's weight names and
    shapes still load unchanged.  Each rank routes its own tokens.  Every rank
    of the group must run the same sequence of forwards (the exchange is
    collective).
    """

    def __init__(self, hidden_size: int, moe_intermediate_size: int, num_experts: int, top_k: int,
                 norm_topk_prob: bool = True, group=None, transport: str | None = None,
                 ep_max_tokens: int | None = None, expert_placement=None):
        super().__init__(hidden_size, moe_intermediate_size, num_experts, top_k, norm_topk_prob)
        self.exchange = ExpertParallelExchange(num_experts, group)
        self.transport = transport or _default_transport(group)
        if self.transport not in ("p2p", "nccl"):
            raise ValueError(f"unknown expert-parallel transport {self.transport!r}")
        self.ep_max_tokens = ep_max_tokens
        N, El, rank = self.exchange.world, self.exchange.E_local, self.exchange.rank
        if expert_placement is None:
            self.local_experts = list(range(rank * El, (rank + 1) * El))
            self._owner_cpu = None
        else:
            pl = [list(map(int, x)) for x in expert_placement]
            if len(pl) != N or sorted(e for x in pl for e in x) != list(range(num_experts)) \
                    or any(len(x) != El for x in pl):
                raise ValueError("expert_placement: N lists of E/N distinct expert ids covering all experts")
            if self.transport != "p2p":
                raise ValueError("expert_placement needs the p2p transport")
            self.local_experts = pl[rank]
            owner = torch.empty(num_experts, dtype=torch.int32)
            for r, x in enumerate(pl):
                for j, e in enumerate(x):
                    owner[e] = (r << 16) | j
            self._owner_cpu = owner
        self.expert_placement = expert_placement
        self._owner = None
        sel = torch.tensor(self.local_experts)
        with torch.no_grad():
            self.gate_up_proj = torch.nn.Parameter(self.gate_up_proj[sel].clone())
            self.down_proj = torch.nn.Parameter(self.down_proj[sel].clone())
        self._ones = None

    def _owner_table(self, device):
        """Device table (rank << 16 | local slot) per expert, or None (plain split)."""
        if self._owner_cpu is None:
            return None
        if self._owner is None or self._owner.device != device:
            self._owner = self._owner_cpu.to(device)
        return self._owner

    def _load_from_state_dict(self, state_dict, prefix, *args, **kwargs):
        sel = torch.tensor(self.local_experts)
        for name in ("gate_up_proj", "down_proj"):
            key = prefix + name
            t = state_dict.get(key)
            if t is not None and t.shape[0] == self.num_experts and len(sel) != self.num_experts:
                state_dict[key] = t[sel.to(t.device)]
        super()._load_from_state_dict(state_dict, prefix, *args, **kwargs)

    # ------------------------------------------------------------ p2p transport
    def _ones_like(self, T: int, N: int, device) -> torch.Tensor:
        if self._ones is None or self._ones.shape[0] < T or self._ones.device != device:
            self._ones = torch.ones(T, N, device=device, dtype=torch.float32)
        return self._ones[:T]

    def p2p_stages(self):
        """The peer-memory expert path as (name, fn(state)) stages, in order:
        ``ep_dispatch`` (rows into the owners' windows, wait for every rank's
        rows), ``ep_experts`` (permutation, gather, grouped GEMMs on the
        received slabs), ``ep_return`` (partials into the senders' windows,
        wait for every rank's partials), ``ep_combine`` (partials + residual).
        ``state`` holds x2d, idx, weights and residual on entry and ``out`` on
        exit.  ``experts`` runs them back to back; the benchmark times them
        one by one."""
        ex = self.exchange
        N, El, rank = ex.world, ex.E_local, ex.rank

        def dispatch(st):
            x2d, idx, w = st["x2d"], st["idx"], st["weights"]
            T, H = x2d.shape
            k = idx.shape[1]
            dev = x2d.device
            win = _window_for(ex.group, dev, N, rank, T, H, k, self.ep_max_tokens)
            stream = torch.cuda.current_stream(dev).cuda_stream
            ret_pos = torch.empty(T, N, device=dev, dtype=torch.int32)
            owner = self._owner_table(dev)
            with torch.cuda.device(dev):
                _lib.call("q35_ep_dispatch", x2d.data_ptr(), idx.data_ptr(), w.data_ptr(), T, k, H,
                          El, N, rank, win.Tcap, None if owner is None else owner.data_ptr(),
                          win.ptr, ret_pos.data_ptr(), stream)
                _lib.call("q35_ep_wait", win.ptr, N, win.Tcap, H, k, 0, WAIT_LIMIT_NS, stream)
            st["win"], st["ret_pos"] = win, ret_pos

        def experts(st):
            win = st["win"]
            lperm = K.moe_permute_slabs(win.idx, N, win.Tcap, win.cnt, El)
            # only offsets[El] of the N*Tcap*k slots hold an expert of this rank
            xs = K.gather_rows(win.rows, lperm.sorted_tok, n_dev=lperm.offsets[El:])
            act = K.grouped_gateup_swiglu(xs, self.gate_up_proj, lperm)
            st["y"] = K.grouped_down(act, self.down_proj, lperm)
            st["slot_pos"] = lperm.slot_pos

        def ret(st):
            win, y = st["win"], st["y"]
            H, k, Tc = win.H, win.k, win.Tcap
            dev = y.device
            stream = torch.cuda.current_stream(dev).cuda_stream
            with torch.cuda.device(dev):
                _lib.call("q35_ep_return", y.data_ptr(), st["slot_pos"].data_ptr(), Tc, k, H, N, rank,
                          win.ptr, stream)
                _lib.call("q35_ep_wait", win.ptr, N, Tc, H, k, 1, WAIT_LIMIT_NS, stream)

        def combine(st):
            T, H = st["x2d"].shape
            dev = st["x2d"].device
            st["out"] = K.moe_combine(st["win"].ret, self._ones_like(T, N, dev), st["ret_pos"],
                                      st["residual"], T, H)

        return [("ep_dispatch", dispatch), ("ep_experts", experts), ("ep_return", ret),
                ("ep_combine", combine)]

    def _experts_p2p(self, x2d, idx, weights, residual):
        st = {"x2d": x2d, "idx": idx, "weights": weights, "residual": residual}
        for _, fn in self.p2p_stages():
            fn(st)
        return st["out"]

    # ------------------------------------------------------------ nccl transport
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

    def _experts_nccl(self, x2d, idx, weights, residual):
        """Tokens are processed in ``ep_chunks`` chunks: all dispatches are issued
        first (asynchronous all-to-alls on the communicator's stream), then each
        chunk's experts run as soon as its rows arrive and its return is issued
        right after, so chunk c+1's dispatch and chunk c's return overlap the
        expert GEMMs of the other chunk."""
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
        use_limit = chunks > 1 and self.ep_sm_reserve and x2d.is_cuda
        if use_limit:
            n_sms = torch.cuda.get_device_properties(x2d.device).multi_processor_count
            K._lib.call("q35_set_sm_limit", max(2, n_sms - self.ep_sm_reserve))
        try:
            for r_rows, r_meta, w1, w2 in inflight:
                w1.wait()
                w2.wait()
                partial = self._chunk_experts(r_rows, r_meta)
                back = torch.empty_like(partial)
                returns.append((back, dist.all_to_all_single(back, partial, group=grp,
                                                             async_op=True)))
        finally:
            if use_limit:
                K._lib.call("q35_set_sm_limit", 0)
        out = torch.empty(T, H, device=x2d.device, dtype=torch.bfloat16)
        ones = torch.ones(max(bounds[1] - bounds[0], 1), N, device=x2d.device, dtype=torch.float32)
        for (a, b), (_, _, ret_pos), (back, work) in zip(zip(bounds[:-1], bounds[1:]), sends, returns):
            work.wait()
            res = None if residual is None else residual[a:b]
            K.moe_combine(back, ones[: b - a], ret_pos, res, b - a, H, out=out[a:b])
        return out

    def experts(self, x2d: torch.Tensor, idx: torch.Tensor, weights: torch.Tensor,
                residual: torch.Tensor | None = None, chunk_counts=None) -> torch.Tensor:
        """Expert compute for routed tokens across the group: (T,H) -> (T,H),
        the weighted combine plus ``residual`` (if given) included.
        ``chunk_counts`` is accepted for signature compatibility and unused:
        the receiving ranks permute what they receive."""
        if self.transport == "p2p":
            try:
                return self._experts_p2p(x2d, idx.contiguous(), weights.contiguous(), residual)
            except RuntimeError as e:
                if "ep_ipc" not in str(e) and "ep_window" not in str(e):
                    raise
                warnings.warn(f"peer-memory exchange unavailable ({e}); using NCCL all-to-all")
                self.transport = "nccl"
        return self._experts_nccl(x2d, idx, weights, residual)
