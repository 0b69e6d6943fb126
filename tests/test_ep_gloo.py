"""Expert-parallel exchange on CPU ranks (gloo): dispatch routes every row to
the rank owning its expert in expert-major order, and combine returns the
expert outputs to the sender in its original sorted order.  Also checks that
a rank that dies before a collective surfaces as an error on the others (a
short process-group timeout), not a hang."""
import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import layer_oracle as O


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=timeout_s))


def _exchange_worker(rank, world, port, E, T, k, H, q):
    try:
        _init(rank, world, port)
        from qwen3_5_vl_cuda_custom_b200.ep import ExpertParallelExchange
        rng = np.random.default_rng(100 + rank)
        idx = np.stack([rng.choice(E, k, replace=False) for _ in range(T)])
        if rank == 0 and T > 3:
            idx[:3] = np.arange(k)  # several tokens on the same experts
        counts, offsets, sorted_tok, slot_pos, _ = O.permutation(idx, E)
        x = torch.randn(T, H, generator=torch.Generator().manual_seed(rank))
        rows = x[torch.from_numpy(sorted_tok).long()]
        ex = ExpertParallelExchange(E)
        em, st = ex.dispatch(rows, torch.from_numpy(counts))
        lo, hi = ex.expert_range
        # expert-major layout: local expert e's rows are contiguous
        offs = st.local_offsets.tolist()
        assert offs[-1] == em.shape[0]
        y = em.clone()
        for e in range(hi - lo):
            y[offs[e]:offs[e + 1]] *= float(lo + e + 1)  # "expert e" = scale by e + 1
        back = ex.combine(y, st)
        expert_of_row = np.repeat(np.arange(E), counts)
        expect = rows * torch.from_numpy(expert_of_row + 1.0).float()[:, None]
        assert torch.allclose(back, expect), "combine did not return the sender's rows"
        # the combine over slot positions equals the per-token weighted sum
        w = torch.rand(T, k)
        out = torch.zeros(T, H)
        sp = torch.from_numpy(slot_pos).long().view(T, k)
        for j in range(k):
            out += w[:, j:j + 1] * back[sp[:, j]]
        ref = torch.zeros(T, H)
        for t in range(T):
            for j in range(k):
                ref[t] += w[t, j] * x[t] * float(idx[t, j] + 1)
        assert torch.allclose(out, ref, atol=1e-5)
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:  # pragma: no cover - reported to the parent
        q.put((rank, traceback.format_exc()))


@pytest.mark.parametrize("world,E,T", [(2, 16, 64), (4, 32, 50), (2, 8, 1)])
def test_ep_dispatch_combine_gloo(world, E, T):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, world, port, E, T, 4, 24, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert all(v == "ok" for v in res.values()), res


def _dying_worker(rank, world, port, q):
    try:
        _init(rank, world, port, timeout_s=5)
        from qwen3_5_vl_cuda_custom_b200.ep import ExpertParallelExchange
        ex = ExpertParallelExchange(8)
        if rank == 1:
            os._exit(3)  # leaves between steps, before the exchange
        rows = torch.randn(4, 8)
        try:
            ex.dispatch(rows, torch.tensor([1, 1, 1, 1, 0, 0, 0, 0]))
            q.put((rank, "no error"))
        except Exception as e:  # the surviving rank must see an error, not hang
            q.put((rank, f"error: {type(e).__name__}"))
    except Exception:
        q.put((rank, traceback.format_exc()))


def test_rank_failure_is_reported_not_hung():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    rank, msg = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert rank == 0 and msg.startswith("error"), msg
