"""Expert-parallel exchange on CPU ranks (gloo): each (token, rank) row with
its slot list, in the fixed per-rank slab layout, reaches the rank that owns
those experts, and the partial sums come back to the sender.  Also checks that
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
        ex = ExpertParallelExchange(E)
        El = ex.E_local
        rng = np.random.default_rng(100 + rank)
        idx = np.stack([rng.choice(E, k, replace=False) for _ in range(T)])
        if rank == 0 and T > 3:
            idx[:3] = np.arange(k)  # several tokens on the same experts
        w = torch.rand(T, k)
        x = torch.randn(T, H, generator=torch.Generator().manual_seed(rank))
        # sender slabs (the q35_ep_scatter layout): row d*T + t, slot lists local to d
        dest = idx // El
        send = torch.zeros(world * T, H)
        meta_idx = torch.full((world * T, k), -1, dtype=torch.int32)
        meta_w = torch.zeros(world * T, k)
        ret_pos = torch.full((T, world), -1, dtype=torch.long)
        for t in range(T):
            for j in range(k):
                d = int(dest[t, j])
                send[d * T + t] = x[t]
                meta_idx[d * T + t, j] = int(idx[t, j]) - d * El
                meta_w[d * T + t, j] = w[t, j]
                ret_pos[t, d] = d * T + t
        r_rows, r_idx, r_w = ex.exchange(send), ex.exchange(meta_idx), ex.exchange(meta_w)
        # receiver: "expert e" scales a row by (global e + 1); weighted per slot
        lo, _ = ex.expert_range
        partial = torch.zeros_like(r_rows)
        for u in range(r_rows.shape[0]):
            for j in range(k):
                if int(r_idx[u, j]) >= 0:
                    partial[u] += r_w[u, j] * r_rows[u] * float(lo + int(r_idx[u, j]) + 1)
        back = ex.exchange(partial)
        out = torch.zeros(T, H)
        for t in range(T):
            for d in range(world):
                if ret_pos[t, d] >= 0:
                    out[t] += back[ret_pos[t, d]]
        ref = torch.zeros(T, H)
        for t in range(T):
            for j in range(k):
                ref[t] += w[t, j] * x[t] * float(idx[t, j] + 1)
        assert torch.allclose(out, ref, atol=1e-5), "returned partial sums are wrong"
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
        try:
            ex.exchange(torch.zeros(4, 8))
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


def test_balanced_placement_spreads_skewed_load():
    """Longest-processing-time placement: E/N experts per rank, every expert
    once, the busiest rank within one expert's load of the mean on a
    Zipf-skewed count vector, never worse than the contiguous split."""
    from qwen3_5_vl_cuda_custom_b200.ep import balanced_placement
    E, N = 128, 8
    rng = np.random.default_rng(3)
    pop = 1.0 / np.arange(1, E + 1) ** 1.2
    counts = (pop[rng.permutation(E)] * 1e6).astype(np.int64)
    pl = balanced_placement(counts, N)
    assert sorted(e for r in pl for e in r) == list(range(E))
    assert all(len(r) == E // N for r in pl)
    loads = [int(counts[r].sum()) for r in pl]
    contiguous = [int(counts[i * 16:(i + 1) * 16].sum()) for i in range(N)]
    assert max(loads) - np.mean(loads) <= counts.max()
    assert max(loads) <= max(contiguous)
    assert balanced_placement(counts, N) == pl  # deterministic
