"""Expert parallelism on 2+ GPUs (NCCL): each rank's output of an
expert-parallel decoder layer matches the single-GPU layer on the same input
within the parity tolerance (the expert rows are computed by the same kernels;
only the summation order of a token's experts and one bf16 rounding of each
rank's partial sum differ), and the router logits are identical.  Skipped
with fewer than 2 GPUs."""
import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        import torch.distributed as dist
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=timedelta(seconds=120))
        from qwen3_5_vl_cuda_custom_b200 import synthetic as syn
        from qwen3_5_vl_cuda_custom_b200.configs import tiny_moe_text, a3b_moe_text
        from qwen3_5_vl_cuda_custom_b200.modules import CudaTextDecoderLayer, TextMRoPE
        results = []
        for cfg, S in ((tiny_moe_text(), 200), (a3b_moe_text(1), 1024)):
            g = torch.Generator().manual_seed(5)
            P = syn.layer_params(cfg, g)
            x = syn.hidden_states((1, S, cfg.hidden_size),
                                  torch.Generator().manual_seed(50 + rank)).cuda().bfloat16()
            pos = syn.text_positions(1, S).cuda()

            def make(group):
                l = CudaTextDecoderLayer(cfg.hidden_size, cfg.num_heads, cfg.num_kv_heads,
                                         cfg.head_dim, cfg.intermediate_size, cfg.rms_norm_eps,
                                         use_moe=True, num_experts=cfg.num_experts,
                                         top_k=cfg.num_experts_per_tok,
                                         moe_intermediate_size=cfg.moe_intermediate_size,
                                         expert_group=group)
                l.load_state_dict(P)
                return l.cuda().bfloat16()

            rot = TextMRoPE(cfg.head_dim, cfg.rope_theta, cfg.mrope_section).cuda()
            ep_layer = make(dist.group.WORLD)
            assert ep_layer.mlp.gate_up_proj.shape[0] == cfg.num_experts // world
            ref_layer = make(None)
            with torch.no_grad():
                y, rl, _ = ep_layer(x, rot.bind(pos))
                yr, rlr, _ = ref_layer(x, rot.bind(pos))
            torch.cuda.synchronize()
            from oracle import layer_oracle as O
            st = O.error_stats(y.float().cpu(), yr.float().cpu())
            results.append(bool(torch.equal(rl, rlr)) and st["max_abs_over_bf16"] <= 2e-2
                           and st["mean_rel"] <= 5e-3)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok" if all(results) else f"mismatch {results}"))
    except Exception:
        q.put((rank, traceback.format_exc()))


def test_expert_parallel_layer_matches_single_gpu():
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs 2 or more GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    assert all(v == "ok" for v in res.values()), res
