"""Expert parallelism on 2+ GPUs (NCCL process group): each rank's output of an
expert-parallel decoder layer matches the single-GPU layer on the same input
within the parity tolerance (the expert rows are computed by the same kernels;
only the summation order of a token's experts and one bf16 rounding of each
rank's partial sum differ) and the fp32 CPU oracle re-run with the GPU's
expert choice; the router logits are identical.  Both transports are checked:
peer-memory stores over NVLink ("p2p") and NCCL all-to-all ("nccl"), on a
uniform router and on the config-4 Zipf-skewed router.  Skipped with fewer
than 2 GPUs."""
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
        from oracle import layer_oracle as O
        from qwen3_5_vl_cuda_custom_b200 import synthetic as syn, kernels as K
        from qwen3_5_vl_cuda_custom_b200.configs import tiny_moe_text, a3b_moe_text
        from qwen3_5_vl_cuda_custom_b200.modules import CudaTextDecoderLayer, TextMRoPE
        from qwen3_5_vl_cuda_custom_b200.ep import release_windows
        results = []
        cases = [(tiny_moe_text(), 200, False), (a3b_moe_text(1), 1024, False),
                 (a3b_moe_text(1), 1024, True)]
        for transport in ("p2p", "nccl"):
            for cfg, S, skew in cases:
                g = torch.Generator().manual_seed(5)
                P = syn.layer_params(cfg, g)
                bias = syn.zipf_router_bias(cfg.num_experts, g) if skew else None
                x_cpu = syn.hidden_states((1, S, cfg.hidden_size),
                                          torch.Generator().manual_seed(50 + rank))
                x = x_cpu.cuda().bfloat16()
                pos = syn.text_positions(1, S).cuda()

                def make(group):
                    l = CudaTextDecoderLayer(cfg.hidden_size, cfg.num_heads, cfg.num_kv_heads,
                                             cfg.head_dim, cfg.intermediate_size, cfg.rms_norm_eps,
                                             use_moe=True, num_experts=cfg.num_experts,
                                             top_k=cfg.num_experts_per_tok,
                                             moe_intermediate_size=cfg.moe_intermediate_size,
                                             expert_group=group)
                    if group is not None:
                        l.mlp.transport = transport
                    l.load_state_dict(P)
                    l = l.cuda().bfloat16()
                    if bias is not None:
                        l.mlp.router_bias = bias.cuda()
                    return l

                rot = TextMRoPE(cfg.head_dim, cfg.rope_theta, cfg.mrope_section).cuda()
                ep_layer = make(dist.group.WORLD)
                assert ep_layer.mlp.gate_up_proj.shape[0] == cfg.num_experts // world
                ref_layer = make(None)
                with torch.no_grad():
                    for _ in range(2):  # the second call reuses the exchange window
                        y, rl, _ = ep_layer(x, rot.bind(pos))
                    yr, rlr, _ = ref_layer(x, rot.bind(pos))
                    h = ref_layer.self_attn(ref_layer.input_layernorm(x), rot.bind(pos),
                                            residual=x, out_dtype=torch.float32)[0]
                    m_in = ref_layer.post_attention_layernorm(h).reshape(-1, cfg.hidden_size)
                    gidx = ref_layer.mlp.route(m_in)[1]
                torch.cuda.synchronize()
                K.device_error_check()
                st = O.error_stats(y.float().cpu(), yr.float().cpu())
                ref = O.decoder_layer(x_cpu, P, cfg, syn.text_positions(1, S), router_bias=bias,
                                      force_idx=gidx.cpu())
                so = O.error_stats(y.float().cpu(), ref["out"])
                ok = (bool(torch.equal(rl, rlr)) and st["max_abs_over_bf16"] <= 2e-2
                      and st["mean_rel"] <= 5e-3 and so["max_abs_over_bf16"] <= 2e-2
                      and so["mean_rel"] <= 5e-3)
                results.append((transport, cfg.hidden_size, skew, ok, so["max_abs_over_bf16"]))
        release_windows()
        dist.barrier()
        dist.destroy_process_group()
        bad = [r for r in results if not r[3]]
        q.put((rank, "ok" if not bad else f"mismatch {bad}"))
    except Exception:
        q.put((rank, traceback.format_exc()))


def test_expert_parallel_layer_matches_single_gpu_and_oracle():
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs 2 or more GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=900) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    assert all(v == "ok" for v in res.values()), res
