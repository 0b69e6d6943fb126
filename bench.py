"""Benchmark: Qwen3-VL-MoE decoder-layer prefill tokens/s on B200.

Workload: one 30B-A3B-shaped MoE decoder layer
(hidden 2048, 32/4 heads x 128, QK-norm, 128 experts top-8, intermediate 768,
mRoPE [24,20,20] theta 5e6), bf16 weights + fp32 router, prefill of
1 x 4096 tokens per GPU, causal, seed 1, random-init weights and N(0,1)
inputs (synthetic: no checkpoint or dataset).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  python bench.py --workload c3   # informational: decode over a KV cache (config 3)

``value`` times the forward replayed from a CUDA graph of the module call
(qwen3_5_vl_cuda_custom_b200.graphs.GraphedDecoderLayer); the eager module
call is reported beside it.

One process per GPU (torchrun for N > 1).  Each rank prefills its own
4096-token sequence (attention data-parallel over sequences) and the experts
are sharded expert-parallel, 128/N per GPU, with NCCL all-to-all dispatch and
return (qwen3_5_vl_cuda_custom_b200.ep); per-GPU work is fixed ("scaling":
"weak").
A step is one layer forward; the L2 is flushed (256 MiB write) between
steps outside the timed events.  ``value`` is whole-job tokens/s from
per-step CUDA events (max over ranks); ``e2e`` re-times the same step through
the public module API with the input copied from pinned host memory and the
output copied back inside the timed region.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

# DRAM bytes (read + write) per launch from `ncu --set full` captures of the C2
# workload (profiles/grouped_gemm_pair_c2_full.md, profiles/attention_tc2_c2_full.md)
TRAFFIC_BYTES_C2 = {"gate_up_swiglu": 1055.5e6, "down": 575.9e6, "attention": 42.9e6}
# algorithmic bytes of the same launches (weights + rows read, outputs written)
ALGO_BYTES_C2 = {"gate_up_swiglu": 989.8e6, "down": 587.2e6, "attention": 75.5e6}
LINK_GBS = 770.0  # measured NVLink peer copy per direction on this pool
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return PEAKS_FALLBACK, "fallback"


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def wait_first(self, timeout: float = 5.0):
        t0 = time.time()
        while not self.lines and time.time() - t0 < timeout and self.proc is not None:
            time.sleep(0.05)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- workload
def build_layer(cfg, seed: int, device, expert_group=None):
    from qwen3_5_vl_cuda_custom_b200 import synthetic as syn
    from qwen3_5_vl_cuda_custom_b200.modules import CudaTextDecoderLayer, TextMRoPE
    g = torch.Generator().manual_seed(seed)
    P = syn.layer_params(cfg, g)
    layer = CudaTextDecoderLayer(cfg.hidden_size, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim,
                                 cfg.intermediate_size, cfg.rms_norm_eps, use_moe=True,
                                 num_experts=cfg.num_experts, top_k=cfg.num_experts_per_tok,
                                 moe_intermediate_size=cfg.moe_intermediate_size,
                                 expert_group=expert_group)
    layer.load_state_dict(P)  # expert-parallel layers keep their slice of the experts
    layer = layer.to(device, torch.bfloat16)
    rot = TextMRoPE(cfg.head_dim, cfg.rope_theta, cfg.mrope_section).to(device)
    return layer, rot, P, g


def stage_table(cfg, T: int, S: int, world: int = 1) -> dict:
    """Algorithmic work per stage: (bound, amount) with FLOPs or bytes."""
    H, D, Hq, Hkv = cfg.hidden_size, cfg.head_dim, cfg.num_heads, cfg.num_kv_heads
    E, k, I = cfg.num_experts, cfg.num_experts_per_tok, cfg.moe_intermediate_size
    B = T // S
    return {
        "input_rmsnorm": ("hbm", 2 * T * H * 2),
        "qkv_gemm": ("tensor", 2 * T * H * (Hq + 2 * Hkv) * D),
        "qknorm_mrope": ("hbm", T * (Hq + 2 * Hkv) * D * 2 * 2),
        "qkv_norm_rope": ("tensor", 2 * T * H * (Hq + 2 * Hkv) * D),
        "attention": ("tensor", B * Hq * 4 * D * S * (S + 1) / 2),
        "o_proj_residual": ("tensor", 2 * T * Hq * D * H),
        "post_rmsnorm": ("hbm", 2 * T * H * 2),
        "router": ("hbm", T * H * 2 + T * E * 4 + T * k * 8),
        "permute": ("hbm", T * k * 4 * 3),
        "gather": ("hbm", T * H * 2 + T * k * H * 2),
        "gate_up_swiglu": ("tensor", T * k * 2 * H * 2 * I),
        "down": ("tensor", T * k * 2 * I * H),
        "combine_residual": ("hbm", T * k * H * 2 + 2 * T * H * 2 + T * k * 4),
        # expert parallelism: one row per (token, destination rank), each
        # direction; expected ranks per token N(1 - (1 - 1/N)^k), N = world
        "ep_dispatch": ("link", T * H * 2 * world * (1 - (1 - 1 / world) ** k)),
        "experts_chunk0": ("tensor", T * k * 2 * 3 * H * I / 2),
        "ep_return": ("link", T * H * 2 * world * (1 - (1 - 1 / world) ** k)),
    }


def staged_forward(layer, rot, x, pos, marks=None):
    """The decoder-layer forward (the same kernel sequence as the module path),
    with an optional CUDA event recorded after each stage."""
    from qwen3_5_vl_cuda_custom_b200 import kernels as K
    att, moe = layer.self_attn, layer.mlp
    B, S, H = x.shape

    def mark(name):
        if marks is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            marks.append((name, ev))

    mark("start")
    xn = K.rmsnorm(x, layer.input_layernorm.weight, layer.input_layernorm.eps)
    mark("input_rmsnorm")
    w, _ = att._qkv_weight()
    if att.fuse_qkv_epilogue and att.head_dim == 128 and B * S >= 256:
        q, k, v = K.qkv_proj_norm_rope(xn, w, att.q_norm.weight, att.k_norm.weight, pos,
                                       rot.inv_freq, rot.mrope_section, att.num_heads,
                                       att.num_kv_heads, att.q_norm.eps)
        mark("qkv_norm_rope")
    else:
        qkv = K.matmul(xn, w)
        mark("qkv_gemm")
        q, k, v = K.qknorm_mrope(qkv, att.q_norm.weight, att.k_norm.weight, pos, rot.inv_freq,
                                 rot.mrope_section, B, S, att.num_heads, att.num_kv_heads,
                                 att.head_dim, att.q_norm.eps)
        mark("qknorm_mrope")
    o = K.attention_tokens(q, k, v, att.scale, True)
    mark("attention")
    h = K.matmul(o, att.o_proj.weight, residual=x, out_dtype=torch.float32)
    mark("o_proj_residual")
    m_in = K.rmsnorm(h, layer.post_attention_layernorm.weight, layer.post_attention_layernorm.eps)
    mark("post_rmsnorm")
    m2 = m_in.reshape(-1, H)
    logits, idx, wts = moe.route(m2)
    mark("router")
    if getattr(moe, "exchange", None) is not None:  # expert parallel
        out = moe.experts(m2, idx, wts, h.reshape(-1, H), mark=mark)
        mark("combine_residual")
        return out.reshape(B, S, H)
    perm = K.moe_permute(idx, moe.num_experts)
    mark("permute")
    xs = K.gather_rows(m2, perm.sorted_tok)
    mark("gather")
    gu_p, dn_p = moe._packed_experts()
    act = K.grouped_gateup_swiglu(xs, moe.gate_up_proj, perm, w_packed=gu_p)
    mark("gate_up_swiglu")
    y = K.grouped_down(act, moe.down_proj, perm, w_packed=dn_p)
    mark("down")
    out = K.moe_combine(y, wts, perm.slot_pos, h.reshape(-1, H), B * S, H)
    mark("combine_residual")
    return out.reshape(B, S, H)


LAUNCHES_PER_LAYER = 16  # rmsnorm, rope table, qkv+norm+rope, attn, o, rmsnorm, router logits,
# router top-k, permute x3 (count, scan, scatter), gather, gate_up, down, combine


def cpu_reference_step_fn(cfg, P, x_cpu, pos_cpu, dtype):
    """The reference's own CudaTextDecoderLayer (baseline/_ref) on CPU tensors,
    or None when the reference is not installed."""
    ref_dir = ROOT / "baseline" / "_ref"
    if not (ref_dir / "cuda_qwen3_vl").exists():
        return None
    os.environ.setdefault("CUDA_QWEN3_VL_AUTO_PRELOAD", "0")
    sys.path.insert(0, str(ref_dir))
    from cuda_qwen3_vl.modules import CudaTextDecoderLayer, TextMRoPE
    layer = CudaTextDecoderLayer(cfg.hidden_size, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim,
                                 cfg.intermediate_size, cfg.rms_norm_eps, use_moe=True,
                                 num_experts=cfg.num_experts, top_k=cfg.num_experts_per_tok,
                                 moe_intermediate_size=cfg.moe_intermediate_size)
    layer.load_state_dict(P)
    layer = layer.to(dtype)
    rot = TextMRoPE(cfg.head_dim, theta=cfg.rope_theta, mrope_section=cfg.mrope_section)
    xr = x_cpu.to(dtype)

    def step():
        with torch.no_grad():
            return layer(xr, lambda q, k: rot.apply(q, k, pos_cpu))[0]
    return step


def time_cpu(step, warmup: int, steps: int) -> list[float]:
    for _ in range(warmup):
        step()
    ts = []
    for _ in range(steps):
        t0 = time.perf_counter()
        step()
        ts.append(time.perf_counter() - t0)
    return ts


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
        dist.init_process_group(backend=backend)
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def allreduce_max(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def run_reference(args, world, rank):
    """--impl reference: the reference's own CPU path on the host cores, rank 0 only."""
    from qwen3_5_vl_cuda_custom_b200 import synthetic as syn
    from qwen3_5_vl_cuda_custom_b200.configs import a3b_moe_text
    if rank != 0:
        return
    cfg = a3b_moe_text(1)
    S = args.tokens
    g = torch.Generator().manual_seed(1)
    P = syn.layer_params(cfg, g)
    x = syn.hidden_states((1, S, cfg.hidden_size), g)
    pos = syn.text_positions(1, S)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    step = cpu_reference_step_fn(cfg, P, x, pos, torch.bfloat16)
    kind = "reference"
    if step is None:
        print(json.dumps({"impl": "reference", "unavailable":
                          "reference package not installed under baseline/_ref"}))
        return
    ts = time_cpu(step, max(1, min(args.warmup, 2)), max(1, args.steps))
    t = statistics.median(ts)
    value = S / t
    line = {
        "impl": "reference", "metric": "moe_layer_prefill_tokens_per_s", "value": value,
        "unit": "tokens/s", "n_gpus": args.gpus, "steps": len(ts), "warmup": args.warmup,
        "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "C2 30B-A3B MoE decoder layer prefill, 1x4096 tokens",
                   "tokens_per_step": S, "device": "cpu"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": kind,
                         "sample": f"full step: one layer over {S} tokens, bf16, median of {len(ts)}"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, world, rank, local):
    from qwen3_5_vl_cuda_custom_b200 import build, kernels as K
    from qwen3_5_vl_cuda_custom_b200 import synthetic as syn
    from qwen3_5_vl_cuda_custom_b200.configs import a3b_moe_text
    build.build()
    dev = torch.device("cuda", local)
    cfg = a3b_moe_text(1)
    S = args.tokens
    T = S
    ep_group = None
    if world > 1:
        import torch.distributed as dist
        ep_group = dist.group.WORLD
    layer, rot, P, g = build_layer(cfg, 1, dev, ep_group)
    if world > 1:  # each rank prefills its own sequence
        g = torch.Generator().manual_seed(1000 + rank)
    x_cpu = syn.hidden_states((1, S, cfg.hidden_size), g)
    x = x_cpu.to(dev, torch.bfloat16)
    pos_cpu = syn.text_positions(1, S)
    pos = pos_cpu.to(dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, device=dev, dtype=torch.float32)
    bpos = rot.bind(pos)

    with torch.no_grad(), ClockSampler(local) as clk:
        clk.wait_first()
        # ---------------- warm-up (the library is AOT-built: no JIT here)
        for _ in range(max(3, args.warmup)):
            layer(x, bpos)
        barrier(world)
        # ---------------- device-timed steps: eager module calls, then the
        # same forward replayed from a CUDA graph (GraphedDecoderLayer)
        from qwen3_5_vl_cuda_custom_b200.graphs import GraphedDecoderLayer

        def timed(step_fn):
            times = []
            barrier(world)
            for _ in range(args.steps):
                flush.zero_()
                s0 = torch.cuda.Event(enable_timing=True)
                s1 = torch.cuda.Event(enable_timing=True)
                s0.record()
                step_fn()
                s1.record()
                times.append((s0, s1))
            barrier(world)
            return allreduce_max(sum(a.elapsed_time(b) for a, b in times), world)

        eager_ms = timed(lambda: layer(x, bpos))

        # ---------------- per-stage breakdown (same kernels, events between)
        samples: dict[str, list[float]] = {}
        for _ in range(7):
            flush.zero_()
            marks = []
            staged_forward(layer, rot, x, pos, marks)
            torch.cuda.synchronize()
            for (_, a), (name, b) in zip(marks[:-1], marks[1:]):
                samples.setdefault(name, []).append(a.elapsed_time(b))
        stage_ms = {k: statistics.median(v) for k, v in samples.items()}

        graphed = None
        try:
            graphed = GraphedDecoderLayer(layer, rot, x, pos)
            total_ms = timed(graphed.replay)
        except Exception as e:  # capture unsupported here: report the eager time
            print(f"graph capture failed ({type(e).__name__}: {e}); eager timing", file=sys.stderr)
            graphed = None
            total_ms = eager_ms
        mode = "CUDA-graph replay" if graphed is not None else "eager"
        if graphed is not None and total_ms > eager_ms:
            total_ms, mode = eager_ms, "eager"  # the faster of the two module paths
        ms_per_step = total_ms / args.steps
        value = world * T * args.steps / (total_ms / 1e3)
        eager_value = world * T * args.steps / (eager_ms / 1e3)

        # ---------------- end to end through the public API: each step copies its
        # input from pinned host memory and its output back.  One GPU: the
        # StreamedLayerRunner overlaps the copies with neighbouring replays.
        x_host = x_cpu.to(torch.bfloat16).pin_memory()
        out_host = torch.empty_like(x_host).pin_memory()
        if graphed is not None:
            from qwen3_5_vl_cuda_custom_b200.graphs import StreamedLayerRunner
            runner = StreamedLayerRunner(graphed)
            run_e2e = lambda n: runner.run(x_host, out_host, n)  # noqa: E731
        else:
            def run_e2e(n):
                for _ in range(n):
                    y, _, _ = layer(x_host.to(dev, non_blocking=True), bpos)
                    out_host.copy_(y, non_blocking=True)
        run_e2e(2)
        barrier(world)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        run_e2e(args.steps)
        e1.record()
        barrier(world)
        e2e_ms = allreduce_max(e0.elapsed_time(e1), world)
        e2e_value = world * T * args.steps / (e2e_ms / 1e3)

    K.device_error_check()

    peaks, peak_src = load_peaks()
    table = stage_table(cfg, T, S, world)
    top = max(stage_ms, key=stage_ms.get)
    bound, amount = table[top]
    t_top = stage_ms[top] / 1e3
    if bound == "tensor":
        achieved = amount / t_top / 1e12
        peak = peaks["bf16_tflops"]
        unit = "TFLOP/s"
    elif bound == "link":
        achieved = amount * (world - 1) / world / t_top / 1e9
        peak = LINK_GBS
        unit = "GB/s"
    else:
        achieved = amount / t_top / 1e9
        peak = peaks["hbm_gbs"]
        unit = "GB/s"
    breakdown = {}
    for name, ms in stage_ms.items():
        b, a = table[name]
        if b == "link":
            a = a * (world - 1) / world
        rate = a / (ms / 1e3) / (1e12 if b == "tensor" else 1e9)
        pk = {"tensor": peaks["bf16_tflops"], "link": LINK_GBS}.get(b, peaks["hbm_gbs"])
        breakdown[name] = {"ms": round(ms, 4), "bound": b,
                           "achieved": round(rate, 1), "frac": round(rate / pk, 3)}

    if rank != 0:
        return
    cpu = None
    if not args.no_cpu_baseline and world == 1:
        threads = os.cpu_count() or 1
        torch.set_num_threads(threads)
        step = cpu_reference_step_fn(cfg, P, x_cpu, pos_cpu, torch.bfloat16)
        kind, sample = "reference", f"reference CudaTextDecoderLayer on CPU, bf16, {S} tokens, median of 2 after 1 warm-up"
        if step is None:
            from oracle import layer_oracle as O
            kind, sample = "port", f"oracle fp32 layer on CPU, {S} tokens"

            def step():
                return O.decoder_layer(x_cpu, P, cfg, pos_cpu)["out"]
        ts = time_cpu(step, 1, 2)
        cpu = {"value": S / statistics.median(ts), "unit": "tokens/s", "cores": threads,
               "kind": kind, "sample": sample}
    clocks = clk.summary()
    in_bytes = x_host.numel() * 2
    line = {
        "metric": "moe_layer_prefill_tokens_per_s", "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": max(3, args.warmup),
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "C2 30B-A3B MoE decoder layer prefill, 1x4096 tokens per GPU",
                   "hidden": cfg.hidden_size, "heads": f"{cfg.num_heads}/{cfg.num_kv_heads}x{cfg.head_dim}",
                   "experts": f"{cfg.num_experts} top-{cfg.num_experts_per_tok} I={cfg.moe_intermediate_size}",
                   "tokens_per_gpu": T, "global_batch": world, "seq_len": S,
                   "parallelism": (f"ep{world}: {cfg.num_experts // world} experts/GPU, NCCL "
                                   f"all-to-all; dp{world} attention over sequences"
                                   if world > 1 else "1 GPU, all experts local"),
                   "mode": mode,
                   "l2": "256 MiB flush between timed steps"},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": in_bytes,
                "d2h_bytes_per_step": in_bytes,
                "api": "StreamedLayerRunner(GraphedDecoderLayer)"},
        "eager": {"value": eager_value, "ms_per_step": eager_ms / args.steps,
                  "note": "same layer through the module API without graph replay"},
        "gpu_launches": LAUNCHES_PER_LAYER * args.steps,
        "roofline": {"bound": bound, "kernel": top, "achieved": achieved, "peak": peak, "unit": unit,
                     "frac": achieved / peak,
                     "traffic": TRAFFIC_BYTES_C2.get(top) if S == 4096 else None,
                     "algorithmic": amount,
                     "algorithmic_bytes": ALGO_BYTES_C2.get(top) if S == 4096 else None,
                     # the kernel's own lower bound max(FLOPs / tensor peak, bytes / HBM peak)
                     # over its measured time (a weight-streaming GEMM can be either)
                     "frac_of_bound": (max(amount / (peaks["bf16_tflops"] * 1e12) if bound == "tensor" else 0.0,
                                           (ALGO_BYTES_C2.get(top) or 0.0) / (peaks["hbm_gbs"] * 1e9))
                                       / t_top) if S == 4096 else None,
                     "peak_source": peak_src},
        "breakdown": breakdown,
        "cpu_baseline": cpu,
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


def run_c3(args, local):
    """Config 3 (decode): 64 sequences x 1 new token over an 8192-position KV
    history, one decoder layer, KV in a preallocated LayerKVCache.  Prints one
    JSON line (decode tokens/s, HBM roofline of the step's bytes)."""
    from qwen3_5_vl_cuda_custom_b200 import build
    from qwen3_5_vl_cuda_custom_b200 import synthetic as syn
    from qwen3_5_vl_cuda_custom_b200.configs import a3b_moe_text
    from qwen3_5_vl_cuda_custom_b200.kv_cache import LayerKVCache
    build.build()
    dev = torch.device("cuda", local)
    cfg = a3b_moe_text(1)
    B, past = 64, 8192
    layer, rot, P, g = build_layer(cfg, 2, dev)
    cache = LayerKVCache(B, cfg.num_kv_heads, past + 1, cfg.head_dim, dev)
    gen = torch.Generator(device=dev).manual_seed(2)
    cache.k[:, :, :past].normal_(generator=gen)
    cache.v[:, :, :past].normal_(generator=gen)
    x = syn.hidden_states((B, 1, cfg.hidden_size), g).to(dev, torch.bfloat16)
    pos = torch.full((3, B, 1), past, dtype=torch.int64, device=dev)
    bpos = rot.bind(pos)
    flush = torch.empty(256 * 1024 * 1024 // 4, device=dev, dtype=torch.float32)

    def step():
        cache.length = past  # every step appends position `past` and attends 8193 keys
        return layer(x, bpos, past_kv=cache)

    def timed(fn):
        ms = 0.0
        for _ in range(args.steps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            b.synchronize()
            ms += a.elapsed_time(b)
        return ms / args.steps

    with torch.no_grad(), ClockSampler(local) as clk:
        clk.wait_first()
        for _ in range(max(3, args.warmup)):
            step()
        eager_ms = timed(step)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            step()
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        graph_ms = timed(graph.replay)
    clocks = clk.summary()
    ms = min(eager_ms, graph_ms)
    peaks, peak_src = load_peaks()
    E, k = cfg.num_experts, cfg.num_experts_per_tok
    experts = E * (1 - (1 - 1 / E) ** (B * k))  # expected distinct experts touched
    per_expert = 3 * cfg.moe_intermediate_size * cfg.hidden_size * 2
    kv_bytes = 2 * B * cfg.num_kv_heads * (past + 1) * cfg.head_dim * 2
    attn_w = (cfg.hidden_size * (cfg.num_heads + 2 * cfg.num_kv_heads) * cfg.head_dim
              + cfg.num_heads * cfg.head_dim * cfg.hidden_size) * 2
    hbm = kv_bytes + experts * per_expert + attn_w
    achieved = hbm / (ms / 1e3) / 1e9
    line = {
        "metric": "moe_layer_decode_tokens_per_s", "value": B / (ms / 1e3), "unit": "tokens/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "C3 decode: 64 sequences x 1 token, 8192-position KV history, "
                               "one 30B-A3B MoE decoder layer", "kv_cache": "LayerKVCache, in place",
                   "mode": "CUDA-graph replay" if graph_ms <= eager_ms else "eager",
                   "l2": "256 MiB flush between timed steps"},
        "eager_ms": eager_ms, "graph_ms": graph_ms,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "algorithmic_bytes": hbm,
                     "kv_bytes": kv_bytes, "expert_bytes": experts * per_expert,
                     "peak_source": peak_src},
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["c2", "c3"], default="c2",
                    help="c2: the headline prefill layer (default); c3: decode over a KV cache "
                         "(one GPU, informational line)")
    args = ap.parse_args()
    if args.workload == "c3":
        run_c3(args, int(os.environ.get("LOCAL_RANK", "0")))
        return
    world, rank, local = dist_setup(args.gpus)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
