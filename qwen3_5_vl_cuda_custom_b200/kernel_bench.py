"""Per-kernel timing of the decoder layer's kernels on config-2-shaped inputs.

    python -m qwen3_5_vl_cuda_custom_b200.kernel_bench [--kernel NAME ...]
        [--tokens 4096] [--iters 20] [--flush]

Builds the inputs of one 30B-A3B MoE layer prefill (hidden 2048, 32/4 heads
x 128, 128 experts top-8, intermediate 768) for ``--tokens`` tokens from a
seeded generator -- the routing comes from the real router on those inputs --
and times each selected kernel with CUDA events on the current stream (median
of ``--iters``; ``--flush`` writes 256 MiB between launches so every launch
reads from HBM).  One JSON line per kernel: the time, the algorithmic bytes
or FLOPs of one launch, and the achieved rate.  Meant for profiling one
kernel at a time, e.g. ``ncu -k regex:gemm_pair -s 5 -c 1 python -m
qwen3_5_vl_cuda_custom_b200.kernel_bench --kernel down --iters 3``.

Kernels: rmsnorm_bf16, rmsnorm_f32in, qkv_norm_rope, attention, o_proj,
router, permute, gather, gate_up, down, combine.
"""
from __future__ import annotations

import argparse
import json
import statistics

import torch

from . import build, kernels as K
from . import synthetic as syn
from .configs import a3b_moe_text

KERNELS = ("rmsnorm_bf16", "rmsnorm_f32in", "qkv_norm_rope", "attention", "o_proj", "router",
           "permute", "gather", "gate_up", "down", "combine")


def _route(moe, m2):
    """(logits, idx, weights, chunk_counts or None) through the module's router."""
    out = moe.route(m2, chunk_counts=True) if _route.counted else moe.route(m2)
    return out if len(out) == 4 else (*out, None)


def _permute(idx, cc, E):
    if cc is not None:
        return K.moe_permute_counted(idx, cc, E)
    return K.moe_permute(idx, E)


def make_case(T: int, seed: int = 1):
    """Device tensors of one layer's intermediate values for T tokens (one sequence)."""
    import inspect
    from .modules import CudaSparseMoE, CudaTextDecoderLayer, TextMRoPE
    _route.counted = "chunk_counts" in inspect.signature(CudaSparseMoE.route).parameters
    cfg = a3b_moe_text(1)
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(seed)
    P = syn.layer_params(cfg, g)
    layer = CudaTextDecoderLayer(cfg.hidden_size, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim,
                                 cfg.intermediate_size, cfg.rms_norm_eps, use_moe=True,
                                 num_experts=cfg.num_experts, top_k=cfg.num_experts_per_tok,
                                 moe_intermediate_size=cfg.moe_intermediate_size)
    layer.load_state_dict(P)
    layer = layer.to(dev, torch.bfloat16)
    rot = TextMRoPE(cfg.head_dim, cfg.rope_theta, cfg.mrope_section).to(dev)
    x = syn.hidden_states((1, T, cfg.hidden_size), g).to(dev, torch.bfloat16)
    pos = syn.text_positions(1, T).to(dev)
    att, moe = layer.self_attn, layer.mlp
    c = {"cfg": cfg, "layer": layer, "rot": rot, "x": x, "pos": pos}
    with torch.no_grad():
        c["xn"] = K.rmsnorm(x, layer.input_layernorm.weight)
        c["w_qkv"] = att._qkv_weight()[0]
        c["q"], c["k"], c["v"] = K.qkv_proj_norm_rope(
            c["xn"], c["w_qkv"], att.q_norm.weight, att.k_norm.weight, pos, rot.inv_freq,
            rot.mrope_section, cfg.num_heads, cfg.num_kv_heads, cfg.rms_norm_eps)
        c["o"] = K.attention_tokens(c["q"], c["k"], c["v"], att.scale, True)
        c["h"] = K.matmul(c["o"], att.o_proj.weight, residual=x, out_dtype=torch.float32)
        c["m2"] = K.rmsnorm(c["h"], layer.post_attention_layernorm.weight).reshape(T, -1)
        c["logits"], c["idx"], c["w"], c["cc"] = _route(moe, c["m2"])
        c["perm"] = _permute(c["idx"], c["cc"], cfg.num_experts)
        c["xs"] = K.gather_rows(c["m2"], c["perm"].sorted_tok)
        c["act"] = K.grouped_gateup_swiglu(c["xs"], moe.gate_up_proj, c["perm"])
        c["y"] = K.grouped_down(c["act"], moe.down_proj, c["perm"])
    torch.cuda.synchronize()
    return c


def kernel_fn(name: str, c: dict):
    """(callable launching the kernel once, algorithmic amount, 'bytes'|'flops')."""
    cfg, layer = c["cfg"], c["layer"]
    att, moe = layer.self_attn, layer.mlp
    T, H = c["m2"].shape
    D, Hq, Hkv = cfg.head_dim, cfg.num_heads, cfg.num_kv_heads
    E, k, I = cfg.num_experts, cfg.num_experts_per_tok, cfg.moe_intermediate_size
    rot, pos = c["rot"], c["pos"]
    table = {
        "rmsnorm_bf16": (lambda: K.rmsnorm(c["x"], layer.input_layernorm.weight),
                         2 * T * H * 2, "bytes"),
        "rmsnorm_f32in": (lambda: K.rmsnorm(c["h"], layer.post_attention_layernorm.weight),
                          T * H * 4 + T * H * 2, "bytes"),
        "qkv_norm_rope": (lambda: K.qkv_proj_norm_rope(
            c["xn"], c["w_qkv"], att.q_norm.weight, att.k_norm.weight, pos, rot.inv_freq,
            rot.mrope_section, Hq, Hkv, cfg.rms_norm_eps), 2 * T * H * (Hq + 2 * Hkv) * D, "flops"),
        "attention": (lambda: K.attention_tokens(c["q"], c["k"], c["v"], att.scale, True),
                      Hq * 4 * D * T * (T + 1) / 2, "flops"),
        "o_proj": (lambda: K.matmul(c["o"], att.o_proj.weight, residual=c["x"],
                                    out_dtype=torch.float32), 2 * T * Hq * D * H, "flops"),
        "router": (lambda: _route(moe, c["m2"]), T * H * 2 + T * E * 4 + T * k * 8, "bytes"),
        "permute": (lambda: _permute(c["idx"], c["cc"], E), T * k * 4 * 3, "bytes"),
        "gather": (lambda: K.gather_rows(c["m2"], c["perm"].sorted_tok),
                   T * H * 2 + T * k * H * 2, "bytes"),
        "gate_up": (lambda: K.grouped_gateup_swiglu(c["xs"], moe.gate_up_proj, c["perm"]),
                    T * k * 2 * H * 2 * I, "flops"),
        "down": (lambda: K.grouped_down(c["act"], moe.down_proj, c["perm"]), T * k * 2 * I * H,
                 "flops"),
        "combine": (lambda: K.moe_combine(c["y"], c["w"], c["perm"].slot_pos, c["h"], T, H),
                    T * k * H * 2 + T * H * 4 + T * H * 2 + T * k * 4, "bytes"),
    }
    if name not in table:
        raise ValueError(f"unknown kernel {name}")
    return table[name]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", nargs="*", default=list(KERNELS))
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--flush", action="store_true")
    args = ap.parse_args()
    build.build()
    c = make_case(args.tokens)
    flush = torch.empty(64 << 20, device="cuda", dtype=torch.float32) if args.flush else None
    for name in args.kernel:
        fn, amount, kind = kernel_fn(name, c)
        with torch.no_grad():
            fn()
            fn()
            ts = []
            for _ in range(args.iters):
                if flush is not None:
                    flush.zero_()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                fn()
                b.record()
                ts.append((a, b))
            torch.cuda.synchronize()
        ms = statistics.median(a.elapsed_time(b) for a, b in ts)
        rate = amount / (ms / 1e3) / (1e12 if kind == "flops" else 1e9)
        print(json.dumps({"kernel": name, "tokens": args.tokens, "ms": round(ms, 4),
                          "algorithmic": amount, "unit": "TFLOP/s" if kind == "flops" else "GB/s",
                          "achieved": round(rate, 1), "l2_flush": bool(args.flush)}), flush=True)
    K.device_error_check()


if __name__ == "__main__":
    main()
