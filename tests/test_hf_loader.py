"""Hugging Face checkpoint loading (CPU): key renames, expert transposes,
vision keys skipped, expert-parallel ranks reading only their experts.  The
name mapping is pinned to the reference's own loader when its package is
installed beside the repository (REF loaders/hf.py:21-109)."""
import os
import socket
import sys
import traceback
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def _tiny_cfg():
    from qwen3_5_vl_cuda_custom_b200.configs import MoETextConfig, moe_config
    t = MoETextConfig(hidden_size=64, intermediate_size=128, num_layers=2, num_heads=4,
                      num_kv_heads=2, head_dim=16, vocab_size=96, rope_theta=1e4,
                      mrope_section=[4, 2, 2], num_experts=8, num_experts_per_tok=2,
                      moe_intermediate_size=32)
    return moe_config(t)


def _to_hf(name: str, t: torch.Tensor) -> tuple[str, torch.Tensor]:
    """Internal name/layout -> the HF Qwen3-VL-MoE on-disk name/layout."""
    if name == "lm_head.weight":
        return name, t
    hf = "model.language_model." + name
    if name.endswith("mlp.gate_up_proj") or name.endswith("mlp.down_proj"):
        hf = hf.replace("mlp.gate_up_proj", "mlp.experts.gate_up_proj")
        hf = hf.replace("mlp.down_proj", "mlp.experts.down_proj")
        t = t.transpose(1, 2)
    hf = hf.replace("mlp.gate_weight", "mlp.gate.weight")
    return hf, t.contiguous()


def _write_checkpoint(path: Path, seed: int = 0) -> dict:
    from safetensors.torch import save_file
    from qwen3_5_vl_cuda_custom_b200.models import CudaQwen3VLMoeModel
    torch.manual_seed(seed)
    src = CudaQwen3VLMoeModel(_tiny_cfg(), vision=False)
    ref = {k: torch.randn_like(v) for k, v in src.state_dict().items()}
    hf = dict(_to_hf(k, v) for k, v in ref.items())
    hf["model.visual.blocks.0.norm1.weight"] = torch.ones(8)
    hf["something.else"] = torch.zeros(2)
    keys = sorted(hf)
    save_file({k: hf[k] for k in keys[: len(keys) // 2]}, str(path / "model-00001.safetensors"))
    save_file({k: hf[k] for k in keys[len(keys) // 2:]}, str(path / "model-00002.safetensors"))
    return ref


def test_load_hf_checkpoint_round_trip(tmp_path):
    from qwen3_5_vl_cuda_custom_b200.loaders import load_hf_weights
    from qwen3_5_vl_cuda_custom_b200.models import CudaQwen3VLMoeModel
    ref = _write_checkpoint(tmp_path)
    model = CudaQwen3VLMoeModel(_tiny_cfg(), vision=False)
    report = load_hf_weights(model, tmp_path)
    assert report["missing"] == [] and report["mismatched"] == []
    assert report["unexpected"] == ["something.else"]
    assert report["skipped"] == ["model.visual.blocks.0.norm1.weight"]
    got = model.state_dict()
    for k, v in ref.items():
        assert torch.equal(got[k], v.to(got[k].dtype)), k
    assert model.layers[0].mlp.gate_weight.dtype == torch.float32


def test_name_mapping_matches_reference_loader():
    ref_dir = ROOT / "baseline" / "_ref"
    if not (ref_dir / "cuda_qwen3_vl").exists():
        pytest.skip("reference package not installed beside the repository")
    os.environ.setdefault("CUDA_QWEN3_VL_AUTO_PRELOAD", "0")
    sys.path.insert(0, str(ref_dir))
    try:
        from cuda_qwen3_vl.loaders import hf as ref_hf
    except Exception as e:  # pragma: no cover - depends on the install
        pytest.skip(f"reference loader not importable: {e}")
    finally:
        sys.path.remove(str(ref_dir))
    from qwen3_5_vl_cuda_custom_b200.loaders import map_hf_name
    from qwen3_5_vl_cuda_custom_b200.models import CudaQwen3VLMoeModel
    model = CudaQwen3VLMoeModel(_tiny_cfg(), vision=False)
    for name, t in model.state_dict().items():
        hf, _ = _to_hf(name, t)
        assert map_hf_name(hf) == ref_hf._map_name(hf) == name
        assert ref_hf._needs_expert_transpose(hf) == (t.dim() == 3)


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ep_worker(rank, world, port, path, q):
    try:
        import torch.distributed as dist
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from qwen3_5_vl_cuda_custom_b200.loaders import load_hf_weights
        from qwen3_5_vl_cuda_custom_b200.models import CudaQwen3VLMoeModel
        model = CudaQwen3VLMoeModel(_tiny_cfg(), expert_group=dist.group.WORLD, vision=False)
        report = load_hf_weights(model, path)
        ref = torch.load(Path(path) / "ref.pt")
        lo, hi = model.layers[0].mlp.exchange.expert_range
        ok = report["missing"] == [] and report["mismatched"] == []
        for i in range(2):
            for n in ("gate_up_proj", "down_proj"):
                got = getattr(model.layers[i].mlp, n)
                ok = ok and torch.equal(got, ref[f"layers.{i}.mlp.{n}"][lo:hi])
        dist.destroy_process_group()
        q.put((rank, "ok" if ok else f"mismatch {report}"))
    except Exception:
        q.put((rank, traceback.format_exc()))


def test_expert_parallel_ranks_load_their_experts(tmp_path):
    import torch.multiprocessing as mp
    ref = _write_checkpoint(tmp_path, seed=3)
    torch.save(ref, tmp_path / "ref.pt")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_ep_worker, args=(r, 2, port, str(tmp_path), q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert all(v == "ok" for v in res.values()), res


def test_vision_key_mapping_matches_reference():
    """HF vision keys map onto the vision tower's parameter names by the
    reference's rule (REF loaders/hf.py:41-52) and all exist in the tower."""
    ref_dir = ROOT / "baseline" / "_ref"
    if not (ref_dir / "cuda_qwen3_vl").exists():
        pytest.skip("reference package not installed under baseline/_ref")
    sys.path.insert(0, str(ref_dir))
    os.environ.setdefault("CUDA_QWEN3_VL_AUTO_PRELOAD", "0")
    from cuda_qwen3_vl.loaders import hf as ref_hf
    from qwen3_5_vl_cuda_custom_b200 import synthetic as syn
    from qwen3_5_vl_cuda_custom_b200.loaders import map_hf_name
    from qwen3_5_vl_cuda_custom_b200.vision import CudaVisionTower
    keys = ["model.visual.patch_embed.proj.weight", "model.visual.patch_embed.proj.bias",
            "model.visual.pos_embed.weight", "model.visual.blocks.2.attn.qkv.bias",
            "model.visual.blocks.0.mlp.linear_fc2.weight", "model.visual.merger.norm.weight",
            "model.visual.deepstack_merger_list.1.linear_fc1.weight"]
    names = set("visual." + k for k in CudaVisionTower(syn.tiny_vision_config()).state_dict())
    for k in keys:
        assert map_hf_name(k) == ref_hf._map_name(k)
        assert map_hf_name(k) in names, k
