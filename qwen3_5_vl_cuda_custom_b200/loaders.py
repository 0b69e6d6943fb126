"""Hugging Face checkpoint loading for CudaQwen3VLMoeModel.

Maps the Qwen3-VL-MoE safetensors key names and layouts onto this library's
parameter names, which are the reference's own (REF loaders/hf.py:21-109):

- ``lm_head.weight`` stays at top level;
- ``model.language_model.<rest>`` -> ``<rest>`` with the MoE renames
  ``mlp.experts.gate_up_proj`` -> ``mlp.gate_up_proj``,
  ``mlp.experts.down_proj`` -> ``mlp.down_proj``,
  ``mlp.gate.weight`` -> ``mlp.gate_weight``;
- the expert tensors are stored transposed on disk ((E, H, 2I) and (E, I, H));
  they are transposed on dims (1, 2) to (E, 2I, H) and (E, H, I);
- ``model.visual.<rest>`` -> ``visual.<rest>`` with ``patch_embed.proj.`` ->
  ``patch_embed.``, ``pos_embed.weight`` -> ``pos_embed.emb.weight`` and
  ``deepstack_merger_list.`` -> ``deepstack_mergers.``; a model built with
  ``vision=False`` reports these keys as ``skipped``.

Expert-parallel models (built with ``expert_group``) read only their own
experts' rows from the files (``safe_open(...).get_slice``), so no rank
materialises the full expert tensors.
"""
from __future__ import annotations

from pathlib import Path

import torch

_EXPERT_KEYS = ("mlp.experts.gate_up_proj", "mlp.experts.down_proj")


def map_hf_name(name: str) -> str | None:
    """Internal parameter name of an HF checkpoint key; None for keys this
    library does not hold."""
    if name == "lm_head.weight":
        return name
    if name.startswith("model.visual."):
        rest = name[len("model.visual."):].replace("patch_embed.proj.", "patch_embed.")
        if rest == "pos_embed.weight":
            rest = "pos_embed.emb.weight"
        return "visual." + rest.replace("deepstack_merger_list.", "deepstack_mergers.")
    prefix = "model.language_model."
    if not name.startswith(prefix):
        return None
    rest = name[len(prefix):]
    rest = rest.replace("mlp.experts.gate_up_proj", "mlp.gate_up_proj")
    rest = rest.replace("mlp.experts.down_proj", "mlp.down_proj")
    rest = rest.replace("mlp.gate.weight", "mlp.gate_weight")
    return rest


def _expert_range(model: torch.nn.Module, internal: str) -> tuple[int, int] | None:
    """(lo, hi) experts held by this rank for an expert tensor of an
    expert-parallel layer, else None (all experts)."""
    mod_name = internal.rsplit(".", 1)[0]
    try:
        mod = model.get_submodule(mod_name)
    except AttributeError:
        return None
    ex = getattr(mod, "exchange", None)
    if ex is None or getattr(mod, "expert_placement", None) is not None:
        return None  # all experts (a placed layer selects its own rows on load)
    return ex.expert_range


def load_hf_weights(model: torch.nn.Module, snapshot_path: str | Path) -> dict:
    """Loads every ``*.safetensors`` file of ``snapshot_path`` into ``model``.

    Returns {'loaded', 'missing', 'unexpected', 'mismatched', 'skipped'}:
    internal names loaded, model parameters no file provided, unmapped
    checkpoint keys, (key, file shape, model shape) mismatches, and the vision
    keys left out by design."""
    from safetensors import safe_open

    files = sorted(Path(snapshot_path).glob("*.safetensors"))
    if not files:
        raise FileNotFoundError(f"no .safetensors files in {snapshot_path}")
    state = dict(model.state_dict())
    remaining = set(state)
    loaded, unexpected, mismatched, skipped = [], [], [], []
    for f in files:
        with safe_open(str(f), framework="pt", device="cpu") as sf:
            for key in sf.keys():
                if key.startswith("model.visual.") and getattr(model, "visual", None) is None:
                    skipped.append(key)
                    continue
                internal = map_hf_name(key)
                if internal is None or internal not in state:
                    unexpected.append(key)
                    continue
                target = state[internal]
                is_expert = any(k in key for k in _EXPERT_KEYS)
                rng = _expert_range(model, internal) if is_expert else None
                if rng is not None:
                    lo, hi = rng
                    tensor = sf.get_slice(key)[lo:hi]
                else:
                    tensor = sf.get_tensor(key)
                if is_expert:
                    tensor = tensor.transpose(1, 2)
                    mod = model.get_submodule(internal.rsplit(".", 1)[0])
                    if rng is None and getattr(mod, "expert_placement", None) is not None:
                        tensor = tensor[torch.tensor(mod.local_experts)]
                if tuple(tensor.shape) != tuple(target.shape):
                    mismatched.append((key, tuple(tensor.shape), tuple(target.shape)))
                    continue
                with torch.no_grad():
                    target.copy_(tensor.to(target.dtype))
                loaded.append(internal)
                remaining.discard(internal)
    return {"loaded": loaded, "missing": sorted(remaining), "unexpected": unexpected,
            "mismatched": mismatched, "skipped": skipped}
