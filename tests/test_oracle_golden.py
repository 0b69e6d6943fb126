"""Pins the CPU oracle to the reference: regenerates the seeded inputs of each
golden case and compares the oracle with the outputs the reference itself
produced (tests/golden/make_golden.py)."""
import numpy as np
import pytest
import torch

from oracle import layer_oracle as O
from qwen3_5_vl_cuda_custom_b200 import synthetic as syn
from qwen3_5_vl_cuda_custom_b200.configs import tiny_moe_text
from tests.golden.make_golden import checksum

CFG = tiny_moe_text()
POS = {
    "c1_unit": syn.text_positions,
    "c1_literal": syn.text_positions,
    "c1_multimodal": lambda B, S: syn.multimodal_positions(B, S, img_off=16, grid=8),
}


def _inputs(case):
    g = torch.Generator().manual_seed(case["seed"])
    P = syn.layer_params(CFG, g, norm_mode=case["norm_mode"])
    x = syn.hidden_states((1, case["S"], CFG.hidden_size), g)
    return g, P, x


@pytest.mark.parametrize("name", ["c1_unit", "c1_literal", "c1_multimodal"])
def test_layer_matches_reference(golden, name):
    case = golden[name]
    g, P, x = _inputs(case)
    pos = POS[name](1, case["S"])
    assert abs(checksum([x, pos.float(), *P.values()]) - case["input_checksum"]) < 1e-6 * abs(case["input_checksum"])
    r = O.decoder_layer(x, P, CFG, pos)
    assert (r["out"] - case["out"]).abs().max() < 2e-5
    assert (r["router_logits"] - case["router_logits"]).abs().max() < 1e-6
    assert (r["k"] - case["k"]).abs().max() < 2e-5
    assert (r["v"] - case["v"]).abs().max() < 2e-5


def test_decode_step_matches_reference(golden):
    case = golden["c1_unit"]
    g, P, x = _inputs(case)
    pos = syn.text_positions(1, case["S"])
    r = O.decoder_layer(x, P, CFG, pos)
    xd = syn.hidden_states((1, 1, CFG.hidden_size), g)
    rd = O.decoder_layer(xd, P, CFG, syn.text_positions(1, 1, start=case["S"]),
                         past_kv=(r["k"], r["v"]))
    assert rd["k"].shape[2] == case["decode_k_len"]
    assert (rd["out"] - case["decode_out"]).abs().max() < 2e-5
    assert (rd["router_logits"] - case["decode_router_logits"]).abs().max() < 1e-6


def test_tiny_moe_module_matches_reference(golden):
    case = golden["moe_tiny"]
    g = torch.Generator().manual_seed(case["seed"])
    shapes = [("gate_weight", (4, 64)), ("gate_up_proj", (4, 64, 64)), ("down_proj", (4, 64, 32))]
    P = {n: torch.empty(s).normal_(0, 0.02, generator=g) for n, s in shapes}
    x = torch.empty(2, 8, 64).normal_(0, 1, generator=g)
    out, logits, *_ = O.moe(x.reshape(-1, 64), P["gate_weight"], P["gate_up_proj"], P["down_proj"], 2)
    assert (out.reshape(2, 8, 64) - case["out"]).abs().max() < 1e-6
    assert (logits - case["router_logits"]).abs().max() < 1e-7


def test_canonical_topk_ties_go_to_lower_index():
    # Known answer of the reference's CUDA top-k (strict '>' keeps the first max).
    p = torch.tensor([[1.0, 1.0, 1.0, 0.0, 1.0]])
    _, idx = O.canonical_topk(p, 3)
    assert idx.tolist() == [[0, 1, 2]]


def test_permutation_is_expert_then_token_order():
    idx = np.array([[2, 0], [0, 1], [2, 1]])
    counts, offsets, sorted_tok, slot_pos, tiles = O.permutation(idx, 3)
    assert counts.tolist() == [2, 2, 2]
    assert offsets.tolist() == [0, 2, 4, 6]
    assert sorted_tok.tolist() == [0, 1, 1, 2, 0, 2]
    # pair (t, j) lands at its sorted row
    for t in range(3):
        for j in range(2):
            r = slot_pos[t * 2 + j]
            assert sorted_tok[r] == t
    assert tiles.tolist() == [0, 1, 2, 3]


def test_permutation_matches_reference_nonzero_loop():
    rng = np.random.default_rng(0)
    T, k, E = 200, 4, 16
    idx = np.stack([rng.choice(E, k, replace=False) for _ in range(T)])
    _, offsets, sorted_tok, _, _ = O.permutation(idx, E)
    ti = torch.from_numpy(idx)
    rows = []
    for e in range(E):  # REF modules/moe.py:71-76
        tok, _slot = (ti == e).nonzero(as_tuple=True)
        rows.extend(tok.tolist())
    assert sorted_tok.tolist() == rows
