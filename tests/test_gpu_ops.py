"""Kernel-level parity on the GPU: each libq35b200 entry point against the CPU
oracle (fp32) on seeded inputs, including the edge cases the reference's own
kernel tests cover (REF tests/test_kernels.py) and ragged / empty shapes."""
import numpy as np
import pytest
import torch

from oracle import layer_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _lib_ready():
    from qwen3_5_vl_cuda_custom_b200 import build
    build.build()
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    yield
    from qwen3_5_vl_cuda_custom_b200 import kernels as K
    K.device_error_check()


def K():
    from qwen3_5_vl_cuda_custom_b200 import kernels
    return kernels


def bf(t):
    return t.to(torch.bfloat16)


def gen(seed):
    return torch.Generator().manual_seed(seed)


# ------------------------------------------------------------------ norms
@pytest.mark.parametrize("rows,cols", [(4, 256), (4096, 2048), (7, 128), (3, 1000), (1, 4096),
                                       (5, 1024)])
@pytest.mark.parametrize("fp32_in", [False, True])
def test_rmsnorm(rows, cols, fp32_in):
    """bf16 input, or the fp32 residual-stream input of the post-attention norm."""
    g = gen(rows * 7 + cols)
    x = torch.randn(rows, cols, generator=g)
    x = x if fp32_in else bf(x)
    w = bf(1 + 0.02 * torch.randn(cols, generator=g))
    y = K().rmsnorm(x.to(DEV), w.to(DEV), 1e-6).float().cpu()
    ref = O.rmsnorm(x.float(), w.float(), 1e-6)
    # one bf16 rounding of the output
    assert (y - ref).abs().max() <= 2 ** -7 * ref.abs().max() + 1e-6


# ------------------------------------------------------------------ GEMM
@pytest.mark.parametrize("M", [64, 17])
def test_gemm_splitk_with_residual_and_fp32_out(M):
    """Decode-sized rows take the split-K path: partial planes summed with the
    bias and the bf16 residual, fp32 or bf16 output."""
    g = gen(M)
    N, K_ = 2048, 4096
    a = bf(torch.randn(M, K_, generator=g))
    b = bf(torch.randn(N, K_, generator=g) * 0.02)
    bias = bf(torch.randn(N, generator=g) * 0.1)
    res = bf(torch.randn(M, N, generator=g))
    Kk = K()
    assert Kk._splitk_factor(M, N, K_, torch.device(DEV)) > 1
    ref = a.float() @ b.float().t() + bias.float() + res.float()
    for dt in (torch.float32, torch.bfloat16):
        out = Kk.matmul(a.to(DEV), b.to(DEV), bias.to(DEV), residual=res.to(DEV), out_dtype=dt)
        err = (out.float().cpu() - ref).abs().max()
        assert err <= 1e-2 * ref.abs().max() + 1e-3, float(err)

def test_gemm_splitk_agrees_with_unsplit_on_same_rows():
    """The split-K path (decode-sized calls) and the single-pass path (what the
    same rows get inside a larger call) agree within the GEMM tolerance; with
    DECODE_SPLITK off a small call is bit-identical to the same rows of a
    large call."""
    g = gen(777)
    N, K_ = 5120, 2048
    a = bf(torch.randn(300, K_, generator=g)).to(DEV)
    b = bf(torch.randn(N, K_, generator=g) * 0.02).to(DEV)
    Kk = K()
    big = Kk.matmul(a, b)  # 300 rows: no split
    assert Kk._splitk_factor(64, N, K_, torch.device(DEV)) > 1
    small = Kk.matmul(a[:64].contiguous(), b)
    ref = a[:64].float() @ b.float().t()
    assert (small.float() - big[:64].float()).abs().max() <= 1e-2 * ref.abs().max() + 1e-3
    try:
        Kk.DECODE_SPLITK = False
        assert Kk._splitk_factor(64, N, K_, torch.device(DEV)) == 1
        unsplit = Kk.matmul(a[:64].contiguous(), b)
    finally:
        Kk.DECODE_SPLITK = True
    assert torch.equal(unsplit, big[:64])


@pytest.mark.parametrize("M,N,K_", [(8, 64, 64), (128, 128, 64), (300, 384, 256), (4096, 5120, 2048),
                                    (4096, 2048, 4096), (1, 256, 128), (129, 2048, 768),
                                    (64, 5120, 2048), (64, 2048, 4096), (3, 96, 640)])
def test_gemm(M, N, K_):
    g = gen(M + N + K_)
    a = bf(torch.randn(M, K_, generator=g))
    b = bf(torch.randn(N, K_, generator=g) * 0.05)
    out = K().matmul(a.to(DEV), b.to(DEV)).float().cpu()
    ref = a.float() @ b.float().t()
    err = (out - ref).abs().max()
    assert err <= 1e-2 * ref.abs().max() + 1e-3, float(err)


def test_gemm_bias_residual():
    g = gen(3)
    a = bf(torch.randn(200, 256, generator=g))
    b = bf(torch.randn(96, 256, generator=g) * 0.05)
    bias = bf(torch.randn(96, generator=g))
    res = bf(torch.randn(200, 96, generator=g))
    out = K().matmul(a.to(DEV), b.to(DEV), bias.to(DEV), residual=res.to(DEV)).float().cpu()
    ref = a.float() @ b.float().t() + bias.float() + res.float()
    assert (out - ref).abs().max() <= 2e-2 * ref.abs().max()


def test_matmul_reference_case():
    """REF tests/test_kernels.py:156-162 shape (bf16 here)."""
    x = bf(torch.randn(8, 64)).to(DEV)
    w = bf(torch.randn(32, 64)).to(DEV)
    b = bf(torch.randn(32)).to(DEV)
    torch.testing.assert_close(K().matmul(x, w, b).float(), torch.nn.functional.linear(
        x.float(), w.float(), b.float()), atol=0.1, rtol=2e-2)


# ------------------------------------------------------------------ router
@pytest.mark.parametrize("T,H,E,k", [(128, 256, 16 * 2, 4), (4096, 2048, 128, 8), (33, 512, 64, 8),
                                     (1, 2048, 128, 8), (100, 256, 256, 16)])
def test_router(T, H, E, k):
    g = gen(T + E)
    x = bf(torch.randn(T, H, generator=g))
    wg = torch.randn(E, H, generator=g) * 0.02
    logits, idx, w = K().router_topk(x.to(DEV), wg.to(DEV), k)
    rl, p, ridx, rw = O.router(x.float(), wg, k)
    assert (logits.cpu() - rl).abs().max() < 1e-5
    tie = O.near_tie_rows(p, k)
    ok = ~tie
    assert torch.equal(idx.cpu().long()[ok], ridx[ok]), "top-k ids differ outside near-tie rows"
    assert (w.cpu()[ok] - rw[ok]).abs().max() < 1e-5


@pytest.mark.parametrize("T,H,E,k", [(4096, 2048, 128, 8), (77, 256, 32, 4), (300, 512, 256, 16),
                                     (1, 2048, 128, 8)])
def test_router_tensor_core_path(T, H, E, k):
    """Logits from the exact bf16 split of the fp32 gate on tcgen05."""
    g = gen(T * 5 + E)
    x = bf(torch.randn(T, H, generator=g))
    wg = torch.randn(E, H, generator=g) * 0.02
    w3 = K().router_split_weights(wg.to(DEV))
    parts = w3.view(E, 3, H).float().sum(1).cpu()
    assert torch.equal(parts, wg), "lo + mid + hi must equal the fp32 weight exactly"
    bias = torch.randn(E, generator=g) * 0.1
    logits, idx, w = K().router_topk(x.to(DEV), wg.to(DEV), k, bias=bias.to(DEV), gate_split=w3)
    rl, p, ridx, rw = O.router(x.float(), wg, k, bias=bias)
    # the tensor core accumulates fp32 with truncation: logits agree to ~1e-5,
    # so rows whose k-th / (k+1)-th probabilities are within 1e-4 may swap
    assert (logits.cpu() - rl).abs().max() < 2e-5
    ok = ~O.near_tie_rows(p, k, rel=1e-4)
    assert torch.equal(idx.cpu().long()[ok], ridx[ok])
    assert (w.cpu()[ok] - rw[ok]).abs().max() < 1e-5


@pytest.mark.parametrize("T,H,E,k", [(4096, 2048, 128, 8), (16384, 2048, 128, 8), (77, 256, 32, 4),
                                     (300, 512, 64, 8), (1, 2048, 128, 8), (129, 1024, 128, 8)])
def test_router_fused_and_counted_permutation(T, H, E, k):
    """Cluster router (three exact bf16 planes in TMEM, partials reduced over
    distributed shared memory) with the permutation's chunk counts, then the
    one-launch scan + scatter: logits vs the fp32 oracle, ids and weights
    outside near ties, chunk counts and the whole permutation bit-exact."""
    Kk = K()
    assert Kk.router_fused_supported(T, H, E, k)
    g = gen(T * 7 + E + H)
    x = bf(torch.randn(T, H, generator=g))
    wg = torch.randn(E, H, generator=g) * 0.02
    bias = torch.randn(E, generator=g) * 0.1
    w3 = Kk.router_split_weights(wg.to(DEV))
    logits, idx, w, cc = Kk.router_topk(x.to(DEV), wg.to(DEV), k, bias=bias.to(DEV), gate_split=w3,
                                        chunk_counts=True)
    assert cc is not None and tuple(cc.shape) == (-(-T // 128), E)
    rl, p, ridx, rw = O.router(x.float(), wg, k, bias=bias)
    assert (logits.cpu() - rl).abs().max() < 2e-5
    ok = ~O.near_tie_rows(p, k, rel=1e-4)
    assert torch.equal(idx.cpu().long()[ok], ridx[ok])
    assert (w.cpu()[ok] - rw[ok]).abs().max() < 1e-5
    gi = idx.cpu().numpy()
    want = np.stack([np.bincount(gi[c * 128:(c + 1) * 128].reshape(-1), minlength=E)
                     for c in range(-(-T // 128))])
    assert cc.cpu().numpy().tolist() == want.tolist()
    perm = Kk.moe_permute_counted(idx, cc, E)
    counts, offsets, sorted_tok, slot_pos, tiles = O.permutation(gi, E)
    assert perm.counts.cpu().numpy().tolist() == counts.tolist()
    assert perm.offsets.cpu().numpy().tolist() == offsets.tolist()
    assert perm.sorted_tok.cpu().numpy().tolist() == sorted_tok.tolist()
    assert perm.slot_pos.cpu().numpy().tolist() == slot_pos.tolist()
    assert perm.tile_offsets.cpu().numpy().tolist() == tiles.tolist()
    Kk.device_error_check()


def test_router_ties_to_lower_index():
    """All-equal logits: every expert ties; the top-k must be 0..k-1."""
    x = torch.zeros(4, 256, dtype=torch.bfloat16, device=DEV)
    wg = torch.randn(32, 256, device=DEV)
    _, idx, w = K().router_topk(x, wg, 4)
    assert idx.cpu().tolist() == [[0, 1, 2, 3]] * 4
    assert torch.allclose(w.cpu(), torch.full((4, 4), 0.25))


def test_router_bias_skews_choice():
    x = bf(torch.randn(64, 256)).to(DEV)
    wg = torch.zeros(32, 256, device=DEV)
    bias = torch.zeros(32, device=DEV)
    bias[5] = 10.0
    logits, idx, _ = K().router_topk(x, wg, 2, bias=bias)
    assert (idx[:, 0] == 5).all()
    assert (logits[:, 5] == 10.0).all()


def test_softmax_and_topk_ops():
    """REF tests/test_kernels.py:102-106 and :278-285."""
    x = torch.randn(8, 256, device=DEV)
    torch.testing.assert_close(K().softmax(x), torch.softmax(x, dim=-1), atol=1e-6, rtol=1e-5)
    x = torch.randn(8, 60, device=DEV)
    v, i = K().cuda_topk(x, 4)
    rv, ri = torch.topk(x, 4, dim=-1)
    torch.testing.assert_close(v, rv)
    assert (i == ri).all()
    t = torch.tensor([[1.0, 1.0, 1.0, 0.0, 1.0]], device=DEV)
    _, i = K().cuda_topk(t, 3)
    assert i.tolist() == [[0, 1, 2]]


# ------------------------------------------------------------------ permutation
def _perm_case(idx_np, E):
    idx = torch.from_numpy(idx_np.astype(np.int32)).to(DEV)
    perm = K().moe_permute(idx, E)
    counts, offsets, sorted_tok, slot_pos, tiles = O.permutation(idx_np, E)
    assert perm.counts.cpu().numpy().tolist() == counts.tolist()
    assert perm.offsets.cpu().numpy().tolist() == offsets.tolist()
    assert perm.sorted_tok.cpu().numpy().tolist() == sorted_tok.tolist()
    assert perm.slot_pos.cpu().numpy().tolist() == slot_pos.tolist()
    assert perm.tile_offsets.cpu().numpy().tolist() == tiles.tolist()


@pytest.mark.parametrize("T,E,k", [(4096, 128, 8), (1, 128, 8), (129, 16, 4), (1000, 64, 8),
                                   (16384, 128, 8), (300, 256, 16)])
def test_permutation_bit_exact(T, E, k):
    rng = np.random.default_rng(T + E)
    idx = np.argsort(rng.random((T, E)), axis=1)[:, :k]
    _perm_case(idx, E)


def test_permutation_all_tokens_one_expert_set_and_empty_experts():
    T, E, k = 700, 128, 8
    idx = np.tile(np.arange(8)[::-1], (T, 1))  # experts 0..7 only, others empty
    _perm_case(idx, E)


def test_permutation_negative_ids_are_empty_slots():
    idx = np.array([[3, -1], [-1, 0], [3, 1], [-1, -1]])
    got = K().moe_permute(torch.from_numpy(idx.astype(np.int32)).to(DEV), 4)
    keep = [(t, j) for t in range(4) for j in range(2) if idx[t, j] >= 0]
    assert got.counts.cpu().tolist() == [1, 1, 0, 2]
    assert got.offsets.cpu().tolist() == [0, 1, 2, 2, 4]
    assert got.sorted_tok.cpu()[:4].tolist() == [1, 2, 0, 2]
    sp = got.slot_pos.cpu().view(4, 2)
    assert all(sp[t, j] == -1 for t in range(4) for j in range(2) if idx[t, j] < 0)
    assert len(keep) == 4
    K().device_error_check()  # negative ids are not errors


def test_permutation_skewed_zipf():
    rng = np.random.default_rng(1)
    T, E, k = 2048, 128, 8
    pop = 1.0 / np.arange(1, E + 1) ** 1.2
    pop /= pop.sum()
    idx = np.stack([rng.choice(E, k, replace=False, p=pop) for _ in range(T)])
    _perm_case(idx, E)


# ------------------------------------------------------------------ grouped GEMMs + combine
@pytest.mark.parametrize("H,I", [(256, 128), (512, 192), (2048, 768)])
def test_grouped_gemm_ragged_groups(H, I):
    """Group sizes around the token sub-tile edges (multiples of 16 up to 256
    columns, balanced sub-tiles above 256 rows) and one hot group of thousands
    of rows; both grouped GEMMs against fp32 per-group products."""
    counts = [1, 15, 16, 17, 33, 64, 127, 128, 129, 200, 255, 256, 257, 300, 0, 384, 385, 520,
              4099]
    E = len(counts)
    g = gen(H + I)
    idx = torch.cat([torch.full((c,), e, dtype=torch.int32) for e, c in enumerate(counts)])
    idx = idx[torch.randperm(idx.numel(), generator=g)].reshape(-1, 1)
    T = idx.shape[0]
    x = bf(torch.randn(T, H, generator=g))
    gu = bf(torch.randn(E, 2 * I, H, generator=g) * 0.05)
    dn = bf(torch.randn(E, H, I, generator=g) * 0.05)
    Kk = K()
    perm = Kk.moe_permute(idx.to(DEV), E)
    xs = Kk.gather_rows(x.to(DEV), perm.sorted_tok)
    act = Kk.grouped_gateup_swiglu(xs, gu.to(DEV), perm)
    y = Kk.grouped_down(act, dn.to(DEV), perm)
    off = perm.offsets.cpu().long().tolist()
    xs_c = xs.float().cpu()
    act_c = act.float().cpu()
    for e in range(E):
        a, b = off[e], off[e + 1]
        assert b - a == counts[e]
        if a == b:
            continue
        h = xs_c[a:b] @ gu[e].float().t()
        ref_act = torch.nn.functional.silu(h[:, :I]) * h[:, I:]
        st = O.error_stats(act_c[a:b], ref_act)
        assert st["max_abs_over_bf16"] <= 2e-2 and st["mean_rel"] <= 5e-3, (e, counts[e], st)
        ref_y = act_c[a:b] @ dn[e].float().t()
        st = O.error_stats(y[a:b].float().cpu(), ref_y)
        assert st["max_abs_over_bf16"] <= 2e-2 and st["mean_rel"] <= 5e-3, (e, counts[e], st)


@pytest.mark.parametrize("T,H,I,E,k", [(128, 256, 128, 16, 4), (1024, 2048, 768, 128, 8),
                                       (37, 256, 64, 8, 2), (512, 512, 96, 32, 4),
                                       (64, 256, 96, 4, 2)])
def test_moe_experts_pipeline(T, H, I, E, k):
    g = gen(T * 3 + E)
    x = bf(torch.randn(T, H, generator=g))
    wg = torch.randn(E, H, generator=g) * 0.02
    gu = bf(torch.randn(E, 2 * I, H, generator=g) * 0.02)
    dn = bf(torch.randn(E, H, I, generator=g) * 0.02)
    res = bf(torch.randn(T, H, generator=g))
    Kk = K()
    xd = x.to(DEV)
    _, idx, w = Kk.router_topk(xd, wg.to(DEV), k)
    perm = Kk.moe_permute(idx, E)
    xs = Kk.gather_rows(xd, perm.sorted_tok)
    assert torch.equal(xs.cpu(), x[perm.sorted_tok.cpu().long()])
    act = Kk.grouped_gateup_swiglu(xs, gu.to(DEV), perm)
    y = Kk.grouped_down(act, dn.to(DEV), perm)
    if I % 128 == 0 and H % 128 == 0:  # tile-packed weights give identical results
        act_p = Kk.grouped_gateup_swiglu(xs, gu.to(DEV), perm, w_packed=Kk.pack_b_tiles(gu.to(DEV)))
        y_p = Kk.grouped_down(act, dn.to(DEV), perm, w_packed=Kk.pack_b_tiles(dn.to(DEV)))
        # the packed path runs the weight rows on the MMA's N side instead of M
        torch.testing.assert_close(act_p.float(), act.float(), rtol=1e-2, atol=1e-3)
        torch.testing.assert_close(y_p.float(), y.float(), rtol=1e-2, atol=1e-3)
    out = Kk.moe_combine(y, w, perm.slot_pos, res.to(DEV), T, H).float().cpu()
    # oracle with the GPU's own routing (routing parity is tested separately)
    offs = perm.offsets.cpu().tolist()
    st = perm.sorted_tok.cpu().long()
    xs_f = x.float()[st]
    act_ref = torch.empty(T * k, I)
    y_ref = torch.empty(T * k, H)
    for e in range(E):
        a, b = offs[e], offs[e + 1]
        if a == b:
            continue
        h = xs_f[a:b] @ gu[e].float().t()
        act_ref[a:b] = torch.nn.functional.silu(h[:, :I]) * h[:, I:]
        y_ref[a:b] = act_ref[a:b] @ dn[e].float().t()
    e_act = (act.float().cpu() - act_ref).abs().max()
    assert e_act <= 1e-2 * act_ref.abs().max() + 1e-4, float(e_act)
    e_y = (y.float().cpu() - y_ref).abs().max()
    assert e_y <= 2e-2 * y_ref.abs().max() + 1e-4, float(e_y)
    sp = perm.slot_pos.cpu().long().view(T, k)
    ref = res.float() + (w.cpu().unsqueeze(-1) * y_ref[sp]).sum(1)
    s = O.error_stats(out, ref)
    assert s["max_abs"] < 2e-2 and s["mean_rel"] < 5e-3, s


def test_index_add_residual_swiglu_ops():
    """REF tests/test_kernels.py:288-297, :49-54, :11-15 (bf16 / fp32)."""
    tgt = torch.zeros(8, 32, device=DEV)
    src = torch.randn(5, 32, device=DEV)
    idx = torch.tensor([0, 2, 4, 6, 7], device=DEV)
    r = tgt.clone().index_add_(0, idx, src)
    K().cuda_index_add(tgt, src, idx)
    torch.testing.assert_close(tgt, r)
    a = bf(torch.randn(4, 16, 64)).to(DEV)
    b = bf(torch.randn(4, 16, 64)).to(DEV)
    torch.testing.assert_close(K().residual_add(a, b), (a.float() + b.float()).bfloat16())
    gte = bf(torch.randn(8, 128)).to(DEV)
    up = bf(torch.randn(8, 128)).to(DEV)
    torch.testing.assert_close(K().swiglu(gte, up).float(),
                               torch.nn.functional.silu(gte.float()) * up.float(), atol=2e-2, rtol=1e-2)


# ------------------------------------------------------------------ rotary
@pytest.mark.parametrize("interleaved", [False, True])
@pytest.mark.parametrize("D,sections,multimodal", [(128, [24, 20, 20], False), (128, [24, 20, 20], True),
                                                   (64, [16, 8, 8], True)])
def test_qknorm_mrope(D, sections, multimodal, interleaved):
    from qwen3_5_vl_cuda_custom_b200 import synthetic as syn
    B, S, Hq, Hkv = 2, 384, 8, 2
    g = gen(D + S)
    qkv = bf(torch.randn(B * S, (Hq + 2 * Hkv) * D, generator=g))
    qw = bf(1 + 0.1 * torch.randn(D, generator=g))
    kw = bf(1 + 0.1 * torch.randn(D, generator=g))
    pos = syn.multimodal_positions(B, S) if multimodal else syn.text_positions(B, S, start=8000)
    inv = O.inv_freq(D, 5e6)
    q, k, v = K().qknorm_mrope(qkv.to(DEV), qw.to(DEV), kw.to(DEV), pos.to(DEV), inv.to(DEV), sections,
                               B, S, Hq, Hkv, D, 1e-6, interleaved)
    x = qkv.float().view(B, S, Hq + 2 * Hkv, D)
    cos3, sin3 = O.mrope_cos_sin(pos, inv)
    cos, sin = O.mrope_select(cos3, sin3, sections, interleaved)
    qr = O.rotate(O.rmsnorm(x[:, :, :Hq], qw, 1e-6).transpose(1, 2), cos, sin)
    kr = O.rotate(O.rmsnorm(x[:, :, Hq:Hq + Hkv], kw, 1e-6).transpose(1, 2), cos, sin)
    vr = x[:, :, Hq + Hkv:].transpose(1, 2)
    for got, ref in ((q, qr), (k, kr), (v, vr)):
        assert (got.float().cpu() - ref).abs().max() <= 2 ** -7 * ref.abs().max() + 1e-3


@pytest.mark.parametrize("B,S,H,Hq,Hkv,sections,multimodal,interleaved", [
    (2, 384, 512, 8, 2, [24, 20, 20], False, False),
    (1, 300, 256, 4, 1, [24, 20, 20], True, False),   # ragged last row tile, MQA
    (2, 256, 2048, 32, 4, [24, 20, 20], True, True),  # A3B head layout
    (3, 100, 136, 6, 2, [16, 24, 24], False, False),  # K tail (136 = 2*64 + 8)
])
def test_qkv_proj_norm_rope(B, S, H, Hq, Hkv, sections, multimodal, interleaved):
    """Projection GEMM with QK-norm + mRoPE + head-major split in its epilogue
    vs the oracle's fp32 projection, RMSNorm and rotation (REF
    modules/attention.py:82-87)."""
    from qwen3_5_vl_cuda_custom_b200 import synthetic as syn
    D = 128
    g = gen(B * S + H)
    x = bf(torch.randn(B, S, H, generator=g))
    w = bf(torch.randn((Hq + 2 * Hkv) * D, H, generator=g) * H ** -0.5)
    qw = bf(1 + 0.1 * torch.randn(D, generator=g))
    kw = bf(1 + 0.1 * torch.randn(D, generator=g))
    pos = syn.multimodal_positions(B, S) if multimodal else syn.text_positions(B, S, start=3000)
    inv = O.inv_freq(D, 5e6)
    q, k, v = K().qkv_proj_norm_rope(x.to(DEV), w.to(DEV), qw.to(DEV), kw.to(DEV), pos.to(DEV),
                                     inv.to(DEV), sections, Hq, Hkv, 1e-6, interleaved)
    xp = (x.float().reshape(B * S, H) @ w.float().t()).view(B, S, Hq + 2 * Hkv, D)
    cos3, sin3 = O.mrope_cos_sin(pos, inv)
    cos, sin = O.mrope_select(cos3, sin3, sections, interleaved)
    qr = O.rotate(O.rmsnorm(xp[:, :, :Hq], qw, 1e-6).transpose(1, 2), cos, sin)
    kr = O.rotate(O.rmsnorm(xp[:, :, Hq:Hq + Hkv], kw, 1e-6).transpose(1, 2), cos, sin)
    vr = xp[:, :, Hq + Hkv:].transpose(1, 2)
    for got, ref in ((q, qr), (k, kr), (v, vr)):
        st = O.error_stats(got.float().cpu(), ref)
        assert st["max_abs_over_bf16"] <= 2e-2 and st["mean_rel"] <= 5e-3, st


def test_mrope_op_matches_oracle():
    from qwen3_5_vl_cuda_custom_b200 import synthetic as syn
    B, H, S, D = 2, 4, 400, 128
    x = bf(torch.randn(B, H, S, D))
    pos = syn.multimodal_positions(B, S)
    inv = O.inv_freq(D, 5e6)
    y = K().mrope(x.to(DEV), pos.to(DEV), inv.to(DEV), [24, 20, 20]).float().cpu()
    cos3, sin3 = O.mrope_cos_sin(pos, inv)
    cos, sin = O.mrope_select(cos3, sin3, [24, 20, 20])
    ref = O.rotate(x.float(), cos, sin)
    assert (y - ref).abs().max() <= 2 ** -7 * ref.abs().max() + 1e-3


# ------------------------------------------------------------------ attention
@pytest.mark.parametrize("B,Hq,Hkv,Sq,Skv,causal", [
    (1, 8, 2, 128, 128, True), (2, 4, 4, 16, 16, True), (1, 8, 2, 200, 200, True), (1, 32, 4, 1000, 1000, True),
    (2, 8, 2, 77, 77, False), (1, 8, 1, 64, 300, True), (1, 4, 2, 200, 450, False),
    (1, 32, 4, 4096, 4096, True)])
def test_attention_prefill(B, Hq, Hkv, Sq, Skv, causal):
    g = gen(Sq * 31 + Skv)
    q = bf(torch.randn(B, Hq, Sq, 128, generator=g))
    k = bf(torch.randn(B, Hkv, Skv, 128, generator=g))
    v = bf(torch.randn(B, Hkv, Skv, 128, generator=g))
    scale = 128 ** -0.5
    out = K().attention_tokens(q.to(DEV), k.to(DEV), v.to(DEV), scale, causal).float().cpu()
    if Sq > 1024:  # keep the CPU oracle quick: check a strided subset of heads
        sel = slice(0, Hq, 8)
        got = out.view(B, Sq, Hq, 128)[:, :, sel].transpose(1, 2)
        # heads 0, 8, 16, 24 map to kv heads 0..3 when Hq/Hkv = 8
        ref = torch.stack([O.attention(q[:, h:h + 1], k[:, h // (Hq // Hkv):h // (Hq // Hkv) + 1],
                                       v[:, h // (Hq // Hkv):h // (Hq // Hkv) + 1], scale, causal)[:, 0]
                           for h in range(0, Hq, 8)], dim=1)
    else:
        ref = O.attention(q, k, v, scale, causal)
        got = out.view(B, Sq, Hq, 128).transpose(1, 2)
    s = O.error_stats(got, ref)
    assert s["max_abs"] < 2e-2 and s["mean_rel"] < 5e-3, s


@pytest.mark.parametrize("B,Hq,Hkv,Sq,Skv", [(4, 32, 4, 1, 8193), (2, 8, 2, 1, 33), (3, 16, 4, 4, 700),
                                             (1, 32, 4, 1, 1)])
def test_attention_decode(B, Hq, Hkv, Sq, Skv):
    g = gen(Skv + Sq)
    q = bf(torch.randn(B, Hq, Sq, 128, generator=g))
    k = bf(torch.randn(B, Hkv, Skv, 128, generator=g))
    v = bf(torch.randn(B, Hkv, Skv, 128, generator=g))
    scale = 128 ** -0.5
    out = K().attention_tokens(q.to(DEV), k.to(DEV), v.to(DEV), scale, False).float().cpu()
    ref = O.attention(q, k, v, scale, False)
    s = O.error_stats(out.view(B, Sq, Hq, 128).transpose(1, 2), ref)
    assert s["max_abs"] < 2e-2 and s["mean_rel"] < 5e-3, s


def test_flash_attention_reference_cases():
    """REF tests/test_kernels.py:184-194 and :261-273 (bf16, head_dim 128)."""
    torch.manual_seed(42)
    q = torch.randn(2, 8, 16, 128, device=DEV, dtype=torch.bfloat16)
    k = torch.randn(2, 2, 16, 128, device=DEV, dtype=torch.bfloat16)
    v = torch.randn(2, 2, 16, 128, device=DEV, dtype=torch.bfloat16)
    scale = 128 ** -0.5
    k_exp = k[:, :, None].expand(2, 2, 4, 16, 128).reshape(2, 8, 16, 128)
    v_exp = v[:, :, None].expand(2, 2, 4, 16, 128).reshape(2, 8, 16, 128)
    for causal in (True, False):
        expected = torch.nn.functional.scaled_dot_product_attention(
            q.float(), k_exp.float(), v_exp.float(), is_causal=causal, scale=scale)
        actual = K().flash_attention(q, k, v, scale=scale, is_causal=causal, num_kv_groups=4)
        torch.testing.assert_close(actual.float(), expected, atol=2e-2, rtol=2e-2)


def test_fp32_residual_stream_ops():
    """o_proj GEMM with fp32 output and the fp32-input RMSNorm the layer uses
    to keep h = x + attn unrounded."""
    g = gen(11)
    a = bf(torch.randn(300, 512, generator=g))
    b = bf(torch.randn(256, 512, generator=g) * 0.05)
    res = bf(torch.randn(300, 256, generator=g))
    out = K().matmul(a.to(DEV), b.to(DEV), residual=res.to(DEV), out_dtype=torch.float32)
    assert out.dtype == torch.float32
    ref = a.float() @ b.float().t() + res.float()
    assert (out.cpu() - ref).abs().max() <= 2e-3 * ref.abs().max()
    w = bf(1 + 0.02 * torch.randn(256, generator=g))
    y = K().rmsnorm(out, w.to(DEV), 1e-6).float().cpu()
    r = O.rmsnorm(out.cpu(), w.float(), 1e-6)
    assert (y - r).abs().max() <= 2 ** -7 * r.abs().max() + 1e-6


@pytest.mark.parametrize("T,E,k", [(1000, 128, 8), (4096, 64, 4), (130, 32, 16)])
def test_counted_permutation_with_empty_slots_and_hot_expert(T, E, k):
    """One-launch scan + scatter from host-computed chunk counts: ids with
    empty (-1) slots and one expert holding a third of the rows, bit-exact
    against the oracle permutation."""
    Kk = K()
    g = gen(T + E + k)
    hot = torch.rand(T, generator=g) < 0.33
    rows = []
    for t in range(T):
        r = torch.randperm(E, generator=g)
        if hot[t]:  # expert 3 first, the rest distinct
            r = torch.cat([r[r == 3], r[r != 3]])
        rows.append(r[:k])
    idx = torch.stack(rows).int()
    idx[torch.rand(T, k, generator=g) < 0.1] = -1
    gi = idx.numpy()
    cc = np.stack([np.bincount(gi[c * 128:(c + 1) * 128].reshape(-1)[gi[c * 128:(c + 1) * 128]
                                                                     .reshape(-1) >= 0],
                               minlength=E) for c in range(-(-T // 128))]).astype(np.int32)
    perm = Kk.moe_permute_counted(idx.to(DEV), torch.from_numpy(cc).to(DEV), E)
    # empty slots as a virtual expert E, ordered after every real expert
    counts, offsets, sorted_tok, slot_pos, _ = O.permutation(np.where(gi < 0, E, gi), E + 1)
    n = int(offsets[E])
    slot_pos = np.where(gi.reshape(-1) < 0, -1, slot_pos)
    tiles = np.concatenate([[0], np.cumsum((counts[:E] + 127) // 128)])
    assert perm.counts.cpu().numpy().tolist() == counts[:E].tolist()
    assert perm.offsets.cpu().numpy().tolist() == offsets[:E + 1].tolist()
    assert perm.sorted_tok.cpu().numpy()[:n].tolist() == sorted_tok[:n].tolist()
    assert perm.slot_pos.cpu().numpy().tolist() == slot_pos.tolist()
    assert perm.tile_offsets.cpu().numpy().tolist() == tiles.tolist()
    Kk.device_error_check()
