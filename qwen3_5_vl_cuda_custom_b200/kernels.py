"""Operator layer: the reference's op wrappers, re-implemented on libq35b200.

The reference exposes one Python function per op (REF cuda_qwen3_vl/kernels/
__init__.py:1-45), each falling back to torch when the tensor is not on CUDA
or the JIT build fails (e.g. REF kernels/matmul.py:62-77).  The functions here
keep the names and argument meanings, but they have no fallback: they require
CUDA tensors of the supported dtype and raise otherwise.  Fused entry points
used by the modules (router, permutation, grouped GEMMs, combine, QK-norm +
mRoPE) live here too.

Tensors passed in are made contiguous; outputs are allocated with
``torch.empty`` on the input's device and the work is enqueued on the current
CUDA stream.
"""
from __future__ import annotations


import torch

from . import _lib

_BF16 = torch.bfloat16


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _require(t: torch.Tensor, name: str, dtype: torch.dtype | tuple = _BF16) -> torch.Tensor:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name}: expected a tensor")
    if not t.is_cuda:
        raise RuntimeError(f"{name}: CUDA tensor required (this library has no CPU path)")
    dts = dtype if isinstance(dtype, tuple) else (dtype,)
    if t.dtype not in dts:
        raise RuntimeError(f"{name}: dtype {t.dtype} unsupported (expected {dts})")
    return t.contiguous()


# ---------------------------------------------------------------- norms
def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """RMSNorm over the last dim (REF kernels/rmsnorm.py:66-77).  x bf16 (or
    fp32: the layer's fp32 residual stream), weight bf16, output bf16."""
    x = _require(x, "rmsnorm.x", (_BF16, torch.float32))
    weight = _require(weight.to(_BF16) if weight.dtype != _BF16 else weight, "rmsnorm.weight")
    cols = x.shape[-1]
    if weight.numel() != cols:
        raise RuntimeError(f"rmsnorm: weight has {weight.numel()} elements, x has {cols} columns")
    y = torch.empty(x.shape, device=x.device, dtype=_BF16)
    name = "q35_rmsnorm_fwd" if x.dtype == _BF16 else "q35_rmsnorm_f32in_fwd"
    with torch.cuda.device(x.device):
        _lib.call(name, x.data_ptr(), weight.data_ptr(), y.data_ptr(),
                  x.numel() // cols if cols else 0, cols, float(eps), _stream(x))
    return y


# ---------------------------------------------------------------- GEMM
def matmul(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
           residual: torch.Tensor | None = None, out_dtype: torch.dtype = _BF16) -> torch.Tensor:
    """y = x @ weight^T (+ bias) (+ residual), REF kernels/matmul.py:62-77.

    bf16 in and out, fp32 accumulation on tcgen05.  ``residual`` (same shape as
    the output) fuses the reference's residual_add into the GEMM epilogue.
    """
    x = _require(x, "matmul.x")
    weight = _require(weight, "matmul.weight")
    K = x.shape[-1]
    N, Kw = weight.shape
    if Kw != K:
        raise RuntimeError(f"matmul: x has K={K}, weight has K={Kw}")
    M = x.numel() // K if K else 0
    if out_dtype not in (_BF16, torch.float32):
        raise RuntimeError(f"matmul: out_dtype {out_dtype} unsupported")
    out = torch.empty(*x.shape[:-1], N, device=x.device, dtype=out_dtype)
    if bias is not None:
        bias = _require(bias, "matmul.bias")
    if residual is not None:
        residual = _require(residual, "matmul.residual")
        if residual.shape != out.shape:
            raise RuntimeError("matmul: residual shape must equal the output shape")
    splits = _splitk_factor(M, N, K, x.device)
    with torch.cuda.device(x.device):
        if splits > 1:
            # few rows: split K so more SMs share the weight stream
            ws = torch.empty(splits * M * N, device=x.device, dtype=torch.float32)
            _lib.call("q35_gemm_bf16_splitk", x.data_ptr(), weight.data_ptr(), _ptr(bias),
                      _ptr(residual), out.data_ptr(), 1 if out_dtype == torch.float32 else 0,
                      M, N, K, splits, ws.data_ptr(), _stream(x))
        else:
            _lib.call("q35_gemm_bf16" if out_dtype == _BF16 else "q35_gemm_bf16_f32out",
                      x.data_ptr(), weight.data_ptr(), _ptr(bias), _ptr(residual),
                      out.data_ptr(), M, N, K, _stream(x))
    return out


_SM_COUNT: dict[int, int] = {}

# Split-K for decode-sized dense GEMMs (M <= 128 rows).  It changes the fp32
# summation order of a row's dot products, so the same row projected in a
# call of <= 128 rows and in a larger call can differ in the last bits (within
# the GEMM tolerance; batch invariance is lost).  Set to False for runs that
# must give bit-identical rows whatever the call size.
DECODE_SPLITK = True


def _splitk_factor(M: int, N: int, K: int, device) -> int:
    """K splits for a dense GEMM of at most 128 rows: the largest power of two
    (<= 16) that divides the 64-wide k-blocks and keeps ceil(N/128) * splits
    CTAs within one wave; 1 (no split) for larger M, when it would not help,
    or when DECODE_SPLITK is off."""
    if not DECODE_SPLITK or M == 0 or M > 128 or K % 64 != 0 or N % 32 != 0:
        return 1
    idx = device.index if device.index is not None else torch.cuda.current_device()
    sms = _SM_COUNT.get(idx)
    if sms is None:
        sms = _SM_COUNT[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    tiles = -(-N // 128)
    splits = 1
    for s in (2, 4, 8, 16):
        if (K // 64) % s == 0 and tiles * s <= sms:
            splits = s
    return splits if tiles * 2 <= sms else 1


# ---------------------------------------------------------------- routing
def softmax(x: torch.Tensor) -> torch.Tensor:
    """Row softmax over the last dim in fp32 (REF kernels/softmax.py:40-51)."""
    x = _require(x, "softmax.x", torch.float32)
    y = torch.empty_like(x)
    cols = x.shape[-1]
    with torch.cuda.device(x.device):
        _lib.call("q35_softmax_fwd", x.data_ptr(), y.data_ptr(), x.numel() // cols, cols, _stream(x))
    return y


def cuda_topk(x: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Top-k over the last dim, sorted descending, ties to the lower index
    (REF kernels/moe_routing.py:55-67).  Returns (values fp32, indices int64)."""
    x = _require(x, "cuda_topk.x", torch.float32)
    cols = x.shape[-1]
    rows = x.numel() // cols
    vals = torch.empty(*x.shape[:-1], k, device=x.device, dtype=torch.float32)
    idx = torch.empty(*x.shape[:-1], k, device=x.device, dtype=torch.int64)
    with torch.cuda.device(x.device):
        _lib.call("q35_topk_fwd", x.data_ptr(), vals.data_ptr(), idx.data_ptr(), rows, cols, int(k),
                  _stream(x))
    return vals, idx


def cuda_index_add(target: torch.Tensor, source: torch.Tensor, index: torch.Tensor) -> torch.Tensor:
    """target[index[r]] += source[r], in place (REF kernels/moe_routing.py:103-121)."""
    if not target.is_contiguous():
        raise RuntimeError("cuda_index_add: target must be contiguous (it is updated in place)")
    _require(target, "cuda_index_add.target", (torch.float32, _BF16))
    source = _require(source.to(target.dtype), "cuda_index_add.source", target.dtype)
    index = _require(index.to(torch.int64), "cuda_index_add.index", torch.int64)
    cols = target[0].numel() if target.shape[0] else 0
    code = 0 if target.dtype == torch.float32 else 1
    with torch.cuda.device(target.device):
        _lib.call("q35_index_add", target.data_ptr(), source.data_ptr(), index.data_ptr(),
                  index.numel(), target.shape[0], cols, code, _stream(target))
    return target


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up, elementwise (REF kernels/swiglu.py:56-67)."""
    gate = _require(gate, "swiglu.gate")
    up = _require(up, "swiglu.up")
    out = torch.empty_like(gate)
    with torch.cuda.device(gate.device):
        _lib.call("q35_swiglu_fwd", gate.data_ptr(), up.data_ptr(), out.data_ptr(), gate.numel(),
                  _stream(gate))
    return out


def residual_add(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """a + b elementwise (REF kernels/residual_add.py)."""
    a = _require(a, "residual_add.a")
    b = _require(b, "residual_add.b")
    out = torch.empty_like(a)
    with torch.cuda.device(a.device):
        _lib.call("q35_residual_add_fwd", a.data_ptr(), b.data_ptr(), out.data_ptr(), a.numel(),
                  _stream(a))
    return out


def router_split_weights(gate_weight: torch.Tensor) -> torch.Tensor:
    """bf16 [E, 3H] planes [hi | mid | lo] summing exactly to the fp32 gate weight."""
    wg = _require(gate_weight, "router_split.gate_weight", torch.float32)
    E, H = wg.shape
    w3 = torch.empty(E, 3 * H, device=wg.device, dtype=_BF16)
    with torch.cuda.device(wg.device):
        _lib.call("q35_router_split_weights", wg.data_ptr(), w3.data_ptr(), E, H, _stream(wg))
    return w3


def router_fused_supported(T: int, H: int, E: int, k: int) -> bool:
    """Whether the tensor-core cluster router (q35_router_topk_fused) takes this
    shape: H a multiple of 256, E in (32, 64, 128), k <= 16."""
    return bool(_lib.query("q35_router_fused_supported", T, H, E, k))


def router_topk(x2d: torch.Tensor, gate_weight: torch.Tensor, top_k: int, renorm: bool = True,
                bias: torch.Tensor | None = None, gate_split: torch.Tensor | None = None,
                chunk_counts: bool = False):
    """Fused fp32 router: logits (T,E) fp32, top-k ids (T,k) int32, weights (T,k) fp32.
    With ``gate_split`` (router_split_weights(gate_weight)) the logits run on the
    tensor cores (exact bf16 products, fp32 accumulation); supported shapes take
    the cluster kernel, which also counts the permutation's chunk counts.
    ``chunk_counts=True`` returns a fourth value: the per-128-token-chunk expert
    counts [ceil(T/128), E] int32 for moe_permute_counted, or None when the
    shape takes another router path."""
    x2d = _require(x2d, "router.x")
    wg = _require(gate_weight, "router.gate_weight", torch.float32)
    T, H = x2d.shape
    E = wg.shape[0]
    logits = torch.empty(T, E, device=x2d.device, dtype=torch.float32)
    idx = torch.empty(T, top_k, device=x2d.device, dtype=torch.int32)
    w = torch.empty(T, top_k, device=x2d.device, dtype=torch.float32)
    if bias is not None:
        bias = _require(bias, "router.bias", torch.float32)
    if gate_split is not None and router_fused_supported(T, H, E, top_k):
        gate_split = _require(gate_split, "router.gate_split")
        cc = (torch.empty(max(1, -(-T // 128)), E, device=x2d.device, dtype=torch.int32)
              if chunk_counts else None)
        with torch.cuda.device(x2d.device):
            _lib.call("q35_router_topk_fused", x2d.data_ptr(), gate_split.data_ptr(), _ptr(bias),
                      logits.data_ptr(), idx.data_ptr(), w.data_ptr(), _ptr(cc), T, H, E,
                      int(top_k), 1 if renorm else 0, _stream(x2d))
        return (logits, idx, w, cc) if chunk_counts else (logits, idx, w)
    ws = None
    if gate_split is not None:
        gate_split = _require(gate_split, "router.gate_split")
        ws = torch.empty(max(1, _lib.query("q35_router_workspace", T, H, E)), device=x2d.device,
                         dtype=torch.float32)
    with torch.cuda.device(x2d.device):
        _lib.call("q35_router_topk_fwd", x2d.data_ptr(), wg.data_ptr(), _ptr(gate_split), _ptr(bias),
                  logits.data_ptr(), idx.data_ptr(), w.data_ptr(), T, H, E, int(top_k),
                  1 if renorm else 0, _ptr(ws), _stream(x2d))
    return (logits, idx, w, None) if chunk_counts else (logits, idx, w)


class Permutation:
    """Device arrays of the (expert, token) sort of the routed pairs."""

    __slots__ = ("counts", "offsets", "sorted_tok", "slot_pos", "tile_offsets", "num_experts")

    def __init__(self, counts, offsets, sorted_tok, slot_pos, tile_offsets, num_experts):
        self.counts = counts
        self.offsets = offsets
        self.sorted_tok = sorted_tok
        self.slot_pos = slot_pos
        self.tile_offsets = tile_offsets
        self.num_experts = num_experts


def moe_permute(idx: torch.Tensor, num_experts: int) -> Permutation:
    """Stable (expert, token) sort of top-k ids idx (T,k) int32 (REF modules/moe.py:71-76)."""
    idx = _require(idx, "moe_permute.idx", torch.int32)
    T, k = idx.shape
    dev = idx.device
    i32 = dict(device=dev, dtype=torch.int32)
    counts = torch.empty(num_experts, **i32)
    offsets = torch.empty(num_experts + 1, **i32)
    tile_offsets = torch.empty(num_experts + 1, **i32)
    sorted_tok = torch.empty(T * k, **i32)
    slot_pos = torch.empty(T * k, **i32)
    ws = torch.empty(max(1, _lib.query("q35_moe_permute_workspace", T, num_experts)), **i32)
    with torch.cuda.device(dev):
        _lib.call("q35_moe_permute", idx.data_ptr(), T, k, num_experts, counts.data_ptr(),
                  offsets.data_ptr(), sorted_tok.data_ptr(), slot_pos.data_ptr(),
                  tile_offsets.data_ptr(), ws.data_ptr(), _stream(idx))
    return Permutation(counts, offsets, sorted_tok, slot_pos, tile_offsets, num_experts)


def moe_permute_counted(idx: torch.Tensor, chunk_counts: torch.Tensor, num_experts: int) -> Permutation:
    """moe_permute from the router's per-chunk expert counts (router_topk with
    chunk_counts=True): one launch instead of count + scan + scatter, the same
    bit-exact result."""
    idx = _require(idx, "moe_permute_counted.idx", torch.int32)
    cc = _require(chunk_counts, "moe_permute_counted.chunk_counts", torch.int32)
    T, k = idx.shape
    if tuple(cc.shape) != (max(1, -(-T // 128)), num_experts):
        raise RuntimeError(f"moe_permute_counted: chunk_counts {tuple(cc.shape)} for T={T}")
    dev = idx.device
    i32 = dict(device=dev, dtype=torch.int32)
    counts = torch.empty(num_experts, **i32)
    offsets = torch.empty(num_experts + 1, **i32)
    tile_offsets = torch.empty(num_experts + 1, **i32)
    sorted_tok = torch.empty(T * k, **i32)
    slot_pos = torch.empty(T * k, **i32)
    with torch.cuda.device(dev):
        _lib.call("q35_moe_permute_counted", idx.data_ptr(), T, k, num_experts, cc.data_ptr(),
                  counts.data_ptr(), offsets.data_ptr(), sorted_tok.data_ptr(), slot_pos.data_ptr(),
                  tile_offsets.data_ptr(), _stream(idx))
    return Permutation(counts, offsets, sorted_tok, slot_pos, tile_offsets, num_experts)


def moe_permute_slabs(idx: torch.Tensor, n_slabs: int, slab_rows: int, slab_cnt: torch.Tensor,
                      num_experts: int) -> Permutation:
    """moe_permute over slab-structured rows: idx (n_slabs*slab_rows, k) int32 where
    only the first slab_cnt[s] rows of slab s take part (the expert-parallel
    receive window); rows past a slab's count are ignored whatever they hold."""
    idx = _require(idx, "moe_permute_slabs.idx", torch.int32)
    slab_cnt = _require(slab_cnt, "moe_permute_slabs.slab_cnt", torch.int32)
    R, k = idx.shape
    if R != n_slabs * slab_rows:
        raise RuntimeError(f"moe_permute_slabs: {R} rows for {n_slabs} slabs of {slab_rows}")
    dev = idx.device
    i32 = dict(device=dev, dtype=torch.int32)
    counts = torch.empty(num_experts, **i32)
    offsets = torch.empty(num_experts + 1, **i32)
    tile_offsets = torch.empty(num_experts + 1, **i32)
    sorted_tok = torch.empty(R * k, **i32)
    slot_pos = torch.empty(R * k, **i32)
    ws = torch.empty(max(1, _lib.query("q35_moe_permute_workspace", R, num_experts)), **i32)
    with torch.cuda.device(dev):
        _lib.call("q35_moe_permute_slabs", idx.data_ptr(), n_slabs, slab_rows, slab_cnt.data_ptr(),
                  k, num_experts, counts.data_ptr(), offsets.data_ptr(), sorted_tok.data_ptr(),
                  slot_pos.data_ptr(), tile_offsets.data_ptr(), ws.data_ptr(), _stream(idx))
    return Permutation(counts, offsets, sorted_tok, slot_pos, tile_offsets, num_experts)


def gather_rows(src: torch.Tensor, rows: torch.Tensor, n_dev: torch.Tensor | None = None) -> torch.Tensor:
    """dst[r] = src[rows[r]] for bf16 rows (rows int32); n_dev (device int32) bounds r."""
    src = _require(src, "gather_rows.src")
    rows = _require(rows, "gather_rows.rows", torch.int32)
    n = rows.numel()
    cols = src.shape[-1]
    dst = torch.empty(n, cols, device=src.device, dtype=src.dtype)
    with torch.cuda.device(src.device):
        _lib.call("q35_gather_rows", src.data_ptr(), rows.data_ptr(), dst.data_ptr(), n,
                  _ptr(n_dev), cols, _stream(src))
    return dst


def embedding(ids: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """weight[ids] for int32/int64 ids of any shape (REF kernels/embedding.py),
    ids checked on the device: out-of-range ids give zero rows and a device
    error report instead of a read outside the table."""
    w = _require(weight, "embedding.weight")
    if ids.device != w.device:
        raise RuntimeError("embedding: ids and weight on different devices")
    flat = ids.reshape(-1)
    flat = flat if flat.dtype == torch.int64 else flat.to(torch.int64)
    flat = flat.contiguous()
    V, C = w.shape
    out = torch.empty(flat.numel(), C, device=w.device, dtype=w.dtype)
    with torch.cuda.device(w.device):
        _lib.call("q35_embedding_fwd", w.data_ptr(), flat.data_ptr(), out.data_ptr(), flat.numel(),
                  V, C, _stream(w))
    return out.reshape(*ids.shape, C)


def pack_b_tiles(w: torch.Tensor) -> torch.Tensor:
    """Copy of a bf16 weight [..., rows, K] as contiguous 128 x 64 tiles (the
    layout the grouped GEMMs stream with one 16 KB read per TMA box)."""
    w = _require(w, "pack_b_tiles.w")
    K = w.shape[-1]
    rows = w.numel() // K
    out = torch.empty_like(w)
    with torch.cuda.device(w.device):
        _lib.call("q35_pack_b_tiles", w.data_ptr(), out.data_ptr(), rows, K, _stream(w))
    return out


def grouped_gateup_swiglu(a: torch.Tensor, w_gate_up: torch.Tensor, perm: Permutation,
                          rows_cap: int | None = None,
                          w_packed: torch.Tensor | None = None) -> torch.Tensor:
    """act[r] = silu(a[r] @ Wg[e]^T) * (a[r] @ Wu[e]^T) for the rows of each expert e.
    ``w_packed`` (pack_b_tiles(w_gate_up)) is read instead of w_gate_up if given."""
    a = _require(a, "gate_up.a")
    w = _require(w_gate_up if w_packed is None else w_packed, "gate_up.w")
    E, I2, H = w_gate_up.shape
    R = a.shape[0] if rows_cap is None else rows_cap
    act = torch.empty(R, I2 // 2, device=a.device, dtype=a.dtype)
    with torch.cuda.device(a.device):
        _lib.call("q35_grouped_gemm_gateup_swiglu", a.data_ptr(), w.data_ptr(), act.data_ptr(),
                  perm.offsets.data_ptr(), perm.tile_offsets.data_ptr(), E, R, H, I2 // 2,
                  0 if w_packed is None else 1, _stream(a))
    return act


def grouped_down(act: torch.Tensor, w_down: torch.Tensor, perm: Permutation,
                 w_packed: torch.Tensor | None = None) -> torch.Tensor:
    """y[r] = act[r] @ Wd[e]^T for the rows of each expert e (``w_packed`` as above)."""
    act = _require(act, "down.act")
    w = _require(w_down if w_packed is None else w_packed, "down.w")
    E, H, I = w_down.shape
    R = act.shape[0]
    y = torch.empty(R, H, device=act.device, dtype=act.dtype)
    with torch.cuda.device(act.device):
        _lib.call("q35_grouped_gemm_down", act.data_ptr(), w.data_ptr(), y.data_ptr(),
                  perm.offsets.data_ptr(), perm.tile_offsets.data_ptr(), E, R, H, I,
                  0 if w_packed is None else 1, _stream(act))
    return y


def moe_combine(y: torch.Tensor, weights: torch.Tensor, slot_pos: torch.Tensor,
                residual: torch.Tensor | None, T: int, H: int,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """out[t] = residual[t] + sum_j weights[t,j] * y[slot_pos[t,j]] (fp32 sum, bf16 out)."""
    y = _require(y, "combine.y")
    weights = _require(weights, "combine.weights", torch.float32)
    slot_pos = _require(slot_pos, "combine.slot_pos", torch.int32)
    k = weights.shape[-1]
    if residual is not None:
        residual = _require(residual, "combine.residual", (_BF16, torch.float32))
    r32 = 1 if residual is not None and residual.dtype == torch.float32 else 0
    if out is None:
        out = torch.empty(T, H, device=weights.device, dtype=_BF16)
    elif out.dtype != _BF16 or not out.is_contiguous() or out.numel() != T * H:
        raise RuntimeError("moe_combine: out must be a contiguous bf16 [T, H] tensor")
    with torch.cuda.device(weights.device):
        _lib.call("q35_moe_combine", y.data_ptr(), weights.data_ptr(), slot_pos.data_ptr(),
                  _ptr(residual), r32, out.data_ptr(), T, k, H, _stream(weights))
    return out


# ---------------------------------------------------------------- rotary
def qknorm_mrope(qkv: torch.Tensor, q_w: torch.Tensor, k_w: torch.Tensor,
                 position_ids: torch.Tensor, inv_freq: torch.Tensor, mrope_section,
                 B: int, S: int, Hq: int, Hkv: int, D: int, eps: float, interleaved: bool = False):
    """Fused QK-RMSNorm + mRoPE + head-major split of the fused qkv projection."""
    qkv = _require(qkv, "qknorm_mrope.qkv")
    q_w = _require(q_w, "qknorm_mrope.q_w")
    k_w = _require(k_w, "qknorm_mrope.k_w")
    pos = _require(position_ids.to(torch.int64), "qknorm_mrope.position_ids", torch.int64)
    inv = _require(inv_freq, "qknorm_mrope.inv_freq", torch.float32)
    dev = qkv.device
    q = torch.empty(B, Hq, S, D, device=dev, dtype=_BF16)
    k = torch.empty(B, Hkv, S, D, device=dev, dtype=_BF16)
    v = torch.empty(B, Hkv, S, D, device=dev, dtype=_BF16)
    with torch.cuda.device(dev):
        _lib.call("q35_qknorm_mrope_fwd", qkv.data_ptr(), q_w.data_ptr(), k_w.data_ptr(),
                  pos.data_ptr(), inv.data_ptr(), _lib.sections_arg(mrope_section),
                  1 if interleaved else 0, q.data_ptr(), k.data_ptr(), v.data_ptr(), B, S, Hq, Hkv,
                  D, float(eps), _stream(qkv))
    return q, k, v


def qkv_proj_norm_rope(x: torch.Tensor, w_qkv: torch.Tensor, q_w: torch.Tensor, k_w: torch.Tensor,
                       position_ids: torch.Tensor, inv_freq: torch.Tensor, mrope_section,
                       Hq: int, Hkv: int, eps: float, interleaved: bool = False):
    """q/k/v projection of x (B,S,H) with QK-RMSNorm + mRoPE + head-major split
    in the GEMM epilogue (head_dim 128, no projection bias): the result of
    matmul(x, w_qkv) followed by qknorm_mrope, with the projection kept in fp32
    until the rotated head is written."""
    x = _require(x, "qkv_proj_norm_rope.x")
    w_qkv = _require(w_qkv, "qkv_proj_norm_rope.w_qkv")
    q_w = _require(q_w, "qkv_proj_norm_rope.q_w")
    k_w = _require(k_w, "qkv_proj_norm_rope.k_w")
    pos = _require(position_ids.to(torch.int64), "qkv_proj_norm_rope.position_ids", torch.int64)
    inv = _require(inv_freq, "qkv_proj_norm_rope.inv_freq", torch.float32)
    B, S, H = x.shape
    if w_qkv.shape != ((Hq + 2 * Hkv) * 128, H):
        raise RuntimeError(f"qkv_proj_norm_rope: w_qkv {tuple(w_qkv.shape)} for Hq={Hq} Hkv={Hkv} H={H}")
    dev = x.device
    q = torch.empty(B, Hq, S, 128, device=dev, dtype=_BF16)
    k = torch.empty(B, Hkv, S, 128, device=dev, dtype=_BF16)
    v = torch.empty(B, Hkv, S, 128, device=dev, dtype=_BF16)
    ws = torch.empty(2 * B * S * 64, device=dev, dtype=torch.float32)
    with torch.cuda.device(dev):
        _lib.call("q35_qkv_proj_norm_rope", x.data_ptr(), w_qkv.data_ptr(), q_w.data_ptr(),
                  k_w.data_ptr(), pos.data_ptr(), inv.data_ptr(), _lib.sections_arg(mrope_section),
                  1 if interleaved else 0, q.data_ptr(), k.data_ptr(), v.data_ptr(), B, S, H, Hq,
                  Hkv, float(eps), ws.data_ptr(), _stream(x))
    return q, k, v


def mrope(x: torch.Tensor, position_ids: torch.Tensor, inv_freq: torch.Tensor, mrope_section,
          interleaved: bool = False) -> torch.Tensor:
    """mRoPE on a head-major (B,H,S,D) tensor, cos/sin computed on the fly from
    (3,B,S) positions (replaces apply_mrope, REF kernels/mrope.py:80-104)."""
    x = _require(x, "mrope.x")
    pos = _require(position_ids.to(torch.int64), "mrope.position_ids", torch.int64)
    inv = _require(inv_freq, "mrope.inv_freq", torch.float32)
    B, H, S, D = x.shape
    y = torch.empty_like(x)
    with torch.cuda.device(x.device):
        _lib.call("q35_mrope_fwd", x.data_ptr(), y.data_ptr(), pos.data_ptr(), inv.data_ptr(),
                  _lib.sections_arg(mrope_section), 1 if interleaved else 0, B, H, S, D, _stream(x))
    return y


# ---------------------------------------------------------------- attention
def attention_tokens(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                     causal: bool) -> torch.Tensor:
    """Attention of head-major q (B,Hq,Sq,D), k/v (B,Hkv,Skv,D); returns the
    token-major (B,Sq,Hq*D) output that feeds o_proj directly.  Causal masking
    is bottom-right aligned.  Decode-shaped calls use the split-KV kernel."""
    q = _require(q, "attention.q")
    k = _require(k, "attention.k")
    v = _require(v, "attention.v")
    B, Hq, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    out = torch.empty(B, Sq, Hq * D, device=q.device, dtype=q.dtype)
    with torch.cuda.device(q.device):
        if (not causal or Sq == 1) and (Hq // Hkv) * Sq <= 16:
            n = _lib.query("q35_attn_decode_workspace", B, Hq, Sq, Skv, D)
            ws = torch.empty(max(1, n), device=q.device, dtype=torch.float32)
            _lib.call("q35_attn_decode_fwd", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                      B, Hq, Hkv, Sq, Skv, D, float(scale), ws.data_ptr(), _stream(q))
        else:
            _lib.call("q35_attn_prefill_fwd", q.data_ptr(), k.data_ptr(), v.data_ptr(),
                      out.data_ptr(), None, B, Hq, Hkv, Sq, Skv, D, float(scale),
                      1 if causal else 0, _stream(q))
    return out


def attention_cache(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, kv_len: int,
                    scale: float, causal: bool) -> torch.Tensor:
    """attention_tokens over the first ``kv_len`` rows of preallocated caches
    k_cache/v_cache (B,Hkv,capacity,D); returns the token-major (B,Sq,Hq*D)."""
    q = _require(q, "attention.q")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise RuntimeError("attention_cache: caches must be contiguous [B, Hkv, capacity, D]")
    k_cache = _require(k_cache, "attention.k_cache")
    v_cache = _require(v_cache, "attention.v_cache")
    B, Hq, Sq, D = q.shape
    Hkv, cap = k_cache.shape[1], k_cache.shape[2]
    if kv_len > cap:
        raise RuntimeError(f"attention_cache: {kv_len} rows exceed the capacity {cap}")
    out = torch.empty(B, Sq, Hq * D, device=q.device, dtype=q.dtype)
    with torch.cuda.device(q.device):
        if (not causal or Sq == 1) and (Hq // Hkv) * Sq <= 16:
            n = _lib.query("q35_attn_decode_workspace", B, Hq, Sq, kv_len, D)
            ws = torch.empty(max(1, n), device=q.device, dtype=torch.float32)
            _lib.call("q35_attn_decode_cache_fwd", q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                      out.data_ptr(), B, Hq, Hkv, Sq, kv_len, cap, D, float(scale), ws.data_ptr(),
                      _stream(q))
        else:
            _lib.call("q35_attn_prefill_cache_fwd", q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                      out.data_ptr(), None, B, Hq, Hkv, Sq, kv_len, cap, D, float(scale),
                      1 if causal else 0, _stream(q))
    return out


def kv_append(k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
              offset: int) -> None:
    """Writes k/v (B,Hkv,S,D) into rows [offset, offset+S) of the caches in place."""
    k = _require(k, "kv_append.k")
    v = _require(v, "kv_append.v")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise RuntimeError("kv_append: caches must be contiguous")
    _require(k_cache, "kv_append.k_cache")
    _require(v_cache, "kv_append.v_cache")
    B, Hkv, S, D = k.shape
    with torch.cuda.device(k.device):
        _lib.call("q35_kv_append", k.data_ptr(), v.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                  B, Hkv, S, D, k_cache.shape[2], offset, _stream(k))


def flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                    is_causal: bool = True, num_kv_groups: int = 1) -> torch.Tensor:
    """Reference op signature (REF kernels/flash_attention.py:82-100): returns
    (B,Hq,Sq,D) (a view of the token-major result)."""
    B, Hq, Sq, D = q.shape
    if Hq != k.shape[1] * num_kv_groups:
        raise RuntimeError("flash_attention: Hq must equal Hkv * num_kv_groups")
    out = attention_tokens(q, k, v, scale, is_causal)
    return out.view(B, Sq, Hq, D).transpose(1, 2)


# ---------------------------------------------------------------- vision ops
def layernorm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
              eps: float = 1e-6) -> torch.Tensor:
    """LayerNorm over the last dim, bf16 (REF kernels/layernorm.py:54)."""
    x = _require(x, "layernorm.x")
    weight = _require(weight.to(_BF16), "layernorm.weight")
    bias = None if bias is None else _require(bias.to(_BF16), "layernorm.bias")
    cols = x.shape[-1]
    y = torch.empty_like(x)
    with torch.cuda.device(x.device):
        _lib.call("q35_layernorm_fwd", x.data_ptr(), weight.data_ptr(),
                  None if bias is None else bias.data_ptr(), y.data_ptr(),
                  x.numel() // cols if cols else 0, cols, float(eps), _stream(x))
    return y


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    """GELU with the tanh approximation, bf16 (REF kernels/gelu_tanh.py:49)."""
    x = _require(x, "gelu_tanh.x")
    y = torch.empty_like(x)
    with torch.cuda.device(x.device):
        _lib.call("q35_gelu_tanh_fwd", x.data_ptr(), y.data_ptr(), x.numel(), _stream(x))
    return y


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE on the first cos.shape[-1] dims of x (B,H,S,D); cos/sin
    (B,S,dr) or (S,dr), cast to x's dtype as in the reference (REF
    kernels/rope.py:58-70)."""
    x = _require(x, "rope.x")
    cos = _require(cos.to(x.dtype), "rope.cos")
    sin = _require(sin.to(x.dtype), "rope.sin")
    B, H, S, D = x.shape
    y = torch.empty_like(x)
    with torch.cuda.device(x.device):
        _lib.call("q35_rope_fwd", x.data_ptr(), cos.data_ptr(), sin.data_ptr(), y.data_ptr(),
                  B, H, S, D, cos.shape[-1], 1 if cos.dim() == 3 else 0, _stream(x))
    return y


def conv3d_patch(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """Non-overlapping 3-D patch embedding (stride == kernel size): x (N, C, T, H, W)
    with (T, H, W) the kernel size, weight (E, C, T, H, W) -> (N, E), as a GEMM of
    the flattened patches on the tensor cores (REF kernels/conv3d_patch.py:17-40)."""
    x = _require(x, "conv3d_patch.x")
    w = _require(weight, "conv3d_patch.weight")
    if tuple(x.shape[2:]) != tuple(w.shape[2:]) or x.shape[1] != w.shape[1]:
        raise RuntimeError(f"conv3d_patch: patch {tuple(x.shape[1:])} vs kernel {tuple(w.shape[1:])}")
    N, E = x.shape[0], w.shape[0]
    K = x[0].numel()
    b = None if bias is None else _require(bias.to(_BF16), "conv3d_patch.bias")
    out = torch.empty(N, E, device=x.device, dtype=x.dtype)
    with torch.cuda.device(x.device):
        _lib.call("q35_conv3d_patch_fwd", x.data_ptr(), w.data_ptr(),
                  None if b is None else b.data_ptr(), out.data_ptr(), N, E, K, _stream(x))
    return out


def default_scale(head_dim: int) -> float:
    return head_dim ** -0.5


def device_error_check():
    """Synchronises and raises if any kernel recorded a device-side error."""
    return _lib.device_error_check()


__all__ = [
    "rmsnorm", "matmul", "softmax", "cuda_topk", "cuda_index_add", "swiglu", "residual_add",
    "router_topk", "router_split_weights", "pack_b_tiles", "embedding", "moe_permute", "moe_permute_slabs", "moe_permute_counted", "router_fused_supported", "Permutation", "gather_rows", "grouped_gateup_swiglu",
    "grouped_down", "moe_combine", "qknorm_mrope", "mrope", "attention_tokens",
    "flash_attention", "attention_cache", "kv_append", "device_error_check", "default_scale",
    "layernorm", "gelu_tanh", "apply_rope", "conv3d_patch",
]
