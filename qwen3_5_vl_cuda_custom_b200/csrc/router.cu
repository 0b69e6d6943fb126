// MoE router: fp32 gate GEMV + softmax + top-k + renormalise, fused.
//
// Reference chain (REF cuda_qwen3_vl/modules/moe.py:60-65): router_logits =
// matmul(x, gate_weight); p = softmax(logits.float()); top_vals, top_idx =
// topk(p, k) (sorted descending, ties to the lower index: strict '>' in
// REF csrc/moe_routing_op.cu:36-53); top_vals /= top_vals.sum(-1).
//
// One CTA owns 32 tokens and all experts.  256 threads = 8 warps; warp w holds
// tokens 4w..4w+3 and lane l experts l, l+32, ...  The K (hidden) dimension is
// streamed through shared memory 32 columns at a time, converting x from bf16
// to fp32 on the way in; every logit is a sequential fp32 FMA chain over h
// (a fixed order, so results are run-to-run deterministic).  Softmax and top-k
// then run on the warp's registers with shuffles.
#include <float.h>

#include "common.cuh"

namespace q35 {
namespace {

constexpr int kTokPerCta = 32;
constexpr int kKc = 32;

// Warp-wide argmax over (value, index) pairs; ties resolve to the lower index.
__device__ __forceinline__ void warp_argmax(float &v, int &i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) {
      v = ov;
      i = oi;
    }
  }
}

template <int EPT>  // experts per lane: E <= 32 * EPT
__global__ void __launch_bounds__(256) router_kernel(
    const uint16_t *__restrict__ x, const float *__restrict__ wg,
    const float *__restrict__ bias, float *__restrict__ logits,
    int32_t *__restrict__ idx_out, float *__restrict__ w_out, int64_t T, int H,
    int E, int k, int renorm) {
  constexpr int EMAX = 32 * EPT;
  __shared__ float xs[kTokPerCta][kKc + 1];
  __shared__ float ws[EMAX][kKc + 1];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kTokPerCta;

  float acc[4][EPT];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < EPT; ++j) acc[i][j] = 0.f;

  for (int h0 = 0; h0 < H; h0 += kKc) {
    // x tile: 32 tokens x 32 columns, 4 bf16 per thread.
    {
      const int r = threadIdx.x >> 3, c = (threadIdx.x & 7) * 4;
      const int64_t t = t0 + r;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      if (t < T) {
        const uint2 u =
            *reinterpret_cast<const uint2 *>(x + t * H + h0 + c);
        unpack_bf2(u.x, a0, a1);
        unpack_bf2(u.y, a2, a3);
      }
      xs[r][c] = a0;
      xs[r][c + 1] = a1;
      xs[r][c + 2] = a2;
      xs[r][c + 3] = a3;
    }
    // gate tile: E rows x 32 columns of fp32.
    for (int q = threadIdx.x; q < EMAX * (kKc / 4); q += 256) {
      const int e = q / (kKc / 4), c = (q % (kKc / 4)) * 4;
      const float4 f = e < E ? *reinterpret_cast<const float4 *>(
                                   wg + static_cast<int64_t>(e) * H + h0 + c)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
      ws[e][c] = f.x;
      ws[e][c + 1] = f.y;
      ws[e][c + 2] = f.z;
      ws[e][c + 3] = f.w;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < kKc; ++kk) {
      float xv[4], wv[EPT];
#pragma unroll
      for (int i = 0; i < 4; ++i) xv[i] = xs[warp * 4 + i][kk];
#pragma unroll
      for (int j = 0; j < EPT; ++j) wv[j] = ws[lane + 32 * j][kk];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < EPT; ++j) acc[i][j] = fmaf(xv[i], wv[j], acc[i][j]);
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t t = t0 + warp * 4 + i;
    if (t >= T) break;  // warp-uniform
    float l[EPT];
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
      const int e = lane + 32 * j;
      if (e < E) {
        l[j] = acc[i][j] + (bias ? bias[e] : 0.f);
        logits[t * E + e] = l[j];
      } else {
        l[j] = -INFINITY;  // padding expert: exp() == 0, never selected
      }
    }
    float m = -FLT_MAX;
#pragma unroll
    for (int j = 0; j < EPT; ++j) m = fmaxf(m, l[j]);
    m = warp_max(m);
    float p[EPT], s = 0.f;
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
      p[j] = expf(l[j] - m);
      s += p[j];
    }
    s = warp_sum(s);
#pragma unroll
    for (int j = 0; j < EPT; ++j) p[j] = (lane + 32 * j < E) ? p[j] / s : -2.f;

    // k rounds of warp argmax; a taken entry is knocked out with -1 (p >= 0).
    float sel_v = 0.f, tot = 0.f;
    int sel_i = 0;
    for (int r = 0; r < k; ++r) {
      float bv = -1.f;
      int bi = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < EPT; ++j)
        if (p[j] > bv) {
          bv = p[j];
          bi = lane + 32 * j;
        }
      warp_argmax(bv, bi);
      if ((bi & 31) == lane) {
#pragma unroll
        for (int j = 0; j < EPT; ++j)
          if (lane + 32 * j == bi) p[j] = -1.f;
      }
      if (lane == r) {
        sel_v = bv;
        sel_i = bi;
      }
      tot += bv;
    }
    if (lane < k) {
      idx_out[t * k + lane] = sel_i;
      w_out[t * k + lane] = renorm ? sel_v / tot : sel_v;
    }
  }
}

// Softmax + top-k + renormalise of the tensor-core router's logits: one warp
// per token, lane l holds experts l, l+32, ...; the logits are the sum of the
// split-K partial planes (+ bias), written to `logits`.
template <int EPT>
__global__ void __launch_bounds__(256) topk_from_logits_kernel(
    const float *__restrict__ partials, int n_partials, float *__restrict__ logits,
    const float *__restrict__ bias, int32_t *__restrict__ idx_out,
    float *__restrict__ w_out, int64_t T, int E, int k, int renorm) {
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  float l[EPT];
#pragma unroll
  for (int j = 0; j < EPT; ++j) {
    const int e = lane + 32 * j;
    if (e < E) {
      // Partial K planes summed in a fixed order (deterministic).
      float v = partials[t * E + e];
      for (int q = 1; q < n_partials; ++q) v += partials[(q * T + t) * E + e];
      if (bias) v += bias[e];
      l[j] = v;
      logits[t * E + e] = v;
    } else {
      l[j] = -INFINITY;
    }
  }
  float m = -FLT_MAX;
#pragma unroll
  for (int j = 0; j < EPT; ++j) m = fmaxf(m, l[j]);
  m = warp_max(m);
  float p[EPT], s = 0.f;
#pragma unroll
  for (int j = 0; j < EPT; ++j) {
    p[j] = expf(l[j] - m);
    s += p[j];
  }
  s = warp_sum(s);
#pragma unroll
  for (int j = 0; j < EPT; ++j) p[j] = (lane + 32 * j < E) ? p[j] / s : -2.f;
  float sel_v = 0.f, tot = 0.f;
  int sel_i = 0;
  for (int r = 0; r < k; ++r) {
    float bv = -1.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < EPT; ++j)
      if (p[j] > bv) {
        bv = p[j];
        bi = lane + 32 * j;
      }
    warp_argmax(bv, bi);
    if ((bi & 31) == lane) {
#pragma unroll
      for (int j = 0; j < EPT; ++j)
        if (lane + 32 * j == bi) p[j] = -1.f;
    }
    if (lane == r) {
      sel_v = bv;
      sel_i = bi;
    }
    tot += bv;
  }
  if (lane < k) {
    idx_out[t * k + lane] = sel_i;
    w_out[t * k + lane] = renorm ? sel_v / tot : sel_v;
  }
}

// w3[e] = [lo | mid | hi] bf16 planes with lo + mid + hi == w[e] exactly:
// hi = rn(w), mid = rn(w - hi), lo = rn(w - hi - mid); each remainder is exact
// in fp32 and each plane holds the next 8 significant bits of w's 24.  The
// small planes come first so the tensor core accumulates them while the
// running sum is still small.
__global__ void split_weights_kernel(const float *__restrict__ wg,
                                     uint16_t *__restrict__ w3, int E, int H) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(E) * H) return;
  const int64_t e = i / H, h = i % H;
  const float w = wg[i];
  const uint16_t hi = f2bf(w);
  const float r1 = w - bf2f(hi);
  const uint16_t mid = f2bf(r1);
  const float r2 = r1 - bf2f(mid);
  const uint16_t lo = f2bf(r2);
  uint16_t *row = w3 + e * 3 * static_cast<int64_t>(H);
  row[h] = lo;
  row[H + h] = mid;
  row[2 * H + h] = hi;
}

// Standalone row softmax (fp32), one warp per row.
__global__ void __launch_bounds__(256) softmax_kernel(const float *__restrict__ x,
                                                      float *__restrict__ y,
                                                      int64_t rows, int cols) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float *xr = x + row * cols;
  float m = -FLT_MAX;
  for (int c = lane; c < cols; c += 32) m = fmaxf(m, xr[c]);
  m = warp_max(m);
  float s = 0.f;
  for (int c = lane; c < cols; c += 32) s += expf(xr[c] - m);
  s = warp_sum(s);
  for (int c = lane; c < cols; c += 32) y[row * cols + c] = expf(xr[c] - m) / s;
}

// Standalone row top-k (fp32 values), one warp per row, k rounds of argmax.
__global__ void __launch_bounds__(256) topk_kernel(const float *__restrict__ x,
                                                   float *__restrict__ vals,
                                                   int64_t *__restrict__ idx,
                                                   int64_t rows, int cols, int k) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float *xr = x + row * cols;
  int taken[16];
  for (int r = 0; r < k; ++r) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int c = lane; c < cols; c += 32) {
      bool used = false;
      for (int q = 0; q < r; ++q) used |= (taken[q] == c);
      const float v = xr[c];
      if (!used && (v > bv || bi == 0x7fffffff)) {
        bv = v;
        bi = c;
      }
    }
    warp_argmax(bv, bi);
    taken[r] = bi;
    if (lane == 0) {
      vals[row * k + r] = bv;
      idx[row * k + r] = bi;
    }
  }
}

}  // namespace
}  // namespace q35

using namespace q35;

extern "C" int q35_router_logits_tc(const void *x, const void *w3,
                                    float *partials, int64_t T, int H, int E,
                                    int k_splits, q35_stream_t stream);

// Split-K factor of the tensor-core router: 4 fresh accumulators when the
// 3H/64 k-blocks divide evenly, else 1.
static int router_splits(int H) { return ((3 * H / 64) % 4 == 0) ? 4 : 1; }

extern "C" int64_t q35_router_workspace(int64_t T, int H, int E) {
  return static_cast<int64_t>(router_splits(H)) * T * E;
}

extern "C" int q35_router_split_weights(const float *wg, void *w3, int E,
                                        int H, q35_stream_t stream) {
  if (!wg || !w3) return fail(Q35_ERR_INVALID, "router_split_weights: null pointer");
  if (E <= 0 || H <= 0) return fail(Q35_ERR_SHAPE, "router_split_weights: bad shape");
  const int64_t n = static_cast<int64_t>(E) * H;
  split_weights_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0,
                         reinterpret_cast<cudaStream_t>(stream)>>>(
      wg, static_cast<uint16_t *>(w3), E, H);
  Q35_LAUNCH_CHECK("router_split_weights launch");
  return Q35_OK;
}

extern "C" int q35_router_topk_fwd(const void *x, const float *wg,
                                   const void *wg_split, const float *bias,
                                   float *logits, int32_t *idx, float *weights,
                                   int64_t T, int H, int E, int k, int renorm,
                                   float *workspace, q35_stream_t stream) {
  if (!x || !wg || !logits || !idx || !weights)
    return fail(Q35_ERR_INVALID, "router: null pointer");
  if (T < 0 || H <= 0 || H % kKc != 0)
    return fail(Q35_ERR_SHAPE, "router: hidden %d must be a multiple of %d", H,
                kKc);
  if (E < 1 || E > 256)
    return fail(Q35_ERR_UNSUPPORTED, "router: num_experts %d (1..256)", E);
  if (k < 1 || k > 16 || k > E)
    return fail(Q35_ERR_SHAPE, "router: top_k %d (1..16, <= E)", k);
  if (!aligned16(wg) || !aligned16(x))
    return fail(Q35_ERR_ALIGN, "router: x / gate weight not 16-byte aligned");
  if (T == 0) return Q35_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (wg_split != nullptr && H % 64 == 0 && E % 32 == 0) {
    // Tensor-core logits, then softmax / top-k on the fp32 logits.
    if (!workspace)
      return fail(Q35_ERR_INVALID, "router: the tensor-core path needs a workspace");
    const int ns = router_splits(H);
    int st = q35_router_logits_tc(x, wg_split, workspace, T, H, E, ns, stream);
    if (st) return st;
    const unsigned g2 = static_cast<unsigned>((T + 7) / 8);
#define Q35_TOPK_CASE(EPT)                                                     \
  case EPT:                                                                    \
    topk_from_logits_kernel<EPT><<<g2, 256, 0, s>>>(workspace, ns, logits,    \
                                                    bias, idx, weights, T, E, \
                                                    k, renorm);                \
    break;
    switch ((E + 31) / 32) {
      Q35_TOPK_CASE(1)
      Q35_TOPK_CASE(2)
      Q35_TOPK_CASE(3)
      Q35_TOPK_CASE(4)
      Q35_TOPK_CASE(5)
      Q35_TOPK_CASE(6)
      Q35_TOPK_CASE(7)
      Q35_TOPK_CASE(8)
    }
#undef Q35_TOPK_CASE
    Q35_LAUNCH_CHECK("router topk launch");
    return Q35_OK;
  }
  const unsigned grid = static_cast<unsigned>((T + kTokPerCta - 1) / kTokPerCta);
  auto xp = static_cast<const uint16_t *>(x);
#define Q35_ROUTER_CASE(EPT)                                              \
  case EPT:                                                               \
    router_kernel<EPT><<<grid, 256, 0, s>>>(xp, wg, bias, logits, idx,    \
                                            weights, T, H, E, k, renorm);    \
    break;
  switch ((E + 31) / 32) {
    Q35_ROUTER_CASE(1)
    Q35_ROUTER_CASE(2)
    Q35_ROUTER_CASE(3)
    Q35_ROUTER_CASE(4)
    Q35_ROUTER_CASE(5)
    Q35_ROUTER_CASE(6)
    Q35_ROUTER_CASE(7)
    Q35_ROUTER_CASE(8)
  }
#undef Q35_ROUTER_CASE
  Q35_LAUNCH_CHECK("router launch");
  return Q35_OK;
}

extern "C" int q35_softmax_fwd(const float *x, float *y, int64_t rows, int cols,
                               q35_stream_t stream) {
  if (!x || !y) return fail(Q35_ERR_INVALID, "softmax: null pointer");
  if (rows < 0 || cols <= 0 || cols > 1 << 20)
    return fail(Q35_ERR_SHAPE, "softmax: bad shape");
  if (rows == 0) return Q35_OK;
  softmax_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0,
                   reinterpret_cast<cudaStream_t>(stream)>>>(x, y, rows, cols);
  Q35_LAUNCH_CHECK("softmax launch");
  return Q35_OK;
}

extern "C" int q35_topk_fwd(const float *x, float *vals, int64_t *idx,
                            int64_t rows, int cols, int k, q35_stream_t stream) {
  if (!x || !vals || !idx) return fail(Q35_ERR_INVALID, "topk: null pointer");
  if (rows < 0 || cols <= 0 || k < 1 || k > 16 || k > cols)
    return fail(Q35_ERR_SHAPE, "topk: k %d cols %d (k <= 16, k <= cols)", k, cols);
  if (rows == 0) return Q35_OK;
  topk_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0,
                reinterpret_cast<cudaStream_t>(stream)>>>(x, vals, idx, rows,
                                                          cols, k);
  Q35_LAUNCH_CHECK("topk launch");
  return Q35_OK;
}
