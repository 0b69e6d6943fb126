// RMSNorm and the fused QK-norm + mRoPE + head-major split.
//
// Both are HBM-bound: one warp owns one row (or one (token, head) vector),
// loads it with 128-bit accesses, reduces the sum of squares with shuffles and
// writes the normalised row once.  Arithmetic follows the reference's fp32
// formula y = (x * rsqrt(mean(x^2) + eps)) * w with a single final rounding
// (REF cuda_qwen3_vl/kernels/rmsnorm.py:12-17, csrc/rmsnorm_op.cu:8-60).
#include "common.cuh"

namespace q35 {
namespace {

__device__ __forceinline__ void load8(const uint16_t *p, float (&v)[8]) {
  uint4 u = *reinterpret_cast<const uint4 *>(p);
  unpack_bf2(u.x, v[0], v[1]);
  unpack_bf2(u.y, v[2], v[3]);
  unpack_bf2(u.z, v[4], v[5]);
  unpack_bf2(u.w, v[6], v[7]);
}
__device__ __forceinline__ void store8(uint16_t *p, const float (&v)[8]) {
  uint4 u;
  u.x = pack_bf2(v[0], v[1]);
  u.y = pack_bf2(v[2], v[3]);
  u.z = pack_bf2(v[4], v[5]);
  u.w = pack_bf2(v[6], v[7]);
  *reinterpret_cast<uint4 *>(p) = u;
}

// cols == NV * 256: the whole row stays in registers (NV uint4 per lane).
template <int NV>
__global__ void __launch_bounds__(256) rmsnorm_reg_kernel(
    const uint16_t *__restrict__ x, const uint16_t *__restrict__ w,
    uint16_t *__restrict__ y, int64_t rows, float eps) {
  constexpr int cols = NV * 256;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const uint16_t *xr = x + row * cols;
  float v[NV][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    load8(xr + i * 256 + lane * 8, v[i]);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(v[i][j], v[i][j], ss);
  }
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(cols) + eps);
  uint16_t *yr = y + row * cols;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    float wv[8];
    load8(w + i * 256 + lane * 8, wv);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[i][j] = (v[i][j] * r) * wv[j];
    store8(yr + i * 256 + lane * 8, v[i]);
  }
}

// Any cols % 8 == 0: two passes over the row (the second from L1/L2).
__global__ void __launch_bounds__(256) rmsnorm_any_kernel(
    const uint16_t *__restrict__ x, const uint16_t *__restrict__ w,
    uint16_t *__restrict__ y, int64_t rows, int64_t cols, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const uint16_t *xr = x + row * cols;
  float ss = 0.f;
  for (int64_t c = lane * 8; c < cols; c += 256) {
    float v[8];
    load8(xr + c, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(v[j], v[j], ss);
  }
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(cols) + eps);
  uint16_t *yr = y + row * cols;
  for (int64_t c = lane * 8; c < cols; c += 256) {
    float v[8], wv[8];
    load8(xr + c, v);
    load8(w + c, wv);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = (v[j] * r) * wv[j];
    store8(yr + c, v);
  }
}

// fp32 input rows (the layer's fp32 residual stream), bf16 output; the row
// stays in registers as NV float4 pairs per lane when cols == NV * 256.
__global__ void __launch_bounds__(256) rmsnorm_f32in_kernel(
    const float *__restrict__ x, const uint16_t *__restrict__ w,
    uint16_t *__restrict__ y, int64_t rows, int64_t cols, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float *xr = x + row * cols;
  float ss = 0.f;
  for (int64_t c = lane * 8; c < cols; c += 256) {
    const float4 a = *reinterpret_cast<const float4 *>(xr + c);
    const float4 b = *reinterpret_cast<const float4 *>(xr + c + 4);
    ss = fmaf(a.x, a.x, ss); ss = fmaf(a.y, a.y, ss); ss = fmaf(a.z, a.z, ss); ss = fmaf(a.w, a.w, ss);
    ss = fmaf(b.x, b.x, ss); ss = fmaf(b.y, b.y, ss); ss = fmaf(b.z, b.z, ss); ss = fmaf(b.w, b.w, ss);
  }
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(cols) + eps);
  uint16_t *yr = y + row * cols;
  for (int64_t c = lane * 8; c < cols; c += 256) {
    const float4 a = *reinterpret_cast<const float4 *>(xr + c);
    const float4 b = *reinterpret_cast<const float4 *>(xr + c + 4);
    float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w}, wv[8];
    load8(w + c, wv);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = (v[j] * r) * wv[j];
    store8(yr + c, v);
  }
}

// cols == NV * 256 fp32 input: the whole row stays in registers (2 x NV
// float4 per lane), all loads issued before the reduction, one pass.
template <int NV>
__global__ void __launch_bounds__(256) rmsnorm_f32in_reg_kernel(
    const float *__restrict__ x, const uint16_t *__restrict__ w,
    uint16_t *__restrict__ y, int64_t rows, float eps) {
  constexpr int cols = NV * 256;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float *xr = x + row * cols;
  float4 a[NV], b[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    a[i] = *reinterpret_cast<const float4 *>(xr + i * 256 + lane * 8);
    b[i] = *reinterpret_cast<const float4 *>(xr + i * 256 + lane * 8 + 4);
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    ss = fmaf(a[i].x, a[i].x, ss); ss = fmaf(a[i].y, a[i].y, ss);
    ss = fmaf(a[i].z, a[i].z, ss); ss = fmaf(a[i].w, a[i].w, ss);
    ss = fmaf(b[i].x, b[i].x, ss); ss = fmaf(b[i].y, b[i].y, ss);
    ss = fmaf(b[i].z, b[i].z, ss); ss = fmaf(b[i].w, b[i].w, ss);
  }
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(cols) + eps);
  uint16_t *yr = y + row * cols;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    float wv[8];
    load8(w + i * 256 + lane * 8, wv);
    float v[8] = {a[i].x, a[i].y, a[i].z, a[i].w, b[i].x, b[i].y, b[i].z, b[i].w};
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = (v[j] * r) * wv[j];
    store8(yr + i * 256 + lane * 8, v);
  }
}

// Rotary angle table for one token: cos/sin of pos[axis(j)] * inv_freq[j] for
// j < D/2.  axis(j) follows the reference's chunked section layout
// (REF kernels/mrope.py:19-35: sections*2 chunks, chunk i from axis i % 3;
// only the first half is read because rotate-half uses c[..., :half] for both
// halves, REF kernels/mrope.py:38-50) or, with interleaved != 0, the
// HF Qwen3-VL layout (H at j % 3 == 1 below 3*s1, W at j % 3 == 2 below 3*s2).
struct RopeSections {
  int s0, s1, s2;
  int interleaved;
};
__device__ __forceinline__ int rope_axis(int j, const RopeSections &sec) {
  if (sec.interleaved) {
    if ((j % 3) == 1 && j < 3 * sec.s1) return 1;
    if ((j % 3) == 2 && j < 3 * sec.s2) return 2;
    return 0;
  }
  if (j < sec.s0) return 0;
  if (j < sec.s0 + sec.s1) return 1;
  return 2;
}

// One block per token; the block's warps walk the token's heads.  q/k heads
// are RMS-normalised over D (fp32), rotated, rounded once; v heads are copied.
// Output layout is head-major [B, H, S, D].
template <int D>
__global__ void __launch_bounds__(256) qknorm_mrope_kernel(
    const uint16_t *__restrict__ qkv, const uint16_t *__restrict__ qw,
    const uint16_t *__restrict__ kw, const int64_t *__restrict__ pos,
    const float *__restrict__ inv_freq, RopeSections sec,
    uint16_t *__restrict__ q, uint16_t *__restrict__ k,
    uint16_t *__restrict__ v, int64_t B, int64_t S, int Hq, int Hkv,
    float eps) {
  constexpr int HALF = D / 2;
  constexpr int EPL = D / 32;  // elements per lane (2 or 4)
  __shared__ float s_cos[HALF], s_sin[HALF];
  const int64_t t = blockIdx.x;  // token = b * S + s
  const int64_t b = t / S, s = t - b * S;
  const int64_t BS = B * S;
  for (int j = threadIdx.x; j < HALF; j += blockDim.x) {
    const int ax = rope_axis(j, sec);
    const float p = static_cast<float>(pos[ax * BS + t]);
    const float ang = p * inv_freq[j];
    float sn, cs;
    sincosf(ang, &sn, &cs);
    s_cos[j] = cs;
    s_sin[j] = sn;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  const int H = Hq + 2 * Hkv;
  const uint16_t *row = qkv + t * static_cast<int64_t>(H) * D;
  const int j0 = lane * EPL;  // first element of this lane
  for (int h = warp; h < H; h += nwarps) {
    const uint16_t *src = row + h * D + j0;
    float xv[EPL];
    if constexpr (EPL == 4) {
      uint2 u = *reinterpret_cast<const uint2 *>(src);
      unpack_bf2(u.x, xv[0], xv[1]);
      unpack_bf2(u.y, xv[2], xv[3]);
    } else if constexpr (EPL == 2) {
      uint32_t u = *reinterpret_cast<const uint32_t *>(src);
      unpack_bf2(u, xv[0], xv[1]);
    } else {
      xv[0] = bf2f(src[0]);
    }
    uint16_t *dst;
    if (h < Hq + Hkv) {
      const bool is_q = h < Hq;
      const uint16_t *wgt = is_q ? qw : kw;
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) ss = fmaf(xv[e], xv[e], ss);
      ss = warp_sum(ss);
      const float r = 1.0f / sqrtf(ss / static_cast<float>(D) + eps);
#pragma unroll
      for (int e = 0; e < EPL; ++e) xv[e] = (xv[e] * r) * bf2f(wgt[j0 + e]);
      // rotate-half: partner element j +- HALF lives 16 lanes away.
      float pv[EPL];
#pragma unroll
      for (int e = 0; e < EPL; ++e)
        pv[e] = __shfl_xor_sync(0xffffffffu, xv[e], 16);
      const bool first = j0 < HALF;
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        const int jj = (j0 + e) & (HALF - 1);
        const float c = s_cos[jj], sn = s_sin[jj];
        xv[e] = first ? (xv[e] * c - pv[e] * sn) : (xv[e] * c + pv[e] * sn);
      }
      if (is_q)
        dst = q + ((b * Hq + h) * S + s) * D;
      else
        dst = k + ((b * Hkv + (h - Hq)) * S + s) * D;
    } else {
      dst = v + ((b * Hkv + (h - Hq - Hkv)) * S + s) * D;
    }
    if constexpr (EPL == 4) {
      uint2 u;
      u.x = pack_bf2(xv[0], xv[1]);
      u.y = pack_bf2(xv[2], xv[3]);
      *reinterpret_cast<uint2 *>(dst + j0) = u;
    } else if constexpr (EPL == 2) {
      *reinterpret_cast<uint32_t *>(dst + j0) = pack_bf2(xv[0], xv[1]);
    } else {
      dst[j0] = f2bf(xv[0]);
    }
  }
}

// mRoPE on a head-major tensor [B, H, S, D]: one warp per (b, h, s) row.
template <int D>
__global__ void __launch_bounds__(256) mrope_kernel(
    const uint16_t *__restrict__ x, uint16_t *__restrict__ y,
    const int64_t *__restrict__ pos, const float *__restrict__ inv_freq,
    RopeSections sec, int64_t B, int H, int64_t S) {
  constexpr int HALF = D / 2;
  constexpr int EPL = D / 32;
  const int lane = threadIdx.x & 31;
  const int64_t rowi = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (rowi >= B * H * S) return;
  const int64_t s = rowi % S;
  const int64_t b = rowi / (S * H);
  const int64_t t = b * S + s;
  const int64_t BS = B * S;
  const int j0 = lane * EPL;
  float xv[EPL], pv[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) xv[e] = bf2f(x[rowi * D + j0 + e]);
#pragma unroll
  for (int e = 0; e < EPL; ++e) pv[e] = __shfl_xor_sync(0xffffffffu, xv[e], 16);
  const bool first = j0 < HALF;
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    const int jj = (j0 + e) & (HALF - 1);
    const int ax = rope_axis(jj, sec);
    float sn, cs;
    sincosf(static_cast<float>(pos[ax * BS + t]) * inv_freq[jj], &sn, &cs);
    const float o = first ? (xv[e] * cs - pv[e] * sn) : (xv[e] * cs + pv[e] * sn);
    y[rowi * D + j0 + e] = f2bf(o);
  }
}

}  // namespace
}  // namespace q35

using namespace q35;

extern "C" int q35_rmsnorm_fwd(const void *x, const void *w, void *y,
                               int64_t rows, int64_t cols, float eps,
                               q35_stream_t stream) {
  if (!x || !w || !y) return fail(Q35_ERR_INVALID, "rmsnorm: null pointer");
  if (rows < 0 || cols <= 0) return fail(Q35_ERR_SHAPE, "rmsnorm: bad shape");
  if (cols % 8 != 0)
    return fail(Q35_ERR_SHAPE, "rmsnorm: cols %lld not a multiple of 8",
                (long long)cols);
  if (!aligned16(x) || !aligned16(w) || !aligned16(y))
    return fail(Q35_ERR_ALIGN, "rmsnorm: pointers must be 16-byte aligned");
  if (rows == 0) return Q35_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>((rows + 7) / 8);
  auto xp = static_cast<const uint16_t *>(x);
  auto wp = static_cast<const uint16_t *>(w);
  auto yp = static_cast<uint16_t *>(y);
  switch (cols) {
    case 256: rmsnorm_reg_kernel<1><<<grid, 256, 0, s>>>(xp, wp, yp, rows, eps); break;
    case 512: rmsnorm_reg_kernel<2><<<grid, 256, 0, s>>>(xp, wp, yp, rows, eps); break;
    case 1024: rmsnorm_reg_kernel<4><<<grid, 256, 0, s>>>(xp, wp, yp, rows, eps); break;
    case 2048: rmsnorm_reg_kernel<8><<<grid, 256, 0, s>>>(xp, wp, yp, rows, eps); break;
    case 4096: rmsnorm_reg_kernel<16><<<grid, 256, 0, s>>>(xp, wp, yp, rows, eps); break;
    default:
      rmsnorm_any_kernel<<<grid, 256, 0, s>>>(xp, wp, yp, rows, cols, eps);
  }
  Q35_LAUNCH_CHECK("rmsnorm launch");
  return Q35_OK;
}

extern "C" int q35_rmsnorm_f32in_fwd(const float *x, const void *w, void *y,
                                     int64_t rows, int64_t cols, float eps,
                                     q35_stream_t stream) {
  if (!x || !w || !y) return fail(Q35_ERR_INVALID, "rmsnorm_f32in: null pointer");
  if (rows < 0 || cols <= 0 || cols % 8 != 0)
    return fail(Q35_ERR_SHAPE, "rmsnorm_f32in: cols %lld must be a positive multiple of 8",
                (long long)cols);
  if (!aligned16(x) || !aligned16(w) || !aligned16(y))
    return fail(Q35_ERR_ALIGN, "rmsnorm_f32in: pointers must be 16-byte aligned");
  if (rows == 0) return Q35_OK;
  const unsigned grid = static_cast<unsigned>((rows + 7) / 8);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  auto wp = static_cast<const uint16_t *>(w);
  auto yp = static_cast<uint16_t *>(y);
  switch (cols) {
    case 1024: rmsnorm_f32in_reg_kernel<4><<<grid, 256, 0, st>>>(x, wp, yp, rows, eps); break;
    case 2048: rmsnorm_f32in_reg_kernel<8><<<grid, 256, 0, st>>>(x, wp, yp, rows, eps); break;
    case 4096: rmsnorm_f32in_reg_kernel<16><<<grid, 256, 0, st>>>(x, wp, yp, rows, eps); break;
    default: rmsnorm_f32in_kernel<<<grid, 256, 0, st>>>(x, wp, yp, rows, cols, eps);
  }
  Q35_LAUNCH_CHECK("rmsnorm_f32in launch");
  return Q35_OK;
}

extern "C" int q35_qknorm_mrope_fwd(const void *qkv, const void *qw,
                                    const void *kw, const int64_t *positions,
                                    const float *inv_freq,
                                    const int32_t *sections, int interleaved,
                                    void *q, void *k, void *v, int64_t B,
                                    int64_t S, int Hq, int Hkv, int D,
                                    float eps, q35_stream_t stream) {
  if (!qkv || !qw || !kw || !positions || !inv_freq || !sections || !q || !k ||
      !v)
    return fail(Q35_ERR_INVALID, "qknorm_mrope: null pointer");
  if (B < 0 || S < 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0)
    return fail(Q35_ERR_SHAPE, "qknorm_mrope: bad head counts %d/%d", Hq, Hkv);
  if (D != 32 && D != 64 && D != 128)
    return fail(Q35_ERR_UNSUPPORTED, "qknorm_mrope: head_dim %d (32, 64, 128)", D);
  if (sections[0] < 0 || sections[1] < 0 || sections[2] < 0 ||
      sections[0] + sections[1] + sections[2] != D / 2)
    return fail(Q35_ERR_SHAPE, "qknorm_mrope: sections must sum to D/2");
  if (B * S == 0) return Q35_OK;
  RopeSections sec{sections[0], sections[1], sections[2], interleaved ? 1 : 0};
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>(B * S);
  auto args = [&](auto kern) {
    kern<<<grid, 256, 0, s>>>(
        static_cast<const uint16_t *>(qkv), static_cast<const uint16_t *>(qw),
        static_cast<const uint16_t *>(kw), positions, inv_freq, sec,
        static_cast<uint16_t *>(q), static_cast<uint16_t *>(k),
        static_cast<uint16_t *>(v), B, S, Hq, Hkv, eps);
  };
  if (D == 128)
    args(qknorm_mrope_kernel<128>);
  else if (D == 64)
    args(qknorm_mrope_kernel<64>);
  else
    args(qknorm_mrope_kernel<32>);
  Q35_LAUNCH_CHECK("qknorm_mrope launch");
  return Q35_OK;
}

extern "C" int q35_mrope_fwd(const void *x, void *y, const int64_t *positions,
                             const float *inv_freq, const int32_t *sections,
                             int interleaved, int64_t B, int H, int64_t S,
                             int D, q35_stream_t stream) {
  if (!x || !y || !positions || !inv_freq || !sections)
    return fail(Q35_ERR_INVALID, "mrope: null pointer");
  if (D != 32 && D != 64 && D != 128)
    return fail(Q35_ERR_UNSUPPORTED, "mrope: head_dim %d (32, 64, 128)", D);
  if (sections[0] + sections[1] + sections[2] != D / 2)
    return fail(Q35_ERR_SHAPE, "mrope: sections must sum to D/2");
  const int64_t rows = B * H * S;
  if (rows == 0) return Q35_OK;
  RopeSections sec{sections[0], sections[1], sections[2], interleaved ? 1 : 0};
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>((rows + 7) / 8);
  if (D == 128)
    mrope_kernel<128><<<grid, 256, 0, s>>>(static_cast<const uint16_t *>(x),
                                           static_cast<uint16_t *>(y), positions,
                                           inv_freq, sec, B, H, S);
  else if (D == 32)
    mrope_kernel<32><<<grid, 256, 0, s>>>(static_cast<const uint16_t *>(x),
                                          static_cast<uint16_t *>(y), positions,
                                          inv_freq, sec, B, H, S);
  else
    mrope_kernel<64><<<grid, 256, 0, s>>>(static_cast<const uint16_t *>(x),
                                          static_cast<uint16_t *>(y), positions,
                                          inv_freq, sec, B, H, S);
  Q35_LAUNCH_CHECK("mrope launch");
  return Q35_OK;
}
