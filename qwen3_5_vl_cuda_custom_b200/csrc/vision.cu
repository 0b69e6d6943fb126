// Vision-tower operators of the reference (bf16 in and out, fp32 math, one
// rounding per output): LayerNorm, GELU (tanh approximation), the
// non-overlapping Conv3d patch embedding and partial rotate-half RoPE.
// They are memory-bound except the patch embedding, which is a GEMM of the
// flattened patches with the flattened filters and runs on the tcgen05 GEMM.
#include "common.cuh"

namespace q35 {
namespace {

__device__ __forceinline__ void ld8(const uint16_t *p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4 *>(p);
  unpack_bf2(u.x, v[0], v[1]);
  unpack_bf2(u.y, v[2], v[3]);
  unpack_bf2(u.z, v[4], v[5]);
  unpack_bf2(u.w, v[6], v[7]);
}
__device__ __forceinline__ void st8(uint16_t *p, const float (&v)[8]) {
  uint4 u;
  u.x = pack_bf2(v[0], v[1]);
  u.y = pack_bf2(v[2], v[3]);
  u.z = pack_bf2(v[4], v[5]);
  u.w = pack_bf2(v[6], v[7]);
  *reinterpret_cast<uint4 *>(p) = u;
}

// y = (x - mean) * rsqrt(var + eps) * w (+ b), var the biased variance (the
// formula of torch.nn.functional.layer_norm, REF kernels/layernorm.py:13-14).
// Warp per row; mean, then the centred sum of squares, then the output
// (passes two and three re-read the row from L1/L2).
__global__ void __launch_bounds__(256) layernorm_kernel(const uint16_t *__restrict__ x,
                                                        const uint16_t *__restrict__ w,
                                                        const uint16_t *__restrict__ b,
                                                        uint16_t *__restrict__ y, int64_t rows,
                                                        int64_t cols, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const uint16_t *xr = x + row * cols;
  float s = 0.f;
  for (int64_t c = lane * 8; c < cols; c += 256) {
    float v[8];
    ld8(xr + c, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) s += v[j];
  }
  const float mean = warp_sum(s) / static_cast<float>(cols);
  float ss = 0.f;
  for (int64_t c = lane * 8; c < cols; c += 256) {
    float v[8];
    ld8(xr + c, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(v[j] - mean, v[j] - mean, ss);
  }
  const float r = 1.0f / sqrtf(warp_sum(ss) / static_cast<float>(cols) + eps);
  uint16_t *yr = y + row * cols;
  for (int64_t c = lane * 8; c < cols; c += 256) {
    float v[8], wv[8], bv[8];
    ld8(xr + c, v);
    ld8(w + c, wv);
    if (b) ld8(b + c, bv);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = (v[j] - mean) * r * wv[j] + (b ? bv[j] : 0.f);
    st8(yr + c, v);
  }
}

// gelu_tanh(x) = 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))
// (torch.nn.functional.gelu(approximate="tanh"), REF kernels/gelu_tanh.py:13-14).
__global__ void __launch_bounds__(256) gelu_tanh_kernel(const uint16_t *__restrict__ x,
                                                        uint16_t *__restrict__ y, int64_t n8) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  float v[8];
  ld8(x + i * 8, v);
  constexpr float kC = 0.7978845608028654f;  // sqrt(2 / pi)
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float a = v[j];
    v[j] = 0.5f * a * (1.f + tanhf(kC * fmaf(0.044715f * a, a * a, a)));
  }
  st8(y + i * 8, v);
}

// Rotate-half RoPE on the first dr of D dims of x (B, H, S, D); the rest pass
// through.  cos/sin bf16 (B, S, dr) when per_batch, else (S, dr); only their
// first half is read, as in the reference (REF kernels/rope.py:12-30).
// Thread = 8 consecutive dims of one (b, h, s) row.
__global__ void __launch_bounds__(256) rope_kernel(const uint16_t *__restrict__ x,
                                                   const uint16_t *__restrict__ cs,
                                                   const uint16_t *__restrict__ sn,
                                                   uint16_t *__restrict__ y, int64_t rows,
                                                   int H, int64_t S, int D, int dr,
                                                   int per_batch) {
  const int vecs = D / 8;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * vecs) return;
  const int64_t row = i / vecs;
  const int d0 = static_cast<int>(i - row * vecs) * 8;
  const int64_t s = row % S, bidx = row / (S * H);
  const uint16_t *xr = x + row * D;
  float v[8];
  ld8(xr + d0, v);
  if (d0 < dr) {
    const int half = dr / 2;
    const int64_t trow = (per_batch ? bidx * S + s : s) * dr;
    const int j0 = d0 < half ? d0 : d0 - half;  // index into the first half of cos/sin
    float c[8], sv[8], pr[8];
    ld8(cs + trow + j0, c);
    ld8(sn + trow + j0, sv);
    ld8(xr + (d0 < half ? d0 + half : d0 - half), pr);  // rotate-half partner
#pragma unroll
    for (int j = 0; j < 8; ++j)
      v[j] = d0 < half ? v[j] * c[j] - pr[j] * sv[j] : v[j] * c[j] + pr[j] * sv[j];
  }
  st8(y + row * D + d0, v);
}

// Vision attention input: the fused projection qkv [S, 3, H, D] (bias already
// added) -> head-major q, k, v [H, S, Dp] with Dp >= D zero-padded, and the
// 2-D rotary on q and k over all D dims (rotate-half, half = D/2; angle of
// dims j and j + D/2 = ang[s, j], REF modules/attention.py:31-39 with
// kernels/rope.py:12-28 and models/common.py:192-195), fp32 math, one
// rounding.  The zero padding lets head dims the attention kernels do not
// take (e.g. 72) run on the D = 128 kernels: padded dims add nothing to a
// score, and the padded output columns are zero.  One warp per (token, head).
__global__ void __launch_bounds__(256) vision_qkv_rope_kernel(
    const uint16_t *__restrict__ qkv, const float *__restrict__ ang, uint16_t *__restrict__ q,
    uint16_t *__restrict__ k, uint16_t *__restrict__ v, int64_t S, int H, int D, int Dp) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (wid >= S * H) return;
  const int64_t s = wid / H;
  const int h = static_cast<int>(wid % H);
  const int half = D / 2;
  const uint16_t *src = qkv + s * 3 * H * D;
  const int64_t dst = (static_cast<int64_t>(h) * S + s) * Dp;
  for (int j = lane; j < Dp; j += 32) {
    float oq = 0.f, ok = 0.f, ov = 0.f;
    if (j < D) {
      const int j0 = j < half ? j : j - half;
      float sn, cs;
      sincosf(ang[s * half + j0], &sn, &cs);
      const float q1 = bf2f(src[h * D + j0]), q2 = bf2f(src[h * D + j0 + half]);
      const float k1 = bf2f(src[(H + h) * D + j0]), k2 = bf2f(src[(H + h) * D + j0 + half]);
      if (j < half) {
        oq = q1 * cs - q2 * sn;
        ok = k1 * cs - k2 * sn;
      } else {
        oq = q2 * cs + q1 * sn;
        ok = k2 * cs + k1 * sn;
      }
      ov = bf2f(src[(2 * H + h) * D + j]);
    }
    q[dst + j] = f2bf(oq);
    k[dst + j] = f2bf(ok);
    v[dst + j] = f2bf(ov);
  }
}

// Token-major attention output [S, H, Dp] -> [S, H, D] (drops the padding).
__global__ void __launch_bounds__(256) unpad_heads_kernel(const uint16_t *__restrict__ x,
                                                          uint16_t *__restrict__ y, int64_t S,
                                                          int H, int D, int Dp) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= S * H * D) return;
  const int64_t sh = i / D;
  const int d = static_cast<int>(i % D);
  y[i] = x[sh * Dp + d];
}

}  // namespace
}  // namespace q35

using namespace q35;

extern "C" int q35_layernorm_fwd(const void *x, const void *w, const void *b, void *y,
                                 int64_t rows, int64_t cols, float eps, q35_stream_t stream) {
  if (!x || !w || !y) return fail(Q35_ERR_INVALID, "layernorm: null pointer");
  if (rows < 0 || cols <= 0 || cols % 8 != 0)
    return fail(Q35_ERR_SHAPE, "layernorm: cols %lld must be a positive multiple of 8",
                (long long)cols);
  if (!aligned16(x) || !aligned16(w) || !aligned16(y) || (b && !aligned16(b)))
    return fail(Q35_ERR_ALIGN, "layernorm: pointers must be 16-byte aligned");
  if (rows == 0) return Q35_OK;
  layernorm_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0,
                     reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t *>(x), static_cast<const uint16_t *>(w),
      static_cast<const uint16_t *>(b), static_cast<uint16_t *>(y), rows, cols, eps);
  Q35_LAUNCH_CHECK("layernorm launch");
  return Q35_OK;
}

extern "C" int q35_gelu_tanh_fwd(const void *x, void *y, int64_t n, q35_stream_t stream) {
  if (!x || !y) return fail(Q35_ERR_INVALID, "gelu_tanh: null pointer");
  if (n < 0 || n % 8 != 0) return fail(Q35_ERR_SHAPE, "gelu_tanh: n %lld (x8)", (long long)n);
  if (!aligned16(x) || !aligned16(y)) return fail(Q35_ERR_ALIGN, "gelu_tanh: alignment");
  if (n == 0) return Q35_OK;
  const int64_t n8 = n / 8;
  gelu_tanh_kernel<<<static_cast<unsigned>((n8 + 255) / 256), 256, 0,
                     reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t *>(x), static_cast<uint16_t *>(y), n8);
  Q35_LAUNCH_CHECK("gelu_tanh launch");
  return Q35_OK;
}

extern "C" int q35_rope_fwd(const void *x, const void *cos_t, const void *sin_t, void *y,
                            int64_t B, int H, int64_t S, int D, int dr, int per_batch,
                            q35_stream_t stream) {
  if (!x || !cos_t || !sin_t || !y) return fail(Q35_ERR_INVALID, "rope: null pointer");
  if (B < 0 || H <= 0 || S < 0 || D <= 0 || D % 8 != 0 || dr <= 0 || dr > D || dr % 16 != 0)
    return fail(Q35_ERR_SHAPE, "rope: D %d (x8), rotary dims %d (x16, <= D)", D, dr);
  if (!aligned16(x) || !aligned16(y) || !aligned16(cos_t) || !aligned16(sin_t))
    return fail(Q35_ERR_ALIGN, "rope: alignment");
  const int64_t rows = B * H * S;
  if (rows == 0) return Q35_OK;
  const int64_t n = rows * (D / 8);
  rope_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0,
                reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t *>(x), static_cast<const uint16_t *>(cos_t),
      static_cast<const uint16_t *>(sin_t), static_cast<uint16_t *>(y), rows, H, S, D, dr,
      per_batch ? 1 : 0);
  Q35_LAUNCH_CHECK("rope launch");
  return Q35_OK;
}

// Non-overlapping Conv3d patch embedding (stride == kernel size): each patch
// flattened to K = C*T*P*P values, out[n, e] = patch[n] . w[e] + bias[e] --
// a GEMM with a bias epilogue on the tensor cores.
extern "C" int q35_gemm_bf16(const void *a, const void *b, const void *bias,
                             const void *residual, void *out, int64_t M, int64_t N,
                             int64_t K, q35_stream_t stream);

extern "C" int q35_conv3d_patch_fwd(const void *patches, const void *w, const void *bias,
                                    void *out, int64_t n_patches, int64_t embed, int64_t K,
                                    q35_stream_t stream) {
  if (!patches || !w || !out) return fail(Q35_ERR_INVALID, "conv3d_patch: null pointer");
  return q35_gemm_bf16(patches, w, bias, nullptr, out, n_patches, embed, K, stream);
}

extern "C" int q35_vision_qkv_rope_pad(const void *qkv, const float *angles, void *q, void *k,
                                       void *v, int64_t S, int H, int D, int Dp,
                                       q35_stream_t stream) {
  if (!qkv || !angles || !q || !k || !v) return fail(Q35_ERR_INVALID, "vision_qkv_rope: null");
  if (S < 0 || H < 1 || D < 2 || D % 2 != 0 || Dp < D)
    return fail(Q35_ERR_SHAPE, "vision_qkv_rope: S %lld H %d D %d (even) Dp %d (>= D)",
                (long long)S, H, D, Dp);
  if (S == 0) return Q35_OK;
  const int64_t warps = S * H;
  vision_qkv_rope_kernel<<<static_cast<unsigned>((warps + 7) / 8), 256, 0,
                           reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t *>(qkv), angles, static_cast<uint16_t *>(q),
      static_cast<uint16_t *>(k), static_cast<uint16_t *>(v), S, H, D, Dp);
  Q35_LAUNCH_CHECK("vision_qkv_rope launch");
  return Q35_OK;
}

extern "C" int q35_unpad_heads(const void *x, void *y, int64_t S, int H, int D, int Dp,
                               q35_stream_t stream) {
  if (!x || !y) return fail(Q35_ERR_INVALID, "unpad_heads: null");
  if (S < 0 || H < 1 || D < 1 || Dp < D) return fail(Q35_ERR_SHAPE, "unpad_heads: bad shape");
  const int64_t n = S * H * D;
  if (n == 0) return Q35_OK;
  unpad_heads_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0,
                       reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t *>(x), static_cast<uint16_t *>(y), S, H, D, Dp);
  Q35_LAUNCH_CHECK("unpad_heads launch");
  return Q35_OK;
}
