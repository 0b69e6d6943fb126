// Causal GQA attention: prefill (flash-attention over 128-query blocks) and
// decode (split-KV with a log-sum-exp merge).
//
// Reference: flash_attn_fwd_kernel (REF cuda_qwen3_vl/csrc/
// flash_attention_op.cu:17-135): one thread per query row, fp32 smem tiles,
// BlockM = 16, BlockN = 32, causal mask n > q, kv head = hq / num_kv_groups.
// Here the score and value products run on bf16 tensor-core MMAs with fp32
// accumulation, the online softmax keeps a running max/sum per row in
// registers, and K/V tiles stream through a two-stage cp.async ring.
//
// Masking is bottom-right aligned: query i of Sq sees keys j <= i + (Skv - Sq).
// With Sq == Skv that is the reference's causal rule; the reference's
// is_causal = (S_q == S_k) choice (REF modules/attention.py:95) is made by the
// caller.
#include <float.h>

#include "common.cuh"

namespace q35 {
namespace {


__device__ __forceinline__ void cp_async16(void *smem, const void *gmem,
                                           bool pred) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s),
               "l"(gmem), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Row-major [rows][D] bf16 tile (element offset), 16-byte chunks XOR-swizzled
// by the row so that ldmatrix row reads hit distinct banks.
template <int D>
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  constexpr int kChunks = D / 8;
  constexpr int kMask = kChunks >= 8 ? 7 : kChunks - 1;
  return static_cast<uint32_t>(row * D + ((chunk ^ (row & kMask)) << 3));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0,
                                        uint32_t &r1, uint32_t &r2,
                                        uint32_t &r3) {
  asm volatile(
      "ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
      : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
      : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0,
                                          uint32_t &r1, uint32_t &r2,
                                          uint32_t &r3) {
  asm volatile(
      "ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
      : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
      : "r"(addr));
}
// D += A(16x16 bf16) * B(16x8 bf16), fp32 accumulate.
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0,
                                         uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Copies rows [r0, r0 + ROWS) of a [n_rows][D] bf16 matrix into a swizzled
// smem tile; rows >= n_rows are zero-filled.
template <int D, int ROWS, int NTHREADS>
__device__ __forceinline__ void load_tile_async(uint16_t *tile,
                                                const uint16_t *src,
                                                int64_t r0, int64_t n_rows,
                                                int tid) {
#pragma unroll
  for (int i = tid; i < ROWS * (D / 8); i += NTHREADS) {
    const int r = i / (D / 8), c = i % (D / 8);
    const int64_t gr = r0 + r;
    const bool ok = gr < n_rows;
    const uint16_t *g = src + (ok ? gr : 0) * D + c * 8;
    cp_async16(tile + swz<D>(r, c), g, ok);
  }
}

// ------------------------------------------------------------------ prefill
constexpr int kPM = 128;  // query rows per CTA (8 warps x 16)
constexpr int kPN = 64;   // keys per tile
constexpr int kPThreads = 256;
template <int D>
constexpr int prefill_smem() { return (kPM + 4 * kPN) * D * 2; }  // Q + 2 x (K, V)

template <int D>
__global__ void __launch_bounds__(kPThreads, 2) attn_prefill_kernel(
    const uint16_t *__restrict__ q, const uint16_t *__restrict__ k,
    const uint16_t *__restrict__ v, uint16_t *__restrict__ out,
    float *__restrict__ lse, int Hq, int Hkv, int64_t Sq, int64_t Skv, int64_t kv_cap,
    float scale_log2, float scale, int causal) {
  extern __shared__ __align__(128) uint16_t smem_attn[];
  uint16_t *sQ = smem_attn;
  uint16_t *sK = sQ + kPM * D;       // [2][kPN][D]
  uint16_t *sV = sK + 2 * kPN * D;   // [2][kPN][D]

  const int n_mblocks = static_cast<int>((Sq + kPM - 1) / kPM);
  // Heaviest (last) query blocks first: better tail balance under causality.
  const int mb = n_mblocks - 1 - static_cast<int>(blockIdx.x);
  const int bh = blockIdx.y;
  const int b = bh / Hq, hq = bh % Hq;
  const int hk = hq / (Hq / Hkv);
  const int64_t m0 = static_cast<int64_t>(mb) * kPM;
  const uint16_t *qg = q + (static_cast<int64_t>(b) * Hq + hq) * Sq * D;
  // a kv head holds kv_cap rows in memory, the first Skv of them valid
  const uint16_t *kg = k + (static_cast<int64_t>(b) * Hkv + hk) * kv_cap * D;
  const uint16_t *vg = v + (static_cast<int64_t>(b) * Hkv + hk) * kv_cap * D;
  const int64_t diag = Skv - Sq;  // key limit of query i is i + diag

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  int64_t kv_end = Skv;
  if (causal) kv_end = min(Skv, m0 + kPM + diag);
  const int n_tiles = kv_end > 0 ? static_cast<int>((kv_end + kPN - 1) / kPN) : 0;

  load_tile_async<D, kPM, kPThreads>(sQ, qg, m0, Sq, tid);
  if (n_tiles > 0) {
    load_tile_async<D, kPN, kPThreads>(sK, kg, 0, Skv, tid);
    load_tile_async<D, kPN, kPThreads>(sV, vg, 0, Skv, tid);
  }
  cp_async_commit();

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float row_m[2] = {-FLT_MAX, -FLT_MAX}, row_l[2] = {0.f, 0.f};
  uint32_t qf[D / 16][4];

  const int g = lane >> 2, t4 = lane & 3;
  const int64_t qrow0 = m0 + warp * 16 + g;  // rows qrow0 and qrow0 + 8
  const uint32_t sQa = static_cast<uint32_t>(__cvta_generic_to_shared(sQ));
  const uint32_t sKa = static_cast<uint32_t>(__cvta_generic_to_shared(sK));
  const uint32_t sVa = static_cast<uint32_t>(__cvta_generic_to_shared(sV));

  for (int it = 0; it < n_tiles; ++it) {
    const int st = it & 1;
    if (it + 1 < n_tiles) {
      load_tile_async<D, kPN, kPThreads>(sK + (st ^ 1) * kPN * D, kg,
                                      static_cast<int64_t>(it + 1) * kPN, Skv, tid);
      load_tile_async<D, kPN, kPThreads>(sV + (st ^ 1) * kPN * D, vg,
                                      static_cast<int64_t>(it + 1) * kPN, Skv, tid);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (it == 0) {
      // Q fragments for this warp's 16 rows, kept in registers.
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const int r = warp * 16 + (lane & 15);
        const int c = kk * 2 + (lane >> 4);
        ldsm_x4(sQa + swz<D>(r, c) * 2, qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }
    const int64_t n0 = static_cast<int64_t>(it) * kPN;
    // S = Q K^T : 16 x 64 per warp.
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
    const uint32_t kbase = sKa + st * kPN * D * 2;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        const int r = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = kk * 2 + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kbase + swz<D>(r, c) * 2, b0, b1, b2, b3);
        mma16816(s[2 * np], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1);
        mma16816(s[2 * np + 1], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b2, b3);
      }
    }
    // Mask: keys beyond Skv, and (causal) keys beyond each row's limit.
    const bool need_mask =
        (n0 + kPN > Skv) || (causal && n0 + kPN - 1 > m0 + warp * 16 + diag);
    if (need_mask) {
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int64_t key = n0 + nt * 8 + 2 * t4 + (e & 1);
          const int64_t qi = qrow0 + ((e >> 1) << 3);
          if (key >= Skv || (causal && key > qi + diag)) s[nt][e] = -INFINITY;
        }
    }
    // Online softmax (base-2 exponent, scale folded in).
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float mx = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) mx = fmaxf(mx, fmaxf(s[nt][2 * h], s[nt][2 * h + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(row_m[h], mx);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = exp2f((row_m[h] - m_use) * scale_log2);
      row_m[h] = m_new;
      float sum = 0.f;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        s[nt][2 * h] = exp2f((s[nt][2 * h] - m_use) * scale_log2);
        s[nt][2 * h + 1] = exp2f((s[nt][2 * h + 1] - m_use) * scale_log2);
        sum += s[nt][2 * h] + s[nt][2 * h + 1];
      }
      row_l[h] = row_l[h] * alpha + sum;
#pragma unroll
      for (int dt = 0; dt < D / 8; ++dt) {
        o[dt][2 * h] *= alpha;
        o[dt][2 * h + 1] *= alpha;
      }
    }
    // O += P V : P re-packed from the S accumulators as A fragments.
    const uint32_t vbase = sVa + st * kPN * D * 2;
#pragma unroll
    for (int j = 0; j < 4; ++j) {  // 16 keys per step
      const uint32_t a0 = pack_bf2(s[2 * j][0], s[2 * j][1]);
      const uint32_t a1 = pack_bf2(s[2 * j][2], s[2 * j][3]);
      const uint32_t a2 = pack_bf2(s[2 * j + 1][0], s[2 * j + 1][1]);
      const uint32_t a3 = pack_bf2(s[2 * j + 1][2], s[2 * j + 1][3]);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {  // two 8-wide d tiles per ldmatrix
        const int r = j * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int c = dp * 2 + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vbase + swz<D>(r, c) * 2, b0, b1, b2, b3);
        mma16816(o[2 * dp], a0, a1, a2, a3, b0, b1);
        mma16816(o[2 * dp + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  // Normalise and store token-major: out[b, s, hq*D + d].
  const int64_t ld = static_cast<int64_t>(Hq) * D;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float l = row_l[h];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    const int64_t qi = qrow0 + 8 * h;
    if (qi >= Sq) continue;
    const float inv = l > 0.f ? 1.0f / l : 0.f;
    uint16_t *orow = out + (static_cast<int64_t>(b) * Sq + qi) * ld + hq * D;
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt)
      *reinterpret_cast<uint32_t *>(orow + dt * 8 + 2 * t4) =
          pack_bf2(o[dt][2 * h] * inv, o[dt][2 * h + 1] * inv);
    if (lse && t4 == 0)
      lse[(static_cast<int64_t>(b) * Hq + hq) * Sq + qi] =
          l > 0.f ? row_m[h] * scale + logf(l) : -INFINITY;
  }
}

// ------------------------------------------------------------------ decode
// CTA = (b, kv head, split, row group).  The R = (Hq/Hkv) * Sq query rows that
// share the kv head form one 16-row MMA tile (row = head_in_group * Sq + s).
// 4 warps walk 32-key tiles of the split round-robin, each with a private
// two-stage cp.async K/V ring; the warps' (max, sum, O) partials are merged in
// shared memory and written to the workspace, and a second kernel merges the
// splits with their log-sum-exp weights.
constexpr int kDN = 32;      // keys per warp tile
constexpr int kDWarps = 4;
constexpr int kDThreads = kDWarps * 32;
template <int D>
constexpr int decode_smem() { return kDWarps * 2 * 2 * kDN * D * 2; }  // warps x stages x (K,V)

struct DecodeShape {
  int Hq, Hkv, G;    // G = Hq / Hkv
  int64_t Sq, Skv;
  int64_t kv_cap;    // rows per kv head in memory (>= Skv)
  int R;             // G * Sq rows per kv head
  int n_splits;
  int64_t split_len;
  float scale_log2;
};

template <int D>
__global__ void __launch_bounds__(kDThreads) attn_decode_kernel(
    const uint16_t *__restrict__ q, const uint16_t *__restrict__ k,
    const uint16_t *__restrict__ v, float *__restrict__ ws, DecodeShape sh) {
  extern __shared__ __align__(128) uint16_t smem_dec[];
  const int split = blockIdx.x;
  const int bh = blockIdx.y;
  const int rg = blockIdx.z;  // row group of 16
  const int b = bh / sh.Hkv, hk = bh % sh.Hkv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int64_t k0 = static_cast<int64_t>(split) * sh.split_len;
  const int64_t k1 = min(sh.Skv, k0 + sh.split_len);
  const uint16_t *kg = k + (static_cast<int64_t>(b) * sh.Hkv + hk) * sh.kv_cap * D;
  const uint16_t *vg = v + (static_cast<int64_t>(b) * sh.Hkv + hk) * sh.kv_cap * D;
  uint16_t *wK = smem_dec + warp * (2 * 2 * kDN * D);  // [stage][K|V][kDN][D]

  // Q fragments straight from global: row r -> (head hq = hk*G + r / Sq, s = r % Sq).
  uint32_t qf[D / 16][4];
  {
    const int r_lo = rg * 16 + g, r_hi = r_lo + 8;
    auto qptr = [&](int r) -> const uint16_t * {
      if (r >= sh.R) return nullptr;
      const int hq = hk * sh.G + r / static_cast<int>(sh.Sq);
      const int64_t s = r % sh.Sq;
      return q + ((static_cast<int64_t>(b) * sh.Hq + hq) * sh.Sq + s) * D;
    };
    const uint16_t *plo = qptr(r_lo), *phi = qptr(r_hi);
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const int c0 = kk * 16 + 2 * t4;
      qf[kk][0] = plo ? *reinterpret_cast<const uint32_t *>(plo + c0) : 0u;
      qf[kk][1] = phi ? *reinterpret_cast<const uint32_t *>(phi + c0) : 0u;
      qf[kk][2] = plo ? *reinterpret_cast<const uint32_t *>(plo + c0 + 8) : 0u;
      qf[kk][3] = phi ? *reinterpret_cast<const uint32_t *>(phi + c0 + 8) : 0u;
    }
  }

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float row_m[2] = {-INFINITY, -INFINITY}, row_l[2] = {0.f, 0.f};

  const int64_t n_tiles = (k1 > k0) ? (k1 - k0 + kDN - 1) / kDN : 0;
  // Warp w handles tiles w, w + 4, ...
  auto issue = [&](int64_t tile, int stage) {
    uint16_t *sk = wK + stage * 2 * kDN * D;
    uint16_t *sv = sk + kDN * D;
    const int64_t r0 = k0 + tile * kDN;
#pragma unroll
    for (int i = lane; i < kDN * (D / 8); i += 32) {
      const int r = i / (D / 8), c = i % (D / 8);
      const int64_t gr = r0 + r;
      const bool ok = gr < k1;
      cp_async16(sk + swz<D>(r, c), kg + (ok ? gr : 0) * D + c * 8, ok);
      cp_async16(sv + swz<D>(r, c), vg + (ok ? gr : 0) * D + c * 8, ok);
    }
  };
  int64_t my_tile = warp;
  if (my_tile < n_tiles) issue(my_tile, 0);
  cp_async_commit();
  for (int step = 0; my_tile < n_tiles; my_tile += kDWarps, ++step) {
    const int st = step & 1;
    if (my_tile + kDWarps < n_tiles) issue(my_tile + kDWarps, st ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncwarp();
    const uint32_t kb = static_cast<uint32_t>(__cvta_generic_to_shared(wK + st * 2 * kDN * D));
    const uint32_t vb = kb + kDN * D * 2;
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk)
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        const int r = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = kk * 2 + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kb + swz<D>(r, c) * 2, b0, b1, b2, b3);
        mma16816(s[2 * np], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1);
        mma16816(s[2 * np + 1], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b2, b3);
      }
    const int64_t n0 = k0 + my_tile * kDN;
    if (n0 + kDN > k1) {
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (n0 + nt * 8 + 2 * t4 + (e & 1) >= k1) s[nt][e] = -INFINITY;
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float mx = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) mx = fmaxf(mx, fmaxf(s[nt][2 * h], s[nt][2 * h + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(row_m[h], mx);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = exp2f((row_m[h] - m_use) * sh.scale_log2);
      row_m[h] = m_new;
      float sum = 0.f;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        s[nt][2 * h] = exp2f((s[nt][2 * h] - m_use) * sh.scale_log2);
        s[nt][2 * h + 1] = exp2f((s[nt][2 * h + 1] - m_use) * sh.scale_log2);
        sum += s[nt][2 * h] + s[nt][2 * h + 1];
      }
      row_l[h] = row_l[h] * alpha + sum;
#pragma unroll
      for (int dt = 0; dt < D / 8; ++dt) {
        o[dt][2 * h] *= alpha;
        o[dt][2 * h + 1] *= alpha;
      }
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint32_t a0 = pack_bf2(s[2 * j][0], s[2 * j][1]);
      const uint32_t a1 = pack_bf2(s[2 * j][2], s[2 * j][3]);
      const uint32_t a2 = pack_bf2(s[2 * j + 1][0], s[2 * j + 1][1]);
      const uint32_t a3 = pack_bf2(s[2 * j + 1][2], s[2 * j + 1][3]);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        const int r = j * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int c = dp * 2 + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vb + swz<D>(r, c) * 2, b0, b1, b2, b3);
        mma16816(o[2 * dp], a0, a1, a2, a3, b0, b1);
        mma16816(o[2 * dp + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncwarp();
  }
  cp_async_wait<0>();
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    row_l[h] += __shfl_xor_sync(0xffffffffu, row_l[h], 1);
    row_l[h] += __shfl_xor_sync(0xffffffffu, row_l[h], 2);
  }
  __syncthreads();
  // Merge the 4 warps' partials through shared memory (reusing the K/V ring).
  float *sm = reinterpret_cast<float *>(smem_dec);  // [warp][16 rows][2 + D]
  constexpr int kRowF = 2 + D;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = g + 8 * h;
    float *dst = sm + (warp * 16 + r) * kRowF;
    if (t4 == 0) {
      dst[0] = row_m[h];
      dst[1] = row_l[h];
    }
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt) {
      dst[2 + dt * 8 + 2 * t4] = o[dt][2 * h];
      dst[2 + dt * 8 + 2 * t4 + 1] = o[dt][2 * h + 1];
    }
  }
  __syncthreads();
  // 128 threads: thread = (row r = tid / 8, column slice c = tid % 8 of D/8).
  {
    constexpr int kSl = D / 8;
    const int r = tid >> 3, cs = (tid & 7) * kSl;
    const int rr = rg * 16 + r;
    float M = -INFINITY;
    for (int w = 0; w < kDWarps; ++w) M = fmaxf(M, sm[(w * 16 + r) * kRowF]);
    const float Mu = (M == -INFINITY) ? 0.f : M;
    float L = 0.f, acc[kSl];
#pragma unroll
    for (int i = 0; i < kSl; ++i) acc[i] = 0.f;
    for (int w = 0; w < kDWarps; ++w) {
      const float *src = sm + (w * 16 + r) * kRowF;
      const float f = exp2f((src[0] - Mu) * sh.scale_log2);
      L += src[1] * f;
#pragma unroll
      for (int i = 0; i < kSl; ++i) acc[i] += src[2 + cs + i] * f;
    }
    if (rr < sh.R) {
      // workspace row: [(b*Hkv + hk) * R + rr][split] x (2 + D)
      float *dst = ws + ((static_cast<int64_t>(bh) * sh.R + rr) * sh.n_splits + split) * kRowF;
      if (cs == 0) {
        dst[0] = M;
        dst[1] = L;
      }
#pragma unroll
      for (int i = 0; i < kSl; ++i) dst[2 + cs + i] = acc[i];
    }
  }
}

// One warp per (b, kv head, row): merges the splits and writes out[b, s, hq*D].
template <int D>
__global__ void __launch_bounds__(256) attn_decode_merge_kernel(
    const float *__restrict__ ws, uint16_t *__restrict__ out, DecodeShape sh,
    int64_t total_rows) {
  const int lane = threadIdx.x & 31;
  const int64_t gr = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (gr >= total_rows) return;
  constexpr int kRowF = 2 + D;
  const int64_t bh = gr / sh.R;
  const int rr = static_cast<int>(gr % sh.R);
  const int b = static_cast<int>(bh / sh.Hkv), hk = static_cast<int>(bh % sh.Hkv);
  const float *src = ws + gr * sh.n_splits * kRowF;
  float M = -INFINITY;
  for (int s = 0; s < sh.n_splits; ++s) M = fmaxf(M, src[s * kRowF]);
  const float Mu = (M == -INFINITY) ? 0.f : M;
  constexpr int EPL = D / 32;
  float L = 0.f, acc[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) acc[i] = 0.f;
  for (int s = 0; s < sh.n_splits; ++s) {
    const float *p = src + s * kRowF;
    const float f = exp2f((p[0] - Mu) * sh.scale_log2);
    L += p[1] * f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) acc[i] += p[2 + lane * EPL + i] * f;
  }
  const float inv = L > 0.f ? 1.0f / L : 0.f;
  const int hq = hk * sh.G + rr / static_cast<int>(sh.Sq);
  const int64_t sidx = rr % sh.Sq;
  uint16_t *o = out + (static_cast<int64_t>(b) * sh.Sq + sidx) * sh.Hq * D + hq * D + lane * EPL;
#pragma unroll
  for (int i = 0; i < EPL; ++i) o[i] = f2bf(acc[i] * inv);
}

DecodeShape decode_shape(int64_t B, int Hq, int Hkv, int64_t Sq, int64_t Skv,
                         float scale) {
  DecodeShape sh{};
  sh.Hq = Hq;
  sh.Hkv = Hkv;
  sh.G = Hq / Hkv;
  sh.Sq = Sq;
  sh.Skv = Skv;
  sh.kv_cap = Skv;
  sh.R = static_cast<int>(sh.G * Sq);
  const int64_t groups = B * Hkv * ((sh.R + 15) / 16);
  const int64_t want = (4LL * 148 + groups - 1) / (groups > 0 ? groups : 1);
  const int64_t max_splits = (Skv + 255) / 256;
  int64_t ns = want < 1 ? 1 : want;
  if (ns > max_splits) ns = max_splits;
  if (ns < 1) ns = 1;
  sh.split_len = ((Skv + ns - 1) / ns + kDN - 1) / kDN * kDN;
  if (sh.split_len < kDN) sh.split_len = kDN;
  sh.n_splits = static_cast<int>((Skv + sh.split_len - 1) / sh.split_len);
  if (sh.n_splits < 1) sh.n_splits = 1;
  sh.scale_log2 = scale * 1.4426950408889634f;
  return sh;
}

}  // namespace
}  // namespace q35

using namespace q35;

int q35_attn_prefill_tc(const void *q, const void *k, const void *v, void *out,
                        float *lse, int64_t B, int Hq, int Hkv, int64_t Sq,
                        int64_t Skv, int64_t kv_cap, float scale, int causal,
                        q35_stream_t stream);

static int attn_prefill_impl(const void *q, const void *k, const void *v, void *out, float *lse,
                             int64_t B, int Hq, int Hkv, int64_t Sq, int64_t Skv, int64_t kv_cap,
                             int D, float scale, int causal, q35_stream_t stream) {
  if (!q || !k || !v || !out) return fail(Q35_ERR_INVALID, "attn_prefill: null");
  if (kv_cap < Skv) return fail(Q35_ERR_SHAPE, "attn_prefill: kv capacity below Skv");
  if (D != 32 && D != 64 && D != 128)
    return fail(Q35_ERR_UNSUPPORTED, "attn_prefill: head_dim %d (32, 64 or 128)", D);
  if (B < 0 || Sq < 0 || Skv < 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0)
    return fail(Q35_ERR_SHAPE, "attn_prefill: bad shape");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
    return fail(Q35_ERR_ALIGN, "attn_prefill: pointers not 16-byte aligned");
  if (B * Sq == 0) return Q35_OK;
  if (B * Hq > 65535) return fail(Q35_ERR_SHAPE, "attn_prefill: B*Hq > 65535");
  if (D == 128)  // tcgen05 path
    return q35_attn_prefill_tc(q, k, v, out, lse, B, Hq, Hkv, Sq, Skv, kv_cap, scale, causal,
                               stream);
  dim3 grid(static_cast<unsigned>((Sq + kPM - 1) / kPM), static_cast<unsigned>(B * Hq));
  auto run = [&](auto kern, int smem) -> int {
    { const int _st = ensure_smem_attr(reinterpret_cast<const void *>(kern), smem); if (_st) return _st; }
    kern<<<grid, kPThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t *>(q), static_cast<const uint16_t *>(k),
        static_cast<const uint16_t *>(v), static_cast<uint16_t *>(out), lse, Hq,
        Hkv, Sq, Skv, kv_cap, scale * 1.4426950408889634f, scale, causal ? 1 : 0);
    return Q35_OK;
  };
  int st;
  if (D == 128) st = run(attn_prefill_kernel<128>, prefill_smem<128>());
  else if (D == 64) st = run(attn_prefill_kernel<64>, prefill_smem<64>());
  else st = run(attn_prefill_kernel<32>, prefill_smem<32>());
  if (st) return st;
  Q35_LAUNCH_CHECK("attn_prefill launch");
  return Q35_OK;
}

extern "C" int q35_attn_prefill_fwd(const void *q, const void *k, const void *v,
                                    void *out, float *lse, int64_t B, int Hq,
                                    int Hkv, int64_t Sq, int64_t Skv, int D,
                                    float scale, int causal,
                                    q35_stream_t stream) {
  return attn_prefill_impl(q, k, v, out, lse, B, Hq, Hkv, Sq, Skv, Skv, D, scale, causal, stream);
}

extern "C" int q35_attn_prefill_cache_fwd(const void *q, const void *k_cache,
                                          const void *v_cache, void *out, float *lse, int64_t B,
                                          int Hq, int Hkv, int64_t Sq, int64_t Skv,
                                          int64_t kv_cap, int D, float scale, int causal,
                                          q35_stream_t stream) {
  return attn_prefill_impl(q, k_cache, v_cache, out, lse, B, Hq, Hkv, Sq, Skv, kv_cap, D, scale,
                           causal, stream);
}

extern "C" int64_t q35_attn_decode_workspace(int64_t B, int Hq, int64_t Sq,
                                             int64_t Skv, int D) {
  if (Hq <= 0 || D <= 0) return 0;
  // Upper bound over any Hkv dividing Hq: rows * splits * (2 + D).
  const int64_t splits = (Skv + 255) / 256 + 1;
  return B * Hq * (Sq > 0 ? Sq : 1) * splits * (2 + static_cast<int64_t>(D)) +
         16 * (2 + static_cast<int64_t>(D)) * splits * B;
}

static int attn_decode_impl(const void *q, const void *k, const void *v, void *out, int64_t B,
                            int Hq, int Hkv, int64_t Sq, int64_t Skv, int64_t kv_cap, int D,
                            float scale, float *workspace, q35_stream_t stream) {
  if (!q || !k || !v || !out || !workspace)
    return fail(Q35_ERR_INVALID, "attn_decode: null pointer");
  if (kv_cap < Skv) return fail(Q35_ERR_SHAPE, "attn_decode: kv capacity below Skv");
  if (D != 32 && D != 64 && D != 128)
    return fail(Q35_ERR_UNSUPPORTED, "attn_decode: head_dim %d (32, 64 or 128)", D);
  if (B < 0 || Sq < 1 || Skv < 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0)
    return fail(Q35_ERR_SHAPE, "attn_decode: bad shape");
  if (static_cast<int64_t>(Hq / Hkv) * Sq > 16)
    return fail(Q35_ERR_SHAPE, "attn_decode: (Hq/Hkv)*Sq must be <= 16");
  if (!aligned16(k) || !aligned16(v) || !aligned16(q))
    return fail(Q35_ERR_ALIGN, "attn_decode: pointers not 16-byte aligned");
  if (B == 0) return Q35_OK;
  if (B * Hkv > 65535) return fail(Q35_ERR_SHAPE, "attn_decode: B*Hkv > 65535");
  DecodeShape sh = decode_shape(B, Hq, Hkv, Sq, Skv, scale);
  sh.kv_cap = kv_cap;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  dim3 grid(sh.n_splits, static_cast<unsigned>(B * Hkv), (sh.R + 15) / 16);
  const int64_t rows = B * Hkv * sh.R;
  const unsigned mgrid = static_cast<unsigned>((rows + 7) / 8);
  auto run = [&](auto kern, auto merge, int smem) -> int {
    { const int _st = ensure_smem_attr(reinterpret_cast<const void *>(kern), smem); if (_st) return _st; }
    kern<<<grid, kDThreads, smem, s>>>(
        static_cast<const uint16_t *>(q), static_cast<const uint16_t *>(k),
        static_cast<const uint16_t *>(v), workspace, sh);
    Q35_LAUNCH_CHECK("attn_decode launch");
    merge<<<mgrid, 256, 0, s>>>(workspace, static_cast<uint16_t *>(out), sh, rows);
    return Q35_OK;
  };
  int st;
  if (D == 128) st = run(attn_decode_kernel<128>, attn_decode_merge_kernel<128>, decode_smem<128>());
  else if (D == 64) st = run(attn_decode_kernel<64>, attn_decode_merge_kernel<64>, decode_smem<64>());
  else st = run(attn_decode_kernel<32>, attn_decode_merge_kernel<32>, decode_smem<32>());
  if (st) return st;
  Q35_LAUNCH_CHECK("attn_decode merge launch");
  return Q35_OK;
}

extern "C" int q35_attn_decode_fwd(const void *q, const void *k, const void *v,
                                   void *out, int64_t B, int Hq, int Hkv,
                                   int64_t Sq, int64_t Skv, int D, float scale,
                                   float *workspace, q35_stream_t stream) {
  return attn_decode_impl(q, k, v, out, B, Hq, Hkv, Sq, Skv, Skv, D, scale, workspace, stream);
}

extern "C" int q35_attn_decode_cache_fwd(const void *q, const void *k_cache, const void *v_cache,
                                         void *out, int64_t B, int Hq, int Hkv, int64_t Sq,
                                         int64_t Skv, int64_t kv_cap, int D, float scale,
                                         float *workspace, q35_stream_t stream) {
  return attn_decode_impl(q, k_cache, v_cache, out, B, Hq, Hkv, Sq, Skv, kv_cap, D, scale,
                          workspace, stream);
}

// dst[b, h, offset + s, :] = src[b, h, s, :] for a [B, Hkv, cap, D] cache; one
// warp per (b, h, s) row, 16-byte vectors.
__global__ void __launch_bounds__(256) kv_append_kernel(const uint16_t *__restrict__ src,
                                                         uint16_t *__restrict__ dst,
                                                         int64_t rows, int64_t S, int64_t D,
                                                         int64_t cap, int64_t offset) {
  const int lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int64_t bh = r / S, s = r - bh * S;
  const uint4 *sp = reinterpret_cast<const uint4 *>(src + r * D);
  uint4 *dp = reinterpret_cast<uint4 *>(dst + (bh * cap + offset + s) * D);
  for (int64_t c = lane; c < D / 8; c += 32) dp[c] = sp[c];
}

extern "C" int q35_kv_append(const void *k_new, const void *v_new, void *k_cache, void *v_cache,
                             int64_t B, int Hkv, int64_t S, int D, int64_t cap, int64_t offset,
                             q35_stream_t stream) {
  if (B < 0 || Hkv <= 0 || S < 0 || D <= 0 || D % 8 != 0 || offset < 0 || offset + S > cap)
    return fail(Q35_ERR_SHAPE, "kv_append: offset %lld + %lld rows exceed capacity %lld",
                (long long)offset, (long long)S, (long long)cap);
  if (B * S == 0) return Q35_OK;  // nothing to append (empty tensors may have null pointers)
  if (!k_new || !v_new || !k_cache || !v_cache) return fail(Q35_ERR_INVALID, "kv_append: null");
  if (!aligned16(k_new) || !aligned16(v_new) || !aligned16(k_cache) || !aligned16(v_cache))
    return fail(Q35_ERR_ALIGN, "kv_append: pointers not 16-byte aligned");
  const int64_t rows = B * Hkv * S;
  if (rows == 0) return Q35_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>((rows + 7) / 8);
  kv_append_kernel<<<grid, 256, 0, st>>>(static_cast<const uint16_t *>(k_new),
                                         static_cast<uint16_t *>(k_cache), rows, S, D, cap, offset);
  kv_append_kernel<<<grid, 256, 0, st>>>(static_cast<const uint16_t *>(v_new),
                                         static_cast<uint16_t *>(v_cache), rows, S, D, cap, offset);
  Q35_LAUNCH_CHECK("kv_append launch");
  return Q35_OK;
}
