// Prefill attention on tcgen05 (head_dim 128): S = Q K^T and O += P V run on
// the 5th-generation tensor cores with S, P and O in tensor memory.
//
// Reference: flash_attn_fwd_kernel (REF cuda_qwen3_vl/csrc/
// flash_attention_op.cu:17-135, one thread per query row on CUDA cores).
//
// CTA = one 128-query tile of one head; it walks the 128-key tiles the causal
// mask leaves (bottom-right aligned: query i sees keys j <= i + Skv - Sq).
// 192 threads:
//   warp 0 lane 0 : TMA producer.  Q once (two 64-column halves, 128-byte
//                   swizzle), then K and V tiles into a 2-stage ring.
//   warp 1 lane 0 : MMA issuer.  S_j = Q K_j^T (M=N=K=128) into TMEM buffer
//                   j%2, then O += P_{j-1} V_{j-1} with P read from TMEM (A
//                   operand) and V from shared memory as an MN-major operand.
//                   Issuing S_j before PV_{j-1} overlaps the tensor core with
//                   the softmax of tile j-1.  Warp 1 owns the 512 TMEM columns.
//   warps 2-5      : softmax.  Thread = query row (TMEM lane): tcgen05.ld of
//                   the 128 scores, mask, row max, exp2, row sum, bf16 P
//                   stored back over its S buffer with tcgen05.st.  The running
//                   max is only raised (and O rescaled in TMEM) when it grows
//                   by more than 2^8 in exp2 units, so P stays <= 256 and the
//                   O correction is rare; the result is exact in real
//                   arithmetic.  At the end: O / l, bf16, token-major store.
// Every mbarrier wait is bounded (sm100::mbar_wait); on timeout the kernel
// records DEV_ERR_WAIT_TIMEOUT and unwinds.
#include "sm100.cuh"

namespace q35 {
namespace {

constexpr int kTile = 128;                    // queries per CTA, keys per tile
constexpr int kHalfBytes = kTile * 64 * 2;    // one 64-column half of a tile
constexpr int kQOff = 0;                      // Q: 2 halves
constexpr int kKOff = kQOff + 2 * kHalfBytes; // K: 2 stages x 2 halves
constexpr int kVOff = kKOff + 4 * kHalfBytes; // V: 2 stages x 2 halves
constexpr int kBarOff = kVOff + 4 * kHalfBytes;
constexpr int kSmem = 1024 + kBarOff + 16 * 8;
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;           // O [0,128), S0 [128,256), S1 [256,384)

// Softmax exponentials, split between two pipes: half on the MUFU unit
// (ex2.approx), half on the FMA pipes.  exp2_fma: x = i + f with i = floor(x),
// 2^f from a degree-3 polynomial fitted to 2^f on [0, 1) (relative-error
// least squares on Chebyshev nodes, max relative error 7.8e-5, below the 2^-9
// rounding P gets when it is packed to bf16), 2^i added to the exponent bits.
__device__ __forceinline__ float exp2_mufu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float exp2_fma(float x) {
  const float xc = fmaxf(x, -126.f);
  const float fi = floorf(xc);
  const float f = xc - fi;
  const float p = fmaf(fmaf(fmaf(0.07790717f, f, 0.22623320f), f, 0.69577712f), f, 0.99992782f);
  const float r = __int_as_float(__float_as_int(p) + (static_cast<int>(fi) << 23));
  return x < -126.f ? 0.f : r;
}

// Paired exp2 on the FMA pipes for two scores at once (Blackwell f32x2
// arithmetic): x = i + f with i = round-to-nearest(x) (the 1.5 * 2^23 shift
// trick), f in [-0.5, 0.5], 2^f from a degree-3 polynomial fitted to 2^f on
// that interval (iteratively reweighted least squares on the relative error,
// max relative error 7.5e-5), and i added to the exponent field of the result.
// Inputs are clamped at -125 so the exponent field never underflows.
__device__ __forceinline__ float2 exp2_fma2(float2 x) {
  x.x = fmaxf(x.x, -125.f);
  x.y = fmaxf(x.y, -125.f);
  const float2 shift = make_float2(12582912.f, 12582912.f);
  const float2 xr = __fadd2_rn(x, shift);                     // 1.5*2^23 + i
  const float2 xi = __fadd2_rn(xr, make_float2(-12582912.f, -12582912.f));
  const float2 f = __ffma2_rn(xi, make_float2(-1.f, -1.f), x);  // x - i
  float2 p = __ffma2_rn(make_float2(0.05517146f, 0.05517146f), f,
                        make_float2(0.24261086f, 0.24261086f));
  p = __ffma2_rn(p, f, make_float2(0.69326097f, 0.69326097f));
  p = __ffma2_rn(p, f, make_float2(0.99992812f, 0.99992812f));
  // the low mantissa bits of xr hold i; shifted by 23 they are i * 2^23 (mod 2^32)
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(xr.x) << 23)),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(xr.y) << 23)));
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

struct AttnParams {
  int Hq, Hkv;
  int64_t Sq, Skv;
  int n_mblocks;
  float sl2;    // scale * log2(e)
  float scale;
  int causal;
  int64_t kv_cap;  // rows per kv head in memory (>= Skv)
  uint16_t *out;
  float *lse;
  int *err;
};

__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                   const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kBarOff);
  uint64_t *q_full = bars + 0;
  uint64_t *kv_full = bars + 1;   // [2]
  uint64_t *kv_empty = bars + 3;  // [2]
  uint64_t *s_full = bars + 5;    // [2]
  uint64_t *p_full = bars + 7;    // [2]
  uint64_t *o_done = bars + 9;
  uint64_t *drain = bars + 10;
  uint32_t *s_tmem = reinterpret_cast<uint32_t *>(bars + 12);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mb = p.n_mblocks - 1 - static_cast<int>(blockIdx.x);  // heavy first
  const int bh = blockIdx.y;
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int hk = h / (p.Hq / p.Hkv);
  const int64_t m0 = static_cast<int64_t>(mb) * kTile;
  const int64_t diag = p.Skv - p.Sq;
  int64_t kv_end = p.Skv;
  if (p.causal) kv_end = min(p.Skv, m0 + kTile + diag);
  const int n_tiles = kv_end > 0 ? static_cast<int>((kv_end + kTile - 1) / kTile) : 0;
  const int32_t q_row = static_cast<int32_t>((static_cast<int64_t>(b) * p.Hq + h) * p.Sq + m0);
  const int32_t kv_row = static_cast<int32_t>((static_cast<int64_t>(b) * p.Hkv + hk) * p.kv_cap);

  if (threadIdx.x == 0) {
    sm100::mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(&kv_full[i], 1);
      sm100::mbar_init(&kv_empty[i], 1);
      sm100::mbar_init(&s_full[i], 1);
      sm100::mbar_init(&p_full[i], 128);
    }
    sm100::mbar_init(o_done, 1);
    sm100::mbar_init(drain, 1);
    sm100::fence_mbar_init();
    sm100::prefetch_tensormap(&tmQ);
    sm100::prefetch_tensormap(&tmK);
    sm100::prefetch_tensormap(&tmV);
  }
  if (warp == 1) sm100::tmem_alloc(s_tmem, kTmemCols);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 0 && lane == 0 && n_tiles > 0) {
    // ------------------------------------------------ TMA producer
    sm100::mbar_arrive_expect_tx(q_full, 2 * kHalfBytes);
    sm100::tma_load_2d(smem + kQOff, &tmQ, q_full, 0, q_row);
    sm100::tma_load_2d(smem + kQOff + kHalfBytes, &tmQ, q_full, 64, q_row);
    for (int j = 0; j < n_tiles; ++j) {
      const int st = j & 1;
      if (!sm100::mbar_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1)) {
        report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 301, j, 0);
        break;
      }
      uint8_t *sk = smem + kKOff + st * 2 * kHalfBytes;
      uint8_t *sv = smem + kVOff + st * 2 * kHalfBytes;
      const int32_t r = kv_row + j * kTile;
      sm100::mbar_arrive_expect_tx(&kv_full[st], 4 * kHalfBytes);
      sm100::tma_load_2d(sk, &tmK, &kv_full[st], 0, r);
      sm100::tma_load_2d(sk + kHalfBytes, &tmK, &kv_full[st], 64, r);
      sm100::tma_load_2d(sv, &tmV, &kv_full[st], 0, r);
      sm100::tma_load_2d(sv + kHalfBytes, &tmV, &kv_full[st], 64, r);
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_s = sm100::idesc_bf16_f32(kTile, kTile);
    constexpr uint32_t idesc_pv = sm100::idesc_bf16_f32(kTile, 128, 0, 1);
    bool ok = n_tiles > 0;
    if (ok && !sm100::mbar_wait(q_full, 0)) {
      report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 302, 0, 0);
      ok = false;
    }
    const uint32_t sq = sm100::smem_u32(smem + kQOff);
    auto issue_pv = [&](int i) -> bool {
      const int st = i & 1;
      if (!sm100::mbar_wait(&p_full[st], (i >> 1) & 1)) {
        report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 303, i, 0);
        return false;
      }
      sm100::tc_fence_after();
      const uint32_t p_tmem = tmem + 128 + st * 128;
      const uint32_t sv = sm100::smem_u32(smem + kVOff + st * 2 * kHalfBytes);
#pragma unroll
      for (int kk = 0; kk < kTile / 16; ++kk) {
        // V as the MN-major B operand: 16 keys = two 8-row swizzle atoms
        // (2048 B); the second 64-wide d half sits one half-tile further.
        const uint64_t bdesc = sm100::sw128_mnmajor_desc(sv + kk * 2048, kHalfBytes, 1024);
        sm100::mma_bf16_ts(tmem, p_tmem + kk * 8, bdesc, idesc_pv, (i > 0 || kk > 0) ? 1u : 0u);
      }
      sm100::mma_commit(o_done);
      sm100::mma_commit(&kv_empty[st]);
      return true;
    };
    for (int j = 0; j < n_tiles && ok; ++j) {
      const int st = j & 1;
      if (!sm100::mbar_wait(&kv_full[st], (j >> 1) & 1)) {
        report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 304, j, 0);
        ok = false;
        break;
      }
      sm100::tc_fence_after();
      const uint32_t sk = sm100::smem_u32(smem + kKOff + st * 2 * kHalfBytes);
      const uint32_t s_tm = tmem + 128 + st * 128;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = (kk >> 2) * kHalfBytes;
        const uint64_t ad = sm100::sw128_kmajor_desc(sq + off) + 2 * (kk & 3);
        const uint64_t bd = sm100::sw128_kmajor_desc(sk + off) + 2 * (kk & 3);
        sm100::mma_bf16_ss(s_tm, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
      }
      sm100::mma_commit(&s_full[st]);
      if (j >= 1 && !issue_pv(j - 1)) {
        ok = false;
        break;
      }
    }
    if (ok) issue_pv(n_tiles - 1);
    sm100::mma_commit(drain);
    if (!sm100::mbar_wait(drain, 0)) report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 305, 0, 0);
  } else if (warp >= 2) {
    // ------------------------------------------------ softmax + epilogue
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int64_t qi = m0 + row;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int st = j & 1;
      if (!sm100::mbar_wait(&s_full[st], (j >> 1) & 1)) {
        report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 306, j, row);
        ok = false;
        break;
      }
      sm100::tc_fence_after();
      const uint32_t sb = tmem + lane_base + 128 + st * 128;
      float s[kTile];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        sm100::tmem_ld32(sb + c * 32, r);
        sm100::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c * 32 + i] = __uint_as_float(r[i]);
      }
      const int64_t n0 = static_cast<int64_t>(j) * kTile;
      const int64_t lim = p.causal ? min(qi + diag, p.Skv - 1) : p.Skv - 1;
      if (n0 + kTile - 1 > lim) {
#pragma unroll
        for (int c = 0; c < kTile; ++c)
          if (n0 + c > lim) s[c] = -INFINITY;
      }
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < kTile; ++c) mx = fmaxf(mx, s[c]);
      const float m_new = fmaxf(m_used, mx);
      bool need = false;
      float alpha = 1.f;
      if (j == 0 || m_used == -INFINITY) {
        m_used = m_new;
      } else if ((m_new - m_used) * p.sl2 > 8.f) {
        need = true;
        alpha = exp2f((m_used - m_new) * p.sl2);
        m_used = m_new;
        l *= alpha;
      }
      const float mu = (m_used == -INFINITY) ? 0.f : m_used;
      const float mus = mu * p.sl2;
      // O may only be touched once PV_{j-1} has finished.
      if (j >= 1 && !sm100::mbar_wait(o_done, (j - 1) & 1)) {
        report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 307, j, row);
        ok = false;
        break;
      }
      if (__any_sync(0xffffffffu, need)) {
        sm100::tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          sm100::tmem_ld32(tmem + lane_base + c * 32, r);
          sm100::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          sm100::tmem_st32(tmem + lane_base + c * 32, r);
        }
        sm100::tmem_wait_st();
      }
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float a = exp2_mufu(fmaf(s[half * 64 + 2 * i], p.sl2, -mus));
          const float b2 = exp2_fma(fmaf(s[half * 64 + 2 * i + 1], p.sl2, -mus));
          l += a + b2;
          pk[i] = pack_bf2(a, b2);
        }
        sm100::tmem_st32(sb + half * 32, pk);
      }
      sm100::tmem_wait_st();
      sm100::tc_fence_before();
      sm100::mbar_arrive(&p_full[st]);
    }
    // ---- epilogue: O / l -> bf16, out[b, qi, h*128 + d]
    const bool valid = qi < p.Sq;
    uint16_t *orow = p.out + ((static_cast<int64_t>(b) * p.Sq + qi) * p.Hq + h) * 128;
    if (n_tiles > 0 && ok) {
      if (!sm100::mbar_wait(o_done, (n_tiles - 1) & 1)) {
        report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 308, n_tiles, row);
      } else {
        sm100::tc_fence_after();
        const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          sm100::tmem_ld32(tmem + lane_base + c * 32, r);
          sm100::tmem_wait_ld();
          if (valid) {
#pragma unroll
            for (int qd = 0; qd < 4; ++qd) {
              uint4 u;
              u.x = pack_bf2(__uint_as_float(r[8 * qd + 0]) * inv, __uint_as_float(r[8 * qd + 1]) * inv);
              u.y = pack_bf2(__uint_as_float(r[8 * qd + 2]) * inv, __uint_as_float(r[8 * qd + 3]) * inv);
              u.z = pack_bf2(__uint_as_float(r[8 * qd + 4]) * inv, __uint_as_float(r[8 * qd + 5]) * inv);
              u.w = pack_bf2(__uint_as_float(r[8 * qd + 6]) * inv, __uint_as_float(r[8 * qd + 7]) * inv);
              reinterpret_cast<uint4 *>(orow + c * 32)[qd] = u;
            }
          }
        }
      }
    } else if (valid) {
      for (int c = 0; c < 16; ++c) reinterpret_cast<uint4 *>(orow)[c] = make_uint4(0, 0, 0, 0);
    }
    if (valid && p.lse)
      p.lse[(static_cast<int64_t>(b) * p.Hq + h) * p.Sq + qi] =
          l > 0.f ? m_used * p.scale + logf(l) : -INFINITY;
  }

  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, kTmemCols);
  }
}


// ---------------------------------------------------------------------------
// Two-tile variant (GQA with an even group): one CTA owns the same 128-query
// block of two heads that share a kv head, so every K/V tile feeds two S
// MMAs and two PV MMAs.  Two softmax warpgroups (one per head) alternate with
// the tensor core: while group a exponentiates S_a(j), the MMA warp computes
// PV_b(j-1) and S_b(j), and vice versa.  TMEM: O_a [0,128), S_a [128,256),
// O_b [256,384), S_b [384,512).  S is single-buffered per head: S_h(j+1) is
// issued only after PV_h(j), which reads P_h(j) from the same columns, and
// tensor operations of one thread complete in issue order, so the commit that
// announces S_h(j+1) also guarantees PV_h(j) has finished (O_h may then be
// rescaled without another wait).
// 384 threads = three warpgroups: WG0 (warp 0 TMA, warp 1 MMA, warps 2-3
// idle) drops to 88 registers per thread with setmaxnreg and the two softmax
// warpgroups (warps 4-7 head a, 8-11 head b) rise to 208, enough to hold a
// whole 128-score row without spilling.  The split uses exactly the launch
// allocation: 128 * 88 + 256 * 208 = 384 * 168 (the kernel must be built with
// 168 registers per thread, which 384 threads and one CTA per SM give).
constexpr int kThreads2 = 384;
constexpr int kRegsLaunch2 = 168, kRegsCtl2 = 88, kRegsSoftmax2 = 208;
static_assert(128 * kRegsCtl2 + 256 * kRegsSoftmax2 <= kThreads2 * kRegsLaunch2,
              "setmaxnreg split exceeds the launch register allocation");
constexpr int kQ2Off = 0;                          // Q_a, Q_b: 2 x 2 halves
constexpr int kK2Off = kQ2Off + 4 * kHalfBytes;    // K: 2 stages x 2 halves
constexpr int kV2Off = kK2Off + 4 * kHalfBytes;    // V: 2 stages x 2 halves
constexpr int kBar2Off = kV2Off + 4 * kHalfBytes;
constexpr int kSmem2 = 1024 + kBar2Off + 20 * 8;

// Pairs (of every 8) whose exponentials use the FMA polynomial instead of MUFU.
template <int kPoly>
constexpr uint32_t kPolyPattern() {
  return kPoly == 2 ? 0x22u : kPoly == 3 ? 0x52u : kPoly == 4 ? 0xAAu : kPoly == 5 ? 0xADu : 0x00u;
}

template <int kPoly>
__global__ void __launch_bounds__(kThreads2, 1)
    attn_tc2_kernel(const __grid_constant__ CUtensorMap tmQ,
                    const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kBar2Off);
  // K and V tiles have separate rings: K(j) is free once both S MMAs of
  // tile j are done, a cycle before the PV MMAs release V(j).
  uint64_t *q_full = bars + 0;
  uint64_t *k_full = bars + 1;    // [2]
  uint64_t *k_empty = bars + 3;   // [2]
  uint64_t *s_full = bars + 5;    // [2] per head
  uint64_t *p_full = bars + 7;    // [2] per head
  uint64_t *o_done = bars + 9;
  uint64_t *drain = bars + 10;
  uint32_t *s_tmem = reinterpret_cast<uint32_t *>(bars + 12);
  uint64_t *v_full = bars + 13;   // [2]
  uint64_t *v_empty = bars + 15;  // [2]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // 1-D grid, heaviest query blocks (most causal key tiles) first across all
  // (batch, head pair) so the tail of the launch is made of short CTAs.
  const int n_pairs_total = static_cast<int>(gridDim.x) / p.n_mblocks;
  const int mb = p.n_mblocks - 1 - static_cast<int>(blockIdx.x) / n_pairs_total;
  const int hp = static_cast<int>(blockIdx.x) % n_pairs_total;  // (b, head pair)
  const int pairs = p.Hq / 2;
  const int b = hp / pairs, h0 = (hp % pairs) * 2;
  const int hk = h0 / (p.Hq / p.Hkv);         // both heads share this kv head
  const int64_t m0 = static_cast<int64_t>(mb) * kTile;
  const int64_t diag = p.Skv - p.Sq;
  int64_t kv_end = p.Skv;
  if (p.causal) kv_end = min(p.Skv, m0 + kTile + diag);
  const int n_tiles = kv_end > 0 ? static_cast<int>((kv_end + kTile - 1) / kTile) : 0;
  const int32_t kv_row = static_cast<int32_t>((static_cast<int64_t>(b) * p.Hkv + hk) * p.kv_cap);

  if (threadIdx.x == 0) {
    sm100::mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(&k_full[i], 1);
      sm100::mbar_init(&k_empty[i], 1);
      sm100::mbar_init(&v_full[i], 1);
      sm100::mbar_init(&v_empty[i], 1);
      sm100::mbar_init(&s_full[i], 1);
      sm100::mbar_init(&p_full[i], 128);
    }
    sm100::mbar_init(o_done, 1);
    sm100::mbar_init(drain, 1);
    sm100::fence_mbar_init();
    sm100::prefetch_tensormap(&tmQ);
    sm100::prefetch_tensormap(&tmK);
    sm100::prefetch_tensormap(&tmV);
  }
  if (warp == 1) sm100::tmem_alloc(s_tmem, kTmemCols);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp < 4) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(kRegsCtl2));
  if (warp == 0 && lane == 0 && n_tiles > 0) {
    // ------------------------------------------------ TMA producer
    sm100::mbar_arrive_expect_tx(q_full, 4 * kHalfBytes);
    for (int hh = 0; hh < 2; ++hh) {
      const int32_t qr = static_cast<int32_t>((static_cast<int64_t>(b) * p.Hq + h0 + hh) * p.Sq + m0);
      sm100::tma_load_2d(smem + kQ2Off + hh * 2 * kHalfBytes, &tmQ, q_full, 0, qr);
      sm100::tma_load_2d(smem + kQ2Off + hh * 2 * kHalfBytes + kHalfBytes, &tmQ, q_full, 64, qr);
    }
    for (int j = 0; j < n_tiles; ++j) {
      const int st = j & 1;
      const uint32_t ph = ((j >> 1) & 1) ^ 1;
      uint8_t *sk = smem + kK2Off + st * 2 * kHalfBytes;
      uint8_t *sv = smem + kV2Off + st * 2 * kHalfBytes;
      const int32_t r = kv_row + j * kTile;
      if (!sm100::mbar_wait(&k_empty[st], ph)) {
        report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 321, j, 0);
        break;
      }
      sm100::mbar_arrive_expect_tx(&k_full[st], 2 * kHalfBytes);
      sm100::tma_load_2d(sk, &tmK, &k_full[st], 0, r);
      sm100::tma_load_2d(sk + kHalfBytes, &tmK, &k_full[st], 64, r);
      if (!sm100::mbar_wait(&v_empty[st], ph)) {
        report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 328, j, 0);
        break;
      }
      sm100::mbar_arrive_expect_tx(&v_full[st], 2 * kHalfBytes);
      sm100::tma_load_2d(sv, &tmV, &v_full[st], 0, r);
      sm100::tma_load_2d(sv + kHalfBytes, &tmV, &v_full[st], 64, r);
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_s = sm100::idesc_bf16_f32(kTile, kTile);
    constexpr uint32_t idesc_pv = sm100::idesc_bf16_f32(kTile, 128, 0, 1);
    bool ok = n_tiles > 0;
    if (ok && !sm100::mbar_wait(q_full, 0)) {
      report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 322, 0, 0);
      ok = false;
    }
    auto issue_s = [&](int hh, int j) {
      const int st = j & 1;
      const uint32_t sq = sm100::smem_u32(smem + kQ2Off + hh * 2 * kHalfBytes);
      const uint32_t sk = sm100::smem_u32(smem + kK2Off + st * 2 * kHalfBytes);
      const uint32_t s_tm = tmem + hh * 256 + 128;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = (kk >> 2) * kHalfBytes;
        const uint64_t ad = sm100::sw128_kmajor_desc(sq + off) + 2 * (kk & 3);
        const uint64_t bd = sm100::sw128_kmajor_desc(sk + off) + 2 * (kk & 3);
        sm100::mma_bf16_ss(s_tm, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
      }
      sm100::mma_commit(&s_full[hh]);
    };
    auto issue_pv = [&](int hh, int i) -> bool {
      if (hh == 0 && !sm100::mbar_wait(&v_full[i & 1], (i >> 1) & 1)) {
        report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 329, i, hh);
        return false;
      }
      if (!sm100::mbar_wait(&p_full[hh], i & 1)) {
        report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 323, i, hh);
        return false;
      }
      sm100::tc_fence_after();
      const int st = i & 1;
      const uint32_t sv = sm100::smem_u32(smem + kV2Off + st * 2 * kHalfBytes);
      const uint32_t o_tm = tmem + hh * 256;
#pragma unroll
      for (int kk = 0; kk < kTile / 16; ++kk) {
        const uint64_t bdesc = sm100::sw128_mnmajor_desc(sv + kk * 2048, kHalfBytes, 1024);
        sm100::mma_bf16_ts(o_tm, o_tm + 128 + kk * 8, bdesc, idesc_pv, (i > 0 || kk > 0) ? 1u : 0u);
      }
      return true;
    };
    for (int j = 0; j < n_tiles && ok; ++j) {
      const int st = j & 1;
      if (!sm100::mbar_wait(&k_full[st], (j >> 1) & 1)) {
        report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 324, j, 0);
        ok = false;
        break;
      }
      sm100::tc_fence_after();
      if (j > 0 && !issue_pv(0, j - 1)) { ok = false; break; }
      issue_s(0, j);
      if (j > 0) {
        if (!issue_pv(1, j - 1)) { ok = false; break; }
        sm100::mma_commit(&v_empty[(j - 1) & 1]);
      }
      issue_s(1, j);
      sm100::mma_commit(&k_empty[st]);
    }
    if (ok) {
      if (issue_pv(0, n_tiles - 1) && issue_pv(1, n_tiles - 1)) {
        sm100::mma_commit(&v_empty[(n_tiles - 1) & 1]);
        sm100::mma_commit(o_done);
      }
    }
    sm100::mma_commit(drain);
    if (!sm100::mbar_wait(drain, 0)) report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 325, 0, 0);
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(kRegsSoftmax2));
    // ------------------------------------------------ softmax, one group per head
    const int hh = (warp - 4) >> 2;          // warps 4-7: head a, 8-11: head b
    const int q = warp & 3;                  // TMEM lane quadrant of this warp
    const int row = q * 32 + lane;
    const int64_t qi = m0 + row;
    const int h = h0 + hh;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t o_tm = tmem + lane_base + hh * 256;
    const uint32_t s_tm = o_tm + 128;
    const int64_t lim_c = p.causal ? min(qi + diag, p.Skv - 1) : p.Skv - 1;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      if (!sm100::mbar_wait(&s_full[hh], j & 1)) {
        report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 326, j, row);
        ok = false;
        break;
      }
      sm100::tc_fence_after();
      const int64_t n0 = static_cast<int64_t>(j) * kTile;
      const bool masked = n0 + kTile - 1 > lim_c;
      // the whole score row in two 64-column loads, one wait
      uint32_t sr[kTile];
      sm100::tmem_ld64(s_tm, sr);
      sm100::tmem_ld64(s_tm + 64, sr + 64);
      sm100::tmem_wait_ld();
      if (masked) {
#pragma unroll
        for (int c = 0; c < kTile; ++c)
          if (n0 + c > lim_c) sr[c] = __float_as_uint(-INFINITY);
      }
      // row max: four independent 3-input max chains
      float mx0 = m_used, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
      for (int c = 0; c < kTile; c += 8) {
        mx0 = max3f(mx0, __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
        mx1 = max3f(mx1, __uint_as_float(sr[c + 2]), __uint_as_float(sr[c + 3]));
        mx2 = max3f(mx2, __uint_as_float(sr[c + 4]), __uint_as_float(sr[c + 5]));
        mx3 = max3f(mx3, __uint_as_float(sr[c + 6]), __uint_as_float(sr[c + 7]));
      }
      const float m_new = max3f(mx0, mx1, fmaxf(mx2, mx3));
      bool need = false;
      float alpha = 1.f;
      if (j == 0 || m_used == -INFINITY) {
        m_used = m_new;
      } else if ((m_new - m_used) * p.sl2 > 8.f) {
        need = true;
        alpha = exp2f((m_used - m_new) * p.sl2);
        m_used = m_new;
        l *= alpha;
      }
      const float mus = ((m_used == -INFINITY) ? 0.f : m_used) * p.sl2;
      // exponentials, bf16 P over the first 64 S columns.  Score pairs are
      // scaled with one f32x2 FMA; pairs alternate between the MUFU unit
      // (ex2.approx) and the paired FMA polynomial; row sums in f32x2.
      const float2 sl2v = make_float2(p.sl2, p.sl2), nmus = make_float2(-mus, -mus);
      float2 lsum0 = make_float2(0.f, 0.f), lsum1 = make_float2(0.f, 0.f);
#pragma unroll
      for (int qtr = 0; qtr < 4; ++qtr) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 sv = make_float2(__uint_as_float(sr[qtr * 32 + 2 * i]),
                                        __uint_as_float(sr[qtr * 32 + 2 * i + 1]));
          const float2 x = __ffma2_rn(sv, sl2v, nmus);
          float2 e;
          if (((kPolyPattern<kPoly>() >> (i & 7)) & 1u)) {
            e = exp2_fma2(x);
          } else {
            e.x = exp2_mufu(x.x);
            e.y = exp2_mufu(x.y);
          }
          if (i & 2) lsum1 = __fadd2_rn(lsum1, e);
          else lsum0 = __fadd2_rn(lsum0, e);
          pk[i] = pack_bf2(e.x, e.y);
        }
        sm100::tmem_st16(s_tm + qtr * 16, pk);
      }
      l += (lsum0.x + lsum0.y) + (lsum1.x + lsum1.y);
      // PV(j-1) is complete (it precedes S(j) in the tensor pipe): O may be scaled
      // (after the exponentials, when the score registers are free).
      if (__any_sync(0xffffffffu, need)) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          sm100::tmem_ld32(o_tm + c * 32, r);
          sm100::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          sm100::tmem_st32(o_tm + c * 32, r);
        }
      }
      sm100::tmem_wait_st();
      sm100::tc_fence_before();
      sm100::mbar_arrive(&p_full[hh]);
    }
    // ---- epilogue: O / l -> bf16, out[b, qi, h*128 + d]
    const bool valid = qi < p.Sq;
    uint16_t *orow = p.out + ((static_cast<int64_t>(b) * p.Sq + qi) * p.Hq + h) * 128;
    if (n_tiles > 0 && ok) {
      if (!sm100::mbar_wait(o_done, 0)) {
        report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 327, n_tiles, row);
      } else {
        sm100::tc_fence_after();
        // a row that saw no unmasked key (m_used still -inf) is all zeros; its
        // l holds only the polynomial's 2^-125 floor for masked scores
        const float inv = (l > 0.f && m_used != -INFINITY) ? 1.f / l : 0.f;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          sm100::tmem_ld32(o_tm + c * 32, r);
          sm100::tmem_wait_ld();
          if (valid) {
#pragma unroll
            for (int qd = 0; qd < 4; ++qd) {
              uint4 u;
              u.x = pack_bf2(__uint_as_float(r[8 * qd + 0]) * inv, __uint_as_float(r[8 * qd + 1]) * inv);
              u.y = pack_bf2(__uint_as_float(r[8 * qd + 2]) * inv, __uint_as_float(r[8 * qd + 3]) * inv);
              u.z = pack_bf2(__uint_as_float(r[8 * qd + 4]) * inv, __uint_as_float(r[8 * qd + 5]) * inv);
              u.w = pack_bf2(__uint_as_float(r[8 * qd + 6]) * inv, __uint_as_float(r[8 * qd + 7]) * inv);
              reinterpret_cast<uint4 *>(orow + c * 32)[qd] = u;
            }
          }
        }
      }
    } else if (valid) {
      for (int c = 0; c < 16; ++c) reinterpret_cast<uint4 *>(orow)[c] = make_uint4(0, 0, 0, 0);
    }
    if (valid && p.lse)
      p.lse[(static_cast<int64_t>(b) * p.Hq + h) * p.Sq + qi] =
          (l > 0.f && m_used != -INFINITY) ? m_used * p.scale + logf(l) : -INFINITY;
  }

  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace
}  // namespace q35

using namespace q35;

// Prefill attention for head_dim 128 on tcgen05 (called by
// q35_attn_prefill_fwd; same arguments and layouts).
int q35_attn_prefill_tc(const void *q, const void *k, const void *v, void *out,
                        float *lse, int64_t B, int Hq, int Hkv, int64_t Sq,
                        int64_t Skv, int64_t kv_cap, float scale, int causal,
                        q35_stream_t stream) {
  const int64_t qrows = B * Hq * Sq, kvrows = B * Hkv * kv_cap;
  if (qrows >= (int64_t(1) << 31) || kvrows >= (int64_t(1) << 31))
    return fail(Q35_ERR_SHAPE, "attn_prefill_tc: too many rows for TMA coordinates");
  int *err = device_error_word();
  if (!err) return fail(Q35_ERR_CUDA, "attn_prefill_tc: no device error word");
  CUtensorMap tq, tk, tv;
  int st = make_tmap_bf16_2d(&tq, q, 128, qrows, 256, 64, kTile);
  if (st) return st;
  st = make_tmap_bf16_2d(&tk, k, 128, kvrows, 256, 64, kTile);
  if (st) return st;
  st = make_tmap_bf16_2d(&tv, v, 128, kvrows, 256, 64, kTile);
  if (st) return st;
  AttnParams p{};
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.Sq = Sq;
  p.Skv = Skv;
  p.kv_cap = kv_cap;
  p.n_mblocks = static_cast<int>((Sq + kTile - 1) / kTile);
  p.scale = scale;
  p.sl2 = scale * 1.4426950408889634f;
  p.causal = causal ? 1 : 0;
  p.out = static_cast<uint16_t *>(out);
  p.lse = lse;
  p.err = err;
  if ((Hq / Hkv) % 2 == 0) {
    // GQA with an even group: two heads per CTA share each K/V tile.
    dim3 grid2(static_cast<unsigned>(p.n_mblocks * B * Hq / 2));
    constexpr int np = 3;  // 3 of 8 score pairs on the FMA-pipe exp2 (measured best of 2..5)
    auto go = [&](auto kern) -> int {
      const int st2 = ensure_smem_attr(reinterpret_cast<const void *>(kern), kSmem2);
      if (st2) return st2;
      // the setmaxnreg split assumes exactly kRegsLaunch2 registers at launch
      static thread_local bool regs_ok = false;
      if (!regs_ok) {
        cudaFuncAttributes fa;
        const cudaError_t fe = cudaFuncGetAttributes(&fa, reinterpret_cast<const void *>(kern));
        if (fe != cudaSuccess) return cuda_fail(fe, "attn_prefill_tc2: cudaFuncGetAttributes");
        if (fa.numRegs != kRegsLaunch2)
          return fail(Q35_ERR_UNSUPPORTED, "attn_prefill_tc2 built with %d registers per thread, "
                      "the register split needs %d", fa.numRegs, kRegsLaunch2);
        regs_ok = true;
      }
      kern<<<grid2, kThreads2, kSmem2, reinterpret_cast<cudaStream_t>(stream)>>>(tq, tk, tv, p);
      return 0;
    };
    int st3 = go(attn_tc2_kernel<np>);
    if (st3) return st3;
    Q35_LAUNCH_CHECK("attn_prefill_tc2 launch");
    return Q35_OK;
  }
  { const int _st = ensure_smem_attr(reinterpret_cast<const void *>(attn_tc_kernel), kSmem); if (_st) return _st; }
  dim3 grid(p.n_mblocks, static_cast<unsigned>(B * Hq));
  attn_tc_kernel<<<grid, kThreads, kSmem, reinterpret_cast<cudaStream_t>(stream)>>>(tq, tk, tv, p);
  Q35_LAUNCH_CHECK("attn_prefill_tc launch");
  return Q35_OK;
}
