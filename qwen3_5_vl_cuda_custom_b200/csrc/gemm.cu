// Persistent tcgen05 GEMM for the dense projections and the grouped expert
// GEMMs (gate_up with SwiGLU fused into the epilogue, down).
//
//   C[m, n] = sum_k A[m, k] * B[n, k]        A, B bf16 K-major, fp32 in TMEM
//
// One CTA per SM (192 threads, 6 warps) loops over output tiles 128 x BN:
//   warp 0  lane 0 : TMA producer.  A tile 128 x 64 and B tile BN x 64 per
//                    k-block into a STAGES-deep shared-memory ring
//                    (128-byte swizzle, the layout UMMA reads directly).
//   warp 1  lane 0 : MMA issuer.  4 x tcgen05.mma (K = 16 each) per k-block
//                    into one of two TMEM accumulators (2 x BN fp32 columns),
//                    tcgen05.commit releases the smem stage / publishes the
//                    accumulator.  Warp 1 also owns the TMEM allocation.
//   warps 2-5      : epilogue.  tcgen05.ld of the accumulator rows (warp w
//                    reads TMEM lanes 32*(w%4)..+31 = tile rows), fused
//                    bias / residual / SwiGLU math, bf16 stores.  The second
//                    accumulator lets the epilogue of tile i overlap the MMAs
//                    of tile i+1.
//
// Grouped mode: rows of A are the permuted (expert-sorted) token rows; group e
// owns rows [offsets[e], offsets[e+1]) and ceil(count/128) M tiles
// (tile_offsets, built by q35_moe_permute).  Tiles are ordered
// (group, n-tile, m-tile) with m fastest, so CTAs running at the same time
// share each weight tile through L2.  The tile count is read from device
// memory: no host synchronisation is needed between routing and the GEMM.
//
// Reference counterparts: matmul_fwd_kernel (REF cuda_qwen3_vl/csrc/
// matmul_op.cu:15-92, SIMT 32x32 tiles) for every projection, and the
// per-expert loop of CudaSparseMoE.forward (REF modules/moe.py:71-83) with
// swiglu_fwd_kernel (REF csrc/swiglu_op.cu:6-18) for the experts.
#include "sm100.cuh"

namespace q35 {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;  // 64 bf16 = one 128-byte swizzle row
constexpr int kThreads = 192;
constexpr int kMaxGroups = 512;

enum Epilogue { EPI_PLAIN = 0, EPI_SWIGLU = 1, EPI_QKV = 2 };

struct GemmParams {
  int M;                       // dense rows (grouped: unused)
  const int32_t *offsets;      // grouped: [E+1] row offsets, else nullptr
  const int32_t *tile_offsets; // grouped: [E+1] M-tile prefix
  int E;                       // groups (1 for dense)
  int N;                       // valid output columns per group
  int K;
  int n_tiles;                 // tiles along N per group
  int b_rows_per_group;        // rows of B owned by one group
  int b_tile_step;             // B row advance per n-tile
  int b_second_off;            // row offset of the second half box of B
  uint16_t *out;
  int64_t ldo;
  const uint16_t *bias;        // [N] or nullptr
  const uint16_t *residual;    // [rows, ldr] or nullptr
  int64_t ldr;
  int *err;
  int out_f32;                 // PLAIN epilogue: store fp32 instead of bf16
  int a_k_wrap;                // > 0: A's K coordinate wraps at this width
  int k_splits;                // dense only: K split into this many partial planes
  int64_t split_stride;        // elements between partial output planes
  int b_packed;                // B stored as contiguous 128 x 64 tiles (see q35_pack_b_tiles)
  // EPI_QKV: the output columns are Hq + 2*Hkv heads of 128; q/k heads get
  // RMSNorm (qk_w: q weight [128] then k weight [128]) and rotate-half RoPE
  // (cos/sin tables fp32 [rows, 64]); q, k, v are written head-major.
  const uint16_t *q_norm_w, *k_norm_w;
  const float *rope_cos, *rope_sin;
  uint16_t *q_out, *k_out, *v_out;
  int Hq, Hkv, seq;
  float eps;
};

template <int BN, int STAGES>
struct SmemLayout {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOff = STAGES * kStageBytes;
  // full[S], empty[S], tfull[2], tempty[2], drain
  static constexpr int kNumBars = 2 * STAGES + 5;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kGroupOff = kMiscOff + 16;
  static constexpr int bytes(int E) {
    return 1024 + kGroupOff + 2 * (E + 1) * 4;
  }
};

struct TileInfo {
  int row0;        // first A row of the tile
  int rows_valid;  // rows of the tile that belong to the group
  int group;
  int nt;          // n-tile index
  int split;       // K split (dense split-K), else 0
  int half;        // pair tile of 128 rows (64 per CTA, M = 128 MMA)
};

__device__ __forceinline__ TileInfo decode_tile(int tile, const GemmParams &p,
                                                const int *s_off,
                                                const int *s_toff) {
  TileInfo ti;
  ti.split = 0;
  if (p.offsets == nullptr) {
    const int mtiles = (p.M + kBM - 1) / kBM;
    const int per_split = mtiles * p.n_tiles;
    ti.split = tile / per_split;
    tile -= ti.split * per_split;
    ti.nt = tile / mtiles;
    const int mt = tile - ti.nt * mtiles;
    ti.group = 0;
    ti.row0 = mt * kBM;
    ti.rows_valid = min(kBM, p.M - ti.row0);
    return ti;
  }
  // Largest e with s_toff[e] * n_tiles <= tile.
  int lo = 0, hi = p.E - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (s_toff[mid] * p.n_tiles <= tile)
      lo = mid;
    else
      hi = mid - 1;
  }
  // Skip empty groups that share the same prefix (they own no tiles).
  while (lo < p.E - 1 && s_toff[lo + 1] * p.n_tiles <= tile) ++lo;
  const int e = lo;
  const int me = s_toff[e + 1] - s_toff[e];
  const int local = tile - s_toff[e] * p.n_tiles;
  ti.nt = local / me;
  const int mt = local - ti.nt * me;
  ti.group = e;
  ti.row0 = s_off[e] + mt * kBM;
  ti.rows_valid = min(kBM, s_off[e + 1] - ti.row0);
  return ti;
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

// Stores 32 consecutive bf16 outputs (fp32 values in v) at dst.
__device__ __forceinline__ void store32(uint16_t *dst, const float *v) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 u;
    u.x = pack_bf2(v[8 * q + 0], v[8 * q + 1]);
    u.y = pack_bf2(v[8 * q + 2], v[8 * q + 3]);
    u.z = pack_bf2(v[8 * q + 4], v[8 * q + 5]);
    u.w = pack_bf2(v[8 * q + 6], v[8 * q + 7]);
    reinterpret_cast<uint4 *>(dst)[q] = u;
  }
}
__device__ __forceinline__ void load32(const uint16_t *src, float *v) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 u = reinterpret_cast<const uint4 *>(src)[q];
    unpack_bf2(u.x, v[8 * q + 0], v[8 * q + 1]);
    unpack_bf2(u.y, v[8 * q + 2], v[8 * q + 3]);
    unpack_bf2(u.z, v[8 * q + 4], v[8 * q + 5]);
    unpack_bf2(u.w, v[8 * q + 6], v[8 * q + 7]);
  }
}

__device__ __forceinline__ void store16(uint16_t *dst, const float *v) {
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    uint4 u;
    u.x = pack_bf2(v[8 * q + 0], v[8 * q + 1]);
    u.y = pack_bf2(v[8 * q + 2], v[8 * q + 3]);
    u.z = pack_bf2(v[8 * q + 4], v[8 * q + 5]);
    u.w = pack_bf2(v[8 * q + 6], v[8 * q + 7]);
    reinterpret_cast<uint4 *>(dst)[q] = u;
  }
}

__device__ __forceinline__ void load16(const uint16_t *src, float *v) {
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const uint4 u = reinterpret_cast<const uint4 *>(src)[q];
    unpack_bf2(u.x, v[8 * q + 0], v[8 * q + 1]);
    unpack_bf2(u.y, v[8 * q + 2], v[8 * q + 3]);
    unpack_bf2(u.z, v[8 * q + 4], v[8 * q + 5]);
    unpack_bf2(u.w, v[8 * q + 6], v[8 * q + 7]);
  }
}

template <int BN, int EPI, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                   const __grid_constant__ CUtensorMap tmB, GemmParams p) {
  using L = SmemLayout<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::kBarOff);
  uint64_t *full = bars;
  uint64_t *empty = bars + STAGES;
  uint64_t *tfull = bars + 2 * STAGES;
  uint64_t *tempty = bars + 2 * STAGES + 2;
  uint64_t *drain = bars + 2 * STAGES + 4;
  uint32_t *s_tmem = reinterpret_cast<uint32_t *>(smem + L::kMiscOff);
  int *s_off = reinterpret_cast<int *>(smem + L::kGroupOff);
  int *s_toff = s_off + (p.E + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (p.offsets != nullptr) {
    for (int i = threadIdx.x; i <= p.E; i += kThreads) {
      s_off[i] = p.offsets[i];
      s_toff[i] = p.tile_offsets[i];
    }
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      sm100::mbar_init(&tfull[a], 1);
      sm100::mbar_init(&tempty[a], 128);
    }
    sm100::mbar_init(drain, 1);
    sm100::fence_mbar_init();
    sm100::prefetch_tensormap(&tmA);
    sm100::prefetch_tensormap(&tmB);
  }
  if (warp == 1) sm100::tmem_alloc(s_tmem, 2 * BN);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem_base = *s_tmem;

  int total;
  if (p.offsets == nullptr)
    total = ((p.M + kBM - 1) / kBM) * p.n_tiles * max(1, p.k_splits);
  else
    total = s_toff[p.E] * p.n_tiles;

  const int k_blocks = (p.K + kBK - 1) / kBK;  // TMA zero-fills the K tail
  // Split-K: split s covers k-blocks [s * kb_per, (s + 1) * kb_per); the host
  // only uses splits that divide k_blocks, so no split is empty.
  const int kb_per = k_blocks / max(1, p.k_splits);

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------ TMA producer
    uint32_t g = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
      const TileInfo ti = decode_tile(tile, p, s_off, s_toff);
      const int brow = ti.group * p.b_rows_per_group + ti.nt * p.b_tile_step;
      const int kb0 = ti.split * kb_per;
      for (int kb = kb0; kb < kb0 + kb_per; ++kb, ++g) {
        const int s = g % STAGES;
        const uint32_t ph = (g / STAGES) & 1u;
        if (!sm100::mbar_wait(&empty[s], ph ^ 1u)) {
          report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 201, tile, kb);
          ok = false;
          break;
        }
        uint8_t *sa = smem + s * L::kStageBytes;
        uint8_t *sb = sa + L::kABytes;
        sm100::mbar_arrive_expect_tx(&full[s], L::kStageBytes);
        const int ka = p.a_k_wrap ? (kb * kBK) % p.a_k_wrap : kb * kBK;
        sm100::tma_load_2d(sa, &tmA, &full[s], ka, ti.row0);
        sm100::tma_load_2d(sb, &tmB, &full[s], kb * kBK, brow);
        sm100::tma_load_2d(sb + L::kBBytes / 2, &tmB, &full[s], kb * kBK,
                           brow + p.b_second_off);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = sm100::idesc_bf16_f32(kBM, BN);
    uint32_t g = 0, j = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++j) {
      const uint32_t acc = j & 1u, use = j >> 1;
      if (!sm100::mbar_wait(&tempty[acc], (use & 1u) ^ 1u)) {
        report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 202, tile, 0);
        break;
      }
      sm100::tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      const int kb0 = decode_tile(tile, p, s_off, s_toff).split * kb_per;
      for (int kb = kb0; kb < kb0 + kb_per; ++kb, ++g) {
        const int s = g % STAGES;
        const uint32_t ph = (g / STAGES) & 1u;
        if (!sm100::mbar_wait(&full[s], ph)) {
          report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 203, tile, kb);
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        const uint32_t sa = sm100::smem_u32(smem + s * L::kStageBytes);
        const uint64_t adesc = sm100::sw128_kmajor_desc(sa);
        const uint64_t bdesc = sm100::sw128_kmajor_desc(sa + L::kABytes);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          sm100::mma_bf16_ss(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc,
                             (kb != kb0 || kk != 0) ? 1u : 0u);
        sm100::mma_commit(&empty[s]);
      }
      sm100::mma_commit(&tfull[acc]);
    }
    // Drain: every MMA issued above has finished before TMEM is released.
    sm100::mma_commit(drain);
    if (!sm100::mbar_wait(drain, 0))
      report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 204, 0, 0);
  } else if (warp >= 2) {
    // ------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int r_in_tile = q * 32 + lane;
    uint32_t j = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++j) {
      const TileInfo ti = decode_tile(tile, p, s_off, s_toff);
      const uint32_t acc = j & 1u, use = j >> 1;
      if (!sm100::mbar_wait(&tfull[acc], use & 1u)) {
        report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 205, tile, 0);
        break;
      }
      sm100::tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                             acc * BN;
      const bool valid = r_in_tile < ti.rows_valid;
      const int64_t row = static_cast<int64_t>(ti.row0) + r_in_tile;
      if constexpr (EPI == EPI_PLAIN) {
        const int n0 = ti.nt * BN;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          sm100::tmem_ld32(t_row + c * 32, r);
          sm100::tmem_wait_ld();
          const int col = n0 + c * 32;
          if (valid && col < p.N) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
            if (p.bias) {
              float bv[32];
              load32(p.bias + col, bv);
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] += bv[i];
            }
            if (p.residual) {
              float rv[32];
              load32(p.residual + row * p.ldr + col, rv);
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = rv[i] + v[i];
            }
            if (p.out_f32) {
              float4 *o = reinterpret_cast<float4 *>(
                  reinterpret_cast<float *>(p.out) + ti.split * p.split_stride + row * p.ldo + col);
#pragma unroll
              for (int q = 0; q < 8; ++q)
                o[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
            } else {
              store32(p.out + row * p.ldo + col, v);
            }
          }
        }
      } else {
        // Accumulator columns [0, BN/2) hold gate, [BN/2, BN) the matching up.
        const int n0 = ti.nt * (BN / 2);
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
          uint32_t rg[32], ru[32];
          sm100::tmem_ld32(t_row + c * 32, rg);
          sm100::tmem_ld32(t_row + BN / 2 + c * 32, ru);
          sm100::tmem_wait_ld();
          const int col = n0 + c * 32;
          if (valid && col < p.N) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i)
              v[i] = silu(__uint_as_float(rg[i])) * __uint_as_float(ru[i]);
            store32(p.out + row * p.ldo + col, v);
          }
        }
      }
      sm100::tc_fence_before();
      sm100::mbar_arrive(&tempty[acc]);
    }
  }

  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem_base, 2 * BN);
  }
}

template <int BN, int EPI, int STAGES>
int launch_gemm(const CUtensorMap &ta, const CUtensorMap &tb,
                const GemmParams &p, int max_tiles, cudaStream_t s) {
  using L = SmemLayout<BN, STAGES>;
  const int smem = L::bytes(p.E);
  auto kern = gemm_tc_kernel<BN, EPI, STAGES>;
  { const int _st = ensure_smem_attr(reinterpret_cast<const void *>(kern), smem); if (_st) return _st; }
  const int grid = max(1, min(max_tiles, num_sms()));
  kern<<<grid, kThreads, smem, s>>>(ta, tb, p);
  Q35_LAUNCH_CHECK("gemm_tc launch");
  return Q35_OK;
}


// ---------------------------------------------------------------------------
// 2-SM variant: a CTA pair (cluster of 2) computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2 (M = 256 across the two SMs' tensor memories).
// Each CTA loads its own 128 rows of A and 128 rows of B per k-block (32 KB,
// half of what one CTA needs for a 128 x 256 tile), so the L2->SM traffic per
// FLOP halves and 6 stages fit.  Both CTAs' TMA loads complete on the leader's
// full barrier (the leader alone expects the 64 KB); the leader issues the MMAs
// and its commits arrive on both CTAs' barriers; each CTA's epilogue drains its
// own 128 accumulator rows and arrives on the leader's accumulator-empty
// barrier.  No TMA multicast is used.
struct PairLayout {
  static constexpr int kStages = 6;
  static constexpr int kHalf = 128 * kBK * 2;           // 16 KB
  static constexpr int kStageBytes = 2 * kHalf;         // A half + B half
  static constexpr int kBarOff = kStages * kStageBytes;
  static constexpr int kNumBars = 2 * kStages + 5;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kGroupOff = kMiscOff + 16;
  static constexpr int bytes(int E) { return 1024 + kGroupOff + 2 * (E + 1) * 4; }
};

__device__ __forceinline__ bool pair_half_ok(const GemmParams &p) {
  return !p.b_packed && !p.bias && !p.residual && !p.out_f32;
}

__device__ __forceinline__ TileInfo decode_pair_tile(int tile, const GemmParams &p,
                                                     const int *s_off, const int *s_pt) {
  TileInfo ti;
  ti.split = 0;
  ti.half = 0;
  if (p.offsets == nullptr) {
    // Rasterise in bands of 8 M tiles: CTAs running together share 8 A tiles
    // and a run of B tiles in L2, whatever the aspect ratio of the problem.
    const int mtiles = (p.M + 255) / 256;
    const int band = tile / (8 * p.n_tiles);
    const int band_m = min(8, mtiles - band * 8);
    const int in_band = tile - band * 8 * p.n_tiles;
    ti.nt = in_band / band_m;
    const int mt = band * 8 + (in_band - ti.nt * band_m);
    ti.group = 0;
    ti.row0 = mt * 256;
    ti.rows_valid = min(256, p.M - ti.row0);
    return ti;
  }
  int lo = 0, hi = p.E - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (s_pt[mid] * p.n_tiles <= tile) lo = mid; else hi = mid - 1;
  }
  while (lo < p.E - 1 && s_pt[lo + 1] * p.n_tiles <= tile) ++lo;
  const int e = lo;
  const int me = s_pt[e + 1] - s_pt[e];
  const int local = tile - s_pt[e] * p.n_tiles;
  ti.nt = local / me;
  const int mt = local - ti.nt * me;
  ti.group = e;
  ti.row0 = s_off[e] + mt * 256;
  ti.rows_valid = min(256, s_off[e + 1] - ti.row0);
  // A group's last <= 128 rows run as an M = 128 pair MMA (half the tensor
  // time of a padded 256-row tile).  Plain stores or SwiGLU, unpacked B only.
  ti.half = (ti.rows_valid <= 128 && pair_half_ok(p)) ? 1 : 0;
  return ti;
}



template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmB64, GemmParams p) {
  using L = PairLayout;
  constexpr int BN = 256;
  constexpr int S = L::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::kBarOff);
  uint64_t *full = bars;
  uint64_t *empty = bars + S;
  uint64_t *tfull = bars + 2 * S;
  uint64_t *tempty = bars + 2 * S + 2;
  uint64_t *drain = bars + 2 * S + 4;
  uint32_t *s_tmem = reinterpret_cast<uint32_t *>(smem + L::kMiscOff);
  int *s_off = reinterpret_cast<int *>(smem + L::kGroupOff);
  int *s_pt = s_off + (p.E + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = sm100::cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (p.offsets != nullptr) {
    for (int i = threadIdx.x; i <= p.E; i += kThreads) s_off[i] = p.offsets[i];
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      sm100::mbar_init(&full[i], 1);
      sm100::mbar_init(&empty[i], 1);
    }
    for (int a = 0; a < 2; ++a) {
      sm100::mbar_init(&tfull[a], 1);
      sm100::mbar_init(&tempty[a], 256);
    }
    sm100::mbar_init(drain, 1);
    sm100::fence_mbar_init();
    sm100::prefetch_tensormap(&tmA);
    sm100::prefetch_tensormap(&tmB);
  }
  __syncthreads();
  if (p.offsets != nullptr && threadIdx.x == 0) {
    // 256-row M tiles per group (prefix over groups).
    int acc = 0;
    s_pt[0] = 0;
    for (int e = 0; e < p.E; ++e) {
      acc += (s_off[e + 1] - s_off[e] + 255) / 256;
      s_pt[e + 1] = acc;
    }
  }
  if (warp == 1) sm100::tmem_alloc_pair(s_tmem, 2 * BN);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::cluster_sync();  // barriers of both CTAs initialised before any remote use
  sm100::tc_fence_after();
  const uint32_t tmem_base = *s_tmem;

  const int total = (p.offsets == nullptr) ? ((p.M + 255) / 256) * p.n_tiles
                                           : s_pt[p.E] * p.n_tiles;
  const int k_blocks = (p.K + kBK - 1) / kBK;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------ TMA producer (both CTAs)
    uint32_t g = 0;
    bool ok = true;
    for (int tile = pair; tile < total && ok; tile += npairs) {
      const TileInfo ti = decode_pair_tile(tile, p, s_off, s_pt);
      const int arow = ti.row0 + static_cast<int>(rank) * (ti.half ? 64 : 128);
      const int brow = ti.group * p.b_rows_per_group + ti.nt * p.b_tile_step +
                       static_cast<int>(rank) * p.b_second_off;
      // SwiGLU half tile: each CTA's B half holds 64 gate rows and the
      // matching 64 up rows, so every accumulator lane gets gate and up
      const bool split_b = EPI == EPI_SWIGLU && ti.half;
      const int brow_g = ti.group * p.b_rows_per_group + ti.nt * p.b_tile_step +
                         static_cast<int>(rank) * 64;
      for (int kb = 0; kb < k_blocks; ++kb, ++g) {
        const int st = g % S;
        const uint32_t ph = (g / S) & 1u;
        if (!sm100::mbar_wait(&empty[st], ph ^ 1u)) {
          report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 211, tile, kb);
          ok = false;
          break;
        }
        uint8_t *sa = smem + st * L::kStageBytes;
        uint8_t *sb = sa + L::kHalf;
        const uint32_t leader_full = sm100::mapa_shared(sm100::smem_u32(&full[st]), 0);
        if (rank == 0) sm100::mbar_arrive_expect_tx(&full[st], 2 * L::kStageBytes);
        sm100::tma_load_2d_pair(sa, &tmA, leader_full, kb * kBK, arow);
        if (split_b) {
          sm100::tma_load_2d_pair(sb, &tmB64, leader_full, kb * kBK, brow_g);
          sm100::tma_load_2d_pair(sb + L::kHalf / 2, &tmB64, leader_full, kb * kBK,
                                  brow_g + p.b_second_off);
        } else if (p.b_packed) {  // tile (brow / 128, kb) is 16 KB contiguous
          sm100::tma_load_2d_pair(sb, &tmB, leader_full, 0, ((brow >> 7) * k_blocks + kb) * 128);
        } else {
          sm100::tma_load_2d_pair(sb, &tmB, leader_full, kb * kBK, brow);
        }
      }
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ------------------------------------------------ MMA issuer (leader CTA)
    constexpr uint32_t idesc256 = sm100::idesc_bf16_f32(256, BN);
    constexpr uint32_t idesc128 = sm100::idesc_bf16_f32(128, BN);
    uint32_t g = 0, j = 0;
    bool ok = true;
    for (int tile = pair; tile < total && ok; tile += npairs, ++j) {
      const uint32_t acc = j & 1u, use = j >> 1;
      const uint32_t idesc = decode_pair_tile(tile, p, s_off, s_pt).half ? idesc128 : idesc256;
      if (!sm100::mbar_wait(&tempty[acc], (use & 1u) ^ 1u)) {
        report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 212, tile, 0);
        break;
      }
      sm100::tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      for (int kb = 0; kb < k_blocks; ++kb, ++g) {
        const int st = g % S;
        const uint32_t ph = (g / S) & 1u;
        if (!sm100::mbar_wait(&full[st], ph)) {
          report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 213, tile, kb);
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        const uint32_t sa = sm100::smem_u32(smem + st * L::kStageBytes);
        const uint64_t adesc = sm100::sw128_kmajor_desc(sa);
        const uint64_t bdesc = sm100::sw128_kmajor_desc(sa + L::kHalf);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          sm100::mma_bf16_ss_pair(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc,
                                  (kb | kk) != 0 ? 1u : 0u);
        sm100::mma_commit_pair_mc(&empty[st], 0x3);
      }
      sm100::mma_commit_pair_mc(&tfull[acc], 0x3);
    }
    sm100::mma_commit_pair_mc(drain, 0x1);
    if (!sm100::mbar_wait(drain, 0)) report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 214, 0, 0);
  } else if (warp >= 2) {
    // ------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    const int r_in_tile = static_cast<int>(rank) * 128 + q * 32 + lane;
    uint32_t j = 0;
    for (int tile = pair; tile < total; tile += npairs, ++j) {
      const TileInfo ti = decode_pair_tile(tile, p, s_off, s_pt);
      const uint32_t acc = j & 1u, use = j >> 1;
      if (!sm100::mbar_wait(&tfull[acc], use & 1u)) {
        report_error(p.err, DEV_ERR_WAIT_TIMEOUT, 215, tile, static_cast<int>(rank));
        break;
      }
      sm100::tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      const bool valid = r_in_tile < ti.rows_valid;
      const int64_t row = static_cast<int64_t>(ti.row0) + r_in_tile;
      if (EPI != EPI_QKV && ti.half) {
        // M = 128 pair accumulator: lane l < 64 holds row 64 * rank + l, tile
        // columns [0, 128); lane 64 + l the same row, columns [128, 256).
        const int tl = q * 32 + lane;
        const int rh = static_cast<int>(rank) * 64 + (tl & 63);
        const int upper = tl >> 6;
        const bool valid_h = rh < ti.rows_valid;
        const int64_t row_h = static_cast<int64_t>(ti.row0) + rh;
        if constexpr (EPI == EPI_SWIGLU) {
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            uint32_t rg[32], ru[32];
            sm100::tmem_ld32(t_row + c * 32, rg);
            sm100::tmem_ld32(t_row + 64 + c * 32, ru);
            sm100::tmem_wait_ld();
            const int col = ti.nt * (BN / 2) + upper * 64 + c * 32;
            if (valid_h && col < p.N) {
              float v[32];
#pragma unroll
              for (int i = 0; i < 32; ++i)
                v[i] = silu(__uint_as_float(rg[i])) * __uint_as_float(ru[i]);
              store32(p.out + row_h * p.ldo + col, v);
            }
          }
        } else {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t r[32];
            sm100::tmem_ld32(t_row + c * 32, r);
            sm100::tmem_wait_ld();
            const int col = ti.nt * BN + upper * 128 + c * 32;
            if (valid_h && col < p.N) {
              float v[32];
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
              store32(p.out + row_h * p.ldo + col, v);
            }
          }
        }
      } else if constexpr (EPI == EPI_PLAIN) {
        const int n0 = ti.nt * BN;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          sm100::tmem_ld32(t_row + c * 32, r);
          sm100::tmem_wait_ld();
          const int col = n0 + c * 32;
          if (valid && col < p.N) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
            if (p.bias) {
              float bv[32];
              load32(p.bias + col, bv);
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] += bv[i];
            }
            if (p.residual) {
              float rv[32];
              load32(p.residual + row * p.ldr + col, rv);
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = rv[i] + v[i];
            }
            if (p.out_f32) {
              float4 *o = reinterpret_cast<float4 *>(reinterpret_cast<float *>(p.out) + row * p.ldo + col);
#pragma unroll
              for (int qq = 0; qq < 8; ++qq)
                o[qq] = make_float4(v[4 * qq], v[4 * qq + 1], v[4 * qq + 2], v[4 * qq + 3]);
            } else {
              store32(p.out + row * p.ldo + col, v);
            }
          }
        }
      } else if constexpr (EPI == EPI_QKV) {
        // Two 128-wide heads per 256-column tile; this thread owns one token.
        // Pass 1: inverse RMS of each q/k head.  Pass 2: 16-column blocks of
        // the rotate-half pairs (c, c + 64); the block's cos/sin (float4
        // loads) serve both heads.
        const int head0 = ti.nt * 2;
        const int n_qk = max(0, min(2, p.Hq + p.Hkv - head0));  // q/k heads in this tile
        float rinv[2] = {1.f, 1.f};
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          if (hh < n_qk) {
            float ss = 0.f;
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
              uint32_t x[32];
              sm100::tmem_ld32(t_row + hh * 128 + c * 32, x);
              sm100::tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) ss = fmaf(__uint_as_float(x[i]), __uint_as_float(x[i]), ss);
            }
            rinv[hh] = rsqrtf(ss * (1.f / 128.f) + p.eps);
          }
        }
        const int64_t b = row / p.seq, sq = row - b * p.seq;
        uint16_t *dst[2];
        const uint16_t *wn[2];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int head = head0 + hh;
          if (head < p.Hq) {
            dst[hh] = p.q_out + ((b * p.Hq + head) * p.seq + sq) * 128;
            wn[hh] = p.q_norm_w;
          } else if (head < p.Hq + p.Hkv) {
            dst[hh] = p.k_out + ((b * p.Hkv + (head - p.Hq)) * p.seq + sq) * 128;
            wn[hh] = p.k_norm_w;
          } else {
            dst[hh] = p.v_out + ((b * p.Hkv + (head - p.Hq - p.Hkv)) * p.seq + sq) * 128;
            wn[hh] = nullptr;
          }
        }
        const float4 *cs4 = reinterpret_cast<const float4 *>(p.rope_cos + (valid ? row : 0) * 64);
        const float4 *sn4 = reinterpret_cast<const float4 *>(p.rope_sin + (valid ? row : 0) * 64);
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float cc[16], sn[16];
          if (valid && n_qk > 0) {
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4) {
              const float4 a = cs4[c * 4 + v4], s4 = sn4[c * 4 + v4];
              cc[4 * v4] = a.x; cc[4 * v4 + 1] = a.y; cc[4 * v4 + 2] = a.z; cc[4 * v4 + 3] = a.w;
              sn[4 * v4] = s4.x; sn[4 * v4 + 1] = s4.y; sn[4 * v4 + 2] = s4.z; sn[4 * v4 + 3] = s4.w;
            }
          }
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            uint32_t x1[16], x2[16];
            sm100::tmem_ld16(t_row + hh * 128 + c * 16, x1);
            sm100::tmem_ld16(t_row + hh * 128 + 64 + c * 16, x2);
            sm100::tmem_wait_ld();
            if (valid) {  // no early exit: every tcgen05.ld needs the whole warp
              float o1[16], o2[16];
              if (hh >= n_qk) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  o1[i] = __uint_as_float(x1[i]);
                  o2[i] = __uint_as_float(x2[i]);
                }
              } else {
                float w1[16], w2[16];
                load16(wn[hh] + c * 16, w1);
                load16(wn[hh] + 64 + c * 16, w2);
                const float r = rinv[hh];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  const float y1 = (__uint_as_float(x1[i]) * r) * w1[i];
                  const float y2 = (__uint_as_float(x2[i]) * r) * w2[i];
                  o1[i] = y1 * cc[i] - y2 * sn[i];
                  o2[i] = y2 * cc[i] + y1 * sn[i];
                }
              }
              store16(dst[hh] + c * 16, o1);
              store16(dst[hh] + 64 + c * 16, o2);
            }
          }
        }
      } else {
        const int n0 = ti.nt * (BN / 2);
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
          uint32_t rg[32], ru[32];
          sm100::tmem_ld32(t_row + c * 32, rg);
          sm100::tmem_ld32(t_row + BN / 2 + c * 32, ru);
          sm100::tmem_wait_ld();
          const int col = n0 + c * 32;
          if (valid && col < p.N) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i)
              v[i] = silu(__uint_as_float(rg[i])) * __uint_as_float(ru[i]);
            store32(p.out + row * p.ldo + col, v);
          }
        }
      }
      sm100::tc_fence_before();
      sm100::mbar_arrive_cluster(sm100::mapa_shared(sm100::smem_u32(&tempty[acc]), 0));
    }
  }

  sm100::tc_fence_before();
  __syncthreads();
  sm100::cluster_sync();  // no CTA leaves while its peer may still signal it
  if (warp == 1) {
    __syncwarp();
    sm100::tc_fence_after();
    sm100::tmem_dealloc_pair(tmem_base, 2 * BN);
  }
}

template <int EPI>
int launch_gemm_pair(const CUtensorMap &ta, const CUtensorMap &tb, const GemmParams &p,
                     int max_pair_tiles, cudaStream_t s, const CUtensorMap *tb64 = nullptr) {
  const int smem = PairLayout::bytes(p.E);
  auto kern = gemm_pair_kernel<EPI>;
  { const int _st = ensure_smem_attr(reinterpret_cast<const void *>(kern), smem); if (_st) return _st; }
  const int npairs = max(1, min(max_pair_tiles, num_sms() / 2));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * npairs, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  Q35_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb, tb64 ? *tb64 : tb, p));
  count_launch();
  return Q35_OK;
}


// dst tile (rb, kb) = src rows [128 rb, 128 rb + 128) x cols [64 kb, 64 kb + 64),
// stored row-major as 128 x 64 contiguous elements (16 KB); one thread moves 16 B.
__global__ void pack_b_tiles_kernel(const uint16_t *__restrict__ src,
                                    uint16_t *__restrict__ dst, int64_t rows, int64_t K) {
  const int64_t kb_n = K / 64;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // 16-B chunk
  if (i >= rows * (K / 8)) return;
  const int64_t r = i / (K / 8), c8 = i % (K / 8);
  const int64_t kb = c8 / 8, cin = (c8 % 8) * 8;
  const int64_t rb = r / 128, rin = r % 128;
  const int64_t d = ((rb * kb_n + kb) * 128 + rin) * 64 + cin;
  *reinterpret_cast<uint4 *>(dst + d) = *reinterpret_cast<const uint4 *>(src + r * K + c8 * 8);
}


// cos/sin [rows, 64] of the rotary angles pos[axis(j)] * inv_freq[j] (fp32,
// precise sincosf), with axis(j) from the mRoPE section layout: chunked
// (interleaved == 0, REF cuda_qwen3_vl/kernels/mrope.py:19-35) or HF's T/H/W
// interleave.  One thread per (row, j).
__global__ void rope_table_kernel(const int64_t *__restrict__ pos, const float *__restrict__ inv_freq,
                                  int s0, int s1, int s2, int interleaved, int64_t rows,
                                  float *__restrict__ cos_t, float *__restrict__ sin_t) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * 64) return;
  const int64_t row = i / 64;
  const int j = static_cast<int>(i % 64);
  int ax;
  if (interleaved)
    ax = ((j % 3) == 1 && j < 3 * s1) ? 1 : (((j % 3) == 2 && j < 3 * s2) ? 2 : 0);
  else
    ax = j < s0 ? 0 : (j < s0 + s1 ? 1 : 2);
  float sn, cs;
  sincosf(static_cast<float>(pos[ax * rows + row]) * inv_freq[j], &sn, &cs);
  cos_t[i] = cs;
  sin_t[i] = sn;
}

}  // namespace
}  // namespace q35

using namespace q35;

static int gemm_dense(const void *a, const void *b, const void *bias,
                      const void *residual, void *out, int64_t M, int64_t N,
                      int64_t K, int out_f32, q35_stream_t stream) {
  if (!a || !b || !out) return fail(Q35_ERR_INVALID, "gemm: null pointer");
  if (M < 0 || N <= 0 || K <= 0) return fail(Q35_ERR_SHAPE, "gemm: bad shape");
  if (K % 8 != 0 || N % 32 != 0)
    return fail(Q35_ERR_SHAPE, "gemm: K %lld must be x8 and N %lld x32",
                (long long)K, (long long)N);
  if (M >= (int64_t(1) << 31) || N >= (int64_t(1) << 24))
    return fail(Q35_ERR_SHAPE, "gemm: M/N too large");
  if (!aligned16(out) || (residual && !aligned16(residual)) ||
      (bias && !aligned16(bias)))
    return fail(Q35_ERR_ALIGN, "gemm: out/bias/residual not 16-byte aligned");
  if (M == 0) return Q35_OK;
  int *err = device_error_word();
  if (!err) return fail(Q35_ERR_CUDA, "gemm: no device error word");
  const int sms = num_sms();
  const int64_t mt = (M + kBM - 1) / kBM;
  // Pick the N tile that finishes the last wave soonest (time ~ waves * BN).
  const int64_t t256 = mt * ((N + 255) / 256), t128 = mt * ((N + 127) / 128);
  const int64_t cost256 = ((t256 + sms - 1) / sms) * 2, cost128 = (t128 + sms - 1) / sms;
  // 256-wide tiles run on CTA pairs (cta_group::2), which sustain a higher
  // fraction of peak than single-CTA 128-wide tiles: prefer them unless they
  // would need clearly more waves.
  const int BN = (N % 256 == 0 && cost256 <= cost128 + 2) ? 256 : 128;
  CUtensorMap ta, tb;
  int st = make_tmap_bf16_2d(&ta, a, K, M, K * 2, kBK, kBM);
  if (st) return st;
  st = make_tmap_bf16_2d(&tb, b, K, N, K * 2, kBK, BN / 2);
  if (st) return st;
  GemmParams p{};
  p.M = static_cast<int>(M);
  p.E = 1;
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.n_tiles = static_cast<int>((N + BN - 1) / BN);
  p.b_rows_per_group = static_cast<int>(N);
  p.b_tile_step = BN;
  p.b_second_off = BN / 2;
  p.out = static_cast<uint16_t *>(out);
  p.ldo = N;
  p.bias = static_cast<const uint16_t *>(bias);
  p.residual = static_cast<const uint16_t *>(residual);
  p.ldr = N;
  p.err = err;
  p.out_f32 = out_f32;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int tiles = static_cast<int>(mt * p.n_tiles);
  if (BN == 256) {
    // CTA pairs (cta_group::2) on 256 x 256 tiles; B boxes are 128 rows per CTA.
    CUtensorMap tb2;
    st = make_tmap_bf16_2d(&tb2, b, K, N, K * 2, kBK, 128);
    if (st) return st;
    const int pair_tiles = static_cast<int>(((M + 255) / 256) * p.n_tiles);
    return launch_gemm_pair<EPI_PLAIN>(ta, tb2, p, pair_tiles, s);
  }
  return launch_gemm<128, EPI_PLAIN, 6>(ta, tb, p, tiles, s);
}

// out[m, n] = sum_s ws[s, m, n] (fixed order) + bias[n] + residual[m, n]; bf16
// or fp32 output.  Thread = 4 consecutive outputs.
__global__ void __launch_bounds__(256) splitk_reduce_kernel(
    const float *__restrict__ ws, int splits, int64_t plane, const uint16_t *__restrict__ bias,
    const uint16_t *__restrict__ residual, void *__restrict__ out, int out_f32, int64_t N) {
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  if (i >= plane) return;
  float4 acc = *reinterpret_cast<const float4 *>(ws + i);
  for (int s = 1; s < splits; ++s) {
    const float4 v = *reinterpret_cast<const float4 *>(ws + s * plane + i);
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
  float r[4] = {acc.x, acc.y, acc.z, acc.w};
  if (bias) {
    const int64_t n = i % N;
#pragma unroll
    for (int j = 0; j < 4; ++j) r[j] += bf2f(bias[n + j]);
  }
  if (residual) {
#pragma unroll
    for (int j = 0; j < 4; ++j) r[j] = bf2f(residual[i + j]) + r[j];
  }
  if (out_f32) {
    *reinterpret_cast<float4 *>(static_cast<float *>(out) + i) = make_float4(r[0], r[1], r[2], r[3]);
  } else {
    uint2 u;
    u.x = pack_bf2(r[0], r[1]);
    u.y = pack_bf2(r[2], r[3]);
    *reinterpret_cast<uint2 *>(static_cast<uint16_t *>(out) + i) = u;
  }
}

// Split-K dense GEMM for few rows (decode-sized M): the 1-CTA tcgen05 kernel
// writes k_splits fp32 partial planes [k_splits, M, N] into `workspace`, so
// ceil(N/128) * k_splits CTAs share the weight stream instead of ceil(N/128);
// the reduce kernel adds them in a fixed order with bias and residual.
extern "C" int q35_gemm_bf16_splitk(const void *a, const void *b, const void *bias,
                                    const void *residual, void *out, int out_f32, int64_t M,
                                    int64_t N, int64_t K, int k_splits, float *workspace,
                                    q35_stream_t stream) {
  if (!a || !b || !out || !workspace) return fail(Q35_ERR_INVALID, "gemm_splitk: null pointer");
  if (M < 0 || N <= 0 || K <= 0 || N % 32 != 0 || K % kBK != 0 || k_splits < 1 ||
      (K / kBK) % k_splits != 0)
    return fail(Q35_ERR_SHAPE, "gemm_splitk: K %lld must be x64 with %d splits dividing its "
                "k-blocks, N %lld x32", (long long)K, k_splits, (long long)N);
  if (M >= (int64_t(1) << 31) || N >= (int64_t(1) << 24))
    return fail(Q35_ERR_SHAPE, "gemm_splitk: M/N too large");
  if (!aligned16(out) || !aligned16(workspace) || (residual && !aligned16(residual)) ||
      (bias && !aligned16(bias)))
    return fail(Q35_ERR_ALIGN, "gemm_splitk: pointers not 16-byte aligned");
  if (M == 0) return Q35_OK;
  int *err = device_error_word();
  if (!err) return fail(Q35_ERR_CUDA, "gemm_splitk: no device error word");
  CUtensorMap ta, tb;
  int st = make_tmap_bf16_2d(&ta, a, K, M, K * 2, kBK, kBM);
  if (st) return st;
  st = make_tmap_bf16_2d(&tb, b, K, N, K * 2, kBK, 64);
  if (st) return st;
  GemmParams p{};
  p.M = static_cast<int>(M);
  p.E = 1;
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.n_tiles = static_cast<int>((N + 127) / 128);
  p.b_rows_per_group = static_cast<int>(N);
  p.b_tile_step = 128;
  p.b_second_off = 64;
  p.out = reinterpret_cast<uint16_t *>(workspace);
  p.ldo = N;
  p.err = err;
  p.out_f32 = 1;
  p.k_splits = k_splits;
  p.split_stride = M * N;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int tiles = static_cast<int>(((M + kBM - 1) / kBM) * p.n_tiles * k_splits);
  st = launch_gemm<128, EPI_PLAIN, 6>(ta, tb, p, tiles, s);
  if (st) return st;
  const int64_t plane = M * N;
  splitk_reduce_kernel<<<static_cast<unsigned>((plane / 4 + 255) / 256), 256, 0, s>>>(
      workspace, k_splits, plane, static_cast<const uint16_t *>(bias),
      static_cast<const uint16_t *>(residual), out, out_f32 ? 1 : 0, N);
  Q35_LAUNCH_CHECK("gemm_splitk reduce launch");
  return Q35_OK;
}

extern "C" int q35_gemm_bf16(const void *a, const void *b, const void *bias,
                             const void *residual, void *out, int64_t M,
                             int64_t N, int64_t K, q35_stream_t stream) {
  return gemm_dense(a, b, bias, residual, out, M, N, K, 0, stream);
}

extern "C" int q35_gemm_bf16_f32out(const void *a, const void *b,
                                    const void *bias, const void *residual,
                                    float *out, int64_t M, int64_t N,
                                    int64_t K, q35_stream_t stream) {
  return gemm_dense(a, b, bias, residual, out, M, N, K, 1, stream);
}

// Router logits on the tensor cores.  The fp32 gate weight is stored as three
// bf16 planes w3[e] = [lo | mid | hi] with lo + mid + hi == w exactly (each
// plane holds 8 significant bits), and x is bf16, so every product x*plane is
// exact in fp32; logits = sum over the 3H columns of x3 * w3 with x3 = [x|x|x]
// (A's K coordinate wraps at H instead of materialising x3).  The tensor
// core's fp32 accumulation truncates relative to the running sum, so the
// small planes are accumulated first and K is split into k_splits fresh
// accumulators written as partial planes [k_splits, T, E]; the top-k kernel
// adds them in a fixed order (deterministic).
extern "C" int q35_router_logits_tc(const void *x, const void *w3,
                                    float *partials, int64_t T, int H, int E,
                                    int k_splits, q35_stream_t stream) {
  if (!x || !w3 || !partials) return fail(Q35_ERR_INVALID, "router_logits_tc: null pointer");
  if (k_splits < 1 || (3 * H / kBK) % k_splits != 0)
    return fail(Q35_ERR_SHAPE, "router_logits_tc: %d splits must divide %d k-blocks", k_splits,
                3 * H / kBK);
  if (T < 0 || H <= 0 || H % kBK != 0 || E <= 0 || E % 32 != 0 || E > 4096)
    return fail(Q35_ERR_SHAPE, "router_logits_tc: H %d (x64) E %d (x32)", H, E);
  if (!aligned16(partials)) return fail(Q35_ERR_ALIGN, "router_logits_tc: output alignment");
  if (T == 0) return Q35_OK;
  int *err = device_error_word();
  if (!err) return fail(Q35_ERR_CUDA, "router_logits_tc: no device error word");
  // One 128-wide N tile when E allows (x and its three planes cross L2 once),
  // else 64-wide tiles.
  const int BN = E % 128 == 0 ? 128 : 64;
  CUtensorMap ta, tb;
  int st = make_tmap_bf16_2d(&ta, x, H, T, static_cast<uint64_t>(H) * 2, kBK, kBM);
  if (st) return st;
  st = make_tmap_bf16_2d(&tb, w3, 3 * static_cast<uint64_t>(H), E,
                         3 * static_cast<uint64_t>(H) * 2, kBK, BN / 2);
  if (st) return st;
  GemmParams p{};
  p.M = static_cast<int>(T);
  p.E = 1;
  p.N = E;
  p.K = 3 * H;
  p.n_tiles = (E + BN - 1) / BN;
  p.b_rows_per_group = E;
  p.b_tile_step = BN;
  p.b_second_off = BN / 2;
  p.out = reinterpret_cast<uint16_t *>(partials);
  p.ldo = E;
  p.err = err;
  p.out_f32 = 1;
  p.a_k_wrap = H;
  p.k_splits = k_splits;
  p.split_stride = T * static_cast<int64_t>(E);
  const int tiles = static_cast<int>(((T + kBM - 1) / kBM) * p.n_tiles * k_splits);
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  if (BN == 128) return launch_gemm<128, EPI_PLAIN, 6>(ta, tb, p, tiles, cs);
  return launch_gemm<64, EPI_PLAIN, 8>(ta, tb, p, tiles, cs);
}

// Re-lays a K-major bf16 matrix [rows, K] (e.g. all experts' weights,
// rows = E * R) as contiguous 128-row x 64-column tiles, so that every TMA box
// the grouped GEMM loads is one 16 KB contiguous read instead of 128 strided
// 128-byte segments.  rows % 128 == 0, K % 64 == 0.
extern "C" int q35_pack_b_tiles(const void *src, void *dst, int64_t rows, int64_t K,
                                q35_stream_t stream) {
  if (!src || !dst) return fail(Q35_ERR_INVALID, "pack_b_tiles: null pointer");
  if (rows <= 0 || K <= 0 || rows % 128 != 0 || K % 64 != 0)
    return fail(Q35_ERR_SHAPE, "pack_b_tiles: rows %lld (x128) K %lld (x64)", (long long)rows,
                (long long)K);
  if (!aligned16(src) || !aligned16(dst)) return fail(Q35_ERR_ALIGN, "pack_b_tiles: alignment");
  const int64_t n = rows * (K / 8);
  pack_b_tiles_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0,
                        reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t *>(src), static_cast<uint16_t *>(dst), rows, K);
  Q35_LAUNCH_CHECK("pack_b_tiles launch");
  return Q35_OK;
}

// Fused q/k/v projection: GEMM of x [B*S, H] with the concatenated weight
// w_qkv [(Hq + 2 Hkv) * 128, H] on CTA pairs, whose epilogue applies the
// per-head RMSNorm (q_norm / k_norm weights) and the mRoPE rotation to the q
// and k heads and writes q [B,Hq,S,128], k and v [B,Hkv,S,128] head-major.
// workspace: fp32 [2 * B * S * 64] for the rotary cos/sin table.
extern "C" int q35_qkv_proj_norm_rope(const void *x, const void *w_qkv, const void *q_w,
                                      const void *k_w, const int64_t *positions,
                                      const float *inv_freq, const int32_t *sections,
                                      int interleaved, void *q, void *k, void *v, int64_t B,
                                      int64_t S, int H, int Hq, int Hkv, float eps,
                                      float *workspace, q35_stream_t stream) {
  if (!x || !w_qkv || !q_w || !k_w || !positions || !inv_freq || !sections || !q || !k || !v ||
      !workspace)
    return fail(Q35_ERR_INVALID, "qkv_proj_norm_rope: null pointer");
  const int64_t M = B * S;
  const int heads = Hq + 2 * Hkv;
  if (M <= 0 || H <= 0 || H % 8 != 0 || Hq <= 0 || Hkv <= 0 || heads % 2 != 0)
    return fail(Q35_ERR_SHAPE, "qkv_proj_norm_rope: H %d (x8), heads %d (even)", H, heads);
  if (sections[0] + sections[1] + sections[2] != 64)
    return fail(Q35_ERR_SHAPE, "qkv_proj_norm_rope: sections must sum to 64 (head_dim 128)");
  if (M >= (int64_t(1) << 31)) return fail(Q35_ERR_SHAPE, "qkv_proj_norm_rope: too many rows");
  int *err = device_error_word();
  if (!err) return fail(Q35_ERR_CUDA, "qkv_proj_norm_rope: no device error word");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  float *cos_t = workspace, *sin_t = workspace + M * 64;
  rope_table_kernel<<<static_cast<unsigned>((M * 64 + 255) / 256), 256, 0, s>>>(
      positions, inv_freq, sections[0], sections[1], sections[2], interleaved ? 1 : 0, M, cos_t,
      sin_t);
  Q35_LAUNCH_CHECK("rope_table launch");
  const int64_t N = static_cast<int64_t>(heads) * 128;
  CUtensorMap ta, tb;
  int st = make_tmap_bf16_2d(&ta, x, H, M, static_cast<uint64_t>(H) * 2, kBK, kBM);
  if (st) return st;
  st = make_tmap_bf16_2d(&tb, w_qkv, H, N, static_cast<uint64_t>(H) * 2, kBK, 128);
  if (st) return st;
  GemmParams p{};
  p.M = static_cast<int>(M);
  p.E = 1;
  p.N = static_cast<int>(N);
  p.K = H;
  p.n_tiles = heads / 2;
  p.b_rows_per_group = static_cast<int>(N);
  p.b_tile_step = 256;
  p.b_second_off = 128;
  p.err = err;
  p.q_norm_w = static_cast<const uint16_t *>(q_w);
  p.k_norm_w = static_cast<const uint16_t *>(k_w);
  p.rope_cos = cos_t;
  p.rope_sin = sin_t;
  p.q_out = static_cast<uint16_t *>(q);
  p.k_out = static_cast<uint16_t *>(k);
  p.v_out = static_cast<uint16_t *>(v);
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.seq = static_cast<int>(S);
  p.eps = eps;
  const int pair_tiles = static_cast<int>(((M + 255) / 256) * p.n_tiles);
  return launch_gemm_pair<EPI_QKV>(ta, tb, p, pair_tiles, s);
}

static int grouped_common(const void *a, const void *w, void *out,
                          const int32_t *offsets, const int32_t *tile_offsets,
                          int E, int64_t rows_cap, int64_t K, int64_t N_out,
                          int64_t b_rows_per_group, int swiglu, int packed,
                          q35_stream_t stream) {
  if (!a || !w || !out || !offsets || !tile_offsets)
    return fail(Q35_ERR_INVALID, "grouped_gemm: null pointer");
  if (E < 1 || E > kMaxGroups)
    return fail(Q35_ERR_SHAPE, "grouped_gemm: groups %d (1..%d)", E, kMaxGroups);
  if (rows_cap < 0 || rows_cap >= (int64_t(1) << 31))
    return fail(Q35_ERR_SHAPE, "grouped_gemm: rows_cap out of range");
  if (K % 8 != 0 || N_out % 32 != 0)
    return fail(Q35_ERR_SHAPE, "grouped_gemm: K %lld (x8) / N %lld (x32)",
                (long long)K, (long long)N_out);
  if (!aligned16(out)) return fail(Q35_ERR_ALIGN, "grouped_gemm: out alignment");
  if (rows_cap == 0) return Q35_OK;
  int *err = device_error_word();
  if (!err) return fail(Q35_ERR_CUDA, "grouped_gemm: no device error word");
  constexpr int BN = 256;
  CUtensorMap ta, tb;
  int st = make_tmap_bf16_2d(&ta, a, K, rows_cap, K * 2, kBK, kBM);
  if (st) return st;
  if (packed) {
    if (K % kBK != 0 || b_rows_per_group % 128 != 0 || (swiglu && N_out % 128 != 0))
      return fail(Q35_ERR_SHAPE, "grouped_gemm: packed weights need K %% 64, rows %% 128");
    // packed tiles viewed as [E * R * K / 64, 64] rows of 128 B
    st = make_tmap_bf16_2d(&tb, w, kBK, static_cast<uint64_t>(E) * b_rows_per_group * (K / kBK),
                           kBK * 2, kBK, BN / 2);
  } else {
    st = make_tmap_bf16_2d(&tb, w, K, static_cast<uint64_t>(E) * b_rows_per_group,
                           K * 2, kBK, BN / 2);
  }
  if (st) return st;
  GemmParams p{};
  p.offsets = offsets;
  p.tile_offsets = tile_offsets;
  p.E = E;
  p.N = static_cast<int>(N_out);
  p.K = static_cast<int>(K);
  p.n_tiles = static_cast<int>(swiglu ? (N_out + BN / 2 - 1) / (BN / 2)
                                      : (N_out + BN - 1) / BN);
  p.b_rows_per_group = static_cast<int>(b_rows_per_group);
  p.b_tile_step = swiglu ? BN / 2 : BN;
  p.b_second_off = swiglu ? static_cast<int>(N_out) : BN / 2;
  p.out = static_cast<uint16_t *>(out);
  p.ldo = N_out;
  p.err = err;
  p.b_packed = packed ? 1 : 0;
  // Upper bound on tiles: every group may add one partial M tile.
  const int64_t max_tiles = ((rows_cap + kBM - 1) / kBM + E) * p.n_tiles;
  const int mt = static_cast<int>(max_tiles < (1 << 30) ? max_tiles : (1 << 30));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // CTA pairs (cta_group::2): 256-row tiles per group, B boxes of 128 rows.
  const int64_t max_pair = ((rows_cap + 255) / 256 + E) * p.n_tiles;
  const int mp = static_cast<int>(max_pair < (1 << 30) ? max_pair : (1 << 30));
  (void)mt;
  if (swiglu) {
    // 64-row B boxes for the gate/up halves of M = 128 pair tiles
    CUtensorMap tb64 = tb;
    if (!packed) {
      st = make_tmap_bf16_2d(&tb64, w, K, static_cast<uint64_t>(E) * b_rows_per_group, K * 2, kBK, 64);
      if (st) return st;
    }
    return launch_gemm_pair<EPI_SWIGLU>(ta, tb, p, mp, s, &tb64);
  }
  return launch_gemm_pair<EPI_PLAIN>(ta, tb, p, mp, s);
}

extern "C" int q35_grouped_gemm_gateup_swiglu(
    const void *a, const void *w_gate_up, void *act, const int32_t *offsets,
    const int32_t *tile_offsets, int E, int64_t rows_cap, int H, int I,
    int w_packed, q35_stream_t stream) {
  if (H <= 0 || I <= 0) return fail(Q35_ERR_SHAPE, "gate_up: bad H/I");
  return grouped_common(a, w_gate_up, act, offsets, tile_offsets, E, rows_cap,
                        H, I, 2 * static_cast<int64_t>(I), 1, w_packed, stream);
}

extern "C" int q35_grouped_gemm_down(const void *act, const void *w_down,
                                     void *y, const int32_t *offsets,
                                     const int32_t *tile_offsets, int E,
                                     int64_t rows_cap, int H, int I,
                                     int w_packed, q35_stream_t stream) {
  if (H <= 0 || I <= 0) return fail(Q35_ERR_SHAPE, "down: bad H/I");
  return grouped_common(act, w_down, y, offsets, tile_offsets, E, rows_cap, I,
                        H, H, 0, w_packed, stream);
}
