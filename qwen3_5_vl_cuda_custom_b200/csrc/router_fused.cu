// Tensor-core MoE router with the permutation's count pass, and the
// one-launch scan + scatter that completes the (expert, token) permutation.
//
// Router (REF cuda_qwen3_vl/modules/moe.py:60-65: logits = x @ gate^T,
// softmax in fp32, top-k sorted descending with ties to the lower index as in
// REF csrc/moe_routing_op.cu:36-53, renormalised), computed in fp32 exactly
// enough to reproduce an fp32 GEMV:
//   * the fp32 gate weight is held as three bf16 planes lo + mid + hi == w
//     (8 significant bits each, q35_router_split_weights); x is bf16, so every
//     product x * plane is exact in fp32;
//   * router_logits_cluster_kernel: a cluster of 4 CTAs owns 128 tokens (one
//     permutation chunk); CTA q of the cluster takes x columns
//     [q*H/4, (q+1)*H/4) and runs the three planes into three separate TMEM
//     accumulators (M = 128 tokens, N = E experts), so x is staged once per
//     k-block for all three planes.  Each CTA sums its planes in fp32
//     ((lo + mid) + hi, small first) and stores the partial rows into the
//     shared memory of the CTA that reduces them (CTA q owns rows
//     [32q, 32q + 32)); after a cluster barrier each CTA adds the four
//     partials in a fixed order (deterministic) plus the bias and writes the
//     fp32 logits.  No split-K partial planes go through HBM;
//   * topk_count_kernel: softmax / top-k / renormalisation, one warp per token
//     (one-instruction warp max/min reductions keep the k selection rounds
//     short), and the per-chunk expert counts of the permutation.
//
// Permutation (REF modules/moe.py:71-76 visits tokens per expert in ascending
// order, i.e. a stable (expert, token) sort): permute_scan_scatter_kernel runs
// one CTA per 128-token chunk; each CTA re-derives its chunk bases and the
// expert offsets from chunk_counts (O(chunks x E) reads, L2-resident), then
// ranks its tokens within the chunk by popcount of per-expert token masks.
// Integer work, bit-exact.
#include <float.h>

#include "sm100.cuh"

namespace q35 {
namespace {

constexpr int kRTok = 128;      // tokens per cluster (= permutation chunk)
constexpr int kRSplit = 4;      // CTAs per cluster (K split)
constexpr int kRBK = 64;        // bf16 columns per k-block (one 128-byte row)
constexpr int kRStages = 3;
constexpr int kRThreads = 256;  // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue; all reduce

template <int E>
struct RouterLayout {
  static constexpr int kA = kRTok * kRBK * 2;        // 16 KB
  static constexpr int kB = E * kRBK * 2;            // one plane
  static constexpr int kStage = kA + 3 * kB;
  static constexpr int kPartStride = E + 4;          // floats per partial row (16-B rows)
  // receive buffer [source CTA][32 rows][E + 4] of the rows this CTA reduces
  static constexpr int kPartBytes = kRSplit * 32 * kPartStride * 4;
  static constexpr int kMain = (kRStages * kStage > kPartBytes) ? kRStages * kStage : kPartBytes;
  static constexpr int kBarOff = kMain;
  static constexpr int kEnd = kBarOff + (2 * kRStages + 1) * 8 + 16;
  // At least 120 KB: one CTA per SM, so no CTA ever waits for another's
  // tensor memory (two CTAs of one cluster on one SM would deadlock there).
  static constexpr int kMinBytes = 120 * 1024;
  static constexpr int kBytes = (1024 + kEnd > kMinBytes) ? 1024 + kEnd : kMinBytes;
  // tensor-memory columns: three E-column accumulators, rounded to a power of two
  static constexpr int kTmemCols = (3 * E <= 128) ? 128 : (3 * E <= 256) ? 256 : 512;
};

__device__ __forceinline__ void st_cluster_v4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b),
               "f"(c), "f"(d)
               : "memory");
}

// Order-preserving map of fp32 onto uint32 (for a one-instruction warp max).
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float from_order_key(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

template <int E>
__global__ void __launch_bounds__(kRThreads, 1) router_logits_cluster_kernel(
    const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
    const float *__restrict__ bias, float *__restrict__ logits, int32_t *__restrict__ chunk_counts,
    int64_t T, int H, int *err) {
  using L = RouterLayout<E>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::kBarOff);
  uint64_t *empty = full + kRStages;
  uint64_t *acc_full = empty + kRStages;
  uint32_t *s_tmem = reinterpret_cast<uint32_t *>(acc_full + 1);
  float *part = reinterpret_cast<float *>(smem);  // reuses the stages after the mainloop

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t q = sm100::cluster_ctarank();
  const int64_t chunk = blockIdx.x / kRSplit;
  const int64_t t0 = chunk * kRTok;
  const int hq = H / kRSplit;
  const int nkb = hq / kRBK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kRStages; ++i) {
      sm100::mbar_init(&full[i], 1);
      sm100::mbar_init(&empty[i], 1);
    }
    sm100::mbar_init(acc_full, 1);
    sm100::fence_mbar_init();
    sm100::prefetch_tensormap(&tmX);
    sm100::prefetch_tensormap(&tmW);
  }
  if (warp == 1) sm100::tmem_alloc(s_tmem, L::kTmemCols);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *s_tmem;
  bool ok = true;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------ TMA producer
    for (int kb = 0; kb < nkb; ++kb) {
      const int st = kb % kRStages;
      const uint32_t ph = (kb / kRStages) & 1u;
      if (!sm100::mbar_wait(&empty[st], ph ^ 1u)) {
        report_error(err, DEV_ERR_WAIT_TIMEOUT, 401, static_cast<int>(chunk), kb);
        break;
      }
      uint8_t *sa = smem + st * L::kStage;
      const int col = static_cast<int>(q) * hq + kb * kRBK;
      sm100::mbar_arrive_expect_tx(&full[st], L::kStage);
      sm100::tma_load_2d(sa, &tmX, &full[st], col, static_cast<int32_t>(t0));
#pragma unroll
      for (int p = 0; p < 3; ++p)
        sm100::tma_load_2d(sa + L::kA + p * L::kB, &tmW, &full[st], p * H + col, 0);
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = sm100::idesc_bf16_f32(kRTok, E);
    for (int kb = 0; kb < nkb; ++kb) {
      const int st = kb % kRStages;
      const uint32_t ph = (kb / kRStages) & 1u;
      if (!sm100::mbar_wait(&full[st], ph)) {
        report_error(err, DEV_ERR_WAIT_TIMEOUT, 402, static_cast<int>(chunk), kb);
        break;
      }
      sm100::tc_fence_after();
      const uint32_t sa = sm100::smem_u32(smem + st * L::kStage);
      const uint64_t adesc = sm100::sw128_kmajor_desc(sa);
#pragma unroll
      for (int p = 0; p < 3; ++p) {
        const uint64_t bdesc = sm100::sw128_kmajor_desc(sa + L::kA + p * L::kB);
#pragma unroll
        for (int kk = 0; kk < kRBK / 16; ++kk)
          sm100::mma_bf16_ss(tmem + p * E, adesc + 2 * kk, bdesc + 2 * kk, idesc,
                             (kb | kk) != 0 ? 1u : 0u);
      }
      sm100::mma_commit(&empty[st]);
    }
    sm100::mma_commit(acc_full);
  }
  // Every CTA of the cluster past its mainloop (the epilogue warps waited for
  // the accumulators first), so every CTA's stage memory may be overwritten.
  if (warp >= 2 && warp < 6) {
    if (!sm100::mbar_wait(acc_full, 0)) {
      report_error(err, DEV_ERR_WAIT_TIMEOUT, 403, static_cast<int>(chunk), static_cast<int>(q));
      ok = false;
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::cluster_sync();
  sm100::tc_fence_after();
  if (warp >= 2 && warp < 6) {
    // ------------------------------------------------ planes -> fp32 partial
    // Row r = 32 q4 + lane of this CTA's accumulators goes to CTA q4 (the CTA
    // that reduces rows [32 q4, 32 q4 + 32)), slot q, with plain stores into
    // its shared memory.
    const int q4 = warp & 3;
    const uint32_t t_row = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    const uint32_t dst0 =
        sm100::mapa_shared(sm100::smem_u32(part), static_cast<uint32_t>(q4)) +
        static_cast<uint32_t>(((q * 32 + lane) * L::kPartStride) * 4);
#pragma unroll 1
    for (int c = 0; c < E / 32; ++c) {
      uint32_t lo[32], mid[32], hi[32];
      sm100::tmem_ld32(t_row + c * 32, lo);
      sm100::tmem_ld32(t_row + E + c * 32, mid);
      sm100::tmem_ld32(t_row + 2 * E + c * 32, hi);
      sm100::tmem_wait_ld();
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i)
        v[i] = ok ? (__uint_as_float(lo[i]) + __uint_as_float(mid[i])) + __uint_as_float(hi[i])
                  : 0.f;
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        st_cluster_v4(dst0 + static_cast<uint32_t>((c * 32 + i) * 4), v[i], v[i + 1], v[i + 2],
                      v[i + 3]);
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::cluster_sync();  // every partial row delivered to its reducing CTA
  if (warp == 1) {
    __syncwarp();
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, L::kTmemCols);
  }
  // ------------------------------------------------ reduce to logits
  // Rows [32 q, 32 q + 32) of the chunk: the four partials in a fixed order
  // (K order), plus the bias; consecutive threads take consecutive experts
  // (coalesced stores).
  for (int i2 = threadIdx.x; i2 < 32 * E; i2 += kRThreads) {
    const int i = i2 / E, e = i2 - i * E;
    const int64_t t = t0 + static_cast<int>(q) * 32 + i;
    if (t >= T) break;
    float v = part[i * L::kPartStride + e];
#pragma unroll
    for (int c = 1; c < kRSplit; ++c) v += part[(c * 32 + i) * L::kPartStride + e];
    if (bias) v += bias[e];
    logits[t * E + e] = v;
  }
  if (q == 0 && chunk_counts != nullptr)
    for (int e = threadIdx.x; e < E; e += kRThreads) chunk_counts[chunk * E + e] = 0;
}

// Softmax, top-k (ties to the lower index) and renormalisation of the fp32
// logits, one warp per token (lane l holds experts l + 32 j); the selected
// experts are counted into chunk_counts[t / 128] (zeroed by the logits
// kernel; integer atomics, so the counts do not depend on their order).
template <int EPT>
__global__ void __launch_bounds__(256) topk_count_kernel(
    const float *__restrict__ logits, int32_t *__restrict__ idx_out, float *__restrict__ w_out,
    int32_t *__restrict__ chunk_counts, int64_t T, int k, int renorm) {
  constexpr int E = 32 * EPT;
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  float l[EPT];
  uint32_t mkey = 0u;
#pragma unroll
  for (int j = 0; j < EPT; ++j) {
    l[j] = logits[t * E + lane + 32 * j];
    mkey = max(mkey, order_key(l[j]));
  }
  const float m = from_order_key(__reduce_max_sync(0xffffffffu, mkey));
  float pr[EPT], s = 0.f;
#pragma unroll
  for (int j = 0; j < EPT; ++j) {
    pr[j] = expf(l[j] - m);
    s += pr[j];
  }
  s = warp_sum(s);
  // selection keys: probability bits + 1 (p >= 0, so the bits order like the
  // values); 0 marks a taken expert
  uint32_t key[EPT];
#pragma unroll
  for (int j = 0; j < EPT; ++j) key[j] = __float_as_uint(pr[j] / s) + 1u;
  float sel_v = 0.f, tot = 0.f;
  int sel_i = 0;
  for (int rr = 0; rr < k; ++rr) {
    uint32_t bk = 0u;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < EPT; ++j)
      if (key[j] > bk) {  // first (lowest index) maximum of this lane
        bk = key[j];
        bi = lane + 32 * j;
      }
    const uint32_t wk = __reduce_max_sync(0xffffffffu, bk);
    const int wi = __reduce_min_sync(0xffffffffu, bk == wk ? bi : 0x7fffffff);
    if ((wi & 31) == lane) {
#pragma unroll
      for (int j = 0; j < EPT; ++j)
        if (lane + 32 * j == wi) key[j] = 0u;
    }
    const float bv = __uint_as_float(wk - 1u);
    if (lane == rr) {
      sel_v = bv;
      sel_i = wi;
    }
    tot += bv;
  }
  if (lane < k) {
    idx_out[t * k + lane] = sel_i;
    w_out[t * k + lane] = renorm ? sel_v / tot : sel_v;
    if (chunk_counts) atomicAdd(&chunk_counts[(t / kRTok) * E + sel_i], 1);
  }
}

// ---------------------------------------------------------------------------
constexpr int kPChunk = 128;
constexpr int kPTile = 128;     // grouped-GEMM M tile of tile_offsets
constexpr int kPThreads = 256;

// One CTA per 128-token chunk.  chunk_counts [n_chunks, E] from the router.
__global__ void __launch_bounds__(kPThreads) permute_scan_scatter_kernel(
    const int32_t *__restrict__ idx, int64_t T, int k, int E, int64_t n_chunks,
    const int32_t *__restrict__ chunk_counts, int32_t *__restrict__ counts,
    int32_t *__restrict__ offsets, int32_t *__restrict__ tile_offsets,
    int32_t *__restrict__ sorted_tok, int32_t *__restrict__ slot_pos, int *err) {
  extern __shared__ int32_t psm[];
  int32_t *s_base = psm;           // [E] this chunk's base within each expert
  int32_t *s_off = psm + E;        // [E] expert offsets
  int32_t *s_tot = psm + 2 * E;    // [E] expert totals
  uint32_t(*mask)[4] = reinterpret_cast<uint32_t(*)[4]>(psm + 3 * E);
  int32_t *s_ids = psm + 7 * E;    // [kPChunk * k] this chunk's expert ids
  const int64_t c = blockIdx.x;
  // The chunk's ids first, as one coalesced sweep: the loads are all in
  // flight together and overlap the chunk-count reads below.
  const int64_t t_lo = c * kPChunk;
  const int n_ids = static_cast<int>(T - t_lo < kPChunk ? T - t_lo : kPChunk) * k;
  const int32_t *ids_g = idx + t_lo * k;
#pragma unroll 4
  for (int i = threadIdx.x; i < n_ids; i += kPThreads) s_ids[i] = __ldg(ids_g + i);
  for (int e = threadIdx.x; e < E; e += kPThreads) {
    s_base[e] = 0;
    s_tot[e] = 0;
  }
  for (int i = threadIdx.x; i < E * 4; i += kPThreads) mask[i >> 2][i & 3] = 0u;
  __syncthreads();
  // Chunk bases and expert totals: one coalesced sweep over all chunk counts
  // by the whole CTA (independent loads, a few in flight per thread), summed
  // with shared-memory atomics -- no per-expert serial walk over the chunks.
  {
    const int n_all = static_cast<int>(n_chunks) * E;
    const int split = static_cast<int>(c) * E;  // entries of the chunks before this one
    for (int i0 = threadIdx.x; i0 < n_all; i0 += 8 * kPThreads) {
      int32_t v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * kPThreads;
        v[u] = i < n_all ? __ldg(chunk_counts + i) : 0;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (v[u] != 0) {
          const int i = i0 + u * kPThreads;
          const int e = i % E;
          atomicAdd(&s_tot[e], v[u]);
          if (i < split) atomicAdd(&s_base[e], v[u]);
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    // exclusive scans over experts: lane l owns a contiguous run of experts
    const int lane = threadIdx.x;
    const int per = (E + 31) / 32;
    const int e0 = lane * per, e1 = min(E, e0 + per);
    int32_t sum = 0, tiles = 0;
    for (int e = e0; e < e1; ++e) {
      sum += s_tot[e];
      tiles += (s_tot[e] + kPTile - 1) / kPTile;
    }
    int32_t isum = sum, itil = tiles;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t a = __shfl_up_sync(0xffffffffu, isum, o);
      const int32_t b = __shfl_up_sync(0xffffffffu, itil, o);
      if (lane >= o) {
        isum += a;
        itil += b;
      }
    }
    int32_t run = isum - sum, trun = itil - tiles;
    for (int e = e0; e < e1; ++e) {
      s_off[e] = run;
      if (c == 0) {
        counts[e] = s_tot[e];
        offsets[e] = run;
        tile_offsets[e] = trun;
      }
      run += s_tot[e];
      trun += (s_tot[e] + kPTile - 1) / kPTile;
    }
    if (c == 0 && lane == 31) {
      offsets[E] = run;
      tile_offsets[E] = trun;
    }
  }
  // this chunk's token masks
  const int64_t t = t_lo + threadIdx.x;
  const bool mine = threadIdx.x < kPChunk && t < T;
  const int32_t *my_ids = s_ids + threadIdx.x * k;
  if (mine) {
    for (int j = 0; j < k; ++j) {
      const int e = my_ids[j];
      if (e < 0) continue;
      if (e >= E) {
        report_error(err, DEV_ERR_INDEX, 411, static_cast<int>(t), e);
        continue;
      }
      atomicOr(&mask[e][threadIdx.x >> 5], 1u << (threadIdx.x & 31));
    }
  }
  __syncthreads();
  if (mine) {
    // each thread overwrites only its own ids with their slot positions
    int32_t *my_pos = s_ids + threadIdx.x * k;
    const int w = threadIdx.x >> 5, b = threadIdx.x & 31;
    for (int j = 0; j < k; ++j) {
      const int e = my_pos[j];
      if (e < 0 || e >= E) {
        my_pos[j] = -1;
        continue;
      }
      int rank = 0;
      for (int qq = 0; qq < w; ++qq) rank += __popc(mask[e][qq]);
      rank += __popc(mask[e][w] & ((1u << b) - 1u));
      const int32_t pos = s_off[e] + s_base[e] + rank;
      sorted_tok[pos] = static_cast<int32_t>(t);
      my_pos[j] = pos;
    }
  }
  __syncthreads();
  int32_t *pos_g = slot_pos + t_lo * k;
  for (int i = threadIdx.x; i < n_ids; i += kPThreads) pos_g[i] = s_ids[i];
}

template <int E>
int launch_router_fused(const void *x, const void *w3, const float *bias, float *logits,
                        int32_t *idx, float *weights, int32_t *chunk_counts, int64_t T, int H,
                        int k, int renorm, int *err, cudaStream_t s) {
  using L = RouterLayout<E>;
  CUtensorMap tx, tw;
  int st = make_tmap_bf16_2d(&tx, x, H, T, static_cast<uint64_t>(H) * 2, kRBK, kRTok);
  if (st) return st;
  st = make_tmap_bf16_2d(&tw, w3, 3 * static_cast<uint64_t>(H), E,
                         3 * static_cast<uint64_t>(H) * 2, kRBK, E);
  if (st) return st;
  auto kern = router_logits_cluster_kernel<E>;
  st = ensure_smem_attr(reinterpret_cast<const void *>(kern), L::kBytes);
  if (st) return st;
  const int64_t chunks = (T + kRTok - 1) / kRTok;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(chunks * kRSplit), 1, 1);
  cfg.blockDim = dim3(kRThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kRSplit;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  Q35_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, tx, tw, bias, logits, chunk_counts, T, H, err));
  count_launch();
  topk_count_kernel<E / 32><<<static_cast<unsigned>((T + 7) / 8), 256, 0, s>>>(
      logits, idx, weights, chunk_counts, T, k, renorm);
  Q35_LAUNCH_CHECK("router topk_count launch");
  return Q35_OK;
}

}  // namespace
}  // namespace q35

using namespace q35;

extern "C" int q35_router_fused_supported(int64_t T, int H, int E, int k) {
  return (T >= 0 && H > 0 && H % (kRSplit * kRBK) == 0 && (E == 32 || E == 64 || E == 128) &&
          k >= 1 && k <= 16 && k <= E)
             ? 1
             : 0;
}

extern "C" int q35_router_topk_fused(const void *x, const void *w3, const float *bias,
                                     float *logits, int32_t *idx, float *weights,
                                     int32_t *chunk_counts, int64_t T, int H, int E, int k,
                                     int renorm, q35_stream_t stream) {
  if (!x || !w3 || !logits || !idx || !weights)
    return fail(Q35_ERR_INVALID, "router_fused: null pointer");
  if (!q35_router_fused_supported(T, H, E, k))
    return fail(Q35_ERR_UNSUPPORTED,
                "router_fused: H %d (multiple of 256), E %d (32, 64 or 128), k %d (1..16)", H, E,
                k);
  if (!aligned16(x) || !aligned16(w3)) return fail(Q35_ERR_ALIGN, "router_fused: alignment");
  if (T == 0) return Q35_OK;
  if (T > (int64_t(1) << 31) - kRTok) return fail(Q35_ERR_SHAPE, "router_fused: T too large");
  int *err = device_error_word();
  if (!err) return fail(Q35_ERR_CUDA, "router_fused: no device error word");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (E) {
    case 32:
      return launch_router_fused<32>(x, w3, bias, logits, idx, weights, chunk_counts, T, H, k,
                                     renorm, err, s);
    case 64:
      return launch_router_fused<64>(x, w3, bias, logits, idx, weights, chunk_counts, T, H, k,
                                     renorm, err, s);
    default:
      return launch_router_fused<128>(x, w3, bias, logits, idx, weights, chunk_counts, T, H, k,
                                      renorm, err, s);
  }
}

extern "C" int q35_moe_permute_counted(const int32_t *idx, int64_t T, int k, int E,
                                       const int32_t *chunk_counts, int32_t *counts,
                                       int32_t *offsets, int32_t *sorted_tok, int32_t *slot_pos,
                                       int32_t *tile_offsets, q35_stream_t stream) {
  if (!chunk_counts || !counts || !offsets || !tile_offsets ||
      (T > 0 && (!idx || !sorted_tok || !slot_pos)))
    return fail(Q35_ERR_INVALID, "moe_permute_counted: null pointer");
  if (T < 0 || k < 1 || k > 16 || E < 1 || E > 1024)
    return fail(Q35_ERR_SHAPE, "moe_permute_counted: T %lld k %d E %d (k <= 16, E <= 1024)",
                (long long)T, k, E);
  if (T * k >= (int64_t(1) << 31))
    return fail(Q35_ERR_SHAPE, "moe_permute_counted: T*k exceeds int32");
  int *err = device_error_word();
  if (!err) return fail(Q35_ERR_CUDA, "moe_permute_counted: no device error word");
  const int64_t chunks = (T + kPChunk - 1) / kPChunk;
  if (chunks * E >= (int64_t(1) << 31))
    return fail(Q35_ERR_SHAPE, "moe_permute_counted: chunk counts exceed int32");
  const size_t smem = static_cast<size_t>(E) * (3 * 4 + 16) + static_cast<size_t>(kPChunk) * k * 4;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // T == 0: one CTA over no rows writes zero counts and offsets
  permute_scan_scatter_kernel<<<static_cast<unsigned>(chunks > 0 ? chunks : 1), kPThreads, smem,
                                s>>>(idx, T, k, E, chunks, chunk_counts, counts, offsets,
                                     tile_offsets, sorted_tok, slot_pos, err);
  Q35_LAUNCH_CHECK("moe_permute_counted launch");
  return Q35_OK;
}
