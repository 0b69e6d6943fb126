// Token permutation for the grouped expert GEMM, the weighted combine, and the
// elementwise ops of the reference op layer.
//
// The reference never materialises a permutation: CudaSparseMoE.forward loops
// over experts in ascending order and, for each, takes mask.nonzero() of
// top_idx == e, which lists tokens in ascending order (REF
// cuda_qwen3_vl/modules/moe.py:71-76).  The canonical order here is therefore
// a stable sort of the T*k (token, slot) pairs by (expert, token).  It is built
// in three passes over 128-token chunks without any host synchronisation:
//   1. count:   per chunk, a 128-bit token mask per expert (shared-memory
//               atomicOr); chunk_counts[c][e] = popcount(mask[e]).
//   2. scan:    per expert, the running sum over chunks; counts, offsets
//               (exclusive scan over experts) and the GEMM M-tile schedule.
//   3. scatter: rank of token t within its chunk for expert e =
//               popcount(mask[e] & bits below t); pos = offsets[e] +
//               chunk_base[c][e] + rank.
// Every step is integer arithmetic, so the result is bit-exact.
#include <mutex>

#include "common.cuh"

namespace q35 {
namespace {

constexpr int kChunk = 128;  // tokens per chunk (one thread each)
constexpr int kTileM = 128;  // grouped-GEMM M tile

// Row t takes part when t < T and, for slab-structured input (slab_cnt !=
// nullptr: rows [s * slab_rows, s * slab_rows + slab_cnt[s]) of slab s are
// filled, the rest hold stale data), when it lies in the filled part of its
// slab.
__device__ __forceinline__ bool row_valid(int64_t t, int64_t T,
                                          const int32_t *__restrict__ slab_cnt,
                                          int64_t slab_rows) {
  if (t >= T) return false;
  if (slab_cnt == nullptr) return true;
  return (t % slab_rows) < static_cast<int64_t>(slab_cnt[t / slab_rows]);
}

__device__ __forceinline__ void build_masks(const int32_t *__restrict__ idx,
                                            int64_t T, int k, int E,
                                            uint32_t (*mask)[4], int *err,
                                            const int32_t *__restrict__ slab_cnt,
                                            int64_t slab_rows) {
  for (int i = threadIdx.x; i < E * 4; i += blockDim.x) mask[i >> 2][i & 3] = 0u;
  __syncthreads();
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kChunk + threadIdx.x;
  if (row_valid(t, T, slab_cnt, slab_rows)) {
    for (int j = 0; j < k; ++j) {
      const int e = idx[t * k + j];
      if (e < 0) continue;  // empty slot (expert-parallel receive side)
      if (e >= E) {
        report_error(err, DEV_ERR_INDEX, 101, static_cast<int>(t), e);
        continue;
      }
      atomicOr(&mask[e][threadIdx.x >> 5], 1u << (threadIdx.x & 31));
    }
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kChunk) permute_count_kernel(
    const int32_t *__restrict__ idx, int64_t T, int k, int E,
    int32_t *__restrict__ chunk_counts, int *err,
    const int32_t *__restrict__ slab_cnt, int64_t slab_rows) {
  extern __shared__ uint32_t smem_mask[];
  auto mask = reinterpret_cast<uint32_t(*)[4]>(smem_mask);
  build_masks(idx, T, k, E, mask, err, slab_cnt, slab_rows);
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    chunk_counts[static_cast<int64_t>(blockIdx.x) * E + e] =
        __popc(mask[e][0]) + __popc(mask[e][1]) + __popc(mask[e][2]) +
        __popc(mask[e][3]);
}

// Single CTA of 1024 threads; E <= 1024.
__global__ void __launch_bounds__(1024) permute_scan_kernel(
    int32_t *__restrict__ chunk_counts, int64_t n_chunks, int E,
    int32_t *__restrict__ counts, int32_t *__restrict__ offsets,
    int32_t *__restrict__ tile_offsets) {
  __shared__ int32_t s_cnt[1024], s_tiles[1024];
  const int e = threadIdx.x;
  int32_t run = 0;
  if (e < E) {
    // 16 chunk counts loaded at a time (independent loads), then rewritten
    // as each chunk's base within expert e
    for (int64_t c0 = 0; c0 < n_chunks; c0 += 16) {
      int32_t v[16];
#pragma unroll
      for (int i = 0; i < 16; ++i)
        v[i] = (c0 + i < n_chunks) ? chunk_counts[(c0 + i) * E + e] : 0;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        if (c0 + i < n_chunks) chunk_counts[(c0 + i) * E + e] = run;
        run += v[i];
      }
    }
    counts[e] = run;
  }
  s_cnt[e] = (e < E) ? run : 0;
  s_tiles[e] = (e < E) ? (run + kTileM - 1) / kTileM : 0;
  __syncthreads();
  // Inclusive Hillis-Steele scans over 1024 entries.
  for (int o = 1; o < 1024; o <<= 1) {
    const int32_t a = (e >= o) ? s_cnt[e - o] : 0;
    const int32_t b = (e >= o) ? s_tiles[e - o] : 0;
    __syncthreads();
    s_cnt[e] += a;
    s_tiles[e] += b;
    __syncthreads();
  }
  if (e < E) {
    offsets[e + 1] = s_cnt[e];
    tile_offsets[e + 1] = s_tiles[e];
  }
  if (e == 0) {
    offsets[0] = 0;
    tile_offsets[0] = 0;
  }
}

__global__ void __launch_bounds__(kChunk) permute_scatter_kernel(
    const int32_t *__restrict__ idx, int64_t T, int k, int E,
    const int32_t *__restrict__ chunk_base, const int32_t *__restrict__ offsets,
    int32_t *__restrict__ sorted_tok, int32_t *__restrict__ slot_pos,
    int *err, const int32_t *__restrict__ slab_cnt, int64_t slab_rows) {
  extern __shared__ uint32_t smem_mask[];
  auto mask = reinterpret_cast<uint32_t(*)[4]>(smem_mask);
  // errors are reported by the count pass
  build_masks(idx, T, k, E, mask, nullptr, slab_cnt, slab_rows);
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kChunk + threadIdx.x;
  if (!row_valid(t, T, slab_cnt, slab_rows)) return;
  const int w = threadIdx.x >> 5, b = threadIdx.x & 31;
  for (int j = 0; j < k; ++j) {
    const int e = idx[t * k + j];
    if (e < 0 || e >= E) {
      slot_pos[t * k + j] = -1;
      continue;
    }
    int rank = 0;
    for (int q = 0; q < w; ++q) rank += __popc(mask[e][q]);
    rank += __popc(mask[e][w] & ((1u << b) - 1u));
    const int32_t pos =
        offsets[e] + chunk_base[static_cast<int64_t>(blockIdx.x) * E + e] + rank;
    sorted_tok[pos] = static_cast<int32_t>(t);
    slot_pos[t * k + j] = pos;
  }
  (void)err;
}

// dst[r,:] = src[rows[r],:]; one warp per row, 16-byte vectors.
__global__ void __launch_bounds__(256) gather_rows_kernel(
    const uint16_t *__restrict__ src, const int32_t *__restrict__ rows,
    uint16_t *__restrict__ dst, int64_t n_max, const int32_t *__restrict__ n_dev,
    int64_t cols) {
  const int lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int64_t n = n_dev ? static_cast<int64_t>(*n_dev) : n_max;
  if (r >= n || r >= n_max) return;
  const int64_t s = rows[r];
  const uint4 *sp = reinterpret_cast<const uint4 *>(src + s * cols);
  uint4 *dp = reinterpret_cast<uint4 *>(dst + r * cols);
  for (int64_t c = lane; c < cols / 8; c += 32) dp[c] = sp[c];
}

// out[t,:] = residual[t,:] + sum_j w[t,j] * y[slot_pos[t*k+j],:]  (fp32 sum,
// slot order, one rounding).  One CTA per token, 8 columns per thread-step.
// KF > 0: k == KF known at compile time; the KF row loads of a column
// block are issued together before the (unchanged, slot-ordered) sum.
template <int KF>
__global__ void __launch_bounds__(256) combine_kernel(
    const uint16_t *__restrict__ y, const float *__restrict__ w,
    const int32_t *__restrict__ slot_pos, const void *__restrict__ residual,
    int residual_f32, uint16_t *__restrict__ out, int k_dyn, int64_t H) {
  const int k = KF > 0 ? KF : k_dyn;
  const int64_t t = blockIdx.x;
  __shared__ int32_t s_pos[16];
  __shared__ float s_w[16];
  if (threadIdx.x < k) {
    s_pos[threadIdx.x] = slot_pos[t * k + threadIdx.x];
    s_w[threadIdx.x] = w[t * k + threadIdx.x];
  }
  __syncthreads();
  for (int64_t c = static_cast<int64_t>(threadIdx.x) * 8; c < H;
       c += static_cast<int64_t>(blockDim.x) * 8) {
    float acc[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] = 0.f;
    if constexpr (KF > 0) {
      uint4 u[KF];
#pragma unroll
      for (int j = 0; j < KF; ++j) {
        const int32_t p = s_pos[j];
        u[j] = p >= 0 ? *reinterpret_cast<const uint4 *>(y + static_cast<int64_t>(p) * H + c)
                      : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int j = 0; j < KF; ++j) {
        if (s_pos[j] < 0) continue;
        float v[8];
        unpack_bf2(u[j].x, v[0], v[1]);
        unpack_bf2(u[j].y, v[2], v[3]);
        unpack_bf2(u[j].z, v[4], v[5]);
        unpack_bf2(u[j].w, v[6], v[7]);
        const float wj = s_w[j];
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] = fmaf(wj, v[q], acc[q]);
      }
    } else {
      for (int j = 0; j < k; ++j) {
        const int32_t p = s_pos[j];
        if (p < 0) continue;
        const uint4 u = *reinterpret_cast<const uint4 *>(y + static_cast<int64_t>(p) * H + c);
        float v[8];
        unpack_bf2(u.x, v[0], v[1]);
        unpack_bf2(u.y, v[2], v[3]);
        unpack_bf2(u.z, v[4], v[5]);
        unpack_bf2(u.w, v[6], v[7]);
        const float wj = s_w[j];
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] = fmaf(wj, v[q], acc[q]);
      }
    }
    if (residual) {
      float v[8];
      if (residual_f32) {
        const float *rp = static_cast<const float *>(residual) + t * H + c;
        const float4 a = *reinterpret_cast<const float4 *>(rp);
        const float4 b = *reinterpret_cast<const float4 *>(rp + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      } else {
        const uint4 u = *reinterpret_cast<const uint4 *>(
            static_cast<const uint16_t *>(residual) + t * H + c);
        unpack_bf2(u.x, v[0], v[1]);
        unpack_bf2(u.y, v[2], v[3]);
        unpack_bf2(u.z, v[4], v[5]);
        unpack_bf2(u.w, v[6], v[7]);
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = v[q] + acc[q];
    }
    uint4 o;
    o.x = pack_bf2(acc[0], acc[1]);
    o.y = pack_bf2(acc[2], acc[3]);
    o.z = pack_bf2(acc[4], acc[5]);
    o.w = pack_bf2(acc[6], acc[7]);
    *reinterpret_cast<uint4 *>(out + t * H + c) = o;
  }
}

__global__ void index_add_f32_kernel(float *__restrict__ target,
                                     const float *__restrict__ src,
                                     const int64_t *__restrict__ index,
                                     int64_t n_target, int64_t cols, int *err) {
  const int64_t r = blockIdx.x;
  const int64_t dst = index[r];
  if (dst < 0 || dst >= n_target) {
    if (threadIdx.x == 0)
      report_error(err, DEV_ERR_INDEX, 102, static_cast<int>(r), static_cast<int>(dst));
    return;
  }
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x)
    atomicAdd(target + dst * cols + c, src[r * cols + c]);
}

__global__ void index_add_bf16_kernel(__nv_bfloat16 *__restrict__ target,
                                      const __nv_bfloat16 *__restrict__ src,
                                      const int64_t *__restrict__ index,
                                      int64_t n_target, int64_t cols, int *err) {
  const int64_t r = blockIdx.x;
  const int64_t dst = index[r];
  if (dst < 0 || dst >= n_target) {
    if (threadIdx.x == 0)
      report_error(err, DEV_ERR_INDEX, 103, static_cast<int>(r), static_cast<int>(dst));
    return;
  }
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x)
    atomicAdd(target + dst * cols + c, src[r * cols + c]);
}

__global__ void swiglu_kernel(const uint16_t *__restrict__ g,
                              const uint16_t *__restrict__ u,
                              uint16_t *__restrict__ o, int64_t n) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float gv = bf2f(g[i]);
  o[i] = f2bf(gv / (1.0f + expf(-gv)) * bf2f(u[i]));
}

__global__ void residual_add_kernel(const uint16_t *__restrict__ a,
                                    const uint16_t *__restrict__ b,
                                    uint16_t *__restrict__ o, int64_t n) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  o[i] = f2bf(bf2f(a[i]) + bf2f(b[i]));
}

}  // namespace
}  // namespace q35

using namespace q35;

extern "C" int64_t q35_moe_permute_workspace(int64_t T, int E) {
  const int64_t chunks = (T + kChunk - 1) / kChunk;
  return chunks * static_cast<int64_t>(E > 0 ? E : 1);
}

namespace {
int permute_impl(const int32_t *idx, int64_t T, int k, int E, int32_t *counts,
                 int32_t *offsets, int32_t *sorted_tok, int32_t *slot_pos,
                 int32_t *tile_offsets, int32_t *workspace,
                 const int32_t *slab_cnt, int64_t slab_rows,
                 q35_stream_t stream) {
  if (!counts || !offsets || !tile_offsets || !workspace ||
      (T > 0 && (!idx || !sorted_tok || !slot_pos)))
    return fail(Q35_ERR_INVALID, "moe_permute: null pointer");
  if (T < 0 || k < 1 || E < 1 || E > 1024)
    return fail(Q35_ERR_SHAPE, "moe_permute: T %lld k %d E %d (E <= 1024)",
                (long long)T, k, E);
  if (T * k >= (int64_t(1) << 31))
    return fail(Q35_ERR_SHAPE, "moe_permute: T*k exceeds int32");
  int *err = device_error_word();
  if (!err) return fail(Q35_ERR_CUDA, "moe_permute: no device error word");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t chunks = (T + kChunk - 1) / kChunk;
  const size_t smem = static_cast<size_t>(E) * 4 * sizeof(uint32_t);
  if (chunks > 0) {
    permute_count_kernel<<<static_cast<unsigned>(chunks), kChunk, smem, s>>>(
        idx, T, k, E, workspace, err, slab_cnt, slab_rows);
    Q35_LAUNCH_CHECK("permute count launch");
  }
  permute_scan_kernel<<<1, 1024, 0, s>>>(workspace, chunks, E, counts, offsets,
                                         tile_offsets);
  Q35_LAUNCH_CHECK("permute scan launch");
  if (chunks > 0) {
    permute_scatter_kernel<<<static_cast<unsigned>(chunks), kChunk, smem, s>>>(
        idx, T, k, E, workspace, offsets, sorted_tok, slot_pos, err, slab_cnt,
        slab_rows);
    Q35_LAUNCH_CHECK("permute scatter launch");
  }
  return Q35_OK;
}
}  // namespace

extern "C" int q35_moe_permute(const int32_t *idx, int64_t T, int k, int E,
                               int32_t *counts, int32_t *offsets,
                               int32_t *sorted_tok, int32_t *slot_pos,
                               int32_t *tile_offsets, int32_t *workspace,
                               q35_stream_t stream) {
  return permute_impl(idx, T, k, E, counts, offsets, sorted_tok, slot_pos,
                      tile_offsets, workspace, nullptr, 0, stream);
}

extern "C" int q35_moe_permute_slabs(const int32_t *idx, int n_slabs,
                                     int64_t slab_rows, const int32_t *slab_cnt,
                                     int k, int E, int32_t *counts,
                                     int32_t *offsets, int32_t *sorted_tok,
                                     int32_t *slot_pos, int32_t *tile_offsets,
                                     int32_t *workspace, q35_stream_t stream) {
  if (!slab_cnt) return fail(Q35_ERR_INVALID, "moe_permute_slabs: null slab counts");
  if (n_slabs < 1 || slab_rows < 1)
    return fail(Q35_ERR_SHAPE, "moe_permute_slabs: %d slabs of %lld rows", n_slabs,
                (long long)slab_rows);
  return permute_impl(idx, n_slabs * slab_rows, k, E, counts, offsets, sorted_tok,
                      slot_pos, tile_offsets, workspace, slab_cnt, slab_rows, stream);
}

namespace q35 {
namespace {
// out[r,:] = table[ids[r],:]; one warp per row, 16-byte vectors; an id outside
// [0, V) writes a zero row and reports DEV_ERR_INDEX (site 104).
__global__ void __launch_bounds__(256) embedding_kernel(const uint16_t *__restrict__ table,
                                                        const int64_t *__restrict__ ids,
                                                        uint16_t *__restrict__ out, int64_t n,
                                                        int64_t V, int64_t cols, int *err) {
  const int lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (r >= n) return;
  const int64_t id = ids[r];
  uint4 *dp = reinterpret_cast<uint4 *>(out + r * cols);
  if (id < 0 || id >= V) {
    if (lane == 0) report_error(err, DEV_ERR_INDEX, 104, static_cast<int>(r), static_cast<int>(id));
    for (int64_t c = lane; c < cols / 8; c += 32) dp[c] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4 *sp = reinterpret_cast<const uint4 *>(table + id * cols);
  for (int64_t c = lane; c < cols / 8; c += 32) dp[c] = sp[c];
}
}  // namespace
}  // namespace q35

extern "C" int q35_embedding_fwd(const void *table, const int64_t *ids, void *out, int64_t n,
                                 int64_t V, int64_t cols, q35_stream_t stream) {
  if (!table || !out || (n > 0 && !ids)) return fail(Q35_ERR_INVALID, "embedding: null pointer");
  if (n < 0 || V < 1 || cols <= 0 || cols % 8 != 0)
    return fail(Q35_ERR_SHAPE, "embedding: n %lld V %lld cols %lld (x8)", (long long)n,
                (long long)V, (long long)cols);
  if (!aligned16(table) || !aligned16(out)) return fail(Q35_ERR_ALIGN, "embedding: alignment");
  if ((n + 7) / 8 >= (int64_t(1) << 31)) return fail(Q35_ERR_SHAPE, "embedding: too many ids");
  if (n == 0) return Q35_OK;
  int *err = device_error_word();
  if (!err) return fail(Q35_ERR_CUDA, "embedding: no device error word");
  embedding_kernel<<<static_cast<unsigned>((n + 7) / 8), 256, 0,
                     reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t *>(table), ids, static_cast<uint16_t *>(out), n, V, cols, err);
  Q35_LAUNCH_CHECK("embedding launch");
  return Q35_OK;
}

extern "C" int q35_gather_rows(const void *src, const int32_t *rows, void *dst,
                               int64_t n_max, const int32_t *n_dev,
                               int64_t cols, q35_stream_t stream) {
  if (!src || !rows || !dst) return fail(Q35_ERR_INVALID, "gather_rows: null");
  if (n_max < 0 || cols <= 0 || cols % 8 != 0)
    return fail(Q35_ERR_SHAPE, "gather_rows: cols %lld must be a multiple of 8",
                (long long)cols);
  if (!aligned16(src) || !aligned16(dst))
    return fail(Q35_ERR_ALIGN, "gather_rows: pointers not 16-byte aligned");
  if (n_max == 0) return Q35_OK;
  gather_rows_kernel<<<static_cast<unsigned>((n_max + 7) / 8), 256, 0,
                       reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t *>(src), rows, static_cast<uint16_t *>(dst),
      n_max, n_dev, cols);
  Q35_LAUNCH_CHECK("gather_rows launch");
  return Q35_OK;
}

extern "C" int q35_moe_combine(const void *y, const float *weights,
                               const int32_t *slot_pos, const void *residual,
                               int residual_f32, void *out, int64_t T, int k,
                               int64_t H, q35_stream_t stream) {
  if (!out || (T > 0 && (!y || !weights || !slot_pos)))
    return fail(Q35_ERR_INVALID, "moe_combine: null pointer");
  if (T < 0 || k < 1 || k > 16 || H <= 0 || H % 8 != 0)
    return fail(Q35_ERR_SHAPE, "moe_combine: k %d (<=16) H %lld (x8)", k,
                (long long)H);
  if (!aligned16(y) || !aligned16(out) || (residual && !aligned16(residual)))
    return fail(Q35_ERR_ALIGN, "moe_combine: pointers not 16-byte aligned");
  if (T == 0) return Q35_OK;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  if (k == 8)
    combine_kernel<8><<<static_cast<unsigned>(T), 256, 0, cs>>>(
        static_cast<const uint16_t *>(y), weights, slot_pos, residual, residual_f32,
        static_cast<uint16_t *>(out), k, H);
  else
    combine_kernel<0><<<static_cast<unsigned>(T), 256, 0, cs>>>(
        static_cast<const uint16_t *>(y), weights, slot_pos, residual, residual_f32,
        static_cast<uint16_t *>(out), k, H);
  Q35_LAUNCH_CHECK("moe_combine launch");
  return Q35_OK;
}

extern "C" int q35_index_add(void *target, const void *source,
                             const int64_t *index, int64_t n_src,
                             int64_t n_target, int64_t cols, int dtype,
                             q35_stream_t stream) {
  if (!target || (n_src > 0 && (!source || !index)))
    return fail(Q35_ERR_INVALID, "index_add: null pointer");
  if (n_src < 0 || cols <= 0) return fail(Q35_ERR_SHAPE, "index_add: bad shape");
  if (n_src == 0) return Q35_OK;
  int *err = device_error_word();
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const unsigned threads = cols >= 256 ? 256 : static_cast<unsigned>(((cols + 31) / 32) * 32);
  if (dtype == 0)
    index_add_f32_kernel<<<static_cast<unsigned>(n_src), threads, 0, s>>>(
        static_cast<float *>(target), static_cast<const float *>(source), index,
        n_target, cols, err);
  else if (dtype == 1)
    index_add_bf16_kernel<<<static_cast<unsigned>(n_src), threads, 0, s>>>(
        static_cast<__nv_bfloat16 *>(target),
        static_cast<const __nv_bfloat16 *>(source), index, n_target, cols, err);
  else
    return fail(Q35_ERR_UNSUPPORTED, "index_add: dtype code %d", dtype);
  Q35_LAUNCH_CHECK("index_add launch");
  return Q35_OK;
}

extern "C" int q35_swiglu_fwd(const void *gate, const void *up, void *out,
                              int64_t n, q35_stream_t stream) {
  if (!gate || !up || !out) return fail(Q35_ERR_INVALID, "swiglu: null pointer");
  if (n <= 0) return n == 0 ? Q35_OK : fail(Q35_ERR_SHAPE, "swiglu: n < 0");
  swiglu_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0,
                  reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t *>(gate), static_cast<const uint16_t *>(up),
      static_cast<uint16_t *>(out), n);
  Q35_LAUNCH_CHECK("swiglu launch");
  return Q35_OK;
}

extern "C" int q35_residual_add_fwd(const void *a, const void *b, void *out,
                                    int64_t n, q35_stream_t stream) {
  if (!a || !b || !out) return fail(Q35_ERR_INVALID, "residual_add: null pointer");
  if (n <= 0) return n == 0 ? Q35_OK : fail(Q35_ERR_SHAPE, "residual_add: n < 0");
  residual_add_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0,
                        reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t *>(a), static_cast<const uint16_t *>(b),
      static_cast<uint16_t *>(out), n);
  Q35_LAUNCH_CHECK("residual_add launch");
  return Q35_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free variant of q35_moe_permute.
//
// Some callers cannot allocate device memory at the point where they route
// tokens: code running inside a pre-sized memory pool that must not grow,
// engines that forbid cudaMalloc on their serving path, or a host that only
// hands out input and output buffers.  For them the per-chunk count scratch
// that q35_moe_permute takes as `workspace` lives in the fixed array below.
// The array is loaded with the library, so every GPU that loads it holds
// 256 KiB until the process exits.
namespace {
constexpr int64_t kNoAllocScratchInts = 65536;  // 256 KiB of int32
static __device__ __align__(256) int32_t g_permute_scratch[kNoAllocScratchInts];

std::mutex g_scratch_mu;
int32_t *g_scratch_ptr[64] = {};

// Device address of g_permute_scratch on the current device, looked up once
// per device.  The symbol's name in host code is only a host-side handle,
// never a device pointer, so kernels get the address from here.
int scratch_address(int32_t **out) {
  int dev = 0;
  Q35_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64)
    return fail(Q35_ERR_NO_DEVICE, "moe_permute_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_permute_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_permute_scratch)");
    g_scratch_ptr[dev] = static_cast<int32_t *>(p);
  }
  *out = g_scratch_ptr[dev];
  return Q35_OK;
}
}  // namespace

extern "C" int64_t q35_moe_permute_noalloc_max_workspace(void) {
  return kNoAllocScratchInts;
}

extern "C" int q35_moe_permute_noalloc(const int32_t *idx, int64_t T, int k,
                                       int E, int32_t *counts,
                                       int32_t *offsets, int32_t *sorted_tok,
                                       int32_t *slot_pos,
                                       int32_t *tile_offsets,
                                       q35_stream_t stream) {
  if (!counts || !offsets || !tile_offsets ||
      (T > 0 && (!idx || !sorted_tok || !slot_pos)))
    return fail(Q35_ERR_INVALID, "moe_permute_noalloc: null pointer");
  if (T < 0 || k < 1 || E < 1 || E > 1024)
    return fail(Q35_ERR_SHAPE, "moe_permute_noalloc: T %lld k %d E %d (E <= 1024)",
                (long long)T, k, E);
  if (T * k >= (int64_t(1) << 31))
    return fail(Q35_ERR_SHAPE, "moe_permute_noalloc: T*k exceeds int32");
  const int64_t need = q35_moe_permute_workspace(T, E);
  if (need > kNoAllocScratchInts)
    return fail(Q35_ERR_SHAPE,
                "moe_permute_noalloc: needs %lld scratch ints (ceil(T/128)*E), the "
                "built-in maximum is %lld; use q35_moe_permute with a caller workspace",
                (long long)need, (long long)kNoAllocScratchInts);
  int32_t *scratch = nullptr;
  const int st = scratch_address(&scratch);
  if (st) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t chunks = (T + kChunk - 1) / kChunk;
  const size_t smem = static_cast<size_t>(E) * 4 * sizeof(uint32_t);
  // The count pass writes every scratch entry the scan and scatter read, so
  // nothing left over from a previous call is ever used.  Expert ids outside
  // [0, E) are dropped (slot_pos = -1) without a device error-word report:
  // that word is allocated on first use, which this entry point must not do.
  if (chunks > 0) {
    permute_count_kernel<<<static_cast<unsigned>(chunks), kChunk, smem, s>>>(
        idx, T, k, E, scratch, nullptr, nullptr, 0);
    Q35_LAUNCH_CHECK("permute_noalloc count launch");
  }
  permute_scan_kernel<<<1, 1024, 0, s>>>(scratch, chunks, E, counts, offsets,
                                         tile_offsets);
  Q35_LAUNCH_CHECK("permute_noalloc scan launch");
  if (chunks > 0) {
    permute_scatter_kernel<<<static_cast<unsigned>(chunks), kChunk, smem, s>>>(
        idx, T, k, E, scratch, offsets, sorted_tok, slot_pos, nullptr, nullptr, 0);
    Q35_LAUNCH_CHECK("permute_noalloc scatter launch");
  }
  return Q35_OK;
}

// ---------------------------------------------------------------------------
// Expert-parallel send slabs.  Each token sends at most one row to each rank
// (the rank that owns one or more of its top-k experts), so a fixed slab of
// T rows per destination holds every possible send: row (d, t) of the send
// buffer is token t's hidden row if token t uses an expert of rank d.  Its
// slot list meta_idx[(d, t), j] is the slot's expert id local to rank d, or -1
// for slots of other ranks (and for every slot of an unused row); meta_w the
// routing weights.  ret_pos[t, d] = d*T + t if token t uses rank d, else -1:
// where rank d's partial sum for token t comes back.  One CTA per token.
namespace q35 {
namespace {
__global__ void __launch_bounds__(256) ep_scatter_kernel(
    const uint16_t *__restrict__ x, const int32_t *__restrict__ idx, const float *__restrict__ w,
    int64_t T, int k, int64_t H, int El, int N, uint16_t *__restrict__ send,
    int32_t *__restrict__ meta_idx, float *__restrict__ meta_w, int64_t meta_slab,
    int32_t *__restrict__ ret_pos) {
  const int64_t t = blockIdx.x;
  __shared__ int s_e[16];
  __shared__ uint32_t s_used;  // bit d: token t sends to rank d (N <= 32)
  if (threadIdx.x == 0) s_used = 0;
  __syncthreads();
  if (threadIdx.x < k) {
    const int e = idx[t * k + threadIdx.x];
    s_e[threadIdx.x] = e;
    if (e >= 0 && e / El < N) atomicOr(&s_used, 1u << (e / El));
  }
  __syncthreads();
  const uint32_t used = s_used;
  // slot lists and return positions
  for (int i = threadIdx.x; i < N * k; i += blockDim.x) {
    const int d = i / k, j = i % k;
    const int e = s_e[j];
    const int64_t m = static_cast<int64_t>(d) * meta_slab + t * k + j;
    const bool mine = e >= 0 && e / El == d;
    meta_idx[m] = mine ? e - d * El : -1;
    meta_w[m] = mine ? w[t * k + j] : 0.f;
  }
  for (int d = threadIdx.x; d < N; d += blockDim.x)
    ret_pos[t * N + d] = ((used >> d) & 1u) ? static_cast<int32_t>(d * T + t) : -1;
  // token row into each used slab
  const uint4 *src = reinterpret_cast<const uint4 *>(x + t * H);
  for (int d = 0; d < N; ++d) {
    if (!((used >> d) & 1u)) continue;
    uint4 *dst = reinterpret_cast<uint4 *>(send + (static_cast<int64_t>(d) * T + t) * H);
    for (int64_t c = threadIdx.x; c < H / 8; c += blockDim.x) dst[c] = src[c];
  }
}
}  // namespace
}  // namespace q35

extern "C" int q35_ep_scatter(const void *x, const int32_t *idx, const float *w, int64_t T,
                              int k, int64_t H, int El, int N, void *send, int32_t *meta_idx,
                              float *meta_w, int64_t meta_slab, int32_t *ret_pos,
                              q35_stream_t stream) {
  if (!send || !meta_idx || !meta_w || !ret_pos || (T > 0 && (!x || !idx || !w)))
    return fail(Q35_ERR_INVALID, "ep_scatter: null pointer");
  if (T < 0 || k < 1 || k > 16 || El < 1 || N < 1 || N > 32 || H <= 0 || H % 8 != 0)
    return fail(Q35_ERR_SHAPE, "ep_scatter: k %d (<=16) N %d (<=32) H %lld (x8)", k, N,
                (long long)H);
  if (!aligned16(x) || !aligned16(send)) return fail(Q35_ERR_ALIGN, "ep_scatter: alignment");
  if (meta_slab < T * k) return fail(Q35_ERR_SHAPE, "ep_scatter: meta_slab < T*k");
  if (T == 0) return Q35_OK;
  ep_scatter_kernel<<<static_cast<unsigned>(T), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t *>(x), idx, w, T, k, H, El, N, static_cast<uint16_t *>(send),
      meta_idx, meta_w, meta_slab, ret_pos);
  Q35_LAUNCH_CHECK("ep_scatter launch");
  return Q35_OK;
}
