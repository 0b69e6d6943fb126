// Expert-parallel token exchange over peer memory (NVLink / NVSwitch).
//
// Rank r of an N-rank group owns experts [r*El, (r+1)*El).  Every rank holds
// one "exchange window" in its own device memory; the windows of all ranks
// are mapped into every rank's address space (CUDA IPC), so the kernels below
// store straight into a peer's window with ordinary st.global instructions
// that travel over NVLink.  No collective library is involved and only the
// rows a token actually needs cross the link.
//
// Window layout (the same offsets on every rank, see window_layout()):
//   rows  [N][Tcap][H] bf16   slab s: token rows sent by rank s (compacted)
//   ret   [N][Tcap][H] bf16   ret[d][t]: owner d's partial sum for my token t
//   idx   [N][Tcap][k] int32  slot lists of the received rows (local expert
//                             id of this rank, -1 for another rank's expert)
//   wts   [N][Tcap][k] fp32   routing weights of those slots
//   tok   [N][Tcap]    int32  the sender's token index of each received row
//   cnt   [N]          int32  rows received from each rank in this call
//   flags [2][N]       u32    per source: epoch of its last dispatch / return
//   ctrl               u32    epoch, two CTA-completion counters, N send
//                             counters (local use only)
//   peers [N]          u64    base address of every rank's window, as mapped
//                             in this process (written once by the host)
//
// One call (one MoE layer forward):
//   1. ep_dispatch_kernel: per CTA of 32 tokens, each token's owner ranks
//      and its rank among the CTA's rows for each of them (shared-memory
//      counters), one global atomicAdd per destination to reserve the CTA's
//      block of that rank's slab, then the hidden rows, slot lists, weights
//      and token indices stored into the peers' windows.  The last CTA
//      to finish publishes the row counts and then the new epoch to every
//      peer (release at system scope, after a system-scope fence).
//   2. ep_wait_kernel: waits (bounded) until every source's dispatch flag has
//      reached this rank's epoch.  The ordinary permutation, gather and
//      grouped-GEMM kernels then run on the received slabs.
//   3. ep_return_kernel: one warp per received row sums its slots' expert
//      outputs (fp32, slot order, weights applied), rounds to bf16 once and
//      stores the partial into the sender's ret[r][token]; the last CTA
//      publishes the return flag to every peer.
//   4. ep_wait_kernel on the return flags, then the combine kernel adds each
//      token's partials (rank order) to its residual.
//
// Reuse safety without extra handshakes: rank r writes slab r of peer d only
// in its own dispatch, which runs after its previous call's return wait; that
// wait completed only after d had returned (so finished reading) everything r
// sent in the previous call.  ret[d][*] of rank r is written by d only after
// d received r's next dispatch, which r issues after its combine consumed the
// previous returns.  Every wait is bounded (default 5 s): on expiry the kernel
// records DEV_ERR_WAIT_TIMEOUT in the device error word and returns, so a
// missing rank ends in an error, never a hang.
//
// The order of rows inside a slab depends on the atomics' order, but no
// result does: a received row's partial depends only on that row, and it is
// returned to its token's fixed position.  The reference runs every expert on
// one GPU (REF cuda_qwen3_vl/modules/moe.py:71-83) and has no counterpart.
#include <string.h>

#include "common.cuh"

namespace q35 {
namespace {

constexpr int kMaxRanks = 32;

struct Layout {
  int64_t rows, ret, idx, wts, tok, cnt, flags, ctrl, peers, total;
};

inline int64_t align256(int64_t v) { return (v + 255) & ~int64_t(255); }

Layout window_layout(int N, int64_t Tcap, int64_t H, int k) {
  Layout L;
  int64_t o = 0;
  L.rows = o;  o = align256(o + int64_t(N) * Tcap * H * 2);
  L.ret = o;   o = align256(o + int64_t(N) * Tcap * H * 2);
  L.idx = o;   o = align256(o + int64_t(N) * Tcap * k * 4);
  L.wts = o;   o = align256(o + int64_t(N) * Tcap * k * 4);
  L.tok = o;   o = align256(o + int64_t(N) * Tcap * 4);
  L.cnt = o;   o = align256(o + int64_t(N) * 4);
  L.flags = o; o = align256(o + int64_t(2) * N * 4);
  L.ctrl = o;  o = align256(o + (3 + int64_t(N)) * 4);
  L.peers = o; o = align256(o + int64_t(N) * 8);
  L.total = o;
  return L;
}

// ctrl words
constexpr int kCtrlEpoch = 0, kCtrlDoneDispatch = 1, kCtrlDoneReturn = 2, kCtrlSend = 3;

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct DevLayout {  // passed by value to the kernels
  int64_t rows, ret, idx, wts, tok, cnt, flags;
};

__device__ __forceinline__ uint8_t *peer_base(const uint64_t *peers, int d) {
  return reinterpret_cast<uint8_t *>(peers[d]);
}

// Called by every CTA once its stores are issued: the last CTA to arrive
// publishes (cnt if `publish_counts`) and the flag `which` (0 dispatch, 1
// return) to every rank, then resets the completion counter.
__device__ void publish_when_last(uint32_t *ctrl, int done_word, bool bump_epoch,
                                  const uint64_t *peers, DevLayout L, int N, int rank,
                                  int which, bool publish_counts) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x != 0) return;
  const uint32_t prev = atomicAdd(&ctrl[done_word], 1u);
  if (prev != gridDim.x - 1) return;
  __threadfence_system();
  uint32_t epoch = ctrl[kCtrlEpoch];
  if (bump_epoch) {
    epoch += 1u;
    ctrl[kCtrlEpoch] = epoch;
  }
  if (publish_counts) {
    for (int d = 0; d < N; ++d) {
      int32_t *cnt = reinterpret_cast<int32_t *>(peer_base(peers, d) + L.cnt);
      volatile int32_t *vc = cnt + rank;
      *vc = static_cast<int32_t>(atomicExch(&ctrl[kCtrlSend + d], 0u));
    }
    __threadfence_system();
  }
  for (int d = 0; d < N; ++d) {
    uint32_t *fl = reinterpret_cast<uint32_t *>(peer_base(peers, d) + L.flags);
    st_release_sys(fl + which * N + rank, epoch);
  }
  ctrl[done_word] = 0u;
}

// dispatch: tokens per CTA.  32 (four per warp) normally; a rank with so few
// tokens that this would leave most SMs idle (fewer CTAs than half the SMs)
// takes one token per warp, spreading its NVLink stores over more SMs.

// Copies one row of H bf16 (H % 8 == 0) with the warp: up to 8 16-byte loads
// per lane issued before their stores.
__device__ __forceinline__ void warp_copy_row(uint4 *__restrict__ dst, const uint4 *__restrict__ src,
                                              int64_t n16, int lane) {
  for (int64_t c0 = 0; c0 < n16; c0 += 256) {
    uint4 v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t c = c0 + lane + 32 * i;
      if (c < n16) v[i] = src[c];
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t c = c0 + lane + 32 * i;
      if (c < n16) dst[c] = v[i];
    }
  }
}

// CTA = TPC consecutive tokens (TPC / 8 per warp).  Pass 1 finds each
// token's owner ranks and its rank among this CTA's rows for each destination
// (shared-memory counters); one global atomicAdd per destination then reserves
// the CTA's block of rows in that destination's slab; pass 2 stores the rows.
// x [T, H] bf16, idx/w [T, k]; ret_pos [T, N]: d*Tcap + t where rank d returns
// token t's partial, else -1.
template <int TPC>
__global__ void __launch_bounds__(256) ep_dispatch_kernel(
    const uint16_t *__restrict__ x, const int32_t *__restrict__ idx,
    const float *__restrict__ w, int64_t T, int k, int64_t H, int El, int N, int rank,
    int64_t Tcap, uint32_t *__restrict__ ctrl, const uint64_t *__restrict__ peers,
    DevLayout L, int32_t *__restrict__ ret_pos, const int32_t *__restrict__ owner, int *err) {
  __shared__ uint32_t s_used[TPC];
  __shared__ int32_t s_rank[TPC][kMaxRanks];
  __shared__ uint32_t s_cnt[kMaxRanks];
  __shared__ int32_t s_base[kMaxRanks];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * TPC;
  if (threadIdx.x < kMaxRanks) s_cnt[threadIdx.x] = 0u;
  __syncthreads();
  // ---- pass 1: owner ranks and local ranks
  for (int i = 0; i < TPC / 8; ++i) {
    const int tl = warp * (TPC / 8) + i;
    const int64_t t = t0 + tl;
    uint32_t used = 0u;
    if (t < T) {
      int dst = -1;
      if (lane < k) {
        const int e = idx[t * k + lane];
        if (e >= N * El) {
          report_error(err, DEV_ERR_INDEX, 301, static_cast<int>(t), e);
        } else if (e >= 0) {
          dst = owner ? (owner[e] >> 16) : e / El;
        }
      }
      used = __reduce_or_sync(0xffffffffu, dst >= 0 ? (1u << dst) : 0u);
      if (lane < N) {
        ret_pos[t * N + lane] = ((used >> lane) & 1u) ? static_cast<int32_t>(lane * Tcap + t) : -1;
        if ((used >> lane) & 1u) s_rank[tl][lane] = static_cast<int32_t>(atomicAdd(&s_cnt[lane], 1u));
      }
    }
    if (lane == 0) s_used[tl] = used;
  }
  __syncthreads();
  if (threadIdx.x < N && s_cnt[threadIdx.x] > 0u)
    s_base[threadIdx.x] = static_cast<int32_t>(atomicAdd(&ctrl[kCtrlSend + threadIdx.x], s_cnt[threadIdx.x]));
  __syncthreads();
  // ---- pass 2: rows, slot lists, weights and token ids into the owners' windows
  for (int i = 0; i < TPC / 8; ++i) {
    const int tl = warp * (TPC / 8) + i;
    const int64_t t = t0 + tl;
    if (t >= T) break;
    int e = -1;
    float wt = 0.f;
    if (lane < k) {
      e = idx[t * k + lane];
      wt = w[t * k + lane];
    }
    const uint4 *src = reinterpret_cast<const uint4 *>(x + t * H);
    for (uint32_t m = s_used[tl]; m != 0u; m &= m - 1u) {
      const int d = __ffs(m) - 1;
      const int64_t p = static_cast<int64_t>(s_base[d]) + s_rank[tl][d];
      if (p >= Tcap) {  // cannot happen: at most one row per token and rank
        if (lane == 0) report_error(err, DEV_ERR_INDEX, 302, static_cast<int>(t), static_cast<int>(p));
        continue;
      }
      uint8_t *base = peer_base(peers, d);
      const int64_t row = static_cast<int64_t>(rank) * Tcap + p;
      warp_copy_row(reinterpret_cast<uint4 *>(base + L.rows) + row * (H / 8), src, H / 8, lane);
      if (lane < k) {
        int dst_e = -1, local = -1;
        if (e >= 0 && e < N * El) {
          dst_e = owner ? (owner[e] >> 16) : e / El;
          local = owner ? (owner[e] & 0xffff) : e - dst_e * El;
        }
        const bool mine = dst_e == d;
        reinterpret_cast<int32_t *>(base + L.idx)[row * k + lane] = mine ? local : -1;
        reinterpret_cast<float *>(base + L.wts)[row * k + lane] = mine ? wt : 0.f;
      }
      if (lane == 0) reinterpret_cast<int32_t *>(base + L.tok)[row] = static_cast<int32_t>(t);
    }
  }
  publish_when_last(ctrl, kCtrlDoneDispatch, true, peers, L, N, rank, 0, true);
}

// Waits until flags[which][s] >= epoch for every source s (lane s).
__global__ void ep_wait_kernel(const uint8_t *__restrict__ window, DevLayout L,
                               const uint32_t *__restrict__ ctrl, int N, int which,
                               uint64_t limit_ns, int *err) {
  const int s = threadIdx.x;
  if (s >= N) return;
  const uint32_t *fl = reinterpret_cast<const uint32_t *>(window + L.flags) + which * N + s;
  const uint32_t epoch = ctrl[kCtrlEpoch];
  const uint64_t t0 = global_timer_ns();
  uint32_t it = 0;
  while (static_cast<int32_t>(ld_acquire_sys(fl) - epoch) < 0) {
    if ((++it & 63u) == 0 && global_timer_ns() - t0 > limit_ns) {
      report_error(err, DEV_ERR_WAIT_TIMEOUT, 310 + which, s, static_cast<int>(epoch));
      return;
    }
    __nanosleep(64);
  }
}

// One warp per received row (s, p), p < cnt[s]: partial = sum over the row's
// slots j with a local expert of w[j] * y[slot_pos[row*k + j]] (fp32, slot
// order, one bf16 rounding), stored into rank s's ret[rank][tok].
__global__ void __launch_bounds__(256) ep_return_kernel(
    const uint16_t *__restrict__ y, const int32_t *__restrict__ slot_pos,
    const uint8_t *__restrict__ window, int64_t Tcap, int k, int64_t H, int N, int rank,
    uint32_t *__restrict__ ctrl, const uint64_t *__restrict__ peers, DevLayout L) {
  const int lane = threadIdx.x & 31;
  const int32_t *cnt = reinterpret_cast<const int32_t *>(window + L.cnt);
  const int32_t *tok = reinterpret_cast<const int32_t *>(window + L.tok);
  const float *wts = reinterpret_cast<const float *>(window + L.wts);
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t R = static_cast<int64_t>(N) * Tcap;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       r < R; r += warps) {
    const int s = static_cast<int>(r / Tcap);
    const int64_t p = r - static_cast<int64_t>(s) * Tcap;
    if (p >= cnt[s]) {  // rows of a slab are contiguous: skip to the next slab
      continue;
    }
    int32_t sp = -1;
    float wj = 0.f;
    if (lane < k) {
      sp = slot_pos[r * k + lane];
      wj = wts[r * k + lane];
    }
    const int32_t t = tok[r];
    uint4 *dst = reinterpret_cast<uint4 *>(peer_base(peers, s) + L.ret) +
                 (static_cast<int64_t>(rank) * Tcap + t) * (H / 8);
    // the row's slots that hold an expert of this rank, compacted in slot
    // order into registers of every lane (at most 8 are kept in registers;
    // rows with more are summed by the general loop below)
    int32_t pv[8];
    float wv8[8];
    int nv = 0;
    bool spill = false;
    for (int j = 0; j < k; ++j) {
      const int32_t pj = __shfl_sync(0xffffffffu, sp, j);
      const float wjj = __shfl_sync(0xffffffffu, wj, j);
      if (pj < 0) continue;
      if (nv < 8) {
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (q == nv) {
            pv[q] = pj;
            wv8[q] = wjj;
          }
        ++nv;
      } else {
        spill = true;
      }
    }
    for (int64_t c = lane; c < H / 8; c += 32) {
      float acc[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = 0.f;
      if (!spill) {
        uint4 u[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (j < nv) u[j] = reinterpret_cast<const uint4 *>(y + static_cast<int64_t>(pv[j]) * H)[c];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (j >= nv) continue;
          float v[8];
          unpack_bf2(u[j].x, v[0], v[1]);
          unpack_bf2(u[j].y, v[2], v[3]);
          unpack_bf2(u[j].z, v[4], v[5]);
          unpack_bf2(u[j].w, v[6], v[7]);
#pragma unroll
          for (int q = 0; q < 8; ++q) acc[q] = fmaf(wv8[j], v[q], acc[q]);
        }
      } else {
        for (int j = 0; j < k; ++j) {
          const int32_t pj = __shfl_sync(0xffffffffu, sp, j);
          const float wjj = __shfl_sync(0xffffffffu, wj, j);
          if (pj < 0) continue;
          const uint4 uu = reinterpret_cast<const uint4 *>(y + static_cast<int64_t>(pj) * H)[c];
          float v[8];
          unpack_bf2(uu.x, v[0], v[1]);
          unpack_bf2(uu.y, v[2], v[3]);
          unpack_bf2(uu.z, v[4], v[5]);
          unpack_bf2(uu.w, v[6], v[7]);
#pragma unroll
          for (int q = 0; q < 8; ++q) acc[q] = fmaf(wjj, v[q], acc[q]);
        }
      }
      uint4 o;
      o.x = pack_bf2(acc[0], acc[1]);
      o.y = pack_bf2(acc[2], acc[3]);
      o.z = pack_bf2(acc[4], acc[5]);
      o.w = pack_bf2(acc[6], acc[7]);
      dst[c] = o;
    }
  }
  publish_when_last(ctrl, kCtrlDoneReturn, false, peers, L, N, rank, 1, false);
}

DevLayout dev_layout(const Layout &L) {
  return DevLayout{L.rows, L.ret, L.idx, L.wts, L.tok, L.cnt, L.flags};
}

int check_dims(int N, int64_t Tcap, int64_t H, int k) {
  if (N < 1 || N > kMaxRanks || Tcap < 1 || H <= 0 || H % 8 != 0 || k < 1 || k > 32)
    return fail(Q35_ERR_SHAPE, "ep window: N %d (1..%d) Tcap %lld H %lld (x8) k %d (1..32)", N,
                kMaxRanks, (long long)Tcap, (long long)H, k);
  if (int64_t(N) * Tcap * k >= (int64_t(1) << 31))
    return fail(Q35_ERR_SHAPE, "ep window: N*Tcap*k exceeds int32");
  return Q35_OK;
}

unsigned grid_for(int64_t warps_needed) {
  const int64_t cap = static_cast<int64_t>(num_sms()) * 8;  // 8 CTAs of 8 warps per SM
  int64_t ctas = (warps_needed + 7) / 8;
  if (ctas > cap) ctas = cap;
  if (ctas < 1) ctas = 1;
  return static_cast<unsigned>(ctas);
}

}  // namespace
}  // namespace q35

using namespace q35;

extern "C" int64_t q35_ep_window_bytes(int N, int64_t Tcap, int64_t H, int k) {
  if (check_dims(N, Tcap, H, k)) return -1;
  return window_layout(N, Tcap, H, k).total;
}

extern "C" int q35_ep_window_offsets(int N, int64_t Tcap, int64_t H, int k, int64_t *out10) {
  if (!out10) return fail(Q35_ERR_INVALID, "ep_window_offsets: null");
  const int st = check_dims(N, Tcap, H, k);
  if (st) return st;
  const Layout L = window_layout(N, Tcap, H, k);
  const int64_t v[10] = {L.rows, L.ret, L.idx, L.wts, L.tok, L.cnt, L.flags, L.ctrl, L.peers, L.total};
  for (int i = 0; i < 10; ++i) out10[i] = v[i];
  return Q35_OK;
}

extern "C" int q35_ep_window_alloc(int N, int64_t Tcap, int64_t H, int k, void **window) {
  if (!window) return fail(Q35_ERR_INVALID, "ep_window_alloc: null");
  const int st = check_dims(N, Tcap, H, k);
  if (st) return st;
  const Layout L = window_layout(N, Tcap, H, k);
  void *p = nullptr;
  Q35_CHECK_CUDA(cudaMalloc(&p, static_cast<size_t>(L.total)));
  // flags, ctrl and counts start at zero; the data areas need no initialisation
  cudaError_t e = cudaMemset(static_cast<uint8_t *>(p) + L.cnt, 0,
                             static_cast<size_t>(L.total - L.cnt));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "ep_window_alloc: clear");
  }
  *window = p;
  return Q35_OK;
}

extern "C" int q35_ep_window_free(void *window) {
  if (!window) return Q35_OK;
  Q35_CHECK_CUDA(cudaFree(window));
  return Q35_OK;
}

// 64-byte cudaIpcMemHandle_t of a window, for the other ranks to open.
extern "C" int q35_ep_ipc_handle(void *window, void *handle64) {
  if (!window || !handle64) return fail(Q35_ERR_INVALID, "ep_ipc_handle: null");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  cudaIpcMemHandle_t h;
  Q35_CHECK_CUDA(cudaIpcGetMemHandle(&h, window));
  memcpy(handle64, &h, sizeof(h));
  return Q35_OK;
}

extern "C" int q35_ep_ipc_open(const void *handle64, void **peer_window) {
  if (!handle64 || !peer_window) return fail(Q35_ERR_INVALID, "ep_ipc_open: null");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  void *p = nullptr;
  Q35_CHECK_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  *peer_window = p;
  return Q35_OK;
}

extern "C" int q35_ep_ipc_close(void *peer_window) {
  if (!peer_window) return Q35_OK;
  Q35_CHECK_CUDA(cudaIpcCloseMemHandle(peer_window));
  return Q35_OK;
}

// Writes the N window base addresses (as mapped in this process; entry `rank`
// is the local window) into the window's peer table.
extern "C" int q35_ep_set_peers(void *window, int N, int64_t Tcap, int64_t H, int k,
                                const uint64_t *peer_bases) {
  if (!window || !peer_bases) return fail(Q35_ERR_INVALID, "ep_set_peers: null");
  const int st = check_dims(N, Tcap, H, k);
  if (st) return st;
  const Layout L = window_layout(N, Tcap, H, k);
  Q35_CHECK_CUDA(cudaMemcpy(static_cast<uint8_t *>(window) + L.peers, peer_bases,
                            sizeof(uint64_t) * N, cudaMemcpyHostToDevice));
  return Q35_OK;
}

extern "C" int q35_ep_dispatch(const void *x, const int32_t *idx, const float *w, int64_t T,
                               int k, int64_t H, int El, int N, int rank, int64_t Tcap,
                               const int32_t *expert_owner, void *window, int32_t *ret_pos,
                               q35_stream_t stream) {
  if (!window || !ret_pos || (T > 0 && (!x || !idx || !w)))
    return fail(Q35_ERR_INVALID, "ep_dispatch: null pointer");
  int st = check_dims(N, Tcap, H, k);
  if (st) return st;
  if (T < 0 || T > Tcap || El < 1 || rank < 0 || rank >= N)
    return fail(Q35_ERR_SHAPE, "ep_dispatch: T %lld (<= Tcap %lld) El %d rank %d of %d",
                (long long)T, (long long)Tcap, El, rank, N);
  if (!aligned16(x)) return fail(Q35_ERR_ALIGN, "ep_dispatch: x not 16-byte aligned");
  int *err = device_error_word();
  if (!err) return fail(Q35_ERR_CUDA, "ep_dispatch: no device error word");
  const Layout L = window_layout(N, Tcap, H, k);
  uint8_t *win = static_cast<uint8_t *>(window);
  // at least one CTA: a rank with no tokens still publishes its (empty) counts
  const int tpc = (T + 31) / 32 < num_sms() / 2 ? 8 : 32;
  const int64_t ctas = T > 0 ? (T + tpc - 1) / tpc : 1;
  auto kern = tpc == 8 ? ep_dispatch_kernel<8> : ep_dispatch_kernel<32>;
  kern<<<static_cast<unsigned>(ctas), 256, 0,
                       reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t *>(x), idx, w, T, k, H, El, N, rank, Tcap,
      reinterpret_cast<uint32_t *>(win + L.ctrl), reinterpret_cast<const uint64_t *>(win + L.peers),
      dev_layout(L), ret_pos, expert_owner, err);
  Q35_LAUNCH_CHECK("ep_dispatch launch");
  return Q35_OK;
}

// which: 0 waits for every rank's dispatch, 1 for every rank's return.
extern "C" int q35_ep_wait(void *window, int N, int64_t Tcap, int64_t H, int k, int which,
                           int64_t limit_ns, q35_stream_t stream) {
  if (!window) return fail(Q35_ERR_INVALID, "ep_wait: null window");
  int st = check_dims(N, Tcap, H, k);
  if (st) return st;
  if (which != 0 && which != 1) return fail(Q35_ERR_INVALID, "ep_wait: which %d", which);
  if (limit_ns <= 0) return fail(Q35_ERR_INVALID, "ep_wait: limit %lld ns", (long long)limit_ns);
  int *err = device_error_word();
  if (!err) return fail(Q35_ERR_CUDA, "ep_wait: no device error word");
  const Layout L = window_layout(N, Tcap, H, k);
  const uint8_t *win = static_cast<const uint8_t *>(window);
  ep_wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      win, dev_layout(L), reinterpret_cast<const uint32_t *>(win + L.ctrl), N, which,
      static_cast<uint64_t>(limit_ns), err);
  Q35_LAUNCH_CHECK("ep_wait launch");
  return Q35_OK;
}

extern "C" int q35_ep_return(const void *y, const int32_t *slot_pos, int64_t Tcap, int k,
                             int64_t H, int N, int rank, void *window, q35_stream_t stream) {
  if (!window || !y || !slot_pos) return fail(Q35_ERR_INVALID, "ep_return: null pointer");
  int st = check_dims(N, Tcap, H, k);
  if (st) return st;
  if (rank < 0 || rank >= N) return fail(Q35_ERR_SHAPE, "ep_return: rank %d of %d", rank, N);
  if (!aligned16(y)) return fail(Q35_ERR_ALIGN, "ep_return: y not 16-byte aligned");
  const Layout L = window_layout(N, Tcap, H, k);
  uint8_t *win = static_cast<uint8_t *>(window);
  ep_return_kernel<<<grid_for(int64_t(N) * Tcap), 256, 0,
                     reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t *>(y), slot_pos, win, Tcap, k, H, N, rank,
      reinterpret_cast<uint32_t *>(win + L.ctrl), reinterpret_cast<const uint64_t *>(win + L.peers),
      dev_layout(L));
  Q35_LAUNCH_CHECK("ep_return launch");
  return Q35_OK;
}
