/*
 * q35b200.h - C ABI of the B200 (sm_100a) Qwen3-VL-MoE decoder-layer kernels.
 *
 * Every entry point takes raw device pointers, sizes and a CUDA stream, enqueues
 * its work on that stream and returns an int status (0 = success, see
 * q35_status).  Nothing in this header depends on torch: any host language that
 * can pass pointers (ctypes, cgo, JNI, N-API) can bind it.
 *
 * Conventions
 *   - "bf16" buffers are IEEE bfloat16 stored as uint16; fp32 buffers are float.
 *   - All buffers are dense row-major (C-contiguous) unless a stride is given.
 *   - Pointers used with TMA (GEMM and attention operands) must be 16-byte
 *     aligned and their row pitch a multiple of 16 bytes; violations return
 *     Q35_ERR_ALIGN before anything is launched.
 *   - A device-side failure (a bounded wait that ran out, an index out of range)
 *     never traps: the kernel records it in a per-device error word and returns.
 *     q35_device_error_check() synchronises the device and reports that word.
 *
 * Each declaration names the reference interface it replaces, as
 * file:line within luozoupi/Qwen3_5_VL_CUDA_CUSTOM (paths relative to
 * CUDA_qwen3_5-main/, REF below).
 */
#ifndef Q35B200_H
#define Q35B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define Q35_API __attribute__((visibility("default")))
#else
#define Q35_API
#endif

typedef struct CUstream_st *q35_stream_t;

enum q35_status {
  Q35_OK = 0,
  Q35_ERR_INVALID = 1,     /* null pointer, negative size, bad enum */
  Q35_ERR_SHAPE = 2,       /* shape outside what the kernel supports */
  Q35_ERR_ALIGN = 3,       /* pointer or pitch not 16-byte aligned */
  Q35_ERR_UNSUPPORTED = 4, /* dtype / head_dim / feature not built */
  Q35_ERR_CUDA = 5,        /* a CUDA runtime/driver call failed */
  Q35_ERR_DEVICE = 6,      /* the device error word is set */
  Q35_ERR_NO_DEVICE = 7    /* no sm_100 device is current */
};

/* ---- status / diagnostics (no reference counterpart: the reference raises
 *      c10::Error through TORCH_CHECK, REF cuda_qwen3_vl/csrc/common.h:10-12) */
Q35_API const char *q35_status_string(int status);
/* Human-readable detail of the last non-zero status returned on this host thread. */
Q35_API const char *q35_last_error_message(void);
/* Synchronises the current device, copies its error word to info[0..3]
 * (code, site, a, b), clears it and returns Q35_OK or Q35_ERR_DEVICE. */
Q35_API int q35_device_error_check(int32_t *info4);
/* Library build identity, e.g. "q35b200 sm_100a". */
Q35_API const char *q35_version(void);
/* Caps the grid of the persistent kernels (GEMMs) launched from this host
 * thread at n SMs (0: all SMs), so that work running at the same time -- e.g.
 * the collective kernels of an overlapped expert-parallel exchange -- keeps
 * some SMs.  No reference counterpart.                                     */
Q35_API int q35_set_sm_limit(int n);
/* Number of kernel launches this library has issued in this process (all
 * devices, all threads).  A CUDA-graph capture issues launches too, so the
 * difference across a capture is the number of library kernels in the graph.
 * No reference counterpart.                                                */
Q35_API int64_t q35_launch_count(void);

/* ---- RMSNorm ------------------------------------------------------------
 * y[r,:] = bf16( x[r,:] * rsqrt(mean(x[r,:]^2) + eps) * w ), fp32 inside.
 * Replaces rmsnorm_forward(Tensor x, Tensor weight, float eps)
 *   REF cuda_qwen3_vl/csrc/rmsnorm_op.cpp:9-12, kernel csrc/rmsnorm_op.cu:8-60.
 * x, y: bf16 [rows, cols]; w: bf16 [cols].  cols % 8 == 0.                   */
Q35_API int q35_rmsnorm_fwd(const void *x, const void *w, void *y, int64_t rows,
                    int64_t cols, float eps, q35_stream_t stream);

/* Same with fp32 input rows x [rows, cols] (the decoder layer keeps its
 * post-attention residual stream in fp32); y bf16.  No separate reference
 * entry: the reference normalises its bf16 residual (REF
 * modules/text_decoder.py:59 -> csrc/rmsnorm_op.cu:8-60).                    */
Q35_API int q35_rmsnorm_f32in_fwd(const float *x, const void *w, void *y,
                                  int64_t rows, int64_t cols, float eps,
                                  q35_stream_t stream);

/* ---- QK-norm + mRoPE + head-major split ---------------------------------
 * Input qkv: bf16 [B*S, (Hq + 2*Hkv) * D], the fused q/k/v projection output
 * (token-major; columns q heads, then k heads, then v heads).
 * Outputs (head-major): q [B,Hq,S,D], k [B,Hkv,S,D], v [B,Hkv,S,D] (bf16).
 * q and k are RMS-normalised over D with qw/kw (bf16 [D]), then rotated with
 * rotate-half RoPE whose angle for rotary index j is
 *     pos[axis(j), b, s] * inv_freq[j mod D/2]      (fp32),
 * axis(j) from the chunked mRoPE section layout (interleaved = 0) or the
 * HF-interleaved T/H/W layout (interleaved = 1).  positions: int64 [3,B,S].
 * Replaces the q_norm/k_norm + TextMRoPE.apply + mrope_forward chain
 *   REF cuda_qwen3_vl/modules/attention.py:82-87, modules/rotary.py:46-59,
 *   kernels/mrope.py:19-50,80-104, csrc/mrope_op.cpp:5-7.
 * D must be 32, 64 or 128; sections is a HOST array of 3 ints summing to D/2;
 * positions and inv_freq (fp32 [D/2]) are device arrays.                   */
Q35_API int q35_qknorm_mrope_fwd(const void *qkv, const void *qw, const void *kw,
                         const int64_t *positions, const float *inv_freq,
                         const int32_t *sections, int interleaved, void *q,
                         void *k, void *v, int64_t B, int64_t S, int Hq,
                         int Hkv, int D, float eps, q35_stream_t stream);

/* The q/k/v projection with QK-norm + mRoPE fused into its epilogue (head_dim
 * 128): x bf16 [B*S, H] times w_qkv bf16 [(Hq + 2 Hkv) * 128, H] (q, k, v
 * projection weights stacked), then per head RMSNorm (q_w / k_w, bf16 [128])
 * and rotate-half mRoPE for q and k, written head-major q [B,Hq,S,128],
 * k, v [B,Hkv,S,128] -- the same results as q35_gemm_bf16 followed by
 * q35_qknorm_mrope_fwd without the [B*S, (Hq+2Hkv)*128] intermediate.
 * workspace: fp32 [2 * B * S * 64] (rotary table).  Hq + 2 Hkv even.
 * Replaces q/k/v CudaLinear + q_norm/k_norm + TextMRoPE.apply
 * (REF modules/attention.py:82-87).                                        */
Q35_API int q35_qkv_proj_norm_rope(const void *x, const void *w_qkv, const void *q_w,
                                   const void *k_w, const int64_t *positions,
                                   const float *inv_freq, const int32_t *sections,
                                   int interleaved, void *q, void *k, void *v, int64_t B,
                                   int64_t S, int H, int Hq, int Hkv, float eps,
                                   float *workspace, q35_stream_t stream);

/* Apply mRoPE to a head-major tensor x [B,H,S,D] in place of
 * mrope_forward(x, cos, sin) (REF csrc/mrope_op.cpp:5-7), computing cos/sin
 * from positions like q35_qknorm_mrope_fwd (no normalisation).             */
Q35_API int q35_mrope_fwd(const void *x, void *y, const int64_t *positions,
                  const float *inv_freq, const int32_t *sections,
                  int interleaved, int64_t B, int H, int64_t S, int D,
                  q35_stream_t stream);

/* ---- Router --------------------------------------------------------------
 * logits[t,e] = sum_h x[t,h] * wg[e,h] (+ bias[e])  in fp32 (x bf16, wg fp32),
 * p = softmax(logits[t,:]); idx[t,0..k) = top-k of p, sorted descending,
 * ties to the lower expert index; weights[t,j] = p[idx] / sum_j p[idx]
 * (renorm != 0) or p[idx] (renorm == 0).
 * Replaces the router of CudaSparseMoE.forward (REF modules/moe.py:60-65):
 *   matmul_forward (csrc/matmul_op.cpp:11-14) -> softmax_forward
 *   (csrc/softmax_op.cpp:6-9) -> topk_forward (csrc/moe_routing_op.cpp:9-13).
 * bias and wg_split may be NULL.  1 <= E <= 256, k <= 16, H % 32 == 0.
 * idx is int32 (the reference returns int64; values are equal).            */
Q35_API int q35_router_topk_fwd(const void *x, const float *wg, const void *wg_split,
                                const float *bias, float *logits, int32_t *idx,
                                float *weights, int64_t T, int H, int E, int k,
                                int renorm, float *workspace, q35_stream_t stream);
/* fp32 elements of `workspace` the tensor-core path needs (wg_split != NULL). */
Q35_API int64_t q35_router_workspace(int64_t T, int H, int E);

/* Tensor-core router inputs.  q35_router_split_weights writes w3 (bf16
 * [E, 3H]) = [lo | mid | hi] with lo + mid + hi == wg exactly (8 significant
 * bits each); passing it as wg_split above (H % 64 == 0, E % 32 == 0) computes
 * the logits as a tcgen05 GEMM of [x | x | x] against w3 -- every product is
 * exact in fp32 and accumulates in fp32 in k_splits partial sums -- instead of
 * the fp32 SIMT GEMV.  q35_router_logits_tc is that GEMM alone, writing
 * partial planes fp32 [k_splits, T, E] (k_splits must divide 3H/64).  No
 * reference counterpart (the reference computes the logits with its SIMT
 * matmul_fwd_kernel, REF csrc/matmul_op.cu:15-92).                           */
Q35_API int q35_router_split_weights(const float *wg, void *w3, int E, int H,
                                     q35_stream_t stream);
Q35_API int q35_router_logits_tc(const void *x, const void *w3, float *partials,
                                 int64_t T, int H, int E, int k_splits,
                                 q35_stream_t stream);

/* Row softmax in fp32, replaces softmax_forward (REF csrc/softmax_op.cpp:6-9).
 * x, y: fp32 [rows, cols], cols <= 4096.                                     */
Q35_API int q35_softmax_fwd(const float *x, float *y, int64_t rows, int cols,
                    q35_stream_t stream);

/* Row top-k of fp32 values, sorted descending, ties to the lower column;
 * replaces topk_forward (REF csrc/moe_routing_op.cpp:9-13, kernel
 * csrc/moe_routing_op.cu:11-63).  vals fp32 [rows,k], idx int64 [rows,k].
 * cols <= 4096, k <= 16.                                                    */
Q35_API int q35_topk_fwd(const float *x, float *vals, int64_t *idx, int64_t rows,
                 int cols, int k, q35_stream_t stream);

/* ---- Permutation ---------------------------------------------------------
 * Sorts the T*k (token, slot) pairs of idx [T,k] by (expert, token): the order
 * the reference's per-expert mask.nonzero loop visits them
 * (REF modules/moe.py:71-76).  Outputs:
 *   counts    int32 [E]        tokens routed to each expert
 *   offsets   int32 [E+1]      exclusive prefix sum of counts
 *   sorted_tok int32 [T*k]     token index of sorted row r
 *   slot_pos  int32 [T*k]      sorted row of pair (t, j) at t*k + j
 *   tile_offsets int32 [E+1]   prefix sum of ceil(counts[e] / 128), the
 *                               grouped-GEMM M-tile schedule
 * workspace: int32 scratch of q35_moe_permute_workspace(T, E) elements.
 * A negative id marks an empty slot (slot_pos = -1, no error: the
 * expert-parallel receiver uses it); ids >= E are recorded in the device
 * error word and the pair is dropped (slot_pos = -1).                      */
Q35_API int64_t q35_moe_permute_workspace(int64_t T, int E);
Q35_API int q35_moe_permute(const int32_t *idx, int64_t T, int k, int E,
                    int32_t *counts, int32_t *offsets, int32_t *sorted_tok,
                    int32_t *slot_pos, int32_t *tile_offsets,
                    int32_t *workspace, q35_stream_t stream);

/* Allocation-free q35_moe_permute.  No counterpart in the reference: it is
 * for callers that cannot allocate device memory while routing (a fixed
 * memory pool that must not grow, a serving path where cudaMalloc is
 * forbidden, a host that only passes input and output buffers).  Same inputs
 * and outputs as q35_moe_permute minus `workspace`: the scratch is a 256 KiB
 * array built into the library, held by every GPU that loads it until exit.
 * Limit: ceil(T/128) * E <= q35_moe_permute_noalloc_max_workspace() (65536,
 * e.g. T = 65536 tokens at E = 128); larger calls return Q35_ERR_SHAPE.
 * The first call on a device looks up the array's device address (once per
 * device); make that first call before any stream capture.  All calls share
 * the one array: calls that overlap on the GPU (other streams, other host
 * threads) race and must be serialised by the caller.  Out-of-range expert
 * ids are dropped (slot_pos = -1) but not reported in the device error word.
 * The call itself allocates nothing.                                        */
Q35_API int64_t q35_moe_permute_noalloc_max_workspace(void);
Q35_API int q35_moe_permute_noalloc(const int32_t *idx, int64_t T, int k, int E,
                                    int32_t *counts, int32_t *offsets,
                                    int32_t *sorted_tok, int32_t *slot_pos,
                                    int32_t *tile_offsets, q35_stream_t stream);

/* Expert-parallel send slabs.  A token sends at most one row to each rank,
 * so the send buffer send bf16 [N, T, H] has a fixed slab of T rows per
 * destination: row (d, t) = x[t] if one of token t's top-k experts
 * (idx int32 [T, k], global ids) is owned by rank d (experts
 * [d*El, (d+1)*El)), else left untouched.  meta_idx int32 [N, T, k] holds, at
 * slot j, the slot's expert id local to rank d or -1, meta_w fp32 [N, T, k]
 * its weight (w fp32 [T, k]) or 0 (slab d of each starts meta_slab >= T*k
 * elements after slab d-1, so both can interleave in one buffer); ret_pos int32 [T, N] = d*T + t for the
 * ranks token t uses, else -1.  k <= 16, N <= 32.  An even-split all-to-all
 * of these slabs needs no host-side sizes.  No reference counterpart.       */
Q35_API int q35_ep_scatter(const void *x, const int32_t *idx, const float *w, int64_t T, int k,
                           int64_t H, int El, int N, void *send, int32_t *meta_idx,
                           float *meta_w, int64_t meta_slab, int32_t *ret_pos,
                           q35_stream_t stream);

/* Tensor-core router in two launches (replaces the matmul -> softmax -> topk
 * chain of REF modules/moe.py:60-65, csrc/softmax_op.cu:8-53 and
 * csrc/moe_routing_op.cu:11-63 for supported shapes): x bf16 [T, H],
 * w3 = q35_router_split_weights(gate) bf16 [E, 3H], bias fp32 [E] or NULL.
 * Outputs as q35_router_topk_fwd, and, if chunk_counts != NULL, int32
 * [ceil(T/128), E]: per 128-token chunk the number of tokens routed to each
 * expert (the permutation's count pass, for q35_moe_permute_counted).
 * Supported when q35_router_fused_supported(T, H, E, k): H % 256 == 0,
 * E in {32, 64, 128}, 1 <= k <= min(16, E).  Logits are summed in a fixed
 * order (deterministic); ties go to the lower expert id.                    */
Q35_API int q35_router_fused_supported(int64_t T, int H, int E, int k);
Q35_API int q35_router_topk_fused(const void *x, const void *w3, const float *bias,
                                  float *logits, int32_t *idx, float *weights,
                                  int32_t *chunk_counts, int64_t T, int H, int E, int k,
                                  int renorm, q35_stream_t stream);

/* q35_moe_permute from the router's chunk_counts in one launch, no workspace:
 * the same outputs bit for bit (REF modules/moe.py:71-76 ordering).         */
Q35_API int q35_moe_permute_counted(const int32_t *idx, int64_t T, int k, int E,
                                    const int32_t *chunk_counts, int32_t *counts,
                                    int32_t *offsets, int32_t *sorted_tok, int32_t *slot_pos,
                                    int32_t *tile_offsets, q35_stream_t stream);

/* q35_moe_permute over slab-structured rows: idx int32 [n_slabs*slab_rows, k]
 * where only rows [s*slab_rows, s*slab_rows + slab_cnt[s]) of slab s take
 * part (slab_cnt int32 [n_slabs] in device memory); the other rows are
 * ignored whatever they hold and their slot_pos entries are left untouched.
 * Outputs sized for n_slabs*slab_rows rows.  This is the receive side of the
 * peer-memory expert-parallel exchange, where slab s holds the rows rank s
 * sent.  No reference counterpart (the reference has no expert parallelism). */
Q35_API int q35_moe_permute_slabs(const int32_t *idx, int n_slabs, int64_t slab_rows,
                                  const int32_t *slab_cnt, int k, int E, int32_t *counts,
                                  int32_t *offsets, int32_t *sorted_tok, int32_t *slot_pos,
                                  int32_t *tile_offsets, int32_t *workspace,
                                  q35_stream_t stream);

/* ---- Expert-parallel exchange over peer memory (NVLink) -----------------
 * No reference counterpart: the reference runs every expert on one GPU
 * (REF cuda_qwen3_vl/modules/moe.py:71-83).  N ranks (one process per GPU),
 * rank r owns experts [r*El, (r+1)*El).  Each rank allocates one exchange
 * window (q35_ep_window_alloc, sized by N, Tcap = max tokens per rank and
 * call, H, k), exports it with q35_ep_ipc_handle, opens every peer's handle
 * with q35_ep_ipc_open and stores the N base addresses (its own at index r)
 * with q35_ep_set_peers.  One forward is then, on every rank, in stream order:
 *   q35_ep_dispatch  token rows + slot lists into the owners' windows,
 *                    ret_pos int32 [T, N] = d*Tcap + t where rank d will
 *                    return token t's partial, else -1;
 *   q35_ep_wait(0)   until every rank's rows have arrived;
 *   q35_moe_permute_slabs / gather / grouped GEMMs on the window's slabs
 *                    (offsets from q35_ep_window_offsets: rows, ret, idx,
 *                    wts, tok, cnt, flags, ctrl, peers, total bytes);
 *   q35_ep_return    each received row's weighted partial (slot_pos of that
 *                    permutation, y the grouped down output) into the
 *                    sender's window;
 *   q35_ep_wait(1)   until every rank's partials have arrived;
 *   q35_moe_combine  y = the window's ret area, weights 1, slot_pos = ret_pos,
 *                    k = N: adds each token's partials to its residual.
 * Every rank must issue the same sequence of calls.  Waits give up after
 * limit_ns and record DEV_ERR_WAIT_TIMEOUT (site 310 dispatch, 311 return) in
 * the device error word; dispatch reports an expert id >= N*El at site 301.
 * N <= 32, k <= 32, H % 8 == 0, T <= Tcap.                                   */
Q35_API int64_t q35_ep_window_bytes(int N, int64_t Tcap, int64_t H, int k);
Q35_API int q35_ep_window_offsets(int N, int64_t Tcap, int64_t H, int k, int64_t *out10);
Q35_API int q35_ep_window_alloc(int N, int64_t Tcap, int64_t H, int k, void **window);
Q35_API int q35_ep_window_free(void *window);
Q35_API int q35_ep_ipc_handle(void *window, void *handle64);
Q35_API int q35_ep_ipc_open(const void *handle64, void **peer_window);
Q35_API int q35_ep_ipc_close(void *peer_window);
Q35_API int q35_ep_set_peers(void *window, int N, int64_t Tcap, int64_t H, int k,
                             const uint64_t *peer_bases);
/* expert_owner: NULL for the contiguous placement (expert e on rank e / El,
 * local slot e % El), else int32 [N*El] in device memory: (rank << 16) | local
 * slot of every expert (balanced placements).                               */
Q35_API int q35_ep_dispatch(const void *x, const int32_t *idx, const float *w, int64_t T, int k,
                            int64_t H, int El, int N, int rank, int64_t Tcap,
                            const int32_t *expert_owner, void *window, int32_t *ret_pos,
                            q35_stream_t stream);
Q35_API int q35_ep_wait(void *window, int N, int64_t Tcap, int64_t H, int k, int which,
                        int64_t limit_ns, q35_stream_t stream);
Q35_API int q35_ep_return(const void *y, const int32_t *slot_pos, int64_t Tcap, int k, int64_t H,
                          int N, int rank, void *window, q35_stream_t stream);

/* Self-test of the bounded waits (no reference counterpart): one kernel
 * waits on an mbarrier phase that nothing completes, gives up after limit_ns
 * (0 < limit_ns <= 2 s), records DEV_ERR_WAIT_TIMEOUT at site 901 (a = the
 * microseconds waited) in the device error word and returns.               */
Q35_API int q35_selftest_wait_timeout(int64_t limit_ns, q35_stream_t stream);

/* Token embedding: out[r,:] = table[ids[r],:] for int64 ids (bf16 [V, cols],
 * cols % 8 == 0).  Replaces embedding_forward (REF csrc/embedding_op.cu:5-97,
 * kernels/embedding.py).  Ids are checked on the device: an id outside [0, V)
 * gives a zero row and DEV_ERR_INDEX (site 104) in the device error word.    */
Q35_API int q35_embedding_fwd(const void *table, const int64_t *ids, void *out, int64_t n,
                              int64_t V, int64_t cols, q35_stream_t stream);

/* dst[r,:] = src[rows[r],:] for r < n (bf16, cols % 8 == 0); n may be read
 * from device memory (n_dev != NULL: *n_dev rows, at most n_max).           */
Q35_API int q35_gather_rows(const void *src, const int32_t *rows, void *dst,
                    int64_t n_max, const int32_t *n_dev, int64_t cols,
                    q35_stream_t stream);

/* ---- GEMMs on tcgen05 (A, B K-major bf16, fp32 accumulate in TMEM) -------
 * Dense: out[m,n] = sum_k a[m,k] * b[n,k]  (+ residual[m,n]) , bf16 out.
 * Replaces matmul_forward(x, weight, bias) (REF csrc/matmul_op.cpp:11-14,
 * csrc/matmul_op.cu:15-149) for the q/k/v/o projections; bias may be NULL
 * (bf16 [N]); residual may be NULL (bf16 [M,N], fuses residual_add,
 * REF csrc/residual_add_op.cpp:5-7).  K % 8 == 0, N % 32 == 0.             */
Q35_API int q35_gemm_bf16(const void *a, const void *b, const void *bias,
                  const void *residual, void *out, int64_t M, int64_t N,
                  int64_t K, q35_stream_t stream);

/* Split-K variant of q35_gemm_bf16 / q35_gemm_bf16_f32out for few rows (decode
 * batches): k_splits fp32 partial planes are written to workspace (fp32
 * [k_splits, M, N]) and summed in a fixed order with bias and residual;
 * out_f32 selects an fp32 output.  K % 64 == 0 with k_splits dividing K/64.
 * Same reference op as q35_gemm_bf16 (REF csrc/matmul_op.cpp:11-14).        */
Q35_API int q35_gemm_bf16_splitk(const void *a, const void *b, const void *bias,
                                 const void *residual, void *out, int out_f32, int64_t M,
                                 int64_t N, int64_t K, int k_splits, float *workspace,
                                 q35_stream_t stream);

/* Same GEMM with an fp32 output: out[m,n] = acc + bias[n] + residual[m,n]
 * stored as fp32 (residual bf16).  The decoder layer uses it for o_proj so the
 * post-attention residual h = x + attn is rounded once, at the layer output
 * (the reference rounds it to bf16: REF modules/text_decoder.py:58).          */
Q35_API int q35_gemm_bf16_f32out(const void *a, const void *b, const void *bias,
                                 const void *residual, float *out, int64_t M,
                                 int64_t N, int64_t K, q35_stream_t stream);

/* Grouped expert GEMMs over the permuted rows of q35_moe_permute.
 * Group e owns rows [offsets[e], offsets[e+1]) of a (rows sorted by expert).
 * gate_up: act[r, j] = bf16( silu(g) * u ), g = a[r,:].w[e, j, :],
 *          u = a[r,:].w[e, I + j, :]; w = gate_up_proj [E, 2I, H], act [R, I].
 *          Replaces matmul(x_sub, gate_up_proj[e]) + swiglu (REF
 *          modules/moe.py:77-80, csrc/swiglu_op.cu:6-18).
 * down:    y[r, n] = bf16( act[r,:].w[e, n, :] ); w = down_proj [E, H, I].
 *          Replaces matmul(activated, down_proj[e]) (REF modules/moe.py:81).
 * offsets/tile_offsets are device arrays ([E+1]); rows_cap bounds R.
 * w_packed != 0: the weight is the q35_pack_b_tiles copy of the same tensor.  */
Q35_API int q35_grouped_gemm_gateup_swiglu(const void *a, const void *w_gate_up,
                                           void *act, const int32_t *offsets,
                                           const int32_t *tile_offsets, int E,
                                           int64_t rows_cap, int H, int I,
                                           int w_packed, q35_stream_t stream);
Q35_API int q35_grouped_gemm_down(const void *act, const void *w_down, void *y,
                                  const int32_t *offsets, const int32_t *tile_offsets,
                                  int E, int64_t rows_cap, int H, int I,
                                  int w_packed, q35_stream_t stream);

/* Packs a K-major bf16 weight matrix [rows, K] (rows % 128 == 0, K % 64 == 0)
 * into contiguous 128-row x 64-column tiles (tile (r, k) at element offset
 * ((r * K/64) + k) * 8192).  The grouped GEMMs read such a copy when called
 * with w_packed != 0: every weight tile is then one contiguous 16 KB read.
 * No reference counterpart (a storage format of this library).               */
Q35_API int q35_pack_b_tiles(const void *src, void *dst, int64_t rows, int64_t K,
                             q35_stream_t stream);

/* ---- Combine --------------------------------------------------------------
 * out[t,:] = bf16( residual[t,:] + sum_j weights[t,j] * y[slot_pos[t*k+j],:] )
 * summed in fp32 in slot order; residual may be NULL, bf16 or (residual_f32)
 * fp32.  slot_pos < 0 marks a
 * slot whose row lives on another rank (skipped).  Replaces the weighted
 * index_add_forward + residual_add_forward pair (REF modules/moe.py:82-83,
 * csrc/moe_routing_op.cpp:9-13, modules/text_decoder.py:64).                 */
Q35_API int q35_moe_combine(const void *y, const float *weights,
                            const int32_t *slot_pos, const void *residual,
                            int residual_f32, void *out, int64_t T, int k,
                            int64_t H, q35_stream_t stream);

/* target[index[r],:] += source[r,:] (bf16 or fp32 rows by dtype code:
 * 0 = fp32, 1 = bf16), replaces index_add_forward
 * (REF csrc/moe_routing_op.cpp:9-13, csrc/moe_routing_op.cu:89-102).       */
Q35_API int q35_index_add(void *target, const void *source, const int64_t *index,
                  int64_t n_src, int64_t n_target, int64_t cols, int dtype,
                  q35_stream_t stream);

/* Elementwise ops of the reference op layer (bf16): swiglu_forward
 * (REF csrc/swiglu_op.cpp:8-11) and residual_add_forward
 * (REF csrc/residual_add_op.cpp:5-7).                                        */
Q35_API int q35_swiglu_fwd(const void *gate, const void *up, void *out, int64_t n,
                   q35_stream_t stream);
Q35_API int q35_residual_add_fwd(const void *a, const void *b, void *out, int64_t n,
                         q35_stream_t stream);

/* ---- Attention ------------------------------------------------------------
 * Prefill: out[b, s, h*D + d] = softmax(q.k^T * scale + mask) . v, GQA with
 * Hq/Hkv query heads per kv head, causal mask bottom-right aligned
 * (query i of Sq sees keys j <= i + Skv - Sq).  q [B,Hq,Sq,D],
 * k/v [B,Hkv,Skv,D] head-major bf16; out token-major bf16 [B,Sq,Hq*D];
 * lse (fp32 [B,Hq,Sq], may be NULL).  D in {32, 64, 128}.
 * Replaces flash_attention_forward(q, k, v, scale, is_causal, num_kv_groups)
 *   REF csrc/flash_attention_op.cpp:13-16, csrc/flash_attention_op.cu:17-180. */
Q35_API int q35_attn_prefill_fwd(const void *q, const void *k, const void *v,
                         void *out, float *lse, int64_t B, int Hq, int Hkv,
                         int64_t Sq, int64_t Skv, int D, float scale,
                         int causal, q35_stream_t stream);

/* Decode (Sq small, long Skv): split-KV attention with an LSE merge.
 * Same layouts as prefill; non-causal over all Skv keys (the reference's
 * S_q != S_k rule, REF modules/attention.py:95).  Sq <= 16.
 * workspace: fp32 scratch of q35_attn_decode_workspace(...) floats.          */
Q35_API int64_t q35_attn_decode_workspace(int64_t B, int Hq, int64_t Sq, int64_t Skv,
                                  int D);
Q35_API int q35_attn_decode_fwd(const void *q, const void *k, const void *v, void *out,
                        int64_t B, int Hq, int Hkv, int64_t Sq, int64_t Skv,
                        int D, float scale, float *workspace,
                        q35_stream_t stream);

/* Attention over a preallocated KV cache: k_cache / v_cache bf16
 * [B, Hkv, kv_cap, D], of which the first Skv rows per head are valid; q and
 * out as in q35_attn_prefill_fwd / q35_attn_decode_fwd (the same kernels with
 * a head stride of kv_cap rows instead of Skv).  kv_cap >= Skv.  Rows past Skv
 * are read by the last key tile and masked, so they must hold finite values
 * (zero-initialise the cache).  Replaces the torch.cat of past and new K/V
 * followed by flash_attention (REF modules/attention.py:89-95).            */
Q35_API int q35_attn_prefill_cache_fwd(const void *q, const void *k_cache, const void *v_cache,
                                       void *out, float *lse, int64_t B, int Hq, int Hkv,
                                       int64_t Sq, int64_t Skv, int64_t kv_cap, int D,
                                       float scale, int causal, q35_stream_t stream);
Q35_API int q35_attn_decode_cache_fwd(const void *q, const void *k_cache, const void *v_cache,
                                      void *out, int64_t B, int Hq, int Hkv, int64_t Sq,
                                      int64_t Skv, int64_t kv_cap, int D, float scale,
                                      float *workspace, q35_stream_t stream);

/* In-place KV-cache append: rows s < S of k_new / v_new bf16 [B, Hkv, S, D]
 * go to rows offset + s of the [B, Hkv, cap, D] caches.  offset + S <= cap,
 * D % 8 == 0.  Replaces k = cat(past_k, k), v = cat(past_v, v)
 * (REF modules/attention.py:89-93) without copying the past rows.         */
Q35_API int q35_kv_append(const void *k_new, const void *v_new, void *k_cache, void *v_cache,
                          int64_t B, int Hkv, int64_t S, int D, int64_t cap, int64_t offset,
                          q35_stream_t stream);

/* ---- Vision-tower operators (bf16, fp32 math) -------------------------- */
/* LayerNorm over the last dim: (x - mean) * rsqrt(var + eps) * w (+ b); b may
 * be NULL.  cols % 8 == 0.  Replaces layernorm_forward
 * (REF kernels/layernorm.py:54, csrc/layernorm_op.cu).                       */
Q35_API int q35_layernorm_fwd(const void *x, const void *w, const void *b, void *y,
                              int64_t rows, int64_t cols, float eps, q35_stream_t stream);
/* GELU, tanh approximation, elementwise over n values (n % 8 == 0).
 * Replaces gelu_tanh_forward (REF kernels/gelu_tanh.py:49).                  */
Q35_API int q35_gelu_tanh_fwd(const void *x, void *y, int64_t n, q35_stream_t stream);
/* Rotate-half RoPE on the first dr of D dims of x [B,H,S,D] (the rest copied);
 * cos/sin bf16 [B,S,dr] (per_batch != 0) or [S,dr].  D % 8 == 0, dr % 16 == 0.
 * Replaces rope_forward (REF kernels/rope.py:58).                            */
Q35_API int q35_rope_fwd(const void *x, const void *cos_t, const void *sin_t, void *y,
                         int64_t B, int H, int64_t S, int D, int dr, int per_batch,
                         q35_stream_t stream);
/* Non-overlapping Conv3d patch embedding as a GEMM: patches bf16
 * [n_patches, K] (each patch flattened C*T*P*P), w bf16 [embed, K], bias bf16
 * [embed] or NULL -> out bf16 [n_patches, embed].  K % 8 == 0, embed % 32 == 0.
 * Replaces conv3d_patch_forward (REF kernels/conv3d_patch.py:17-40).        */
Q35_API int q35_conv3d_patch_fwd(const void *patches, const void *w, const void *bias,
                                 void *out, int64_t n_patches, int64_t embed, int64_t K,
                                 q35_stream_t stream);

/* Vision attention input (replaces the qkv reshape + apply_rope pair of
 * REF modules/attention.py:31-39): qkv bf16 [S, 3, H, D] (the fused projection
 * with its bias) -> q, k, v bf16 [H, S, Dp], Dp >= D, zero-padded, with the
 * rotate-half rotary over all D dims of q and k; angles fp32 [S, D/2]: the
 * angle of dims j and j + D/2 (fp32 sin/cos).  Padding lets head dims the
 * attention kernels do not take (72 in Qwen3-VL's vision tower) run on the
 * head_dim 128 kernels.                                                     */
Q35_API int q35_vision_qkv_rope_pad(const void *qkv, const float *angles, void *q, void *k,
                                    void *v, int64_t S, int H, int D, int Dp,
                                    q35_stream_t stream);
/* Token-major [S, H, Dp] -> [S, H, D]: drops the head padding of the
 * attention output (no reference counterpart; the reference needs no padding). */
Q35_API int q35_unpad_heads(const void *x, void *y, int64_t S, int H, int D, int Dp,
                            q35_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* Q35B200_H */
