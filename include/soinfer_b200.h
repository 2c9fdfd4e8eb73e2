/*
 * soinfer_b200.h -- C ABI of the B200 (sm_100a) decode hot path of soinfer.
 *
 * Every entry point takes plain device/host pointers, 64-bit sizes and a CUDA
 * stream handle (`void* stream`, a cudaStream_t; NULL = legacy default
 * stream), launches asynchronously on that stream, and returns a status code
 * (SOINFER_OK == 0).  No entry point aborts the process: argument errors are
 * reported as SOINFER_ERR_INVALID_ARGUMENT before anything is launched, and
 * launch failures as SOINFER_ERR_CUDA.  soinfer_last_error() returns the
 * message of the most recent failure on the calling thread.
 *
 * Data formats (identical to the reference's packing contract,
 * csrc/include/layout.h:19-67 of sparse-offload-infer):
 *   - INT4 weights: uint8 [N, ceil(K/8)*4]; each 4-byte group holds 8 signed
 *     two's-complement nibbles in AWQ order [0,2,4,6,1,3,5,7]
 *     (byte0 = v0|v2<<4, byte1 = v4|v6<<4, byte2 = v1|v3<<4, byte3 = v5|v7<<4).
 *   - INT8 weights: int8 [N, K], one value per byte.
 *   - scales: fp32 [N, num_groups] row-major, element k of row n uses
 *     scale[n, k / group_size]; num_groups == ceil(K / group_size).
 *   - activations / outputs: IEEE fp16 (stored as uint16_t bit patterns).
 *
 * Each declaration names the reference interface it replaces as
 * path:line inside the sparse-offload-infer repository.
 */
#ifndef SOINFER_B200_H_
#define SOINFER_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef uint16_t soinfer_half; /* IEEE binary16 bit pattern */

enum soinfer_status {
  SOINFER_OK = 0,
  SOINFER_ERR_INVALID_ARGUMENT = 1, /* a precondition failed; nothing launched */
  SOINFER_ERR_CUDA = 2,             /* a CUDA runtime call or launch failed     */
  SOINFER_ERR_UNSUPPORTED = 3,      /* valid request this build cannot serve    */
  SOINFER_ERR_HOST = 4              /* host-side failure (thread pool, memcpy)  */
};

/* ABI version of this header (bumped on any signature change). */
int soinfer_abi_version(void);
/* Message of the last failed call on this thread ("" if none). */
const char* soinfer_last_error(void);
/* Static name of a status code. */
const char* soinfer_status_string(int status);

/* Reads and clears the device-side error bits set by kernels whose bounded
 * waits gave up instead of hanging (bit 0: an asynchronous copy into shared
 * memory did not complete within its time limit).  Synchronous; *flags = 0
 * means no kernel reported a problem since the previous call.  No reference
 * counterpart. */
int soinfer_device_errors(int* flags);

/* ---------------------------------------------------------------- GEMV --- */

/* y[n] = fp16( sum_k scale[n, k/g] * q[n,k] * x[k] ), fp32 accumulation.
 * Wq: uint8 [N, ceil(K/8)*4]; scale: fp32 [N, num_groups]; x: fp16 [K];
 * y: fp16 [N].  group_size must be a positive multiple of 8 and num_groups
 * == ceil(K/group_size).
 * Replaces: csrc/bindings.cpp:300-303 (gemv_w4a16_group) and
 *           csrc/kernels/gemv_w4a16_group.cu:23-63. */
int soinfer_gemv_w4a16_group(const uint8_t* Wq, const float* scale, const soinfer_half* x,
                             soinfer_half* y, int64_t N, int64_t K, int64_t group_size,
                             int64_t num_groups, void* stream);

/* Same contract and same kernel as soinfer_gemv_w4a16_group (the two reference
 * variants differ only in how the nibbles are unpacked; here both names run
 * the one sm_100a kernel, so their outputs are identical by construction).
 * Replaces: csrc/bindings.cpp:305-309 (gemv_w4a16_group_lop3) and
 *           csrc/kernels/gemv_w4a16_group.cu:77-134. */
int soinfer_gemv_w4a16_group_lop3(const uint8_t* Wq, const float* scale, const soinfer_half* x,
                                  soinfer_half* y, int64_t N, int64_t K, int64_t group_size,
                                  int64_t num_groups, void* stream);

/* Launch flags for the *_ex entry points. */
#define SOINFER_FLAG_PDL 1u /* programmatic dependent launch: the kernel may start before the
                               previous kernel in the stream has finished and streams its weights
                               meanwhile; only x is waited for.  Set it only when the weights are
                               not written by the kernel that precedes this one in the stream. */

/* soinfer_gemv_w4a16_group_lop3 with launch flags (SOINFER_FLAG_*).
 * No reference counterpart (the reference launches on the legacy stream). */
int soinfer_gemv_w4a16_group_ex(const uint8_t* Wq, const float* scale, const soinfer_half* x,
                                soinfer_half* y, int64_t N, int64_t K, int64_t group_size,
                                int64_t num_groups, uint32_t flags, void* stream);

/* One INT4 GEMV of a batch: y = dequant(Wq, scale) @ x (shapes as in
 * soinfer_gemv_w4a16_group).  dep = index of an earlier task of the same
 * batch whose output this task's x depends on (x is read only after that
 * task has finished), or -1 if x is ready when the batch starts. */
typedef struct soinfer_gemv_task {
  const uint8_t* Wq;
  const float* scale;
  const soinfer_half* x;
  soinfer_half* y;
  int64_t N, K, group_size, num_groups;
  int64_t dep;
  /* Optional epilogue (NULL = off), applied to d = fp16(dot) in this order:
   * glu_gate: d = fp16(silu(float(glu_gate[n])) * float(d))  (SwiGLU: y = the
   *   MLP hidden state when this task is up_proj and glu_gate gate_proj's y);
   * residual: d = fp16(float(residual[n]) + float(d))  (the residual add).
   * Each equals the unfused op on the fp16 GEMV output.  A glu_gate /
   * residual buffer is either ready before the launch or the y of an earlier
   * task of the batch with the same N. */
  const soinfer_half* residual;
  const soinfer_half* glu_gate;
  /* Optional prologue (NULL = off): the task multiplies RMSNorm(x) * norm_weight
   * (fp16 [K], eps norm_eps) instead of x -- each CTA normalises x in shared
   * memory as soinfer_rmsnorm computes it (v * rsqrt(mean(v^2) + eps) * w,
   * rounded to fp16), so the normalised vector is never written.  Needs the
   * persistent path (K and group_size multiples of 128). */
  const soinfer_half* norm_weight;
  float norm_eps;
  /* With norm_weight: if not NULL, the normalised x (fp16 [K]) is also written
   * here, complete when the launch is (for kernels that need it later). */
  soinfer_half* norm_out;
} soinfer_gemv_task;

/* Bytes of zero-initialised device workspace soinfer_gemv_w4a16_batch needs
 * for num_tasks tasks (per-task completion counters; left zeroed on return). */
int64_t soinfer_gemv_batch_workspace_bytes(int64_t num_tasks);

/* Runs up to 256 INT4 GEMVs, in task order, as one persistent kernel: a
 * producer warp per SM streams the weights of task after task through a deep
 * shared-memory ring (weights never wait for activations) while consumer
 * warps compute each task once its x is ready.  Dependencies are expressed
 * with soinfer_gemv_task.dep.  Tasks outside the fast-path constraints (K and
 * group_size multiples of 128, num_groups % 4 == 0, 16-byte aligned operands,
 * N <= 128 * #SMs) make the whole batch run as ordered single-GEMV launches.
 * No reference counterpart: the reference launches one GEMV per weight
 * (runtime/generate.py:116-138). */
int soinfer_gemv_w4a16_batch(const soinfer_gemv_task* tasks, int64_t num_tasks, void* workspace,
                             int64_t workspace_bytes, void* stream);

/* Row-indirect INT4 GEMV over HBM-resident weights: y[r] = row rows[r] of
 * dequant(Wq, scale) dotted with x, for r in [0, num_sel).  Equivalent to
 * gathering rows (Wq[rows], scale[rows]) and calling
 * soinfer_gemv_w4a16_group_lop3 on them (bit-identical), without the copy.
 * rows: int32 [num_sel] device, each in [0, N).
 * Replaces the pair at runtime/generate.py:286-302 (gather_rows_staged of the
 * selected up_proj rows + gemv_w4a16_group_lop3 with N = k) when the matrix is
 * resident in device memory.  glu_gate (optional, fp16 [N]): y[r] =
 * fp16(silu(glu_gate[rows[r]]) * y[r]) -- DIP's SwiGLU on the selected
 * channels (generate.py:300-302), equal to soinfer_swiglu after the GEMV. */
int soinfer_gemv_w4a16_rows(const uint8_t* Wq, const float* scale, int64_t N, const int32_t* rows,
                            int64_t num_sel, const soinfer_half* x, soinfer_half* y, int64_t K,
                            int64_t group_size, int64_t num_groups, const soinfer_half* glu_gate,
                            void* stream);

/* y = dequant(Wq, scale) @ x for symmetric INT8 weights.
 * Wq: int8 [N, K]; scale: fp32 [N or 1, num_groups]; scale_row_stride = 0
 * broadcasts one scale row (per-tensor) else num_groups.  num_groups is 1
 * (per-tensor / per-channel) or ceil(K/group_size) with group_size % 4 == 0.
 * Replaces: csrc/bindings.cpp:239-262, csrc/kernels/gemv_w8a16.cu:22-70. */
int soinfer_gemv_w8a16(const int8_t* Wq, const float* scale, const soinfer_half* x, soinfer_half* y,
                       int64_t N, int64_t K, int64_t group_size, int64_t num_groups,
                       int64_t scale_row_stride, void* stream);

/* ------------------------------------------------------------ selection --- */

/* Reference-compatible DIP channel selector ("ref mode", bit-exact with the
 * reference): lo = 0, hi = max(0, max v) + 1e-3f, 24 fp32 bisection steps
 * mid = 0.5f*(lo+hi) keeping count(v >= lo) >= k, tau = lo; out_idx receives
 * the first min(k, count(v >= tau)) indices i in ascending order with
 * v[i] >= tau and *out_count the number written.  Entries of out_idx past
 * *out_count are set to -1.  abs_g: fp32 [n] device; out_idx: int32 [k];
 * out_count: int32 [1].  Requires 1 <= k <= n.  Values are expected to be
 * non-negative magnitudes (not checked, as in the reference).
 * Replaces: csrc/bindings.cpp:507-518, csrc/kernels/topk_select.cu:10-102. */
int soinfer_topk_threshold_select(const float* abs_g, int64_t n, int64_t k, int32_t* out_idx,
                                  int32_t* out_count, void* stream);

/* soinfer_topk_threshold_select on |gate| of an fp16 gate vector: the values
 * selected on are exactly the fp32 |float(gate[i])| the reference computes
 * with gate.float().abs() before selecting (runtime/generate.py:276-278).
 * No reference counterpart (fuses that conversion into the selector). */
int soinfer_topk_threshold_select_abs_f16(const soinfer_half* gate, int64_t n, int64_t k,
                                          int32_t* out_idx, int32_t* out_count, void* stream);

/* Exact top-k ("exact mode"): the k largest values, ties at the k-th value
 * broken by the lower index, written in ascending index order; *out_count = k.
 * NaN ranks below every number.  Same buffers as the ref-mode selector.
 * No reference counterpart (the reference selector is threshold-based). */
int soinfer_topk_select_exact(const float* abs_g, int64_t n, int64_t k, int32_t* out_idx,
                              int32_t* out_count, void* stream);

/* Cache descriptors: desc[j] = slot_of[sel[j]] when >= 0 (hot-cache hit),
 * else (m | 0x80000000) where m is the miss position; miss[m] = sel[j].
 * Misses are compacted in ascending j order (deterministic; the reference's
 * atomic order is arbitrary).  *miss_count = number of misses.
 * sel: int32 [k], each in [0, I); slot_of: int32 [I].
 * Replaces: csrc/bindings.cpp:341-359, csrc/kernels/gemv_dip_fused.cu:17-42. */
int soinfer_build_dip_descriptors(const int32_t* sel, int64_t k, const int32_t* slot_of, int64_t I,
                                  int32_t* desc, int32_t* miss, int32_t* miss_count, void* stream);

/* ------------------------------------------------- DIP fused GEMVs ------- */

/* 'Up' direction of cache-or-stream DIP: y[j] = row j of the selected matrix
 * dotted with x, where row j lives in cache (desc[j] >= 0: cache row
 * desc[j]) or in staging (desc[j] < 0: staging row desc[j] & 0x7fffffff).
 * Bit-identical to soinfer_gemv_w4a16_group_lop3 on the same logical rows.
 * cache_Wq: uint8 [C, ceil(K/8)*4]; staging_Wq: uint8 [M, ...]; scales fp32
 * [C|M, num_groups]; desc: int32 [k]; x: fp16 [K]; y: fp16 [k].
 * Replaces: csrc/bindings.cpp:388-408, csrc/kernels/gemv_dip_fused.cu:48-102. */
int soinfer_gemv_dip_fused_up(const uint8_t* cache_Wq, const float* cache_scale, int64_t C,
                              const uint8_t* staging_Wq, const float* staging_scale, int64_t M,
                              const int32_t* desc, int64_t k, const soinfer_half* x, soinfer_half* y,
                              int64_t K, int64_t group_size, int64_t num_groups, void* stream);

/* fp16 GEMV: y[n] = fp16( sum_k W[n, k] * x[k] ), fp32 accumulation.  The
 * decode LM head.  W: fp16 [N, K] row-major (16-byte aligned), x: fp16 [K],
 * y: fp16 [N]; K % 8 == 0.
 * Replaces: csrc/bindings.cpp:201-208 (gemv_fp16_v3), csrc/kernels/gemv_fp16.cu:60-95. */
int soinfer_gemv_fp16(const soinfer_half* W, const soinfer_half* x, soinfer_half* y, int64_t N,
                      int64_t K, void* stream);

/* Bytes of zero-initialised workspace soinfer_gemv_fp16_argmax needs (left
 * zeroed on return). */
int64_t soinfer_lm_head_argmax_workspace_bytes(void);

/* soinfer_gemv_fp16 fused with the greedy token choice: *out_idx = the
 * argmax of the fp16 logits (lowest index among equal maxima, as
 * torch.argmax).  y may be NULL when the logits are not needed.
 * Replaces the reference's gemv_fp16_v3 + torch.argmax pair
 * (python/soinfer/runtime/generate.py:452-454). */
int soinfer_gemv_fp16_argmax(const soinfer_half* W, const soinfer_half* x, soinfer_half* y, int64_t N,
                             int64_t K, int32_t* out_idx, void* workspace, int64_t workspace_bytes,
                             void* stream);

/* Bytes of zero-initialised device workspace the sparse 'down' GEMVs need for
 * an output width H over k selected rows.  The kernels leave the workspace
 * zeroed again on return, so a caller allocates (and clears) it once and
 * reuses it for every call on one stream. */
int64_t soinfer_sparse_workspace_bytes(int64_t H, int64_t k);

/* 'Down' direction: y[c] = fp16( sum_{i<k} h[i] * scale[i, c/g] * q[i, c] )
 * over k selected (already gathered) rows of the transposed down_proj.
 * Wq_sel: uint8 [k, ceil(H/8)*4]; scale_sel: fp32 [k, num_groups];
 * h: fp16 [k]; y: fp16 [H].  Deterministic fixed-order reduction.
 * Replaces: csrc/bindings.cpp:311-339, csrc/kernels/gemv_sparse_accumulate.cu:10-47. */
int soinfer_gemv_w4a16_sparse_accumulate(const uint8_t* Wq_sel, const float* scale_sel,
                                         const soinfer_half* h, soinfer_half* y, int64_t H, int64_t k,
                                         int64_t group_size, int64_t num_groups, void* workspace,
                                         int64_t workspace_bytes, void* stream);

/* No-allocation form of soinfer_gemv_w4a16_sparse_accumulate (no reference
 * counterpart: the reference allocates its output and has no workspace).
 * Same arguments, results bit-identical, but the scratch is a per-device
 * static device array of 512 KiB instead of a caller workspace, for callers
 * that cannot hand over memory (e.g. a decode loop with no allocator at
 * hand).  Limits: soinfer_sparse_workspace_bytes(H, k) must fit in 512 KiB
 * (every shape up to H = 16384 needs ~0.3 MiB; larger ones return
 * SOINFER_ERR_INVALID_ARGUMENT); the scratch is shared, so two calls on one
 * device that overlap in time (different streams, or host threads) race on
 * it -- serialise them; the first call on each device does a one-time set-up
 * (symbol lookup and an async clear of the scratch's tickets on `stream`),
 * so make that call before capturing a stream into a CUDA graph. */
int soinfer_gemv_w4a16_sparse_accumulate_noalloc(const uint8_t* Wq_sel, const float* scale_sel,
                                                 const soinfer_half* h, soinfer_half* y, int64_t H,
                                                 int64_t k, int64_t group_size, int64_t num_groups,
                                                 void* stream);

/* Row-indirect form of the sparse 'down' GEMV over a resident transposed
 * matrix: row j of the sum is Wq_T[rows[j]] with scale_T[rows[j]].
 * Bit-identical to gathering those rows and calling
 * soinfer_gemv_w4a16_sparse_accumulate.  rows: int32 [k] in [0, I).
 * residual (optional, fp16 [H]): y = fp16(residual + fp16(sum)) -- the
 * layer's residual add (generate.py:310), equal to adding after the GEMV. */
int soinfer_gemv_w4a16_sparse_rows(const uint8_t* Wq_T, const float* scale_T, int64_t I,
                                   const int32_t* rows, const soinfer_half* h, soinfer_half* y,
                                   int64_t H, int64_t k, int64_t group_size, int64_t num_groups,
                                   void* workspace, int64_t workspace_bytes, const soinfer_half* residual,
                                   void* stream);

/* Cache-or-stream 'down' direction: same as the sparse accumulate with each
 * row resolved through desc (see soinfer_gemv_dip_fused_up).  Bit-identical
 * to soinfer_gemv_w4a16_sparse_accumulate on the same logical rows.
 * Replaces: csrc/bindings.cpp:410-432, csrc/kernels/gemv_dip_fused.cu:116-164. */
int soinfer_gemv_dip_fused_down(const uint8_t* cache_Wq, const float* cache_scale, int64_t C,
                                const uint8_t* staging_Wq, const float* staging_scale, int64_t M,
                                const int32_t* desc, const soinfer_half* h, soinfer_half* y, int64_t H,
                                int64_t k, int64_t group_size, int64_t num_groups, void* workspace,
                                int64_t workspace_bytes, void* stream);

/* ------------------------------------------------------------- gathers --- */

/* Copies rows indices[0..k) of a pinned host matrix [num_rows, row_nbytes]
 * into pinned staging (host memcpy, multi-threaded for large k), then one
 * cudaMemcpyAsync of k*row_nbytes bytes to gpu_dst on `stream`.  Byte-exact.
 * indices: int64 host; staging: pinned host >= k*row_nbytes bytes.  The host
 * copy is complete on return; the H2D copy is asynchronous.
 * Replaces: csrc/bindings.cpp:538-549, csrc/kernels/gather_rows.cu:6-13. */
int soinfer_gather_rows_staged(const uint8_t* matrix, int64_t num_rows, int64_t row_nbytes,
                               const int64_t* indices, int64_t k, uint8_t* staging,
                               int64_t staging_bytes, uint8_t* gpu_dst, int64_t dst_bytes, void* stream);

/* One cudaMemcpyAsync per selected row straight from the pinned matrix.
 * Replaces: csrc/bindings.cpp:551-559, csrc/kernels/gather_rows.cu:15-21. */
int soinfer_gather_rows_naive(const uint8_t* matrix, int64_t num_rows, int64_t row_nbytes,
                              const int64_t* indices, int64_t k, uint8_t* gpu_dst, int64_t dst_bytes,
                              void* stream);

/* Device-driven gather: an SM kernel copies rows rows[0..k) (int32, device
 * memory) of `matrix` into gpu_dst.  `matrix` may be device memory or pinned
 * host memory mapped into the device address space (zero-copy over PCIe), so
 * the selection never has to visit the host.  No reference counterpart (the
 * reference gathers on the host after an index download, generate.py:282). */
int soinfer_gather_rows_device(const uint8_t* matrix, int64_t num_rows, int64_t row_nbytes,
                               const int32_t* rows, int64_t k, uint8_t* gpu_dst, void* stream);

/* One source of soinfer_gather_rows_device_multi. */
typedef struct soinfer_gather_src {
  const uint8_t* matrix; /* [num_rows, row_nbytes]: device or pinned host memory (zero-copy) */
  int64_t num_rows;
  int64_t row_nbytes;    /* a positive multiple of 4 */
  uint8_t* dst;          /* device [max_k, row_nbytes] */
} soinfer_gather_src;

/* Device-driven gather of the same rows from up to 4 matrices in one launch,
 * with the row count read from device memory: rows[j] of every source for
 * j < min(*count, max_k) (count NULL: max_k rows); rows at or past the count
 * are not touched.  This is the cache-aware DIP miss gather (the missed
 * channels' up_proj and down_proj_T rows and their scale rows) without the
 * host ever learning the miss count, so the step can be captured in a CUDA
 * graph.  Replaces runtime/generate.py:376-388 of the reference (the
 * miss-count download, then gather_rows_staged per matrix). */
int soinfer_gather_rows_device_multi(const soinfer_gather_src* srcs, int32_t num_srcs, const int32_t* rows,
                                     const int32_t* count, int64_t max_k, void* stream);

/* ---------------------------------------------- attention-side glue ------ */

/* out[r, :] = fp16( x[r,:] * rsqrt(mean(x[r,:]^2) + eps) * weight ), fp32 math.
 * x, out: fp16 [rows, hidden]; weight: fp16 [hidden]; hidden even.
 * Replaces: csrc/bindings.cpp:141-152, csrc/kernels/rmsnorm.cu:9-48. */
int soinfer_rmsnorm(const soinfer_half* x, const soinfer_half* weight, soinfer_half* out, int64_t rows,
                    int64_t hidden, float eps, void* stream);

/* Rotate-half RoPE in place on x: fp16 [num_heads, head_dim]; cos/sin: fp32
 * [head_dim/2].  Replaces: csrc/bindings.cpp:490-505, csrc/kernels/rope.cu:5-25. */
int soinfer_rope_apply(soinfer_half* x, const float* cos_vals, const float* sin_vals, int64_t num_heads,
                       int64_t head_dim, void* stream);

/* k_cache/v_cache: fp16 [num_kv_heads, max_seq_len, head_dim]; k_new/v_new:
 * fp16 [num_kv_heads, head_dim] written at position pos (0 <= pos < max_seq_len).
 * Replaces: csrc/bindings.cpp:450-466, csrc/kernels/kv_cache.cu:7-27. */
int soinfer_kv_cache_append(soinfer_half* k_cache, soinfer_half* v_cache, const soinfer_half* k_new,
                            const soinfer_half* v_new, int64_t num_kv_heads, int64_t max_seq_len,
                            int64_t head_dim, int64_t pos, void* stream);

/* Bytes of device workspace soinfer_decode_attention needs (split-KV partials). */
int64_t soinfer_decode_attention_workspace_bytes(int64_t num_q_heads, int64_t max_seq_len,
                                                 int64_t head_dim);

/* Single-query GQA attention: q fp16 [NQ, hd]; caches fp16 [NKV, max_seq, hd];
 * query head h reads kv head h / (NQ/NKV); scale 1/sqrt(hd); softmax in fp32
 * over positions [0, cur_len); out fp16 [NQ, hd].  head_dim must be a
 * multiple of 8 and at most 256.
 * Replaces: csrc/bindings.cpp:468-488, csrc/kernels/decode_attention.cu:17-63. */
int soinfer_decode_attention(const soinfer_half* q, const soinfer_half* k_cache,
                             const soinfer_half* v_cache, soinfer_half* out, int64_t num_q_heads,
                             int64_t num_kv_heads, int64_t max_seq_len, int64_t head_dim, int64_t cur_len,
                             void* workspace, int64_t workspace_bytes, void* stream);

/* Fused decode-layer glue (no reference counterpart; each equals the
 * reference's unfused composition).
 * add_rmsnorm: sum_out = fp16(x + x2) (fp32 add, one rounding: the fp16
 * residual add), out = rmsnorm(sum_out, weight) as soinfer_rmsnorm;
 * bit-identical to the two ops.  x, x2, out, sum_out: fp16 [rows, hidden].
 * swiglu: out[i] = fp16(silu(float(g_i)) * float(up[i])) with g_i = gate[idx[i]]
 * (idx may be NULL: gate[i]); silu(x) = x / (1 + exp(-x)) in fp32 -- the
 * reference's (F.silu(g.float()) * u.float()).half(), generate.py:300-302.
 * head_norm_rope: after the q / k / v GEMVs of one token: RMSNorm of every q
 * and k head (q_norm / k_norm weights, fp16 [head_dim]), rotate-half RoPE of
 * the normalised values (q rewritten in place), k and v appended to the
 * caches at pos -- or, when pos_dev is not NULL, at *pos_dev with cos / sin
 * tables [table_rows, head_dim/2] indexed by it (out-of-range: nothing
 * written).  q: fp16 [num_q_heads, head_dim]; k, v: [num_kv_heads, head_dim];
 * head_dim even and <= 256.  Replaces the reference's qk_norm x2, rope x2 and
 * kv_cache_append sequence (generate.py:243-252). */
int soinfer_add_rmsnorm(const soinfer_half* x, const soinfer_half* x2, const soinfer_half* weight,
                        soinfer_half* out, soinfer_half* sum_out, int64_t rows, int64_t hidden,
                        float eps, void* stream);
int soinfer_swiglu(const soinfer_half* gate, const soinfer_half* up, const int32_t* idx,
                   soinfer_half* out, int64_t n, void* stream);
int soinfer_head_norm_rope(soinfer_half* q, const soinfer_half* k, const soinfer_half* v,
                           const soinfer_half* q_norm, const soinfer_half* k_norm,
                           const float* cos_vals, const float* sin_vals, int64_t table_rows,
                           soinfer_half* k_cache, soinfer_half* v_cache, int64_t num_q_heads,
                           int64_t num_kv_heads, int64_t head_dim, int64_t max_seq_len, int64_t pos,
                           const int32_t* pos_dev, float eps, void* stream);

/* Device-position forms (no reference counterpart): the same kernels with the
 * token position read from device memory when they run (*pos_dev), so a whole
 * decode step -- its position advanced by a device op -- can be captured in a
 * CUDA graph and replayed.  rope: cos_table / sin_table fp32
 * [table_rows, head_dim/2], row *pos_dev (positions outside the table: no
 * change).  kv append: written at *pos_dev (outside [0, max_seq_len): no
 * write).  attention: over positions [0, *pos_dev + 1), clamped to
 * [1, max_seq_len]; the launch is planned for max_seq_len. */
int soinfer_rope_apply_at(soinfer_half* x, const float* cos_table, const float* sin_table,
                          int64_t table_rows, int64_t num_heads, int64_t head_dim,
                          const int32_t* pos_dev, void* stream);
int soinfer_kv_cache_append_at(soinfer_half* k_cache, soinfer_half* v_cache, const soinfer_half* k_new,
                               const soinfer_half* v_new, int64_t num_kv_heads, int64_t max_seq_len,
                               int64_t head_dim, const int32_t* pos_dev, void* stream);
int soinfer_decode_attention_at(const soinfer_half* q, const soinfer_half* k_cache,
                                const soinfer_half* v_cache, soinfer_half* out, int64_t num_q_heads,
                                int64_t num_kv_heads, int64_t max_seq_len, int64_t head_dim,
                                const int32_t* pos_dev, void* workspace, int64_t workspace_bytes,
                                void* stream);

/* The graph decode step's token bookkeeping on the device (no reference
 * counterpart: the reference embeds and appends the token on the host,
 * python/soinfer/runtime/generate.py:446-458).  embed: x [hidden] =
 * embed[ids[*pos_dev]] (fp16 [vocab, hidden]); a position outside
 * [0, ids_len) or a token id outside [0, vocab) writes nothing.  advance: once
 * the step's token is in *next (int32, e.g. the LM head's argmax),
 * ids[*pos_dev + 1] = *next unless *pos_dev + 1 < *prompt_len (a prompt token
 * stays), then *pos_dev += 1; nothing when *pos_dev + 1 is outside
 * [0, ids_len). */
int soinfer_decode_step_embed(const soinfer_half* embed, int64_t vocab, int64_t hidden, const int32_t* ids,
                              int64_t ids_len, const int32_t* pos_dev, soinfer_half* x, void* stream);
int soinfer_decode_step_advance(int32_t* ids, int64_t ids_len, int32_t* pos_dev, const int32_t* prompt_len,
                                const int32_t* next, void* stream);

/* Multi-token INT4 GEMM for batched decode (no reference counterpart; the
 * reference GEMV applied to M tokens): Y[m, 0:N] = dequant(W) X[m, 0:K] for
 * m < M <= 8, X fp16 with row stride ldx, Y fp16 with row stride ldy, the
 * weights / scales of soinfer_gemv_w4a16_group.  One pass over the weights:
 * the tensor-core MMA's 8 columns carry the M tokens (a long K whose X does
 * not fit in shared memory is staged K-segment by K-segment, same sums).
 * Shapes outside the one-pass kernel (K or group size not multiples of 128,
 * scale rows not 16-byte multiples, more shared memory than an SM has) run
 * the single-token GEMV per row. */
int soinfer_gemm_w4a16(const uint8_t* Wq_packed, const float* scale, const soinfer_half* X, int64_t ldx,
                       soinfer_half* Y, int64_t ldy, int64_t M, int64_t N, int64_t K, int64_t group_size,
                       int64_t num_groups, void* stream);

/* One task of soinfer_gemm_w4a16_batch: Y[m, 0:N] = dequant(Wq) X[m, 0:K]
 * for the batch's M tokens (X row stride ldx, Y row stride ldy, elements). */
typedef struct soinfer_gemm_task {
  const uint8_t* Wq;
  const float* scale;
  const soinfer_half* X;
  soinfer_half* Y;
  int64_t N, K, group_size, num_groups, ldx, ldy;
} soinfer_gemm_task;

/* Bytes of zero-initialised device workspace soinfer_gemm_w4a16_batch needs
 * (a work ticket and an exit count; left zeroed on return). */
int64_t soinfer_gemm_batch_workspace_bytes(void);

/* Batched decode of M <= 8 tokens over a list of up to 256 independent INT4
 * matrices in ONE launch: every task's Y = X W^T as in soinfer_gemm_w4a16,
 * with the weights of all tasks streamed by the same kernel as
 * soinfer_gemv_w4a16_batch's independent GEMVs (a warp per 48-row unit over
 * the full K, the M tokens in the tensor-core MMA's columns).  No task may
 * read another's Y.  Needs K and group_size multiples of 128, 16-byte aligned
 * Wq and X rows (ldx * 2 % 16 == 0), 4-byte aligned scales; otherwise
 * SOINFER_ERR_UNSUPPORTED.  No reference counterpart (the reference decodes
 * one token at a time, runtime/generate.py:429-463). */
int soinfer_gemm_w4a16_batch(const soinfer_gemm_task* tasks, int64_t num_tasks, int64_t M, void* workspace,
                             int64_t workspace_bytes, void* stream);

/* One decoder layer of soinfer_decode_layers_fused: the packed INT4 weights
 * (group size 128, scales [N, K/128]) of q, k, v, o, gate, up, down in that
 * order, the four RMSNorm weights and the layer's KV cache
 * ([num_kv_heads, max_seq, 128] fp16 each). */
typedef struct soinfer_fused_layer {
  const uint8_t* Wq[7];
  const float* scale[7];
  const soinfer_half* input_norm;
  const soinfer_half* post_norm;
  const soinfer_half* q_norm;
  const soinfer_half* k_norm;
  soinfer_half* k_cache;
  soinfer_half* v_cache;
} soinfer_fused_layer;

/* Bytes of device workspace soinfer_decode_layers_fused needs (its first 256
 * bytes must be zero on the first call; every call leaves them zero). */
int64_t soinfer_decode_fused_workspace_bytes(int64_t hidden, int64_t intermediate, int64_t num_heads,
                                             int64_t num_kv_heads, int64_t head_dim);

/* Every decoder layer of one batch-1 decode step in ONE cooperative launch
 * (no reference counterpart: the reference runs the layer as separate kernels,
 * python/soinfer/runtime/generate.py:141-182, dense streaming layer).  x
 * [hidden] holds the step's input embedding and receives the last layer's
 * output; the token's position is read from pos_dev (device int32) when the
 * kernel runs (CUDA-graph capturable); each layer appends its K / V row at
 * that position.  Per layer: RMSNorm -> q/k/v -> q/k head norm + RoPE (tables
 * [max_seq, 64] fp32) -> GQA attention -> o + residual -> RMSNorm -> gate/up
 * -> SwiGLU -> down + residual, bit-identical to the per-kernel path
 * (soinfer_gemv_w4a16_batch with its prologue / epilogues,
 * soinfer_head_norm_rope, soinfer_decode_attention_at).  Needs head_dim 128,
 * num_heads / num_kv_heads in {1, 2, 4}, hidden and intermediate multiples of
 * 128, group size 128, at most 64 layers, 16-byte aligned weight rows;
 * otherwise SOINFER_ERR_UNSUPPORTED.  Grid barriers are bounded (1 s): a wait
 * that runs out sets a soinfer_device_errors bit. */
int soinfer_decode_layers_fused(const soinfer_fused_layer* layers, int64_t num_layers, int64_t hidden,
                                int64_t intermediate, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                                int64_t group_size, int64_t max_seq, float eps, const float* cos_table,
                                const float* sin_table, const int32_t* pos_dev, soinfer_half* x, void* workspace,
                                int64_t workspace_bytes, void* stream);

/* Load-time INT4 quantization + packing on the GPU (reference
 * python/soinfer/quant/formats.py:77-110 with calibrate.min_max:22-27 and
 * quant/pack.py:31-69): w [N, K] with row stride ld (dtype 0 fp32, 1 fp16,
 * 2 bf16) -> packed uint8 [N, ceil(Kp/8)*4] (AWQ nibble order) and scale fp32
 * [N, Kp/group_size], Kp = K rounded up to group_size (a power of two in
 * [8, 256]); scale = max(amax/7, FLT_MIN), q = clamp(rint(w/scale), -7, 7)
 * with IEEE division -- bit-exact with the reference's CPU quantizer, in one
 * pass over the weights. */
int soinfer_quantize_pack_int4(const void* w, int32_t dtype, int64_t N, int64_t K, int64_t ld,
                               int64_t group_size, uint8_t* packed, float* scale, void* stream);

/* ---- Tensor-parallel exchange over peer memory (no reference counterpart:
 * the reference runs on one GPU; this is the row-parallel all-reduce, the
 * all-gather and the greedy-token agreement of tensor-parallel decode across
 * the GPUs of one node, one process per GPU).
 *
 * Each rank creates one exchange buffer (soinfer_peer_buffer_create: device
 * memory, zeroed, plus a CUDA IPC handle of SOINFER_IPC_HANDLE_BYTES bytes),
 * hands the handle to the other ranks (any host channel), and maps theirs
 * (soinfer_peer_buffer_open).  A soinfer_peer_set lists every rank's buffer as
 * mapped in this process (base[rank] = its own), the rank, the world size
 * (1..8) and the inbox slot size (a multiple of 16 bytes, at least the
 * largest payload).  Kernels store straight into the peers' buffers over
 * NVLink, then signal them with system-scope release flags; every wait is
 * bounded (1 s) and a timeout raises a device error bit
 * (soinfer_device_errors) instead of hanging.  All ranks must issue the same
 * sequence of exchange calls on their streams.  A timed-out exchange leaves
 * the ranks out of step: after the error bit (bit 1) every rank calls
 * soinfer_peer_buffer_reset on its own buffer between steps, with a host
 * barrier before and after, before the next exchange.
 *
 * allreduce_add_rmsnorm: out_sum = fp16(residual + fp16(sum over ranks of
 * partial)) (sum in fp32, rank order; residual may be NULL), and when
 * out_norm is not NULL out_norm = RMSNorm(out_sum) * weight (eps); n % 8 == 0.
 * partial == NULL: the partials were already pushed by
 * soinfer_gemv_w4a16_tp_partial, which computes the row-parallel INT4 GEMV
 * (same arguments and arithmetic as soinfer_gemv_w4a16_group_lop3) and stores
 * its fp16 rows into every rank's inbox instead of an output vector (K and
 * group_size multiples of 128, 16-byte aligned rows).
 * allgather: out [world * nbytes] = every rank's local [nbytes] in rank order
 * (nbytes % 16 == 0).
 * argmax: with a vocabulary-parallel LM head (rank r owns rows from offset),
 * out_idx int32 [1] = the global greedy token -- the largest fp16
 * logits[local_idx] over ranks, ties to the lowest global index (the rule of
 * soinfer_gemv_fp16_argmax). */
#define SOINFER_IPC_HANDLE_BYTES 64
#define SOINFER_MAX_PEERS 8
typedef struct soinfer_peer_set {
  void* base[SOINFER_MAX_PEERS];
  int32_t rank;
  int32_t world;
  int64_t slot_bytes;
} soinfer_peer_set;

int64_t soinfer_peer_buffer_bytes(int64_t slot_bytes, int32_t world);
int soinfer_peer_buffer_create(int64_t bytes, void** dptr, void* ipc_handle);
int soinfer_peer_buffer_open(const void* ipc_handle, void** dptr);
int soinfer_peer_buffer_close(void* dptr);
int soinfer_peer_buffer_destroy(void* dptr);
/* Zeroes this rank's exchange header (flags, exchange count, ticket) on
 * `stream`: the recovery step after a peer timeout (see above). */
int soinfer_peer_buffer_reset(void* dptr, void* stream);
int soinfer_tp_allreduce_add_rmsnorm(const soinfer_peer_set* peers, const soinfer_half* partial,
                                     const soinfer_half* residual, const soinfer_half* weight,
                                     soinfer_half* out_sum, soinfer_half* out_norm, int64_t n, float eps,
                                     void* stream);
int soinfer_gemv_w4a16_tp_partial(const soinfer_peer_set* peers, const uint8_t* Wq_packed,
                                  const float* scale, const soinfer_half* x, int64_t N, int64_t K,
                                  int64_t group_size, int64_t num_groups, void* stream);
/* Tensor-parallel form of soinfer_gemv_w4a16_batch: at most one task may have
 * y == NULL (no glu_gate / residual); its rows go to every rank's inbox as
 * with soinfer_gemv_w4a16_tp_partial, signalled when the whole launch is done.
 * Finish with soinfer_tp_allreduce_add_rmsnorm(partial = NULL). */
int soinfer_gemv_w4a16_batch_tp(const soinfer_peer_set* peers, const soinfer_gemv_task* tasks,
                                int64_t num_tasks, void* workspace, int64_t workspace_bytes, void* stream);
int soinfer_tp_allgather(const soinfer_peer_set* peers, const void* local, int64_t nbytes, void* out,
                         void* stream);
int soinfer_tp_argmax(const soinfer_peer_set* peers, const soinfer_half* logits, const int32_t* local_idx,
                      int64_t offset, int32_t* out_idx, void* stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* SOINFER_B200_H_ */
