// Internal launcher interface between the C ABI (capi.cu) and the kernels.
// Launchers validate nothing (capi.cu does) and return the launch status.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace soinfer {

// How a logical output row of an INT4 GEMV finds its packed bytes and scales.
enum class RowMode : int { kPlain = 0, kIndexed = 1, kDesc = 2 };

struct RowSource {
  const uint8_t* W = nullptr;   // plain rows / indexed matrix / hot-cache rows
  const float* S = nullptr;
  const uint8_t* W2 = nullptr;  // staging rows (descriptor mode)
  const float* S2 = nullptr;
  const int32_t* idx = nullptr; // row indices (indexed) or descriptors (desc)
  int64_t rows1 = 0;            // rows available behind W/S (bounds clamp)
  int64_t rows2 = 0;            // rows available behind W2/S2
  int64_t row_bytes = 0;        // packed bytes per row = ceil(K/8)*4
  int64_t num_groups = 0;       // scale columns per row
};

// Tensor-parallel peer exchange (peer.cuh has the buffer layout and protocol).
constexpr int kMaxPeers = 8;
constexpr int64_t kPeerHeaderBytes = 256;
struct PeerSet {
  uint8_t* base[kMaxPeers];  // every rank's exchange buffer as mapped in this process (own at [rank])
  int rank, world;
  int64_t slot_bytes;        // one inbox slot (multiple of 16)
};
inline int64_t peer_buffer_bytes(int64_t slot_bytes, int world) {
  return kPeerHeaderBytes + 2 * (int64_t)world * slot_bytes;
}

struct LaunchOpts {
  bool pdl = false;  // programmatic dependent launch (weights not produced by the previous kernel)
  // Optional output epilogues (the bulk INT4 GEMV / the sparse down GEMV):
  const half* glu = nullptr;    // y[r] = fp16(silu(glu[idx[r]]) * fp16(dot))  (indexed rows: SwiGLU of DIP)
  const half* resid = nullptr;  // y[c] = fp16(resid[c] + fp16(sum))           (sparse down: the residual add)
};

// y[r] = dot(row r of src, x) for r < nrows (INT4, AWQ order, fp32 accumulation).
cudaError_t launch_gemv_w4(RowMode mode, const RowSource& src, const half* x, half* y, int64_t nrows,
                           int64_t K, int64_t group_size, cudaStream_t stream, LaunchOpts opts = {});

// Multi-token INT4 GEMM (gemm_w4.cu): Y[m, :] = W X[m, :] for m < M <= 8 in one pass over W.
// plan_gemm_w4: whether the one-pass kernel takes the shape (else run per token).
bool plan_gemm_w4(int64_t M, int64_t N, int64_t K, int64_t group_size, int64_t G);
cudaError_t launch_gemm_w4(const uint8_t* W, const float* S, const half* X, int64_t ldx, half* Y, int64_t ldy,
                           int64_t M, int64_t N, int64_t K, int64_t group_size, int64_t G, cudaStream_t stream);
cudaError_t read_and_clear_gemm_w4_error(int* out);

// Group-wise INT4 quantization + AWQ packing of w [N, K] (row stride ld; dtype 0 fp32, 1 fp16,
// 2 bf16): packed uint8 [N, ceil(Kp/8)*4], scale fp32 [N, Kp/g], Kp = K rounded up to g
// (g a power of two in [8, 256]).  Bit-exact with the reference's CPU torch quantizer.
cudaError_t launch_quantize_pack_int4(const void* w, int dtype, int64_t N, int64_t K, int64_t ld, int64_t group_size,
                                      uint8_t* packed, float* scale, cudaStream_t stream);

// Reads and clears the INT4 GEMV module's device error bits (DeviceError).
cudaError_t read_and_clear_gemv_w4_error(int* out);

// Row-parallel INT4 GEMV whose output rows go straight into every rank's
// inbox slot of the next exchange (peer stores over NVLink); the last CTA
// signals the exchange.  Finish it with launch_tp_allreduce_norm(partial =
// nullptr).  Needs the bulk-path layout (K, group size multiples of 128,
// 16-byte aligned rows); returns cudaErrorNotSupported otherwise.
cudaError_t launch_gemv_w4_peer(const RowSource& src, const half* x, int64_t nrows, int64_t K, int64_t group_size,
                                const PeerSet& ps, cudaStream_t stream);

// Exchanges (tp_comm.cu), one CTA each:
// all-reduce of fp16 [n] partials (summed in fp32 in rank order, rounded
// once), then out_sum = fp16(residual + sum) (residual optional) and, if
// out_norm, out_norm = rmsnorm(out_sum) * w.  partial == nullptr: the data was
// already pushed and signalled by launch_gemv_w4_peer.
cudaError_t launch_tp_allreduce_norm(const PeerSet& ps, const half* partial, const half* residual, const half* w,
                                     half* out_sum, half* out_norm, int64_t n, float eps, cudaStream_t stream);
// out [world * nbytes] = every rank's `local` [nbytes] in rank order.
cudaError_t launch_tp_allgather(const PeerSet& ps, const void* local, int64_t nbytes, void* out, cudaStream_t stream);
// Global greedy token of a vocabulary-parallel LM head: every rank's
// (logits[local_idx], local_idx + offset), the largest fp16 logit, ties to the
// lowest global index; out_idx int32 [1].
cudaError_t launch_tp_argmax(const PeerSet& ps, const half* logits, const int32_t* local_idx, int64_t offset,
                             int32_t* out_idx, cudaStream_t stream);
cudaError_t read_and_clear_tp_error(int* out);

// Persistent batched INT4 GEMV (gemv_batch.cu).  Tasks run in order; a task
// with dep >= 0 reads x only after every CTA finished task `dep`.
struct GemvBatchTask {
  const uint8_t* W;
  const float* S;
  const half* x;
  half* y;
  const half* resid;  // optional epilogue: y = fp16(resid + fp16(dot))
  const half* glu;    // optional epilogue: y = fp16(silu(glu) * fp16(dot)), applied before resid
  const half* norm_w; // optional prologue: x -> fp16(x * rsqrt(mean(x^2) + eps) * norm_w) in shared memory
  half* norm_out;     // with the prologue: CTA 0 also writes the normalised x here (for later kernels)
  int N, K, G, cpg, dep;
  // filled by plan_gemv_batch: rows per CTA, 16-row tiles per item, publish (a later task depends on it),
  // ks / nsegs (K split into segments of ks 128-chunks when a 16-row tile is too long for one item),
  // scale_plain (scale rows staged by plain loads: not 16-byte rows, or segmented)
  int rows_per_cta, tiles_per_item, publish, ks, nsegs, scale_plain;
  int peer;           // y == nullptr: rows go to every rank's exchange inbox (PeerSet), the last CTA signals
  float eps;
};
constexpr int kMaxBatchTasks = 256;
constexpr int kSmallBatchTasks = 8;  // decode-layer batches: a small kernel-parameter block launches faster
template <int MaxTasks>
struct GemvBatchParamsT {
  int num, grid, x_bytes, ring_bytes, smem_bytes;
  int any_cp_async;  // some task stages scales with cp.async (proxy fence before later bulk copies)
  int norm_bytes;    // shared scratch for the norm weights of prologue tasks (0: none)
  int need_counters; // some task is depended on or sends to peers: count CTAs / reset at the end
  PeerSet peers;  // used by a peer task (at most one per batch)
  GemvBatchTask tasks[MaxTasks];
};
using GemvBatchParams = GemvBatchParamsT<kMaxBatchTasks>;
int64_t gemv_batch_workspace_bytes(int64_t num_tasks);
// Fills the derived fields; false when the batch needs the per-task fallback.
bool plan_gemv_batch(GemvBatchParams& B, int sms);
cudaError_t launch_gemv_batch(const GemvBatchParams& B, int* counters, cudaStream_t stream);
cudaError_t read_and_clear_gemv_batch_error(int* out);

// Streaming INT4 GEMV over a list of tasks (gemv_stream.cu): no epilogue, K
// and group size multiples of 128; a task may wait for an earlier one (dep:
// its x is that task's y), in which case its units start once every unit of
// that task is stored.
struct GemvStreamTask {
  const uint8_t* W;
  const float* S;
  const half* x;  // [m, K], row stride ldx (m tokens)
  half* y;        // [m, N], row stride ldy
  int N, K, G, cpg;
  int ldx, ldy;   // token strides in elements (multi-token form)
  int dep;        // index of the task this one waits for, or -1 (caller order; plan_gemv_stream remaps it)
  int ubegin;     // filled by plan_gemv_stream: first unit of the task
  int dneed;      // filled by plan_gemv_stream: units of the dep task (its completion count)
  int publish;    // filled by plan_gemv_stream: 1 if another task waits for this one
};
template <int MaxTasks>
struct GemvStreamParamsT {
  int num, grid, total_units, total_warps;
  int m;  // tokens per task: 1 (GEMV) or 2..8 (every task multiplies m token rows)
  GemvStreamTask tasks[MaxTasks];
};
using GemvStreamParams = GemvStreamParamsT<kMaxBatchTasks>;
#ifndef SOINFER_STREAM_TILES
#define SOINFER_STREAM_TILES 3
#endif
#ifndef SOINFER_STREAM_STAGES
#define SOINFER_STREAM_STAGES 2
#endif
#ifndef SOINFER_STREAM_WARPS
#define SOINFER_STREAM_WARPS 16
#endif
constexpr int kStreamTiles = SOINFER_STREAM_TILES;    // 16-row tiles per unit
constexpr int kStreamStages = SOINFER_STREAM_STAGES;  // chunks in flight per warp
constexpr int kStreamWarps = SOINFER_STREAM_WARPS;    // warps per CTA (one CTA per SM)
// Zeroed workspace bytes for num_tasks tasks (a unit ticket, an exit count and
// one completion count per task; left zeroed on return).
int64_t gemv_stream_workspace_bytes(int64_t num_tasks);
// Orders the tasks (dependency level, then decreasing K), fills the unit
// offsets and remaps dep to the new order; false if the shape is not served.
bool plan_gemv_stream(GemvStreamParams& B, int sms);
cudaError_t launch_gemv_stream(const GemvStreamParams& B, int* ctr, cudaStream_t stream);
cudaError_t read_and_clear_gemv_stream_error(int* out);

// INT8 GEMV (per-tensor / per-channel / grouped scales).
cudaError_t launch_gemv_w8(const int8_t* Wq, const float* scale, const half* x, half* y, int64_t N,
                           int64_t K, int64_t group_size, int64_t num_groups, int64_t scale_row_stride,
                           cudaStream_t stream, LaunchOpts opts = {});

// Sparse 'down' accumulate: y[c] = sum_j h[j] * scale(j, c/g) * q(j, c).
int64_t sparse_workspace_bytes(int64_t H, int64_t k);
// Per-device static scratch usable as the sparse workspace (no allocation):
// its size, and its address on the current device (first call per device
// resolves the symbol and clears the tickets on `stream`).
int64_t sparse_static_scratch_bytes();
cudaError_t sparse_static_scratch(void** scratch, cudaStream_t stream);
cudaError_t launch_sparse_down(RowMode mode, const RowSource& src, const half* h, half* y, int64_t H,
                               int64_t k, int64_t group_size, void* workspace, cudaStream_t stream,
                               LaunchOpts opts = {});

// Selectors.
cudaError_t launch_topk(bool exact, const float* v, int64_t n, int64_t k, int32_t* out_idx,
                        int32_t* out_count, cudaStream_t stream);
cudaError_t launch_build_descriptors(const int32_t* sel, int64_t k, const int32_t* slot_of, int64_t I,
                                     int32_t* desc, int32_t* miss, int32_t* miss_count, cudaStream_t stream);

// Gathers.
// Multi-source device gather (glue.cu): rows rows[0 .. min(*count, max_k)) of
// up to kMaxGatherSrc matrices into their destinations (count NULL: max_k rows).
constexpr int kMaxGatherSrc = 4;
struct GatherSrc {
  const uint8_t* matrix;
  int64_t num_rows, row_nbytes;
  uint8_t* dst;
  int vec16;  // 16-byte pieces (rows, matrix and dst 16-byte aligned) or 4-byte pieces
};
struct GatherMulti {
  GatherSrc src[kMaxGatherSrc];
  int num;
  const int32_t* rows;
  const int32_t* count;
  int64_t max_k;
};
cudaError_t launch_gather_multi(const GatherMulti& P, cudaStream_t stream);
cudaError_t launch_gather_rows_device(const uint8_t* matrix, int64_t num_rows, int64_t row_nbytes,
                                      const int32_t* rows, int64_t k, uint8_t* dst, cudaStream_t stream);

// fp16 GEMV (LM head) and the fused greedy argmax (lm_head.cu).  The argmax
// workspace (lm_head_argmax_workspace_bytes, zero-initialised) is left zeroed.
cudaError_t launch_gemv_fp16(const half* W, const half* x, half* y, int64_t N, int64_t K, cudaStream_t stream);
int64_t lm_head_argmax_workspace_bytes();
cudaError_t launch_gemv_fp16_argmax(const half* W, const half* x, half* y, int64_t N, int64_t K, void* workspace,
                                    int32_t* out_idx, cudaStream_t stream);

// Attention-side glue.
cudaError_t launch_rmsnorm(const half* x, const half* w, half* out, int64_t rows, int64_t hidden, float eps,
                           cudaStream_t stream);
cudaError_t launch_rope(half* x, const float* cos_v, const float* sin_v, int64_t heads, int64_t head_dim,
                        cudaStream_t stream);
cudaError_t launch_kv_append(half* kc, half* vc, const half* kn, const half* vn, int64_t nkv, int64_t max_seq,
                             int64_t hd, int64_t pos, cudaStream_t stream);
// Fused decode glue: residual add + RMSNorm (sum_out = fp16(x + x2), out =
// rmsnorm(sum_out), bit-identical to the two ops); SwiGLU (optionally over
// gate[idx[i]]); per-head q / k RMSNorm + RoPE + KV append (head_dim <= 256).
cudaError_t launch_add_rmsnorm(const half* x, const half* x2, const half* w, half* out, half* sum_out, int64_t rows,
                               int64_t hidden, float eps, cudaStream_t stream);
cudaError_t launch_swiglu(const half* gate, const half* up, const int32_t* idx, half* out, int64_t n,
                          cudaStream_t stream);
// out = fp16(float(a) + float(b)) elementwise (the fp16 tensor add).
cudaError_t launch_add_half(const half* a, const half* b, half* out, int64_t n, cudaStream_t stream);
cudaError_t launch_head_norm_rope(half* q, const half* k, const half* v, const half* qw, const half* kw,
                                  const float* cv, const float* sv, half* kc, half* vc, int64_t nq, int64_t nkv,
                                  int64_t hd, int64_t max_seq, int64_t pos, const int32_t* pos_dev,
                                  int64_t table_rows, float eps, cudaStream_t stream);
cudaError_t launch_topk_abs_half(bool exact, const half* v, int64_t n, int64_t k, int32_t* out_idx,
                                 int32_t* out_count, cudaStream_t stream);

// Device-position forms (CUDA-graph capturable decode step): the position is
// read from device memory when the kernel runs.
cudaError_t launch_rope_at(half* x, const float* cos_table, const float* sin_table, int64_t table_rows, int64_t heads,
                           int64_t head_dim, const int32_t* pos_dev, cudaStream_t stream);
cudaError_t launch_kv_append_at(half* kc, half* vc, const half* kn, const half* vn, int64_t nkv, int64_t max_seq,
                                int64_t hd, const int32_t* pos_dev, cudaStream_t stream);
// The graph decode step's embedding lookup and state advance (glue.cu).
cudaError_t launch_step_embed(const half* embed, int64_t vocab, int64_t H, const int32_t* ids, int64_t ids_len,
                              const int32_t* pos_dev, half* x, cudaStream_t stream);
cudaError_t launch_step_advance(int32_t* ids, int64_t ids_len, int32_t* pos_dev, const int32_t* prompt_len,
                                const int32_t* next, cudaStream_t stream);
int64_t attention_workspace_bytes(int64_t nq, int64_t max_seq, int64_t hd);
cudaError_t launch_decode_attention_at(const half* q, const half* kc, const half* vc, half* out, int64_t nq,
                                       int64_t nkv, int64_t max_seq, int64_t hd, const int32_t* pos_dev,
                                       void* workspace, cudaStream_t stream);
cudaError_t launch_decode_attention(const half* q, const half* kc, const half* vc, half* out, int64_t nq,
                                    int64_t nkv, int64_t max_seq, int64_t hd, int64_t cur_len, void* workspace,
                                    cudaStream_t stream);

// Fused dense decode step (decode_fused.cu): every decoder layer of a batch-1
// Qwen3-style model with HBM-resident INT4 weights (group size 128) in one
// cooperative launch, phases separated by grid barriers.
constexpr int kFusedMaxLayers = 64;
struct FusedLayer {
  const uint8_t* w[7];  // packed rows of q, k, v, o, gate, up, down
  const float* s[7];    // their scales [N, K / 128]
  const half* in_norm;
  const half* post_norm;
  const half* q_norm;
  const half* k_norm;
  half* kc;             // [NKV, max_seq, HD]
  half* vc;
};
struct FusedDecodeParams {
  int layers, H, I, NQ, NKV, HD;
  int cap;    // attention splits per kv head at most (the split kernel's layout)
  int lmax;   // score-row stride: positions per split at most
  int64_t max_seq;
  float eps, scale_log2;
  const float* cos_t;  // [max_seq, HD / 2]
  const float* sin_t;
  const int32_t* pos;  // the token's position (device)
  half* x;             // [H] hidden state: layer 0's input, the last layer's output
  half *q, *k, *v, *attn, *h2, *hid;  // scratch activations
  float* ws_acc;       // [NQ, 128 splits, HD]
  float* ws_ml;        // [NQ, 128 splits, 2]
  int* bar;            // [0] barrier arrivals, [1] exit count: zeroed, left zeroed
  FusedLayer layer[kFusedMaxLayers];
};
// Workspace bytes for the fused step (barrier words + activations + attention partials).
int64_t decode_fused_workspace_bytes(int64_t H, int64_t I, int64_t NQ, int64_t NKV, int64_t HD);
// Fills the scratch pointers of P from the workspace; checks the shapes; false if not served.
bool plan_decode_fused(FusedDecodeParams& P, void* workspace, int64_t workspace_bytes, int sms);
cudaError_t launch_decode_fused(const FusedDecodeParams& P, int sms, cudaStream_t stream);
cudaError_t read_and_clear_decode_fused_error(int* out);

}  // namespace soinfer
