// Attention-side glue: RMSNorm (also per-head QK-norm), rotate-half RoPE,
// KV-cache append, and the device-driven row gather.
//
// Reference semantics: csrc/kernels/rmsnorm.cu:9-42 (fp32 sum of squares,
// rsqrtf(mean + eps), out = half((v * inv) * w)), csrc/kernels/rope.cu:5-19
// (x1' = x1*c - x2*s, x2' = x2*c + x1*s over pairs (i, i + hd/2)),
// csrc/kernels/kv_cache.cu:7-20 (cache[h, pos, :] = new[h, :]).
#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"

namespace soinfer {
namespace {

// Every kernel here starts with griddepcontrol.wait (before touching any
// activation memory), so each is launched as a programmatic dependent: its
// launch overlaps the tail of the kernel before it.
constexpr bool kPdl = true;
constexpr int kNormThreads = 256;

// ADD: the normalised row is v = fp16(x + x2) (fp32 add, one rounding -- the
// fp16 tensor add of the reference's residual), also written to sum_out.
template <bool ADD>
__device__ __forceinline__ half2 norm_input(const half2* xr, const half2* x2r, int64_t i) {
  if (!ADD) return xr[i];
  const float2 a = __half22float2(xr[i]), b = __half22float2(x2r[i]);
  return __floats2half2_rn(a.x + b.x, a.y + b.y);
}

template <bool ADD>
__global__ void __launch_bounds__(kNormThreads)
    rmsnorm_kernel(const half* __restrict__ x, const half* __restrict__ x2, const half* __restrict__ w,
                   half* __restrict__ out, half* __restrict__ sum_out, const int64_t hidden, const float eps) {
  __shared__ float s_part[kNormThreads / 32];
  __shared__ float s_inv;
  pdl_launch_dependents();
  pdl_wait();
  const int64_t row = blockIdx.x;
  const half2* xr = reinterpret_cast<const half2*>(x + row * hidden);
  const half2* x2r = ADD ? reinterpret_cast<const half2*>(x2 + row * hidden) : nullptr;
  half2* orow = reinterpret_cast<half2*>(out + row * hidden);
  const half2* w2 = reinterpret_cast<const half2*>(w);
  const int64_t h2 = hidden / 2;
  float ss = 0.f;
  for (int64_t i = threadIdx.x; i < h2; i += kNormThreads) {
    const half2 hv = norm_input<ADD>(xr, x2r, i);
    if (ADD) reinterpret_cast<half2*>(sum_out + row * hidden)[i] = hv;
    const float2 f = __half22float2(hv);
    ss += f.x * f.x + f.y * f.y;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < kNormThreads / 32; ++i) t += s_part[i];
    s_inv = rsqrtf(t / (float)hidden + eps);
  }
  __syncthreads();
  const float inv = s_inv;
  for (int64_t i = threadIdx.x; i < h2; i += kNormThreads) {
    const float2 f = __half22float2(norm_input<ADD>(xr, x2r, i));
    const float2 g = __half22float2(w2[i]);
    orow[i] = __floats2half2_rn(f.x * inv * g.x, f.y * inv * g.y);
  }
}

// out[i] = fp16( silu(float(g)) * float(up[i]) ), g = gate[idx[i]] (or gate[i]);
// silu(x) = x / (1 + exp(-x)), the fp32 expression of torch's F.silu.
__global__ void swiglu_kernel(const half* __restrict__ gate, const half* __restrict__ up,
                              const int32_t* __restrict__ idx, half* __restrict__ out, const int64_t n) {
  pdl_launch_dependents();
  pdl_wait();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float g = __half2float(gate[idx ? idx[i] : i]);
    const float s = g / (1.0f + expf(-g));
    out[i] = __float2half_rn(s * __half2float(up[i]));
  }
}

__global__ void add_half_kernel(const half* __restrict__ a, const half* __restrict__ b, half* __restrict__ out,
                                const int64_t n) {
  pdl_launch_dependents();
  pdl_wait();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = __float2half_rn(__half2float(a[i]) + __half2float(b[i]));
}

// After the q / k / v GEMVs of one decode token (rows: q heads, then k heads,
// then v heads; one warp per row): q and k rows get RMSNorm over the head
// (fp32 sum of squares, out = fp16((x * rsqrt(mean + eps)) * w)) followed by
// rotate-half RoPE on the normalised fp16 values; q is rewritten in place,
// the k and v rows are appended to the caches at `pos` (or *pos_dev).
// cv / sv: the position's cos / sin, or with pos_dev tables indexed by it.
constexpr int kHeadRowsPerBlock = 4;

__global__ void __launch_bounds__(kHeadRowsPerBlock * 32)
    head_norm_rope_kernel(half* __restrict__ q, const half* __restrict__ k, const half* __restrict__ v,
                          const half* __restrict__ qw, const half* __restrict__ kw, const float* __restrict__ cv,
                          const float* __restrict__ sv, half* __restrict__ kc, half* __restrict__ vc, const int nq,
                          const int nkv, const int hd, const int64_t max_seq, int64_t pos,
                          const int32_t* __restrict__ pos_dev, const int64_t table_rows, const float eps) {
  pdl_launch_dependents();
  pdl_wait();
  const int row = blockIdx.x * kHeadRowsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= nq + 2 * nkv) return;
  if (pos_dev) {
    pos = *pos_dev;
    if (pos < 0 || pos >= max_seq || pos >= table_rows) return;
    cv += pos * (hd / 2);
    sv += pos * (hd / 2);
  }
  const int half_dim = hd / 2;
  if (row >= nq + nkv) {  // v: copy into the cache
    const int h = row - nq - nkv;
    const half* src = v + (int64_t)h * hd;
    half* dst = vc + ((int64_t)h * max_seq + pos) * hd;
    for (int i = lane; i < hd; i += 32) dst[i] = src[i];
    return;
  }
  const bool is_q = row < nq;
  const int h = is_q ? row : row - nq;
  const half* src = is_q ? q + (int64_t)h * hd : k + (int64_t)h * hd;
  const half* w = is_q ? qw : kw;
  float ss = 0.f;
  for (int i = lane; i < hd; i += 32) {
    const float f = __half2float(src[i]);
    ss = fmaf(f, f, ss);
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / (float)hd + eps);
  half* dst = is_q ? q + (int64_t)h * hd : kc + ((int64_t)h * max_seq + pos) * hd;
  // pairs (i, i + hd/2): normalise both (rounded to fp16), then rotate
  float x1[4], x2[4];
  int n = 0;
  for (int i = lane; i < half_dim; i += 32, ++n) {
    x1[n] = __half2float(__float2half_rn(__fmul_rn(__fmul_rn(__half2float(src[i]), inv), __half2float(w[i]))));
    x2[n] = __half2float(
        __float2half_rn(__fmul_rn(__fmul_rn(__half2float(src[i + half_dim]), inv), __half2float(w[i + half_dim]))));
  }
  __syncwarp();  // every lane has read its q values before any lane rewrites q in place
  n = 0;
  for (int i = lane; i < half_dim; i += 32, ++n) {
    const float c = cv[i], s = sv[i];
    // explicit roundings (no contraction), so every kernel that rotates a head row gets the same bits
    dst[i] = __float2half_rn(__fsub_rn(__fmul_rn(x1[n], c), __fmul_rn(x2[n], s)));
    dst[i + half_dim] = __float2half_rn(__fadd_rn(__fmul_rn(x2[n], c), __fmul_rn(x1[n], s)));
  }
}

// cv / sv: the position's cos / sin [head_dim / 2], or -- with pos_dev -- tables
// [table_rows, head_dim / 2] indexed by *pos_dev (out-of-range positions: no-op).
__global__ void rope_kernel(half* __restrict__ x, const float* __restrict__ cv, const float* __restrict__ sv,
                            const int64_t head_dim, const int32_t* __restrict__ pos_dev, const int64_t table_rows) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t half_dim = head_dim / 2;
  if (pos_dev) {
    const int64_t pos = *pos_dev;
    if (pos < 0 || pos >= table_rows) return;
    cv += pos * half_dim;
    sv += pos * half_dim;
  }
  half* row = x + (int64_t)blockIdx.x * head_dim;
  for (int64_t i = threadIdx.x; i < half_dim; i += blockDim.x) {
    const float c = cv[i], s = sv[i];
    const float x1 = __half2float(row[i]);
    const float x2 = __half2float(row[i + half_dim]);
    row[i] = __float2half_rn(x1 * c - x2 * s);
    row[i + half_dim] = __float2half_rn(x2 * c + x1 * s);
  }
}

__global__ void kv_append_kernel(half* __restrict__ kc, half* __restrict__ vc, const half* __restrict__ kn,
                                 const half* __restrict__ vn, const int64_t max_seq, const int64_t hd,
                                 int64_t pos, const int32_t* __restrict__ pos_dev) {
  pdl_launch_dependents();
  pdl_wait();
  if (pos_dev) {  // device-position form: out-of-range positions write nothing
    pos = *pos_dev;
    if (pos < 0 || pos >= max_seq) return;
  }
  const int64_t h = blockIdx.x;
  half* kd = kc + (h * max_seq + pos) * hd;
  half* vd = vc + (h * max_seq + pos) * hd;
  const half* ks = kn + h * hd;
  const half* vs = vn + h * hd;
  for (int64_t i = threadIdx.x; i < hd; i += blockDim.x) {
    kd[i] = ks[i];
    vd[i] = vs[i];
  }
}

// The graph decode step's input row: x = embed[ids[*pos_dev]] (fp16 [vocab, H]),
// the position and the token id read when the kernel runs; an out-of-range
// position or id writes nothing.  VEC16: 16-byte pieces.
template <bool VEC16>
__global__ void step_embed_kernel(const half* __restrict__ embed, const int64_t vocab, const int64_t H,
                                  const int32_t* __restrict__ ids, const int64_t ids_len,
                                  const int32_t* __restrict__ pos_dev, half* __restrict__ x) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t pos = *pos_dev;
  if (pos < 0 || pos >= ids_len) return;
  const int64_t id = ids[pos];
  if (id < 0 || id >= vocab) return;
  const int64_t n = VEC16 ? H / 8 : H;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    if (VEC16)
      reinterpret_cast<uint4*>(x)[i] = reinterpret_cast<const uint4*>(embed + id * H)[i];
    else
      x[i] = embed[id * H + i];
  }
}

// Advances the graph decode step's device state once the step's token is in
// *next: ids[pos + 1] = *next unless pos + 1 is still a prompt position
// (< *prompt_len, the prompt's token stays), then pos += 1.  Nothing when
// pos + 1 is outside [0, ids_len).
__global__ void step_advance_kernel(int32_t* __restrict__ ids, const int64_t ids_len, int32_t* __restrict__ pos_dev,
                                    const int32_t* __restrict__ prompt_len, const int32_t* __restrict__ next) {
  pdl_launch_dependents();
  pdl_wait();
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const int64_t p = *pos_dev;
  if (p < 0 || p + 1 >= ids_len) return;
  if (p + 1 >= *prompt_len) ids[p + 1] = *next;
  *pos_dev = (int32_t)(p + 1);
}

template <bool VEC16>
__global__ void gather_rows_kernel(const uint8_t* __restrict__ matrix, const int64_t num_rows, const int64_t row_nbytes,
                                   const int32_t* __restrict__ rows, const int64_t k, uint8_t* __restrict__ dst) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t unit = VEC16 ? 16 : 1;
  const int64_t per_row = row_nbytes / unit;
  const int64_t total = k * per_row;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
    const int64_t j = e / per_row;
    const int64_t c = e - j * per_row;
    int64_t r = rows[j];
    r = r < 0 ? 0 : (r >= num_rows ? num_rows - 1 : r);
    if (VEC16) {
      const uint4 v = ldg_stream_u4(matrix + r * row_nbytes + c * 16);
      *reinterpret_cast<uint4*>(dst + j * row_nbytes + c * 16) = v;
    } else {
      dst[j * row_nbytes + c] = matrix[r * row_nbytes + c];
    }
  }
}

// Multi-source gather with the row count in device memory: every thread
// copies 16-byte pieces (4-byte pieces for a source whose rows are not
// 16-byte aligned) of rows rows[j], j < min(*count, max_k), of every source;
// a warp's lanes read consecutive pieces of one row, so each warp load is one
// contiguous burst (over PCIe when the matrix is pinned host memory).
__global__ void gather_multi_kernel(const GatherMulti P) {
  pdl_launch_dependents();
  pdl_wait();
  int64_t n = P.max_k;
  if (P.count != nullptr) {
    const int64_t c = *P.count;
    n = c < 0 ? 0 : (c < n ? c : n);
  }
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
#pragma unroll 1
  for (int s = 0; s < P.num; ++s) {
    const GatherSrc& g = P.src[s];
    const int64_t unit = g.vec16 ? 16 : 4;
    const int64_t per_row = g.row_nbytes / unit;
    const int64_t total = P.max_k * per_row;
    for (int64_t e = tid; e < total; e += stride) {
      const int64_t j = e / per_row;
      if (j >= n) break;  // rows are in j order: nothing further in this source
      const int64_t c = e - j * per_row;
      int64_t r = P.rows[j];
      r = r < 0 ? 0 : (r >= g.num_rows ? g.num_rows - 1 : r);
      if (g.vec16) {
        const uint4 v = ldg_stream_u4(g.matrix + r * g.row_nbytes + c * 16);
        *reinterpret_cast<uint4*>(g.dst + j * g.row_nbytes + c * 16) = v;
      } else {
        const uint32_t v = ldg_stream_u32(g.matrix + r * g.row_nbytes + c * 4);
        *reinterpret_cast<uint32_t*>(g.dst + j * g.row_nbytes + c * 4) = v;
      }
    }
  }
}

}  // namespace

cudaError_t launch_gather_multi(const GatherMulti& P, cudaStream_t stream) {
  int64_t total = 0;
  for (int s = 0; s < P.num; ++s) total += P.max_k * (P.src[s].row_nbytes / (P.src[s].vec16 ? 16 : 4));
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  return launch_ex(gather_multi_kernel, dim3((unsigned)blocks), dim3(256), 0, stream, 1, kPdl, P);
}

cudaError_t launch_rmsnorm(const half* x, const half* w, half* out, int64_t rows, int64_t hidden, float eps,
                           cudaStream_t stream) {
  return launch_ex(rmsnorm_kernel<false>, dim3((unsigned)rows), dim3(kNormThreads), 0, stream, 1, kPdl, x,
                   (const half*)nullptr, w, out, (half*)nullptr, hidden, eps);
}

cudaError_t launch_add_rmsnorm(const half* x, const half* x2, const half* w, half* out, half* sum_out, int64_t rows,
                               int64_t hidden, float eps, cudaStream_t stream) {
  return launch_ex(rmsnorm_kernel<true>, dim3((unsigned)rows), dim3(kNormThreads), 0, stream, 1, kPdl, x, x2, w, out,
                   sum_out, hidden, eps);
}

cudaError_t launch_swiglu(const half* gate, const half* up, const int32_t* idx, half* out, int64_t n,
                          cudaStream_t stream) {
  const int threads = 256;
  int64_t blocks = (n + threads - 1) / threads;
  if (blocks > 1184) blocks = 1184;
  if (blocks < 1) blocks = 1;
  return launch_ex(swiglu_kernel, dim3((unsigned)blocks), dim3(threads), 0, stream, 1, kPdl, gate, up, idx, out, n);
}

cudaError_t launch_add_half(const half* a, const half* b, half* out, int64_t n, cudaStream_t stream) {
  const int threads = 256;
  int64_t blocks = (n + threads - 1) / threads;
  if (blocks > 1184) blocks = 1184;
  if (blocks < 1) blocks = 1;
  return launch_ex(add_half_kernel, dim3((unsigned)blocks), dim3(threads), 0, stream, 1, kPdl, a, b, out, n);
}

cudaError_t launch_head_norm_rope(half* q, const half* k, const half* v, const half* qw, const half* kw,
                                  const float* cv, const float* sv, half* kc, half* vc, int64_t nq, int64_t nkv,
                                  int64_t hd, int64_t max_seq, int64_t pos, const int32_t* pos_dev,
                                  int64_t table_rows, float eps, cudaStream_t stream) {
  const int64_t rows = nq + 2 * nkv;
  const unsigned blocks = (unsigned)((rows + kHeadRowsPerBlock - 1) / kHeadRowsPerBlock);
  return launch_ex(head_norm_rope_kernel, dim3(blocks), dim3(kHeadRowsPerBlock * 32), 0, stream, 1, kPdl, q, k, v,
                   qw, kw, cv, sv, kc, vc, (int)nq, (int)nkv, (int)hd, max_seq, pos, pos_dev, table_rows, eps);
}

cudaError_t launch_rope(half* x, const float* cv, const float* sv, int64_t heads, int64_t head_dim,
                        cudaStream_t stream) {
  int threads = (int)(head_dim / 2);
  threads = threads < 32 ? 32 : (threads > 1024 ? 1024 : threads);
  return launch_ex(rope_kernel, dim3((unsigned)heads), dim3(threads), 0, stream, 1, kPdl, x, cv, sv, head_dim,
                   (const int32_t*)nullptr, (int64_t)0);
}

cudaError_t launch_rope_at(half* x, const float* cos_table, const float* sin_table, int64_t table_rows, int64_t heads,
                           int64_t head_dim, const int32_t* pos_dev, cudaStream_t stream) {
  int threads = (int)(head_dim / 2);
  threads = threads < 32 ? 32 : (threads > 1024 ? 1024 : threads);
  return launch_ex(rope_kernel, dim3((unsigned)heads), dim3(threads), 0, stream, 1, kPdl, x, cos_table, sin_table,
                   head_dim, pos_dev, table_rows);
}

cudaError_t launch_kv_append(half* kc, half* vc, const half* kn, const half* vn, int64_t nkv, int64_t max_seq,
                             int64_t hd, int64_t pos, cudaStream_t stream) {
  int threads = hd < 32 ? 32 : (hd > 256 ? 256 : (int)hd);
  return launch_ex(kv_append_kernel, dim3((unsigned)nkv), dim3(threads), 0, stream, 1, kPdl, kc, vc, kn, vn, max_seq,
                   hd, pos, (const int32_t*)nullptr);
}

cudaError_t launch_kv_append_at(half* kc, half* vc, const half* kn, const half* vn, int64_t nkv, int64_t max_seq,
                                int64_t hd, const int32_t* pos_dev, cudaStream_t stream) {
  int threads = hd < 32 ? 32 : (hd > 256 ? 256 : (int)hd);
  return launch_ex(kv_append_kernel, dim3((unsigned)nkv), dim3(threads), 0, stream, 1, kPdl, kc, vc, kn, vn, max_seq,
                   hd, (int64_t)0, pos_dev);
}

cudaError_t launch_step_embed(const half* embed, int64_t vocab, int64_t H, const int32_t* ids, int64_t ids_len,
                              const int32_t* pos_dev, half* x, cudaStream_t stream) {
  const bool vec = H % 8 == 0 && ((reinterpret_cast<uintptr_t>(embed) | reinterpret_cast<uintptr_t>(x)) & 15u) == 0;
  const int64_t n = vec ? H / 8 : H;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 64) blocks = 64;
  if (vec)
    return launch_ex(step_embed_kernel<true>, dim3((unsigned)blocks), dim3(256), 0, stream, 1, kPdl, embed, vocab, H,
                     ids, ids_len, pos_dev, x);
  return launch_ex(step_embed_kernel<false>, dim3((unsigned)blocks), dim3(256), 0, stream, 1, kPdl, embed, vocab, H,
                   ids, ids_len, pos_dev, x);
}

cudaError_t launch_step_advance(int32_t* ids, int64_t ids_len, int32_t* pos_dev, const int32_t* prompt_len,
                                const int32_t* next, cudaStream_t stream) {
  return launch_ex(step_advance_kernel, dim3(1), dim3(32), 0, stream, 1, kPdl, ids, ids_len, pos_dev, prompt_len,
                   next);
}

cudaError_t launch_gather_rows_device(const uint8_t* matrix, int64_t num_rows, int64_t row_nbytes,
                                      const int32_t* rows, int64_t k, uint8_t* dst, cudaStream_t stream) {
  const bool vec = (row_nbytes % 16 == 0) && ((reinterpret_cast<uintptr_t>(matrix) & 15u) == 0) &&
                   ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0);
  const int64_t total = k * (vec ? row_nbytes / 16 : row_nbytes);
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  if (vec)
    return launch_ex(gather_rows_kernel<true>, dim3((unsigned)blocks), dim3(256), 0, stream, 1, kPdl, matrix,
                     num_rows, row_nbytes, rows, k, dst);
  return launch_ex(gather_rows_kernel<false>, dim3((unsigned)blocks), dim3(256), 0, stream, 1, kPdl, matrix,
                   num_rows, row_nbytes, rows, k, dst);
}

}  // namespace soinfer
