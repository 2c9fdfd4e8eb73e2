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

constexpr int kNormThreads = 256;

__global__ void __launch_bounds__(kNormThreads)
    rmsnorm_kernel(const half* __restrict__ x, const half* __restrict__ w, half* __restrict__ out, const int64_t hidden,
                   const float eps) {
  __shared__ float s_part[kNormThreads / 32];
  __shared__ float s_inv;
  pdl_launch_dependents();
  pdl_wait();
  const int64_t row = blockIdx.x;
  const half2* xr = reinterpret_cast<const half2*>(x + row * hidden);
  half2* orow = reinterpret_cast<half2*>(out + row * hidden);
  const half2* w2 = reinterpret_cast<const half2*>(w);
  const int64_t h2 = hidden / 2;
  float ss = 0.f;
  for (int64_t i = threadIdx.x; i < h2; i += kNormThreads) {
    const float2 f = __half22float2(xr[i]);
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
    const float2 f = __half22float2(xr[i]);
    const float2 g = __half22float2(w2[i]);
    orow[i] = __floats2half2_rn(f.x * inv * g.x, f.y * inv * g.y);
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

}  // namespace

cudaError_t launch_rmsnorm(const half* x, const half* w, half* out, int64_t rows, int64_t hidden, float eps,
                           cudaStream_t stream) {
  return launch_ex(rmsnorm_kernel, dim3((unsigned)rows), dim3(kNormThreads), 0, stream, 1, false, x, w, out, hidden,
                   eps);
}

cudaError_t launch_rope(half* x, const float* cv, const float* sv, int64_t heads, int64_t head_dim,
                        cudaStream_t stream) {
  int threads = (int)(head_dim / 2);
  threads = threads < 32 ? 32 : (threads > 1024 ? 1024 : threads);
  return launch_ex(rope_kernel, dim3((unsigned)heads), dim3(threads), 0, stream, 1, false, x, cv, sv, head_dim,
                   (const int32_t*)nullptr, (int64_t)0);
}

cudaError_t launch_rope_at(half* x, const float* cos_table, const float* sin_table, int64_t table_rows, int64_t heads,
                           int64_t head_dim, const int32_t* pos_dev, cudaStream_t stream) {
  int threads = (int)(head_dim / 2);
  threads = threads < 32 ? 32 : (threads > 1024 ? 1024 : threads);
  return launch_ex(rope_kernel, dim3((unsigned)heads), dim3(threads), 0, stream, 1, false, x, cos_table, sin_table,
                   head_dim, pos_dev, table_rows);
}

cudaError_t launch_kv_append(half* kc, half* vc, const half* kn, const half* vn, int64_t nkv, int64_t max_seq,
                             int64_t hd, int64_t pos, cudaStream_t stream) {
  int threads = hd < 32 ? 32 : (hd > 256 ? 256 : (int)hd);
  return launch_ex(kv_append_kernel, dim3((unsigned)nkv), dim3(threads), 0, stream, 1, false, kc, vc, kn, vn, max_seq,
                   hd, pos, (const int32_t*)nullptr);
}

cudaError_t launch_kv_append_at(half* kc, half* vc, const half* kn, const half* vn, int64_t nkv, int64_t max_seq,
                                int64_t hd, const int32_t* pos_dev, cudaStream_t stream) {
  int threads = hd < 32 ? 32 : (hd > 256 ? 256 : (int)hd);
  return launch_ex(kv_append_kernel, dim3((unsigned)nkv), dim3(threads), 0, stream, 1, false, kc, vc, kn, vn, max_seq,
                   hd, (int64_t)0, pos_dev);
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
    return launch_ex(gather_rows_kernel<true>, dim3((unsigned)blocks), dim3(256), 0, stream, 1, false, matrix,
                     num_rows, row_nbytes, rows, k, dst);
  return launch_ex(gather_rows_kernel<false>, dim3((unsigned)blocks), dim3(256), 0, stream, 1, false, matrix,
                   num_rows, row_nbytes, rows, k, dst);
}

}  // namespace soinfer
