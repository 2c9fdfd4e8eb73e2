// Sparse 'down' GEMV over k selected rows of the transposed down_proj:
//   y[c] = fp16( sum_{j<k} (h[j] * scale[j, c/g]) * q[j, c] )
// (reference csrc/kernels/gemv_sparse_accumulate.cu:10-38 and the
// descriptor-sourced csrc/kernels/gemv_dip_fused.cu:116-154, which run one
// thread per output column serially over j -- 8 CTAs at H=2048).
//
// Here the k rows are split into row slabs and the H columns into column
// slabs; each thread owns a 32-column (16-byte) slice of a row and walks the
// slab's rows with a fixed stride, so every row is read exactly once with
// fully coalesced 128-bit loads.  Each value is converted to fp32 exactly
// without a conversion instruction: OR-ing nibble n (at bit offset p) under
// the exponent of 2^23 gives 2^23 + n*2^p, and one FADD removes the bias,
// leaving s*2^p; the FFMA then uses the coefficient pre-scaled by 2^-p, so
// the product equals coef*s exactly, as in the reference's fp32 expression.
// Partials: per-thread registers -> fixed-order shared-memory reduction over
// the CTA's row phases -> one fp32 partial row per (row slab, column slab)
// in the workspace -> the last CTA of each column slab (atomic ticket) sums
// the slab partials in row-slab order.  The reduction order depends only on
// (H, k), never on which buffer a row came from, so cache / staging /
// indexed / plain sources give bit-identical outputs.
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"

namespace soinfer {
namespace {

constexpr int kThreads = 256;
constexpr int kColChunks = 8;            // 16-byte column chunks per column slab (256 columns)
constexpr int kPhases = kThreads / kColChunks;
constexpr int kTargetCtas = 296;
constexpr int64_t kCounterBytes = 4096;  // tickets that every workspace starts with: 1024 column slabs
constexpr int64_t kStaticScratchBytes = 512 * 1024;
constexpr int kMaxDevices = 64;

// Scratch of the no-alloc entry point, one copy per device (file-scope device
// memory: no allocation at call time).  Same layout as a caller workspace:
// the column-slab tickets (ticket_bytes(H): kCounterBytes, more for H above
// 65536), which must start at zero and which every call leaves at zero, then
// the fp32 partial rows (overwritten by each call).  Workspaces of up to kStaticScratchBytes fit: every shape from H =
// 2048 to H = 16384 needs about 0.3 MiB.
static __device__ __align__(256) unsigned char g_sparse_scratch[kStaticScratchBytes];

struct DownShape {
  int64_t H, k;
  int vec;         // 4: 16-byte chunks of 32 columns; 1: 4-byte chunks of 8 columns
  int64_t chunks;  // column chunks per row
  int64_t col_slabs, row_slabs, rows_per_slab;
};

DownShape down_shape(int64_t H, int64_t k, bool vec4) {
  DownShape s;
  s.H = H;
  s.k = k;
  s.vec = vec4 ? 4 : 1;
  s.chunks = vec4 ? H / 32 : (H + 7) / 8;
  s.col_slabs = (s.chunks + kColChunks - 1) / kColChunks;
  int64_t want_rows = (kTargetCtas + s.col_slabs - 1) / s.col_slabs;
  if (want_rows < 1) want_rows = 1;
  s.rows_per_slab = (k + want_rows - 1) / want_rows;
  if (s.rows_per_slab < kPhases) s.rows_per_slab = kPhases < k ? kPhases : k;
  if (s.rows_per_slab < 1) s.rows_per_slab = 1;
  s.row_slabs = (k + s.rows_per_slab - 1) / s.rows_per_slab;
  return s;
}

// Ticket area of a workspace for H output columns: one int per column slab of
// the wider of the two kernel shapes, at least kCounterBytes.  The first
// kCounterBytes are kept zeroed by every call; a launch that needs more clears
// the rest first (it may hold partial rows of an earlier, narrower call).
int64_t ticket_bytes(int64_t H) {
  const int64_t a = down_shape(H, 1, true).col_slabs, b = down_shape(H, 1, false).col_slabs;
  const int64_t need = ((a > b ? a : b) * 4 + 255) / 256 * 256;
  return need > kCounterBytes ? need : kCounterBytes;
}

template <RowMode M>
__device__ __forceinline__ void down_row(const RowSource& src, int64_t j, const uint8_t*& w, const float*& s) {
  if constexpr (M == RowMode::kPlain) {
    w = src.W + j * src.row_bytes;
    s = src.S + j * src.num_groups;
  } else if constexpr (M == RowMode::kIndexed) {
    int64_t r = src.idx[j];
    r = r < 0 ? 0 : (r >= src.rows1 ? src.rows1 - 1 : r);
    w = src.W + r * src.row_bytes;
    s = src.S + r * src.num_groups;
  } else {
    const int32_t d = src.idx[j];
    const bool staging = (desc_is_staging(d) && src.rows2 > 0) || src.rows1 == 0;
    int64_t r = desc_offset(d);
    const int64_t rows = staging ? src.rows2 : src.rows1;
    r = r >= rows ? rows - 1 : r;
    w = (staging ? src.W2 : src.W) + r * src.row_bytes;
    s = (staging ? src.S2 : src.S) + r * src.num_groups;
  }
}

// acc[8] += coef * values of word w (logical K order v0..v7).
__device__ __forceinline__ void fma_word(uint32_t w, const float c[5], float* acc) {
  // nibble slots 0..4 sit at bit offsets 0,4,8,12,16; slots 5..7 are brought
  // to offsets 8,12,16 by w >> 12.  slot -> logical index: 0,2,4,6,1,3,5,7.
  const uint32_t top = w >> 12;
  const float f0 = __uint_as_float(lop3_and_xor(w, 0x0000000fu, 0x4b000008u)) - 8388616.0f;         // v0
  const float f1 = __uint_as_float(lop3_and_xor(w, 0x000000f0u, 0x4b000080u)) - 8388736.0f;         // v2 *16
  const float f2 = __uint_as_float(lop3_and_xor(w, 0x00000f00u, 0x4b000800u)) - 8390656.0f;         // v4 *256
  const float f3 = __uint_as_float(lop3_and_xor(w, 0x0000f000u, 0x4b008000u)) - 8421376.0f;         // v6 *4096
  const float f4 = __uint_as_float(lop3_and_xor(w, 0x000f0000u, 0x4b080000u)) - 8912896.0f;         // v1 *65536
  const float f5 = __uint_as_float(lop3_and_xor(top, 0x00000f00u, 0x4b000800u)) - 8390656.0f;       // v3 *256
  const float f6 = __uint_as_float(lop3_and_xor(top, 0x0000f000u, 0x4b008000u)) - 8421376.0f;       // v5 *4096
  const float f7 = __uint_as_float(lop3_and_xor(top, 0x000f0000u, 0x4b080000u)) - 8912896.0f;       // v7 *65536
  acc[0] = fmaf(c[0], f0, acc[0]);
  acc[1] = fmaf(c[4], f4, acc[1]);
  acc[2] = fmaf(c[1], f1, acc[2]);
  acc[3] = fmaf(c[2], f5, acc[3]);
  acc[4] = fmaf(c[2], f2, acc[4]);
  acc[5] = fmaf(c[3], f6, acc[5]);
  acc[6] = fmaf(c[3], f3, acc[6]);
  acc[7] = fmaf(c[4], f7, acc[7]);
}

template <RowMode M, int VEC>
__global__ void __launch_bounds__(kThreads)
    sparse_down_kernel(const RowSource src, const half* __restrict__ h, half* __restrict__ y, const int64_t H,
                       const int64_t k, const int64_t gsz, const int64_t chunks, const int64_t rows_per_slab,
                       float* __restrict__ partials, int* __restrict__ tickets, const half* __restrict__ resid) {
  constexpr int kCols = VEC * 8;  // columns per chunk
  extern __shared__ float red[];  // [kPhases][kColChunks * kCols]
  __shared__ int is_last;

  const int cl = threadIdx.x % kColChunks;
  const int phase = threadIdx.x / kColChunks;
  const int64_t col_slab = blockIdx.x;
  const int64_t row_slab = blockIdx.y;
  const int64_t chunk = col_slab * kColChunks + cl;
  const bool active = chunk < chunks;
  const int64_t j0 = row_slab * rows_per_slab;
  const int64_t j1 = (j0 + rows_per_slab < k) ? j0 + rows_per_slab : k;
  const int64_t col0 = chunk * kCols;
  const int64_t grp = active ? col0 / gsz : 0;  // g % kCols == 0 on the vector path

  pdl_launch_dependents();
  pdl_wait();  // h and the row indices come from preceding kernels

  float acc[kCols];
#pragma unroll
  for (int i = 0; i < kCols; ++i) acc[i] = 0.f;

  if (active) {
    // kBatch rows per pass: every row's index, weight, scale and h loads are
    // issued before the first FMA (one latency chain per pass, not per row);
    // the FMAs still run in ascending j, so the sums are unchanged.
    constexpr int kBatch = 4;
    for (int64_t jb = j0 + phase; jb < j1; jb += (int64_t)kPhases * kBatch) {
      const uint8_t* w[kBatch];
      const float* s[kBatch];
      float hj[kBatch];
#pragma unroll
      for (int r = 0; r < kBatch; ++r) {
        const int64_t j = jb + (int64_t)r * kPhases;
        const int64_t jj = j < j1 ? j : jb;  // past the slab: reload row jb, its terms are skipped
        down_row<M>(src, jj, w[r], s[r]);
        hj[r] = __half2float(h[jj]);
      }
      float sc[kBatch];
      if constexpr (VEC == 4) {
        uint4 q[kBatch];
#pragma unroll
        for (int r = 0; r < kBatch; ++r) {
          q[r] = ldg_stream_u4(w[r] + chunk * 16);
          sc[r] = __ldg(s[r] + grp);
        }
#pragma unroll
        for (int r = 0; r < kBatch; ++r) {
          if (jb + (int64_t)r * kPhases >= j1) break;
          float c[5];
          c[0] = hj[r] * sc[r];
          c[1] = c[0] * 0.0625f;
          c[2] = c[0] * 0.00390625f;
          c[3] = c[0] * 0.000244140625f;
          c[4] = c[0] * 0.0000152587890625f;
          fma_word(q[r].x, c, acc + 0);
          fma_word(q[r].y, c, acc + 8);
          fma_word(q[r].z, c, acc + 16);
          fma_word(q[r].w, c, acc + 24);
        }
      } else {
        uint32_t q[kBatch];
#pragma unroll
        for (int r = 0; r < kBatch; ++r) {
          q[r] = ldg_stream_u32(w[r] + chunk * 4);
          sc[r] = __ldg(s[r] + col0 / gsz);
        }
#pragma unroll
        for (int r = 0; r < kBatch; ++r) {
          if (jb + (int64_t)r * kPhases >= j1) break;
          float c[5];
          c[0] = hj[r] * sc[r];
          c[1] = c[0] * 0.0625f;
          c[2] = c[0] * 0.00390625f;
          c[3] = c[0] * 0.000244140625f;
          c[4] = c[0] * 0.0000152587890625f;
          fma_word(q[r], c, acc);
        }
      }
    }
  }

  // fixed-order reduction over the CTA's row phases
  constexpr int kSlabCols = kColChunks * kCols;
#pragma unroll
  for (int i = 0; i < kCols; ++i) red[phase * kSlabCols + cl * kCols + i] = acc[i];
  __syncthreads();
  const int64_t slab_col0 = col_slab * kSlabCols;
  for (int c = threadIdx.x; c < kSlabCols; c += kThreads) {
    float sum = 0.f;
    for (int p = 0; p < kPhases; ++p) sum += red[p * kSlabCols + c];
    if (slab_col0 + c < H) partials[row_slab * H + slab_col0 + c] = sum;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int ticket = atomicAdd(&tickets[col_slab], 1);
    is_last = (ticket == (int)gridDim.y - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int c = threadIdx.x; c < kSlabCols; c += kThreads) {
    const int64_t col = slab_col0 + c;
    if (col >= H) continue;
    float sum = 0.f;
    const int slabs = (int)gridDim.y;
    constexpr int kLoads = 32;  // partial rows loaded per pass, summed in row-slab order
    for (int r0 = 0; r0 < slabs; r0 += kLoads) {
      float v[kLoads];
#pragma unroll
      for (int i = 0; i < kLoads; ++i)
        v[i] = r0 + i < slabs ? __ldcg(partials + (int64_t)(r0 + i) * H + col) : 0.f;
#pragma unroll
      for (int i = 0; i < kLoads; ++i)
        if (r0 + i < slabs) sum += v[i];
    }
    half out = __float2half_rn(sum);
    if (resid != nullptr) out = __float2half_rn(__half2float(resid[col]) + __half2float(out));  // residual epilogue
    y[col] = out;
  }
  if (threadIdx.x == 0) tickets[col_slab] = 0;  // leave the workspace ready for the next call
}

template <RowMode M>
cudaError_t launch_mode(const RowSource& src, const half* h, half* y, int64_t H, int64_t k, int64_t gsz,
                        void* workspace, cudaStream_t stream, LaunchOpts opts) {
  auto aligned16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const bool vec4 = (H % 32 == 0) && (gsz % 32 == 0) && src.row_bytes % 16 == 0 && aligned16(src.W) &&
                    (M != RowMode::kDesc || aligned16(src.W2));
  const DownShape s = down_shape(H, k, vec4);
  int* tickets = reinterpret_cast<int*>(workspace);
  const int64_t tb = ticket_bytes(H);
  float* partials = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + tb);
  if (tb > kCounterBytes) {
    cudaError_t e = cudaMemsetAsync(reinterpret_cast<char*>(workspace) + kCounterBytes, 0, (size_t)(tb - kCounterBytes),
                                    stream);
    if (e != cudaSuccess) return e;
  }
  const dim3 grid((unsigned)s.col_slabs, (unsigned)s.row_slabs);
  if (vec4) {
    const size_t smem = (size_t)kPhases * kColChunks * 32 * sizeof(float);
    auto kernel = sparse_down_kernel<M, 4>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    return launch_ex(kernel, grid, dim3(kThreads), smem, stream, 1, opts.pdl, src, h, y, H, k, gsz, s.chunks,
                     s.rows_per_slab, partials, tickets, opts.resid);
  }
  const size_t smem = (size_t)kPhases * kColChunks * 8 * sizeof(float);
  return launch_ex(sparse_down_kernel<M, 1>, grid, dim3(kThreads), smem, stream, 1, opts.pdl, src, h, y, H, k, gsz,
                   s.chunks, s.rows_per_slab, partials, tickets, opts.resid);
}

}  // namespace

int64_t sparse_workspace_bytes(int64_t H, int64_t k) {
  // the vector and scalar shapes differ; reserve the larger of the two
  const DownShape a = down_shape(H, k, true);
  const DownShape b = down_shape(H, k, false);
  const int64_t slabs = a.row_slabs > b.row_slabs ? a.row_slabs : b.row_slabs;
  return ticket_bytes(H) + slabs * H * (int64_t)sizeof(float);
}

int64_t sparse_static_scratch_bytes() { return kStaticScratchBytes; }

cudaError_t sparse_static_scratch(void** scratch, cudaStream_t stream) {
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {  // first use on this device: resolve the symbol, clear the tickets
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_sparse_scratch);
    if (e != cudaSuccess) return e;
    e = cudaMemsetAsync(p, 0, (size_t)kCounterBytes, stream);
    if (e != cudaSuccess) return e;
    addr[dev] = p;
  }
  *scratch = addr[dev];
  return cudaSuccess;
}

cudaError_t launch_sparse_down(RowMode mode, const RowSource& src, const half* h, half* y, int64_t H, int64_t k,
                               int64_t group_size, void* workspace, cudaStream_t stream, LaunchOpts opts) {
  switch (mode) {
    case RowMode::kPlain:
      return launch_mode<RowMode::kPlain>(src, h, y, H, k, group_size, workspace, stream, opts);
    case RowMode::kIndexed:
      return launch_mode<RowMode::kIndexed>(src, h, y, H, k, group_size, workspace, stream, opts);
    case RowMode::kDesc:
      return launch_mode<RowMode::kDesc>(src, h, y, H, k, group_size, workspace, stream, opts);
  }
  return cudaErrorInvalidValue;
}

}  // namespace soinfer
