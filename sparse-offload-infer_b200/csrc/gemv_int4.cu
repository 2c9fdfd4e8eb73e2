// INT4 (AWQ-order, symmetric, fp32 group scales) GEMV for batch-1 decode.
//
// Fast path (group_size % 128 == 0, K % 128 == 0, 16-byte aligned operands):
// the weights stream through 128-bit non-allocating loads; each 32-bit word
// is unpacked to exact fp16 integers in registers (one LOP3 per half2, see
// common.cuh), and the dot products run on the tensor pipe with
// mma.sync.m16n8k16 (fp16 x fp16 products are exact, accumulation is fp32),
// one MMA group per 128-wide K chunk.  At batch 1 the B operand is x
// replicated across the 8 MMA columns, so every column of D holds the same
// row sums and no cross-lane reduction is needed.  The per-row group scale is
// applied in fp32 once per 128-K chunk.
//
// Why the tensor pipe at batch 1: B200 streams ~23 HBM bytes per SM per
// clock, i.e. ~2.8 SIMT instructions per INT4 value at full bandwidth.  An
// fp32 SIMT dot product costs >= 3 instructions per value; an fp16 HFMA2 dot
// product fits the budget but its fp16 partial sums miss the rel-L2 1e-3
// parity bar against the fp32-accumulated reference.  Offloading the
// multiply-add to the MMA leaves ~1.1 SIMT instructions per value (unpack).
//
// Work split: one CTA = 4 warps owns a 16-row tile; its warps interleave over
// 128-K chunks.  When the tile count is too small to fill the GPU the K range
// is split across a thread-block cluster of 2..8 CTAs (cluster dims along y)
// whose partial sums are reduced through distributed shared memory in a fixed
// order, so results are deterministic and independent of the row source.
//
// Reference semantics followed: csrc/kernels/gemv_w4a16_group.cu:77-127
// (y[n] = half(sum_w s[n, 8w/g] * dot(dq(word w), x[8w..8w+8)))) and
// csrc/kernels/gemv_dip_fused.cu:48-102 (descriptor row source).
#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"

namespace cg = cooperative_groups;

namespace soinfer {
namespace {

constexpr int kWarps = 4;   // warps per CTA (fast path)
constexpr int kUnroll = 4;  // 128-K chunks in flight per warp
constexpr int kTargetCtas = 296;

__device__ __forceinline__ int64_t clamp_row(int64_t r, int64_t rows) {
  return r < 0 ? 0 : (r >= rows ? rows - 1 : r);
}

template <RowMode M>
__device__ __forceinline__ void row_ptrs(const RowSource& src, int64_t row, const uint8_t*& w, const float*& s) {
  if constexpr (M == RowMode::kPlain) {
    w = src.W + row * src.row_bytes;
    s = src.S + row * src.num_groups;
  } else if constexpr (M == RowMode::kIndexed) {
    const int64_t r = clamp_row(src.idx[row], src.rows1);
    w = src.W + r * src.row_bytes;
    s = src.S + r * src.num_groups;
  } else {
    const int32_t d = src.idx[row];
    const bool staging = (desc_is_staging(d) && src.rows2 > 0) || src.rows1 == 0;
    if (staging) {
      const int64_t r = clamp_row(desc_offset(d), src.rows2);
      w = src.W2 + r * src.row_bytes;
      s = src.S2 + r * src.num_groups;
    } else {
      const int64_t r = clamp_row(desc_offset(d), src.rows1);
      w = src.W + r * src.row_bytes;
      s = src.S + r * src.num_groups;
    }
  }
}

template <RowMode M>
__global__ void __launch_bounds__(kWarps * 32)
    gemv_w4_mma_kernel(const RowSource src, const half* __restrict__ x, half* __restrict__ y, const int nrows,
                       const int chunks, const int chunks_per_group) {
  extern __shared__ uint4 xs[];  // this CTA's slice of x, 16 uint4 (128 halfs) per chunk
  __shared__ float red[kWarps][16];
  __shared__ float tile_sum[16];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2;  // MMA groupID: rows g and g + 8 of the tile
  const int t = lane & 3;   // MMA thread-in-group: 32-K slice of each chunk
  const int splits = gridDim.y;
  const int split = blockIdx.y;
  const int64_t row0 = (int64_t)blockIdx.x * 16 + g;
  const int64_t row1 = row0 + 8;
  const int c_begin = (int)(((int64_t)chunks * split) / splits);
  const int c_end = (int)(((int64_t)chunks * (split + 1)) / splits);

  pdl_launch_dependents();
  // Row indices / descriptors come from the preceding kernel.
  if constexpr (M != RowMode::kPlain) pdl_wait();

  const uint8_t *w0, *w1;
  const float *s0, *s1;
  row_ptrs<M>(src, row0 < nrows ? row0 : nrows - 1, w0, s0);
  row_ptrs<M>(src, row1 < nrows ? row1 : nrows - 1, w1, s1);
  w0 += t * 16;
  w1 += t * 16;

  uint4 wa[kUnroll], wb[kUnroll];
  auto load_batch = [&](int cb, uint4* a, uint4* b) {
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int c = cb + u * kWarps;
      if (c < c_end) {
        a[u] = ldg_stream_u4(w0 + (int64_t)c * 64);
        b[u] = ldg_stream_u4(w1 + (int64_t)c * 64);
      } else {
        a[u] = make_uint4(0u, 0u, 0u, 0u);
        b[u] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
  };

  int cb = c_begin + warp;
  load_batch(cb, wa, wb);  // weights never depend on the preceding kernel in plain mode

  if constexpr (M == RowMode::kPlain) pdl_wait();
  // Stage x[c_begin*128, c_end*128) into shared memory (L2-coherent loads).
  {
    const uint4* xg = reinterpret_cast<const uint4*>(x) + (int64_t)c_begin * 16;
    const int n16 = (c_end - c_begin) * 16;
    for (int i = threadIdx.x; i < n16; i += kWarps * 32) xs[i] = __ldcg(xg + i);
  }
  __syncthreads();

  float acc0 = 0.f, acc1 = 0.f;
  while (cb < c_end) {
    const int next = cb + kWarps * kUnroll;
    uint4 na[kUnroll], nb[kUnroll];
    if (next < c_end) load_batch(next, na, nb);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int c = cb + u * kWarps;
      if (c < c_end) {
        const uint4* xc = xs + (c - c_begin) * 16 + t * 4;
        const uint32_t r0[4] = {wa[u].x, wa[u].y, wa[u].z, wa[u].w};
        const uint32_t r1[4] = {wb[u].x, wb[u].y, wb[u].z, wb[u].w};
        float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 xv = xc[j];  // x[c*128 + 32t + 8j .. +8): pairs 0..3 of word j
          uint32_t p0[4], p1[4];
          unpack_int4x8(r0[j], p0);
          unpack_int4x8(r1[j], p1);
          const uint32_t a_lo[4] = {p0[0], p1[0], p0[1], p1[1]};
          mma_16816(d, a_lo, xv.x, xv.y);
          const uint32_t a_hi[4] = {p0[2], p1[2], p0[3], p1[3]};
          mma_16816(d, a_hi, xv.z, xv.w);
        }
        const int grp = c / chunks_per_group;
        acc0 = fmaf(__ldg(s0 + grp), d[0], acc0);
        acc1 = fmaf(__ldg(s1 + grp), d[2], acc1);
      }
    }
    if (next < c_end) {
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        wa[u] = na[u];
        wb[u] = nb[u];
      }
    }
    cb = next;
  }

  if (t == 0) {
    red[warp][g] = acc0;
    red[warp][g + 8] = acc1;
  }
  __syncthreads();
  float total = 0.f;
  if (threadIdx.x < 16) {
#pragma unroll
    for (int w = 0; w < kWarps; ++w) total += red[w][threadIdx.x];
    tile_sum[threadIdx.x] = total;
  }
  const int64_t out_row = (int64_t)blockIdx.x * 16 + threadIdx.x;
  if (splits == 1) {
    if (threadIdx.x < 16 && out_row < nrows) y[out_row] = __float2half_rn(total);
    return;
  }
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  if (split == 0 && threadIdx.x < 16) {
    float sum = 0.f;
    for (int r = 0; r < splits; ++r) sum += cluster.map_shared_rank(tile_sum, r)[threadIdx.x];
    if (out_row < nrows) y[out_row] = __float2half_rn(sum);
  }
  cluster.sync();  // keep every CTA's shared memory alive until rank 0 has read it
}

// Generic path: any group_size % 8 == 0, any K, 4-byte aligned rows.  One
// warp per row, lanes strided over packed words, fp32 arithmetic in the
// reference's per-word form acc += s * (dq0*x0 + dq1*x1) per K pair.
template <RowMode M>
__global__ void __launch_bounds__(128)
    gemv_w4_simt_kernel(const RowSource src, const half* __restrict__ x, half* __restrict__ y, const int64_t nrows,
                        const int64_t K, const int64_t gsz) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 4 + warp;
  pdl_launch_dependents();
  pdl_wait();
  if (row >= nrows) return;
  const uint8_t* w;
  const float* s;
  row_ptrs<M>(src, row, w, s);
  const int64_t words = (K + 7) / 8;
  const uint32_t* wp = reinterpret_cast<const uint32_t*>(w);
  float acc = 0.f;
  for (int64_t wi = lane; wi < words; wi += 32) {
    const int64_t k = wi * 8;
    const float sc = s[k / gsz];
    uint32_t p[4];
    unpack_int4x8(ldg_stream_u32(wp + wi), p);
    const int64_t rem = K - k;
    if (rem >= 8) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 d = __half22float2(u32_as_h2(p[j]));
        const float x0 = __half2float(x[k + 2 * j]);
        const float x1 = __half2float(x[k + 2 * j + 1]);
        acc += sc * (d.x * x0 + d.y * x1);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 d = __half22float2(u32_as_h2(p[j]));
        if (2 * j < rem) acc += sc * d.x * __half2float(x[k + 2 * j]);
        if (2 * j + 1 < rem) acc += sc * d.y * __half2float(x[k + 2 * j + 1]);
      }
    }
  }
  acc = warp_sum(acc);
  if (lane == 0) y[row] = __float2half_rn(acc);
}

template <RowMode M>
cudaError_t launch_mode(const RowSource& src, const half* x, half* y, int64_t nrows, int64_t K, int64_t gsz,
                        cudaStream_t stream, LaunchOpts opts) {
  auto aligned16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const bool mma_ok = (K % 128 == 0) && (gsz % 128 == 0) && src.row_bytes % 16 == 0 && aligned16(src.W) &&
                      (M != RowMode::kDesc || aligned16(src.W2)) && aligned16(x) && nrows < (1ll << 31) &&
                      K / 128 < (1 << 30);
  if (mma_ok) {
    const int chunks = (int)(K / 128);
    const int tiles = (int)((nrows + 15) / 16);
    int splits = 1;
    while ((int64_t)tiles * splits < kTargetCtas && splits < 8 && chunks / (splits * 2) >= kWarps) splits *= 2;
    const int max_chunks = (chunks + splits - 1) / splits;
    const size_t smem = (size_t)max_chunks * 256;
    auto kernel = gemv_w4_mma_kernel<M>;
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
    }
    return launch_ex(kernel, dim3(tiles, splits), dim3(kWarps * 32), smem, stream, splits, opts.pdl, src, x, y,
                     (int)nrows, chunks, (int)(gsz / 128));
  }
  const int64_t blocks = (nrows + 3) / 4;
  return launch_ex(gemv_w4_simt_kernel<M>, dim3((unsigned)blocks), dim3(128), 0, stream, 1, opts.pdl, src, x, y,
                   nrows, K, gsz);
}

}  // namespace

cudaError_t launch_gemv_w4(RowMode mode, const RowSource& src, const half* x, half* y, int64_t nrows, int64_t K,
                           int64_t group_size, cudaStream_t stream, LaunchOpts opts) {
  switch (mode) {
    case RowMode::kPlain:
      return launch_mode<RowMode::kPlain>(src, x, y, nrows, K, group_size, stream, opts);
    case RowMode::kIndexed:
      return launch_mode<RowMode::kIndexed>(src, x, y, nrows, K, group_size, stream, opts);
    case RowMode::kDesc:
      return launch_mode<RowMode::kDesc>(src, x, y, nrows, K, group_size, stream, opts);
  }
  return cudaErrorInvalidValue;
}

}  // namespace soinfer
