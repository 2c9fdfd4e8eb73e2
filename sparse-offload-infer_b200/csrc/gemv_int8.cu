// INT8 (symmetric, fp32 per-tensor / per-channel / group scales) GEMV.
//
// Fast path (K % 64 == 0, 16-byte aligned, one scale per row or group_size %
// 64 == 0): 128-bit streaming weight loads, int8 -> exact fp16 via PRMT of the
// biased bytes under the fp16 exponent of 1024 (value 1024 + v + 128, minus
// 1152), and mma.sync.m16n8k16 dot products with fp32 accumulation, one
// 64-wide K chunk per MMA group (4 MMAs).  Same tile / cluster split-K scheme
// as the INT4 kernel (gemv_int4.cu).
//
// Reference semantics followed: csrc/kernels/gemv_w8a16.cu:22-62
// (y[n] = half(sum_k scale[n*stride + k/g] * q[n,k] * x[k])).
#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"

namespace cg = cooperative_groups;

namespace soinfer {
namespace {

constexpr int kWarps = 4;
constexpr int kUnroll = 4;
constexpr int kTargetCtas = 296;

// Four int8 (one word) -> two half2 {v0,v1}, {v2,v3}, exact.
__device__ __forceinline__ void unpack_int8x4(uint32_t w, uint32_t& p01, uint32_t& p23) {
  const uint32_t u = w ^ 0x80808080u;  // byte' = v + 128
  const half2 k1152 = __floats2half2_rn(1152.f, 1152.f);
  p01 = h2_as_u32(__hsub2(u32_as_h2(__byte_perm(u, 0x64646464u, 0x4140)), k1152));
  p23 = h2_as_u32(__hsub2(u32_as_h2(__byte_perm(u, 0x64646464u, 0x4342)), k1152));
}

// chunk = 64 K values = 64 bytes per row; thread t of a row quad reads bytes
// [64c + 16t, +16), i.e. words 16c + 4t + j covering k = 64c + 16t + 4j + {0..3}.
__global__ void __launch_bounds__(kWarps * 32)
    gemv_w8_mma_kernel(const int8_t* __restrict__ Wq, const float* __restrict__ scale, const half* __restrict__ x,
                       half* __restrict__ y, const int nrows, const int64_t K, const int chunks,
                       const int chunks_per_group, const int scale_row_stride, const int per_row_scale) {
  extern __shared__ uint2 xs2[];  // 4 halfs per uint2; 16 uint2 per chunk
  __shared__ float red[kWarps][16];
  __shared__ float tile_sum[16];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2;
  const int t = lane & 3;
  const int splits = gridDim.y;
  const int split = blockIdx.y;
  const int64_t row0 = (int64_t)blockIdx.x * 16 + g;
  const int64_t row1 = row0 + 8;
  const int c_begin = (int)(((int64_t)chunks * split) / splits);
  const int c_end = (int)(((int64_t)chunks * (split + 1)) / splits);
  pdl_launch_dependents();

  const int64_t r0 = row0 < nrows ? row0 : nrows - 1;
  const int64_t r1 = row1 < nrows ? row1 : nrows - 1;
  const int8_t* w0 = Wq + r0 * K + t * 16;
  const int8_t* w1 = Wq + r1 * K + t * 16;
  const float* s0 = scale + r0 * scale_row_stride;
  const float* s1 = scale + r1 * scale_row_stride;

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
  load_batch(cb, wa, wb);
  pdl_wait();
  {
    const uint2* xg = reinterpret_cast<const uint2*>(x) + (int64_t)c_begin * 16;
    const int n = (c_end - c_begin) * 16;
    for (int i = threadIdx.x; i < n; i += kWarps * 32) xs2[i] = __ldcg(xg + i);
  }
  __syncthreads();

  float acc0 = 0.f, acc1 = 0.f;
  float grp0 = 0.f, grp1 = 0.f;  // running sums within one scale group (per-row-scale mode)
  while (cb < c_end) {
    const int next = cb + kWarps * kUnroll;
    uint4 na[kUnroll], nb[kUnroll];
    if (next < c_end) load_batch(next, na, nb);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int c = cb + u * kWarps;
      if (c < c_end) {
        const uint2* xc = xs2 + (c - c_begin) * 16 + t * 4;
        const uint32_t q0[4] = {wa[u].x, wa[u].y, wa[u].z, wa[u].w};
        const uint32_t q1[4] = {wb[u].x, wb[u].y, wb[u].z, wb[u].w};
        float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint2 xv = xc[j];  // x[64c + 16t + 4j .. +4)
          uint32_t a01, a23, b01, b23;
          unpack_int8x4(q0[j], a01, a23);
          unpack_int8x4(q1[j], b01, b23);
          const uint32_t a[4] = {a01, b01, a23, b23};
          mma_16816(d, a, xv.x, xv.y);
        }
        if (per_row_scale) {
          grp0 += d[0];
          grp1 += d[2];
        } else {
          const int grp = c / chunks_per_group;
          acc0 = fmaf(__ldg(s0 + grp), d[0], acc0);
          acc1 = fmaf(__ldg(s1 + grp), d[2], acc1);
        }
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
  if (per_row_scale) {
    acc0 = __ldg(s0) * grp0;
    acc1 = __ldg(s1) * grp1;
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
  cluster.sync();
}

// Generic path: warp per row, lanes strided over bytes in 4-byte words when
// aligned, scalar otherwise; fp32 arithmetic.
__global__ void __launch_bounds__(128)
    gemv_w8_simt_kernel(const int8_t* __restrict__ Wq, const float* __restrict__ scale, const half* __restrict__ x,
                        half* __restrict__ y, const int64_t nrows, const int64_t K, const int64_t gsz,
                        const int64_t scale_row_stride) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 4 + warp;
  pdl_launch_dependents();
  pdl_wait();
  if (row >= nrows) return;
  const int8_t* w = Wq + row * K;
  const float* s = scale + row * scale_row_stride;
  float acc = 0.f;
  for (int64_t k = lane; k < K; k += 32) acc += s[k / gsz] * (float)w[k] * __half2float(x[k]);
  acc = warp_sum(acc);
  if (lane == 0) y[row] = __float2half_rn(acc);
}

}  // namespace

cudaError_t launch_gemv_w8(const int8_t* Wq, const float* scale, const half* x, half* y, int64_t N, int64_t K,
                           int64_t group_size, int64_t num_groups, int64_t scale_row_stride, cudaStream_t stream,
                           LaunchOpts opts) {
  auto aligned16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const bool per_row = (num_groups == 1);
  const bool mma_ok = (K % 64 == 0) && aligned16(Wq) && aligned16(x) && (per_row || group_size % 64 == 0) &&
                      N < (1ll << 31) && K / 64 < (1 << 30);
  // per-row scale: the whole row is one group
  const int64_t gsz = per_row ? K : group_size;
  if (mma_ok) {
    const int chunks = (int)(K / 64);
    const int tiles = (int)((N + 15) / 16);
    int splits = 1;
    while ((int64_t)tiles * splits < kTargetCtas && splits < 8 && chunks / (splits * 2) >= kWarps) splits *= 2;
    const int max_chunks = (chunks + splits - 1) / splits;
    const size_t smem = (size_t)max_chunks * 128;
    if (smem > 48 * 1024) {
      cudaError_t e =
          cudaFuncSetAttribute(gemv_w8_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
    }
    const int cpg = per_row ? chunks : (int)(group_size / 64);
    return launch_ex(gemv_w8_mma_kernel, dim3(tiles, splits), dim3(kWarps * 32), smem, stream, splits, opts.pdl,
                     Wq, scale, x, y, (int)N, K, chunks, cpg, (int)scale_row_stride, per_row ? 1 : 0);
  }
  const int64_t blocks = (N + 3) / 4;
  return launch_ex(gemv_w8_simt_kernel, dim3((unsigned)blocks), dim3(128), 0, stream, 1, opts.pdl, Wq, scale, x, y,
                   N, K, gsz, scale_row_stride);
}

}  // namespace soinfer
