// fp16 GEMV for the LM head (y = W x, W fp16 [N, K] row-major, fp32
// accumulation, fp16 output; reference csrc/kernels/gemv_fp16.cu:60-95 and
// csrc/bindings.cpp:201-208, gemv_fp16_v3) and the greedy-decode argmax
// fused into it.
//
// At batch 1 the LM head is the largest single matrix of a decode step
// (151936 x 2048 fp16 = 622 MB at 1.7B): pure HBM streaming.  Each warp owns
// rows r = global_warp + i * total_warps and keeps two rows in flight, each
// lane issuing K/256 independent 16-byte loads per row; x is staged once per
// CTA in shared memory.  Grid: a whole number of CTAs per SM.
//
// Argmax: every logit is rounded to fp16 first (the reference takes
// torch.argmax of the fp16 logits), mapped to an order-preserving 32-bit key,
// and packed with the complement of its row index into one 64-bit key, so a
// plain atomicMax picks the largest logit and, among equal ones, the lowest
// index -- torch.argmax's first-occurrence rule -- in any execution order.
// The last CTA (ticket) publishes the index and resets the workspace to zero.
#include "common.cuh"
#include "kernels.h"

namespace soinfer {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kCtasPerSm = 4;

// fp16 bits -> order-preserving unsigned key (NaN sorts above +inf; -0 == +0).
__device__ __forceinline__ uint32_t half_order_key(half h) {
  uint32_t b = __half_as_ushort(h);
  if (b == 0x8000u) b = 0;  // -0 -> +0
  return (b & 0x8000u) ? (0xFFFFu - b) : (b | 0x8000u);
}

__device__ __forceinline__ float dot8(const uint4 w, const uint4 x, float acc) {
  const half2* wh = reinterpret_cast<const half2*>(&w);
  const half2* xh = reinterpret_cast<const half2*>(&x);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 wf = __half22float2(wh[j]);
    const float2 xf = __half22float2(xh[j]);
    acc = fmaf(wf.x, xf.x, acc);
    acc = fmaf(wf.y, xf.y, acc);
  }
  return acc;
}

template <bool ARGMAX>
__global__ void __launch_bounds__(kThreads)
    gemv_fp16_kernel(const half* __restrict__ W, const half* __restrict__ x, half* __restrict__ y, int64_t N,
                     int K, unsigned long long* __restrict__ best, int* __restrict__ ticket,
                     int32_t* __restrict__ out_idx) {
  extern __shared__ __align__(16) uint4 xs[];  // K / 8
  __shared__ unsigned long long s_best[kWarps];
  __shared__ bool s_last;
  const int k8 = K / 8;
  for (int i = threadIdx.x; i < k8; i += kThreads) xs[i] = reinterpret_cast<const uint4*>(x)[i];
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t total_warps = (int64_t)gridDim.x * kWarps;
  unsigned long long my_best = 0;
  for (int64_t r0 = (int64_t)blockIdx.x * kWarps + warp; r0 < N; r0 += 2 * total_warps) {
    const int64_t r1 = r0 + total_warps;
    const bool has1 = r1 < N;
    const uint4* w0 = reinterpret_cast<const uint4*>(W + r0 * K);
    const uint4* w1 = reinterpret_cast<const uint4*>(W + (has1 ? r1 : r0) * K);
    float a0 = 0.f, a1 = 0.f;
    int k = lane;
    for (; k + 96 < k8; k += 128) {  // 4 loads per row in flight per lane
      uint4 u[4], v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) u[j] = ldg_stream_u4(w0 + k + 32 * j);
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = ldg_stream_u4(w1 + k + 32 * j);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 xv = xs[k + 32 * j];
        a0 = dot8(u[j], xv, a0);
        a1 = dot8(v[j], xv, a1);
      }
    }
    for (; k < k8; k += 32) {
      const uint4 xv = xs[k];
      a0 = dot8(ldg_stream_u4(w0 + k), xv, a0);
      a1 = dot8(ldg_stream_u4(w1 + k), xv, a1);
    }
    a0 = warp_sum(a0);
    a1 = warp_sum(a1);
    if (lane == 0) {
      const half h0 = __float2half_rn(a0), h1 = __float2half_rn(a1);
      if (y) {
        y[r0] = h0;
        if (has1) y[r1] = h1;
      }
      if (ARGMAX) {
        const unsigned long long k0 =
            ((unsigned long long)half_order_key(h0) << 32) | (0xFFFFFFFFull - (unsigned long long)r0);
        my_best = k0 > my_best ? k0 : my_best;
        if (has1) {
          const unsigned long long k1 =
              ((unsigned long long)half_order_key(h1) << 32) | (0xFFFFFFFFull - (unsigned long long)r1);
          my_best = k1 > my_best ? k1 : my_best;
        }
      }
    }
  }
  if (!ARGMAX) return;
  if (lane == 0) s_best[warp] = my_best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = 0;
    for (int w = 0; w < kWarps; ++w) b = s_best[w] > b ? s_best[w] : b;
    atomicMax(best, b);
    __threadfence();
    s_last = atomicAdd(ticket, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    __threadfence();
    const unsigned long long b = atomicAdd(best, 0ull);
    *out_idx = (int32_t)(0xFFFFFFFFull - (b & 0xFFFFFFFFull));
    *best = 0;  // leave the workspace zeroed for the next call
    *ticket = 0;
  }
}

int grid_for(int64_t N) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t need = (N + 2 * kWarps - 1) / (2 * kWarps);
  const int64_t g = (int64_t)sms * kCtasPerSm;
  return (int)(need < g ? (need < 1 ? 1 : need) : g);
}

template <bool ARGMAX>
cudaError_t launch(const half* W, const half* x, half* y, int64_t N, int64_t K, unsigned long long* best,
                   int* ticket, int32_t* out_idx, cudaStream_t stream) {
  const size_t smem = (size_t)K * 2;
  auto kernel = gemv_fp16_kernel<ARGMAX>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  kernel<<<grid_for(N), kThreads, smem, stream>>>(W, x, y, N, (int)K, best, ticket, out_idx);
  return cudaGetLastError();
}

}  // namespace

int64_t lm_head_argmax_workspace_bytes() { return 256; }

cudaError_t launch_gemv_fp16(const half* W, const half* x, half* y, int64_t N, int64_t K, cudaStream_t stream) {
  return launch<false>(W, x, y, N, K, nullptr, nullptr, nullptr, stream);
}

cudaError_t launch_gemv_fp16_argmax(const half* W, const half* x, half* y, int64_t N, int64_t K, void* workspace,
                                    int32_t* out_idx, cudaStream_t stream) {
  auto* best = reinterpret_cast<unsigned long long*>(workspace);
  auto* ticket = reinterpret_cast<int*>(reinterpret_cast<char*>(workspace) + 8);
  return launch<true>(W, x, y, N, K, best, ticket, out_idx, stream);
}

}  // namespace soinfer
