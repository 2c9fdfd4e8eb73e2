// Tensor-parallel exchanges over peer memory (NVLink P2P stores; no
// multicast, no library collective): the row-parallel all-reduce fused with
// the residual add and the next RMSNorm, an all-gather, and the cross-rank
// greedy-token agreement.  Protocol and buffer layout: peer.cuh.
//
// Each exchange is one CTA: the payloads are small at batch-1 decode (a
// 5120-wide fp16 partial is 10 KB per rank), so latency -- one push, one
// flag round trip -- is what matters, and a single CTA keeps the RMSNorm's
// sum of squares on chip.  Pushes are 16-byte stores into every rank's inbox;
// the reduction reads only local memory, in rank order, so every rank
// computes bit-identical results.
#include "common.cuh"
#include "kernels.h"
#include "peer.cuh"

namespace soinfer {
namespace {

__device__ int g_tp_error;

constexpr int kThreads = 512;

__global__ void __launch_bounds__(kThreads)
    tp_allreduce_norm_kernel(const PeerSet ps, const half* __restrict__ partial, const half* __restrict__ residual,
                             const half* __restrict__ w, half* __restrict__ out_sum, half* __restrict__ out_norm,
                             const int n, const float eps) {
  __shared__ float s_part[kThreads / 32];
  __shared__ float s_inv;
  pdl_wait();
  const int tid = threadIdx.x;
  const uint32_t e = peer_next_epoch(ps);
  const int par = (int)(e & 1u);
  const int n8 = n / 8;
  if (partial != nullptr) {
    for (int i = tid; i < n8; i += kThreads) {
      const uint4 v = __ldcg(reinterpret_cast<const uint4*>(partial) + i);
      for (int r = 0; r < ps.world; ++r) reinterpret_cast<uint4*>(peer_slot(ps, r, par, ps.rank))[i] = v;
    }
    peer_signal_all(ps, par, e);
  }
  const bool ok = peer_wait_all(ps, par, e, &g_tp_error, kErrPeerTimeout);
  if (ok) {
    float ss = 0.f;
    for (int i = tid; i < n8; i += kThreads) {
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
      for (int r = 0; r < ps.world; ++r) {
        const uint4 v = __ldcg(reinterpret_cast<const uint4*>(peer_slot(ps, ps.rank, par, r)) + i);
        const half2* h = reinterpret_cast<const half2*>(&v);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(h[j]);
          acc[2 * j] += f.x;
          acc[2 * j + 1] += f.y;
        }
      }
      uint4 res = make_uint4(0, 0, 0, 0);
      if (residual) res = __ldcg(reinterpret_cast<const uint4*>(residual) + i);
      const half2* rh = reinterpret_cast<const half2*>(&res);
      uint4 outv;
      half2* oh = reinterpret_cast<half2*>(&outv);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const half2 o = __floats2half2_rn(acc[2 * j], acc[2 * j + 1]);  // the all-reduced fp16 partial sum
        half2 hv = o;
        if (residual) {
          const float2 a = __half22float2(rh[j]), b = __half22float2(o);
          hv = __floats2half2_rn(a.x + b.x, a.y + b.y);
        }
        oh[j] = hv;
        const float2 f = __half22float2(hv);
        ss += f.x * f.x + f.y * f.y;
      }
      reinterpret_cast<uint4*>(out_sum)[i] = outv;
    }
    if (out_norm != nullptr) {
      ss = warp_sum(ss);
      if ((tid & 31) == 0) s_part[tid >> 5] = ss;
      __syncthreads();
      if (tid == 0) {
        float t = 0.f;
        for (int i = 0; i < kThreads / 32; ++i) t += s_part[i];
        s_inv = rsqrtf(t / (float)n + eps);
      }
      __syncthreads();
      const float inv = s_inv;
      for (int i = tid; i < n8; i += kThreads) {
        const uint4 hv = reinterpret_cast<const uint4*>(out_sum)[i];  // written by this thread above
        const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w) + i);
        const half2* hh = reinterpret_cast<const half2*>(&hv);
        const half2* wh = reinterpret_cast<const half2*>(&wv);
        uint4 nv;
        half2* nh = reinterpret_cast<half2*>(&nv);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(hh[j]), g = __half22float2(wh[j]);
          nh[j] = __floats2half2_rn(f.x * inv * g.x, f.y * inv * g.y);
        }
        reinterpret_cast<uint4*>(out_norm)[i] = nv;
      }
    }
  }
  __syncthreads();
  if (tid == 0 && ok) *peer_epoch(ps) = (int)e;  // a timed-out exchange is not counted (see peer.cuh)
}

__global__ void __launch_bounds__(kThreads)
    tp_allgather_kernel(const PeerSet ps, const uint4* __restrict__ local, const int n16, uint4* __restrict__ out) {
  pdl_wait();
  const int tid = threadIdx.x;
  const uint32_t e = peer_next_epoch(ps);
  const int par = (int)(e & 1u);
  for (int i = tid; i < n16; i += kThreads) {
    const uint4 v = __ldcg(local + i);
    for (int r = 0; r < ps.world; ++r) reinterpret_cast<uint4*>(peer_slot(ps, r, par, ps.rank))[i] = v;
  }
  peer_signal_all(ps, par, e);
  const bool ok = peer_wait_all(ps, par, e, &g_tp_error, kErrPeerTimeout);
  if (ok) {
    for (int r = 0; r < ps.world; ++r) {
      const uint4* src = reinterpret_cast<const uint4*>(peer_slot(ps, ps.rank, par, r));
      for (int i = tid; i < n16; i += kThreads) out[(int64_t)r * n16 + i] = __ldcg(src + i);
    }
  }
  __syncthreads();
  if (tid == 0 && ok) *peer_epoch(ps) = (int)e;  // a timed-out exchange is not counted (see peer.cuh)
}

// fp16 bits -> order-preserving key (the fused LM-head argmax's key).
__device__ __forceinline__ uint32_t half_order_key(half h) {
  uint32_t b = __half_as_ushort(h);
  if (b == 0x8000u) b = 0;
  return (b & 0x8000u) ? (0xFFFFu - b) : (b | 0x8000u);
}

__global__ void tp_argmax_kernel(const PeerSet ps, const half* __restrict__ logits,
                                 const int32_t* __restrict__ local_idx, const int64_t offset,
                                 int32_t* __restrict__ out_idx) {
  pdl_wait();
  const int tid = threadIdx.x;
  const uint32_t e = peer_next_epoch(ps);
  const int par = (int)(e & 1u);
  if (tid < ps.world) {
    const int32_t li = __ldcg(local_idx);
    const half h = logits[li];
    const uint32_t gi = (uint32_t)(li + offset);
    const unsigned long long key = ((unsigned long long)half_order_key(h) << 32) | (0xFFFFFFFFu - gi);
    *reinterpret_cast<unsigned long long*>(peer_slot(ps, tid, par, ps.rank)) = key;
  }
  peer_signal_all(ps, par, e);
  const bool ok = peer_wait_all(ps, par, e, &g_tp_error, kErrPeerTimeout);
  if (ok && tid == 0) {
    unsigned long long best = 0;
    for (int r = 0; r < ps.world; ++r) {
      const unsigned long long k = __ldcg(reinterpret_cast<const unsigned long long*>(peer_slot(ps, ps.rank, par, r)));
      best = k > best ? k : best;
    }
    *out_idx = (int32_t)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
  }
  __syncthreads();
  if (tid == 0 && ok) *peer_epoch(ps) = (int)e;  // a timed-out exchange is not counted (see peer.cuh)
}

}  // namespace

cudaError_t launch_tp_allreduce_norm(const PeerSet& ps, const half* partial, const half* residual, const half* w,
                                     half* out_sum, half* out_norm, int64_t n, float eps, cudaStream_t stream) {
  tp_allreduce_norm_kernel<<<1, kThreads, 0, stream>>>(ps, partial, residual, w, out_sum, out_norm, (int)n, eps);
  return cudaGetLastError();
}

cudaError_t launch_tp_allgather(const PeerSet& ps, const void* local, int64_t nbytes, void* out, cudaStream_t stream) {
  tp_allgather_kernel<<<1, kThreads, 0, stream>>>(ps, reinterpret_cast<const uint4*>(local), (int)(nbytes / 16),
                                                  reinterpret_cast<uint4*>(out));
  return cudaGetLastError();
}

cudaError_t launch_tp_argmax(const PeerSet& ps, const half* logits, const int32_t* local_idx, int64_t offset,
                             int32_t* out_idx, cudaStream_t stream) {
  tp_argmax_kernel<<<1, 32, 0, stream>>>(ps, logits, local_idx, offset, out_idx);
  return cudaGetLastError();
}

cudaError_t read_and_clear_tp_error(int* out) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(out, g_tp_error, sizeof(int));
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(g_tp_error, &zero, sizeof(int));
}

}  // namespace soinfer
