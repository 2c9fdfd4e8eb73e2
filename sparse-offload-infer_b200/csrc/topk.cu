// DIP channel selectors and cache descriptors.
//
// Reference selector (csrc/kernels/topk_select.cu:17-95): lo = 0,
// hi = max(0, max v) + 1e-3f, 24 fp32 bisection steps mid = 0.5f*(lo+hi)
// keeping count(v >= lo) >= k, then a single-thread ascending scan writes the
// first k indices with v >= lo.  It runs 24 counting passes on one CTA plus an
// O(n) serial scan.
//
// Here: count(v >= mid) >= k holds exactly when the k-th largest value is
// >= mid, so one radix select (4 passes of 8 bits over order-preserving float
// keys, warp-aggregated shared-memory histograms) yields the k-th largest
// value, one thread replays the 24 bisection steps on that single number
// (bit-identical tau, no counting), and a block-wide ballot/prefix-scan
// compaction writes the qualifying indices in ascending order.  The exact
// mode reuses the radix select and resolves ties at the k-th value by the
// lower index.  One CTA of 1024 threads; keys stay in shared memory when n
// fits (n <= 49152), otherwise every pass re-reads v from L2.
//
// The DIP decode path selects on |fp16 gate| (reference: gate.float().abs()):
// those values are exact fp16 magnitudes, so their order is the order of the
// 15-bit |h| patterns -- topk_abs_half_kernel radix-selects on 16-bit keys in
// two 8-bit passes, replays the same bisection, and compacts with one
// block-wide scan (each warp owns a contiguous run of indices), in a fraction
// of the general kernel's barriers.
#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"

namespace soinfer {
namespace {

constexpr int kThreads = 1024;
constexpr int kWarpsPerBlock = kThreads / 32;
constexpr int64_t kSmemKeysMax = 49152;
constexpr int kBisectionSteps = 24;  // reference topk_select.cu:7
constexpr int kLoadBatch = 4;        // 16-byte input loads in flight per thread

// Order-preserving map float -> uint32 (larger float -> larger key).
// NaN -> 0 (below -inf), -0 -> +0.
__device__ __forceinline__ uint32_t float_key(float f) {
  uint32_t u = __float_as_uint(f);
  if (f != f) return 0u;
  if (u == 0x80000000u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);  // key 0 -> NaN
}

// Exclusive prefix over the block's warp totals.  Returns this warp's offset;
// *total receives the block total.  Contains two __syncthreads().
__device__ __forceinline__ int block_warp_scan(int warp_total, int* s_warp, int* s_total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) s_warp[warp] = warp_total;
  __syncthreads();
  if (warp == 0) {
    const int v = s_warp[lane];
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += u;
    }
    s_warp[lane] = incl - v;
    if (lane == 31) *s_total = incl;
  }
  __syncthreads();
  return s_warp[warp];
}

// Selector input: fp32 values, or (HALF_ABS) |x| of fp16 values -- exactly
// the fp32 tensor gate.float().abs() that the reference feeds the selector.
template <bool HALF_ABS>
__device__ __forceinline__ float sel_value(const void* v, int i) {
  if (HALF_ABS) return fabsf(__half2float(static_cast<const half*>(v)[i]));
  return static_cast<const float*>(v)[i];
}

template <bool EXACT, bool SMEM, bool HALF_ABS>
__global__ void __launch_bounds__(kThreads)
    topk_kernel(const void* __restrict__ v, const int n, const int k, int32_t* __restrict__ out_idx,
                int32_t* __restrict__ out_count) {
  extern __shared__ __align__(16) uint32_t skeys[];
  __shared__ uint32_t hist[256];
  __shared__ int s_warp[kWarpsPerBlock];
  __shared__ int s_warp2[kWarpsPerBlock];
  __shared__ int s_total, s_total2;
  __shared__ float s_wmax[kWarpsPerBlock];
  __shared__ uint32_t s_prefix;
  __shared__ int s_remaining;
  __shared__ float s_tau;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_launch_dependents();
  pdl_wait();

  // 1) keys (+ max for the reference's upper bisection bound)
  float lmax = 0.f;  // reference: local_max starts at 0 (topk_select.cu:19)
  if (SMEM && !HALF_ABS && (n & 3) == 0 && (reinterpret_cast<uintptr_t>(v) & 15u) == 0) {
    // 16-byte loads, kLoadBatch per thread in flight before the first use
    const float4* v4 = static_cast<const float4*>(v);
    const int n4 = n >> 2;
    for (int i0 = tid; i0 < n4; i0 += kThreads * kLoadBatch) {
      float4 f[kLoadBatch];
#pragma unroll
      for (int r = 0; r < kLoadBatch; ++r) {
        const int i = i0 + r * kThreads;
        f[r] = i < n4 ? __ldcg(v4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int r = 0; r < kLoadBatch; ++r) {
        const int i = i0 + r * kThreads;
        if (i < n4) {
          lmax = fmaxf(fmaxf(lmax, fmaxf(f[r].x, f[r].y)), fmaxf(f[r].z, f[r].w));
          reinterpret_cast<uint4*>(skeys)[i] =
              make_uint4(float_key(f[r].x), float_key(f[r].y), float_key(f[r].z), float_key(f[r].w));
        }
      }
    }
  } else {
    for (int i = tid; i < n; i += kThreads) {
      const float f = sel_value<HALF_ABS>(v, i);
      lmax = fmaxf(lmax, f);
      if (SMEM) skeys[i] = float_key(f);
    }
  }
  lmax = warp_max(lmax);
  if (lane == 0) s_wmax[warp] = lmax;
  __syncthreads();

  // 2) radix select of the k-th largest key
  uint32_t prefix = 0, mask = 0;
  int remaining = k;
  const int tiles = (n + kThreads - 1) / kThreads;
#pragma unroll 1
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += kThreads) hist[i] = 0;
    __syncthreads();
    for (int tile = 0; tile < tiles; ++tile) {
      const int i = tile * kThreads + tid;
      bool match = false;
      uint32_t bin = 0;
      if (i < n) {
        const uint32_t key = SMEM ? skeys[i] : float_key(sel_value<HALF_ABS>(v, i));
        match = (key & mask) == prefix;
        bin = (key >> shift) & 255u;
      }
      const unsigned active = __ballot_sync(0xffffffffu, match);
      if (match) {
        const unsigned peers = __match_any_sync(active, bin);
        if (lane == __ffs(peers) - 1) atomicAdd(&hist[bin], (uint32_t)__popc(peers));
      }
    }
    __syncthreads();
    if (warp == 0) {
      int c[8];
      int lsum = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = (int)hist[lane * 8 + j];
        lsum += c[j];
      }
      int suf = lsum;  // inclusive suffix sum over lanes >= lane
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_down_sync(0xffffffffu, suf, o);
        if (lane + o < 32) suf += u;
      }
      int cum = suf - lsum;  // keys in bins above this lane's bins
#pragma unroll
      for (int j = 7; j >= 0; --j) {
        if (cum < remaining && cum + c[j] >= remaining) {
          s_prefix = prefix | ((uint32_t)(lane * 8 + j) << shift);
          s_remaining = remaining - cum;
        }
        cum += c[j];
      }
    }
    __syncthreads();
    prefix = s_prefix;
    remaining = s_remaining;
    mask |= 255u << shift;
  }
  const uint32_t kth = prefix;  // k-th largest key; `remaining` of its copies are in the top k

  // 3) reference threshold: replay the bisection on the k-th value
  if (!EXACT && tid == 0) {
    float m = 0.f;
    for (int w = 0; w < kWarpsPerBlock; ++w) m = fmaxf(m, s_wmax[w]);
    const float kv = key_float(kth);
    float lo = 0.f, hi = m + 1e-3f;
#pragma unroll 1
    for (int it = 0; it < kBisectionSteps; ++it) {
      const float mid = 0.5f * (lo + hi);
      if (kv >= mid)  // == (count(v >= mid) >= k); false for NaN
        lo = mid;
      else
        hi = mid;
    }
    s_tau = lo;
  }
  __syncthreads();
  const float tau = EXACT ? 0.f : s_tau;

  // 4) ordered compaction
  int base = 0, tie_base = 0;
  for (int tile = 0; tile < tiles && base < k; ++tile) {
    const int i = tile * kThreads + tid;
    const bool valid = i < n;
    const uint32_t key = valid ? (SMEM ? skeys[i] : float_key(sel_value<HALF_ABS>(v, i))) : 0u;
    const unsigned lt_mask = (1u << lane) - 1u;
    bool sel;
    if (EXACT) {
      const bool gt = valid && key > kth;
      const bool tie = valid && key == kth;
      const unsigned bt = __ballot_sync(0xffffffffu, tie);
      const int tie_off = block_warp_scan(__popc(bt), s_warp2, &s_total2);
      const int tie_rank = tie_base + tie_off + __popc(bt & lt_mask);
      sel = gt || (tie && tie_rank < remaining);
      tie_base += s_total2;
    } else {
      sel = valid && key_float(key) >= tau;
    }
    const unsigned bs = __ballot_sync(0xffffffffu, sel);
    const int off = block_warp_scan(__popc(bs), s_warp, &s_total);
    const int pos = base + off + __popc(bs & lt_mask);
    if (sel && pos < k) out_idx[pos] = i;
    base += s_total;
    __syncthreads();  // s_warp / s_total are rewritten by the next tile
  }
  const int count = base < k ? base : k;
  for (int p = count + tid; p < k; p += kThreads) out_idx[p] = -1;
  if (tid == 0) *out_count = count;
}

// |fp16| keys: the magnitude bits; NaN ranks below every number (key 0), as
// float_key does for the general kernel.
__device__ __forceinline__ uint32_t abs_half_key(uint16_t bits) {
  const uint32_t m = bits & 0x7fffu;
  return m > 0x7c00u ? 0u : m;
}

// Selects bin b with sum(counts of bins > b) < remaining <= sum(counts of bins >= b)
// over hist[256] (warp 0); writes s_bin / s_rem (remaining within the bin).
__device__ __forceinline__ void pick_bin(const uint32_t* hist, int remaining, uint32_t* s_bin, int* s_rem) {
  const int lane = threadIdx.x & 31;
  int c[8];
  int lsum = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    c[j] = (int)hist[lane * 8 + j];
    lsum += c[j];
  }
  int suf = lsum;  // inclusive suffix sum over lanes >= lane
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_down_sync(0xffffffffu, suf, o);
    if (lane + o < 32) suf += u;
  }
  int cum = suf - lsum;
#pragma unroll
  for (int j = 7; j >= 0; --j) {
    if (cum < remaining && cum + c[j] >= remaining) {
      *s_bin = (uint32_t)(lane * 8 + j);
      *s_rem = remaining - cum;
    }
    cum += c[j];
  }
}

__global__ void __launch_bounds__(kThreads)
    topk_abs_half_kernel(const half* __restrict__ v, const int n, const int k, int32_t* __restrict__ out_idx,
                         int32_t* __restrict__ out_count) {
  extern __shared__ __align__(16) uint16_t sbits[];  // [n] raw fp16 bits
  __shared__ uint32_t hist[256];
  __shared__ int s_warp[kWarpsPerBlock];
  __shared__ int s_total;
  __shared__ float s_wmax[kWarpsPerBlock];
  __shared__ uint32_t s_bin;
  __shared__ int s_rem;
  __shared__ float s_tau;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_launch_dependents();
  pdl_wait();
  const uint16_t* vb = reinterpret_cast<const uint16_t*>(v);
  float lmax = 0.f;  // reference: local_max starts at 0 (topk_select.cu:19)
  if ((n & 7) == 0 && (reinterpret_cast<uintptr_t>(v) & 15u) == 0) {
    // 16-byte loads, kLoadBatch per thread in flight before the first use
    const uint4* v8 = reinterpret_cast<const uint4*>(v);
    const int n8 = n >> 3;
    for (int i0 = tid; i0 < n8; i0 += kThreads * kLoadBatch) {
      uint4 u[kLoadBatch];
#pragma unroll
      for (int r = 0; r < kLoadBatch; ++r) {
        const int i = i0 + r * kThreads;
        u[r] = i < n8 ? __ldcg(v8 + i) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int r = 0; r < kLoadBatch; ++r) {
        const int i = i0 + r * kThreads;
        if (i < n8) {
          reinterpret_cast<uint4*>(sbits)[i] = u[r];
          const half2* hp = reinterpret_cast<const half2*>(&u[r]);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(hp[e]);
            lmax = fmaxf(lmax, fmaxf(fabsf(f.x), fabsf(f.y)));
          }
        }
      }
    }
  } else {
    for (int i = tid; i < n; i += kThreads) {
      const uint16_t b = vb[i];
      sbits[i] = b;
      lmax = fmaxf(lmax, fabsf(__half2float(__ushort_as_half(b))));
    }
  }
  for (int i = tid; i < 256; i += kThreads) hist[i] = 0;
  lmax = warp_max(lmax);
  if (lane == 0) s_wmax[warp] = lmax;
  __syncthreads();
  // pass 1: high byte of the 16-bit key
  for (int i = tid; i < n; i += kThreads) atomicAdd(&hist[abs_half_key(sbits[i]) >> 8], 1u);
  __syncthreads();
  if (warp == 0) pick_bin(hist, k, &s_bin, &s_rem);
  __syncthreads();
  const uint32_t hi = s_bin;
  const int rem1 = s_rem;
  for (int i = tid; i < 256; i += kThreads) hist[i] = 0;
  __syncthreads();
  // pass 2: low byte among the keys in that bin
  for (int i = tid; i < n; i += kThreads) {
    const uint32_t key = abs_half_key(sbits[i]);
    if ((key >> 8) == hi) atomicAdd(&hist[key & 255u], 1u);
  }
  __syncthreads();
  if (warp == 0) pick_bin(hist, rem1, &s_bin, &s_rem);
  __syncthreads();
  const uint32_t kth = (hi << 8) | s_bin;  // the k-th largest |h| (NaN-free: key 0 == +0)
  // the reference threshold: replay the bisection on the k-th value
  if (tid == 0) {
    float m = 0.f;
    for (int w = 0; w < kWarpsPerBlock; ++w) m = fmaxf(m, s_wmax[w]);
    const float kv = __half2float(__ushort_as_half((uint16_t)kth));
    float lo = 0.f, hi_b = m + 1e-3f;
#pragma unroll 1
    for (int it = 0; it < kBisectionSteps; ++it) {
      const float mid = 0.5f * (lo + hi_b);
      if (kv >= mid)
        lo = mid;
      else
        hi_b = mid;
    }
    s_tau = lo;
  }
  __syncthreads();
  const float tau = s_tau;
  // ordered compaction: warp w owns indices [w * chunk, (w + 1) * chunk)
  const int chunk = ((n + kWarpsPerBlock - 1) / kWarpsPerBlock + 31) & ~31;
  const int c0 = warp * chunk, c1 = min(n, c0 + chunk);
  int wcount = 0;
  for (int i0 = c0; i0 < c1; i0 += 32) {
    const int i = i0 + lane;
    const bool sel = i < c1 && fabsf(__half2float(__ushort_as_half(sbits[i]))) >= tau;
    wcount += __popc(__ballot_sync(0xffffffffu, sel));
  }
  const int wbase = block_warp_scan(wcount, s_warp, &s_total);
  int run = wbase;
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int i0 = c0; i0 < c1 && run < k; i0 += 32) {
    const int i = i0 + lane;
    const bool sel = i < c1 && fabsf(__half2float(__ushort_as_half(sbits[i]))) >= tau;
    const unsigned bs = __ballot_sync(0xffffffffu, sel);
    const int pos = run + __popc(bs & lt_mask);
    if (sel && pos < k) out_idx[pos] = i;
    run += __popc(bs);
  }
  const int total = s_total;
  const int count = total < k ? total : k;
  for (int p = count + tid; p < k; p += kThreads) out_idx[p] = -1;
  if (tid == 0) *out_count = count;
}

__global__ void __launch_bounds__(kThreads)
    descriptors_kernel(const int32_t* __restrict__ sel, const int k, const int32_t* __restrict__ slot_of, const int I,
                       int32_t* __restrict__ desc, int32_t* __restrict__ miss, int32_t* __restrict__ miss_count) {
  __shared__ int s_warp[kWarpsPerBlock];
  __shared__ int s_total;
  const int tid = threadIdx.x, lane = tid & 31;
  pdl_launch_dependents();
  pdl_wait();
  int base = 0;
  const int tiles = (k + kThreads - 1) / kThreads;
  for (int tile = 0; tile < tiles; ++tile) {
    const int j = tile * kThreads + tid;
    const bool valid = j < k;
    int c = 0, slot = 0;
    if (valid) {
      c = sel[j];
      c = c < 0 ? 0 : (c >= I ? I - 1 : c);
      slot = slot_of[c];
    }
    const bool is_miss = valid && slot < 0;
    const unsigned bm = __ballot_sync(0xffffffffu, is_miss);
    const int off = block_warp_scan(__popc(bm), s_warp, &s_total);
    const int pos = base + off + __popc(bm & ((1u << lane) - 1u));
    if (valid) desc[j] = is_miss ? (int32_t)((uint32_t)pos | 0x80000000u) : slot;
    if (is_miss) miss[pos] = c;
    base += s_total;
    __syncthreads();
  }
  if (tid == 0) *miss_count = base;
}

}  // namespace

namespace {

template <bool HALF_ABS>
cudaError_t launch_topk_impl(bool exact, const void* v, int64_t n, int64_t k, int32_t* out_idx, int32_t* out_count,
                             cudaStream_t stream) {
  const bool smem = n <= kSmemKeysMax;
  const size_t bytes = smem ? (size_t)n * sizeof(uint32_t) : 0;
  void (*kernel)(const void*, int, int, int32_t*, int32_t*);
  if (exact)
    kernel = smem ? topk_kernel<true, true, HALF_ABS> : topk_kernel<true, false, HALF_ABS>;
  else
    kernel = smem ? topk_kernel<false, true, HALF_ABS> : topk_kernel<false, false, HALF_ABS>;
  if (bytes > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) return e;
  }
  return launch_ex(kernel, dim3(1), dim3(kThreads), bytes, stream, 1, true /* programmatic dependent: waits first */, v, (int)n, (int)k, out_idx, out_count);
}

}  // namespace

cudaError_t launch_topk(bool exact, const float* v, int64_t n, int64_t k, int32_t* out_idx, int32_t* out_count,
                        cudaStream_t stream) {
  return launch_topk_impl<false>(exact, v, n, k, out_idx, out_count, stream);
}

cudaError_t launch_topk_abs_half(bool exact, const half* v, int64_t n, int64_t k, int32_t* out_idx,
                                 int32_t* out_count, cudaStream_t stream) {
  if (!exact && n <= 2 * kSmemKeysMax) {
    const size_t bytes = (size_t)n * sizeof(uint16_t);
    if (bytes > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(topk_abs_half_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)bytes);
      if (e != cudaSuccess) return e;
    }
    return launch_ex(topk_abs_half_kernel, dim3(1), dim3(kThreads), bytes, stream, 1, true, v, (int)n, (int)k,
                     out_idx, out_count);
  }
  return launch_topk_impl<true>(exact, v, n, k, out_idx, out_count, stream);
}

cudaError_t launch_build_descriptors(const int32_t* sel, int64_t k, const int32_t* slot_of, int64_t I, int32_t* desc,
                                     int32_t* miss, int32_t* miss_count, cudaStream_t stream) {
  return launch_ex(descriptors_kernel, dim3(1), dim3(kThreads), 0, stream, 1, true /* programmatic dependent: waits first */, sel, (int)k, slot_of, (int)I,
                   desc, miss, miss_count);
}

}  // namespace soinfer
