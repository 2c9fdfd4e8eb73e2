// Shared device helpers for the sm_100a soinfer kernels.
//
// INT4 unpack: the packing contract (AWQ nibble order [0,2,4,6,1,3,5,7] per
// 32-bit word, two's-complement nibbles; reference csrc/include/layout.h:19-51)
// puts (v0,v1) in nibbles 0/4, (v2,v3) in nibbles 1/5, (v4,v5) in 2/6 and
// (v6,v7) in 3/7.  Masking one nibble per 16-bit half and OR-ing in the fp16
// exponent of 1024 (0x6400) yields the half2 {1024 + n_lo, 1024 + n_hi} with no
// int->float conversion (the published "magic number" int4->fp16 method used
// by FasterTransformer and AWQ).  Signed nibbles are biased by flipping bit 3
// (n ^ 8 == s + 8 for the sign-extended value s), and that XOR is folded into
// the same single LOP3: (w & mask) ^ (0x6400 | 0x8-in-nibble) per half.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace soinfer {

template <typename T>
__host__ __device__ __forceinline__ T ceil_div(T a, T b) {
  return (a + b - 1) / b;
}

// (a & b) ^ c in one LOP3 (truth-table 0x6a = (0xF0 & 0xCC) ^ 0xAA).
__device__ __forceinline__ uint32_t lop3_and_xor(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint32_t h2_as_u32(half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<half2*>(&u); }

// One packed word -> four half2 holding the exact signed values
// {v0,v1}, {v2,v3}, {v4,v5}, {v6,v7} (consecutive K pairs).
__device__ __forceinline__ void unpack_int4x8(uint32_t w, uint32_t out[4]) {
  const uint32_t top = w >> 8;
  const uint32_t lo0 = lop3_and_xor(w, 0x000f000fu, 0x64086408u);    // 1024 + (n ^ 8)
  const uint32_t hi0 = lop3_and_xor(w, 0x00f000f0u, 0x64806480u);    // 1024 + 16 (n ^ 8)
  const uint32_t lo1 = lop3_and_xor(top, 0x000f000fu, 0x64086408u);
  const uint32_t hi1 = lop3_and_xor(top, 0x00f000f0u, 0x64806480u);
  const half2 k1032 = __floats2half2_rn(1032.f, 1032.f);
  const half2 k1_16 = __floats2half2_rn(1.f / 16.f, 1.f / 16.f);
  const half2 km72 = __floats2half2_rn(-72.f, -72.f);
  out[0] = h2_as_u32(__hsub2(u32_as_h2(lo0), k1032));            // (1024+s+8) - 1032 = s
  out[1] = h2_as_u32(__hfma2(u32_as_h2(hi0), k1_16, km72));      // (1024+16(s+8))/16 - 72 = s
  out[2] = h2_as_u32(__hsub2(u32_as_h2(lo1), k1032));
  out[3] = h2_as_u32(__hfma2(u32_as_h2(hi1), k1_16, km72));
}

// Signed value of nibble position j (0..7, logical K order) of a packed word.
__device__ __forceinline__ int int4_value(uint32_t w, int j) {
  // logical j -> nibble slot: even j -> j/2, odd j -> 4 + j/2
  const int slot = (j & 1) ? (4 + (j >> 1)) : (j >> 1);
  const int n = (w >> (4 * slot)) & 0xF;
  return (n ^ 8) - 8;
}

// D(16x8,f32) += A(16x16,f16,row) * B(16x8,f16,col).  Register fragments
// follow the PTX ISA m16n8k16 layout (groupID = lane/4, tig = lane%4).
__device__ __forceinline__ void mma_16816(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Streaming 128-bit global load that does not allocate in L1 (weights are
// touched exactly once per call).
__device__ __forceinline__ uint4 ldg_stream_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t ldg_stream_u32(const void* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// Programmatic dependent launch: block until the preceding grid in the
// stream has completed and flushed its writes (no-op when the kernel was not
// launched with the programmatic-serialization attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---------------------------------------------------------------------------
// Bulk async copies (global -> shared) completing on an mbarrier.

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

// Order this thread's earlier generic-proxy shared-memory accesses before
// subsequent async-proxy (bulk copy) writes to shared memory.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits for the phase of `bar` with the given parity; gives up after
// timeout_ns (measured on %globaltimer) and returns false instead of hanging.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint64_t timeout_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > timeout_ns) return false;
  }
  return true;
}

// 1-D bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned)
// from global memory into this CTA's shared memory, signalling `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Device-side error bits (reported through soinfer_device_errors()).
enum DeviceError : int { kErrCopyTimeout = 1, kErrPeerTimeout = 2 };

// Row source of a cache-or-stream descriptor (reference gemv_dip_fused.cu:11-12).
__device__ __forceinline__ bool desc_is_staging(int32_t d) { return d < 0; }
__device__ __forceinline__ int32_t desc_offset(int32_t d) { return d & 0x7fffffff; }

}  // namespace soinfer
