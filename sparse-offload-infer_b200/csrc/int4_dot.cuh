// INT4 x fp16 dot products of one 128-K chunk on mma.sync.m16n8k16, shared by
// the persistent batched GEMV (gemv_batch.cu) and the fused decode step
// (decode_fused.cu), so that both produce the same bits for the same chunk.
#pragma once

#include "common.cuh"

namespace soinfer {

// Bias of one 128-K chunk of x as seen by chunk_dot: the MMAs there multiply
// x by 1024 + (s + 8) (low-nibble positions: x0 x1 x4 x5 of each 8-group) and
// 1024 + 16 (s + 8) (high positions x2 x3 x6 x7, later scaled by 1/16), so
// sum q x = chunk_dot - bias with bias = 1032 XL + 72 XH.  One MMA computes it:
// A = 1032 in k-columns 0..7 and 72 in 8..15 (every row), and column n of B
// holds the 16 values of x groups 2n and 2n + 1 (low pairs in k 0..7, high
// pairs in k 8..15), so D[*][n] is the bias share of 16 of the chunk's 128
// values; the 8 columns are summed across the 4 lanes of a row group.
// `xc` is the chunk's 256 bytes of x in shared memory; every lane gets the value.
__device__ __forceinline__ float chunk_bias(const uint8_t* xc, int g, int t) {
  const uint32_t* xw = reinterpret_cast<const uint32_t*>(xc + (2 * g + (t >> 1)) * 16 + (t & 1) * 8);
  const uint32_t a[4] = {0x64086408u, 0x64086408u, 0x54805480u, 0x54805480u};  // 1032 1032 | 72 72
  float d[4] = {0.f, 0.f, 0.f, 0.f};
  mma_16816(d, a, xw[0], xw[1]);  // b0 = (x0, x1) or (x4, x5), b1 = (x2, x3) or (x6, x7)
  float bias = d[0] + d[1];
  bias += __shfl_xor_sync(0xffffffffu, bias, 1);
  bias += __shfl_xor_sync(0xffffffffu, bias, 2);
  return bias;
}

// Biased row sums of one 128-K chunk for the thread's two MMA rows (see file
// comment): returns E + O / 16 for rows g and g + 8, in two MMA chains (one
// per nibble position class) of depth four.
__device__ __forceinline__ void chunk_dot(const uint4 wa, const uint4 wb, const uint4 xf[4], float& s0, float& s1) {
  const uint32_t r0[4] = {wa.x, wa.y, wa.z, wa.w};
  const uint32_t r1[4] = {wb.x, wb.y, wb.z, wb.w};
  float e[4] = {0.f, 0.f, 0.f, 0.f}, o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t t0 = r0[j] >> 8, t1 = r1[j] >> 8;
    const uint32_t ae[4] = {lop3_and_xor(r0[j], 0x000f000fu, 0x64086408u), lop3_and_xor(r1[j], 0x000f000fu, 0x64086408u),
                            lop3_and_xor(t0, 0x000f000fu, 0x64086408u), lop3_and_xor(t1, 0x000f000fu, 0x64086408u)};
    mma_16816(e, ae, xf[j].x, xf[j].z);  // (v0,v1) with x0x1, (v4,v5) with x4x5
    const uint32_t ao[4] = {lop3_and_xor(r0[j], 0x00f000f0u, 0x64806480u), lop3_and_xor(r1[j], 0x00f000f0u, 0x64806480u),
                            lop3_and_xor(t0, 0x00f000f0u, 0x64806480u), lop3_and_xor(t1, 0x00f000f0u, 0x64806480u)};
    mma_16816(o, ao, xf[j].y, xf[j].w);  // (v2,v3) with x2x3, (v6,v7) with x6x7
  }
  s0 = fmaf(o[0], 0.0625f, e[0]);
  s1 = fmaf(o[2], 0.0625f, e[2]);
}

// RMSNorm of K fp16 values (n16 = K / 8 16-byte pieces) in shared memory, in
// two parts: warp_rmsnorm_inv -- one warp: fp32 sum of squares (per-lane
// strided, then a butterfly sum), inv = rsqrt(ss / K + eps) -- and
// rmsnorm_piece -- x = fp16(x * inv * w) per 16-byte piece, the rmsnorm
// kernel's expression (any thread, any order).
__device__ __forceinline__ float warp_rmsnorm_inv(const uint4* x, int n16, int K, float eps, int lane) {
  constexpr int kB = 4;  // pieces loaded ahead of the (in-order) accumulation
  float ss = 0.f;
  for (int u0 = lane; u0 < n16; u0 += 32 * kB) {
    uint4 v[kB];
#pragma unroll
    for (int r = 0; r < kB; ++r) v[r] = u0 + 32 * r < n16 ? x[u0 + 32 * r] : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int r = 0; r < kB; ++r) {
      if (u0 + 32 * r >= n16) break;
      const half2* h = reinterpret_cast<const half2*>(&v[r]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h[j]);
        ss = __fadd_rn(ss, __fadd_rn(__fmul_rn(f.x, f.x), __fmul_rn(f.y, f.y)));  // no contraction: same bits everywhere
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  return rsqrtf(ss / (float)K + eps);
}

__device__ __forceinline__ uint4 rmsnorm_piece(const uint4 v, const uint4 wv, float inv) {
  const half2* h = reinterpret_cast<const half2*>(&v);
  const half2* wh = reinterpret_cast<const half2*>(&wv);
  uint4 o;
  half2* oh = reinterpret_cast<half2*>(&o);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __half22float2(h[j]), gw = __half22float2(wh[j]);
    oh[j] = __floats2half2_rn(f.x * inv * gw.x, f.y * inv * gw.y);
  }
  return o;
}

// Both parts by one warp, in place; out (optional) receives a copy.
__device__ __forceinline__ void warp_rmsnorm_inplace(uint4* x, const uint4* w, int n16, int K, float eps, int lane,
                                                     uint4* out) {
  const float inv = warp_rmsnorm_inv(x, n16, K, eps, lane);
  constexpr int kB = 4;
  for (int u0 = lane; u0 < n16; u0 += 32 * kB) {
    uint4 xv[kB], wv[kB];
#pragma unroll
    for (int r = 0; r < kB; ++r)
      if (u0 + 32 * r < n16) xv[r] = x[u0 + 32 * r], wv[r] = w[u0 + 32 * r];
#pragma unroll
    for (int r = 0; r < kB; ++r) {
      if (u0 + 32 * r >= n16) break;
      const uint4 o = rmsnorm_piece(xv[r], wv[r], inv);
      x[u0 + 32 * r] = o;
      if (out != nullptr) out[u0 + 32 * r] = o;
    }
  }
}

}  // namespace soinfer
