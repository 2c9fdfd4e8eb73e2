// Load-time group-wise INT4 quantization + AWQ packing on the GPU, one pass
// over the weights (reference python/soinfer/quant/formats.py:77-110 with
// calibrate.min_max, and quant/pack.py:31-69 / csrc/include/layout.h:19-51).
//
// Semantics, bit-exact with the reference's torch path on the same input:
//   w -> fp32 (w.float()); K zero-padded to a multiple of g;
//   scale[n, j] = max(amax_j / 7, FLT_MIN)            (IEEE fp32 division)
//   q = clamp(rint(w / scale), -7, 7)                   (IEEE division, ties to even)
//   packed word of values v0..v7 (K order) = nibbles in AWQ order
//     byte0 = v0 | v2 << 4, byte1 = v4 | v6 << 4, byte2 = v1 | v3 << 4, byte3 = v5 | v7 << 4.
// (Compiled without fast-math: '/' is the correctly rounded division.)
//
// One thread per packed word (8 values); the g / 8 threads of a group are
// consecutive lanes (g / 8 a power of two <= 32, so a group never straddles a
// warp) and reduce |w| with xor shuffles.  HBM-bound: reads the weights once,
// writes 1/8 of their fp32 size.
#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.h"

namespace soinfer {
namespace {

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_f32<half>(half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename T>
__global__ void __launch_bounds__(256)
    quantize_pack_int4_kernel(const T* __restrict__ w, const int64_t N, const int64_t K, const int64_t ld,
                              const int words_per_row, const int words_per_group, const int G,
                              uint32_t* __restrict__ packed, float* __restrict__ scale) {
  const int64_t total = N * (int64_t)words_per_row;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  // the whole warp iterates together (shuffles); words past the end act as zeros
  for (int64_t base = (int64_t)blockIdx.x * blockDim.x; base < total; base += stride) {
    const int64_t id = base + threadIdx.x;
    const bool live = id < total;
    const int64_t row = live ? id / words_per_row : 0;
    const int word = live ? (int)(id - row * words_per_row) : 0;
    float v[8];
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t k = (int64_t)word * 8 + i;
      v[i] = (live && k < K) ? to_f32<T>(w[row * ld + k]) : 0.f;
      amax = fmaxf(amax, fabsf(v[i]));
    }
    for (int o = 1; o < words_per_group; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float s = fmaxf(amax / 7.0f, 1.17549435e-38f);  // torch.finfo(float32).tiny
    uint32_t nib[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float q = fminf(fmaxf(rintf(v[i] / s), -7.f), 7.f);
      nib[i] = (uint32_t)((int)q) & 0xFu;
    }
    if (live) {
      packed[id] = nib[0] | (nib[2] << 4) | (nib[4] << 8) | (nib[6] << 12) | (nib[1] << 16) | (nib[3] << 20) |
                   (nib[5] << 24) | (nib[7] << 28);
      if (word % words_per_group == 0) scale[row * G + word / words_per_group] = s;
    }
  }
}

}  // namespace

cudaError_t launch_quantize_pack_int4(const void* w, int dtype, int64_t N, int64_t K, int64_t ld, int64_t group_size,
                                      uint8_t* packed, float* scale, cudaStream_t stream) {
  const int64_t Kp = (K + group_size - 1) / group_size * group_size;
  const int words_per_row = (int)(Kp / 8);
  const int words_per_group = (int)(group_size / 8);
  const int G = (int)(Kp / group_size);
  const int64_t total = N * (int64_t)words_per_row;
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t blocks_needed = (total + 255) / 256;
  const int grid = (int)(blocks_needed < (int64_t)sms * 8 ? blocks_needed : (int64_t)sms * 8);
  uint32_t* out = reinterpret_cast<uint32_t*>(packed);
  switch (dtype) {
    case 0:
      quantize_pack_int4_kernel<float><<<grid, 256, 0, stream>>>(static_cast<const float*>(w), N, K, ld,
                                                                  words_per_row, words_per_group, G, out, scale);
      break;
    case 1:
      quantize_pack_int4_kernel<half><<<grid, 256, 0, stream>>>(static_cast<const half*>(w), N, K, ld, words_per_row,
                                                                 words_per_group, G, out, scale);
      break;
    case 2:
      quantize_pack_int4_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
          static_cast<const __nv_bfloat16*>(w), N, K, ld, words_per_row, words_per_group, G, out, scale);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace soinfer
