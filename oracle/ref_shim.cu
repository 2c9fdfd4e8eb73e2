// TEST INFRASTRUCTURE ONLY: extern "C" entry points over the reference's own
// CUDA launchers (compiled from sparse-offload-infer's csrc/kernels/*.cu in
// place by oracle/Makefile), so tests can run the reference kernels on a
// B200 through ctypes and pin the oracle / compare against them.  Every
// reference launcher runs on the legacy default stream and aborts on error.
#include <cstdint>
#include <cuda_fp16.h>

#include "decode_attention.cuh"
#include "gemv_dip_fused.cuh"
#include "gemv_sparse_accumulate.cuh"
#include "gemv_w4a16_group.cuh"
#include "gemv_w8a16.cuh"
#include "kv_cache.cuh"
#include "rmsnorm.cuh"
#include "rope.cuh"
#include "topk_select.cuh"

extern "C" {

void ref_gemv_w4a16_group(const void* Wq, const void* s, const void* x, void* y, int N, int K, int g, int G) {
  launch_gemv_w4a16_group((const uint8_t*)Wq, (const float*)s, (const half*)x, (half*)y, N, K, g, G);
}
void ref_gemv_w4a16_group_lop3(const void* Wq, const void* s, const void* x, void* y, int N, int K, int g, int G) {
  launch_gemv_w4a16_group_lop3((const uint8_t*)Wq, (const float*)s, (const half*)x, (half*)y, N, K, g, G);
}
void ref_gemv_w8a16(const void* Wq, const void* s, const void* x, void* y, int N, int K, int g, int G, int stride) {
  launch_gemv_w8a16((const int8_t*)Wq, (const float*)s, (const half*)x, (half*)y, N, K, g, G, stride);
}
void ref_topk_threshold_select(const void* v, int n, int k, void* idx, void* count) {
  launch_topk_threshold_select((const float*)v, n, k, (int*)idx, (int*)count);
}
void ref_sparse_accumulate(const void* Wq, const void* s, const void* h, void* y, int H, int k, int g, int G) {
  launch_gemv_w4a16_sparse_accumulate((const uint8_t*)Wq, (const float*)s, (const half*)h, (half*)y, H, k, g, G);
}
void ref_build_dip_descriptors(const void* sel, int k, const void* slot_of, void* desc, void* miss, void* count) {
  launch_build_dip_descriptors((const int32_t*)sel, k, (const int32_t*)slot_of, (int32_t*)desc, (int32_t*)miss,
                               (int32_t*)count);
}
void ref_gemv_dip_fused_up(const void* cW, const void* cS, const void* sW, const void* sS, const void* desc,
                           const void* x, void* y, int k, int K, int g, int G) {
  launch_gemv_dip_fused_up((const uint8_t*)cW, (const float*)cS, (const uint8_t*)sW, (const float*)sS,
                           (const int32_t*)desc, (const half*)x, (half*)y, k, K, g, G);
}
void ref_gemv_dip_fused_down(const void* cW, const void* cS, const void* sW, const void* sS, const void* desc,
                             const void* h, void* y, int H, int k, int g, int G) {
  launch_gemv_dip_fused_down((const uint8_t*)cW, (const float*)cS, (const uint8_t*)sW, (const float*)sS,
                             (const int32_t*)desc, (const half*)h, (half*)y, H, k, g, G);
}
void ref_decode_attention(const void* q, const void* kc, const void* vc, void* out, int nq, int nkv, int max_seq,
                          int hd, int cur_len, float scale) {
  launch_decode_attention((const half*)q, (const half*)kc, (const half*)vc, (half*)out, nq, nkv, max_seq, hd,
                          cur_len, scale);
}
void ref_rmsnorm(const void* x, const void* w, void* out, int rows, int hidden, float eps) {
  launch_rmsnorm((const half*)x, (const half*)w, (half*)out, rows, hidden, eps);
}
void ref_rope_apply(void* x, const void* c, const void* s, int heads, int hd) {
  launch_rope_apply((half*)x, (const float*)c, (const float*)s, heads, hd);
}
}
