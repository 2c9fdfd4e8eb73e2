// Single-query GQA decode attention over a contiguous fp16 KV cache.
//
// Reference semantics (csrc/kernels/decode_attention.cu:17-55): query head qh
// reads kv head qh / (NQ/NKV); scores q.k * (1/sqrt(hd)); online softmax in
// fp32; out = fp16(sum p v / sum p).  The reference runs one CTA per query
// head with a block-wide reduction and two __syncthreads per cached position,
// re-reading K/V once per query head.
//
// Here (split-KV / flash-decoding): CTA (kv head, position split, head group)
// reads each K and V row of its split exactly once with 16-byte loads and
// serves all REP query heads of the group from registers.  A team of hd/8
// lanes owns one position (8 dims per lane); scores go to shared memory in
// the log2 domain, the split's max / exp2 / sum are taken per head, V rows are
// accumulated in fp32, and the split writes (m, l, acc[hd]) to the workspace.
// A combine kernel rescales and sums the splits in a fixed order.  With a
// single split the CTA writes the output directly.
//
// Each lane keeps kU K (then V) row loads in flight per iteration.
//
// Split layout: for the attended length c, want = min(cap, ceil(c/16))
// splits of L = ceil(c/want) positions (cap: enough CTAs to fill the GPU).
// Both forms compute it in the kernel from c, so the device-position form
// (launched once for max_seq, c read from device memory at run time) uses
// exactly the layout of the host-length form at the same c -- every split
// busy at any length, and bit-identical results between the two forms.
#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"

namespace soinfer {
namespace {

constexpr int kThreads = 128;
constexpr int kMaxSplits = 128;
constexpr int kTargetCtas = 592;   // 4 CTAs per SM (measured best with kU = 4; 8 per SM slowed short contexts)
constexpr int kU = 4;              // positions per team per iteration (loads in flight per lane)
constexpr float kLog2e = 1.4426950408889634f;

// Attended length of the device-position form: *pos_dev + 1, clamped to [1, max_seq].
__device__ __forceinline__ int device_cur_len(const int32_t* pos_dev, int64_t max_seq) {
  const int64_t len = (int64_t)*pos_dev + 1;
  return (int)(len < 1 ? 1 : (len > max_seq ? max_seq : len));
}

__host__ __device__ __forceinline__ int split_want(int c, int cap) {
  const int w = (c + 15) / 16;
  return w < 1 ? 1 : (w > cap ? cap : w);
}

template <int TEAM, int REP>
__global__ void __launch_bounds__(kThreads)
    attn_split_kernel(const half* __restrict__ q, const half* __restrict__ kc, const half* __restrict__ vc,
                      half* __restrict__ out, float* __restrict__ ws_acc, float* __restrict__ ws_ml, const int nq,
                      const int nkv, const int64_t max_seq, const int hd, const int cur_len_host, const int L,
                      const int cap, const float scale_log2, const int32_t* __restrict__ pos_dev) {
  constexpr int kTeams = kThreads / TEAM;
  extern __shared__ float smem[];
  float* s_p = smem;                        // [REP][L] scores, then probabilities
  float* s_red = smem + REP * L;            // [kTeams][REP][hd]
  __shared__ float s_m[REP], s_l[REP];

  const int kvh = blockIdx.x;
  const int split = blockIdx.y;
  const int n_rep = nq / nkv;
  const int qh0 = kvh * n_rep + blockIdx.z * REP;
  const int team = threadIdx.x / TEAM;
  const int tl = threadIdx.x % TEAM;
  const int d0 = tl * 8;
  const bool lane_on = d0 < hd;
  const half* kb = kc + (int64_t)kvh * max_seq * hd;
  const half* vb = vc + (int64_t)kvh * max_seq * hd;

  pdl_launch_dependents();
  pdl_wait();
  // device-position form: cur_len = *pos_dev + 1, read after the producer of
  // pos_dev has finished (the launch holds enough splits for any length)
  const int cur_len = pos_dev ? device_cur_len(pos_dev, max_seq) : cur_len_host;
  const int want = split_want(cur_len, cap);
  const int Ld = (cur_len + want - 1) / want;      // positions per split (<= L, the score-row stride)
  const int nsplit = (cur_len + Ld - 1) / Ld;
  const int t0 = split * Ld;
  if (split >= nsplit) return;
  const int t1 = (t0 + Ld < cur_len) ? t0 + Ld : cur_len;

  float qf[REP][8];
#pragma unroll
  for (int h = 0; h < REP; ++h) {
    if (lane_on) {
      const uint4 u = *reinterpret_cast<const uint4*>(q + (int64_t)(qh0 + h) * hd + d0);
      const half2* p = reinterpret_cast<const half2*>(&u);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(p[i]);
        qf[h][2 * i] = f.x;
        qf[h][2 * i + 1] = f.y;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) qf[h][i] = 0.f;
    }
  }

  // phase A: scores, kU positions per team per iteration (their K rows loaded
  // together, so each lane has kU 16-byte loads in flight); the trip count is
  // uniform across the warp (the team shuffles below need every lane)
  for (int tb = t0; tb < t1; tb += kTeams * kU) {
    uint4 ku[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int t = tb + u * kTeams + team;
      ku[u] = (lane_on && t < t1) ? ldg_stream_u4(kb + (int64_t)t * hd + d0) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int t = tb + u * kTeams + team;
      const bool pos_on = t < t1;
      float kf[8];
      const half2* p = reinterpret_cast<const half2*>(&ku[u]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(p[i]);
        kf[2 * i] = f.x;
        kf[2 * i + 1] = f.y;
      }
#pragma unroll
      for (int h = 0; h < REP; ++h) {
        float dot = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) dot = fmaf(qf[h][i], kf[i], dot);
#pragma unroll
        for (int o = TEAM / 2; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        if (tl == 0 && pos_on) s_p[h * L + (t - t0)] = dot * scale_log2;
      }
    }
  }
  __syncthreads();

  // phase B: per-head max, exp2, sum over the split
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_pos = t1 - t0;
  for (int h = warp; h < REP; h += kThreads / 32) {
    float m = -INFINITY;
    for (int i = lane; i < n_pos; i += 32) m = fmaxf(m, s_p[h * L + i]);
    m = warp_max(m);
    float l = 0.f;
    for (int i = lane; i < n_pos; i += 32) {
      const float p = exp2f(s_p[h * L + i] - m);
      s_p[h * L + i] = p;
      l += p;
    }
    l = warp_sum(l);
    if (lane == 0) {
      s_m[h] = m;
      s_l[h] = l;
    }
  }
  __syncthreads();

  // phase C: acc = sum p v
  float acc[REP][8];
#pragma unroll
  for (int h = 0; h < REP; ++h)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[h][i] = 0.f;
  for (int tb = t0 + team; tb < t1; tb += kTeams * kU) {
    if (!lane_on) continue;
    uint4 vu[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int t = tb + u * kTeams;
      vu[u] = t < t1 ? ldg_stream_u4(vb + (int64_t)t * hd + d0) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int t = tb + u * kTeams;
      if (t >= t1) break;
      const half2* p = reinterpret_cast<const half2*>(&vu[u]);
      float vf[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(p[i]);
        vf[2 * i] = f.x;
        vf[2 * i + 1] = f.y;
      }
#pragma unroll
      for (int h = 0; h < REP; ++h) {
        const float pr = s_p[h * L + (t - t0)];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[h][i] = fmaf(pr, vf[i], acc[h][i]);
      }
    }
  }
  if (lane_on) {
#pragma unroll
    for (int h = 0; h < REP; ++h)
#pragma unroll
      for (int i = 0; i < 8; ++i) s_red[(team * REP + h) * hd + d0 + i] = acc[h][i];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < REP * hd; e += kThreads) {
    const int h = e / hd, d = e - h * hd;
    float sum = 0.f;
    for (int tm = 0; tm < kTeams; ++tm) sum += s_red[(tm * REP + h) * hd + d];
    const int qh = qh0 + h;
    if (nsplit == 1) {
      out[(int64_t)qh * hd + d] = __float2half_rn(sum / s_l[h]);
    } else {
      ws_acc[((int64_t)qh * kMaxSplits + split) * hd + d] = sum;
      if (d == 0) {
        ws_ml[((int64_t)qh * kMaxSplits + split) * 2 + 0] = s_m[h];
        ws_ml[((int64_t)qh * kMaxSplits + split) * 2 + 1] = s_l[h];
      }
    }
  }
}

__global__ void attn_combine_kernel(const float* __restrict__ ws_acc, const float* __restrict__ ws_ml,
                                    half* __restrict__ out, const int hd, const int cur_len_host, const int cap,
                                    const int64_t max_seq, const int32_t* __restrict__ pos_dev) {
  pdl_launch_dependents();
  pdl_wait();
  // the split layout of this length (see the file comment)
  const int cur_len = pos_dev ? device_cur_len(pos_dev, max_seq) : cur_len_host;
  const int want = split_want(cur_len, cap);
  const int Ld = (cur_len + want - 1) / want;
  const int nsplit = (cur_len + Ld - 1) / Ld;
  if (nsplit == 1) return;  // the single split wrote the output itself
  const int qh = blockIdx.x;
  const float* ml = ws_ml + (int64_t)qh * kMaxSplits * 2;
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, ml[2 * s]);
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float num = 0.f, den = 0.f;
    for (int s = 0; s < nsplit; ++s) {
      const float w = exp2f(ml[2 * s] - M);
      num = fmaf(w, ws_acc[((int64_t)qh * kMaxSplits + s) * hd + d], num);
      den = fmaf(w, ml[2 * s + 1], den);
    }
    out[(int64_t)qh * hd + d] = __float2half_rn(num / den);
  }
}

template <int TEAM, int REP>
cudaError_t launch_split(const half* q, const half* kc, const half* vc, half* out, float* ws_acc, float* ws_ml,
                         int nq, int nkv, int64_t max_seq, int hd, int cur_len, int nsplit, int L, int cap,
                         float scale_log2, int groups, const int32_t* pos_dev, cudaStream_t stream) {
  constexpr int kTeams = kThreads / TEAM;
  const size_t smem = (size_t)(REP * L + kTeams * REP * hd) * sizeof(float);
  auto kernel = attn_split_kernel<TEAM, REP>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  return launch_ex(kernel, dim3(nkv, nsplit, groups), dim3(kThreads), smem, stream, 1, true /* programmatic dependent: both kernels wait first */, q, kc, vc, out, ws_acc,
                   ws_ml, nq, nkv, max_seq, hd, cur_len, L, cap, scale_log2, pos_dev);
}

template <int TEAM>
cudaError_t dispatch_rep(int rep, const half* q, const half* kc, const half* vc, half* out, float* ws_acc,
                         float* ws_ml, int nq, int nkv, int64_t max_seq, int hd, int cur_len, int nsplit, int L,
                         int cap, float sl2, int groups, const int32_t* pd, cudaStream_t st) {
  switch (rep) {
    case 1: return launch_split<TEAM, 1>(q, kc, vc, out, ws_acc, ws_ml, nq, nkv, max_seq, hd, cur_len, nsplit, L, cap, sl2, groups, pd, st);
    case 2: return launch_split<TEAM, 2>(q, kc, vc, out, ws_acc, ws_ml, nq, nkv, max_seq, hd, cur_len, nsplit, L, cap, sl2, groups, pd, st);
    case 4: return launch_split<TEAM, 4>(q, kc, vc, out, ws_acc, ws_ml, nq, nkv, max_seq, hd, cur_len, nsplit, L, cap, sl2, groups, pd, st);
    case 5: return launch_split<TEAM, 5>(q, kc, vc, out, ws_acc, ws_ml, nq, nkv, max_seq, hd, cur_len, nsplit, L, cap, sl2, groups, pd, st);
    case 8: return launch_split<TEAM, 8>(q, kc, vc, out, ws_acc, ws_ml, nq, nkv, max_seq, hd, cur_len, nsplit, L, cap, sl2, groups, pd, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

int64_t attention_workspace_bytes(int64_t nq, int64_t max_seq, int64_t hd) {
  (void)max_seq;
  return nq * kMaxSplits * (hd + 2) * (int64_t)sizeof(float);
}

namespace {

cudaError_t decode_attention_impl(const half* q, const half* kc, const half* vc, half* out, int64_t nq, int64_t nkv,
                                  int64_t max_seq, int64_t hd, int64_t plan_len, const int32_t* pos_dev,
                                  void* workspace, cudaStream_t stream) {
  const int n_rep = (int)(nq / nkv);
  int rep;
  if (n_rep == 1 || n_rep == 2 || n_rep == 4 || n_rep == 5 || n_rep == 8)
    rep = n_rep;
  else if (n_rep % 4 == 0)
    rep = 4;
  else if (n_rep % 2 == 0)
    rep = 2;
  else
    rep = 1;
  const int groups = n_rep / rep;
  int64_t cap64 = (kTargetCtas + nkv * groups - 1) / (nkv * groups);
  const int cap = (int)(cap64 > kMaxSplits ? kMaxSplits : cap64);
  const int want = split_want((int)plan_len, cap);
  const int L_plan = (int)((plan_len + want - 1) / want);
  // score-row stride: the longest split of any length <= plan_len (<= max(L_plan, 16))
  const int L = L_plan > 16 ? L_plan : 16;
  // splits launched: the host form's own count; the device form enough for any length
  const int nsplit = pos_dev ? want : (int)((plan_len + L_plan - 1) / L_plan);
  float* ws_acc = reinterpret_cast<float*>(workspace);
  float* ws_ml = ws_acc + nq * kMaxSplits * hd;
  const float sl2 = (1.0f / sqrtf((float)hd)) * kLog2e;
  const int chunks = (int)((hd + 7) / 8);
  int team = 4;
  while (team < chunks) team <<= 1;
  cudaError_t e;
  const int inq = (int)nq, inkv = (int)nkv, ihd = (int)hd, icl = (int)plan_len;
  switch (team) {
    case 4: e = dispatch_rep<4>(rep, q, kc, vc, out, ws_acc, ws_ml, inq, inkv, max_seq, ihd, icl, nsplit, L, cap, sl2, groups, pos_dev, stream); break;
    case 8: e = dispatch_rep<8>(rep, q, kc, vc, out, ws_acc, ws_ml, inq, inkv, max_seq, ihd, icl, nsplit, L, cap, sl2, groups, pos_dev, stream); break;
    case 16: e = dispatch_rep<16>(rep, q, kc, vc, out, ws_acc, ws_ml, inq, inkv, max_seq, ihd, icl, nsplit, L, cap, sl2, groups, pos_dev, stream); break;
    case 32: e = dispatch_rep<32>(rep, q, kc, vc, out, ws_acc, ws_ml, inq, inkv, max_seq, ihd, icl, nsplit, L, cap, sl2, groups, pos_dev, stream); break;
    default: return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess || nsplit == 1) return e;
  const int threads = ihd < 32 ? 32 : (ihd > 256 ? 256 : ihd);
  return launch_ex(attn_combine_kernel, dim3(inq), dim3(threads), 0, stream, 1, true /* programmatic dependent: both kernels wait first */, ws_acc, ws_ml, out, ihd, icl,
                   cap, max_seq, pos_dev);
}

}  // namespace

cudaError_t launch_decode_attention(const half* q, const half* kc, const half* vc, half* out, int64_t nq, int64_t nkv,
                                    int64_t max_seq, int64_t hd, int64_t cur_len, void* workspace,
                                    cudaStream_t stream) {
  return decode_attention_impl(q, kc, vc, out, nq, nkv, max_seq, hd, cur_len, nullptr, workspace, stream);
}

cudaError_t launch_decode_attention_at(const half* q, const half* kc, const half* vc, half* out, int64_t nq,
                                       int64_t nkv, int64_t max_seq, int64_t hd, const int32_t* pos_dev,
                                       void* workspace, cudaStream_t stream) {
  return decode_attention_impl(q, kc, vc, out, nq, nkv, max_seq, hd, max_seq, pos_dev, workspace, stream);
}

}  // namespace soinfer
