// Fused dense decode step: all decoder layers of a batch-1 Qwen3-style model
// (HBM-resident INT4 weights, group size 128, head_dim 128) in ONE cooperative
// launch -- one CTA of 16 warps per SM, the layer's phases separated by grid
// barriers instead of kernel boundaries:
//
//   1 x -> RMSNorm (input_layernorm) -> q / k / v GEMVs
//   2 per (kv head, split) unit: q head norm + RoPE, the new K / V row
//     (k head norm + RoPE) appended by the unit that holds the position,
//     split-KV attention partials
//   3 combine of the splits (skipped when the length needs one split)
//   4 o GEMV + residual -> h2
//   5 h2 -> RMSNorm (post_attention_layernorm) -> gate / up GEMVs -> SwiGLU
//   6 down GEMV + residual -> x (the next layer's input)
//
// Why: in the per-kernel decode step each launch pays the launch, the first
// weight fetch from HBM and the drain of its tail, and a 1.7B-class layer's
// kernels move only a few MB each, so launch latency -- not bandwidth -- set
// the step time.  Here each CTA bulk-copies its tiles of the coming GEMV phase
// (cp.async.bulk into one of two shared-memory weight buffers, completing on
// an mbarrier) a phase or more ahead, so a phase finds its weights on chip
// and costs a barrier plus one round trip for its input vector.
//
// Arithmetic: every value equals the per-kernel path's (gemv_batch.cu with
// its RMSNorm prologue and SwiGLU / residual epilogues, glue.cu's head norm +
// RoPE + KV append, attention.cu's split and combine kernels): a 16-row tile's
// 128-K chunks are split over 8 warps exactly as the persistent kernel splits
// them (warp w: chunks w, w + 8, ..., accumulated in chunk order), the 8
// partial rows are summed in warp order, the attention layout is computed
// from the same length and cap, and the shared helpers (int4_dot.cuh) are the
// same code -- so the fused step produces the same bits and the same greedy
// tokens.
//
// Grid barrier: one arrival counter that only grows (target = barrier index x
// grid), acquire/release at GPU scope, bounded (1 s) -- a wait that runs out
// sets a device error bit and every CTA leaves; the last CTA out resets the
// counters.  Reference semantics per layer: python/soinfer/runtime/generate.py
// :141-182 of sparse-offload-infer (the dense streaming layer).
#include "common.cuh"
#include "int4_dot.cuh"
#include "kernels.h"
#include "launch.cuh"

namespace soinfer {

__device__ int g_decode_fused_error;

namespace {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kGroupWarps = 8;          // warps per 16-row tile (the persistent kernel's split)
constexpr int kMaxSlots = 16;           // tiles per CTA per phase
constexpr int kAttnGroups = 4;          // attention: 4 units of 128 threads per CTA
constexpr int kAttnThreads = 128;
constexpr int kTeam = 16;               // lanes per position (head_dim 128 / 8)
constexpr int kTeams = kAttnThreads / kTeam;
constexpr int kU = 4;                   // positions per team per iteration
constexpr int kMaxSplits = 128;         // the attention workspace's split stride
constexpr int kHD = 128;
constexpr uint64_t kWaitNs = 1000000000ull;

__device__ __forceinline__ int ld_acquire_i32(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Loads through L2 (data written by other CTAs of this launch; never a stale
// L1 line).  Plain intrinsics, so the compiler may batch them.
__device__ __forceinline__ uint4 ld_cg_u4(const void* p) { return __ldcg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ half ld_cg_half(const half* p) { return __ldcg(p); }
__device__ __forceinline__ float ld_cg_f32(const float* p) { return __ldcg(p); }

__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Grid barrier number nb (1, 2, ...): every CTA's writes before it are
// visible to every CTA after it.  False (uniform over the CTA) if the wait ran
// out: the caller returns.
__device__ __forceinline__ bool grid_sync(int* bar, int nb, int grid, int* s_ok) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(bar, 1);
    const int target = nb * grid;
    int ok = 1;
    if (ld_acquire_i32(bar) < target) {
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_i32(bar) < target) {
        if (globaltimer_ns() - t0 > kWaitNs) {
          atomicOr(&g_decode_fused_error, kErrCopyTimeout);
          ok = 0;
          break;
        }
      }
    }
    *s_ok = ok;
  }
  __syncthreads();
  return *s_ok != 0;
}

// One GEMV phase's matrices: up to three matrices of the same K, their tiles
// numbered one after another (q / k / v), or two matrices paired tile by tile
// (gate / up: a unit is gate tile j and up tile j, on the same CTA).
struct Mat {
  const uint8_t* w;
  const float* s;
  int tiles;
};

struct Mat3 {
  Mat m[3];
};

// K fp16 values from global memory (written by other CTAs) into shared memory.
__device__ __forceinline__ void load_x(const half* src, int K, half* xs) {
  for (int u = threadIdx.x; u < K / 8; u += kThreads)
    reinterpret_cast<uint4*>(xs)[u] = ld_cg_u4(reinterpret_cast<const uint4*>(src) + u);
}

// Every chunk's bias (chunk_bias) of the phase input, one warp per chunk.
__device__ __forceinline__ void chunk_biases(const half* xs, int nch, float* sb, int warp, int lane) {
  const int g = lane >> 2, t = lane & 3;
  for (int c = warp; c < nch; c += kWarps) {
    const float b = chunk_bias(reinterpret_cast<const uint8_t*>(xs) + c * 256, g, t);
    if (lane == 0) sb[c] = b;
  }
}

// Slots of a phase on this CTA: units cta, cta + grid, ...; NT tiles per unit.
__device__ __forceinline__ int owned_units(int units, int cta, int grid) {
  return units > cta ? (units - cta + grid - 1) / grid : 0;
}

// The (matrix, tile) of slot s; matrices picked with constant indices so the
// descriptors stay in registers.
template <int NMAT, bool PAIRED>
__device__ __forceinline__ void slot_tile(const Mat (&mats)[NMAT], int s, int cta, int grid, int& mi, int& tile) {
  constexpr int NT = PAIRED ? 2 : 1;
  const int u = cta + grid * (s / NT);
  if (PAIRED) {
    mi = s % NT;
    tile = u;
  } else {
    mi = 0;
    tile = u;
#pragma unroll
    for (int m = 0; m < NMAT - 1; ++m)
      if (mi == m && tile >= mats[m].tiles) {
        tile -= mats[m].tiles;
        mi = m + 1;
      }
  }
}

template <int NMAT>
__device__ __forceinline__ const Mat& pick(const Mat (&mats)[NMAT], int mi) {
  if (NMAT > 2 && mi == 2) return mats[NMAT > 2 ? 2 : 0];
  if (NMAT > 1 && mi == 1) return mats[NMAT > 1 ? 1 : 0];
  return mats[0];
}

// Bytes of one slot in a weight buffer: the tile's 16 packed rows, then its
// 16 scale rows.
__host__ __device__ __forceinline__ int slot_bytes(int K) { return 16 * (K / 2) + 16 * (K / 128) * 4; }

// The warp that issues the weight-buffer fills (it has no epilogue rows, so
// the issue overlaps the epilogue).
constexpr int kFillWarp = kWarps - 1;

// Starts the bulk copies of this CTA's tiles of one GEMV phase (and, if given,
// an RMSNorm weight vector after them) into a weight buffer, completing on
// `bar`: lane j copies slot j's rows and scale rows, lane 31 the norm vector.
// The fill warp only; the buffer's earlier readers have passed a CTA barrier.
template <int NMAT, bool PAIRED>
__device__ __forceinline__ void fill_weights(const Mat (&mats)[NMAT], int K, int units, int cta, int grid,
                                             uint8_t* buf, const half* norm, int normK, uint64_t* bar, int lane) {
  constexpr int NT = PAIRED ? 2 : 1;
  const int nslots = owned_units(units, cta, grid) * NT;
  const int sbytes = slot_bytes(K), wbytes = 16 * (K / 2), nch = K / 128;
  fence_proxy_async_smem();  // the buffer's earlier generic reads precede these async writes
  if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)(nslots * sbytes + (norm != nullptr ? normK * 2 : 0)));
  __syncwarp();
  for (int j = lane; j < nslots; j += 32) {
    int mi, tile;
    slot_tile<NMAT, PAIRED>(mats, j, cta, grid, mi, tile);
    const Mat& mt = pick<NMAT>(mats, mi);
    bulk_g2s(buf + j * sbytes, mt.w + (int64_t)tile * wbytes, (uint32_t)wbytes, bar);
    bulk_g2s(buf + j * sbytes + wbytes, mt.s + (int64_t)tile * 16 * nch, (uint32_t)(16 * nch * 4), bar);
  }
  if (norm != nullptr && lane == 31) bulk_g2s(buf + nslots * sbytes, norm, (uint32_t)(normK * 2), bar);
}

// One GEMV phase from a weight buffer: the CTA's slots as fp32 partial rows
// red[slot][w8][16] (summed over the 8 warps by the caller's epilogue).  Slot
// s belongs to the warp group s & 1; warp gw of the group takes the tile's
// chunks gw, gw + 8, ... in order and accumulates them in registers -- the
// persistent kernel's split and order; sb holds every chunk's bias.  Two
// slots advance together (their dot products
// are independent, so their MMA chains overlap).
__device__ __forceinline__ void gemv_compute(const uint8_t* buf, int K, int nslots, const half* xs, const float* sb,
                                             float* red, int warp, int lane) {
  const int nch = K / 128, rb = K / 2, sbytes = slot_bytes(K);
  const int g = lane >> 2, t = lane & 3;
  const int grp = warp / kGroupWarps, gw = warp % kGroupWarps;
  const int nmine = nch > gw ? (nch - gw + kGroupWarps - 1) / kGroupWarps : 0;
  const uint4* xq = reinterpret_cast<const uint4*>(xs) + gw * 16 + t * 4;
  for (int s = grp; s < nslots; s += 4) {
    const bool two = s + 2 < nslots;
    const uint8_t* wt0 = buf + s * sbytes;
    const uint8_t* wt1 = buf + (two ? s + 2 : s) * sbytes;
    const uint8_t* a0 = wt0 + g * rb + gw * 64 + t * 16;
    const uint8_t* b0 = wt1 + g * rb + gw * 64 + t * 16;
    const float* sa = reinterpret_cast<const float*>(wt0 + 16 * rb) + g * nch + gw;
    const float* sbb = reinterpret_cast<const float*>(wt1 + 16 * rb) + g * nch + gw;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};  // slot s rows g, g + 8; slot s + 2 rows g, g + 8
    for (int i = 0; i < nmine; ++i) {
      const int off = i * kGroupWarps;
      uint4 xf[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) xf[q] = xq[off * 16 + q];
      const uint4 wa0 = *reinterpret_cast<const uint4*>(a0 + off * 64);
      const uint4 wb0 = *reinterpret_cast<const uint4*>(a0 + 8 * rb + off * 64);
      const uint4 wa1 = *reinterpret_cast<const uint4*>(b0 + off * 64);
      const uint4 wb1 = *reinterpret_cast<const uint4*>(b0 + 8 * rb + off * 64);
      float d0, d1, d2, d3;
      chunk_dot(wa0, wb0, xf, d0, d1);
      chunk_dot(wa1, wb1, xf, d2, d3);
      const float b = sb[gw + off];
      acc[0] = fmaf(sa[off], d0 - b, acc[0]);
      acc[1] = fmaf(sa[8 * nch + off], d1 - b, acc[1]);
      acc[2] = fmaf(sbb[off], d2 - b, acc[2]);
      acc[3] = fmaf(sbb[8 * nch + off], d3 - b, acc[3]);
    }
    if (t == 0) {
      red[(s * kGroupWarps + gw) * 16 + g] = acc[0];
      red[(s * kGroupWarps + gw) * 16 + g + 8] = acc[1];
      if (two) {
        red[((s + 2) * kGroupWarps + gw) * 16 + g] = acc[2];
        red[((s + 2) * kGroupWarps + gw) * 16 + g + 8] = acc[3];
      }
    }
  }
}

// RMSNorm of the phase input in shared memory with weights w (shared memory):
// warp 0 takes the sum of squares in the persistent kernel's order, then every
// thread scales pieces.  Ends with a CTA barrier.
__device__ __forceinline__ void cta_rmsnorm(half* xs, const half* w, int K, float eps, float* s_inv, int warp,
                                            int lane) {
  if (warp == 0) {
    const float inv = warp_rmsnorm_inv(reinterpret_cast<const uint4*>(xs), K / 8, K, eps, lane);
    if (lane == 0) *s_inv = inv;
  }
  __syncthreads();
  const float inv = *s_inv;
  for (int u = threadIdx.x; u < K / 8; u += kThreads)
    reinterpret_cast<uint4*>(xs)[u] =
        rmsnorm_piece(reinterpret_cast<const uint4*>(xs)[u], reinterpret_cast<const uint4*>(w)[u], inv);
  __syncthreads();
}

// Waits (every thread, bounded) for a weight buffer's fill; uniform result.
__device__ __forceinline__ bool wait_weights(uint64_t* bar, int parity) {
  const bool ok = mbar_wait_bounded(bar, (uint32_t)parity, kWaitNs);
  if (!ok && (threadIdx.x & 31) == 0) atomicOr(&g_decode_fused_error, kErrCopyTimeout);
  return __syncthreads_and(ok ? 1 : 0) != 0;
}

// Sum of the 8 warp partials of (slot, row r), in warp order.
__device__ __forceinline__ float slot_sum(const float* red, int slot, int r) {
  float sum = 0.f;
#pragma unroll
  for (int w = 0; w < kGroupWarps; ++w) sum += red[(slot * kGroupWarps + w) * 16 + r];
  return sum;
}

__host__ __device__ __forceinline__ int split_want(int c, int cap) {
  const int w = (c + 15) / 16;
  return w < 1 ? 1 : (w > cap ? cap : w);
}

// One head row: RMSNorm with the head norm weights (rounded to fp16), then
// RoPE at the position (cos / sin rows cv / sv) -- glue.cu head_norm_rope's
// per-warp arithmetic; src read from L2 (written earlier in this launch).
// Every load the row needs is issued first (one round trip), then the math.
__device__ __forceinline__ void head_norm_rope_row(const half* src, const half* w, const float* cv, const float* sv,
                                                   half* dst, float eps, int lane, half* dst2 = nullptr) {
  constexpr int half_dim = kHD / 2;
  float xv[4], wv[4], cs[2], sn[2];
#pragma unroll
  for (int n = 0; n < 4; ++n) {
    xv[n] = __half2float(ld_cg_half(src + lane + 32 * n));
    wv[n] = __half2float(w[lane + 32 * n]);
  }
#pragma unroll
  for (int n = 0; n < 2; ++n) {
    cs[n] = cv[lane + 32 * n];
    sn[n] = sv[lane + 32 * n];
  }
  float ss = 0.f;
#pragma unroll
  for (int n = 0; n < 4; ++n) ss = fmaf(xv[n], xv[n], ss);
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / (float)kHD + eps);
#pragma unroll
  for (int n = 0; n < 2; ++n) {  // pairs (i, i + 64), i = lane + 32 n
    // explicit roundings (no contraction): the same bits as glue.cu's kernel
    const float x1 = __half2float(__float2half_rn(__fmul_rn(__fmul_rn(xv[n], inv), wv[n])));
    const float x2 = __half2float(__float2half_rn(__fmul_rn(__fmul_rn(xv[n + 2], inv), wv[n + 2])));
    const half lo = __float2half_rn(__fsub_rn(__fmul_rn(x1, cs[n]), __fmul_rn(x2, sn[n])));
    const half hi = __float2half_rn(__fadd_rn(__fmul_rn(x2, cs[n]), __fmul_rn(x1, sn[n])));
    const int i = lane + 32 * n;
    dst[i] = lo;
    dst[i + half_dim] = hi;
    if (dst2 != nullptr) {
      dst2[i] = lo;
      dst2[i + half_dim] = hi;
    }
  }
}

// Shared-memory bytes of one attention group for REP query heads per unit:
// the new K / V rows, the q rows, scores, partial sums; rounded up to 128 so
// every group's region (rows are read as 16-byte vectors) starts aligned.
__host__ __device__ __forceinline__ int attn_group_bytes(int rep, int lmax) {
  return (2 * kHD * 2 + rep * kHD * 2 + rep * lmax * 4 + kTeams * rep * kHD * 4 + 2 * rep * 4 + 127) / 128 * 128;
}

// One attention unit (kv head kvh, positions [t0, t1) of split `split`) by a
// group of 128 threads (named barrier bar_id): attention.cu attn_split_kernel's
// arithmetic, with the unit's q rows normalised and rotated here and, in the
// unit that holds the new position, its K / V row appended first.
template <int REP>
__device__ void attn_unit(const FusedDecodeParams& P, const FusedLayer& Ly, int kvh, int split, int Ld, int nsplit,
                          int cur_len, int pos, uint8_t* gsm, int gtid, int bar_id) {
  half* s_kv = reinterpret_cast<half*>(gsm);                       // [2][128] the new position's K and V rows
  half* s_q = s_kv + 2 * kHD;                                      // [REP][128] normalised + rotated q
  float* s_p = reinterpret_cast<float*>(gsm + (2 + REP) * kHD * 2);  // [REP][lmax] scores, then probabilities
  float* s_red = s_p + REP * P.lmax;                               // [kTeams][REP][128]
  float* s_m = s_red + kTeams * REP * kHD;                         // [REP]
  float* s_l = s_m + REP;                                          // [REP]
  const int L = P.lmax;
  const int gwarp = gtid >> 5, lane = gtid & 31;
  const int t0 = split * Ld;
  const int t1 = (t0 + Ld < cur_len) ? t0 + Ld : cur_len;
  const int qh0 = kvh * REP;
  const int team = gtid / kTeam, tl = gtid % kTeam, d0 = tl * 8;
  const half* kb = Ly.kc + (int64_t)kvh * P.max_seq * kHD;
  const half* vb = Ly.vc + (int64_t)kvh * P.max_seq * kHD;
  // the first iteration's cached K / V rows (positions before the new one) do
  // not depend on this step: their loads overlap the q rows' norm and RoPE
  uint4 kpre[kU], vpre[kU];
#pragma unroll
  for (int u = 0; u < kU; ++u) {
    const int t = t0 + u * kTeams + team;
    const bool cached = t < t1 && t != pos;
    kpre[u] = cached ? ld_cg_u4(kb + (int64_t)t * kHD + d0) : make_uint4(0, 0, 0, 0);
    vpre[u] = cached ? ld_cg_u4(vb + (int64_t)t * kHD + d0) : make_uint4(0, 0, 0, 0);
  }
  const float* cv = P.cos_t + (int64_t)pos * (kHD / 2);
  const float* sv = P.sin_t + (int64_t)pos * (kHD / 2);
  for (int h = gwarp; h < REP; h += kAttnThreads / 32)
    head_norm_rope_row(P.q + (int64_t)(qh0 + h) * kHD, Ly.q_norm, cv, sv, s_q + h * kHD, P.eps, lane);
  if (split == nsplit - 1) {  // this unit attends to the new position: append its K / V row first
    // on warps without a q row when there are any (REP < 4), so the rows run side by side
    if (gwarp == REP % 4) {
      head_norm_rope_row(P.k + (int64_t)kvh * kHD, Ly.k_norm, cv, sv, Ly.kc + ((int64_t)kvh * P.max_seq + pos) * kHD,
                         P.eps, lane, s_kv);
    } else if (gwarp == (REP + 1) % 4) {
      for (int i = lane; i < kHD; i += 32) {
        const half v = ld_cg_half(P.v + (int64_t)kvh * kHD + i);
        Ly.vc[((int64_t)kvh * P.max_seq + pos) * kHD + i] = v;
        s_kv[kHD + i] = v;
      }
    }
  }
  named_sync(bar_id, kAttnThreads);

  float qf[REP][8];
#pragma unroll
  for (int h = 0; h < REP; ++h) {
    const uint4 u = *reinterpret_cast<const uint4*>(s_q + h * kHD + d0);
    const half2* p = reinterpret_cast<const half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(p[i]);
      qf[h][2 * i] = f.x;
      qf[h][2 * i + 1] = f.y;
    }
  }
  // phase A: scores
  for (int tb = t0; tb < t1; tb += kTeams * kU) {
    uint4 ku[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int t = tb + u * kTeams + team;
      ku[u] = t == pos ? *reinterpret_cast<const uint4*>(s_kv + d0)
                       : (tb == t0 ? kpre[u] : (t < t1 ? ld_cg_u4(kb + (int64_t)t * kHD + d0) : make_uint4(0, 0, 0, 0)));
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
        for (int o = kTeam / 2; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        if (tl == 0 && pos_on) s_p[h * L + (t - t0)] = dot * P.scale_log2;
      }
    }
  }
  named_sync(bar_id, kAttnThreads);
  // phase B: per-head max, exp2, sum
  const int n_pos = t1 - t0;
  for (int h = gwarp; h < REP; h += kAttnThreads / 32) {
    float m = -INFINITY;
    for (int i = lane; i < n_pos; i += 32) m = fmaxf(m, s_p[h * L + i]);
    m = warp_max(m);
    float l = 0.f;
    for (int i = lane; i < n_pos; i += 32) {
      const float pr = exp2f(s_p[h * L + i] - m);
      s_p[h * L + i] = pr;
      l += pr;
    }
    l = warp_sum(l);
    if (lane == 0) {
      s_m[h] = m;
      s_l[h] = l;
    }
  }
  named_sync(bar_id, kAttnThreads);
  // phase C: acc = sum p v
  float acc[REP][8];
#pragma unroll
  for (int h = 0; h < REP; ++h)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[h][i] = 0.f;
  for (int tb = t0 + team; tb < t1; tb += kTeams * kU) {
    uint4 vu[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int t = tb + u * kTeams;
      vu[u] = t == pos ? *reinterpret_cast<const uint4*>(s_kv + kHD + d0)
                       : (tb == t0 + team ? vpre[u]
                                          : (t < t1 ? ld_cg_u4(vb + (int64_t)t * kHD + d0) : make_uint4(0, 0, 0, 0)));
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
#pragma unroll
  for (int h = 0; h < REP; ++h)
#pragma unroll
    for (int i = 0; i < 8; ++i) s_red[(team * REP + h) * kHD + d0 + i] = acc[h][i];
  named_sync(bar_id, kAttnThreads);
  for (int e = gtid; e < REP * kHD; e += kAttnThreads) {
    const int h = e / kHD, d = e - h * kHD;
    float sum = 0.f;
    for (int tm = 0; tm < kTeams; ++tm) sum += s_red[(tm * REP + h) * kHD + d];
    const int qh = qh0 + h;
    if (nsplit == 1) {
      P.attn[(int64_t)qh * kHD + d] = __float2half_rn(sum / s_l[h]);
    } else {
      P.ws_acc[((int64_t)qh * kMaxSplits + split) * kHD + d] = sum;
      if (d == 0) {
        P.ws_ml[((int64_t)qh * kMaxSplits + split) * 2 + 0] = s_m[h];
        P.ws_ml[((int64_t)qh * kMaxSplits + split) * 2 + 1] = s_l[h];
      }
    }
  }
  named_sync(bar_id, kAttnThreads);  // the group's shared memory is free for its next unit
}

// Element d of query head qh's attention output from its splits (attention.cu
// attn_combine_kernel's arithmetic).
__device__ __forceinline__ half combine_one(const FusedDecodeParams& P, int qh, int d, int nsplit) {
  const float* ml = P.ws_ml + (int64_t)qh * kMaxSplits * 2;
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, ld_cg_f32(ml + 2 * s));
  float num = 0.f, den = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    const float w = exp2f(ld_cg_f32(ml + 2 * s) - M);
    num = fmaf(w, ld_cg_f32(P.ws_acc + ((int64_t)qh * kMaxSplits + s) * kHD + d), num);
    den = fmaf(w, ld_cg_f32(ml + 2 * s + 1), den);
  }
  return __float2half_rn(num / den);
}



// Shared-memory layout: weight buffer A (q/k/v + input norm, then gate/up +
// post-attention norm) | weight buffer B (o, then down) | scratch, shared by
// the GEMV phases (x | chunk biases | partial rows) and the attention groups.
struct FusedSmem {
  int a_bytes, b_bytes, xbytes, sbbytes, redbytes, attn_bytes, total;
};
__host__ __device__ __forceinline__ FusedSmem fused_smem(int H, int I, int NQD, int NKVD, int rep, int lmax,
                                                         int grid) {
  auto own = [&](int units) { return (units + grid - 1) / grid; };
  FusedSmem f;
  const int qkv = own((NQD + 2 * NKVD) / 16) * slot_bytes(H) + H * 2;
  const int gu = own(I / 16) * 2 * slot_bytes(H) + H * 2;
  f.a_bytes = ((qkv > gu ? qkv : gu) + 127) / 128 * 128;
  const int o = own(H / 16) * slot_bytes(NQD), dn = own(H / 16) * slot_bytes(I);
  f.b_bytes = ((o > dn ? o : dn) + 127) / 128 * 128;
  int kmax = H > I ? H : I;
  if (NQD > kmax) kmax = NQD;
  f.xbytes = (kmax * 2 + 127) / 128 * 128;
  f.sbbytes = ((kmax / 128) * 4 + 127) / 128 * 128;
  f.redbytes = kMaxSlots * kGroupWarps * 16 * 4;
  f.attn_bytes = kAttnGroups * attn_group_bytes(rep, lmax);
  const int g = f.xbytes + f.sbbytes + f.redbytes;
  f.total = f.a_bytes + f.b_bytes + (g > f.attn_bytes ? g : f.attn_bytes);
  return f;
}

template <int REP>
__global__ void __launch_bounds__(kThreads, 1) decode_fused_kernel(const __grid_constant__ FusedDecodeParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_ok;
  __shared__ float s_inv;
  __shared__ __align__(8) uint64_t s_wbar[2];  // weight buffers A, B: fill complete
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x, grid = gridDim.x;
  const int pos = *P.pos;
  if (pos < 0 || pos >= P.max_seq) return;  // the same for every CTA: no barrier is left waiting
  const int cur_len = pos + 1;
  const int want = split_want(cur_len, P.cap);
  const int Ld = (cur_len + want - 1) / want;
  const int nsplit = (cur_len + Ld - 1) / Ld;
  const int H = P.H, I = P.I, NQD = P.NQ * kHD, NKVD = P.NKV * kHD;
  const FusedSmem fs = fused_smem(H, I, NQD, NKVD, REP, P.lmax, grid);
  uint8_t* bufA = smem;
  uint8_t* bufB = smem + fs.a_bytes;
  uint8_t* scratch = bufB + fs.b_bytes;
  half* xs = reinterpret_cast<half*>(scratch);
  float* sb = reinterpret_cast<float*>(scratch + fs.xbytes);
  float* red = reinterpret_cast<float*>(scratch + fs.xbytes + fs.sbbytes);
  const int agrp = warp / (kAttnThreads / 32), gtid = threadIdx.x % kAttnThreads;
  uint8_t* gsm = scratch + agrp * attn_group_bytes(REP, P.lmax);
  const int qkv_units = (NQD + 2 * NKVD) / 16;
  const int n_qkv = owned_units(qkv_units, cta, grid), n_h = owned_units(H / 16, cta, grid);
  const int n_gu = owned_units(I / 16, cta, grid);
  int ph[2] = {0, 0};         // next parity to wait for, per buffer
  bool pend[2] = {false, false};  // a fill is in flight (the fill warp's view)
  auto qkv_mats = [&](const FusedLayer& L) {
    return Mat3{{{L.w[0], L.s[0], NQD / 16}, {L.w[1], L.s[1], NKVD / 16}, {L.w[2], L.s[2], NKVD / 16}}};
  };
  // leave after a failed wait: first let this CTA's copies in flight land (bounded)
  auto bail = [&]() {
    if (warp == kFillWarp && lane == 0)
      for (int b = 0; b < 2; ++b)
        if (pend[b]) (void)mbar_wait_bounded(&s_wbar[b], (uint32_t)ph[b], kWaitNs);
  };
  if (threadIdx.x == 0) {
    mbar_init(&s_wbar[0], 1);
    mbar_init(&s_wbar[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == kFillWarp) {
    const FusedLayer& L0 = P.layer[0];
    const Mat3 mq = qkv_mats(L0);
    fill_weights<3, false>(mq.m, H, qkv_units, cta, grid, bufA, L0.in_norm, H, &s_wbar[0], lane);
    const Mat mo[1] = {{L0.w[3], L0.s[3], H / 16}};
    fill_weights<1, false>(mo, NQD, H / 16, cta, grid, bufB, nullptr, 0, &s_wbar[1], lane);
    pend[0] = pend[1] = true;
  }
  __syncthreads();
  int nb = 0;
  for (int li = 0; li < P.layers; ++li) {
    const FusedLayer& Ly = P.layer[li];
    const bool last = li + 1 == P.layers;
    // ---- phase 1: RMSNorm(x) -> q / k / v from buffer A
    load_x(P.x, H, xs);
    if (!wait_weights(&s_wbar[0], ph[0])) return bail();
    ph[0] ^= 1;
    pend[0] = false;
    cta_rmsnorm(xs, reinterpret_cast<const half*>(bufA + n_qkv * slot_bytes(H)), H, P.eps, &s_inv, warp, lane);
    chunk_biases(xs, H / 128, sb, warp, lane);
    __syncthreads();
    gemv_compute(bufA, H, n_qkv, xs, sb, red, warp, lane);
    __syncthreads();
    {
      const Mat3 mq = qkv_mats(Ly);
      for (int e = threadIdx.x; e < n_qkv * 16; e += kThreads) {
        const int slot = e >> 4, r = e & 15;
        int mi, tile;
        slot_tile<3, false>(mq.m, slot, cta, grid, mi, tile);
        half* dst = mi == 0 ? P.q : (mi == 1 ? P.k : P.v);
        dst[tile * 16 + r] = __float2half_rn(slot_sum(red, slot, r));
      }
    }
    if (!grid_sync(P.bar, ++nb, grid, &s_ok)) return bail();
    // ---- phase 2: head norm + RoPE, KV append, split attention
    if (warp == kFillWarp) {  // buffer A: this layer's gate / up (+ post-attention norm)
      const Mat mgu[2] = {{Ly.w[4], Ly.s[4], I / 16}, {Ly.w[5], Ly.s[5], I / 16}};
      fill_weights<2, true>(mgu, H, I / 16, cta, grid, bufA, Ly.post_norm, H, &s_wbar[0], lane);
      pend[0] = true;
    }
    for (int u = cta * kAttnGroups + agrp; u < P.NKV * nsplit; u += grid * kAttnGroups)
      attn_unit<REP>(P, Ly, u % P.NKV, u / P.NKV, Ld, nsplit, cur_len, pos, gsm, gtid, 1 + agrp);
    if (!grid_sync(P.bar, ++nb, grid, &s_ok)) return bail();
    // ---- phase 3: combine the splits, spread over the whole grid
    if (nsplit > 1) {
      for (int e = cta * kThreads + threadIdx.x; e < NQD; e += grid * kThreads)
        P.attn[e] = combine_one(P, e / kHD, e % kHD, nsplit);
      if (!grid_sync(P.bar, ++nb, grid, &s_ok)) return bail();
    }
    // ---- phase 4: o + residual -> h2, from buffer B
    load_x(P.attn, NQD, xs);
    if (!wait_weights(&s_wbar[1], ph[1])) return bail();
    ph[1] ^= 1;
    pend[1] = false;
    chunk_biases(xs, NQD / 128, sb, warp, lane);
    __syncthreads();
    gemv_compute(bufB, NQD, n_h, xs, sb, red, warp, lane);
    __syncthreads();
    for (int e = threadIdx.x; e < n_h * 16; e += kThreads) {
      const int slot = e >> 4, r = e & 15;
      const int row = (cta + grid * slot) * 16 + r;
      half hv = __float2half_rn(slot_sum(red, slot, r));
      hv = __float2half_rn(__half2float(ld_cg_half(P.x + row)) + __half2float(hv));
      P.h2[row] = hv;
    }
    if (!grid_sync(P.bar, ++nb, grid, &s_ok)) return bail();
    // ---- phase 5: RMSNorm(h2) -> gate / up -> SwiGLU, from buffer A
    if (warp == kFillWarp) {  // buffer B: this layer's down
      const Mat md[1] = {{Ly.w[6], Ly.s[6], H / 16}};
      fill_weights<1, false>(md, I, H / 16, cta, grid, bufB, nullptr, 0, &s_wbar[1], lane);
      pend[1] = true;
    }
    load_x(P.h2, H, xs);
    if (!wait_weights(&s_wbar[0], ph[0])) return bail();
    ph[0] ^= 1;
    pend[0] = false;
    cta_rmsnorm(xs, reinterpret_cast<const half*>(bufA + 2 * n_gu * slot_bytes(H)), H, P.eps, &s_inv, warp, lane);
    chunk_biases(xs, H / 128, sb, warp, lane);
    __syncthreads();
    gemv_compute(bufA, H, 2 * n_gu, xs, sb, red, warp, lane);
    __syncthreads();
    for (int e = threadIdx.x; e < n_gu * 16; e += kThreads) {
      const int m = e >> 4, r = e & 15;
      const int row = (cta + grid * m) * 16 + r;
      const float gv = __half2float(__float2half_rn(slot_sum(red, 2 * m, r)));
      half hv = __float2half_rn(slot_sum(red, 2 * m + 1, r));
      hv = __float2half_rn((gv / (1.0f + expf(-gv))) * __half2float(hv));
      P.hid[row] = hv;
    }
    if (!grid_sync(P.bar, ++nb, grid, &s_ok)) return bail();
    // ---- phase 6: down + residual -> x, from buffer B
    if (warp == kFillWarp && !last) {  // buffer A: the next layer's q / k / v (+ its input norm)
      const FusedLayer& Ln = P.layer[li + 1];
      const Mat3 mq = qkv_mats(Ln);
      fill_weights<3, false>(mq.m, H, qkv_units, cta, grid, bufA, Ln.in_norm, H, &s_wbar[0], lane);
      pend[0] = true;
    }
    load_x(P.hid, I, xs);
    if (!wait_weights(&s_wbar[1], ph[1])) return bail();
    ph[1] ^= 1;
    pend[1] = false;
    chunk_biases(xs, I / 128, sb, warp, lane);
    __syncthreads();
    gemv_compute(bufB, I, n_h, xs, sb, red, warp, lane);
    __syncthreads();
    for (int e = threadIdx.x; e < n_h * 16; e += kThreads) {
      const int slot = e >> 4, r = e & 15;
      const int row = (cta + grid * slot) * 16 + r;
      half hv = __float2half_rn(slot_sum(red, slot, r));
      hv = __float2half_rn(__half2float(ld_cg_half(P.h2 + row)) + __half2float(hv));
      P.x[row] = hv;
    }
    if (!last && !grid_sync(P.bar, ++nb, grid, &s_ok)) return bail();
    if (warp == kFillWarp && !last) {  // buffer B: the next layer's o
      const FusedLayer& Ln = P.layer[li + 1];
      const Mat mo[1] = {{Ln.w[3], Ln.s[3], H / 16}};
      fill_weights<1, false>(mo, NQD, H / 16, cta, grid, bufB, nullptr, 0, &s_wbar[1], lane);
      pend[1] = true;
    }
  }
  // every CTA is past its last barrier wait: the last one out resets the counters
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int done = atomicAdd(P.bar + 1, 1);
    if (done == grid - 1) {
      atomicExch(P.bar, 0);
      atomicExch(P.bar + 1, 0);
    }
  }
}

int64_t round256(int64_t v) { return (v + 255) / 256 * 256; }

int fused_smem_bytes(const FusedDecodeParams& P, int sms) {
  return fused_smem(P.H, P.I, P.NQ * kHD, P.NKV * kHD, P.NQ / P.NKV, P.lmax, sms).total;
}

template <int REP>
cudaError_t launch_rep(const FusedDecodeParams& P, int sms, cudaStream_t stream) {
  auto kernel = decode_fused_kernel<REP>;
  const int smem = fused_smem_bytes(P, sms);
  if (cudaError_t e = ensure_smem_attr<decode_fused_kernel<REP>>(smem); e != cudaSuccess) return e;
  int per_sm = 0;
  if (cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem); e != cudaSuccess)
    return e;
  if (per_sm < 1) return cudaErrorCooperativeLaunchTooLarge;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sms);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: they meet at grid barriers
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, P);
}

}  // namespace

int64_t decode_fused_workspace_bytes(int64_t H, int64_t I, int64_t NQ, int64_t NKV, int64_t HD) {
  return 256 + round256(NQ * HD * 2) * 2 + round256(NKV * HD * 2) * 2 + round256(H * 2) + round256(I * 2) +
         round256(NQ * kMaxSplits * HD * 4) + round256(NQ * kMaxSplits * 2 * 4);
}

bool plan_decode_fused(FusedDecodeParams& P, void* workspace, int64_t workspace_bytes, int sms) {
  if (P.layers < 1 || P.layers > kFusedMaxLayers || P.HD != kHD || P.NKV < 1 || P.NQ % P.NKV != 0) return false;
  const int rep = P.NQ / P.NKV;
  if (rep != 1 && rep != 2 && rep != 4) return false;
  if (P.H % 128 != 0 || P.I % 128 != 0 || P.max_seq < 1) return false;
  const int NQD = P.NQ * kHD, NKVD = P.NKV * kHD;
  auto slots = [&](int units, int nt) { return (units + sms - 1) / sms * nt; };
  if (slots((NQD + 2 * NKVD) / 16, 1) > kMaxSlots || slots(P.H / 16, 1) > kMaxSlots || slots(P.I / 16, 2) > kMaxSlots)
    return false;
  // the split layout of attention.cu (one group of all the kv head's query heads)
  int cap = (592 + P.NKV - 1) / P.NKV;
  if (cap > kMaxSplits) cap = kMaxSplits;
  P.cap = cap;
  const int64_t want = split_want((int)(P.max_seq < (1 << 30) ? P.max_seq : (1 << 30)), cap);
  const int64_t lplan = (P.max_seq + want - 1) / want;
  P.lmax = (int)(lplan > 16 ? lplan : 16);
  P.scale_log2 = (1.0f / sqrtf((float)kHD)) * 1.4426950408889634f;
  if (workspace_bytes < decode_fused_workspace_bytes(P.H, P.I, P.NQ, P.NKV, kHD)) return false;
  uint8_t* w = reinterpret_cast<uint8_t*>(workspace);
  P.bar = reinterpret_cast<int*>(w);
  w += 256;
  P.q = reinterpret_cast<half*>(w);
  w += round256(NQD * 2);
  P.attn = reinterpret_cast<half*>(w);
  w += round256(NQD * 2);
  P.k = reinterpret_cast<half*>(w);
  w += round256(NKVD * 2);
  P.v = reinterpret_cast<half*>(w);
  w += round256(NKVD * 2);
  P.h2 = reinterpret_cast<half*>(w);
  w += round256((int64_t)P.H * 2);
  P.hid = reinterpret_cast<half*>(w);
  w += round256((int64_t)P.I * 2);
  P.ws_acc = reinterpret_cast<float*>(w);
  w += round256((int64_t)P.NQ * kMaxSplits * kHD * 4);
  P.ws_ml = reinterpret_cast<float*>(w);
  return fused_smem_bytes(P, sms) <= 227 * 1024 - 256;  // room for the static shared variables
}

cudaError_t launch_decode_fused(const FusedDecodeParams& P, int sms, cudaStream_t stream) {
  switch (P.NQ / P.NKV) {
    case 1: return launch_rep<1>(P, sms, stream);
    case 2: return launch_rep<2>(P, sms, stream);
    case 4: return launch_rep<4>(P, sms, stream);
  }
  return cudaErrorInvalidValue;
}

cudaError_t read_and_clear_decode_fused_error(int* out) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(out, g_decode_fused_error, sizeof(int));
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(g_decode_fused_error, &zero, sizeof(int));
}

}  // namespace soinfer
