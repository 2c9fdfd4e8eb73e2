// Streaming INT4 GEMV over a list of independent GEMVs: the weight stream of
// many matrices in one launch, every warp its own pipeline.
//
// Why a second batched kernel: in the persistent batched GEMV (gemv_batch.cu)
// a CTA's slab of each task is split along K across a group of warps, so
// every task costs a hand-off chain (x ready -> items -> partial rows ->
// epilogue sum) and the consumer warps spend most cycles waiting on it.  When
// no task of a launch reads another task's output, none of that is needed:
// here a warp owns whole units -- T 16-row tiles over the full K -- so its
// row sums never leave registers, and it fetches its own operands.
//
// Work split: units (task, 16*T rows) are handed out in task order by a
// global ticket (one atomicAdd per unit, grabbed one unit ahead); the planner
// orders the tasks by decreasing K (bigger units first, so the launch ends on
// the smallest ones).  Rows past N are clamped on load and never stored.
//
// Dependencies (a task whose x is an earlier task's y): the planner puts every
// task after the one it waits for (dependency level first, then K), so all of
// a task's units are numbered before any unit that waits for it.  A warp
// counts each finished unit of a waited-for task (release); when its fetch
// cursor reaches a waiting unit whose dependency is not complete it leaves a
// bubble stage instead of blocking, and polls again as the bubble comes round,
// so it always finishes the units it already holds first.  The lowest-numbered
// unfinished unit therefore never waits, and the launch cannot deadlock on a
// dependency; the wait is still bounded (kStreamWaitNs, then an error bit).
//
// Per warp: a private ring of D shared-memory stages, each one 128-K chunk of
// the unit -- 16*T rows x 64 B of packed weights (cp.async 16 B per lane per
// 8 rows), the chunk's 256 B of x (8 B per lane) and the rows' scales for the
// chunk's group (4 B per lane) -- plus a 16-byte tag (task, row0, chunk,
// flags) written by lane 0.  The fetch of chunk i + D is issued right after
// chunk i is read out of its stage, so D chunks per warp are always in flight
// (16 warps x D x 16T x 64 B per SM); completion is cp.async.wait_group, no
// mbarrier and no cross-warp synchronisation.  The fetch cursor runs ahead
// across unit boundaries, so the pipeline never drains between units.
//
// Math per chunk (identical to gemv_batch.cu's): the biased LOP3 unpack into
// exact fp16 (1024 + (n ^ 8), 1024 + 16 (n ^ 8)) feeding mma.sync.m16n8k16
// with x in B column 0 (fp32 accumulation; rows g, g + 8 of the result live in
// the lanes with t == 0, which store them), the bias removed
// with the chunk's x sums (one MMA), then acc = fma(scale, dot - bias, acc)
// in chunk order -- so a row's result depends only on its own bytes and x.
//
// Reference semantics per GEMV: csrc/kernels/gemv_w4a16_group.cu:77-127 of
// sparse-offload-infer (y[n] = half(sum_k s[n, k/g] * q[n,k] * x[k]), fp32
// accumulation).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"

namespace soinfer {

__device__ int g_gemv_stream_error;

namespace {

constexpr uint32_t kStreamWaitNs = 1000000000u;  // 1 s: a dependency that never completes sets an error bit

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}


// Stage layout for units of T 16-row tiles and MT token columns (1, or up
// to 8 for the multi-token form).
template <int T, int MT>
struct StageLayout {
  static constexpr int kRows = 16 * T;
  static constexpr int kW = 0;                   // [2T row groups][32 lanes][16 B]
  static constexpr int kX = kRows * 64;          // per token: the chunk's 256 B of x, t-pieces 2 / 3 shifted by 16 B
  static constexpr int kS = kX + 288 * MT;       // [kRows] fp32 scales
  static constexpr int kTag = kS + kRows * 4;    // int4 tag
  static constexpr int kBytes = kTag + 16;
};

__device__ __forceinline__ void cpa16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cpa8(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cpa4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cpa_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cpa_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// The LOP3 constants of the unpack, held in registers for the whole kernel
// (asm-defined, so the compiler cannot re-materialise them at every use).
struct UnpackK {
  uint32_t lo, hi;  // 0x6408 / 0x6480 per half: the fp16 1024 exponent with the n ^ 8 bias bit
  __device__ __forceinline__ UnpackK() {
    asm volatile("mov.b32 %0, 0x64086408;" : "=r"(lo));
    asm volatile("mov.b32 %0, 0x64806480;" : "=r"(hi));
  }
};

// D = A * B with a zero accumulator (the first MMA of a chain).
__device__ __forceinline__ void mma_16816_c0(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
}

// Biased row sums of one 128-K chunk for rows g and g + 8 of a 16-row tile
// (see gemv_batch.cu): returns E + O / 16 per row.  PAIRED: each 16-byte x
// fragment holds (x0x1, x4x5, x2x3, x6x7) -- the stage stores x that way --
// so each MMA's two B registers are adjacent; otherwise (x0x1, x2x3, x4x5,
// x6x7) as in memory.
template <bool PAIRED>
__device__ __forceinline__ void st_chunk_dot(const uint4 wa, const uint4 wb, const uint4 xf[4], const UnpackK& k,
                                             float& s0, float& s1) {
  const uint32_t r0[4] = {wa.x, wa.y, wa.z, wa.w};
  const uint32_t r1[4] = {wb.x, wb.y, wb.z, wb.w};
  float e[4], o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t t0 = r0[j] >> 8, t1 = r1[j] >> 8;
    const uint32_t ae[4] = {lop3_and_xor(r0[j], 0x000f000fu, k.lo), lop3_and_xor(r1[j], 0x000f000fu, k.lo),
                            lop3_and_xor(t0, 0x000f000fu, k.lo), lop3_and_xor(t1, 0x000f000fu, k.lo)};
    const uint32_t be0 = xf[j].x, be1 = PAIRED ? xf[j].y : xf[j].z;
    if (j == 0) mma_16816_c0(e, ae, be0, be1);
    else mma_16816(e, ae, be0, be1);  // (v0,v1) with x0x1, (v4,v5) with x4x5
    const uint32_t ao[4] = {lop3_and_xor(r0[j], 0x00f000f0u, k.hi), lop3_and_xor(r1[j], 0x00f000f0u, k.hi),
                            lop3_and_xor(t0, 0x00f000f0u, k.hi), lop3_and_xor(t1, 0x00f000f0u, k.hi)};
    const uint32_t bo0 = PAIRED ? xf[j].z : xf[j].y, bo1 = xf[j].w;
    if (j == 0) mma_16816_c0(o, ao, bo0, bo1);
    else mma_16816(o, ao, bo0, bo1);  // (v2,v3) with x2x3, (v6,v7) with x6x7
  }
  s0 = fmaf(o[0], 0.0625f, e[0]);
  s1 = fmaf(o[2], 0.0625f, e[2]);
}

// Multi-token form of st_chunk_dot: B column n carries token n, so every D
// element is a distinct (row, token) sum: s[0] = (g, 2t), s[1] = (g, 2t + 1),
// s[2] = (g + 8, 2t), s[3] = (g + 8, 2t + 1).
__device__ __forceinline__ void st_chunk_dot4(const uint4 wa, const uint4 wb, const uint4 xf[4], const UnpackK& k,
                                              float s[4]) {
  const uint32_t r0[4] = {wa.x, wa.y, wa.z, wa.w};
  const uint32_t r1[4] = {wb.x, wb.y, wb.z, wb.w};
  float e[4] = {0.f, 0.f, 0.f, 0.f}, o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t t0 = r0[j] >> 8, t1 = r1[j] >> 8;
    const uint32_t ae[4] = {lop3_and_xor(r0[j], 0x000f000fu, k.lo), lop3_and_xor(r1[j], 0x000f000fu, k.lo),
                            lop3_and_xor(t0, 0x000f000fu, k.lo), lop3_and_xor(t1, 0x000f000fu, k.lo)};
    mma_16816(e, ae, xf[j].x, xf[j].z);
    const uint32_t ao[4] = {lop3_and_xor(r0[j], 0x00f000f0u, k.hi), lop3_and_xor(r1[j], 0x00f000f0u, k.hi),
                            lop3_and_xor(t0, 0x00f000f0u, k.hi), lop3_and_xor(t1, 0x00f000f0u, k.hi)};
    mma_16816(o, ao, xf[j].y, xf[j].w);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) s[i] = fmaf(o[i], 0.0625f, e[i]);
}

// Per-token chunk biases for the multi-token form, from the x fragments the
// lane already holds: with A uniform (1032 for the low-nibble positions x0
// x1 x4 x5 of each 8-group, 72 for the high ones), column n of D sums
// token n's x over the positions its B operand covers; eight MMAs cover the
// chunk, so b[0] / b[1] = the bias of tokens 2t / 2t + 1.
__device__ __forceinline__ void st_chunk_bias_tokens(const uint4 xf[4], float b[2]) {
  const uint32_t lo[4] = {0x64086408u, 0x64086408u, 0x64086408u, 0x64086408u};  // 1032
  const uint32_t hi[4] = {0x54805480u, 0x54805480u, 0x54805480u, 0x54805480u};  // 72
  float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    mma_16816(d, lo, xf[j].x, xf[j].z);
    mma_16816(d, hi, xf[j].y, xf[j].w);
  }
  b[0] = d[0];
  b[1] = d[1];
}

// The chunk's bias 1032 XL + 72 XH (gemv_batch.cu chunk_bias) from this
// lane's 8 bytes of the chunk's paired x (stage bytes 8 * lane ..): lanes with
// even t hold two low-position pairs (x0x1, x4x5 of an 8-group), lanes with
// odd t two high-position pairs, so the lane's A is 1032 or 72 throughout;
// column n of D sums 16 of the chunk's 128 values, and the 8 columns are
// summed across the 4 lanes of a row group.
__device__ __forceinline__ float st_chunk_bias(uint2 xw, int t) {
  const uint32_t c = (t & 1) ? 0x54805480u : 0x64086408u;  // 72 | 1032
  const uint32_t a[4] = {c, c, c, c};
  float d[4];
  mma_16816_c0(d, a, xw.x, xw.y);
  float bias = d[0] + d[1];
  bias += __shfl_xor_sync(0xffffffffu, bias, 1);
  bias += __shfl_xor_sync(0xffffffffu, bias, 2);
  return bias;
}

// Fetch cursor: the unit being fetched and this lane's source pointers at
// the current chunk (set once per unit, advanced by adds per chunk).
template <int T, int MT>
struct Cursor {
  static constexpr int kSP = (16 * T + 31) / 32;  // scale rows per lane
  static constexpr int kXP = MT == 1 ? 1 : MT / 2;  // x pieces per lane (8 B for one token, else 16 B)
  const uint8_t* wp[2 * T];  // 16 B of row row0 + g + 8r (clamped to N - 1) at the chunk
  const float* sp[kSP];      // scale of row row0 + lane + 32i (clamped) at the chunk's group
  const half* xp[kXP];       // this lane's x pieces at the chunk (token (lane + 32i) / 16, clamped to m - 1)
  int task, row0, chunk, nch, sub, cpg;
  bool done, ready;  // ready: the unit's dependency (if any) is complete
};

template <int T, int MT, class P>
__device__ __forceinline__ void st_resolve(const P& B, int u, int lane, Cursor<T, MT>& c) {
  if (u >= B.total_units) {
    c.done = true;
    return;
  }
  int lo = 0, hi = B.num - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (B.tasks[mid].ubegin <= u) lo = mid;
    else hi = mid - 1;
  }
  const auto& tk = B.tasks[lo];
  c.task = lo;
  c.row0 = (u - tk.ubegin) * (16 * T);
  c.chunk = 0;
  c.nch = tk.K >> 7;
  c.sub = 0;
  c.cpg = tk.cpg;
  c.ready = tk.dep < 0;
  const int64_t rb = tk.K >> 1;
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int r = 0; r < 2 * T; ++r) c.wp[r] = tk.W + (int64_t)min(c.row0 + g + 8 * r, tk.N - 1) * rb + t * 16;
#pragma unroll
  for (int i = 0; i < Cursor<T, MT>::kSP; ++i)
    c.sp[i] = tk.S + (int64_t)min(c.row0 + lane + 32 * i, tk.N - 1) * tk.G;
  if constexpr (MT == 1) {
    c.xp[0] = tk.x + lane * 4;
  } else {
#pragma unroll
    for (int i = 0; i < Cursor<T, MT>::kXP; ++i) {
      const int p = lane + 32 * i;
      c.xp[i] = tk.x + (int64_t)min(p >> 4, B.m - 1) * tk.ldx + (p & 15) * 8;
    }
  }
}

template <int T, int D, int W, int MT, class P>
__global__ void __launch_bounds__(W * 32, 1) gemv_stream_kernel(const __grid_constant__ P B, int* __restrict__ ctr) {
  using L = StageLayout<T, MT>;
  using C = Cursor<T, MT>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  uint8_t* ring = smem + warp * (D * L::kBytes);
  const uint32_t ring_u32 = smem_u32(ring);
  // per-warp bubble-run state after the rings: [start (low clock bits), length]; the
  // address is re-derived where used (tid read in asm) so no register holds it
  auto wait_state = [&]() {
    uint32_t tid;
    asm volatile("mov.u32 %0, %%tid.x;" : "=r"(tid));
    return reinterpret_cast<uint32_t*>(smem + W * D * L::kBytes) + 2 * (tid >> 5);
  };
  if (lane == 0) wait_state()[1] = 0;

  // first unit, and the next one grabbed ahead (lane 0 holds it)
  int nxt = 0, first = 0;
  if (lane == 0) {
    first = atomicAdd(ctr, 1);
    nxt = atomicAdd(ctr, 1);
  }
  C f;
  f.done = false;
  st_resolve(B, __shfl_sync(0xffffffffu, first, 0), lane, f);
  const UnpackK uk;

  auto fetch = [&](int s) {
    const uint32_t st = ring_u32 + s * L::kBytes;
    if (f.done) {
      if (lane == 0) *reinterpret_cast<int4*>(ring + s * L::kBytes + L::kTag) = make_int4(0, 0, 0, 0);
      cpa_commit();
      return;
    }
    if (!f.ready) {  // a waiting unit: every unit of its dependency stored yet?
      const auto& tk = B.tasks[f.task];
      int have = 0;
      if (lane == 0) have = ld_acquire_gpu(ctr + 2 + tk.dep);
      if (__shfl_sync(0xffffffffu, have, 0) < tk.dneed) {
        if (lane == 0) *reinterpret_cast<int4*>(ring + s * L::kBytes + L::kTag) = make_int4(0, 0, 0, 4);
        cpa_commit();
        return;  // a bubble stage; polled again when the consumer reaches it
      }
      f.ready = true;
      if (lane == 0) wait_state()[1] = 0;  // the run of bubbles (if any) ends here
      __syncwarp();  // lane 0's acquire before any lane's copy of x
    }
#pragma unroll
    for (int r = 0; r < 2 * T; ++r) cpa16(st + L::kW + r * 512 + lane * 16, f.wp[r]);
    if constexpr (MT == 1) {
      // paired layout: word i of the chunk (4 bytes) goes to slot i with its
      // two middle words of every 4 swapped, then the t-piece padding
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int i = 2 * lane + h;
        const int b = ((i & ~3) | ((i & 1) << 1) | ((i >> 1) & 1)) * 4;
        cpa4(st + L::kX + b + ((b >> 7) << 4), f.xp[0] + 2 * h);
      }
    } else {
#pragma unroll
      for (int i = 0; i < C::kXP; ++i) {
        const int p = lane + 32 * i, c16 = p & 15;
        cpa16(st + L::kX + (p >> 4) * 288 + c16 * 16 + ((c16 >> 3) << 4), f.xp[i]);
      }
    }
#pragma unroll
    for (int i = 0; i < C::kSP; ++i)
      if (lane + 32 * i < L::kRows) cpa4(st + L::kS + (lane + 32 * i) * 4, f.sp[i]);
    if (lane == 0)
      *reinterpret_cast<int4*>(ring + s * L::kBytes + L::kTag) =
          make_int4(f.task, f.row0, f.chunk, (f.chunk == f.nch - 1 ? 2 : 0) | 1);
    cpa_commit();
    // advance the cursor (chunk -> scale group -> next unit)
    if (++f.chunk == f.nch) {
      const int u = __shfl_sync(0xffffffffu, nxt, 0);
      if (lane == 0) nxt = atomicAdd(ctr, 1);
      st_resolve(B, u, lane, f);
    } else {
#pragma unroll
      for (int r = 0; r < 2 * T; ++r) f.wp[r] += 64;
#pragma unroll
      for (int i = 0; i < C::kXP; ++i) f.xp[i] += 128;
      if (++f.sub == f.cpg) {
        f.sub = 0;
#pragma unroll
        for (int i = 0; i < C::kSP; ++i) ++f.sp[i];
      }
    }
  };

#pragma unroll
  for (int s = 0; s < D; ++s) fetch(s);

  constexpr int kAcc = MT == 1 ? 2 * T : 4 * T;  // per tile: rows g, g + 8 (x tokens 2t, 2t + 1)
  float acc[kAcc];
#pragma unroll
  for (int r = 0; r < kAcc; ++r) acc[r] = 0.f;
  const int xoff = L::kX + (MT == 1 ? 0 : g * 288) + t * 64 + ((t >> 1) << 4);
  const int boff = L::kX + lane * 8 + ((lane >> 4) << 4);
  int s = 0;
  while (true) {
    cpa_wait<D - 1>();
    __syncwarp();
    const uint8_t* stg = ring + s * L::kBytes;
    const int4 tag = *reinterpret_cast<const int4*>(stg + L::kTag);
    if (tag.w & 4) {  // a bubble: the fetch cursor waits for a dependency
      __syncwarp();   // every lane has read the tag before fetch rewrites it
      if (!f.done) {
        int give_up = 0;
        if (lane == 0) {  // wait[0]: start of this run of bubbles (low clock bits), wait[1]: its length
          uint32_t* wait = wait_state();
          const uint32_t now = (uint32_t)globaltimer_ns();
          if (wait[1]++ == 0) wait[0] = now;
          else give_up = now - wait[0] > kStreamWaitNs;  // modular: valid for waits under 4 s
        }
        if (__shfl_sync(0xffffffffu, give_up, 0)) {
          if (lane == 0) atomicOr(&g_gemv_stream_error, kErrCopyTimeout);
          f.done = true;  // give up: the warp drains its ring and exits
        }
        __nanosleep(256);
      }
      fetch(s);
      s = (s + 1 == D) ? 0 : s + 1;
      continue;
    }
    if (!(tag.w & 1)) break;
    uint4 w[2 * T];
#pragma unroll
    for (int r = 0; r < 2 * T; ++r) w[r] = *reinterpret_cast<const uint4*>(stg + L::kW + r * 512 + lane * 16);
    uint4 xf[4];
    if constexpr (MT == 1) {
      // one token: only B column 0 (lanes g == 0) carries x, the other seven
      // columns are zero -- D column 0 is the same sum (the columns are
      // independent), with 1/8 of the x reads from shared memory and far less
      // multiplier switching (measured at the power cap: +1.2% sustained)
#pragma unroll
      for (int j = 0; j < 4; ++j) xf[j] = make_uint4(0u, 0u, 0u, 0u);
      if (g == 0) {
#pragma unroll
        for (int j = 0; j < 4; ++j) xf[j] = *reinterpret_cast<const uint4*>(stg + xoff + j * 16);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) xf[j] = *reinterpret_cast<const uint4*>(stg + xoff + j * 16);
    }
    uint2 xb = make_uint2(0, 0);
    if constexpr (MT == 1) xb = *reinterpret_cast<const uint2*>(stg + boff);
    float sc[2 * T];
#pragma unroll
    for (int r = 0; r < 2 * T; ++r) sc[r] = reinterpret_cast<const float*>(stg + L::kS)[g + 8 * r];
    __syncwarp();  // every lane has read the stage: refill it with the chunk D ahead
    fetch(s);
    if constexpr (MT == 1) {
      const float bias = st_chunk_bias(xb, t);
#pragma unroll
      for (int tt = 0; tt < T; ++tt) {
        float d0, d1;
        st_chunk_dot<true>(w[2 * tt], w[2 * tt + 1], xf, uk, d0, d1);
        acc[2 * tt] = fmaf(sc[2 * tt], d0 - bias, acc[2 * tt]);
        acc[2 * tt + 1] = fmaf(sc[2 * tt + 1], d1 - bias, acc[2 * tt + 1]);
      }
    } else {
      float bt[2];
      st_chunk_bias_tokens(xf, bt);
#pragma unroll
      for (int tt = 0; tt < T; ++tt) {
        float d[4];
        st_chunk_dot4(w[2 * tt], w[2 * tt + 1], xf, uk, d);
        acc[4 * tt + 0] = fmaf(sc[2 * tt], d[0] - bt[0], acc[4 * tt + 0]);
        acc[4 * tt + 1] = fmaf(sc[2 * tt], d[1] - bt[1], acc[4 * tt + 1]);
        acc[4 * tt + 2] = fmaf(sc[2 * tt + 1], d[2] - bt[0], acc[4 * tt + 2]);
        acc[4 * tt + 3] = fmaf(sc[2 * tt + 1], d[3] - bt[1], acc[4 * tt + 3]);
      }
    }
    if (tag.w & 2) {  // last chunk of the unit: rows g + 8r of the unit
      const auto& tk = B.tasks[tag.x];
      if constexpr (MT == 1) {
        if (t == 0) {
#pragma unroll
          for (int r = 0; r < 2 * T; ++r) {
            const int row = tag.y + g + 8 * r;
            if (row < tk.N) tk.y[row] = __float2half_rn(acc[r]);
          }
        }
      } else {
#pragma unroll
        for (int tt = 0; tt < T; ++tt)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int row = tag.y + 16 * tt + g + 8 * (q >> 1), tok = 2 * t + (q & 1);
            if (row < tk.N && tok < B.m) tk.y[(int64_t)tok * tk.ldy + row] = __float2half_rn(acc[4 * tt + q]);
          }
      }
#pragma unroll
      for (int r = 0; r < kAcc; ++r) acc[r] = 0.f;
      if (tk.publish) {  // a task that others wait for: count the stored unit (release)
        __syncwarp();
        if (lane == 0) {
          __threadfence();
          atomicAdd(ctr + 2 + tag.x, 1);
        }
      }
    }
    s = (s + 1 == D) ? 0 : s + 1;
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  // the last warp out resets the ticket and the exit count for the next launch
  if (lane == 0) {
    __threadfence();
    const int done = atomicAdd(ctr + 1, 1);
    if (done == B.total_warps - 1) {
      for (int i = 0; i < B.num; ++i)
        if (B.tasks[i].publish) atomicExch(ctr + 2 + i, 0);
      atomicExch(ctr, 0);
      atomicExch(ctr + 1, 0);
    }
  }
}

template <int T, int D, int W, int MT, class P>
cudaError_t launch_stream_params(const P& B, int* ctr, cudaStream_t stream) {
  auto kernel = gemv_stream_kernel<T, D, W, MT, P>;
  const int smem = W * D * StageLayout<T, MT>::kBytes + W * 8;
  if (cudaError_t e = ensure_smem_attr<gemv_stream_kernel<T, D, W, MT, P>>(smem); e != cudaSuccess) return e;
  kernel<<<B.grid, W * 32, smem, stream>>>(B, ctr);
  return cudaGetLastError();
}

}  // namespace

int64_t gemv_stream_workspace_bytes(int64_t num_tasks) { return ((num_tasks + 2) * 4 + 255) / 256 * 256; }

cudaError_t read_and_clear_gemv_stream_error(int* out) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(out, g_gemv_stream_error, sizeof(int));
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(g_gemv_stream_error, &zero, sizeof(int));
}

bool plan_gemv_stream(GemvStreamParams& B, int sms) {
  if (B.num < 1 || B.num > kMaxBatchTasks) return false;
  // Order: dependency level first (a task after the one it waits for), then
  // bigger units first -- decreasing K, stable.  (Measured: smaller units at
  // the end of the order, to shorten the tail, cost more in per-unit overhead
  // than they saved.)
  int level[kMaxBatchTasks], order[kMaxBatchTasks], where[kMaxBatchTasks];
  for (int i = 0; i < B.num; ++i) {
    const int d = B.tasks[i].dep;
    if (d >= i || d < -1) return false;  // deps name earlier tasks only
    level[i] = d < 0 ? 0 : level[d] + 1;
    order[i] = i;
  }
  std::stable_sort(order, order + B.num, [&](int a, int b) {
    if (level[a] != level[b]) return level[a] < level[b];
    return B.tasks[a].K > B.tasks[b].K;
  });
  GemvStreamTask sorted[kMaxBatchTasks];
  for (int i = 0; i < B.num; ++i) {
    sorted[i] = B.tasks[order[i]];
    where[order[i]] = i;
  }
  int64_t u = 0;
  for (int i = 0; i < B.num; ++i) {
    GemvStreamTask& tk = sorted[i];
    if (tk.K % 128 != 0 || tk.cpg < 1 || tk.N < 1) return false;
    tk.ubegin = (int)u;
    tk.publish = 0;
    u += (tk.N + 16 * kStreamTiles - 1) / (16 * kStreamTiles);
  }
  if (u >= (1 << 30)) return false;
  for (int i = 0; i < B.num; ++i) {
    GemvStreamTask& tk = sorted[i];
    if (tk.dep >= 0) {
      const int d = where[tk.dep];
      tk.dep = d;
      tk.dneed = (sorted[d].N + 16 * kStreamTiles - 1) / (16 * kStreamTiles);
      sorted[d].publish = 1;
    } else {
      tk.dneed = 0;
    }
  }
  for (int i = 0; i < B.num; ++i) B.tasks[i] = sorted[i];
  B.total_units = (int)u;
  B.grid = sms;
  B.total_warps = sms * kStreamWarps;
  return true;
}

cudaError_t launch_gemv_stream(const GemvStreamParams& B, int* ctr, cudaStream_t stream) {
  if (B.m > 1) return launch_stream_params<kStreamTiles, kStreamStages, kStreamWarps, 8>(B, ctr, stream);
  if (B.num <= kSmallBatchTasks) {
    GemvStreamParamsT<kSmallBatchTasks> S;
    S.num = B.num;
    S.grid = B.grid;
    S.total_units = B.total_units;
    S.total_warps = B.total_warps;
    S.m = B.m;
    for (int i = 0; i < B.num; ++i) S.tasks[i] = B.tasks[i];
    return launch_stream_params<kStreamTiles, kStreamStages, kStreamWarps, 1>(S, ctr, stream);
  }
  return launch_stream_params<kStreamTiles, kStreamStages, kStreamWarps, 1>(B, ctr, stream);
}

}  // namespace soinfer
