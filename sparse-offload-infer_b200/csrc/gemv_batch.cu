// Persistent batched INT4 GEMV: one cooperative launch runs a list of GEMVs
// (y_i = dequant(W_i, S_i) x_i), optionally chained (x_i = y_j of an earlier
// task j) -- a decode layer's or a whole token's weight stream in one kernel.
//
// Why: a batch-1 decode GEMV moves ~6.7 MB, i.e. ~42 KB per SM, while an SM
// needs ~100 KB of copies in flight to run HBM at full rate; a single GEMV
// launch is therefore latency-bound no matter how it is written.  Weights do
// not depend on activations, so here a producer warp per CTA streams the
// weight pieces of task after task through a deep shared-memory ring
// (cp.async.bulk + full/empty mbarriers) without ever waiting for x; a loader
// warp double-buffers each task's x (bulk copy), waiting first for the task it
// depends on (a per-task completion counter in global memory reaching the grid
// size); consumer warps compute as weights and x land.
//
// Per task each CTA owns a contiguous, equal slab of output rows (no
// cross-CTA reduction).  Dot products: each packed word is turned into fp16
// values biased by a constant with a single LOP3 per half2 -- (n^8)+1024 for
// the low nibble of each byte pair, 16(n^8)+1024 for the high nibble -- and
// fed to mma.sync.m16n8k16 (exact products, fp32 accumulation) in two chains
// (low / high nibbles); the bias is removed per 128-K chunk with the chunk's
// x sums: sum q x = (E - 1032 XL) + (O - 1152 XH) / 16.  That leaves ~0.6
// SIMT instructions per INT4 value.
//
// Every wait is bounded (%globaltimer); a timeout sets a device error bit and
// the CTA drains its in-flight copies and exits.  The completion counters
// (workspace) are reset to zero by the last CTA to finish, so a zeroed
// workspace stays reusable across launches and CUDA-graph replays.
//
// Reference semantics per task: csrc/kernels/gemv_w4a16_group.cu:77-127 of
// sparse-offload-infer.
#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"

namespace soinfer {

namespace {

__device__ int g_gemv_batch_error;

constexpr int kCWarps = 16;                   // consumer warps (0..15)
constexpr int kCThreads = kCWarps * 32;
constexpr int kPWarps = 4;                    // producer warps (16..19): one warp issues copies serially,
                                              // so the 16 row copies of a stage are spread over 4 warps
constexpr int kLoaderWarp = kCWarps + kPWarps;
constexpr int kThreads = (kCWarps + kPWarps + 1) * 32;
constexpr int kMaxStages = 10;
constexpr int kPieceChunks = 16;              // 128-K chunks per stage row piece: one per consumer warp
constexpr int kMaxPieces = 16;                // K <= 32768
constexpr int kSlotPad = 64;
constexpr int kMaxTilesPerTask = 8;           // 16-row tiles per CTA per task
constexpr uint64_t kWaitNs = 1000000000ull;   // 1 s
constexpr int kSmemBudget = 220 * 1024;

__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// Named barrier over `n` threads that also ORs `pred` across them: every
// participant gets the same answer (uniform control flow after the barrier).
__device__ __forceinline__ bool named_sync_or(int id, int n, bool pred) {
  uint32_t out;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(out)
      : "r"((uint32_t)pred), "r"(id), "r"(n)
      : "memory");
  return out != 0;
}

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Row sums of one 128-K chunk for the thread's two MMA rows (see file comment).
__device__ __forceinline__ void chunk_dot_biased(const uint4 wa, const uint4 wb, const uint4 xf[4], float xl,
                                                 float xh, float& s0, float& s1) {
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
  const float bl = 1032.f * xl, bh = 1152.f * xh;
  s0 = (e[0] - bl) + (o[0] - bh) * 0.0625f;
  s1 = (e[2] - bl) + (o[2] - bh) * 0.0625f;
}

struct TaskView {
  int rows, tiles, chunks, pieces;
  int64_t row0;
};

__device__ __forceinline__ TaskView task_view(const GemvBatchTask& tk, int cta) {
  TaskView v;
  v.row0 = (int64_t)cta * tk.rows_per_cta;
  int rows = tk.N - (int)v.row0;
  v.rows = rows < 0 ? 0 : (rows > tk.rows_per_cta ? tk.rows_per_cta : rows);
  v.tiles = (v.rows + 15) / 16;
  v.chunks = tk.K / 128;
  v.pieces = (v.chunks + kPieceChunks - 1) / kPieceChunks;
  return v;
}

// Lane 0 polls the barrier (with back-off) while the other lanes park in
// __syncwarp; the result is broadcast so the warp decides uniformly.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, uint64_t timeout_ns) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) {
    if (!mbar_try_wait(bar, parity)) {
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(bar, parity)) {
        if (globaltimer_ns() - t0 > timeout_ns) {
          ok = 0;
          break;
        }
        __nanosleep(20);
      }
    }
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok != 0;
}

__device__ __forceinline__ void red_release_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Low- / high-nibble-position sums of one 128-K chunk of x: each thread sums
// its 32-value slice, then the 4 lanes of a groupID (t = 0..3) combine.
__device__ __forceinline__ void chunk_xsums(const uint4 xf[4], float& xl, float& xh) {
  float lo = 0.f, hi = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 a = __half22float2(u32_as_h2(xf[j].x)), b = __half22float2(u32_as_h2(xf[j].y));
    const float2 c = __half22float2(u32_as_h2(xf[j].z)), d = __half22float2(u32_as_h2(xf[j].w));
    lo += (a.x + a.y) + (c.x + c.y);
    hi += (b.x + b.y) + (d.x + d.y);
  }
  lo += __shfl_xor_sync(0xffffffffu, lo, 1);
  hi += __shfl_xor_sync(0xffffffffu, hi, 1);
  lo += __shfl_xor_sync(0xffffffffu, lo, 2);
  hi += __shfl_xor_sync(0xffffffffu, hi, 2);
  xl = lo;
  xh = hi;
}

__global__ void __launch_bounds__(kThreads, 1)
    gemv_batch_kernel(const __grid_constant__ GemvBatchParams B, int* __restrict__ counters) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* xbuf = smem;                                     // [2][x_bytes]
  uint8_t* slots = smem + 2 * B.x_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(slots + B.stages * B.slot_bytes);
  uint64_t* empty = full + kMaxStages;
  uint64_t* xfull = empty + kMaxStages;
  uint64_t* xempty = xfull + 2;
  float* red = reinterpret_cast<float*>(xempty + 2);        // [kCWarps][kMaxTilesPerTask*16]
  __shared__ int s_abort;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int cta = blockIdx.x;
  const int grid = gridDim.x;
  const int S = B.stages;
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCWarps);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], kCWarps);
    }
    fence_mbar_init();
    s_abort = 0;
  }
  __syncthreads();

  if (warp >= kCWarps && warp < kLoaderWarp) {
    // ------------------------------------------------------------ producers
    // Items are ordered piece-major within a task (piece p of every tile,
    // then piece p + 1), matching the consumers.  Producer warp pw issues the
    // row copies of rows pw, pw + 4, ... (lanes 0..3); warp 0 also posts the
    // stage's expected byte count and copies the tile's scale rows.
    const int pw = warp - kCWarps;
    int item = 0;
    bool stop = false;
    for (int ti = 0; ti < B.num && !stop; ++ti) {
      const GemvBatchTask& tk = B.tasks[ti];
      const TaskView v = task_view(tk, cta);
      const int64_t row_bytes = tk.K / 2;
      const uint32_t srow = (uint32_t)tk.G * 4u;
      for (int piece = 0; piece < v.pieces && !stop; ++piece) {
        const int c0 = piece * kPieceChunks;
        const int pc = min(kPieceChunks, v.chunks - c0);
        for (int tile = 0; tile < v.tiles; ++tile, ++item) {
          const int slot = item % S;
          if (item >= S && !mbar_wait_bounded(&empty[slot], (uint32_t)(((item / S) - 1) & 1), kWaitNs)) {
            stop = true;
            break;
          }
          if (s_abort) {
            stop = true;
            break;
          }
          const int valid = min(16, v.rows - tile * 16);
          const int64_t r = v.row0 + tile * 16;
          uint8_t* sb = slots + slot * B.slot_bytes;
          if (pw == 0 && lane == 0)
            mbar_arrive_expect_tx(&full[slot], (uint32_t)(valid * pc * 64) + (uint32_t)valid * srow);
          const int row = lane * kPWarps + pw;
          if (lane < 4 && row < valid)
            bulk_g2s(sb + row * B.slot_stride, tk.W + (r + row) * row_bytes + (int64_t)c0 * 64, (uint32_t)(pc * 64),
                     &full[slot]);
          if (pw == 0 && lane == 4) bulk_g2s(sb + B.scale_off, tk.S + r * tk.G, (uint32_t)valid * srow, &full[slot]);
        }
      }
    }
    if (stop && lane == 0) {
      s_abort = 1;
      atomicOr(&g_gemv_batch_error, kErrCopyTimeout);
    }
    // drain: every issued stage must land before this CTA's shared memory is released
    for (int q = item - S; q < item; ++q)
      if (q >= 0) (void)mbar_wait_bounded(&full[q % S], (uint32_t)((q / S) & 1), kWaitNs / 4);
  } else if (warp == kLoaderWarp) {
    // ------------------------------------------------------------ x loader
    int issued = 0;
    bool stop = false;
    for (int ti = 0; ti < B.num && !stop; ++ti) {
      const GemvBatchTask& tk = B.tasks[ti];
      const int xs = ti & 1;
      int ok = 1;
      if (lane == 0) {
        if (ti >= 2 && !mbar_wait_bounded(&xempty[xs], (uint32_t)(((ti >> 1) - 1) & 1), kWaitNs)) ok = 0;
        if (ok && tk.dep >= 0) {
          const uint64_t t0 = globaltimer_ns();
          while (ld_acquire(counters + tk.dep) < grid) {
            if (s_abort || globaltimer_ns() - t0 > kWaitNs) {
              ok = 0;
              break;
            }
            __nanosleep(32);
          }
          fence_proxy_async_global();  // x was written by other SMs through the generic proxy
        }
        if (s_abort) ok = 0;
        if (ok) mbar_arrive_expect_tx(&xfull[xs], (uint32_t)tk.K * 2u);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        stop = true;
        break;
      }
      if (lane == 0) bulk_g2s(xbuf + xs * B.x_bytes, tk.x, (uint32_t)tk.K * 2u, &xfull[xs]);
      __syncwarp();
      issued = ti + 1;
    }
    if (stop && lane == 0) {
      s_abort = 1;
      atomicOr(&g_gemv_batch_error, kErrCopyTimeout);
    }
    if (lane == 0)
      for (int q = issued - 2; q < issued; ++q)
        if (q >= 0) (void)mbar_wait_bounded(&xfull[q & 1], (uint32_t)((q >> 1) & 1), kWaitNs / 4);
    __syncwarp();
  } else {
    // ------------------------------------------------------------ consumers
    // Abort decisions are made only through named_sync_or, so all consumer
    // threads leave the task loop together; a failed wait marks the thread
    // `bad`, after which it stops waiting and skips work until that barrier.
    const int g = lane >> 2, t = lane & 3;
    const int lr0 = g, lr1 = g + 8;
    int item = 0;
    bool bad = false;
    for (int ti = 0; ti < B.num; ++ti) {
      const GemvBatchTask& tk = B.tasks[ti];
      const TaskView v = task_view(tk, cta);
      const int xsl = ti & 1;
      if (!bad && !warp_wait(&xfull[xsl], (uint32_t)((ti >> 1) & 1), kWaitNs)) bad = true;
      const uint4* xs = reinterpret_cast<const uint4*>(xbuf + xsl * B.x_bytes);
      float acc0[kMaxTilesPerTask], acc1[kMaxTilesPerTask];
#pragma unroll
      for (int i = 0; i < kMaxTilesPerTask; ++i) acc0[i] = acc1[i] = 0.f;
      for (int piece = 0; piece < v.pieces; ++piece) {
        const int cg = piece * kPieceChunks + warp;  // the one chunk of this piece this warp owns
        const bool mine = cg < v.chunks;
        uint4 xf[4];
        float xl = 0.f, xh = 0.f;
        if (!bad && mine) {
          const uint4* xc = xs + cg * 16 + t * 4;
#pragma unroll
          for (int j = 0; j < 4; ++j) xf[j] = xc[j];
          chunk_xsums(xf, xl, xh);
        }
        const int grp = cg / tk.cpg;
#pragma unroll
        for (int tile = 0; tile < kMaxTilesPerTask; ++tile) {
          if (tile < v.tiles) {
            const int slot = item % S;
            if (!bad && !warp_wait(&full[slot], (uint32_t)((item / S) & 1), kWaitNs)) bad = true;
            if (!bad && mine) {
              const uint8_t* sb = slots + slot * B.slot_bytes;
              const float* sc = reinterpret_cast<const float*>(sb + B.scale_off);
              const uint4 wa = *reinterpret_cast<const uint4*>(sb + lr0 * B.slot_stride + warp * 64 + t * 16);
              const uint4 wb = *reinterpret_cast<const uint4*>(sb + lr1 * B.slot_stride + warp * 64 + t * 16);
              const int sr0 = min(tile * 16 + lr0, v.rows - 1) - tile * 16;
              const int sr1 = min(tile * 16 + lr1, v.rows - 1) - tile * 16;
              float d0, d1;
              chunk_dot_biased(wa, wb, xf, xl, xh, d0, d1);
              acc0[tile] = fmaf(sc[sr0 * tk.G + grp], d0, acc0[tile]);
              acc1[tile] = fmaf(sc[sr1 * tk.G + grp], d1, acc1[tile]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            ++item;
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&xempty[xsl]);  // this warp is done with the task's x
      if (t == 0) {
#pragma unroll
        for (int tile = 0; tile < kMaxTilesPerTask; ++tile) {
          if (tile < v.tiles) {
            red[warp * (kMaxTilesPerTask * 16) + tile * 16 + lr0] = acc0[tile];
            red[warp * (kMaxTilesPerTask * 16) + tile * 16 + lr1] = acc1[tile];
          }
        }
      }
      if (named_sync_or(1, kCThreads, bad || s_abort)) {
        bad = true;
        break;
      }
      for (int r = tid; r < v.rows; r += kCThreads) {
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < kCWarps; ++w) sum += red[w * (kMaxTilesPerTask * 16) + r];
        tk.y[v.row0 + r] = __float2half_rn(sum);
      }
      named_sync(1, kCThreads);  // all y rows of this CTA written; red free again
      if (tid == 0) red_release_add(counters + ti, 1);  // release: cumulative over the barrier
    }
    if (bad && tid == 0) {
      s_abort = 1;
      atomicOr(&g_gemv_batch_error, kErrCopyTimeout);
    }
  }
  __syncthreads();
  if (tid == 0 && !s_abort) {
    __threadfence();
    const int done = atomicAdd(counters + B.num, 1);
    if (done == grid - 1) {  // every CTA is past every dependency wait: reset for the next launch
      for (int i = 0; i <= B.num; ++i) atomicExch(counters + i, 0);
      __threadfence();
    }
  }
}

}  // namespace

int64_t gemv_batch_workspace_bytes(int64_t num_tasks) { return ((num_tasks + 1) * 4 + 255) / 256 * 256; }

bool plan_gemv_batch(GemvBatchParams& B, int sms) {
  int max_k = 0, max_g = 0;
  for (int i = 0; i < B.num; ++i) {
    GemvBatchTask& tk = B.tasks[i];
    tk.rows_per_cta = (tk.N + sms - 1) / sms;
    if (tk.rows_per_cta > kMaxTilesPerTask * 16) return false;
    max_k = tk.K > max_k ? tk.K : max_k;
    max_g = tk.G > max_g ? tk.G : max_g;
  }
  B.grid = sms;
  if (max_k / 128 > kMaxPieces * kPieceChunks) return false;
  B.x_bytes = (max_k * 2 + 127) / 128 * 128;
  B.xsum_bytes = 0;
  B.slot_stride = kPieceChunks * 64 + kSlotPad;
  B.scale_off = 16 * B.slot_stride;
  B.slot_bytes = B.scale_off + ((16 * max_g * 4 + 127) / 128) * 128;
  const int fixed = 2 * B.x_bytes + (2 * kMaxStages + 4) * 8 + kCWarps * kMaxTilesPerTask * 16 * 4 + B.xsum_bytes;
  int stages = (kSmemBudget - fixed) / B.slot_bytes;
  if (stages > kMaxStages) stages = kMaxStages;
  if (stages < 2) return false;
  B.stages = stages;
  B.smem_bytes = fixed + stages * B.slot_bytes;
  return true;
}

cudaError_t launch_gemv_batch(const GemvBatchParams& B, int* counters, cudaStream_t stream) {
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(gemv_batch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(B.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = (size_t)B.smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident: they wait on each other's counters
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv_batch_kernel, B, counters);
}

cudaError_t read_and_clear_gemv_batch_error(int* out) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(out, g_gemv_batch_error, sizeof(int));
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(g_gemv_batch_error, &zero, sizeof(int));
}

}  // namespace soinfer
