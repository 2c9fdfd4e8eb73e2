// Persistent batched INT4 GEMV: one cooperative launch runs a list of GEMVs
// (y_i = dequant(W_i, S_i) x_i), optionally chained (x_i = y_j of an earlier
// task j) -- a decode layer's or a whole token's weight stream in one kernel.
//
// Why: a batch-1 decode GEMV moves a few MB, i.e. tens of KB per SM, while an
// SM needs well over 100 KB of copies in flight to run HBM at full rate; a
// single GEMV launch is latency-bound however it is written.  Weights do not
// depend on activations, so here one producer thread per CTA streams the
// weight slabs of task after task into a shared-memory byte ring and never
// waits for x.
//
// Work split: per task every CTA owns a contiguous, equal slab of output rows
// (rows_per_cta = ceil(N / grid)), so a CTA's weights for a task are one
// contiguous byte range of the packed matrix and its scales another.  The
// slab is cut into items of whole 16-row tiles (as many as fit in
// kMaxItemBytes); each item is exactly two bulk copies (cp.async.bulk, one
// for the packed rows, one for their scale rows) completing on one mbarrier.
// A tile too long for one item (K above ~6K, e.g. a 14B down_proj) is cut
// along K into segments of ks 128-chunks, one item each (one bulk copy per
// row); a warp carries its chain for a tile from segment to segment through
// its partial rows, so the sums do not depend on where the segments fall.
// Scale rows that are not whole 16-byte pieces (tensor-parallel shards with
// 5, 10, 17 or 34 groups per row) are staged with 4-byte cp.async copies that
// arrive on the item's barrier; segment scales go as one bulk copy per row.  Items of any size
// share a circular byte ring, so the bytes in flight stay near the ring size
// whatever the matrix shape.
//
// Roles (one CTA per SM, 19 warps):
//   warps 0..15  consumers in two groups of 8 that take alternate tasks; a
//                group splits K across its warps (chunk c of every tile goes
//                to group warp c mod 8), tensor-core dot products, per-warp
//                partial row sums into a double-buffered reduction area;
//   warp 16      producer: ring allocation + the item copies;
//   warp 17      x loader: waits for the task's dependency (a completion
//                counter in global memory reaching the grid size), then loads
//                x (L2) into a double-buffered x slot;
//   warp 18      epilogue: sums the 8 partials per row, frees the partial
//                buffer, writes y and -- only for a task that a later task
//                depends on -- fences and publishes its completion counter.
//                A peer task (tensor parallelism) stores its rows into every
//                rank's exchange inbox instead (NVLink stores); the last CTA
//                to finish the launch signals the exchange (peer.cuh).
// All lanes of a warp wait on an mbarrier together: a lane-0 poll with the
// rest of the warp parked in __syncwarp delays the hand-offs measurably.
//
// Dot products: each packed word becomes fp16 values biased by a constant
// with one LOP3 per half2 -- (n^8)+1024 for the low nibble of each byte pair,
// 16(n^8)+1024 for the high nibble -- fed to mma.sync.m16n8k16 (exact
// products, fp32 accumulation) in two chains; the bias is removed per 128-K
// chunk with the chunk's x sums: sum q x = (E - 1032 XL) + (O - 1152 XH) / 16.
//
// Every wait is bounded (%globaltimer) and also gives up once another warp of
// the CTA has raised the abort flag; a timeout sets a device error bit, the
// producer waits (bounded) for its copies in flight, and the CTA
// exits.  The completion counters (workspace) are reset to zero by the last
// CTA to finish, so a zeroed workspace stays reusable across launches and
// CUDA-graph replays; after a reported error the caller re-zeroes it.
//
// Launch overlap: a batch without a peer task is launched as a programmatic
// dependent of the kernel before it, so its CTAs start (and the producer
// streams weights, which no earlier kernel writes) while that kernel is still
// finishing; the x loader and the epilogue warp -- the only roles that read
// an earlier kernel's output (x, residual) or write memory another kernel may
// still read (y, norm_out, the workspace counters) -- wait for the earlier
// grid first (griddepcontrol.wait).  The last counter update follows a CTA
// barrier behind both.  A peer batch keeps the cooperative launch: its CTA 0
// reads the exchange epoch at entry.
//
// Reference semantics per task: csrc/kernels/gemv_w4a16_group.cu:77-127 of
// sparse-offload-infer.
#include "common.cuh"
#include "int4_dot.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "peer.cuh"
#include "ring_place.h"

namespace soinfer {

namespace {

__device__ int g_gemv_batch_error;

constexpr int kCWarps = 16;
constexpr int kGroupWarps = 8;                // consumer warps per task (two groups alternate tasks)
constexpr int kProducerWarp = kCWarps;
constexpr int kLoaderWarp = kCWarps + 1;
constexpr int kEpilogueWarp = kCWarps + 2;
constexpr int kThreads = (kCWarps + 3) * 32;
constexpr int kMaxItems = 16;                 // item descriptors (mbarrier pairs) in flight
constexpr int kMaxTiles = 8;                  // 16-row tiles per CTA per task
constexpr int kRedRows = kMaxTiles * 16;
constexpr int kRedBytes = 2 * kGroupWarps * kRedRows * 4;
constexpr int kMaxItemBytes = 52 * 1024;
constexpr int kMaxChunksPerWarp = 24;         // K <= kGroupWarps * kMaxChunksPerWarp * 128 = 24576
constexpr int kSmemLimit = 227 * 1024;
constexpr uint64_t kWaitNs = 1000000000ull;   // 1 s

__host__ __device__ __forceinline__ int round128(int v) { return (v + 127) & ~127; }

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// 16-byte asynchronous global -> shared copy through L2 (x may have been
// written by other SMs during this kernel), and the arrive-on that signals
// an mbarrier once all of this thread's earlier cp.async copies have landed.
__device__ __forceinline__ void cp_async_16(void* dst_smem, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst_smem)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// 4-byte form (scale rows of any length), and the counted arrive-on: the
// barrier's pending count is raised now and lowered when this thread's
// earlier cp.async copies have landed (net zero: the init count is unchanged).
__device__ __forceinline__ void cp_async_4(void* dst_smem, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst_smem)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait for the phase of `bar` with the given parity, giving up early
// once the CTA's abort flag is raised.  Called by every lane of a warp; the
// result is made warp-uniform.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, const volatile int* abort_flag) {
  bool ok = mbar_try_wait(bar, parity);
  if (!ok) {
    const uint64_t t0 = globaltimer_ns();
    while (true) {
      if (mbar_try_wait(bar, parity)) {
        ok = true;
        break;
      }
      if (*abort_flag || globaltimer_ns() - t0 > kWaitNs) break;
    }
  }
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void raise_abort(volatile int* abort_flag) {
  if ((threadIdx.x & 31) == 0) {
    *abort_flag = 1;
    atomicOr(&g_gemv_batch_error, kErrCopyTimeout);
  }
}

struct TaskView {
  int rows, tiles, chunks;
  int64_t row0;
};

// Item k of a task (in issue order): tiles [tile0, tile0 + nt), K-segment seg.
struct ItemView {
  int tile0, nt, seg;
};

__device__ __forceinline__ int task_items(const GemvBatchTask& tk, const TaskView& v) {
  return (v.tiles + tk.tiles_per_item - 1) / tk.tiles_per_item * tk.nsegs;
}

__device__ __forceinline__ TaskView task_view(const GemvBatchTask& tk, int cta) {
  TaskView v;
  v.row0 = (int64_t)cta * tk.rows_per_cta;
  const int rows = tk.N - (int)v.row0;
  v.rows = rows < 0 ? 0 : (rows > tk.rows_per_cta ? tk.rows_per_cta : rows);
  v.tiles = (v.rows + 15) / 16;
  v.chunks = tk.K / 128;
  return v;
}

// Rows of the item covering tiles [tile0, tile0 + nt) of the CTA's slab.
__device__ __forceinline__ int item_rows(const TaskView& v, int tile0, int nt) {
  const int r = v.rows - tile0 * 16;
  return r < nt * 16 ? r : nt * 16;
}

// Per-task state of one consumer warp (everything that depends only on the
// task is computed once; the kernel is issue-bound).
struct ConsumerTask {
  const uint4* xq;        // this lane's 64 x bytes of its first chunk
  const float* sbias;     // chunk_bias of each owned chunk (shared memory)
  float* rr;              // this warp's partial rows
  int row_bytes, G, g, cpg, c_first;
  uint32_t tmask;         // tiles this warp works on
};

// One unit: 16 rows x one 128-K chunk (chunk c_first + i * kGroupWarps);
// w0 / w1 point at rows g / g + 8 of the tile at the first owned chunk.
__device__ __forceinline__ void consume_unit(const uint4 xf[4], const uint8_t* w0, const uint8_t* w1, float sc0,
                                             float sc1, float bias, int i, float& acc0, float& acc1) {
  const uint4 wa = *reinterpret_cast<const uint4*>(w0 + i * (kGroupWarps * 64));
  const uint4 wb = *reinterpret_cast<const uint4*>(w1 + i * (kGroupWarps * 64));
  float d0, d1;
  chunk_dot(wa, wb, xf, d0, d1);
  acc0 = fmaf(sc0, d0 - bias, acc0);
  acc1 = fmaf(sc1, d1 - bias, acc1);
}

// The warp's units of one item: for each owned tile of the item, nm chunks
// (stride kGroupWarps); the tile's partial rows go to the reduction buffer
// (the 4 lanes of a row group hold the same value and all store it).  NM is
// the chunk count when it is 1 or 2 (x fragments and biases stay in
// registers, every offset is an immediate); NM == 0 is the rolled loop over
// nm chunks.  G128: group size 128, one scale column per chunk.
template <int NM, bool G128>
__device__ __forceinline__ void consume_tiles(const ConsumerTask& ct, const uint8_t* wbase, const float* sbase,
                                              int rows, int tile0, int nt, int nm, bool accum) {
  uint4 xr[2][4];
  float br[2] = {0.f, 0.f};
#pragma unroll
  for (int i = 0; i < NM; ++i) {
#pragma unroll
    for (int j = 0; j < 4; ++j) xr[i][j] = ct.xq[i * (kGroupWarps * 16) + j];
    br[i] = ct.sbias[i];
  }
  const int rstep = 16 * ct.row_bytes, sstep = 16 * ct.G;
  const uint8_t* w0 = wbase + ct.g * ct.row_bytes;
  const float* s0p = sbase + ct.g * ct.G + (G128 ? ct.c_first : 0);
  for (int tt = tile0; tt < tile0 + nt; ++tt, w0 += rstep, s0p += sstep) {
    if (!((ct.tmask >> tt) & 1u)) continue;
    const uint8_t* w1 = w0 + 8 * ct.row_bytes;
    const float* s1p = s0p + 8 * ct.G;
    const int last = rows - 1 - (tt - tile0) * 16;  // last valid row of this tile (ragged tile: repeat it)
    const uint8_t* wa = w0;
    const float* sa = s0p;
    if (ct.g > last) wa -= (ct.g - last) * ct.row_bytes, sa -= (ct.g - last) * ct.G;
    if (ct.g + 8 > last) w1 -= (ct.g + 8 - last) * ct.row_bytes, s1p -= (ct.g + 8 - last) * ct.G;
    // a later K-segment continues the warp's chain from its stored partial,
    // so the sums are those of the unsegmented tile (the same fma sequence)
    float acc0 = accum ? ct.rr[tt * 16 + ct.g] : 0.f, acc1 = accum ? ct.rr[tt * 16 + ct.g + 8] : 0.f;
    if (NM > 0) {
#pragma unroll
      for (int i = 0; i < NM; ++i) consume_unit(xr[i], wa, w1, sa[i * kGroupWarps], s1p[i * kGroupWarps], br[i], i, acc0, acc1);
    } else {
      // two chunks per iteration: their dot products are independent and
      // interleave; the accumulation keeps chunk order (same rounding)
      int i = 0;
#pragma unroll 1
      for (; i + 1 < nm; i += 2) {
        uint4 xf0[4], xf1[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          xf0[j] = ct.xq[i * (kGroupWarps * 16) + j];
          xf1[j] = ct.xq[(i + 1) * (kGroupWarps * 16) + j];
        }
        const int sc0 = G128 ? i * kGroupWarps : (ct.c_first + i * kGroupWarps) / ct.cpg;
        const int sc1 = G128 ? (i + 1) * kGroupWarps : (ct.c_first + (i + 1) * kGroupWarps) / ct.cpg;
        const uint4 wa0 = *reinterpret_cast<const uint4*>(wa + i * (kGroupWarps * 64));
        const uint4 wb0 = *reinterpret_cast<const uint4*>(w1 + i * (kGroupWarps * 64));
        const uint4 wa1 = *reinterpret_cast<const uint4*>(wa + (i + 1) * (kGroupWarps * 64));
        const uint4 wb1 = *reinterpret_cast<const uint4*>(w1 + (i + 1) * (kGroupWarps * 64));
        float d00, d01, d10, d11;
        chunk_dot(wa0, wb0, xf0, d00, d01);
        chunk_dot(wa1, wb1, xf1, d10, d11);
        acc0 = fmaf(sa[sc0], d00 - ct.sbias[i], acc0);
        acc1 = fmaf(s1p[sc0], d01 - ct.sbias[i], acc1);
        acc0 = fmaf(sa[sc1], d10 - ct.sbias[i + 1], acc0);
        acc1 = fmaf(s1p[sc1], d11 - ct.sbias[i + 1], acc1);
      }
      if (i < nm) {
        uint4 xf[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) xf[j] = ct.xq[i * (kGroupWarps * 16) + j];
        const int sc = G128 ? i * kGroupWarps : (ct.c_first + i * kGroupWarps) / ct.cpg;
        consume_unit(xf, wa, w1, sa[sc], s1p[sc], ct.sbias[i], i, acc0, acc1);
      }
    }
    ct.rr[tt * 16 + ct.g] = acc0;
    ct.rr[tt * 16 + ct.g + 8] = acc1;
  }
}

// The producer warp's loop.
template <class Params>
__device__ __forceinline__ void producer_loop(const Params& B, int cta, int lane, uint8_t* ring,
                                           uint64_t* full, uint64_t* empty, int* item_off,
                                           volatile int* abort_flag) {
  // ------------------------------------------------------------ producer
  // Ring allocation is FIFO: the producer frees items in issue order (it
  // waits on each one's empty barrier, whichever consumer group takes it), so
  // the occupied bytes are [item_off[oldest], head) circularly.
  int head = 0, issued = 0, oldest = 0;
  bool stop = false;
  for (int ti = 0; ti < B.num && !stop; ++ti) {
    const GemvBatchTask& tk = B.tasks[ti];
    const TaskView v = task_view(tk, cta);
    const int row_bytes = tk.K / 2;
    const bool segd = tk.nsegs > 1;
    const int wrow = segd ? tk.ks * 64 : row_bytes;     // weight row stride in the item
    const int srow_f = segd ? tk.ks / tk.cpg : tk.G;    // scale row stride in the item (floats)
    const int nitems = task_items(tk, v);
    int tile0 = 0, seg = 0;  // item (tile0, seg): segments of a tile are consecutive
    for (int it = 0; it < nitems && !stop; ++it, seg = (seg + 1 == tk.nsegs) ? (tile0 += tk.tiles_per_item, 0) : seg + 1) {
      const int nt = min(tk.tiles_per_item, v.tiles - tile0);
      const int rows = item_rows(v, tile0, nt);
      const int nks = segd ? min(tk.ks, v.chunks - seg * tk.ks) : v.chunks;
      const int wb = rows * wrow, sb = rows * srow_f * 4;
      const int bytes = round128(wb) + round128(sb);
      // place the item (ring_place.h); otherwise wait for the oldest item
      while (true) {
        const int live = issued - oldest;
        const int at = ring_place(head, live > 0 ? item_off[oldest % kMaxItems] : 0, live, bytes, B.ring_bytes,
                                  kMaxItems);
        if (at >= 0) {
          head = at;
          break;
        }
        if (!warp_wait(&empty[oldest % kMaxItems], (uint32_t)((oldest / kMaxItems) & 1), abort_flag)) {
          stop = true;
          break;
        }
        ++oldest;
      }
      if (stop) break;
      const int d = issued % kMaxItems;
      __syncwarp();  // every lane has read item_off[] before lane 0 rewrites a slot
      const int64_t r0 = v.row0 + tile0 * 16;
      if (!segd && !tk.scale_plain) {
        // whole 16-row tiles with 16-byte scale rows: one bulk copy each for rows and scales
        if (lane == 0) {
          item_off[d] = head;
          mbar_arrive_expect_tx(&full[d], (uint32_t)(wb + sb));
          bulk_g2s(ring + head, tk.W + r0 * row_bytes, (uint32_t)wb, &full[d]);
          bulk_g2s(ring + head + round128(wb), tk.S + r0 * tk.G, (uint32_t)sb, &full[d]);
        }
      } else {
        if (lane == 0) item_off[d] = head;
        if (B.any_cp_async) fence_proxy_async_smem();  // earlier cp.async writes into the ring precede bulk writes
        float* sdst = reinterpret_cast<float*>(ring + head + round128(wb));
        const int gs = segd ? nks / tk.cpg : tk.G;  // scale columns of the item's rows
        // segment scales as one bulk copy per row when every piece is whole 16 bytes
        const bool seg_bulk = segd && (tk.G % 4) == 0 && (srow_f % 4) == 0 && (gs % 4) == 0;
        if (!seg_bulk) {
          // scale rows not in 16-byte pieces: 4-byte cp.async copies; each
          // lane's arrive-on (counted before lane 0's arrive below) completes
          // when its copies have landed, so the producer never waits on them
          const float* src = tk.S + r0 * tk.G + (segd ? seg * srow_f : 0);
          for (int i = lane; i < rows * gs; i += 32) {
            const int rr = i / gs, c = i - rr * gs;
            cp_async_4(sdst + rr * srow_f + c, src + (int64_t)rr * tk.G + c);
          }
          cp_async_arrive(&full[d]);
          __syncwarp();
        }
        if (!segd) {
          if (lane == 0) {
            mbar_arrive_expect_tx(&full[d], (uint32_t)wb);
            bulk_g2s(ring + head, tk.W + r0 * row_bytes, (uint32_t)wb, &full[d]);
          }
        } else {
          if (lane == 0) mbar_arrive_expect_tx(&full[d], (uint32_t)(rows * (nks * 64 + (seg_bulk ? gs * 4 : 0))));
          if (lane < rows)
            bulk_g2s(ring + head + lane * wrow, tk.W + (r0 + lane) * row_bytes + (int64_t)seg * tk.ks * 64,
                     (uint32_t)(nks * 64), &full[d]);
          if (seg_bulk && lane >= 16 && lane - 16 < rows)
            bulk_g2s(sdst + (lane - 16) * srow_f, tk.S + (r0 + lane - 16) * tk.G + seg * srow_f, (uint32_t)(gs * 4),
                     &full[d]);
        }
      }
      __syncwarp();
      head += bytes;
      ++issued;
    }
  }
  if (stop) raise_abort(abort_flag);
  // every issued copy must land before this CTA's shared memory is released
  for (int q = max(oldest, issued - kMaxItems); q < issued; ++q)
    (void)mbar_wait_bounded(&full[q % kMaxItems], (uint32_t)((q / kMaxItems) & 1), kWaitNs / 4);
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// The epilogue warp's loop.
template <class Params>
__device__ __forceinline__ void epilogue_loop(const Params& B, int cta, int lane, const float* red,
                                           uint64_t* rfull, uint64_t* rempty, uint8_t* const* s_inbox,
                                           int* counters, volatile int* abort_flag) {
  // ------------------------------------------------------------ epilogue
  int a = 0;
  bool stop = false;
  for (int ti = 0; ti < B.num && !stop; ++ti) {
    const GemvBatchTask& tk = B.tasks[ti];
    const TaskView v = task_view(tk, cta);
    if (v.rows > 0) {
      const int rb = a & 1;
      if (!warp_wait(&rfull[rb], (uint32_t)((a >> 1) & 1), abort_flag)) {
        stop = true;
        break;
      }
      const float* rr = red + rb * (kGroupWarps * kRedRows);
      // warps holding partials of a row: the whole group, or -- with fewer chunks
      // than group warps -- the `chunks` warps that own the row's tile
      const int nsplit = v.chunks >= kGroupWarps ? 1 : kGroupWarps / v.chunks;
      const int nw = v.chunks >= kGroupWarps ? kGroupWarps : v.chunks;
      float sums[kRedRows / 32];
#pragma unroll
      for (int i = 0; i < kRedRows / 32; ++i) {
        const int r = lane + 32 * i;
        sums[i] = 0.f;
        if (r < v.rows) {
          const int w0 = ((r >> 4) % nsplit) * nw;
          for (int w = w0; w < w0 + nw; ++w) sums[i] += rr[w * kRedRows + r];
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&rempty[rb]);  // partials consumed: the consumers may refill the buffer
#pragma unroll
      for (int i = 0; i < kRedRows / 32; ++i) {
        const int r = lane + 32 * i;
        if (r < v.rows) {
          // optional epilogues; a glu / resid row written by an earlier task of
          // this batch was stored by this same lane (same N, same row split)
          half hv = __float2half_rn(sums[i]);
          if (tk.glu) {
            const float gv = __half2float(__ldcg(tk.glu + v.row0 + r));
            hv = __float2half_rn((gv / (1.0f + expf(-gv))) * __half2float(hv));
          }
          if (tk.resid) hv = __float2half_rn(__half2float(__ldcg(tk.resid + v.row0 + r)) + __half2float(hv));
          if (tk.peer) {
            for (int pr = 0; pr < B.peers.world; ++pr) reinterpret_cast<half*>(s_inbox[pr])[v.row0 + r] = hv;
          } else {
            tk.y[v.row0 + r] = hv;
          }
        }
      }
      ++a;
    }
    if (tk.peer) {  // rows pushed: system-visible before this CTA counts itself done (kernel end)
      __threadfence_system();
    } else if (tk.publish) {  // a later task reads this y: make it visible GPU-wide, then count this CTA in
      __threadfence();
      __syncwarp();
      if (lane == 0) red_release_add(counters + ti, 1);
    }
    __syncwarp();
  }
  if (stop) raise_abort(abort_flag);
}

// 19 warps put 5 warps on some of the SM's four 16K-register partitions:
// at most 96 registers per thread.
template <class Params>
__global__ void __launch_bounds__(kThreads, 1)
    gemv_batch_kernel(const __grid_constant__ Params B, int* __restrict__ counters) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;                                                  // [ring_bytes]
  uint8_t* xbuf = smem + B.ring_bytes;                                   // [2][x_bytes]
  float* red = reinterpret_cast<float*>(xbuf + 2 * B.x_bytes);          // [2][kGroupWarps][kRedRows]
  uint8_t* nscr = reinterpret_cast<uint8_t*>(red) + kRedBytes;          // [norm_bytes] norm weights
  __shared__ uint64_t full[kMaxItems], empty[kMaxItems];
  __shared__ uint64_t xfull[2], xempty[2], rfull[2], rempty[2];
  __shared__ int item_off[kMaxItems];
  __shared__ float s_bias[kCWarps][kMaxChunksPerWarp];  // 1.5 KB
  __shared__ int s_abort;
  __shared__ uint8_t* s_inbox[kMaxPeers];  // peer task: rank r's inbox slot (parity, this rank)
  __shared__ uint32_t* s_flag[kMaxPeers];  // and its flag for this rank
  __shared__ uint32_t s_epoch;             // the exchange this launch signals
  volatile int* abort_flag = &s_abort;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int cta = blockIdx.x;
  const int grid = gridDim.x;
  if (tid == 0) {
    for (int s = 0; s < kMaxItems; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kGroupWarps);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&xfull[s], 32);  // one cp.async arrive-on per loader lane
      mbar_init(&xempty[s], kGroupWarps);
      mbar_init(&rfull[s], kGroupWarps);
      mbar_init(&rempty[s], 1);
    }
    fence_mbar_init();
    s_abort = 0;
    if (B.peers.world > 0) {
      const uint32_t e = peer_next_epoch(B.peers);
      const int par = (int)(e & 1u);
      s_epoch = e;
#pragma unroll
      for (int r = 0; r < kMaxPeers; ++r) {
        s_inbox[r] = B.peers.base[r] + kPeerHeaderBytes + ((int64_t)par * B.peers.world + B.peers.rank) * B.peers.slot_bytes;
        s_flag[r] = reinterpret_cast<uint32_t*>(B.peers.base[r]) + par * kMaxPeers + B.peers.rank;
      }
    }
  }
  __syncthreads();
  // let the next kernel (launched as a programmatic dependent; it waits for
  // this grid's completion before touching memory) be scheduled early
  pdl_launch_dependents();

  if (warp == kProducerWarp) {
    producer_loop(B, cta, lane, ring, full, empty, item_off, abort_flag);
  } else if (warp == kLoaderWarp) {
    pdl_wait();  // x (and the dependency counters) come from earlier kernels
    // ------------------------------------------------------------ x loader
    int a = 0;  // index among this CTA's active (rows > 0) tasks
    bool stop = false;
    for (int ti = 0; ti < B.num && !stop; ++ti) {
      const GemvBatchTask& tk = B.tasks[ti];
      if (task_view(tk, cta).rows == 0) continue;
      const int xs = a & 1;
      if (a >= 2 && !warp_wait(&xempty[xs], (uint32_t)(((a >> 1) - 1) & 1), abort_flag)) {
        stop = true;
        break;
      }
      if (tk.dep >= 0) {
        // every lane polls the same word (one request); the exit is uniform
        const uint64_t t0 = globaltimer_ns();
        while (true) {
          const bool done = ld_acquire(counters + tk.dep) >= grid;
          if (__all_sync(0xffffffffu, done)) break;
          const bool give_up = *abort_flag || globaltimer_ns() - t0 > kWaitNs;
          if (__any_sync(0xffffffffu, give_up)) {
            stop = true;
            break;
          }
        }
        if (stop) break;
      }
      // x through cp.async (all 16-byte pieces in flight at once), not a bulk
      // copy: a bulk copy would queue behind the producer's weight copies in
      // this SM's copy engine.  Each lane's arrive-on fires when its copies land.
      const uint4* src = reinterpret_cast<const uint4*>(tk.x);
      uint4* dst = reinterpret_cast<uint4*>(xbuf + xs * B.x_bytes);
      const int n16 = tk.K / 8;
      if (tk.norm_w == nullptr) {
        for (int u = lane; u < n16; u += 32) cp_async_16(dst + u, src + u);
        cp_async_arrive_noinc(&xfull[xs]);
      } else {
        // RMSNorm prologue: x and the norm weights land, then the warp
        // normalises x in place -- f * inv * w in fp32, rounded to fp16, as
        // the rmsnorm kernel does -- and arrives (32 arrivals, like the copies)
        uint4* wsc = reinterpret_cast<uint4*>(nscr);
        const uint4* wsrc = reinterpret_cast<const uint4*>(tk.norm_w);
        for (int u = lane; u < n16; u += 32) {
          cp_async_16(dst + u, src + u);
          cp_async_16(wsc + u, wsrc + u);
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncwarp();
        warp_rmsnorm_inplace(dst, wsc, n16, tk.K, tk.eps, lane,
                             tk.norm_out != nullptr && blockIdx.x == 0 ? reinterpret_cast<uint4*>(tk.norm_out)
                                                                       : nullptr);
        __syncwarp();
        mbar_arrive(&xfull[xs]);
      }
      ++a;
    }
    if (stop) raise_abort(abort_flag);
    asm volatile("cp.async.wait_all;" ::: "memory");  // no copy into this CTA's shared memory outlives it
  } else if (warp == kEpilogueWarp) {
    pdl_wait();  // residual inputs from earlier kernels; y may alias a buffer they read
    epilogue_loop(B, cta, lane, red, rfull, rempty, s_inbox, counters, abort_flag);
  } else {
    // ------------------------------------------------------------ consumers
    // Two groups of kGroupWarps warps alternate over this CTA's active tasks
    // (group = active index & 1, matching the x and partial double buffers),
    // so each warp works on every other task with twice the chunks: the
    // per-task overhead is paid by half the warps.
    const int group = warp / kGroupWarps, gw = warp % kGroupWarps;
    const int g = lane >> 2, t = lane & 3;
    int item = 0, a = 0;
    bool stop = false;
    for (int ti = 0; ti < B.num && !stop; ++ti) {
      const GemvBatchTask& tk = B.tasks[ti];
      const TaskView v = task_view(tk, cta);
      if (v.rows == 0) continue;
      const int tpi = tk.tiles_per_item;
      const int nitems = task_items(tk, v);
      if ((a & 1) != group) {  // the other group's task
        item += nitems;
        ++a;
        continue;
      }
      const int row_bytes = tk.K / 2;
      int c_first, nmine;
      uint32_t tmask = 0xffu;
      if (v.chunks >= kGroupWarps) {
        c_first = gw, nmine = (v.chunks - gw + kGroupWarps - 1) / kGroupWarps;
      } else {  // fewer chunks than group warps: warps also split the tiles
        const int nsplit = kGroupWarps / v.chunks, tsel = gw / v.chunks;
        c_first = gw % v.chunks, nmine = tsel < nsplit ? 1 : 0;
        tmask = 0;
        for (int tt = tsel; tt < kMaxTiles; tt += nsplit) tmask |= 1u << tt;
      }
      const int xs = a & 1, rb = a & 1;
      if (!warp_wait(&xfull[xs], (uint32_t)((a >> 1) & 1), abort_flag)) {
        stop = true;
        break;
      }
      ConsumerTask ct;
      ct.xq = reinterpret_cast<const uint4*>(xbuf + xs * B.x_bytes) + c_first * 16 + t * 4;
      ct.sbias = s_bias[warp];
      ct.rr = red + rb * (kGroupWarps * kRedRows) + gw * kRedRows;
      ct.row_bytes = row_bytes;
      ct.G = tk.G;
      ct.g = g;
      ct.cpg = tk.cpg;
      ct.c_first = c_first;
      ct.tmask = tmask;
      for (int i = 0; i < nmine; ++i) {
        const float bias = chunk_bias(xbuf + xs * B.x_bytes + (c_first + i * kGroupWarps) * 256, g, t);
        if (lane == 0) s_bias[warp][i] = bias;
      }
      __syncwarp();
      if (a >= 2 && !warp_wait(&rempty[rb], (uint32_t)(((a >> 1) - 1) & 1), abort_flag)) {
        stop = true;
        break;
      }
      // 1, 2: unrolled (group size 128); 3: rolled, group size 128; 4: rolled, general; 0: idle
      const int kind = nmine == 0 ? 0 : (tk.cpg == 1 ? (nmine <= 2 ? nmine : 3) : 4);
      if (tk.nsegs == 1) {
        for (int tile0 = 0; tile0 < v.tiles; tile0 += tpi) {
          const int nt = min(tpi, v.tiles - tile0);
          const int rows = item_rows(v, tile0, nt);
          const int d = item % kMaxItems;
          if (!warp_wait(&full[d], (uint32_t)((item / kMaxItems) & 1), abort_flag)) {
            stop = true;
            break;
          }
          const uint8_t* ib = ring + item_off[d];
          const uint8_t* wbase = ib + c_first * 64 + t * 16;
          const float* sbase = reinterpret_cast<const float*>(ib + round128(rows * row_bytes));
          if (kind == 1) consume_tiles<1, true>(ct, wbase, sbase, rows, tile0, nt, 1, false);
          else if (kind == 2) consume_tiles<2, true>(ct, wbase, sbase, rows, tile0, nt, 2, false);
          else if (kind == 3) consume_tiles<0, true>(ct, wbase, sbase, rows, tile0, nt, nmine, false);
          else if (kind == 4) consume_tiles<0, false>(ct, wbase, sbase, rows, tile0, nt, nmine, false);
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[d]);
          ++item;
        }
      } else {
        // K-segmented task: items are (tile, segment), segments of a tile consecutive; item rows
        // hold one segment, scale columns are segment-local (the item holds the segment's groups)
        ct.row_bytes = tk.ks * 64;
        ct.G = tk.ks / tk.cpg;
        for (int tile0 = 0; tile0 < v.tiles && !stop; ++tile0) {
          const int rows = item_rows(v, tile0, 1);
          for (int seg = 0; seg < tk.nsegs; ++seg) {
            const int d = item % kMaxItems;
            if (!warp_wait(&full[d], (uint32_t)((item / kMaxItems) & 1), abort_flag)) {
              stop = true;
              break;
            }
            const uint8_t* ib = ring + item_off[d];
            const uint8_t* wbase = ib + c_first * 64 + t * 16;
            const float* sbase = reinterpret_cast<const float*>(ib + round128(rows * ct.row_bytes));
            // owned chunks gw + 8j of the segment (ks is a multiple of 8), their x and biases
            const int nks = min(tk.ks, v.chunks - seg * tk.ks);
            const int nm = nks > gw ? (nks - gw + kGroupWarps - 1) / kGroupWarps : 0;
            ct.xq = reinterpret_cast<const uint4*>(xbuf + xs * B.x_bytes) + (c_first + seg * tk.ks) * 16 + t * 4;
            ct.sbias = s_bias[warp] + seg * (tk.ks / kGroupWarps);
            if (nm > 0) {
              if (tk.cpg == 1) consume_tiles<0, true>(ct, wbase, sbase, rows, tile0, 1, nm, seg > 0);
              else consume_tiles<0, false>(ct, wbase, sbase, rows, tile0, 1, nm, seg > 0);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[d]);
            ++item;
          }
        }
      }
      if (stop) break;
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&xempty[xs]);  // this warp is done with the task's x
        mbar_arrive(&rfull[rb]);   // and has written its partials
      }
      ++a;
    }
    if (stop) raise_abort(abort_flag);
  }
  __syncthreads();
  if (B.need_counters && tid == 0 && !s_abort) {
    __threadfence();
    const int done = atomicAdd(counters + B.num, 1);
    if (done == grid - 1) {  // every CTA is past every dependency wait: reset for the next launch
      for (int i = 0; i <= B.num; ++i) atomicExch(counters + i, 0);
      __threadfence();
      if (B.peers.world > 0) {  // every CTA pushed its rows of the peer task: signal every rank
        __threadfence_system();
        for (int pr = 0; pr < B.peers.world; ++pr) st_release_sys_u32(s_flag[pr], s_epoch);
      }
    }
  }
}

}  // namespace

// Also large enough for the streaming kernel's counters (gemv_stream_workspace_bytes),
// which the same batch entry point may choose.
int64_t gemv_batch_workspace_bytes(int64_t num_tasks) { return ((num_tasks + 2) * 4 + 255) / 256 * 256; }

bool plan_gemv_batch(GemvBatchParams& B, int sms) {
  int max_k = 0;
  for (int i = 0; i < B.num; ++i) B.tasks[i].publish = 0;
  for (int i = 0; i < B.num; ++i)
    if (B.tasks[i].dep >= 0) B.tasks[B.tasks[i].dep].publish = 1;
  int npeer = 0;
  B.any_cp_async = 0;
  int norm_k = 0;
  for (int i = 0; i < B.num; ++i) {
    GemvBatchTask& tk = B.tasks[i];
    tk.rows_per_cta = (tk.N + sms - 1) / sms;
    if (tk.rows_per_cta > kMaxTiles * 16) return false;
    if (tk.K % 128 != 0 || tk.K / 128 > kGroupWarps * kMaxChunksPerWarp) return false;
    const int chunks = tk.K / 128;
    tk.scale_plain = (tk.G * 4) % 16 != 0 ? 1 : 0;
    const int tile_bytes = round128(16 * (tk.K / 2)) + round128(16 * tk.G * 4);
    if (tile_bytes <= kMaxItemBytes) {
      tk.nsegs = 1;
      tk.ks = chunks;
      tk.tiles_per_item = kMaxItemBytes / tile_bytes;
    } else {
      // K-segments of ks chunks: whole scale groups, a multiple of the group's warps
      if (chunks % tk.cpg != 0 || tk.G != chunks / tk.cpg) return false;
      const int step = kGroupWarps * tk.cpg;
      int ks = 0;
      for (int c = step; c <= chunks; c += step)
        if (round128(16 * c * 64) + round128(16 * (c / tk.cpg) * 4) <= kMaxItemBytes) ks = c;
      if (ks == 0) return false;
      tk.ks = ks;
      tk.nsegs = (chunks + ks - 1) / ks;
      tk.tiles_per_item = 1;
      tk.scale_plain = 1;
    }
    if (tk.peer) ++npeer;
    if (tk.norm_w != nullptr) norm_k = tk.K > norm_k ? tk.K : norm_k;
    if (tk.scale_plain && !(tk.nsegs > 1 && tk.G % 4 == 0 && (tk.ks / tk.cpg) % 4 == 0 &&
                            ((chunks - (tk.nsegs - 1) * tk.ks) / tk.cpg) % 4 == 0))
      B.any_cp_async = 1;  // the producer's seg_bulk test fails for some item of this task
    max_k = tk.K > max_k ? tk.K : max_k;
  }
  if (npeer > 1 || (npeer == 1 && B.peers.world < 1)) return false;
  // A task whose glu / resid rows are an earlier task's y reads each row in
  // the epilogue lane that wrote it, which needs the same base and row split;
  // anything else goes to the ordered per-task fallback.
  for (int i = 0; i < B.num; ++i) {
    const GemvBatchTask& tk = B.tasks[i];
    for (int j = 0; j < i; ++j) {
      const GemvBatchTask& p = B.tasks[j];
      if (p.y == nullptr) continue;
      const half* lo = p.y;
      const half* hi = p.y + p.N;
      for (const half* e : {tk.glu, tk.resid})
        if (e != nullptr && e < hi && e + tk.N > lo && (e != p.y || p.N != tk.N)) return false;
    }
  }
  B.need_counters = npeer > 0 ? 1 : 0;
  for (int i = 0; i < B.num; ++i) B.need_counters |= B.tasks[i].publish;
  B.grid = sms;
  B.x_bytes = round128(max_k * 2);
  const int static_smem = 3072;  // mbarriers, item offsets, per-warp biases, flags (~2 KB used)
  B.norm_bytes = norm_k > 0 ? round128(norm_k * 2) : 0;
  B.ring_bytes = ((kSmemLimit - static_smem - 2 * B.x_bytes - kRedBytes - B.norm_bytes - 256) / 128) * 128;
  if (B.ring_bytes < kMaxItemBytes + 128) return false;
  B.smem_bytes = B.ring_bytes + 2 * B.x_bytes + kRedBytes + B.norm_bytes;
  return true;
}

namespace {

template <class Params>
cudaError_t launch_params(const Params& B, int* counters, cudaStream_t stream) {
  auto kernel = gemv_batch_kernel<Params>;
  if (cudaError_t e = ensure_smem_attr<gemv_batch_kernel<Params>>(B.smem_bytes); e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(B.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = (size_t)B.smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  if (B.peers.world > 0) {
    at[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident: they wait on each other's counters
    at[0].val.cooperative = 1;
  } else {
    // one CTA per SM and grid = SM count: every CTA becomes resident once the
    // earlier kernel drains, before any dependency wait (those follow the
    // grid wait), so the CTAs still meet; start them early to overlap it
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
  }
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, B, counters);
}

}  // namespace

cudaError_t launch_gemv_batch(const GemvBatchParams& B, int* counters, cudaStream_t stream) {
  if (B.num <= kSmallBatchTasks) {
    // a decode layer's batch: the same kernel with a ~1 KB parameter block
    static GemvBatchParamsT<kSmallBatchTasks> S;  // callers serialise launches
    S.num = B.num;
    S.grid = B.grid;
    S.x_bytes = B.x_bytes;
    S.ring_bytes = B.ring_bytes;
    S.smem_bytes = B.smem_bytes;
    S.any_cp_async = B.any_cp_async;
    S.norm_bytes = B.norm_bytes;
    S.need_counters = B.need_counters;
    S.peers = B.peers;
    for (int i = 0; i < B.num; ++i) S.tasks[i] = B.tasks[i];
    return launch_params(S, counters, stream);
  }
  return launch_params(B, counters, stream);
}

cudaError_t read_and_clear_gemv_batch_error(int* out) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(out, g_gemv_batch_error, sizeof(int));
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(g_gemv_batch_error, &zero, sizeof(int));
}

}  // namespace soinfer
