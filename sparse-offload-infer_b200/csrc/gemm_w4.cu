// Multi-token INT4 GEMM for batched decode: Y[m, n] = sum_k W[n, k] X[m, k]
// for M <= 8 token rows (group-wise INT4 weights, AWQ order, fp32 scales,
// fp16 activations, fp32 accumulation) -- the reference's per-token GEMV
// (csrc/kernels/gemv_w4a16_group.cu:77-127) applied to M tokens, sharing one
// pass over the weights.
//
// Why tensor cores pay here: at batch 1 the mma.sync.m16n8k16 B operand
// carries one x replicated over its 8 columns; with M tokens column m holds
// token m, so the same MMAs (same count, same weight unpack) produce M
// outputs per weight row.  The weight stream -- the HBM roofline -- is
// unchanged, the useful work grows M-fold.
//
// Structure (one CTA per SM, 512 threads): the CTA owns a contiguous slab of
// output rows; warp 0 streams 16-row x 24-chunk pieces of it into a ring of
// shared-memory stages with cp.async.bulk (one copy per row piece, mbarrier
// per stage, bounded waits); X [M, K] and the slab's scale rows are staged
// once in shared memory (long K, where X [M, K] does not fit: the pieces run
// K-segment by K-segment over the slab's tiles, X is staged one segment at a
// time and each warp keeps its per-tile partial rows in shared memory between
// segments -- the same per-warp accumulation order, so the same bits); the
// 16 warps split each piece's 128-K chunks, unpack
// each packed word to biased exact fp16 values (one LOP3 per pair, the bias
// removed per chunk and token with a precomputed table) and run two MMA chains; at each tile's end the per-warp partials [16 rows x 8
// tokens] are summed in warp order (deterministic) and written.
#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"

namespace soinfer {
namespace {

__device__ int g_gemm_w4_error;

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kStages = 4;        // stage barriers held (the plan uses up to this many)
constexpr int kPieceChunks = 48;   // most 128-K chunks per piece
constexpr int kSlotPad = 64;
constexpr int kTokens = 8;
constexpr uint64_t kWaitNs = 2000000000ull;

struct GemmPlan {
  int rows_per_cta, chunks, piece_chunks, pieces, stages, cpg, G, slot_stride;
  int m;    // tokens
  int seg;  // 1: K-segment-major order, X staged one piece's chunks at a time
  int cpg_shift;  // log2(cpg): chunks per scale group are a power of two
  int smem_x, smem_scale, smem_stage, smem_red, smem_bias, smem_total;
};

// x in shared memory: token m's K values at uint4 offset m * K/8, each
// 64-byte segment's four uint4 swizzled so a chunk's four lane-groups read
// distinct banks (same layout as the single-token GEMV).
__device__ __forceinline__ int x_slot(int q) {
  const int t = (q >> 2) & 3;
  return (q & ~3) | ((q & 3) ^ ((t >> 1) & 1));
}

// One 128-K chunk of two rows (g, g + 8) against the thread's token columns
// (2t, 2t + 1): d[0..1] row g, d[2..3] row g + 8, biased -- each packed word
// becomes exact fp16 values 1024 + (n ^ 8) (nibble positions v0 v1 v4 v5) and
// 1024 + 16 (n ^ 8) (v2 v3 v6 v7) with one LOP3 per half2, in two MMA chains
// (one per position class); d = E + O / 16 is the dot product plus the
// chunk's per-token bias 1032 XL + 72 XH (chunk_bias8), which the caller
// subtracts.
__device__ __forceinline__ void chunk_mma(const uint4 wa, const uint4 wb, const uint4 xf[4], float d[4]) {
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
#pragma unroll
  for (int c = 0; c < 4; ++c) d[c] = fmaf(o[c], 0.0625f, e[c]);
}

// The chunk's bias for the thread's token columns 2t, 2t + 1: with A uniform
// (1032 in the v0 v1 v4 v5 positions' k, 72 in the others'), column n of D
// sums token n's x weighted by position class over the 128 values.
__device__ __forceinline__ void chunk_bias8(const uint4 xf[4], float b[2]) {
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

__global__ void __launch_bounds__(kThreads, 1)
    gemm_w4_kernel(const uint8_t* __restrict__ W, const float* __restrict__ S, const half* __restrict__ X,
                   const int64_t ldx, half* __restrict__ Y, const int64_t ldy, const int nrows, const int K,
                   const GemmPlan p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint4* xs = reinterpret_cast<uint4*>(smem);
  float* ss = reinterpret_cast<float*>(smem + p.smem_x);
  uint8_t* stage_base = smem + p.smem_x + p.smem_scale;
  float* red = reinterpret_cast<float*>(stage_base + p.smem_stage);  // [kWarps][16][kTokens]
  float* cbias = reinterpret_cast<float*>(stage_base + p.smem_stage + p.smem_red);  // [staged chunks][kTokens]
  __shared__ uint64_t bars[kStages + 1];  // stage full (tx), then the scale rows
  __shared__ uint64_t empty[kStages];     // stage released by every warp
  __shared__ int s_abort_v;
  uint64_t* scale_bar = bars + kStages;
  int* s_abort = &s_abort_v;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int64_t row_begin = (int64_t)blockIdx.x * p.rows_per_cta;
  int rows_here = nrows - (int)row_begin;
  rows_here = rows_here < 0 ? 0 : (rows_here > p.rows_per_cta ? p.rows_per_cta : rows_here);
  const int n_tiles = (rows_here + 15) / 16;
  const int total = n_tiles * p.pieces;
  const int slot_bytes = 16 * p.slot_stride;
  const int64_t row_bytes = K / 2;

  if (tid == 0) {
    for (int s = 0; s <= kStages; ++s) mbar_init(&bars[s], 1);
    for (int s = 0; s < kStages; ++s) mbar_init(&empty[s], kWarps);
    s_abort_v = 0;
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  // stage s -> (tile, piece): tile-major, or K-segment-major for long K
  auto coords = [&](int s, int& tile, int& piece) {
    if (p.seg) {
      piece = s / n_tiles;
      tile = s - piece * n_tiles;
    } else {
      tile = s / p.pieces;
      piece = s - tile * p.pieces;
    }
  };
  auto issue = [&](int s) {  // warp 0: lane r < 16 copies row r of stage s's piece
    const int slot = s % p.stages;
    int tile, piece;
    coords(s, tile, piece);
    const int c0 = piece * p.piece_chunks;
    const int pc = min(p.piece_chunks, p.chunks - c0);
    const int valid = min(16, rows_here - tile * 16);
    if (lane == 0) mbar_arrive_expect_tx(&bars[slot], (uint32_t)(valid * pc * 64));
    if (lane < valid)
      bulk_g2s(stage_base + slot * slot_bytes + lane * p.slot_stride,
               W + (row_begin + tile * 16 + lane) * row_bytes + (int64_t)c0 * 64, (uint32_t)(pc * 64), &bars[slot]);
  };
  if (warp == 0 && total > 0) {
    if (lane == 0) {
      const uint32_t bytes = (uint32_t)rows_here * (uint32_t)p.G * 4u;
      mbar_arrive_expect_tx(scale_bar, bytes);
      bulk_g2s(ss, S + row_begin * p.G, bytes, scale_bar);
    }
    const int first = total < p.stages ? total : p.stages;
    for (int s = 0; s < first; ++s) issue(s);
  }
  pdl_wait();  // X may come from the previous kernel
  // X chunks [c0, c0 + nc) of every token into shared memory (token stride xk16 uint4)
  const int xk16 = p.seg ? p.piece_chunks * 16 : K / 8;
  auto load_x = [&](int c0, int nc) {
    const int k16 = nc * 16;
    for (int i = tid; i < p.m * k16; i += kThreads) {
      const int m = i / k16, q = i - m * k16;
      xs[m * xk16 + x_slot(q)] = __ldcg(reinterpret_cast<const uint4*>(X + m * ldx) + c0 * 16 + q);
    }
  };
  // every staged chunk's per-token bias (warp w: chunks w, w + 16, ...)
  auto chunk_biases = [&](int nc) {
    for (int c = warp; c < nc; c += kWarps) {
      uint4 xf[4];
      const uint4* xc = xs + (g < p.m ? g : 0) * xk16 + c * 16 + t * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j) xf[j] = xc[j ^ ((t >> 1) & 1)];
      float b[2];
      chunk_bias8(xf, b);
      if (g == 0) {
        cbias[c * kTokens + 2 * t] = b[0];
        cbias[c * kTokens + 2 * t + 1] = b[1];
      }
    }
  };
  if (!p.seg) load_x(0, p.chunks);
  if (total == 0) return;
  __syncthreads();  // X staged for every warp
  if (!p.seg) {
    chunk_biases(p.chunks);
    __syncthreads();
  }
  // A failed (timed-out) wait sets s_abort; every warp then skips its work but
  // still takes the same CTA barriers, so nothing is left waiting, and the
  // issuing warp waits (bounded) for the copies it started before leaving.
  auto wait_bar = [&](uint64_t* bar, uint32_t parity) -> bool {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity)) {
      if (*s_abort != 0 || globaltimer_ns() - t0 > kWaitNs) return false;
    }
    return true;
  };
  auto fail = [&]() {
    if (lane == 0) {
      atomicOr(&g_gemm_w4_error, kErrCopyTimeout);
      *s_abort = 1;
    }
  };
  bool ab = !wait_bar(scale_bar, 0);
  if (ab) fail();
  // this lane's token (columns past M read token 0; their outputs are dropped)
  const uint4* xtok = xs + (g < p.m ? g : 0) * xk16;
  const int lr0 = g, lr1 = g + 8;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  int issued = total < p.stages ? total : p.stages;  // warp 0: stages whose copies were started
  int tile = 0, piece = 0;  // stage s's coordinates, advanced at the end of each iteration
  for (int s = 0; s < total; ++s) {
    const int slot = s % p.stages;
    if (p.seg && tile == 0) {  // a new K segment: its X (every warp is done with the previous one)
      __syncthreads();
      load_x(piece * p.piece_chunks, min(p.piece_chunks, p.chunks - piece * p.piece_chunks));
      __syncthreads();
      chunk_biases(min(p.piece_chunks, p.chunks - piece * p.piece_chunks));
      __syncthreads();
    }
    ab = ab || *s_abort != 0;
    if (!ab && !wait_bar(&bars[slot], (uint32_t)((s / p.stages) & 1))) {
      ab = true;
      fail();
    }
    const int c0 = piece * p.piece_chunks;
    const int pc = min(p.piece_chunks, p.chunks - c0);
    const uint8_t* sb = stage_base + slot * slot_bytes;
    const int sr0 = min(tile * 16 + lr0, rows_here - 1) * p.G;
    const int sr1 = min(tile * 16 + lr1, rows_here - 1) * p.G;
    for (int c = warp; c < pc && !ab; c += kWarps) {
      const uint4 wa = *reinterpret_cast<const uint4*>(sb + lr0 * p.slot_stride + c * 64 + t * 16);
      const uint4 wb = *reinterpret_cast<const uint4*>(sb + lr1 * p.slot_stride + c * 64 + t * 16);
      const int cg = c0 + c;
      uint4 xf[4];
      const uint4* xc = xtok + (p.seg ? c : cg) * 16 + t * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j) xf[j] = xc[j ^ ((t >> 1) & 1)];
      float d[4];
      chunk_mma(wa, wb, xf, d);
      const int grp = cg >> p.cpg_shift;
      const float s0 = ss[sr0 + grp], s1 = ss[sr1 + grp];
      const float2 b = *reinterpret_cast<const float2*>(cbias + (p.seg ? c : cg) * kTokens + 2 * t);
      acc[0] = fmaf(s0, d[0] - b.x, acc[0]);
      acc[1] = fmaf(s0, d[1] - b.y, acc[1]);
      acc[2] = fmaf(s1, d[2] - b.x, acc[2]);
      acc[3] = fmaf(s1, d[3] - b.y, acc[3]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);  // this warp is done with the stage's slot
    const bool tile_end = (piece == p.pieces - 1);
    // this warp's partial rows of the tile: written at the tile's end, or (long
    // K) carried across segments in the tile's own region (same sums, in order)
    float* tred = red + (p.seg ? tile * (kWarps * 16 * kTokens) : 0);
    if (p.seg || tile_end) {
      float* rw = tred + warp * (16 * kTokens);
      if (p.seg && piece > 0) {
        acc[0] += rw[lr0 * kTokens + 2 * t];
        acc[1] += rw[lr0 * kTokens + 2 * t + 1];
        acc[2] += rw[lr1 * kTokens + 2 * t];
        acc[3] += rw[lr1 * kTokens + 2 * t + 1];
      }
      rw[lr0 * kTokens + 2 * t] = acc[0];
      rw[lr0 * kTokens + 2 * t + 1] = acc[1];
      rw[lr1 * kTokens + 2 * t] = acc[2];
      rw[lr1 * kTokens + 2 * t + 1] = acc[3];
      acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
    }
    if (tile_end) {
      __syncthreads();  // every warp's partial rows of the tile are written
      if (tid < 16 * kTokens && *s_abort == 0) {
        const int r = tid / kTokens, m = tid - r * kTokens;
        const int lr = tile * 16 + r;
        if (m < p.m && lr < rows_here) {
          float sum = 0.f;
#pragma unroll
          for (int w = 0; w < kWarps; ++w) sum += tred[w * (16 * kTokens) + r * kTokens + m];
          Y[m * ldy + row_begin + lr] = __float2half_rn(sum);
        }
      }
      if (!p.seg) __syncthreads();  // partials read before the next tile overwrites them
    }
    // warp 0 refills the slot with the stage `stages` ahead once every warp released it
    if (warp == 0 && !ab && s + p.stages < total) {
      if (!wait_bar(&empty[slot], (uint32_t)((s / p.stages) & 1))) {
        ab = true;
        fail();
      } else {
        fence_proxy_async_smem();
        issue(s + p.stages);
        issued = s + p.stages + 1;
      }
    }
    if (p.seg) {
      if (++tile == n_tiles) tile = 0, ++piece;
    } else if (++piece == p.pieces) {
      piece = 0;
      ++tile;
    }
  }
  if (warp == 0 && *s_abort != 0) {  // leave no copy in flight into this CTA's shared memory
    for (int q = issued - p.stages; q < issued; ++q)
      if (q >= 0) (void)mbar_wait_bounded(&bars[q % p.stages], (uint32_t)((q / p.stages) & 1), kWaitNs / 4);
  }
}

int sms_now() {
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

}  // namespace

bool plan_gemm_w4(int64_t M, int64_t N, int64_t K, int64_t group_size, int64_t G) {
  return M >= 1 && M <= kTokens && K % 128 == 0 && group_size % 128 == 0 && (G * 4) % 16 == 0 &&
         N >= 1 && N < (1ll << 31) && K < (1 << 24);
}

cudaError_t launch_gemm_w4(const uint8_t* W, const float* S, const half* X, int64_t ldx, half* Y, int64_t ldy,
                           int64_t M, int64_t N, int64_t K, int64_t group_size, int64_t G, cudaStream_t stream) {
  GemmPlan p;
  const int sms = sms_now();
  int grid = (int)(N < sms ? N : sms);
  p.rows_per_cta = (int)((N + grid - 1) / grid);
  grid = (int)((N + p.rows_per_cta - 1) / p.rows_per_cta);
  p.m = (int)M;
  p.chunks = (int)(K / 128);
  p.cpg = (int)(group_size / 128);
  if (p.cpg & (p.cpg - 1)) return cudaErrorNotSupported;  // the per-token path serves other group sizes
  p.cpg_shift = 0;
  while ((1 << p.cpg_shift) < p.cpg) ++p.cpg_shift;
  p.G = (int)G;
  // The largest piece that fits with two stages, then as many stages as fit
  // (measured: one piece per tile -- K <= 48 chunks -- beats a deeper ring of
  // smaller pieces; the per-stage hand-off, not the copy latency, bounds this
  // kernel).
  p.seg = M * K * 2 > 112 * 1024 ? 1 : 0;
  auto size = [&](int pc, int stages) {
    p.piece_chunks = pc;
    p.stages = stages;
    p.pieces = (p.chunks + p.piece_chunks - 1) / p.piece_chunks;
    p.slot_stride = p.piece_chunks * 64 + kSlotPad;
    p.smem_x = p.seg ? (int)(M * p.piece_chunks * 256) : (int)(M * K * 2);
    p.smem_scale = (int)(((int64_t)p.rows_per_cta * G * 4 + 127) / 128 * 128);
    p.smem_stage = p.stages * 16 * p.slot_stride;
    p.smem_red = (p.seg ? (p.rows_per_cta + 15) / 16 : 1) * kWarps * 16 * kTokens * 4;
    p.smem_bias = (p.seg ? p.piece_chunks : p.chunks) * kTokens * 4;
    p.smem_total = p.smem_x + p.smem_scale + p.smem_stage + p.smem_red + p.smem_bias;
    return p.smem_total <= 226 * 1024;
  };
  int pc = p.chunks < kPieceChunks ? p.chunks : kPieceChunks;
  while (!size(pc, 2) && pc > 8) pc -= 8;
  if (p.smem_total <= 226 * 1024) {
    int st = 2;
    while (st < kStages && size(pc, st + 1)) ++st;
    size(pc, st);
  }
  if (p.smem_total > 226 * 1024) return cudaErrorNotSupported;
  if (cudaError_t e = ensure_smem_attr<gemm_w4_kernel>(p.smem_total); e != cudaSuccess) return e;
  // a programmatic dependent of the previous kernel: the weight copies and
  // scale rows start while it drains; X is read after griddepcontrol.wait
  return launch_ex(gemm_w4_kernel, dim3(grid), dim3(kThreads), (size_t)p.smem_total, stream, 1, true, W, S, X, ldx,
                   Y, ldy, (int)N, (int)K, p);
}

cudaError_t read_and_clear_gemm_w4_error(int* out) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(out, g_gemm_w4_error, sizeof(int));
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(g_gemm_w4_error, &zero, sizeof(int));
}

}  // namespace soinfer
