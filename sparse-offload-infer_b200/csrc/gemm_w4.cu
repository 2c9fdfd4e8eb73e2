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
// each packed word to exact fp16 values (LOP3 + one half2 op per pair) and
// run two MMA chains; at each tile's end the per-warp partials [16 rows x 8
// tokens] are summed in warp order (deterministic) and written.
#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"

namespace soinfer {
namespace {

__device__ int g_gemm_w4_error;

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kStages = 4;
constexpr int kPieceChunks = 24;
constexpr int kSlotPad = 64;
constexpr int kTokens = 8;
constexpr uint64_t kWaitNs = 2000000000ull;

struct GemmPlan {
  int rows_per_cta, chunks, piece_chunks, pieces, stages, cpg, G, slot_stride;
  int m;    // tokens
  int seg;  // 1: K-segment-major order, X staged one piece's chunks at a time
  int smem_x, smem_scale, smem_stage, smem_red, smem_total;
};

// x in shared memory: token m's K values at uint4 offset m * K/8, each
// 64-byte segment's four uint4 swizzled so a chunk's four lane-groups read
// distinct banks (same layout as the single-token GEMV).
__device__ __forceinline__ int x_slot(int q) {
  const int t = (q >> 2) & 3;
  return (q & ~3) | ((q & 3) ^ ((t >> 1) & 1));
}

// One 128-K chunk of two rows (g, g + 8) against the thread's token columns
// (2t, 2t + 1): d[0..1] row g, d[2..3] row g + 8.
__device__ __forceinline__ void chunk_mma(const uint4 wa, const uint4 wb, const uint4 xf[4], float d[4]) {
  const uint32_t r0[4] = {wa.x, wa.y, wa.z, wa.w};
  const uint32_t r1[4] = {wb.x, wb.y, wb.z, wb.w};
  float e[4] = {0.f, 0.f, 0.f, 0.f}, o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t p0[4], p1[4];
    unpack_int4x8(r0[j], p0);
    unpack_int4x8(r1[j], p1);
    const uint32_t a_lo[4] = {p0[0], p1[0], p0[1], p1[1]};
    mma_16816(e, a_lo, xf[j].x, xf[j].y);
    const uint32_t a_hi[4] = {p0[2], p1[2], p0[3], p1[3]};
    mma_16816(o, a_hi, xf[j].z, xf[j].w);
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) d[c] = e[c] + o[c];
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
  __shared__ uint64_t bars[kStages + 1];
  uint64_t* scale_bar = bars + kStages;

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
  if (!p.seg) load_x(0, p.chunks);
  if (total == 0) return;
  const bool scales_ok = mbar_wait_bounded(scale_bar, 0, kWaitNs);
  if (__syncthreads_or(!scales_ok)) {
    if (tid == 0) atomicOr(&g_gemm_w4_error, kErrCopyTimeout);
    for (int q = 0; q < total && q < p.stages; ++q)
      (void)mbar_wait_bounded(&bars[q % p.stages], 0, kWaitNs / 4);
    return;
  }
  // this lane's token (columns past M read token 0; their outputs are dropped)
  const uint4* xtok = xs + (g < p.m ? g : 0) * xk16;
  const int lr0 = g, lr1 = g + 8;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int s = 0; s < total; ++s) {
    const int slot = s % p.stages;
    int tile, piece;
    coords(s, tile, piece);
    if (p.seg && tile == 0) {  // a new K segment: its X (every warp is done with the previous one)
      __syncthreads();
      load_x(piece * p.piece_chunks, min(p.piece_chunks, p.chunks - piece * p.piece_chunks));
      __syncthreads();
    }
    const bool ok = mbar_wait_bounded(&bars[slot], (uint32_t)((s / p.stages) & 1), kWaitNs);
    if (__syncthreads_or(!ok)) {
      if (tid == 0) atomicOr(&g_gemm_w4_error, kErrCopyTimeout);
      for (int q = s; q < total && q < s + p.stages; ++q)
        (void)mbar_wait_bounded(&bars[q % p.stages], (uint32_t)((q / p.stages) & 1), kWaitNs / 4);
      return;
    }
    const int c0 = piece * p.piece_chunks;
    const int pc = min(p.piece_chunks, p.chunks - c0);
    const uint8_t* sb = stage_base + slot * slot_bytes;
    const int sr0 = min(tile * 16 + lr0, rows_here - 1) * p.G;
    const int sr1 = min(tile * 16 + lr1, rows_here - 1) * p.G;
    for (int c = warp; c < pc; c += kWarps) {
      const uint4 wa = *reinterpret_cast<const uint4*>(sb + lr0 * p.slot_stride + c * 64 + t * 16);
      const uint4 wb = *reinterpret_cast<const uint4*>(sb + lr1 * p.slot_stride + c * 64 + t * 16);
      const int cg = c0 + c;
      uint4 xf[4];
      const uint4* xc = xtok + (p.seg ? c : cg) * 16 + t * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j) xf[j] = xc[j ^ ((t >> 1) & 1)];
      float d[4];
      chunk_mma(wa, wb, xf, d);
      const int grp = cg / p.cpg;
      const float s0 = ss[sr0 + grp], s1 = ss[sr1 + grp];
      acc[0] = fmaf(s0, d[0], acc[0]);
      acc[1] = fmaf(s0, d[1], acc[1]);
      acc[2] = fmaf(s1, d[2], acc[2]);
      acc[3] = fmaf(s1, d[3], acc[3]);
    }
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
    __syncthreads();  // stage slot consumed; partials visible
    if (tile_end && tid < 16 * kTokens) {
      const int r = tid / kTokens, m = tid - r * kTokens;
      const int lr = tile * 16 + r;
      if (m < p.m && lr < rows_here) {
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) sum += tred[w * (16 * kTokens) + r * kTokens + m];
        Y[m * ldy + row_begin + lr] = __float2half_rn(sum);
      }
    }
    if (warp == 0 && s + p.stages < total) {
      fence_proxy_async_smem();
      issue(s + p.stages);
    }
    if (tile_end && !p.seg) __syncthreads();  // partials read before the next tile overwrites them
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
  p.G = (int)G;
  p.piece_chunks = p.chunks < kPieceChunks ? p.chunks : kPieceChunks;
  p.pieces = (p.chunks + p.piece_chunks - 1) / p.piece_chunks;
  p.slot_stride = p.piece_chunks * 64 + kSlotPad;
  p.stages = kStages;
  p.seg = M * K * 2 > 112 * 1024 ? 1 : 0;
  p.smem_x = p.seg ? (int)(M * p.piece_chunks * 256) : (int)(M * K * 2);
  p.smem_scale = (int)(((int64_t)p.rows_per_cta * G * 4 + 127) / 128 * 128);
  p.smem_stage = p.stages * 16 * p.slot_stride;
  p.smem_red = (p.seg ? (p.rows_per_cta + 15) / 16 : 1) * kWarps * 16 * kTokens * 4;
  p.smem_total = p.smem_x + p.smem_scale + p.smem_stage + p.smem_red;
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
