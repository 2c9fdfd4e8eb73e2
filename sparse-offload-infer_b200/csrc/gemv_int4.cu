// INT4 (AWQ-order, symmetric, fp32 group scales) GEMV for batch-1 decode.
//
// Reference semantics: csrc/kernels/gemv_w4a16_group.cu:77-127 of
// sparse-offload-infer (y[n] = half(sum_k s[n, k/g] * q[n,k] * x[k]), fp32
// accumulation) and csrc/kernels/gemv_dip_fused.cu:48-102 (the same per row,
// with the row taken from a hot cache or a staging buffer per descriptor).
//
// Fast path (group_size % 128 == 0, K % 128 == 0, 16-byte aligned rows, the
// common decode case):
//  * Work split: the N output rows are cut into one contiguous, equal slab per
//    CTA (grid = min(#SMs, N)), so every SM streams the same number of bytes
//    and no cross-CTA reduction is needed.
//  * Streaming: one warp issues cp.async.bulk copies (one per row piece) into
//    a ring of shared-memory stages completing on mbarriers, so each row is
//    read as one contiguous burst.  In plain mode the copies are issued before
//    griddepcontrol.wait: launched with programmatic dependent launch, the
//    kernel streams its weights while the previous kernel in the stream is
//    still running and only waits for x.
//  * Math: each packed 32-bit word is unpacked to exact fp16 integers in
//    registers (one LOP3 per half2, see common.cuh) and the dot products run
//    on the tensor pipe with mma.sync.m16n8k16 (exact fp16 x fp16 products,
//    fp32 accumulation).  At batch 1 the B operand is x replicated over the 8
//    MMA columns, so every D column holds the row sums.  The fp32 group scale
//    is applied once per 128-wide K chunk.
//    Why the tensor pipe at batch 1: B200 streams ~23 HBM bytes per SM per
//    clock, ~2.8 SIMT instructions per INT4 value; an fp32 SIMT dot product
//    costs >= 3, and an fp16 HFMA2 dot product misses the rel-L2 1e-3 parity
//    bar.  With the MMA doing the multiply-adds ~1.1 instructions per value
//    remain (the unpack).
//  * The reduction order depends only on (N, K, group size, #SMs), never on
//    where a row's bytes came from, so plain / indexed / descriptor sources
//    produce bit-identical outputs.
//  * Every mbarrier wait is bounded (2 s); on timeout the CTA sets a device
//    error bit (soinfer_device_errors) and exits instead of hanging.
//
// Generic path (any group_size % 8 == 0, ragged K, unaligned views): one warp
// per row, fp32 SIMT arithmetic in the reference's per-word form.
#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "peer.cuh"

namespace soinfer {

namespace {

__device__ int g_gemv_w4_error;

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxStages = 4;         // ring depth when the CTA's slab does not fit
constexpr int kMaxResident = 16;      // stages when the whole slab is resident
constexpr int kMaxResidentBytes = 96 * 1024;
constexpr int kMaxTiles = 4;          // 16-row tiles per CTA in resident mode
constexpr int kMaxPieceChunks = 24;   // 16 rows x 24 chunks x 64 B = 24 KB per stage
constexpr int kSlotPad = 64;          // row stride padding inside a stage: conflict-free LDS.128
constexpr uint64_t kWaitNs = 2000000000ull;

struct BulkPlan {
  int rows_per_cta;
  int chunks;        // K / 128
  int piece_chunks;  // 128-K chunks per stage row piece
  int pieces;        // pieces per 16-row tile
  int stages;        // shared-memory stage slots
  int resident;      // 1: every stage of the CTA has its own slot
  int cpg;           // chunks per scale group (group_size / 128)
  int G;             // scale columns per row
  int scale_simt;    // 1: scale rows are not 16-byte multiples -- staged with plain loads, not bulk copies
  int slot_stride;   // bytes between rows inside a stage slot
  int smem_x, smem_scale, smem_stage, smem_total;
};

__device__ __forceinline__ int64_t clamp_row(int64_t r, int64_t rows) {
  return r < 0 ? 0 : (r >= rows ? rows - 1 : r);
}

template <RowMode M>
__device__ __forceinline__ void row_ptrs(const RowSource& src, int64_t row, const uint8_t*& w, const float*& s) {
  if constexpr (M == RowMode::kPlain) {
    w = src.W + row * src.row_bytes;
    s = src.S + row * src.num_groups;
  } else if constexpr (M == RowMode::kIndexed) {
    const int64_t r = clamp_row(src.idx[row], src.rows1);
    w = src.W + r * src.row_bytes;
    s = src.S + r * src.num_groups;
  } else {
    const int32_t d = src.idx[row];
    const bool staging = (desc_is_staging(d) && src.rows2 > 0) || src.rows1 == 0;
    if (staging) {
      const int64_t r = clamp_row(desc_offset(d), src.rows2);
      w = src.W2 + r * src.row_bytes;
      s = src.S2 + r * src.num_groups;
    } else {
      const int64_t r = clamp_row(desc_offset(d), src.rows1);
      w = src.W + r * src.row_bytes;
      s = src.S + r * src.num_groups;
    }
  }
}

// x is stored in shared memory with the uint4 j of each 64-byte (t) segment
// at slot j ^ ((t >> 1) & 1), which makes the per-chunk LDS.128 of the four
// MMA thread-in-group lanes hit distinct banks.
__device__ __forceinline__ int x_slot(int q) {  // q = logical uint4 index within x
  const int t = (q >> 2) & 3;
  return (q & ~3) | ((q & 3) ^ ((t >> 1) & 1));
}

// One 128-K chunk of two rows (this thread's MMA fragments): returns the row
// sums for rows g (d[0]) and g + 8 (d[2]).  Two independent MMA chains (even
// and odd K pairs) halve the dependent-MMA latency.
__device__ __forceinline__ void chunk_dot(const uint4 wa, const uint4 wb, const uint4 xf[4], float& s0, float& s1) {
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
  s0 = e[0] + o[0];
  s1 = e[2] + o[2];
}

// PEER: row-parallel tensor-parallel form -- each output row is stored into
// slot (parity, rank) of every rank's exchange inbox instead of y, and the
// last CTA to finish (ticket) signals the exchange to every rank.
template <RowMode M, bool PEER>
__global__ void __launch_bounds__(kThreads, 2)
    gemv_w4_bulk_kernel(const RowSource src, const half* __restrict__ x, half* __restrict__ y, const int nrows,
                        const int K, const BulkPlan p, const PeerSet ps, const half* __restrict__ glu) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint4* xs = reinterpret_cast<uint4*>(smem);
  float* ss = reinterpret_cast<float*>(smem + p.smem_x);
  uint8_t* stage_base = smem + p.smem_x + p.smem_scale;
  uint64_t* bars = reinterpret_cast<uint64_t*>(stage_base + p.smem_stage);  // [kMaxResident] + scale barrier
  uint64_t* scale_bar = bars + kMaxResident;
  float* red = reinterpret_cast<float*>(bars + kMaxResident + 1);  // [kWarps][kMaxTiles * 16]

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int64_t row_begin = (int64_t)blockIdx.x * p.rows_per_cta;
  int rows_here = nrows - (int)row_begin;
  rows_here = rows_here < 0 ? 0 : (rows_here > p.rows_per_cta ? p.rows_per_cta : rows_here);
  const int n_tiles = (rows_here + 15) / 16;
  const int total = n_tiles * p.pieces;
  const int slot_bytes = 16 * p.slot_stride;
  const uint32_t scale_row_bytes = (uint32_t)p.G * 4u;

  if (tid == 0) {
    for (int s = 0; s <= kMaxResident; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();
  // Row indices / descriptors are produced by the preceding kernel.
  if constexpr (M != RowMode::kPlain) pdl_wait();

  // producer: warp 0, lane r < 16 copies row r of the stage's tile piece
  auto issue = [&](int s) {
    const int slot = s % p.stages;
    const int tile = s / p.pieces, piece = s - tile * p.pieces;
    const int c0 = piece * p.piece_chunks;
    const int pc = min(p.piece_chunks, p.chunks - c0);
    const int valid = min(16, rows_here - tile * 16);
    if (lane == 0) mbar_arrive_expect_tx(&bars[slot], (uint32_t)(valid * pc * 64));
    if (lane < valid) {
      const uint8_t* w;
      const float* sc;
      row_ptrs<M>(src, row_begin + tile * 16 + lane, w, sc);
      bulk_g2s(stage_base + slot * slot_bytes + lane * p.slot_stride, w + (int64_t)c0 * 64, (uint32_t)(pc * 64),
               &bars[slot]);
    }
  };
  if (warp == 0) {
    // scale rows of this CTA (contiguous in plain mode)
    if (p.scale_simt) {
      // staged by all threads below
    } else if constexpr (M == RowMode::kPlain) {
      if (lane == 0) {
        const uint32_t bytes = (uint32_t)rows_here * scale_row_bytes;
        mbar_arrive_expect_tx(scale_bar, bytes);
        bulk_g2s(ss, src.S + row_begin * src.num_groups, bytes, scale_bar);
      }
    } else {
      if (lane == 0) mbar_arrive_expect_tx(scale_bar, (uint32_t)rows_here * scale_row_bytes);
      __syncwarp();
      for (int r = lane; r < rows_here; r += 32) {
        const uint8_t* w;
        const float* sc;
        row_ptrs<M>(src, row_begin + r, w, sc);
        bulk_g2s(ss + r * p.G, sc, scale_row_bytes, scale_bar);
      }
    }
    const int first = total < p.stages ? total : p.stages;
    for (int s = 0; s < first; ++s) issue(s);
  }
  if constexpr (M == RowMode::kPlain) pdl_wait();
  uint32_t epoch = 0;
  int par = 0;
  if constexpr (PEER) {
    epoch = peer_next_epoch(ps);
    par = (int)(epoch & 1u);
  }
  auto put = [&](int64_t row, float v) {
    half h = __float2half_rn(v);
    if (glu != nullptr) {  // SwiGLU epilogue on the selected row's gate value (x / (1 + exp(-x)) in fp32)
      const float gv = __half2float(glu[M == RowMode::kIndexed ? src.idx[row] : row]);
      h = __float2half_rn((gv / (1.0f + expf(-gv))) * __half2float(h));
    }
    if constexpr (PEER) {
      for (int r = 0; r < ps.world; ++r) reinterpret_cast<half*>(peer_slot(ps, r, par, ps.rank))[row] = h;
    } else {
      y[row] = h;
    }
  };
  // every row stored: the last CTA signals the exchange (PEER only)
  auto finish = [&]() {
    if constexpr (PEER) {
      __threadfence_system();  // every thread's row stores, before the CTA counts itself done
      __syncthreads();
      if (tid == 0) {
        const unsigned prev = atomicAdd(peer_ticket(ps), 1u);
        if (prev == gridDim.x - 1) {
          *peer_ticket(ps) = 0u;
          __threadfence_system();
          for (int r = 0; r < ps.world; ++r) st_release_sys_u32(peer_flag(ps, r, par, ps.rank), epoch);
        }
      }
    }
  };
  // x -> shared memory (L2-coherent loads: x may come from the previous kernel)
  {
    const uint4* xg = reinterpret_cast<const uint4*>(x);
    const int n16 = K / 8;
    for (int i = tid; i < n16; i += kThreads) xs[x_slot(i)] = __ldcg(xg + i);
  }
  if (p.scale_simt) {
    // (tensor-parallel shards: e.g. 10 or 17 groups per row) -- made visible by the barrier below
    for (int i = tid; i < rows_here * p.G; i += kThreads) {
      const int r = i / p.G, gi = i - r * p.G;
      const uint8_t* w;
      const float* sc;
      row_ptrs<M>(src, row_begin + r, w, sc);
      ss[i] = __ldg(sc + gi);
    }
  }
  const bool scales_ok = p.scale_simt ? true : mbar_wait_bounded(scale_bar, 0, kWaitNs);
  const int lr0 = g, lr1 = g + 8;

  if (p.resident) {
    // every stage has its own slot: wait for all of them, then compute
    // chunk-major so each x fragment is loaded once and reused by all tiles
    bool ok = scales_ok;
    for (int s = 0; s < total; ++s) ok = mbar_wait_bounded(&bars[s], 0, kWaitNs) && ok;
    if (__syncthreads_or(!ok)) {
      if (tid == 0) atomicOr(&g_gemv_w4_error, kErrCopyTimeout);
      return;
    }
    float acc0[kMaxTiles], acc1[kMaxTiles];
#pragma unroll
    for (int i = 0; i < kMaxTiles; ++i) acc0[i] = acc1[i] = 0.f;
    for (int c = warp; c < p.chunks; c += kWarps) {
      uint4 xf[4];
      const uint4* xc = xs + c * 16 + t * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j) xf[j] = xc[j ^ ((t >> 1) & 1)];
      const int piece = c / p.piece_chunks, cc = c - piece * p.piece_chunks;
      const int grp = c / p.cpg;
#pragma unroll
      for (int tile = 0; tile < kMaxTiles; ++tile) {
        if (tile < n_tiles) {
          const uint8_t* sb = stage_base + (tile * p.pieces + piece) * slot_bytes + cc * 64 + t * 16;
          const uint4 wa = *reinterpret_cast<const uint4*>(sb + lr0 * p.slot_stride);
          const uint4 wb = *reinterpret_cast<const uint4*>(sb + lr1 * p.slot_stride);
          float d0, d1;
          chunk_dot(wa, wb, xf, d0, d1);
          const int sr0 = min(tile * 16 + lr0, rows_here - 1) * p.G;
          const int sr1 = min(tile * 16 + lr1, rows_here - 1) * p.G;
          acc0[tile] = fmaf(ss[sr0 + grp], d0, acc0[tile]);
          acc1[tile] = fmaf(ss[sr1 + grp], d1, acc1[tile]);
        }
      }
    }
    if (t == 0) {
#pragma unroll
      for (int tile = 0; tile < kMaxTiles; ++tile) {
        if (tile < n_tiles) {
          red[warp * (kMaxTiles * 16) + tile * 16 + lr0] = acc0[tile];
          red[warp * (kMaxTiles * 16) + tile * 16 + lr1] = acc1[tile];
        }
      }
    }
    __syncthreads();
    for (int r = tid; r < rows_here; r += kThreads) {
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) sum += red[w * (kMaxTiles * 16) + r];
      put(row_begin + r, sum);
    }
    finish();
    return;
  }

  // streaming: ring of p.stages slots, refilled as tiles are consumed
  if (__syncthreads_or(!scales_ok)) {
    if (tid == 0) atomicOr(&g_gemv_w4_error, kErrCopyTimeout);
    return;
  }
  float acc0 = 0.f, acc1 = 0.f;
  for (int s = 0; s < total; ++s) {
    const int slot = s % p.stages;
    const bool ok = mbar_wait_bounded(&bars[slot], (uint32_t)((s / p.stages) & 1), kWaitNs);
    if (__syncthreads_or(!ok)) {
      if (tid == 0) atomicOr(&g_gemv_w4_error, kErrCopyTimeout);
      // give copies still in flight into this CTA's shared memory a bounded chance to land
      for (int q = s; q < total && q < s + p.stages; ++q)
        (void)mbar_wait_bounded(&bars[q % p.stages], (uint32_t)((q / p.stages) & 1), kWaitNs / 4);
      return;
    }
    const int tile = s / p.pieces, piece = s - tile * p.pieces;
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
      const uint4* xc = xs + cg * 16 + t * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j) xf[j] = xc[j ^ ((t >> 1) & 1)];
      float d0, d1;
      chunk_dot(wa, wb, xf, d0, d1);
      const int grp = cg / p.cpg;
      acc0 = fmaf(ss[sr0 + grp], d0, acc0);
      acc1 = fmaf(ss[sr1 + grp], d1, acc1);
    }
    const bool tile_end = (piece == p.pieces - 1);
    if (tile_end) {
      if (t == 0) {
        red[warp * 16 + lr0] = acc0;
        red[warp * 16 + lr1] = acc1;
      }
      acc0 = 0.f;
      acc1 = 0.f;
    }
    __syncthreads();  // stage slot fully consumed, partial sums visible
    if (tile_end && tid < 16) {
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) sum += red[w * 16 + tid];
      const int lr = tile * 16 + tid;
      if (lr < rows_here) put(row_begin + lr, sum);
    }
    if (warp == 0 && s + p.stages < total) {
      fence_proxy_async_smem();
      issue(s + p.stages);
    }
  }
  finish();
}

// Generic path: any group_size % 8 == 0, any K, 4-byte aligned rows.
template <RowMode M>
__global__ void __launch_bounds__(128)
    gemv_w4_simt_kernel(const RowSource src, const half* __restrict__ x, half* __restrict__ y, const int64_t nrows,
                        const int64_t K, const int64_t gsz) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 4 + warp;
  pdl_launch_dependents();
  pdl_wait();
  if (row >= nrows) return;
  const uint8_t* w;
  const float* s;
  row_ptrs<M>(src, row, w, s);
  const int64_t words = (K + 7) / 8;
  const uint32_t* wp = reinterpret_cast<const uint32_t*>(w);
  float acc = 0.f;
  for (int64_t wi = lane; wi < words; wi += 32) {
    const int64_t k = wi * 8;
    const float sc = s[k / gsz];
    uint32_t q[4];
    unpack_int4x8(ldg_stream_u32(wp + wi), q);
    const int64_t rem = K - k;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 dq = __half22float2(u32_as_h2(q[j]));
      if (rem >= 8) {
        acc += sc * (dq.x * __half2float(x[k + 2 * j]) + dq.y * __half2float(x[k + 2 * j + 1]));
      } else {
        if (2 * j < rem) acc += sc * dq.x * __half2float(x[k + 2 * j]);
        if (2 * j + 1 < rem) acc += sc * dq.y * __half2float(x[k + 2 * j + 1]);
      }
    }
  }
  acc = warp_sum(acc);
  if (lane == 0) y[row] = __float2half_rn(acc);
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

bool make_plan(int64_t nrows, int64_t K, int64_t gsz, int64_t G, BulkPlan& p, int& grid) {
  const int64_t sms = sm_count();
  grid = (int)(nrows < sms ? nrows : sms);
  p.rows_per_cta = (int)((nrows + grid - 1) / grid);
  grid = (int)((nrows + p.rows_per_cta - 1) / p.rows_per_cta);
  p.chunks = (int)(K / 128);
  p.cpg = (int)(gsz / 128);
  p.G = (int)G;
  p.scale_simt = (G * 4) % 16 != 0 ? 1 : 0;
  p.piece_chunks = p.chunks < kMaxPieceChunks ? p.chunks : kMaxPieceChunks;
  p.pieces = (p.chunks + p.piece_chunks - 1) / p.piece_chunks;
  p.slot_stride = p.piece_chunks * 64 + kSlotPad;
  const int tiles = (p.rows_per_cta + 15) / 16;
  const int total = tiles * p.pieces;
  p.resident = (tiles <= kMaxTiles && total <= kMaxResident && total * 16 * p.slot_stride <= kMaxResidentBytes) ? 1 : 0;
  p.stages = p.resident ? total : (total < kMaxStages ? total : kMaxStages);
  p.smem_x = (int)(K * 2);
  p.smem_scale = (int)(((int64_t)p.rows_per_cta * G * 4 + 15) / 16 * 16);
  p.smem_stage = p.stages * 16 * p.slot_stride;
  p.smem_total = p.smem_x + p.smem_scale + p.smem_stage + (kMaxResident + 1) * 8 + kWarps * kMaxTiles * 16 * 4;
  return p.smem_total <= 200 * 1024;
}

template <RowMode M>
bool bulk_ok(const RowSource& src, const half* x, int64_t nrows, int64_t K, int64_t gsz, BulkPlan& plan, int& grid) {
  auto aligned16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return (K % 128 == 0) && (gsz % 128 == 0) && src.row_bytes % 16 == 0 && aligned16(src.W) &&
         (M != RowMode::kDesc || aligned16(src.W2)) && aligned16(x) && nrows < (1ll << 31) &&
         (((src.num_groups * 4) % 16 == 0 && aligned16(src.S) && (M != RowMode::kDesc || aligned16(src.S2))) ||
          ((src.num_groups * 4) % 16 != 0 && (reinterpret_cast<uintptr_t>(src.S) & 3u) == 0)) &&
         K < (1ll << 30) && make_plan(nrows, K, gsz, src.num_groups, plan, grid);
}

template <RowMode M, bool PEER>
cudaError_t launch_bulk(const RowSource& src, const half* x, half* y, int64_t nrows, int64_t K, const BulkPlan& plan,
                        int grid, const PeerSet& ps, cudaStream_t stream, bool pdl, const half* glu = nullptr) {
  auto kernel = gemv_w4_bulk_kernel<M, PEER>;
  if (cudaError_t e = ensure_smem_attr<gemv_w4_bulk_kernel<M, PEER>>(200 * 1024); e != cudaSuccess) return e;
  return launch_ex(kernel, dim3(grid), dim3(kThreads), (size_t)plan.smem_total, stream, 1, pdl, src, x, y,
                   (int)nrows, (int)K, plan, ps, glu);
}

template <RowMode M>
cudaError_t launch_mode(const RowSource& src, const half* x, half* y, int64_t nrows, int64_t K, int64_t gsz,
                        cudaStream_t stream, LaunchOpts opts) {
  BulkPlan plan;
  int grid = 0;
  if (bulk_ok<M>(src, x, nrows, K, gsz, plan, grid)) {
    return launch_bulk<M, false>(src, x, y, nrows, K, plan, grid, PeerSet{}, stream, opts.pdl, opts.glu);
  }
  if (opts.glu != nullptr) return cudaErrorNotSupported;  // the caller applies the epilogue separately
  const int64_t blocks = (nrows + 3) / 4;
  return launch_ex(gemv_w4_simt_kernel<M>, dim3((unsigned)blocks), dim3(128), 0, stream, 1, opts.pdl, src, x, y,
                   nrows, K, gsz);
}

}  // namespace

cudaError_t launch_gemv_w4(RowMode mode, const RowSource& src, const half* x, half* y, int64_t nrows, int64_t K,
                           int64_t group_size, cudaStream_t stream, LaunchOpts opts) {
  switch (mode) {
    case RowMode::kPlain:
      return launch_mode<RowMode::kPlain>(src, x, y, nrows, K, group_size, stream, opts);
    case RowMode::kIndexed:
      return launch_mode<RowMode::kIndexed>(src, x, y, nrows, K, group_size, stream, opts);
    case RowMode::kDesc:
      return launch_mode<RowMode::kDesc>(src, x, y, nrows, K, group_size, stream, opts);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_gemv_w4_peer(const RowSource& src, const half* x, int64_t nrows, int64_t K, int64_t group_size,
                                const PeerSet& ps, cudaStream_t stream) {
  BulkPlan plan;
  int grid = 0;
  if (!bulk_ok<RowMode::kPlain>(src, x, nrows, K, group_size, plan, grid)) return cudaErrorNotSupported;
  return launch_bulk<RowMode::kPlain, true>(src, x, nullptr, nrows, K, plan, grid, ps, stream, false);
}

cudaError_t read_and_clear_gemv_w4_error(int* out) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(out, g_gemv_w4_error, sizeof(int));
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(g_gemv_w4_error, &zero, sizeof(int));
}

}  // namespace soinfer
