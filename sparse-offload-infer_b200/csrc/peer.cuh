// Peer-memory exchange between the ranks of one node (tensor parallelism).
//
// Every rank owns one exchange buffer (cudaMalloc'd, shared with the other
// processes through CUDA IPC handles) and maps every peer's buffer, so a
// kernel can store straight into another GPU's memory over NVLink.  Layout of
// each buffer (PeerSet::base[r] is rank r's, as mapped in this process):
//   [0, 64)    flags u32 [2 parities][kMaxPeers]: flags[p][s] = epoch of the
//              last exchange whose data rank s finished pushing here
//   [64, 68)   epoch i32 (local: the number of exchanges this rank completed)
//   [128, 132) ticket u32 (local: completion count of a pushing GEMV's CTAs)
//   [256, ..)  inbox [2 parities][world][slot_bytes]: slot (p, s) holds what
//              rank s pushed for an exchange of parity p
//
// Protocol of exchange number e (e = epoch + 1, parity e & 1): every rank
// pushes its data into slot (parity, rank) of every rank's inbox (its own
// included), then -- after a system-scope fence -- release-stores e into
// flags[parity][rank] of every rank; every rank then acquire-polls its own
// flags[parity][0..world) until all equal e, reads its inbox, and sets its
// epoch to e.  Reusing parity p again (exchange e + 2) is safe: a rank pushes
// for e + 2 only after it saw everybody's e + 1 flag, which each rank sets
// only after it finished reading its e inbox.  All ranks must run the same
// sequence of exchanges.  Every poll is bounded (kPeerWaitNs): on timeout the
// kernel records kErrPeerTimeout and returns (no hang) without advancing its
// epoch.  The ranks are then out of step (this rank already signalled e, a
// late rank may not have), so after kErrPeerTimeout every rank resets its own
// buffer's header (flags, epoch, ticket: soinfer_peer_buffer_reset) between
// steps, with a host barrier before and after, and the exchanges restart at 1.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace soinfer {

constexpr uint64_t kPeerWaitNs = 1000000000ull;

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ps.base[r] by selects over constant indices (a runtime index into the
// kernel-parameter array would copy it to local memory).
__device__ __forceinline__ uint8_t* peer_base(const PeerSet& ps, int r) {
  uint8_t* b = ps.base[0];
#pragma unroll
  for (int i = 1; i < kMaxPeers; ++i) b = (r == i) ? ps.base[i] : b;
  return b;
}

__device__ __forceinline__ uint32_t* peer_flag(const PeerSet& ps, int owner, int parity, int src) {
  return reinterpret_cast<uint32_t*>(peer_base(ps, owner)) + parity * kMaxPeers + src;
}

__device__ __forceinline__ int* peer_epoch(const PeerSet& ps) {
  return reinterpret_cast<int*>(peer_base(ps, ps.rank) + 64);
}

__device__ __forceinline__ unsigned* peer_ticket(const PeerSet& ps) {
  return reinterpret_cast<unsigned*>(peer_base(ps, ps.rank) + 128);
}

__device__ __forceinline__ uint8_t* peer_slot(const PeerSet& ps, int owner, int parity, int src) {
  return peer_base(ps, owner) + kPeerHeaderBytes + ((int64_t)parity * ps.world + src) * ps.slot_bytes;
}

// Number of the exchange about to run (read after the previous kernel finished).
__device__ __forceinline__ uint32_t peer_next_epoch(const PeerSet& ps) {
  return (uint32_t)(*reinterpret_cast<volatile int*>(peer_epoch(ps))) + 1u;
}

// Flag stores to every rank.  Every thread of the CTA calls it after its own
// pushes: each fences them at system scope, the barrier gathers the CTA, and
// threads [0, world) then each signal one rank.
__device__ __forceinline__ void peer_signal_all(const PeerSet& ps, int parity, uint32_t e) {
  __threadfence_system();
  __syncthreads();
  if ((int)threadIdx.x < ps.world) st_release_sys_u32(peer_flag(ps, threadIdx.x, parity, ps.rank), e);
}

// Bounded wait (whole CTA) until every rank signalled exchange e here.
// Returns false (error bit set) on timeout.
__device__ __forceinline__ bool peer_wait_all(const PeerSet& ps, int parity, uint32_t e, int* error_word,
                                              int error_bit) {
  bool ok = true;
  if ((int)threadIdx.x < ps.world) {
    const uint32_t* f = peer_flag(ps, ps.rank, parity, threadIdx.x);
    if ((int)(ld_acquire_sys_u32(f) - e) < 0) {
      const uint64_t t0 = globaltimer_ns();
      while ((int)(ld_acquire_sys_u32(f) - e) < 0) {
        if (globaltimer_ns() - t0 > kPeerWaitNs) {
          ok = false;
          break;
        }
        __nanosleep(32);
      }
    }
  }
  const bool bad = __syncthreads_or(!ok);
  if (bad && threadIdx.x == 0) atomicOr(error_word, error_bit);
  return !bad;
}

}  // namespace soinfer
