// Placement rule of the batched GEMV's shared-memory byte ring.  Plain C++
// (no CUDA types) so that a host program can exercise it directly.
#pragma once

#ifdef __CUDACC__
#define SOINFER_RING_FN __host__ __device__ __forceinline__
#else
#define SOINFER_RING_FN inline
#endif

namespace soinfer {

// Where an item of `bytes` goes in a ring of `ring_bytes`: the producer frees
// items in issue order, so the live items occupy [tail, head) -- tail = the
// oldest live item's offset, head = the end of the newest -- or, after head has
// wrapped while the oldest item still lies beyond it, [tail, ring end) and
// [0, head), where only [head, tail) is free (tail == head with live items:
// full).  Returns the item's offset, or -1 when the producer must first wait
// for the oldest item (also when `live` has reached `max_items` descriptors).
SOINFER_RING_FN int ring_place(int head, int tail, int live, int bytes, int ring_bytes, int max_items) {
  if (live == 0) return head + bytes > ring_bytes ? 0 : head;
  if (live >= max_items) return -1;
  if (tail < head) {
    if (head + bytes <= ring_bytes) return head;
    return bytes <= tail ? 0 : -1;
  }
  return head + bytes <= tail ? head : -1;
}

}  // namespace soinfer
