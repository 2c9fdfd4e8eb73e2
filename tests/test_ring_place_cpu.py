"""The batched GEMV's ring placement rule (csrc/ring_place.h, the function the
kernel's producer calls), compiled for the host with g++ and driven by a
producer / consumer simulation: items of mixed sizes are issued in order,
consumed out of order (two consumer groups take alternate tasks), and freed
by the producer in issue order only when it has to wait -- the kernel's
protocol.  A placement must never overlap an item that is not yet consumed,
must stay inside the ring, and may keep at most the descriptor limit in
flight.

The fixed case is the sequence that corrupted live items under the earlier
rule (which checked a new item only against the oldest live item's start):
four 45696-byte items, a 13056-byte item at the ring's end, then large items
again, with the small item still unconsumed when head wraps a second time."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "sparse-offload-infer_b200", "csrc")

DRIVER = r"""
#include <cstdio>
#include <cstdlib>
#include <deque>
#include <random>
#include <vector>
#include "ring_place.h"

struct Item { int off, bytes; bool consumed; };

// returns the number of violations; prints the first one
static int simulate(unsigned seed, int ring, int max_items, const std::vector<int>& sizes, double p_consume,
                    bool hold_small) {
  std::mt19937 rng(seed);
  std::uniform_real_distribution<double> u(0.0, 1.0);
  std::deque<Item> live;  // issued and not yet freed, oldest first
  int head = 0, bad = 0;
  for (size_t n = 0; n < sizes.size(); ++n) {
    const int b = sizes[n];
    int at;
    while (true) {
      for (auto& it : live)  // consumers make progress in any order
        if (!it.consumed && u(rng) < p_consume && !(hold_small && it.bytes < 20000)) it.consumed = true;
      const int tail = live.empty() ? 0 : live.front().off;
      at = soinfer::ring_place(head, tail, (int)live.size(), b, ring, max_items);
      if (at >= 0) break;
      live.front().consumed = true;  // the producer waits for the oldest item, then frees it
      live.pop_front();
    }
    if (at < 0 || at + b > ring) { if (!bad) std::printf("out of ring: [%d,%d)\n", at, at + b); ++bad; }
    if ((int)live.size() >= max_items) { if (!bad) std::printf("descriptor limit exceeded\n"); ++bad; }
    for (const auto& it : live)
      if (!it.consumed && at < it.off + it.bytes && it.off < at + b) {
        if (!bad) std::printf("overlap: new [%d,%d) live [%d,%d)\n", at, at + b, it.off, it.off + it.bytes);
        ++bad;
      }
    live.push_back({at, b, false});
    head = at + b;
  }
  return bad;
}

int main() {
  const int ring = 196352, max_items = 16;  // the headline batch's ring and descriptor count
  int bad = 0;
  // fixed case: the small item stays unconsumed while head wraps twice
  std::vector<int> fixed = {45696, 45696, 45696, 45696, 13056};
  for (int i = 0; i < 12; ++i) fixed.push_back(45696);
  bad += simulate(1, ring, max_items, fixed, 0.5, true);
  // random mixes of the kernel's item sizes (whole-tile, ragged, segment items)
  const int kinds[] = {45696, 13056, 52224, 3328, 26112, 17408, 5504};
  for (unsigned seed = 0; seed < 300; ++seed) {
    std::mt19937 rng(seed);
    std::vector<int> sizes(2000);
    for (auto& s : sizes) s = kinds[rng() % 7];
    bad += simulate(seed, ring, max_items, sizes, seed % 3 == 0 ? 0.05 : 0.3, false);
  }
  // uniform sizes (the headline's per-CTA stream) and a tiny ring
  bad += simulate(7, ring, max_items, std::vector<int>(3000, 45696), 0.3, false);
  bad += simulate(8, 60000, 4, std::vector<int>(3000, 13056), 0.2, false);
  std::printf("violations %d\n", bad);
  return bad == 0 ? 0 : 1;
}
"""


def test_ring_placement_never_overwrites_live_items(tmp_path):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("no host C++ compiler")
    src = tmp_path / "ring_driver.cpp"
    exe = tmp_path / "ring_driver"
    src.write_text(DRIVER)
    subprocess.run([gxx, "-O2", "-std=c++17", "-I", CSRC, str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "violations 0" in out.stdout
