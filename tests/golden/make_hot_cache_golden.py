"""Generates tests/golden/hot_cache_golden.json from the reference implementation.

Imports the reference's own python/soinfer/offload/hot_cache.py
(sparse-offload-infer) from $SOINFER_REF_PYTHON (the reference checkout's
python/ folder) -- its policy half is pure Python -- and records, for
seeded synthetic selection traces (Zipf-skewed channel popularity, as in
the cache-aware DIP benchmark), the hot set of the static policy and the hit counts of
the static, LRU and LFU-with-decay policies at several cache sizes.  The
committed JSON pins soinfer.offload.hot_cache; this script only runs where
the reference source is available.

    python tests/golden/make_hot_cache_golden.py
"""
from __future__ import annotations

import importlib.util
import json
import os
import sys

import numpy as np

REF = os.environ.get("SOINFER_REF_PYTHON", "")  # the reference checkout's python/ directory (required)
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "hot_cache_golden.json")


def make_trace(seed: int, channels: int, k: int, tokens: int) -> list[list[int]]:
    """Per token, k distinct channels drawn with Zipf(1.1) popularity over a seeded permutation."""
    rng = np.random.default_rng(seed)
    perm = rng.permutation(channels)
    w = 1.0 / np.arange(1, channels + 1) ** 1.1
    p = np.empty(channels)
    p[perm] = w / w.sum()
    return [sorted(int(c) for c in rng.choice(channels, size=k, replace=False, p=p)) for _ in range(tokens)]


def main() -> None:
    spec = importlib.util.spec_from_file_location("ref_hot_cache", os.path.join(REF, "soinfer/offload/hot_cache.py"))
    ref = importlib.util.module_from_spec(spec)
    sys.modules["ref_hot_cache"] = ref
    spec.loader.exec_module(ref)  # the reference's own module (policy half needs only torch)
    cases = []
    for seed, (channels, k, tokens, sizes, lfu) in enumerate([
        (64, 16, 40, [0, 4, 16, 48], {}),
        (256, 96, 60, [8, 32, 128], {"decay": 0.9, "decay_every": 7}),
        (1024, 512, 30, [100, 307], {"decay": 0.98, "decay_every": 5}),
    ]):
        trace = make_trace(seed, channels, k, tokens)
        counts = [0] * channels
        for t in trace:
            for c in t:
                counts[c] += 1
        results = ref.compare_policies(trace, sizes, frequencies=counts, **lfu)
        hot = {str(s): sorted(ref.StaticFrequencyPolicy(counts, s).hot_set) for s in sizes}
        cases.append({"seed": seed, "channels": channels, "k": k, "tokens": tokens, "sizes": sizes, "lfu": lfu,
                      "trace": trace, "hot_sets": hot,
                      "results": [[r.policy, r.cache_size, r.hits, r.total] for r in results]})
    with open(OUT, "w") as f:
        json.dump({"source": "reference python/soinfer/offload/hot_cache.py", "cases": cases}, f)
    print("wrote", OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
