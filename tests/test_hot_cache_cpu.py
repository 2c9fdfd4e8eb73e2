"""Hot-channel cache policies (soinfer.offload.hot_cache) against golden
results of the reference's own policy code (tests/golden/make_hot_cache_golden.py):
the static hot set and the hit counts of static / LRU / LFU-with-decay on
seeded Zipf-skewed traces, plus the selector-order independence and the
argument checks."""
import json
import os
import random

import pytest
import torch

from soinfer.offload import hot_cache as hc

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "hot_cache_golden.json")


def _cases():
    with open(GOLDEN) as f:
        return json.load(f)["cases"]


@pytest.mark.parametrize("case", _cases(), ids=lambda c: f"seed{c['seed']}")
def test_policies_match_reference_golden(case):
    trace = case["trace"]
    counts = [0] * case["channels"]
    for t in trace:
        for c in t:
            counts[c] += 1
    got = hc.compare_policies(trace, case["sizes"], frequencies=counts, **case["lfu"])
    assert [[r.policy, r.cache_size, r.hits, r.total] for r in got] == case["results"]
    for size, hot in case["hot_sets"].items():
        assert sorted(hc.StaticFrequencyPolicy(counts, int(size)).hot_set) == hot


def test_policies_ignore_selector_output_order():
    case = _cases()[1]
    rng = random.Random(0)
    shuffled = []
    for t in case["trace"]:
        t = list(t)
        rng.shuffle(t)
        shuffled.append(torch.tensor(t, dtype=torch.int32))
    got = hc.compare_policies(shuffled, case["sizes"], **case["lfu"])
    counts = [0] * case["channels"]
    for t in case["trace"]:
        for c in t:
            counts[c] += 1
    ref = hc.compare_policies(case["trace"], case["sizes"], frequencies=counts, **case["lfu"])
    assert [(r.policy, r.hits, r.total) for r in got] == [(r.policy, r.hits, r.total) for r in ref]


def test_static_ties_keep_lower_index_and_clamp_size():
    p = hc.StaticFrequencyPolicy([5, 7, 7, 1, 7], cache_size=2)
    assert sorted(p.hot_set) == [1, 2]
    assert hc.StaticFrequencyPolicy([1, 2], cache_size=10).cache_size == 2
    r = hc.StaticFrequencyPolicy([0, 3, 3], 1).simulate([[1, 2], [2]])
    assert (r.hits, r.total, r.hit_rate) == (1, 3, pytest.approx(1 / 3))


def test_lfu_rejects_bad_decay_and_empty_trace():
    with pytest.raises(ValueError):
        hc.LFUDecayPolicy(4, decay=0.0)
    with pytest.raises(ValueError):
        hc.LFUDecayPolicy(4, decay=1.5)
    assert hc.LRUPolicy(4).simulate([]).hit_rate == 0.0
