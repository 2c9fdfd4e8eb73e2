"""TEST INFRASTRUCTURE: runs the reference implementation's own decode loops
(sparse-offload-infer's soinfer package, installed with its CUDA extension
under baseline/_ref) on a Hugging Face checkpoint directory and writes the
greedy token ids as JSON.  Run in a subprocess by
tests/test_reference_runtime_gpu.py -- the reference's package is also named
soinfer, so it must not share a process with this build's.

    python tests/reference_runner.py REF_ROOT MODEL_DIR OUT_JSON PROMPT_JSON N_NEW DIP_K HOT_JSON

Calls (reference python/soinfer/runtime): loader.load_streaming_model
(loader.py:33-82), generate.generate_streaming (generate.py:429-463),
generate_dip (:466-500), generate_cached_dip (:503-542) with
offload.hot_cache.HotCache.build (hot_cache.py:67-96).
"""
import json
import sys


def main() -> None:
    ref_root, model_dir, out, prompt, n_new, dip_k, hot = sys.argv[1:8]
    sys.path.insert(0, ref_root)
    import soinfer
    from soinfer.offload.hot_cache import HotCache
    from soinfer.runtime import generate as g
    from soinfer.runtime.loader import load_streaming_model

    assert soinfer.__file__.startswith(ref_root), soinfer.__file__
    prompt, n_new, dip_k, hot = json.loads(prompt), int(n_new), int(dip_k), json.loads(hot)
    model = load_streaming_model(model_dir, group_size=128, include_dip=True)
    max_seq = len(prompt) + n_new + 1
    res = {"dense": g.generate_streaming(model, prompt, n_new, max_seq_len=max_seq),
           "dip": g.generate_dip(model, prompt, n_new, dip_k, max_seq_len=max_seq)}
    caches = [HotCache.build(model, layer, hot) for layer in range(model.num_layers)]
    res["cached_dip"] = g.generate_cached_dip(model, prompt, n_new, dip_k, caches, max_seq_len=max_seq)
    with open(out, "w") as f:
        json.dump(res, f)


if __name__ == "__main__":
    main()
