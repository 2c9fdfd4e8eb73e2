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
    # teacher-forced logits along the reference's own DIP token sequence
    # (the loop of generate.teacher_forced_nll:545-582, keeping the logits)
    seq = res["dip"]
    pipe = g.WeightPipeline(model)
    res["tf_dense"] = teacher_forced_logits(
        g, model, lambda m, li, x, p, kc, vc: g.run_decoder_layer_streaming(pipe, m, li, x, p, kc, vc), seq, max_seq)
    pipe_d = g.WeightPipeline(model, suffixes=g.DIP_DENSE_SUFFIXES)
    bufs = g.DipBuffers.make(model, max_k=dip_k)
    sel = [[] for _ in range(model.num_layers)]
    res["tf_dip"] = teacher_forced_logits(
        g, model, lambda m, li, x, p, kc, vc: g.run_decoder_layer_dip(pipe_d, m, li, x, p, kc, vc, dip_k, bufs,
                                                                      selected_out=sel), seq, max_seq)
    res["tf_dip_selected"] = sel
    with open(out, "w") as f:
        json.dump(res, f)


def teacher_forced_logits(g, model, layer_fn, token_ids, max_seq_len):
    import torch

    ops = g.ops
    shape = (model.num_key_value_heads, max_seq_len, model.head_dim)
    kcs = [torch.zeros(shape, device="cuda", dtype=torch.float16) for _ in range(model.num_layers)]
    vcs = [torch.zeros(shape, device="cuda", dtype=torch.float16) for _ in range(model.num_layers)]
    out = []
    for pos, tok in enumerate(token_ids[:-1]):
        x = model.embed_tokens[tok].contiguous()
        for li in range(model.num_layers):
            x = layer_fn(model, li, x, pos, kcs[li], vcs[li])
        xn = ops.rmsnorm(x.unsqueeze(0), model.final_norm, model.rms_norm_eps).squeeze(0).contiguous()
        out.append(ops.gemv_fp16_v3(model.lm_head, xn).float().cpu().tolist())
    return out


if __name__ == "__main__":
    main()
