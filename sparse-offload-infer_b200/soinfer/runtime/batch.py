"""Batched greedy decode: B <= 8 sequences in lockstep (BASELINE configs[4]'s
batch-8 decode).  No reference counterpart -- the reference decodes one token
at a time (runtime/generate.py:429-463); each sequence here follows that loop's
arithmetic with its own KV cache.

Layout: the B sequences' KV caches are stacked by head, [B * n_kv, max_seq,
head_dim] per layer, and their query heads likewise [B * n_q, head_dim], so
one head-norm + RoPE + append launch and one GQA attention launch serve the
whole batch (query head b * n_q + h reads kv head b * n_kv + h / (n_q /
n_kv): sequence b's own cache).  Every INT4 projection is one multi-token
GEMM (soinfer_gemm_w4a16: the B tokens ride the tensor-core MMA's columns, one
pass over the weights); the fp16 LM head is a plain cuBLAS GEMM
(torch.matmul) with a per-row argmax (first maximum, as the batch-1 path).
All sequences share one position (prompts of equal length), held on the
device, so a step is captured once in a CUDA graph and replayed."""
from __future__ import annotations

import torch

from .. import ops
from ..offload.load_hf_checkpoint import LINEAR_SUFFIXES
from .generate import StreamingModel

MAX_BATCH = 8


class BatchDecoder:
    """Greedy decode of up to 8 equal-length prompts together, one CUDA graph
    per step.  Weights must be HBM-resident INT4 (StreamingModel.resident)."""

    def __init__(self, model: StreamingModel, batch: int, max_seq_len: int = 4096):
        if not 1 <= batch <= MAX_BATCH:
            raise ValueError(f"batch must be in [1, {MAX_BATCH}]")
        names = [f"model.layers.{i}.{s}" for i in range(model.num_layers) for s in LINEAR_SUFFIXES]
        if not all(model.is_resident(n) for n in names):
            raise ValueError("BatchDecoder needs every decoder weight resident in HBM (StreamingModel.resident)")
        if any(model.matrices[n].bits != 4 for n in names):
            raise ValueError("BatchDecoder runs INT4 weights")
        self.model, self.B, self.max_seq_len = model, batch, max_seq_len
        dev = model.device
        self.stream = torch.cuda.Stream(dev)
        self.ids = torch.zeros(batch, max_seq_len + 1, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.prompt_len = torch.zeros(1, dtype=torch.int32, device=dev)
        self.cos_t, self.sin_t = ops.precompute_rope_table(model.head_dim, model.rope_theta, max_seq_len, dev)
        shape = (batch * model.num_key_value_heads, max_seq_len, model.head_dim)
        self.k_caches = [torch.zeros(shape, dtype=torch.float16, device=dev) for _ in range(model.num_layers)]
        self.v_caches = [torch.zeros(shape, dtype=torch.float16, device=dev) for _ in range(model.num_layers)]
        self.graph = None

    def _gemm(self, li: int, suffix: str, X: torch.Tensor) -> torch.Tensor:
        name = f"model.layers.{li}.{suffix}"
        m = self.model.matrices[name]
        return ops.gemm_w4a16(self.model.resident[name], m.scale, X, m.packed_k, self.model.group_size)

    def _layer(self, li: int, x: torch.Tensor) -> torch.Tensor:
        """One decoder layer for the B tokens x [B, hidden]."""
        m, B = self.model, self.B
        NQ, NKV, HD, eps = m.num_attention_heads, m.num_key_value_heads, m.head_dim, m.rms_norm_eps
        norms = m.layer_norms[li]
        h = ops.rmsnorm(x, norms["input_layernorm"], eps)
        q = self._gemm(li, "self_attn.q_proj.weight", h).view(B * NQ, HD)
        k = self._gemm(li, "self_attn.k_proj.weight", h).view(B * NKV, HD)
        v = self._gemm(li, "self_attn.v_proj.weight", h).view(B * NKV, HD)
        ops.head_norm_rope(q, k, v, norms["q_norm"], norms["k_norm"], self.cos_t, self.sin_t, self.k_caches[li],
                           self.v_caches[li], pos_dev=self.pos, eps=eps)
        attn = ops.decode_attention_at(q, self.k_caches[li], self.v_caches[li], self.pos).reshape(B, NQ * HD)
        o = self._gemm(li, "self_attn.o_proj.weight", attn)
        h3, h2 = ops.add_rmsnorm(x, o, norms["post_attention_layernorm"], eps)
        gate = self._gemm(li, "mlp.gate_proj.weight", h3)
        up = self._gemm(li, "mlp.up_proj.weight", h3)
        hs = ops.swiglu(gate.view(-1), up.view(-1)).view(B, -1)
        return h2 + self._gemm(li, "mlp.down_proj.weight", hs)

    def _step(self) -> None:
        m, B = self.model, self.B
        cur = self.ids.index_select(1, self.pos.long()).view(B)
        x = m.embed_tokens.index_select(0, cur.long())
        for li in range(m.num_layers):
            x = self._layer(li, x)
        xn = ops.rmsnorm(x, m.final_norm, m.rms_norm_eps)
        nxt = torch.matmul(xn, m.lm_head.t()).argmax(dim=1).to(torch.int32).view(B, 1)
        at = (self.pos + 1).long()
        keep = (self.pos + 1) < self.prompt_len  # still inside the prompts: keep their tokens
        self.ids.index_copy_(1, at, torch.where(keep, self.ids.index_select(1, at), nxt))
        self.pos.add_(1)

    def _capture(self) -> None:
        self.stream.wait_stream(torch.cuda.current_stream(self.model.device))
        with torch.cuda.stream(self.stream):
            self.pos.zero_()
            self._step()  # warm-up: workspaces and lazy initialisation outside the capture
            self.stream.synchronize()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=self.stream):
                self._step()
        torch.cuda.synchronize(self.model.device)

    def generate(self, prompts: list[list[int]], n_new: int, timings: dict | None = None) -> list[list[int]]:
        """Greedy-decode n_new tokens after each of the B prompts (equal
        lengths).  timings (optional): CUDA-event milliseconds of the prompt
        steps ("prefill_ms") and of the n_new - 1 generating steps
        ("decode_ms"); every step advances all B sequences."""
        if len(prompts) != self.B or len({len(p) for p in prompts}) != 1:
            raise ValueError(f"need {self.B} prompts of equal length")
        P = len(prompts[0])
        if P < 1 or P + n_new > self.max_seq_len:
            raise ValueError(f"need 1 <= prompt length and prompt + n_new <= max_seq_len ({self.max_seq_len})")
        if self.graph is None:
            self._capture()
        self.stream.wait_stream(torch.cuda.current_stream(self.model.device))
        with torch.cuda.stream(self.stream):
            self.ids.zero_()
            self.ids[:, :P].copy_(torch.tensor(prompts, dtype=torch.int32), non_blocking=False)
            self.prompt_len.fill_(P)
            self.pos.zero_()
            for kc, vc in zip(self.k_caches, self.v_caches):
                kc.zero_()
                vc.zero_()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            ev[0].record(self.stream)
            for _ in range(P):
                self.graph.replay()
            ev[1].record(self.stream)
            for _ in range(n_new - 1):
                self.graph.replay()
            ev[2].record(self.stream)
        self.stream.synchronize()
        if timings is not None:
            timings["prefill_ms"] = ev[0].elapsed_time(ev[1])
            timings["decode_ms"] = ev[1].elapsed_time(ev[2])
        return self.ids[:, : P + n_new].cpu().tolist()
