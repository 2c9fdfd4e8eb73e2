#!/usr/bin/env python
"""Benchmark of the soinfer B200 decode hot path on the reference's headline
metric: INT4 g128 GEMV HBM throughput (GB/s, % of measured HBM peak).

Workload (configs[0] shapes, run on the GPU): per layer copy one gate_proj
GEMV [6144 x 2048] and one down_proj GEMV [2048 x 6144]; one launch = one
pass over LAYERS distinct layer copies (default 64 -> 128 GEMVs over 858 MB of
packed weights, far above the 126 MB L2, so no L2 flush is needed) through
soinfer_gemv_w4a16_batch (independent GEMVs: the streaming kernel,
gemv_stream.cu); one step = LAUNCHES_PER_STEP (16) such launches back to back,
so that the default 200 timed steps span ~0.5 s.  Weights ~N(0, 0.02)
quantized to group-128 INT4 on the GPU with soinfer.quant; x ~N(0, 1) fp16;
seeded.  `value` = algorithmic bytes (packed weights + fp32 scales + x + y
per GEMV, 6,701,056 B) of all ranks / max rank time, timed with CUDA events.
The GEMVs of a launch are independent (every x is ready); the same stream
with each down_proj reading its gate_proj output (a dependency inside the
launch: the streaming kernel numbers every gate unit first and a down unit
starts once its gate is stored) is reported as config.chained_gate_down.

`e2e`: the same chain through the public streaming API (WeightPipeline: packed
weights streamed from the pinned host arena by the copy engine, double
buffered, x uploaded from pinned memory and the result read back every step).

`--impl reference`: the reference's CPU path (formats.dequantize + fp32
matvec, restated in oracle/) on this host's cores, same metric.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "sparse-offload-infer_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

H, I, G = 2048, 6144, 128
LAUNCHES_PER_STEP = 16
METRIC = "INT4 g128 GEMV HBM GB/s"
UNIT = "GB/s"


def gemv_bytes(n: int, k: int, g: int = G) -> int:
    """Algorithmic bytes of one GEMV: packed INT4 weights + fp32 scales + fp16 x + fp16 y."""
    return n * (-(-k // 8) * 4) + n * (-(-k // g)) * 4 + 2 * k + 2 * n


BYTES_PER_GEMV = gemv_bytes(I, H)  # == gemv_bytes(H, I) == 6,701,056
assert BYTES_PER_GEMV == gemv_bytes(H, I) == 6_701_056


def measured_peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except OSError:
        return {}


def profile_traffic(kernel_tag: str):
    """Per-launch DRAM traffic recorded from an ncu capture in profiles/ (a line
    'traffic_bytes_per_launch[<tag>]: <int>'), or None."""
    pdir = os.path.join(ROOT, "profiles")
    if not os.path.isdir(pdir):
        return None
    key = f"traffic_bytes_per_launch[{kernel_tag}]:"
    for name in sorted(os.listdir(pdir)):
        try:
            for line in open(os.path.join(pdir, name)):
                if line.strip().startswith(key):
                    return int(float(line.split(":", 1)[1].strip()))
        except (OSError, ValueError):
            continue
    return None


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML every ~10 ms."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting", 0x1: "gpu_idle"}

    def __init__(self, device_index: int):
        self.samples: list[int] = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            phys = int(vis.split(",")[device_index]) if vis else device_index
            self._h = pynvml.nvmlDeviceGetHandleByIndex(phys)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:  # no NVML: clocks unreported
            self._nv = None

    def _run(self):
        nv = self._nv
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.reasons |= int(get_reasons(self._h)) & ~0x1
            except Exception:
                pass
            time.sleep(0.01)

    def __enter__(self):
        if self._nv is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self) -> dict | None:
        if self._nv is None:
            return None
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit]
        return {"sm_mhz": float(np.median(self.samples)) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


# --------------------------------------------------------------- CPU side
def cpu_gemv_sample(seconds: float, threads: int):
    """The reference's CPU path restated (oracle): fp32 matvec of the
    pre-dequantized INT4 weights, dequantization outside the timer
    (the reference's tests/test_m4_kernels.py:157-168 oracle).
    Returns (GB/s of algorithmic INT4 bytes, sample description, gemvs run)."""
    from oracle import reference_port as port

    rng = np.random.default_rng(0)
    mats = []
    for i, (n, k) in enumerate([(I, H), (H, I), (I, H), (H, I)]):
        w = (rng.standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float32)
        q, s = port.quantize_group(w, G)
        mats.append(port.dequant_int4(port.pack_int4(q), s, k, G))
    x0 = rng.standard_normal(H).astype(np.float16).astype(np.float32)
    n_gemv = 0
    t0 = time.perf_counter()
    while True:
        x = x0
        for j in range(0, 4, 2):
            y = mats[j] @ x
            x = (mats[j + 1] @ y.astype(np.float16).astype(np.float32)).astype(np.float32)
            n_gemv += 2
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    gbs = n_gemv * BYTES_PER_GEMV / dt / 1e9
    desc = (f"{n_gemv} fp32 matvecs (2x gate {I}x{H} + 2x down {H}x{I}, dequantized outside the timer) "
            f"in {dt:.2f} s on {threads} threads")
    return gbs, desc, n_gemv


def op_suite(ops, formats, pack, device, capturable: bool, iters: int = 200) -> dict:
    """Per-call latency of the hot-path ops at the benchmark configs' shapes,
    through the given `ops` module with the same names and arguments -- this
    build's soinfer.ops, or the reference's own (its extension compiled for
    sm_100a, baseline/_ref) in the reference arm.  Inputs come from the
    module's own quantizer (bit-exact between the two), seeded identically.
    Per op: call_us, the mean of `iters` back-to-back calls on the current
    stream after 20 warm-up calls (CUDA events: the binding's host cost shows
    when it exceeds the kernel's), and device_us, the device time per call
    (see timed); the weights of one call fit in L2, as in decode."""
    gen = torch.Generator().manual_seed(0)
    cfg = formats.QuantConfig(bits=4, granularity="group", group_size=G)

    def q4(n, k):
        qt = formats.quantize(torch.randn(n, k, generator=gen) * 0.02, cfg)
        p, _ = pack.pack_int4(qt.qweight)
        return p.contiguous().to(device), qt.scale.contiguous().to(device)

    def timed(fn):
        """(call us, device us): back-to-back calls timed with CUDA events
        (includes each binding's host cost when it exceeds the kernel's), and
        the device time of one call: a CUDA graph of `iters` calls replayed
        (this build's ops launch on the current stream), or the CUPTI
        durations of the launched kernels through torch.profiler (the
        reference's ops launch on the legacy default stream, which cannot be
        captured; they use no programmatic dependent launch, so their kernel
        durations do not overlap)."""
        for _ in range(20):
            fn()
        torch.cuda.synchronize(device)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters):
            fn()
        e.record()
        torch.cuda.synchronize(device)
        call_us = s.elapsed_time(e) * 1e3 / iters
        dev_us = None
        if capturable:
            st = torch.cuda.Stream(device)
            st.wait_stream(torch.cuda.current_stream(device))
            with torch.cuda.stream(st):
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=st):
                    for _ in range(iters):
                        fn()
                graph.replay()
                s.record(st)
                graph.replay()
                e.record(st)
            torch.cuda.synchronize(device)
            dev_us = s.elapsed_time(e) * 1e3 / iters
            del graph
        else:
            try:
                from torch.autograd import DeviceType
                from torch.profiler import ProfilerActivity, profile

                n = 50
                with profile(activities=[ProfilerActivity.CUDA]) as prof:
                    for _ in range(n):
                        fn()
                    torch.cuda.synchronize(device)
                tot = 0.0
                for ev in prof.events():
                    if getattr(ev, "device_type", None) == DeviceType.CUDA:
                        tot += float(getattr(ev, "device_time", None) or getattr(ev, "cuda_time", 0.0) or 0.0)
                dev_us = tot / n if tot > 0 else None
            except Exception:  # no CUPTI here: the call time stands alone
                dev_us = None
        return call_us, dev_us

    out = {}

    def rec(name, t, nbytes):
        call_us, dev_us = t
        out[name] = {"call_us": round(call_us, 2), "device_us": round(dev_us, 2) if dev_us else None,
                     "device_gbs": round(nbytes / dev_us / 1e3, 1) if dev_us else None}

    for n, k in ((I, H), (H, I)):
        W, S = q4(n, k)
        x = torch.randn(k, generator=gen).half().to(device)
        rec(f"gemv_int4_{n}x{k}", timed(lambda: ops.gemv_w4a16_group_lop3(W, S, x, k, G)), gemv_bytes(n, k))
    for n in (I, 17408):
        a = torch.randn(n, generator=gen).abs().to(device)
        rec(f"topk_{n}_k{n // 2}", timed(lambda: ops.topk_threshold_select(a, n // 2)), n * 4 + (n // 2) * 4)
    k_sel = I // 2
    WT, ST = q4(I, H)  # down_proj_T rows
    idx = torch.sort(torch.randperm(I, generator=gen)[:k_sel]).values
    Wsel, Ssel = WT[idx.to(device)].contiguous(), ST[idx.to(device)].contiguous()
    h = torch.randn(k_sel, generator=gen).half().to(device)
    sel_bytes = k_sel * (H // 2 + (H // G) * 4) + 2 * k_sel + 2 * H
    rec(f"sparse_accumulate_{k_sel}x{H}", timed(lambda: ops.gemv_w4a16_sparse_accumulate(Wsel, Ssel, h, H, G)),
        sel_bytes)
    hot = torch.arange(0, I, 5)  # a 20% hot set
    slot_of = torch.full((I,), -1, dtype=torch.int32)
    slot_of[hot] = torch.arange(hot.numel(), dtype=torch.int32)
    idx32 = idx.to(torch.int32).to(device)
    desc, miss, mc = ops.build_dip_descriptors(idx32, slot_of.to(device))
    miss = miss[: int(mc.item())].long()
    cW, cS = WT[hot.to(device)].contiguous(), ST[hot.to(device)].contiguous()
    sW, sS = WT[miss].contiguous(), ST[miss].contiguous()
    rec(f"fused_down_20pct_{k_sel}x{H}",
        timed(lambda: ops.gemv_dip_fused_down(cW, cS, sW, sS, desc, h, H, G)), sel_bytes)
    for nq, ctx in ((16, 2048), (40, 4096)):
        q = torch.randn(nq, 128, generator=gen).half().to(device)
        kc = torch.randn(8, ctx, 128, generator=gen).half().to(device)
        vc = torch.randn(8, ctx, 128, generator=gen).half().to(device)
        rec(f"decode_attention_{nq}q8kv_ctx{ctx}", timed(lambda: ops.decode_attention(q, kc, vc, ctx)),
            2 * 8 * ctx * 128 * 2 + 2 * nq * 128 * 2)
    W8 = torch.randint(-127, 128, (5120, 5120), generator=gen, dtype=torch.int8).to(device)
    S8 = (torch.rand(5120, 1, generator=gen) * 0.01).to(device)
    x8 = torch.randn(5120, generator=gen).half().to(device)
    rec("gemv_int8_5120x5120_per_channel", timed(lambda: ops.gemv_w8a16(W8, S8, x8, 5120)),
        5120 * 5120 + 5120 * 4 + 4 * 5120)
    return out


def run_reference(args) -> None:
    """The reference arm: sparse-offload-infer's own CPU path for the
    headline op -- soinfer.quant.formats.dequantize once outside the timer,
    then fp32 torch.mv on every host core (the reference tests' oracle,
    tests/test_m4_kernels.py:157-168) -- from the reference package installed
    under baseline/_ref, or the oracle's numpy restatement when that install
    is absent.  Also times the reference's own CUDA ops (its extension built
    for sm_100a) at the benchmark configs' shapes on this GPU (config.ref_ops_b200)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    ref_root = os.path.join(ROOT, "baseline", "_ref")
    have_ref = os.path.isfile(os.path.join(ref_root, "soinfer", "quant", "formats.py"))
    per_step = []
    if have_ref:
        for p in (ROOT, os.path.join(ROOT, "sparse-offload-infer_b200")):
            while p in sys.path:
                sys.path.remove(p)
        sys.path.insert(0, ref_root)
        import soinfer  # the reference package
        from soinfer.quant import formats, pack

        assert soinfer.__file__.startswith(ref_root), soinfer.__file__
        torch.set_num_threads(threads)
        cfg = formats.QuantConfig(bits=4, granularity="group", group_size=G)
        gen = torch.Generator().manual_seed(0)
        mats = []
        for n, k in [(I, H), (H, I), (I, H), (H, I)]:
            qt = formats.quantize(torch.randn(n, k, generator=gen) * 0.02, cfg)
            mats.append(formats.dequantize(qt).float().contiguous())
        x0 = torch.randn(H, generator=gen).half().float()

        def step():
            x = x0
            for j in range(0, 4, 2):
                y = torch.mv(mats[j], x).half().float()
                x = torch.mv(mats[j + 1], y)
            return x

        kind = "reference"
        sample = (f"per step 4 fp32 torch.mv (2x gate {I}x{H} + 2x down {H}x{I}) of weights dequantized by the "
                  f"reference's soinfer.quant.formats.dequantize outside the timer, {threads} torch threads")
    else:
        from oracle import reference_port as port

        rng = np.random.default_rng(0)
        mats = []
        for n, k in [(I, H), (H, I), (I, H), (H, I)]:
            w = (rng.standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float32)
            q, s_ = port.quantize_group(w, G)
            mats.append(port.dequant_int4(port.pack_int4(q), s_, k, G))
        x0 = rng.standard_normal(H).astype(np.float16).astype(np.float32)

        def step():
            x = x0
            for j in range(0, 4, 2):
                y = (mats[j] @ x).astype(np.float16).astype(np.float32)
                x = mats[j + 1] @ y
            return x

        kind = "port"
        sample = (f"per step 4 fp32 matvecs (2x gate {I}x{H} + 2x down {H}x{I}) of pre-dequantized INT4 weights "
                  f"(oracle restatement; no reference install), numpy BLAS on {threads} threads")
    for _ in range(args.warmup):
        step()
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        per_step.append(time.perf_counter() - t0)
    total = sum(per_step)
    value = 4 * args.steps * BYTES_PER_GEMV / total / 1e9
    ref_ops = None
    if have_ref and torch.cuda.is_available() and not args.no_ref_ops:
        try:
            from soinfer import ops as ref_ops_mod

            ref_ops = op_suite(ref_ops_mod, formats, pack, torch.device("cuda", 0), capturable=False)
        except Exception as exc:  # the extension could not run here: report why, keep the CPU line
            ref_ops = {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * total / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "configs[0]: INT4 g128 GEMV gate_proj 6144x2048 + down_proj 2048x6144 "
                               "(the reference's CPU torch path)",
                   "gemvs_per_step": 4, "bytes_per_gemv": BYTES_PER_GEMV, "parallelism": "host cores",
                   "ref_ops_b200": ref_ops},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------- GPU side
def build_layers(layers: int, device, seed: int):
    """Per layer: (gate packed [I, H/2], gate scale [I, 16], down packed [H, I/2], down scale [H, 48]) on device."""
    from soinfer.quant import formats, pack

    cfg = formats.QuantConfig(bits=4, granularity="group", group_size=G)
    out = []
    gen = torch.Generator(device=device)
    for layer in range(layers):
        mats = []
        for n, k in ((I, H), (H, I)):
            gen.manual_seed(seed * 1000 + 2 * layer + (n == H))
            w = torch.randn(n, k, generator=gen, device=device) * 0.02
            qt = formats.quantize(w, cfg)
            packed, _ = pack.pack_int4(qt.qweight)
            mats += [packed.contiguous(), qt.scale.contiguous()]
            del w, qt
        out.append(tuple(mats))
    torch.cuda.synchronize(device)
    return out


def run_ours(args) -> None:
    import torch.distributed as dist

    from soinfer import _C

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    _C.lib()  # fail loudly if the CUDA library is missing

    L = args.layers
    layers = build_layers(L, device, seed=rank + 1)
    gen = torch.Generator(device=device).manual_seed(12345 + rank)
    x = (torch.randn(H, generator=gen, device=device)).half()
    xd = (torch.randn(I, generator=gen, device=device)).half()
    ys = [torch.empty(I, dtype=torch.float16, device=device) for _ in range(L)]
    outs = [torch.empty(H, dtype=torch.float16, device=device) for _ in range(L)]

    # one step: every layer copy's gate and down GEMV, independent inputs
    tasks = []
    for li, (gw, gs, dw, ds) in enumerate(layers):
        tasks.append((gw, gs, x, ys[li], H, G, -1))
        tasks.append((dw, ds, xd, outs[li], I, G, -1))
    batch = _C.GemvBatch(tasks)
    # the same stream with each down_proj consuming its gate_proj output
    chained = _C.GemvBatch([(t[0], t[1], ys[i // 2] if i % 2 else t[2], t[3], t[4], t[5], i - 1 if i % 2 else -1)
                            for i, t in enumerate(tasks)])

    # correctness spot check against the oracle (first gate, first down)
    batch.run()
    torch.cuda.synchronize(device)
    assert _C.device_errors() == 0, "device error flag set by the batched GEMV"
    from oracle import reference_port as port

    gw, gs, dw, ds = layers[0]
    for got, (w, s_, xin, k) in ((ys[0], (gw, gs, x, H)), (outs[0], (dw, ds, xd, I))):
        ref = port.gemv_w4a16(w.cpu().numpy(), s_.cpu().numpy(), xin.cpu().numpy(), k, G)
        err = float(np.abs(got.double().cpu().numpy() - ref).max())
        assert err < 1e-2 * max(1.0, float(np.abs(ref).max())), f"gemv spot check failed: max-abs {err}"

    launches_per_step = LAUNCHES_PER_STEP
    gemvs_per_step = 2 * L * launches_per_step
    bytes_per_step = gemvs_per_step * BYTES_PER_GEMV
    for _ in range(args.warmup * launches_per_step):
        batch.run()
    torch.cuda.synchronize(device)

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    with sampler:
        cur = torch.cuda.current_stream(device)
        start.record(cur)
        for _ in range(args.steps * launches_per_step):
            batch.run()
        end.record(cur)
        torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    assert _C.device_errors() == 0, "device error flag set by the batched GEMV"
    elapsed_ms = start.elapsed_time(end)
    t = torch.tensor([elapsed_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    value = world * args.steps * bytes_per_step / (max_ms / 1e3) / 1e9
    per_launch_s = (elapsed_ms / 1e3) / (args.steps * launches_per_step)
    achieved = 2 * L * BYTES_PER_GEMV / per_launch_s / 1e9

    # chained variant (reported, not the headline)
    for _ in range(2):
        chained.run()
    torch.cuda.synchronize(device)
    cs, ce = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    csteps = max(3, args.steps // 4) * launches_per_step
    cs.record(cur)
    for _ in range(csteps):
        chained.run()
    ce.record(cur)
    torch.cuda.synchronize(device)
    assert _C.device_errors() == 0, "device error flag set by the chained batched GEMV"
    chained_gbs = csteps * 2 * L * BYTES_PER_GEMV / (cs.elapsed_time(ce) / 1e3) / 1e9

    gemm_m8 = run_gemm_m8(layers, device) if args.gemm_m8 else None

    # ---- e2e through the public streaming API (weights from the pinned arena)
    e2e = run_e2e(args, layers, device, world, dist)
    del layers
    decode = run_decode(args, device) if args.decode and rank == 0 and world == 1 else None
    decode_tp = run_decode_tp(args, device, world, rank, dist) if args.tp_decode else None
    nccl_sweep = None
    if world > 1 and args.nccl_sweep:
        from soinfer.runtime.tp import PeerExchange, allreduce_sweep

        ex = PeerExchange(device=device)
        nccl_sweep = allreduce_sweep(device, exchange=ex)
        torch.cuda.synchronize(device)
        dist.barrier()
        ex.close()
    decode_int8 = run_decode_int8(args, device) if args.int8_decode and world == 1 else None
    decode_b8 = run_decode_batch8(args, device) if args.batch8_decode and world == 1 else None
    dip_blocks = run_dip_blocks(args, device) if args.dip_blocks and world == 1 else None
    ops_b200 = None
    if args.ops and world == 1:
        from soinfer import ops as our_ops
        from soinfer.quant import formats, pack

        ops_b200 = op_suite(our_ops, formats, pack, device, capturable=True)

    peaks = measured_peaks()
    peak = peaks.get("hbm_gbs")
    peak_src = "measured" if peak else "fallback"
    peak = peak or 6650.0
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        gbs, desc, _ = cpu_gemv_sample(args.cpu_seconds, threads)
        cpu = {"value": round(gbs, 3), "unit": UNIT, "cores": threads, "kind": "port", "sample": desc}
    del batch, chained
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(max_ms / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int4w-f16a-f32acc", "data": "synthetic",
        "config": {"workload": "configs[0]: INT4 g128 GEMV, gate_proj 6144x2048 + down_proj 2048x6144 per layer "
                               f"copy, {L} layer copies per launch (one soinfer_gemv_w4a16_batch call), "
                               f"{launches_per_step} launches per step",
                   "layers": L, "launches_per_step": launches_per_step, "gemvs_per_step": gemvs_per_step,
                   "bytes_per_gemv": BYTES_PER_GEMV,
                   "weights_bytes": L * 2 * (I * H // 2),
                   "l2": "inputs larger than L2 (weights far above the 126 MB L2), no flush",
                   "chained_gate_down": {"value": round(chained_gbs, 2), "unit": UNIT, "launches": csteps,
                                         "note": "each down_proj reads its gate_proj output (in-kernel dependency; "
                                                 "streaming kernel: gate units first, each down unit waits for its "
                                                 "gate's completion count)"},
                   "gemm_m8": gemm_m8,
                   "decode": decode,
                   "decode_14b_tp": decode_tp,
                   "allreduce_sweep": nccl_sweep,
                   "decode_14b_int8": decode_int8,
                   "decode_14b_batch8": decode_b8,
                   "dip_blocks": dip_blocks,
                   "ops_b200": ops_b200,
                   "parallelism": f"{world} independent replicas (no collective)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": UNIT,
                     "frac": round(achieved / peak, 4), "peak_source": peak_src,
                     "traffic": profile_traffic("gemv_stream_kernel"),
                     "kernel": "gemv_stream_kernel (one launch = 128 INT4 g128 GEMVs; achieved = bytes per launch / "
                               "mean launch time)"},
        "e2e": e2e,
        "gpu_launches": args.steps * launches_per_step,
        "clocks": sampler.summary(),
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)


def run_gemm_m8(layers, device, reps: int = 40) -> dict:
    """configs[4]'s batch-8 variant on the headline stream: the same 64 layer
    copies x (gate, down), each matrix multiplying 8 token rows, all 128
    matrices in ONE launch (soinfer_gemm_w4a16_batch: the streaming kernel
    with the 8 tokens in the MMA columns); the older per-matrix kernel
    (soinfer_gemm_w4a16, 128 launches in one CUDA graph) is reported beside it."""
    from soinfer import _C

    M = 8
    gen = torch.Generator(device=device).manual_seed(99)
    Xg = torch.randn(M, H, generator=gen, device=device).half()
    Xd = torch.randn(M, I, generator=gen, device=device).half()
    Yg = [torch.empty(M, I, dtype=torch.float16, device=device) for _ in layers]
    Yd = [torch.empty(M, H, dtype=torch.float16, device=device) for _ in layers]
    L = len(layers)
    w_bytes = 2 * L * (I * H // 2 + I * H // 128 * 4)
    act_bytes = L * M * 2 * (H + I) * 2
    tasks = []
    for li, (gw, gs, dw, ds) in enumerate(layers):
        tasks += [(gw, gs, Xg, Yg[li], H, G), (dw, ds, Xd, Yd[li], I, G)]
    batch = _C.GemmBatch(tasks)
    for _ in range(3):
        batch.run()
    torch.cuda.synchronize(device)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        batch.run()
    e.record()
    torch.cuda.synchronize(device)
    assert _C.device_errors() == 0, "device error flag set by the batched multi-token GEMM"
    ms = s.elapsed_time(e) / reps
    # spot check: one token row of the first gate against the single-matrix kernel
    ref = _C.gemm_w4a16(layers[0][0], layers[0][1], Xg, H, G)
    assert (Yg[0].float() - ref.float()).abs().max().item() < 1e-2 * max(1.0, ref.float().abs().max().item())

    def step_old():
        for li, (gw, gs, dw, ds) in enumerate(layers):
            _C.gemm_w4a16(gw, gs, Xg, H, G, out=Yg[li])
            _C.gemm_w4a16(dw, ds, Xd, I, G, out=Yd[li])

    st = torch.cuda.Stream(device)
    st.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(st):
        step_old()
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            step_old()
        for _ in range(3):
            graph.replay()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record(st)
        for _ in range(20):
            graph.replay()
        e2.record(st)
    torch.cuda.synchronize(device)
    ms_old = s2.elapsed_time(e2) / 20
    del graph
    return {"m": M, "value": round((w_bytes + act_bytes) / (ms / 1e3) / 1e9, 2), "unit": UNIT,
            "ms_per_launch": round(ms, 4), "gemms_per_launch": 2 * L,
            "token_gemvs_per_s": round(2 * L * M / (ms / 1e3), 1),
            "per_matrix_kernel": {"value": round((w_bytes + act_bytes) / (ms_old / 1e3) / 1e9, 2), "unit": UNIT,
                                  "ms_per_step": round(ms_old, 4),
                                  "note": "soinfer_gemm_w4a16, one launch per matrix, 128 launches in a CUDA graph"},
            "note": "one soinfer_gemm_w4a16_batch launch = 128 matrices x 8 tokens (streaming kernel, tokens in "
                    "the mma.sync columns)"}


def run_e2e(args, layers, device, world, dist) -> dict:
    from soinfer.offload.load_hf_checkpoint import LoadedMatrix
    from soinfer.offload.weight_store import PinnedWeightStore
    from soinfer.runtime.generate import StreamingModel, WeightPipeline

    L = len(layers)
    total = sum(t[0].numel() + t[2].numel() for t in layers)
    store = PinnedWeightStore(total)
    matrices = {}
    for li, (gw, gs, dw, ds) in enumerate(layers):
        for suffix, w, s, n, k in (("mlp.gate_proj.weight", gw, gs, I, H), ("mlp.down_proj.weight", dw, ds, H, I)):
            name = f"model.layers.{li}.{suffix}"
            matrices[name] = LoadedMatrix(store.register(name, w.cpu()), s, k, n, k)
    torch.cuda.synchronize(device)
    model = StreamingModel(store=store, matrices=matrices, num_layers=L, embed_tokens=None, lm_head=None,
                           final_norm=None, layer_norms=[], hidden_size=H, num_attention_heads=16,
                           num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-6, rope_theta=1e6, group_size=G)
    pipe = WeightPipeline(model, suffixes=("mlp.gate_proj.weight", "mlp.down_proj.weight"))
    x_host = torch.randn(H, generator=torch.Generator().manual_seed(7)).half().pin_memory()
    out_host = torch.empty(H, dtype=torch.float16).pin_memory()
    x_dev = torch.empty(H, dtype=torch.float16, device=device)

    def e2e_step():
        x_dev.copy_(x_host, non_blocking=True)
        o = None
        for _ in range(L):
            y = pipe.next_gemv(x_dev)
            o = pipe.next_gemv(y)
        out_host.copy_(o, non_blocking=True)

    steps = max(3, min(args.steps, args.e2e_steps))
    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    cur = torch.cuda.current_stream(device)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(cur)
    for _ in range(steps):
        e2e_step()
    e.record(cur)
    torch.cuda.synchronize(device)
    ms = s.elapsed_time(e)
    t = torch.tensor([ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    h2d = 2 * L * (I * H // 2) + 2 * H
    value = world * steps * 2 * L * BYTES_PER_GEMV / (ms / 1e3) / 1e9
    return {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 2 * H,
            "steps": steps, "ms_per_step": round(ms / steps, 3), "h2d_gbs": round(world * steps * h2d / (ms / 1e3) / 1e9, 2),
            "path": "soinfer.runtime.generate.WeightPipeline (copy-engine double buffering from the pinned arena)"}


def zipf_hot_set(I: int, frac: float, seed: int = 0):
    """configs[2]'s hot channel set: a Zipf(s=1.1) frequency ranking over a
    seeded permutation of the I channels, the top round(frac * I) kept by the
    reference's StaticFrequencyPolicy."""
    from soinfer.offload.hot_cache import StaticFrequencyPolicy

    rng = np.random.default_rng(seed)
    freq = np.empty(I, dtype=np.int64)
    freq[rng.permutation(I)] = (1e9 / np.arange(1, I + 1) ** 1.1).astype(np.int64)
    return StaticFrequencyPolicy(freq, round(frac * I)).hot_list


def run_decode(args, device) -> dict:
    """batch-1 greedy decode of the Qwen3-1.7B-shaped INT4 model
    (random-init weights), 70 random prompt tokens then args.decode_tokens new
    tokens.  Resident variants, one CUDA graph per token (GraphDecoder): dense,
    DIP k/I = 0.5, and cache-aware DIP k/I = 0.5 with a 20% Zipf hot cache in
    HBM and the other up_proj / down_proj_T rows read from the pinned arena by
    the device (zero-copy over PCIe) -- its tokens must equal DIP's.  Offload
    variant: streamed dense (every matrix copied from the pinned arena by the
    copy engine each token, double-buffered: WeightPipeline, eager).  tok/s
    counts the generating steps only (prompt timed apart)."""
    import copy

    from soinfer.offload.hot_cache import HotCache
    from soinfer.runtime import generate as gen
    from soinfer.runtime.loader import QWEN3_1_7B, synthetic_streaming_model

    arch = QWEN3_1_7B
    model = synthetic_streaming_model(arch, seed=1, resident=True, offload=True, include_dip=True, device=device)
    prompt = torch.randint(0, arch.vocab_size, (70,), generator=torch.Generator().manual_seed(0)).tolist()
    n_new = args.decode_tokens
    peak = pcie_h2d_peak(device)
    out = {"model": "Qwen3-1.7B-shaped: 28 layers, hidden 2048, intermediate 6144, 16 q / 8 kv heads, head_dim 128, "
                    "vocab 151936; INT4 g128 random-init weights",
           "prompt_tokens": len(prompt), "new_tokens": n_new, "max_seq_len": 2048,
           "step": "one CUDA graph per token (soinfer.runtime.generate.GraphDecoder)",
           "pcie_h2d_peak_gbs": round(peak, 2)}
    toks = {}
    for name, dip_k in (("dense", None), ("dip_k3072", 3072)):
        gd = gen.GraphDecoder(model, dip_k=dip_k, max_seq_len=2048)
        gd.generate(prompt, 4)  # capture + warm-up
        tm = {}
        toks[name] = gd.generate(prompt, n_new, timings=tm)
        n = n_new - 1
        out[name] = {"tok_s": round(n / (tm["decode_ms"] / 1e3), 1), "ms_per_token": round(tm["decode_ms"] / n, 4),
                     "prefill_ms": round(tm["prefill_ms"], 2)}
        del gd
    # the dense step as one cooperative kernel for all layers (same bits, same tokens)
    gd = gen.GraphDecoder(model, max_seq_len=2048, fused=True)
    gd.generate(prompt, 4)
    tm = {}
    ids_f = gd.generate(prompt, n_new, timings=tm)
    n = n_new - 1
    out["dense_fused"] = {"tok_s": round(n / (tm["decode_ms"] / 1e3), 1), "ms_per_token": round(tm["decode_ms"] / n, 4),
                          "prefill_ms": round(tm["prefill_ms"], 2), "tokens_equal_dense": ids_f == toks["dense"],
                          "note": "one CUDA graph per token whose decoder layers are ONE cooperative kernel "
                                  "(soinfer_decode_layers_fused: grid barriers between phases, each phase's weights "
                                  "bulk-copied into shared memory a phase ahead)"}
    assert ids_f == toks["dense"], "fused decode tokens differ from the per-kernel step's"
    del gd
    # cache-aware DIP: 20% hot cache resident, misses from the pinned arena
    hot = zipf_hot_set(arch.intermediate_size, 0.2)
    caches = [HotCache.build(model, li, hot) for li in range(arch.num_layers)]
    host = copy.copy(model)
    host.resident = {n_: t for n_, t in model.resident.items()
                     if not (n_.endswith("mlp.up_proj.weight") or n_.endswith(gen.DOWN_PROJ_T_SUFFIX))}
    gd = gen.GraphDecoder(host, dip_k=3072, max_seq_len=2048, caches=caches)
    gd.generate(prompt, 4)
    tm = {}
    ids = gd.generate(prompt, n_new, timings=tm)
    misses = gd.miss_counts.sum().item()  # over every replay of this generate (prompt + new tokens)
    steps = len(prompt) + n_new - 1
    h2d_per_token = misses / steps * gen.miss_row_bytes(host)
    n = n_new - 1
    ms_tok = tm["decode_ms"] / n
    out["cached_dip_k3072"] = {
        "tok_s": round(n / (tm["decode_ms"] / 1e3), 1), "ms_per_token": round(ms_tok, 4),
        "prefill_ms": round(tm["prefill_ms"], 2), "hot_channels": len(hot),
        "tokens_equal_dip": ids == toks["dip_k3072"],
        "h2d_bytes_per_token": int(h2d_per_token), "h2d_gbs": round(h2d_per_token / (ms_tok / 1e3) / 1e9, 2),
        "h2d_frac_of_peak": round(h2d_per_token / (ms_tok / 1e3) / 1e9 / peak, 4),
        "note": "one CUDA graph per token: descriptors, miss gather (zero-copy from the pinned arena, count read on "
                "the device) and fused cache-or-stream GEMVs; 20% Zipf(1.1) hot set"}
    assert ids == toks["dip_k3072"], "cache-aware DIP tokens differ from DIP's"
    del gd, caches, host
    # offload-streamed dense: every matrix from the pinned arena each token
    streamed = copy.copy(model)
    streamed.resident = {}
    ns = min(n_new, 24)
    s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ids_s = gen.generate_streaming(streamed, prompt[:8], 2, max_seq_len=64)  # warm-up
    s_.record()
    ids_s = gen.generate_streaming(streamed, prompt[:1], ns, max_seq_len=64)
    e_.record()
    torch.cuda.synchronize(device)
    wbytes = sum(m.n * m.handle.row_nbytes for nm, m in model.matrices.items()
                 if not nm.endswith(gen.DOWN_PROJ_T_SUFFIX))
    ms_tok = s_.elapsed_time(e_) / (ns + 1)  # 1 prompt step + ns generating steps
    out["streamed_dense"] = {"tok_s": round(1e3 / ms_tok, 1), "ms_per_token": round(ms_tok, 3),
                             "tokens": ns, "h2d_bytes_per_token": int(wbytes),
                             "h2d_gbs": round(wbytes / (ms_tok / 1e3) / 1e9, 2),
                             "h2d_frac_of_peak": round(wbytes / (ms_tok / 1e3) / 1e9 / peak, 4),
                             "note": "eager; each matrix copied by the copy engine on a side stream, double "
                                     "buffered (WeightPipeline); 1-token prompt, timed over every step"}
    assert ids_s[:1] == prompt[:1]
    del model, streamed
    torch.cuda.empty_cache()
    return out


def run_decode_batch8(args, device) -> dict:
    """configs[4] at batch 8: the Qwen3-14B-shaped INT4 model on one GPU,
    8 random prompts of args.tp_prompt tokens decoded together, then
    args.tp_tokens new tokens each (4096 context), one CUDA graph per step
    (soinfer.runtime.batch.BatchDecoder: multi-token INT4 GEMMs, one attention
    launch over the 8 stacked caches).  tok/s counts every sequence's tokens."""
    from soinfer.runtime.batch import BatchDecoder
    from soinfer.runtime.loader import QWEN3_14B, synthetic_streaming_model

    arch, B = QWEN3_14B, 8
    model = synthetic_streaming_model(arch, seed=2, resident=True, offload=False, include_dip=False, device=device)
    g = torch.Generator().manual_seed(3)
    prompts = torch.randint(0, arch.vocab_size, (B, args.tp_prompt), generator=g).tolist()
    bd = BatchDecoder(model, B, max_seq_len=4096)
    bd.generate([p[:8] for p in prompts], 4)  # capture + warm-up
    tm = {}
    out = bd.generate(prompts, args.tp_tokens, timings=tm)
    n = args.tp_tokens - 1
    weight_bytes = sum(t.numel() for t in model.resident.values()) + sum(
        m.scale.numel() * m.scale.element_size() for m in model.matrices.values())
    kv_per_pos = 2 * arch.num_key_value_heads * arch.head_dim * 2 * arch.num_layers
    step_bytes = weight_bytes + arch.vocab_size * arch.hidden_size * 2 + B * kv_per_pos * (
        args.tp_prompt + args.tp_tokens / 2)
    ms_step = tm["decode_ms"] / n
    del bd, model
    torch.cuda.empty_cache()
    return {"model": "Qwen3-14B-shaped, INT4 g128, resident; batch 8", "batch": B, "prompt_tokens": args.tp_prompt,
            "new_tokens": args.tp_tokens, "tok_s": round(B * n / (tm["decode_ms"] / 1e3), 1),
            "ms_per_step": round(ms_step, 4), "prefill_ms": round(tm["prefill_ms"], 1),
            "hbm_bytes_per_step": int(step_bytes),
            "hbm_floor_ms": round(step_bytes / (measured_peaks().get("hbm_gbs") or 6650.0) / 1e6, 4),
            "distinct_sequences": len({tuple(o) for o in out}),
            "step": "one CUDA graph per step: per layer rmsnorm, q/k/v/o/gate/up/down as multi-token INT4 GEMMs "
                    "(soinfer_gemm_w4a16), one head-norm+RoPE+append and one attention launch for the 8 stacked "
                    "caches, SwiGLU; fp16 LM head as a cuBLAS GEMM"}


def run_decode_tp(args, device, world, rank, dist) -> dict:
    """batch-1 greedy decode of the Qwen3-14B-shaped INT4 model,
    tensor-parallel over the `world` GPUs (one process each; q/k/v/gate/up
    split by output rows, o/down by input columns with one NCCL all-reduce
    after each, vocabulary-parallel LM head); world 1 runs the unsharded
    model.  A random prompt of args.tp_prompt tokens fills the KV cache, then
    args.tp_tokens tokens are generated, one CUDA graph per token (collectives
    captured in it).  ms/token is the max over ranks of the CUDA-event time."""
    from soinfer.runtime import generate as gen
    from soinfer.runtime.loader import QWEN3_14B, synthetic_streaming_model
    from soinfer.runtime.tp import PeerExchange, ShardPlan, build_tp_model, graph_decoder_tp

    arch = QWEN3_14B
    max_seq = 4096
    n_prompt, n_new = args.tp_prompt, args.tp_tokens
    if n_prompt + n_new > max_seq:
        raise ValueError("tp prompt + tokens must fit the 4096 context")
    exchange = None
    if world == 1:
        model = synthetic_streaming_model(arch, seed=2, resident=True, offload=False, include_dip=False,
                                          device=device)
        gd = gen.GraphDecoder(model, max_seq_len=max_seq)
    else:
        plan = ShardPlan(rank, world, arch.num_attention_heads, arch.num_key_value_heads, arch.head_dim,
                         arch.hidden_size, arch.intermediate_size, arch.vocab_size)
        model = build_tp_model(arch, plan, seed=2, device=device)
        if not args.tp_nccl:
            exchange = PeerExchange(device=device)
        gd = graph_decoder_tp(model, plan, max_seq_len=max_seq, exchange=exchange)
    weight_bytes = sum(t.numel() for t in model.resident.values()) + sum(
        m.scale.numel() * m.scale.element_size() for m in model.matrices.values())
    prompt = torch.randint(0, arch.vocab_size, (n_prompt,), generator=torch.Generator().manual_seed(1)).tolist()
    gd.generate(prompt[:8], 4)  # capture + warm-up
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    tm = {}
    ids = gd.generate(prompt, n_new, timings=tm)
    t = torch.tensor([tm["decode_ms"], tm["prefill_ms"]], dtype=torch.float64, device=device)
    same = torch.tensor(ids[-n_new:], dtype=torch.int64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ref = same.clone()
        dist.broadcast(ref, 0)
        agree = bool(torch.equal(ref, same))
    else:
        agree = True
    decode_ms, prefill_ms = (float(v) for v in t.tolist())
    del gd
    if exchange is not None:
        from soinfer import _C

        assert _C.device_errors() == 0, "device error bits set during TP decode (peer exchange)"
        exchange.close()
    del model
    torch.cuda.empty_cache()
    n = n_new - 1
    ms_tok = decode_ms / n
    # per-token HBM floor of one rank: its weight shard + LM-head shard + KV read at the mean context
    kv_per_pos = 2 * (arch.num_key_value_heads // world) * arch.head_dim * 2 * arch.num_layers
    mean_ctx = n_prompt + n_new / 2
    lm_bytes = -(-arch.vocab_size // world) * arch.hidden_size * 2
    rank_bytes = weight_bytes + lm_bytes + kv_per_pos * mean_ctx
    return {"model": "Qwen3-14B-shaped: 40 layers, hidden 5120, intermediate 17408, 40 q / 8 kv heads, head_dim 128, "
                     "vocab 151936; INT4 g128 random-init weights resident in HBM",
            "tp": world, "prompt_tokens": n_prompt, "new_tokens": n_new, "max_seq_len": max_seq,
            "tok_s": round(n / (decode_ms / 1e3), 1), "ms_per_token": round(ms_tok, 4),
            "prefill_ms": round(prefill_ms, 1), "tokens_agree_across_ranks": agree,
            "hbm_bytes_per_token_per_rank": int(rank_bytes),
            "hbm_floor_ms": round(rank_bytes / (measured_peaks().get("hbm_gbs") or 6650.0) / 1e6, 4),
            "collectives_per_token": 2 * arch.num_layers + 1,
            "step": "one CUDA graph per token; " + (
                "NCCL fp32 all-reduce of the o / down partials" if world > 1 and args.tp_nccl else
                "row-parallel GEMV stores its rows into every rank's inbox over NVLink, one exchange kernel "
                "sums + residual + RMSNorm (soinfer.runtime.tp.PeerExchange)" if world > 1 else "single GPU")}


def pcie_h2d_peak(device, reps: int = 3) -> float:
    """Pinned host -> device copy bandwidth (GB/s): the best over copy sizes
    (64 MB, 256 MB, 1 GB) and over 1 or 2 copies in flight on separate
    streams (each of the two moving half of the bytes), best of `reps`."""
    best = 0.0
    big = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    dst = torch.empty(1 << 30, dtype=torch.uint8, device=device)
    streams = [torch.cuda.Stream(device) for _ in range(2)]
    for nbytes in (64 << 20, 256 << 20, 1 << 30):
        for ways in (1, 2):
            part = nbytes // ways
            for _ in range(reps + 1):
                torch.cuda.synchronize(device)
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                cur = torch.cuda.current_stream(device)
                s.record(cur)
                for w in range(ways):
                    streams[w].wait_stream(cur)
                    with torch.cuda.stream(streams[w]):
                        dst[w * part:(w + 1) * part].copy_(big[w * part:(w + 1) * part], non_blocking=True)
                for w in range(ways):
                    cur.wait_stream(streams[w])
                e.record(cur)
                torch.cuda.synchronize(device)
                best = max(best, nbytes / (s.elapsed_time(e) / 1e3) / 1e9)
    del big, dst
    return best


def run_dip_blocks(args, device, reps: int = 20) -> dict:
    """configs[1] and configs[2] on the Qwen3-1.7B MLP shapes (H 2048, I 6144,
    k = I/2), 28 layer copies per step (weights far above L2):
    * DIP block: gate GEMV, |gate| top-k, up_proj on the selected rows,
      SwiGLU, down_proj_T sparse accumulate -- all on the device, one CUDA
      graph per step; algorithmic bytes per block 13,443,072;
    * cache-aware DIP block: 20% hot cache (Zipf s=1.1 ranking over a seeded
      permutation), the misses' rows streamed from the pinned arena by the
      device-driven gather (the miss count stays on the device: one CUDA
      graph per step); H2D bytes = misses x (up + down_T row bytes), against
      the measured pinned H2D peak."""
    import copy

    from soinfer import ops
    from soinfer.offload.hot_cache import HotCache, StaticFrequencyPolicy
    from soinfer.runtime import generate as gen
    from soinfer.runtime.loader import QWEN3_1_7B, synthetic_streaming_model

    arch = QWEN3_1_7B
    L, Hh, Ii = arch.num_layers, arch.hidden_size, arch.intermediate_size
    k = Ii // 2
    model = synthetic_streaming_model(arch, seed=3, resident=True, offload=True, include_dip=True, device=device)
    g = model.group_size
    gen_x = torch.Generator(device=device).manual_seed(17)
    h3 = [torch.randn(Hh, generator=gen_x, device=device).half() for _ in range(L)]
    bufs = gen.DipBuffers.make(model, k)
    outs = [None] * L

    def gate_and_select(li):
        m = model.matrix(li, "mlp.gate_proj.weight")
        gate = ops.gemv_w4a16_group_lop3(model.resident[m.handle.name], m.scale, h3[li], m.packed_k, g)
        return gate, ops.topk_threshold_select_abs(gate, k)

    def dip_step():
        for li in range(L):
            gate, idx = gate_and_select(li)
            outs[li] = gen.dip_mlp_tail(model, li, h3[li], gate, idx, k, bufs)

    st = torch.cuda.Stream(device)
    st.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(st):
        dip_step()
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            dip_step()
        for _ in range(3):
            graph.replay()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(st)
        for _ in range(reps):
            graph.replay()
        e.record(st)
    torch.cuda.synchronize(device)
    dip_ms = s.elapsed_time(e) / reps
    ref = [o.clone() for o in outs]
    del graph
    block_bytes = 13_443_072

    # cache-aware DIP: hot rows resident, misses from the pinned arena (device-side miss count)
    hot = zipf_hot_set(Ii, 0.2)
    caches = [HotCache.build(model, li, hot) for li in range(L)]
    host_model = copy.copy(model)  # same matrices; up / down_T rows read from the arena
    host_model.resident = {n: t for n, t in model.resident.items()
                           if not (n.endswith("mlp.up_proj.weight") or n.endswith(gen.DOWN_PROJ_T_SUFFIX))}
    misses = torch.zeros(L, dtype=torch.int64, device=device)

    def cached_step():
        for li in range(L):
            gate, idx = gate_and_select(li)
            outs[li] = gen.cached_dip_mlp_tail(host_model, li, h3[li], gate, idx, bufs, caches[li], misses)

    creps = 10
    with torch.cuda.stream(st):
        cached_step()
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            cached_step()
        for _ in range(2):
            graph.replay()
        torch.cuda.synchronize(device)
        misses.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(st)
        for _ in range(creps):
            graph.replay()
        e.record(st)
    torch.cuda.synchronize(device)
    cached_ms = s.elapsed_time(e) / creps
    identical = all(torch.equal(a, b) for a, b in zip(outs, ref))
    assert identical, "cache-aware DIP differs from DIP"
    miss_bytes = int(misses.sum().item()) * gen.miss_row_bytes(host_model) / creps
    peak = pcie_h2d_peak(device)
    del graph, model, host_model, caches, bufs
    torch.cuda.empty_cache()
    return {"shapes": "Qwen3-1.7B MLP: H 2048, I 6144, k 3072, INT4 g128; 28 layer copies per step",
            "dip_block": {"us_per_block": round(dip_ms * 1e3 / L, 2),
                          "value": round(L * block_bytes / (dip_ms / 1e3) / 1e9, 1), "unit": UNIT,
                          "bytes_per_block": block_bytes, "steps": reps,
                          "note": "CUDA graph per step; the fraction of HBM peak is value / roofline.peak"},
            "cached_dip_block": {"us_per_block": round(cached_ms * 1e3 / L, 2), "hot_channels": len(hot),
                                 "h2d_bytes_per_block": int(miss_bytes / L),
                                 "h2d_gbs": round(miss_bytes / (cached_ms / 1e3) / 1e9, 2),
                                 "pcie_h2d_peak_gbs": round(peak, 2),
                                 "h2d_frac_of_peak": round(miss_bytes / (cached_ms / 1e3) / 1e9 / peak, 4),
                                 "bit_identical_to_dip": identical, "layers_compared": L, "steps": creps,
                                 "note": "CUDA graph per step (the miss count never leaves the device); misses "
                                         "gathered zero-copy over PCIe from the pinned arena by one device gather "
                                         "per block; all 28 block outputs of the last replay equal DIP's"}}


def run_decode_int8(args, device) -> dict:
    """configs[4]'s INT8 per-channel variant: the 14B-shaped model with int8
    rows and one fp32 scale per row (the reference's gemv_w8a16 per GEMV),
    batch-1 greedy decode on one GPU, same prompt / token counts as the TP run."""
    from soinfer.runtime import generate as gen
    from soinfer.runtime.loader import QWEN3_14B, synthetic_streaming_model

    arch = QWEN3_14B
    model = synthetic_streaming_model(arch, seed=2, resident=True, offload=False, include_dip=False, device=device,
                                      bits=8)
    weight_bytes = sum(t.numel() for t in model.resident.values()) + sum(
        m.scale.numel() * 4 for m in model.matrices.values())
    gd = gen.GraphDecoder(model, max_seq_len=4096)
    prompt = torch.randint(0, arch.vocab_size, (args.tp_prompt,), generator=torch.Generator().manual_seed(1)).tolist()
    gd.generate(prompt[:8], 4)
    tm = {}
    gd.generate(prompt, args.tp_tokens, timings=tm)
    del gd, model
    torch.cuda.empty_cache()
    n = args.tp_tokens - 1
    ms = tm["decode_ms"] / n
    kv = 2 * arch.num_key_value_heads * arch.head_dim * 2 * arch.num_layers * (args.tp_prompt + args.tp_tokens / 2)
    floor_bytes = weight_bytes + arch.vocab_size * arch.hidden_size * 2 + kv
    return {"model": "Qwen3-14B-shaped, INT8 per-channel weights (int8 rows + fp32 row scale), resident in HBM",
            "prompt_tokens": args.tp_prompt, "new_tokens": args.tp_tokens, "tok_s": round(n / (tm["decode_ms"] / 1e3), 1),
            "ms_per_token": round(ms, 4), "weight_bytes": int(weight_bytes),
            "hbm_floor_ms": round(floor_bytes / (measured_peaks().get("hbm_gbs") or 6650.0) / 1e6, 4)}


def decode_trace(args) -> None:
    """--decode-trace: where one graph-replayed decode step's time goes
    (Qwen3-1.7B-shaped, resident INT4, 70-token prompt then 40 tokens):
    CUPTI kernel records of 5 replays (torch.profiler), per kernel name its
    launches, mean duration and its increment of the step's end time (kernels
    launched as programmatic dependents overlap, so durations overstate);
    for the per-kernel, fused and DIP steps.  Prints a table; no JSON line."""
    from torch.profiler import ProfilerActivity, profile

    from soinfer.runtime import generate as gen
    from soinfer.runtime.loader import QWEN3_1_7B, synthetic_streaming_model

    device = torch.device("cuda", 0)
    model = synthetic_streaming_model(QWEN3_1_7B, seed=1, resident=True, offload=False, include_dip=True,
                                      device=device)
    prompt = torch.randint(0, QWEN3_1_7B.vocab_size, (70,), generator=torch.Generator().manual_seed(0)).tolist()
    for name, dip_k, fused in (("per-kernel dense", None, False), ("fused dense", None, True),
                               ("per-kernel DIP k/I=0.5", 3072, False)):
        gd = gen.GraphDecoder(model, dip_k=dip_k, max_seq_len=2048, fused=fused)
        tm = {}
        gd.generate(prompt, 40, timings=tm)
        reps = 5
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            with torch.cuda.stream(gd.stream):
                for _ in range(reps):
                    gd.graph.replay()
            torch.cuda.synchronize(device)
        ev = sorted((e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA),
                    key=lambda e: e.time_range.start)
        span = (ev[-1].time_range.end - ev[0].time_range.start) / reps
        agg, prev_end = {}, ev[0].time_range.start
        for e in ev:
            k = e.name.replace("(anonymous namespace)::", "").replace("void ", "").replace("soinfer::", "")
            k = k.split("(")[0][:56]
            a = agg.setdefault(k, [0, 0.0, 0.0])
            a[0] += 1
            a[1] += e.time_range.elapsed_us()
            a[2] += max(0.0, e.time_range.end - prev_end)
            prev_end = max(prev_end, e.time_range.end)
        print(f"== {name}: {tm['decode_ms'] / 39:.4f} ms/token (CUDA events); traced {span:.1f} us/step, "
              f"{len(ev) // reps} kernels/step")
        print(f"   {'increment us/step':>18s} {'launches/step':>14s} {'mean us':>8s}  kernel")
        for k, (n, t, c) in sorted(agg.items(), key=lambda kv: -kv[1][2])[:10]:
            print(f"   {c / reps:18.1f} {n // reps:14d} {t / n:8.2f}  {k}")
        del gd


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=64)
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ref-ops", action="store_true", help="reference arm: skip timing its CUDA ops")
    ap.add_argument("--nccl-sweep", type=int, default=1,
                    help="N>1: NCCL all-reduce latency / bus bandwidth sweep (10 KB .. 1 GiB) and the peer exchange")
    ap.add_argument("--ops", type=int, default=1, help="also time this build's hot-path ops (config.ops_b200)")
    ap.add_argument("--decode", type=int, default=1, help="also measure configs[3] decode tok/s (reported in config)")
    ap.add_argument("--decode-tokens", type=int, default=128)
    ap.add_argument("--tp-decode", type=int, default=1, help="also measure configs[4] 14B TP decode (in config)")
    ap.add_argument("--gemm-m8", type=int, default=1, help="also measure the batch-8 GEMM stream (in config)")
    ap.add_argument("--batch8-decode", type=int, default=1, help="also measure configs[4] batch-8 14B decode (N=1)")
    ap.add_argument("--decode-trace", action="store_true", help="print where a 1.7B decode step's time goes and exit")
    ap.add_argument("--int8-decode", type=int, default=1, help="also measure the 14B INT8 per-channel decode (N=1)")
    ap.add_argument("--dip-blocks", type=int, default=1, help="also measure configs[1] / configs[2] blocks (N=1)")
    ap.add_argument("--tp-prompt", type=int, default=3840)
    ap.add_argument("--tp-tokens", type=int, default=256)
    ap.add_argument("--tp-nccl", type=int, default=0, help="TP collectives through NCCL instead of the peer exchange")
    args = ap.parse_args()
    if args.decode_trace:
        decode_trace(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
