#!/usr/bin/env python
"""Benchmark of the grouped MoE-LoRA expert layer, forward + backward, on B200s (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl meep2b|reference] [--config qwen3_30b|...]

A step is one forward + backward of the routed layer (routing, gather, gate/up with SwiGLU, down, un-permute and
the whole backward, adapters' gradients included) over one batch of T tokens of BASELINE config 2 (Qwen3-30B-A3B:
T=16384, hidden 2048, moe_intermediate 768, 128 experts, top-8, LoRA r=16 alpha 32, bf16). Synthetic seeded data
(router logits ~N(0,1), stacks ~N(0,0.02)); every per-step tensor is far larger than the 126 MB L2, so no flush.
At N>1 each rank runs its own batch (weak scaling) and the LoRA gradients are averaged with NCCL all-reduces
(the reference's DDP exchange). Rank 0 prints one JSON line.

Beside the library's own numbers the line carries two baselines, both the reference's path restated with PyTorch
operations (reference_routed_forward below, meepsquared/_moe.py:48-126 on its non-kernel branch):
  gpu_baseline  that path on the same GPU in bf16: what the reference runs on a compute capability 10.0 GPU, where
                its Triton kernel is not chosen (_grouped.wanted, _grouped.py:57-67) and the products are PyTorch's
                grouped matmuls;
  cpu_baseline  that path on the host cores in float32 (the reference's CPU path), rank 0 at N=1 only.
--impl reference times the same CPU path alone (rank 0), with the same config, metric and unit.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    "qwen3_30b": dict(tokens=16384, hidden=2048, inter=768, experts=128, top_k=8, rank=16, alpha=32),
    "mixtral": dict(tokens=8192, hidden=4096, inter=14336, experts=8, top_k=2, rank=16, alpha=32),
    "qwen3_30b_nf4": dict(tokens=16384, hidden=2048, inter=768, experts=128, top_k=8, rank=16, alpha=32, quant="nf4"),
    "qwen3_235b_fp8": dict(tokens=32768, hidden=4096, inter=1536, experts=128, top_k=8, rank=16, alpha=32, zipf=1.1,
                           quant="fp8_block128"),
    "small": dict(tokens=2048, hidden=2048, inter=768, experts=128, top_k=8, rank=16, alpha=32),
    "small_fp8": dict(tokens=2048, hidden=2048, inter=768, experts=128, top_k=8, rank=16, alpha=32,
                      quant="fp8_block128"),
    "small_nf4": dict(tokens=2048, hidden=2048, inter=768, experts=128, top_k=8, rank=16, alpha=32, quant="nf4"),
    "half": dict(tokens=8192, hidden=2048, inter=768, experts=128, top_k=8, rank=16, alpha=32),
    # a whole Qwen3-30B-A3B-shaped model (its decoder layers at the real sizes, fewer of them, a smaller vocabulary):
    # the model-level step with the routed layer installed on every experts module (meepsquared_b200.model)
    "qwen3_30b_model": dict(tokens=16384, hidden=2048, inter=768, experts=128, top_k=8, rank=16, alpha=32,
                            model=True, layers=4, seq=4096, vocab=16384, heads=32, kv_heads=4, head_dim=128),
}
METRIC = "MoE-LoRA layer fwd+bwd tokens/s"
# DRAM bytes (read + write) per grouped-product launch at config 2, averaged over the step's four launches: from an
# ncu capture of the four products at the full config-2 size (dram__bytes_read.sum + dram__bytes_write.sum).
GEMM_TRAFFIC_BYTES_PER_LAUNCH = 1.643e9


def flop_per_token(c):
    """k [12 H I + 6 r (2H + 3I)]: frozen base forward + input gradient, LoRA forward, input gradient and dA/dB."""
    return c["top_k"] * (12 * c["hidden"] * c["inter"] + 6 * c["rank"] * (2 * c["hidden"] + 3 * c["inter"]))


def peaks():
    """(bf16 sustained, bf16 burst, HBM GB/s, "measured" | "fallback") from MEASURED_PEAKS.json."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        p = json.load(open(path))
        return float(p["bf16_tflops_sustained"]), float(p["bf16_tflops"]), float(p["hbm_gbs"]), "measured"
    return 1400.0, 1590.0, 6650.0, "fallback"


def pick_peak(clocks, sustained, burst):
    """The bf16 peak that matches the clock regime of the timed region: the burst figure (a GEMM timed alone, at
    full clock) when the median SM clock sampled under load is within 5% of the maximum with no power cap seen;
    the sustained one (seconds of GEMMs under the power cap) otherwise."""
    sm, mx = clocks.get("sm_mhz"), clocks.get("sm_max_mhz")
    full = sm is not None and mx and sm >= 0.95 * mx and "sw_power_cap" not in clocks.get("reasons", [])
    return (burst, "burst") if full else (sustained, "sustained")


class ClockSampler:
    """nvidia-smi sampled every 100 ms from before the warm-up; the summary keeps the samples that arrived while
    the timed region ran (between mark_start and mark_stop)."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []
        self.t0 = self.t1 = None

    def __enter__(self):
        import threading

        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self

        def read():
            for ln in self.proc.stdout:
                self.lines.append((time.monotonic(), ln.strip()))

        self.reader = threading.Thread(target=read, daemon=True)
        self.reader.start()
        return self

    def mark_start(self):
        self.t0 = time.monotonic()

    def mark_stop(self):
        self.t1 = time.monotonic()

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for t, ln in list(self.lines):
            if self.t0 is not None and (t < self.t0 or (self.t1 is not None and t > self.t1 + 0.1)):
                continue
            f = [x.strip() for x in ln.split(",")]
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


class GemmTimer:
    """CUDA events around every grouped-product launch, on the launching stream; totals over the timed steps."""

    def __init__(self):
        import torch

        self.torch = torch
        self.pending = []
        self.active = False

    def before(self, x):
        if self.active:
            ev = self.torch.cuda.Event(enable_timing=True)
            ev.record(self.torch.cuda.current_stream(x.device))
            self._start = ev

    def after(self, x, flops):
        if self.active:
            ev = self.torch.cuda.Event(enable_timing=True)
            ev.record(self.torch.cuda.current_stream(x.device))
            self.pending.append((self._start, ev, flops))

    def totals(self):
        ms = sum(a.elapsed_time(b) for a, b, _ in self.pending)
        return ms, sum(f for _, _, f in self.pending), len(self.pending)


def setup_dist():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def make_layer(c, device, seed):
    import torch

    import meepsquared_b200 as mb  # noqa: F401

    g = torch.Generator(device=device).manual_seed(seed)
    T, H, I, E, k, r = c["tokens"], c["hidden"], c["inter"], c["experts"], c["top_k"], c["rank"]
    logits = torch.randn(T, E, device=device, generator=g)
    if c.get("zipf"):
        order = torch.randperm(E, device=device, generator=g)
        p = torch.arange(1, E + 1, device=device, dtype=torch.float32) ** (-c["zipf"])
        logits = logits + torch.log(p / p.sum())[order]
    probs = torch.softmax(logits, dim=-1, dtype=torch.float32)
    w, idx = torch.topk(probs, k, dim=-1)
    w = w / w.sum(dim=-1, keepdim=True)

    class Experts(torch.nn.Module):
        pass

    ex = Experts()
    ex.num_experts, ex.has_gate, ex.has_bias, ex.is_transposed = E, True, False, False
    ex.gate_up_proj = torch.nn.Parameter((torch.randn(E, 2 * I, H, device=device, generator=g) * 0.02).to(torch.bfloat16),
                                         requires_grad=False)
    ex.down_proj = torch.nn.Parameter((torch.randn(E, H, I, device=device, generator=g) * 0.02).to(torch.bfloat16),
                                      requires_grad=False)
    if c.get("quant") == "nf4":  # QLoRA: NF4 blocks of 64, absmax double-quantised (blocks of 256)
        mb._nf4.convert_stacks(ex)
    elif c.get("quant") == "fp8_block128":  # e4m3 with a 128 x 128 grid of scales per expert matrix
        mb._fp8.convert_stacks(ex, block=128)
    bound1, bound2 = 1.0 / H ** 0.5, 1.0 / I ** 0.5
    lora = {
        "lhs1": (torch.randn(E, 2 * I, r, device=device, generator=g) * 0.01).to(torch.bfloat16),
        "rhs1": ((torch.rand(E, r, H, device=device, generator=g) * 2 - 1) * bound1).to(torch.bfloat16),
        "lhs2": (torch.randn(E, H, r, device=device, generator=g) * 0.01).to(torch.bfloat16),
        "rhs2": ((torch.rand(E, r, I, device=device, generator=g) * 2 - 1) * bound2).to(torch.bfloat16),
    }
    for t in lora.values():
        t.requires_grad_()
    hidden = torch.randn(T, H, device=device, generator=g).to(torch.bfloat16)
    grad = torch.randn(T, H, device=device, generator=g).to(torch.bfloat16)
    return ex, lora, hidden, idx, w, grad


def run_meep2b(a):
    import torch
    import torch.distributed as dist

    import meepsquared_b200 as mb
    from meepsquared_b200 import _grouped, ddp

    world, rank, local = setup_dist()
    c = CONFIGS[a.config]
    device = torch.device("cuda", local)
    ex, lora, hidden, idx, w, grad = make_layer(c, device, seed=1234 + rank)
    s = c["alpha"] / c["rank"]
    factors = {"gate_up_proj": (lora["lhs1"], lora["rhs1"], s), "down_proj": (lora["lhs2"], lora["rhs2"], s)}
    # the down projection's adapter gradients are ready first: their average starts while the gate/up input gradient
    # runs, the gate/up adapters' at the end of the step
    bucket = ddp.LoraGradBucket(list(lora.values()),
                                segments=[[lora["lhs2"], lora["rhs2"]], [lora["lhs1"], lora["rhs1"]]])
    hidden_leaf = hidden.clone().requires_grad_()

    def step(h, ids, wts, g):
        bucket.release()  # the layer's reductions write the adapters' gradients into the bucket
        h.grad = None  # the input gradient is made fresh each step (in a model it flows on to the previous layer)
        out = mb.routed_forward(ex, h, ids, wts, factors)
        out.backward(g)
        bucket.reduce()
        return out

    def sync():
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()
            torch.cuda.synchronize(device)

    clocks = ClockSampler(local).__enter__()
    for _ in range(a.warmup):
        step(hidden_leaf, idx, w, grad)
    sync()

    timer = GemmTimer()
    _grouped.set_launch_observer(timer)
    timer.active = True
    stream = torch.cuda.current_stream(device)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sync()
    clocks.mark_start()
    launches_before = mb._lib.launch_count()
    start.record(stream)
    for _ in range(a.steps):
        step(hidden_leaf, idx, w, grad)
    stop.record(stream)
    timed_launches = mb._lib.launch_count() - launches_before
    sync()
    clocks.mark_stop()
    timer.active = False
    _grouped.set_launch_observer(None)
    ms = start.elapsed_time(stop)
    gemm_ms, gemm_flops, gemm_launches = timer.totals()

    # End to end through the public API with host buffers: every step copies its inputs in from pinned host memory
    # (hidden states, routing, upstream gradient) and reads its result back: the LoRA gradients, what the optimizer
    # steps on (the layer output and input gradient stay on the device, where the neighbouring layers of a model
    # consume them). As a training loop with a prefetching data loader does, the copies run beside the compute:
    # step i+1's inputs go in on one stream and step i's gradients come out on another while step i+1 computes. The
    # timed region covers every step's copies in both directions.
    h_host = hidden.cpu().pin_memory()
    i_host = idx.cpu().pin_memory()
    w_host = w.cpu().pin_memory()
    g_host = grad.cpu().pin_memory()
    lg_host = [torch.empty(bucket.flat.shape, dtype=bucket.flat.dtype).pin_memory() for _ in range(2)]
    d_in = [(torch.empty_like(hidden), torch.empty_like(idx), torch.empty_like(w), torch.empty_like(grad))
            for _ in range(2)]
    lg_stage = [torch.empty_like(bucket.flat) for _ in range(2)]
    copy_in, copy_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    in_ready = [torch.cuda.Event() for _ in range(2)]
    inputs_free = [None, None]   # the step that last read this input slot has finished
    outputs_free = [None, None]  # the read-back of this slot's staged LoRA gradients has finished

    def h2d(slot):
        if inputs_free[slot] is not None:
            copy_in.wait_event(inputs_free[slot])
        with torch.cuda.stream(copy_in):
            for dst, src in zip(d_in[slot], (h_host, i_host, w_host, g_host)):
                dst.copy_(src, non_blocking=True)
            in_ready[slot].record(copy_in)

    def e2e_run(n):
        inputs_free[:] = [None, None]
        outputs_free[:] = [None, None]
        h2d(0)
        for i in range(n):
            cur = i % 2
            stream.wait_event(in_ready[cur])
            if i + 1 < n:
                h2d(1 - cur)
            hd, ids, wts, g = d_in[cur]
            h = hd.detach().requires_grad_()
            step(h, ids, wts, g)
            if outputs_free[cur] is not None:
                stream.wait_event(outputs_free[cur])
            lg_stage[cur].copy_(bucket.flat)
            done = torch.cuda.Event()
            done.record(stream)
            inputs_free[cur] = done
            copy_out.wait_event(done)
            with torch.cuda.stream(copy_out):
                lg_host[cur].copy_(lg_stage[cur], non_blocking=True)
            fin = torch.cuda.Event()
            fin.record(copy_out)
            outputs_free[cur] = fin
        stream.wait_stream(copy_in)
        stream.wait_stream(copy_out)

    e2e_run(max(2, a.warmup))
    sync()
    e_start, e_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_steps = max(3, a.steps // 2)
    sync()
    e_start.record(stream)
    e2e_run(e_steps)
    e_stop.record(stream)
    sync()
    e_ms = e_start.elapsed_time(e_stop)

    # the reference's own path on this GPU (bf16 stacks only: the reference has no NF4 stacks)
    gpu_base = None
    if not a.no_gpu_baseline:
        gpu_base = gpu_baseline(c, ex, lora, hidden, idx, w, grad, s, a.steps, a.warmup, device)
        sync()
    clocks.__exit__()

    times = torch.tensor([ms, e_ms, gpu_base["ms_per_step"] if gpu_base and "ms_per_step" in gpu_base else 0.0],
                         device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms, e_ms, base_ms = times.tolist()
    clock_summary = clocks.summary()
    rank_clocks = [clock_summary]
    if world > 1:  # every rank's clock record (the power cap is box-wide: it shows on all of them)
        rank_clocks = [None] * world
        dist.all_gather_object(rank_clocks, clock_summary)
    T = c["tokens"]
    value = world * T * a.steps / (ms / 1e3)
    e_value = world * T * e_steps / (e_ms / 1e3)
    sustained, burst, hbm, peak_source = peaks()
    bf16_peak, regime = pick_peak(clock_summary, sustained, burst)
    # MEEPSQUARED_FP8_PRODUCTS=1 on an FP8 stack: the frozen stack's products run e4m3 x e4m3 (the activations
    # quantised per row and 128-column tile); their roofline is the dense FP8 rate, the measured bf16 peak of the
    # regime times the measured FP8 / bf16 ratio (FP8_OVER_BF16)
    fp8_products = str(c.get("quant", "")).startswith("fp8") and os.environ.get("MEEPSQUARED_FP8_PRODUCTS") == "1"
    fp8_scale = FP8_OVER_BF16 if fp8_products else 1
    gemm_peak = round(fp8_scale * bf16_peak, 1)
    achieved = gemm_flops / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 else None
    layer_tflops = flop_per_token(c) * value / world / 1e12
    h2d = hidden.numel() * 2 + idx.numel() * idx.element_size() + w.numel() * 4 + grad.numel() * 2
    d2h = bucket.flat.numel() * bucket.flat.element_size()
    if gpu_base and "ms_per_step" in gpu_base:
        gpu_base["ms_per_step"] = round(base_ms, 4)
        gpu_base["value"] = round(world * T / (base_ms / 1e3), 1)
        gpu_base["frac_of_bf16_peak_layer"] = round(flop_per_token(c) * T / (base_ms / 1e3) / 1e12 / bf16_peak, 4)
    result = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(ms / a.steps, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "e4m3 products, bf16 adapters" if fp8_products else "bf16",
        "data": "synthetic (seeded, BASELINE config shapes)",
        "config": bench_config(a, c, world),
        "roofline": {"bound": "tensor", "kernel": "grouped_gemm (tcgen05), all product launches of the step",
                     "achieved": round(achieved, 1) if achieved else None, "peak": gemm_peak,
                     "unit": "TFLOP/s", "frac": round(achieved / gemm_peak, 4) if achieved else None,
                     "peak_kind": (f"fp8 = {FP8_OVER_BF16} x bf16 {regime} (measured ratio), {peak_source}" if fp8_products
                                   else f"bf16 {regime} ({'median SM clock at max' if regime == 'burst' else 'clock below max or power-capped'}), {peak_source}"),
                     "frac_of_burst": round(achieved / (fp8_scale * burst), 4) if achieved else None,
                     "frac_of_sustained": (round(achieved / (fp8_scale * sustained), 4)
                                           if achieved else None),
                     "launches_timed": gemm_launches, "gemm_ms_per_step": round(gemm_ms / a.steps, 4),
                     "traffic": GEMM_TRAFFIC_BYTES_PER_LAUNCH if a.config == "qwen3_30b" else None,
                     "traffic_unit": "DRAM bytes per launch (ncu capture of the four products at full size)",
                     "layer": {"achieved": round(layer_tflops, 1), "peak": bf16_peak,
                               "frac": round(layer_tflops / bf16_peak, 4),
                               "flop_per_token": flop_per_token(c),
                               "note": "algorithmic FLOPs of the whole layer step / step time, per GPU"}},
        "e2e": {"value": round(e_value, 1), "unit": "tokens/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h)},
        "gpu_launches": timed_launches,  # libmeep2b kernels launched in the timed steps (counted per call)
        "clocks": clock_summary,
    }
    if world > 1:
        result["clocks_per_rank"] = rank_clocks
        result["nccl_ranks"] = dist.get_world_size()
        result["exchange"] = ("LoRA-gradient average, two NCCL all-reduces per step: the down adapters' slice "
                              "started during the backward pass, the gate/up adapters' at its end")
    if gpu_base is not None:
        result["gpu_baseline"] = gpu_base
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(c)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


def bench_config(a, c, world):
    """The `config` object of the JSON line: the same for both arms of the same run."""
    return {"workload": a.config + " routed MoE-LoRA layer fwd+bwd", **c, "tokens_per_gpu": c["tokens"],
            "parallelism": f"dp{world}", "l2": "per-step tensors >> 126 MB L2, no flush"}


# ------------------------------------------------------------------------ the reference's path, restated

def reference_lora_delta(x, lhs, rhs, scaling, offsets, is_transposed):
    """scaling * x @ delta for each expert's rows, delta = lhs @ rhs in the stack's layout: the reference's
    _grouped_lora (meepsquared/_moe.py:48-67). Two grouped matmuls of rank depth; the rank is padded with zeros to
    a 16-byte row (the grouped matmul's stride rule) and the scaling goes into the small factor."""
    import torch
    from transformers.integrations.moe import _grouped_mm

    pad = -lhs.shape[-1] % (16 // lhs.element_size())
    if pad:
        lhs = torch.nn.functional.pad(lhs, (0, pad))
        rhs = torch.nn.functional.pad(rhs, (0, 0, 0, pad))
    if is_transposed:  # stack (experts, in, out): x @ lhs @ rhs
        first, second = (lhs * scaling).contiguous(), rhs.contiguous()
    else:  # stack (experts, out, in): x @ rhs^T @ lhs^T
        first, second = (rhs * scaling).transpose(-2, -1).contiguous(), lhs.transpose(-2, -1).contiguous()
    return _grouped_mm(_grouped_mm(x, first, offs=offsets), second, offs=offsets)


def reference_routed_forward(experts, hidden_states, top_k_index, top_k_weights, factors):
    """The reference's routed layer (meepsquared/_moe.py:_routed_forward, :70-126) on the branch it takes where its
    kernel is not wanted (every CPU, and a compute capability 10.0 GPU: _grouped.py:57-67): sort the flat expert
    ids, gather the rows, Transformers' grouped linear for each stack plus the adapters' change in place, sentinel
    rows zeroed, the gate, the weighted un-permute. bf16 stacks (or float32 on the CPU) without FP8 scales."""
    import torch
    from transformers.integrations.moe import _grouped_linear

    device = hidden_states.device
    k = top_k_index.size(-1)
    tokens, hidden_dim = hidden_states.size(0), hidden_states.size(-1)
    experts_n = experts.num_experts
    flat_ids = top_k_index.reshape(-1)
    ids_sorted, perm = torch.sort(flat_ids)
    rows = hidden_states[perm // k]
    weights_sorted = top_k_weights.reshape(-1)[perm]
    counts = torch.histc(ids_sorted.float() if device.type in ("cpu", "mps") else ids_sorted.int(),
                         bins=experts_n, min=0, max=experts_n - 1)
    offsets = torch.cumsum(counts, dim=0, dtype=torch.int32)
    sentinel = (ids_sorted >= experts_n).unsqueeze(-1)
    ids_sorted.clamp_(max=experts_n - 1)
    rows = rows.masked_fill(sentinel, 0.0)

    def project(x, name, bias_name):
        lhs, rhs, scaling = factors.get(name, (None, None, 1.0))
        bias = getattr(experts, bias_name)[ids_sorted] if experts.has_bias else None
        out = _grouped_linear(x, getattr(experts, name), offsets, bias=bias, is_transposed=experts.is_transposed)
        if lhs is not None:
            out = out.add_(reference_lora_delta(x.to(lhs.dtype), lhs, rhs, scaling, offsets, experts.is_transposed))
        return out.masked_fill_(sentinel, 0.0)

    if experts.has_gate:
        gate_up = project(rows, "gate_up_proj", "gate_up_proj_bias")
        if hasattr(experts, "_apply_gate"):
            h = experts._apply_gate(gate_up)
        else:  # Transformers' default gate with the SiLU activation (Qwen3, Mixtral)
            gate, up = gate_up.chunk(2, dim=-1)
            h = torch.nn.functional.silu(gate) * up
    else:
        h = experts.act_fn(project(rows, "up_proj", "up_proj_bias"))
    y = project(h, "down_proj", "down_proj_bias")
    weighted = y * weights_sorted.unsqueeze(-1)
    inverse = torch.empty_like(perm)
    inverse[perm] = torch.arange(perm.size(0), device=device)
    return weighted[inverse].view(tokens, k, hidden_dim).sum(dim=1).to(hidden_states.dtype)


def gpu_baseline(c, ex, lora, hidden, idx, w, grad, scaling, steps, warmup, device):
    """The reference's path on this GPU (reference_routed_forward, bf16), forward + backward with the gradients of
    the hidden states, the routing weights and the four factors: W untimed steps, then K steps timed with CUDA
    events on the launching stream."""
    import torch

    if c.get("quant"):
        return {"unavailable": "quantised stacks: the reference dequantises FP8 per product and has no NF4 stacks"}
    leaves = {n: t.detach().clone().requires_grad_() for n, t in lora.items()}
    factors = {"gate_up_proj": (leaves["lhs1"], leaves["rhs1"], scaling),
               "down_proj": (leaves["lhs2"], leaves["rhs2"], scaling)}
    weights = w.detach().clone().requires_grad_()

    def step():
        h = hidden.detach().requires_grad_()
        weights.grad = None
        for t in leaves.values():
            t.grad = None
        out = reference_routed_forward(ex, h, idx, weights, factors)
        out.backward(grad)

    for _ in range(max(1, warmup)):
        step()
    stream = torch.cuda.current_stream(device)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    start.record(stream)
    for _ in range(steps):
        step()
    stop.record(stream)
    torch.cuda.synchronize(device)
    ms = start.elapsed_time(stop) / steps
    return {"ms_per_step": ms, "unit": "tokens/s", "steps": steps, "warmup": max(1, warmup),
            "impl": "the reference's _routed_forward, non-kernel branch (torch grouped_mm + _grouped_lora), bf16",
            "kind": "port"}


# ------------------------------------------------------------------------ the reference's path on the host cores

def cpu_inputs(c, tokens):
    """The workload's seeded inputs (float32, CPU) for its first `tokens` tokens: the per-token tensors of the full
    batch cut to a sample, the full stacks and adapters."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import layer_inputs

    cfg = {k: v for k, v in c.items() if k not in ("quant",)}  # a quantised config's CPU leg runs bf16-valued stacks
    inp = layer_inputs.layer(**cfg)
    if tokens < c["tokens"]:
        for n in ("hidden", "top_k_index", "top_k_weights", "grad"):
            inp[n] = inp[n][:tokens].contiguous()
    return inp


def run_cpu_reference(inp, c, steps, warmup):
    """Seconds per step of reference_routed_forward + backward on the host cores, float32, all host threads."""
    import types

    import torch

    torch.set_num_threads(os.cpu_count() or 1)  # a launcher (torchrun) sets OMP_NUM_THREADS=1 for its ranks
    ex = types.SimpleNamespace(num_experts=c["experts"], has_gate=True, has_bias=False, is_transposed=False,
                               gate_up_proj=inp["gate_up"], down_proj=inp["down"])
    s = inp["scaling"]

    def once():
        leaves = {n: inp[n].clone().requires_grad_() for n in ("gate_up_lhs", "gate_up_rhs", "down_lhs", "down_rhs")}
        factors = {"gate_up_proj": (leaves["gate_up_lhs"], leaves["gate_up_rhs"], s),
                   "down_proj": (leaves["down_lhs"], leaves["down_rhs"], s)}
        h = inp["hidden"].clone().requires_grad_()
        wts = inp["top_k_weights"].clone().requires_grad_()
        t0 = time.perf_counter()
        out = reference_routed_forward(ex, h, inp["top_k_index"], wts, factors)
        out.backward(inp["grad"])
        return time.perf_counter() - t0

    for _ in range(warmup):
        once()
    return [once() for _ in range(steps)], torch.get_num_threads()


def sample_tokens(c, seconds_full, steps, budget_s):
    """Tokens per step of a CPU leg: the whole batch when `steps` steps of it fit in `budget_s`, else the largest
    power of two (at least 2048, every expert still ~128 routed rows at config 2) that does."""
    T = c["tokens"]
    if seconds_full * steps <= budget_s:
        return T
    t = 2048
    while t * 2 < T and seconds_full * (t * 2 / T) * steps <= budget_s:
        t *= 2
    return min(t, T)


def cpu_baseline(c):
    """The reference's CPU path timed on the host cores: the benchmarked workload (its whole batch when a step
    fits the ~30 s budget, else a leading sample of its tokens) and BASELINE config 1 in full."""
    import torch

    full = cpu_inputs(c, c["tokens"])
    probe, _ = run_cpu_reference(full, c, 1, 1)
    tokens = sample_tokens(c, probe[0], 3, 30.0)
    inp = full if tokens == c["tokens"] else cpu_inputs(c, tokens)
    reps, threads = run_cpu_reference(inp, c, 3, 0 if tokens == c["tokens"] else 1)
    sec = statistics.median(reps + (probe if tokens == c["tokens"] else []))
    c1 = dict(tokens=512, hidden=256, inter=512, experts=8, top_k=2, rank=8, alpha=16)
    r1, _ = run_cpu_reference(cpu_inputs(c1, 512), c1, 20, 3)
    sec1 = statistics.median(r1)
    del torch
    return {"value": round(tokens / sec, 1), "unit": "tokens/s", "cores": threads, "kind": "port",
            "host_cpus": os.cpu_count(),
            "sample": (f"{tokens} of the workload's {c['tokens']} tokens per step (all {c['experts']} experts), "
                       f"fwd+bwd, float32 eager PyTorch (the reference's _routed_forward restated), median of "
                       f"{len(reps)}" + (", stacks bf16-valued" if c.get("quant") else "")),
            "config1": {"value": round(512 / sec1, 1), "unit": "tokens/s", "ms_per_step": round(sec1 * 1e3, 3),
                        "config": c1, "sample": "the whole config (512 tokens), median of 20 after 3 warm-ups"}}


def run_reference(a):
    """--impl reference: the reference's path on the host cores (rank 0 alone), float32, the same config, metric and
    unit as the library's arm. Each step runs the whole batch when W + K steps fit in ~4 minutes, else the same
    leading sample of its tokens every step."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    c = CONFIGS[a.config]
    full = cpu_inputs(c, c["tokens"])
    probe, _ = run_cpu_reference(full, c, 1, 1)
    tokens = sample_tokens(c, probe[0], a.steps + a.warmup, 240.0)
    inp = full if tokens == c["tokens"] else cpu_inputs(c, tokens)
    reps, threads = run_cpu_reference(inp, c, a.steps, a.warmup)
    sec = sum(reps) / len(reps)
    value = round(tokens / sec, 1)
    sample = (f"{tokens} of the workload's {c['tokens']} tokens per step (all {c['experts']} experts), fwd+bwd, "
              f"float32 eager PyTorch (the reference's _routed_forward restated), mean of {a.steps} steps after "
              f"{a.warmup} warm-ups")
    print(json.dumps({
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": round(1e3 * sec, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, BASELINE config shapes)", "impl": "reference",
        "config": bench_config(a, c, world),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "host_cpus": os.cpu_count(), "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}), flush=True)


def run_model(a):
    """--config qwen3_30b_model: a training step of a whole Qwen3-MoE model (random weights of the configured
    sizes, Transformers' Qwen3MoeForCausalLM) with LoRA on every expert stack: forward, the language-model loss on
    the batch itself, backward, AdamW on the adapters. The experts run the routed layer (meepsquared_b200.model);
    the same model with its experts on the reference's PyTorch path (reference_routed_forward) is the GPU baseline."""
    import types

    import torch
    from transformers import Qwen3MoeConfig, Qwen3MoeForCausalLM

    import meepsquared_b200 as mb
    from meepsquared_b200 import _grouped

    c = CONFIGS[a.config]
    torch.cuda.set_device(0)
    device = torch.device("cuda", 0)
    cfg = Qwen3MoeConfig(vocab_size=c["vocab"], hidden_size=c["hidden"], intermediate_size=4 * c["hidden"],
                         moe_intermediate_size=c["inter"], num_hidden_layers=c["layers"],
                         num_attention_heads=c["heads"], num_key_value_heads=c["kv_heads"], head_dim=c["head_dim"],
                         num_experts=c["experts"], num_experts_per_tok=c["top_k"], decoder_sparse_step=1,
                         mlp_only_layers=[], norm_topk_prob=True, max_position_embeddings=c["seq"])
    torch.manual_seed(1234)
    with torch.device(device):
        model = Qwen3MoeForCausalLM(cfg).to(torch.bfloat16)
    for p in model.parameters():
        p.requires_grad_(False)
    mb.model.install(model, rank=c["rank"], alpha=c["alpha"], generator=torch.Generator().manual_seed(0))
    params = mb.model.lora_parameters(model)
    opt = torch.optim.AdamW(params, lr=1e-4)
    batch = c["tokens"] // c["seq"]
    ids = torch.randint(0, c["vocab"], (batch, c["seq"]), generator=torch.Generator().manual_seed(1)).to(device)

    def step():
        opt.zero_grad(set_to_none=True)
        out = model(input_ids=ids, labels=ids)
        out.loss.backward()
        opt.step()
        return out.loss

    def timed(n):
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        start.record()
        for _ in range(n):
            step()
        stop.record()
        torch.cuda.synchronize()
        return start.elapsed_time(stop) / n

    clocks = ClockSampler(0).__enter__()
    for _ in range(a.warmup):
        step()
    timer = GemmTimer()
    _grouped.set_launch_observer(timer)
    timer.active = True
    clocks.mark_start()
    launches_before = mb._lib.launch_count()
    ms = timed(a.steps)
    timed_launches = mb._lib.launch_count() - launches_before
    clocks.mark_stop()
    timer.active = False
    _grouped.set_launch_observer(None)
    gemm_ms, gemm_flops, _ = timer.totals()
    # the same model with its experts on the reference's PyTorch path
    def reference_forward(self, hidden_states, top_k_index, top_k_weights):
        factors = {name: (getattr(self, f"lora_{name}_lhs"), getattr(self, f"lora_{name}_rhs"), self.lora_scaling)
                   for name in self.lora_stacks}
        return reference_routed_forward(self, hidden_states, top_k_index, top_k_weights, factors)

    saved = {}
    for name, e in mb.model.experts_modules(model):
        saved[name] = e.forward
        e.forward = types.MethodType(reference_forward, e)
    for _ in range(max(1, a.warmup)):
        step()
    base_ms = timed(a.steps)
    clocks.__exit__()
    T = c["tokens"]
    sustained, burst, hbm, peak_source = peaks()
    clock_summary = clocks.summary()
    bf16_peak, regime = pick_peak(clock_summary, sustained, burst)
    achieved = gemm_flops / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 else None
    print(json.dumps({
        "metric": "MoE-LoRA model training step tokens/s", "value": round(T / (ms / 1e3), 1), "unit": "tokens/s",
        "n_gpus": 1, "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random weights and token ids)",
        "config": {"workload": "qwen3_30b_model: Qwen3-MoE decoder layers at Qwen3-30B-A3B sizes, LoRA on the experts, "
                               "fwd + loss + bwd + AdamW", **{k: v for k, v in c.items() if k != "model"}},
        "roofline": {"bound": "tensor", "kernel": "grouped_gemm (tcgen05), all product launches of the step",
                     "achieved": round(achieved, 1) if achieved else None, "peak": bf16_peak, "unit": "TFLOP/s",
                     "frac": round(achieved / bf16_peak, 4) if achieved else None,
                     "peak_kind": f"bf16 {regime}, {peak_source}", "gemm_ms_per_step": round(gemm_ms / a.steps, 4)},
        "gpu_launches": timed_launches, "clocks": clock_summary,
        "gpu_baseline": {"ms_per_step": round(base_ms, 4), "value": round(T / (base_ms / 1e3), 1),
                         "unit": "tokens/s", "impl": "the same model, experts on the reference's _routed_forward "
                                                     "non-kernel branch (torch grouped_mm + _grouped_lora)"}}),
          flush=True)


# Dense e4m3 GEMM rate over the bf16 one on a B200, measured with `bench.py --measure-fp8-peak` (torch._scaled_mm
# e4m3 x e4m3 -> bf16 at 8192^3: 3,082 and 3,070 TFLOP/s against torch.matmul bf16 at 1,622 and 1,618 in the same
# processes), below the nominal 2 (4.5 / 2.25 PFLOP/s)
FP8_OVER_BF16 = 1.90


def measure_fp8_peak():
    """The dense e4m3 GEMM rate of this GPU through the vendor library (torch._scaled_mm, e4m3 x e4m3 -> bf16,
    8192^3, per-tensor scales): best of 10 launches after 5 warm-ups, CUDA events, with a bf16 matmul of the same
    size beside it. The FP8 products' roofline uses this figure; one JSON line."""
    import torch

    n = 8192
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    a = torch.randn(n, n, device=dev, generator=g).to(torch.float8_e4m3fn)
    b = torch.randn(n, n, device=dev, generator=g).to(torch.float8_e4m3fn).t()  # column-major, as the call wants
    one = torch.ones((), device=dev)
    ab = torch.randn(n, n, device=dev, generator=g, dtype=torch.bfloat16)
    bb = torch.randn(n, n, device=dev, generator=g, dtype=torch.bfloat16)

    def best(fn):
        for _ in range(5):
            fn()
        ts = []
        for _ in range(10):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            ts.append(s.elapsed_time(e))
        return min(ts)

    ms8 = best(lambda: torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16))
    ms16 = best(lambda: torch.matmul(ab, bb))
    flop = 2 * n ** 3
    print(json.dumps({"fp8_e4m3_tflops": round(flop / ms8 / 1e9, 1), "bf16_tflops": round(flop / ms16 / 1e9, 1),
                      "shape": [n, n, n], "how": "torch._scaled_mm e4m3 x e4m3 -> bf16 and torch.matmul bf16, "
                      "best of 10 after 5 warm-ups, CUDA events"}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="meep2b", choices=["meep2b", "reference"])
    ap.add_argument("--config", default="qwen3_30b", choices=sorted(CONFIGS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gpu-baseline", action="store_true")
    ap.add_argument("--measure-fp8-peak", action="store_true", help="print this GPU's dense e4m3 GEMM rate and exit")
    a = ap.parse_args()
    if a.measure_fp8_peak:
        measure_fp8_peak()
        return
    if a.warmup < 3 and a.impl == "meep2b":
        a.warmup = 3
    if CONFIGS[a.config].get("model"):
        if a.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the model config's reference arm is its "
                                                                   "gpu_baseline (the same model on the reference's "
                                                                   "PyTorch path), in the meep2b line"}))
            return
        run_model(a)
    elif a.impl == "reference":
        run_reference(a)
    else:
        run_meep2b(a)


if __name__ == "__main__":
    main()
