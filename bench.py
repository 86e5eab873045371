"""Benchmark of the B200 MoE expert path (prints ONE JSON line on rank 0).

Workload (N = 1 per GPU): the MoE path of the synthetic Qwen3-30B-A3B-shaped
model (benchmark configuration 2): 48 MoE FFN layers, hidden 2048, 128
experts top-8 (softmax, selected weights renormalised), expert intermediate
768, Q4_K experts synthesised in HBM from seed 0 (16.3 GB pool), F32 routers
~N(0, 0.02), F32 ffn_norm = 1.  One step = one decode token through all 48
layers: hidden += MoE_l(rms_norm(hidden, ffn_norm_l)) for l = 0..47.  The
attention half of each decoder layer is outside this path.

  value   decode tokens/s with inputs resident in HBM (CUDA events, max over ranks)
  e2e     the same through pokit_cuda_moe_decode_layers_host: host hidden in
          (pinned) -> device -> 48 layers -> host hidden out, every step
  roofline  the dominant kernel, moe_chain_kernel: the whole 48-layer chain is
          one cooperative launch per token, so its algorithmic bytes per
          launch are 48 x 22,298,624 (router + 8 routed experts + in/out per
          layer) / its average launch duration (CUDA events around launches
          back to back, after the timed region); traffic = DRAM bytes per
          layer of the committed ncu capture x 48
  chain_phases  per-layer phase times of the chain kernel from one traced
          launch (globaltimer stamps of every CTA); gate_up_* is the in-kernel
          Q4_K gate/up matvec: 8 experts x (gate + up) x 884,736 B + x' in +
          act out / the window from the first CTA's routes to the last CTA's
          gate/up products
  block_roofline  per MoE block: 22,298,624 algorithmic bytes (router 1 MiB +
          8 experts x 2,654,208 B + 16 KiB in/out) / (step time / 48)

Between steps nothing is flushed: one step streams 1.07 GB of distinct expert
and router bytes, far above the 126 MB L2.

  grouped  (N = 1) benchmark configuration 4 beside the headline: 512 tokens,
          BF16 activations ~N(0, 1), router logits ~N(0, 1) + a Zipf(1.1)
          popularity bias, one MoE block (hidden 2048, 128 experts top-8,
          inter 768, Q4_K) through the grouped-expert tensor-core GEMM
          (pokit_cuda_moe_forward_batch); L2 flushed (256 MiB write) between
          timed batches; per-kernel times from pokit_cuda_moe_time_batch.

With N > 1 (torchrun) every rank decodes its own sequence on its own copy of the
model (independent replicas: the 16.3 GB pool fits one GPU; no data-path
collective); value = N tokens per step / the slowest rank's step time, and
`parity` checks that every rank gives the same bits on a common input.

  decoder (N = 1) benchmark configuration 2 end to end: the whole 48-layer
          decoder (attention, MoE, Q6_K LM head) greedy-decoding 128 tokens
          after a 32-token prompt (pokit_cuda_decoder_*).
  config5 (every N) benchmark configuration 5 through expert parallelism over
          all ranks (128 / N experts per GPU, NCCL all-reduce of the partial
          outputs inside the step's CUDA graph), strong scaling, with a parity
          object and the exchange step timed as an all-reduce and as two
          all-to-alls.

--impl reference times the PokitLMs reference's own CPU kernels and row
executor (oracle/_ref) on the host cores, same metric and unit.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

H, I, E, K_TOP, LAYERS = 2048, 768, 128, 8, 48
SEED = 0
EPS = 1e-6
EXPERT_BYTES = 3 * 884_736                     # gate + up + down, Q4_K
ROUTER_BYTES = E * H * 4
BLOCK_BYTES = ROUTER_BYTES + K_TOP * EXPERT_BYTES + 2 * H * 4
ROUTED_BYTES = K_TOP * EXPERT_BYTES
# gate/up phase: 8 experts x (gate + up) Q4_K + x' (F32 [H]) in + 8 x 768 act
# floats out.
GATE_UP_BYTES = K_TOP * 2 * 884_736 + H * 4 + K_TOP * I * 4
TRAFFIC_FILE = ROOT / "profiles" / "moe_chain_q4k_h2048_e128_k8.md"
TRAFFIC_SOURCE = ("committed ncu capture (profiles/moe_chain_q4k_h2048_e128_k8.md) of a 4-layer launch, "
                  "per-layer DRAM bytes x layers")
METRIC = "decode tokens/sec and routed-expert HBM GB/s (% of peak) at 1/2/4/8 B200"
WORKLOAD = ("qwen3-30b-a3b-shaped MoE expert path: 48 MoE FFN layers (hidden 2048, 128 experts "
            "top-8 renormalised, inter 768, Q4_K experts, F32 router), decode batch 1")


def ncu_traffic_bytes(layers: int) -> float | None:
    """DRAM bytes (read + write) of one chain launch over `layers` layers, from
    the committed ncu summary of a shorter launch (line
    'traffic_bytes_per_layer: N', scaled by the layer count: every layer
    streams its own distinct weights)."""
    try:
        for line in TRAFFIC_FILE.read_text().splitlines():
            if line.strip().startswith("traffic_bytes_per_layer:"):
                return float(line.split(":", 1)[1]) * layers
    except OSError:
        pass
    return None


def chain_phases(be, layers: int, work, stream) -> dict:
    """Per-layer phase times of the chain kernel from one traced launch
    (pokit_cuda_moe_trace_decode; globaltimer stamps of every CTA): medians
    over the inner layers.  gate_up_us: first CTA's routes ready -> last CTA's
    gate/up products done (the window in which the layer's 14.2 MB of gate/up
    weights stream in); act_exchange_down_us: last CTA's activation words
    stored -> last D unit's down products combined (the tagged-word exchange
    plus the down MMA); partials_us: -> last D unit's next-layer router
    partials added and its route arrival."""
    import torch
    grid = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    st = torch.zeros(layers * grid * 16, dtype=torch.int64, device="cuda")
    g = be.trace_decode(0, layers, work, st, stream)
    torch.cuda.synchronize()
    ns = st.cpu().numpy().reshape(layers, g, 16)[:, :, :8].astype(np.float64)
    units = H // 16
    inner = range(1, layers - 1) if layers > 2 else range(layers)
    med = lambda v: float(np.median(v)) / 1e3  # noqa: E731
    return {
        "layer_us": med([ns[l, :units, 7].max() - ns[l - 1, :units, 7].max() for l in inner if l > 0]) if layers > 1 else None,
        "route_us": med([ns[l, :, 1].max() - ns[l, :, 0].min() for l in inner]),
        "gate_up_us": med([ns[l, :, 2].max() - ns[l, :, 1].min() for l in inner]),
        "act_exchange_down_us": med([ns[l, :units, 5].max() - ns[l, :, 3].max() for l in inner]),
        "partials_us": med([ns[l, :units, 7].max() - ns[l, :units, 5].max() for l in inner]),
        "how": "pokit_cuda_moe_trace_decode: globaltimer stamps per CTA and phase, medians over layers "
               "(globaltimer ticks are coarse: sub-microsecond phases are approximate)",
    }


def host_cpu() -> dict:
    """The box's CPU: logical cores and model name (the reference's row
    executor uses min(6, cores - 1) worker threads, src/tensor_linear.cpp:27)."""
    model = None
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"host_cores": os.cpu_count(), "cpu_model": model}


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clock/throttle samples while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (FileNotFoundError, OSError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def build_model(be, layers: int, router_dtype=None) -> None:
    from pokitlms_b200 import synth
    from pokitlms_b200._lib import DOWN, FFN_NORM, GATE, ROUTER, UP
    ones = np.ones(H, dtype=np.float32)
    for l in range(layers):
        be.upload_tensor(l, ROUTER, synth.router_weights(E, H, SEED, l))
        be.upload_tensor(l, FFN_NORM, ones)
        for t in (GATE, UP, DOWN):
            be.synthesize_tensor(l, t, SEED, synth.stream_id(l, t))


def cpu_reference_rate(target_seconds: float, max_tokens: int | None = None):
    """Decode tokens/s of the reference's CPU path: the reference's kernels and
    multi-threaded row executor (oracle/_ref) when built, else the oracle's C
    restatement.  Sample: 2 synthesised layers (layer l uses the weights of
    layer l % 2) stand for the 48; every token runs all 48 layer evaluations.
    Returns (tokens_per_s, kind, cores, sample_text)."""
    sys.path.insert(0, str(ROOT / "tests"))
    import cases
    from oracle import oracle as O
    from pokitlms_b200 import synth
    layers = [cases.moe_layer(seed=SEED, layer=l, with_norm=True) for l in range(2)]
    hw = os.cpu_count() or 1
    if O.ref_available():
        kind = "reference"
        cores = min(6, max(2, hw - 1))           # TensorRowExecutor workers, tensor_linear.cpp:27
        runners = [O.RefMoe(L) for L in layers]
        norm = O.ref_rms_norm

        def block(l, x):
            return runners[l % 2].forward(x)[0]
    else:
        kind = "port"
        cores = 1
        norm = O.rms_norm

        def block(l, x):
            return O.moe_forward(layers[l % 2], x)[0]
    ones = np.ones(H, dtype=np.float32)
    tokens = 0
    t0 = time.perf_counter()
    while True:
        h = synth.activation(H, SEED, 10_000 + tokens)
        for l in range(LAYERS):
            h = (h + block(l, norm(h, ones, EPS))).astype(np.float32)
        tokens += 1
        el = time.perf_counter() - t0
        if el >= target_seconds or (max_tokens and tokens >= max_tokens):
            break
    sample = (f"{tokens} decode tokens x 48 MoE layers (2 synthesised layers cycled), "
              f"{el:.1f} s of CPU work")
    return tokens / el, kind, cores, sample


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT / "tests"))
    import cases
    from oracle import oracle as O
    from pokitlms_b200 import synth
    layers = [cases.moe_layer(seed=SEED, layer=l, with_norm=True) for l in range(2)]
    hw = os.cpu_count() or 1
    if O.ref_available():
        kind, cores = "reference", min(6, max(2, hw - 1))
        runners = [O.RefMoe(L) for L in layers]
        norm = O.ref_rms_norm

        def block(l, x):
            return runners[l % 2].forward(x)[0]
    else:
        kind, cores, norm = "port", 1, O.rms_norm

        def block(l, x):
            return O.moe_forward(layers[l % 2], x)[0]
    ones = np.ones(H, dtype=np.float32)

    def step(i):
        h = synth.activation(H, SEED, 20_000 + i)
        for l in range(LAYERS):
            h = (h + block(l, norm(h, ones, EPS))).astype(np.float32)
        return h

    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(args.warmup + i)
    el = time.perf_counter() - t0
    v = args.steps / el
    sample = (f"each step = 1 decode token x 48 MoE layers (2 synthesised layers cycled) on "
              f"{cores} host thread(s)")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seed 0)",
        "config": {"workload": WORKLOAD, "layers": LAYERS, "hidden": H, "experts": E,
                   "top_k": K_TOP, "inter": I, "expert_type": "Q4_K"},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": kind,
                         "sample": sample, **host_cpu()},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }))


GROUPED_TOKENS = 512
GROUPED_FLOPS = GROUPED_TOKENS * K_TOP * 2 * 3 * I * H          # 38.65 GFLOP
GATE_UP_SLICE = 2 * 884_736                                      # gate + up of one expert


def measure_grouped(device: int, stream) -> dict:
    """Benchmark configuration 4 through the grouped-expert GEMM (see the
    module docstring).  Returns the "grouped" object of the JSON line."""
    import torch
    from pokitlms_b200 import backend as B
    from pokitlms_b200 import synth
    from pokitlms_b200._lib import DOWN, GATE, ROUTER, UP
    be = B.CudaMoeBackend(layers=1, hidden=H, inter=I, experts=E, top_k=K_TOP, rms_epsilon=EPS, device=device)
    be.upload_tensor(0, ROUTER, synth.router_weights(E, H, SEED, 0))
    for t in (GATE, UP, DOWN):
        be.synthesize_tensor(0, t, SEED, synth.stream_id(0, t))
    bits, _, logits = synth.grouped_inputs(GROUPED_TOKENS, E, H, seed=SEED)
    x = torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16)
    lg = torch.from_numpy(logits).cuda()
    out = torch.empty(GROUPED_TOKENS, H, device="cuda")
    ids = torch.empty(GROUPED_TOKENS, K_TOP, dtype=torch.int32, device="cuda")
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")   # 256 MiB > L2
    for _ in range(3):
        be.forward_batch(0, x, out, logits=lg, route_ids=ids, stream=stream)
    be.synchronize(stream)
    launches0 = be.stats()["kernel_launches"]
    times = []
    for i in range(20):
        flush.fill_(float(i))
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        be.forward_batch(0, x, out, logits=lg, stream=stream)
        b.record(stream)
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b) * 1e3)
    be.synchronize(stream)
    launches = (be.stats()["kernel_launches"] - launches0) // 20
    us = statistics.median(times)
    stage_names = ["route", "group", "pack_x", "gate_up_gemm", "pack_act", "down_gemm", "combine"]
    stages = be.time_batch(0, x, out, logits=lg, reps=10, stream=stream)
    stage_us = dict(zip(stage_names, stages))
    touched = int(np.unique(ids.cpu().numpy()).size)
    # End to end: BF16 rows and logits from the host, output and routes back.
    for _ in range(2):
        be.forward_batch_host(0, bits, bf16_bits=True, logits=logits)
    t0 = time.perf_counter()
    reps = 10
    for _ in range(reps):
        be.forward_batch_host(0, bits, bf16_bits=True, logits=logits)
    e2e_us = (time.perf_counter() - t0) / reps * 1e6
    be.close()
    peaks = measured_peaks()
    weight_bytes = touched * EXPERT_BYTES
    act_bytes = GROUPED_TOKENS * H * (2 + 4) + logits.nbytes
    gu_us = stage_us["gate_up_gemm"]
    gu_bytes = touched * GATE_UP_SLICE
    tflops = GROUPED_FLOPS / (us * 1e-6) / 1e12
    return {
        "workload": ("benchmark configuration 4: 512 tokens, BF16 x ~N(0,1), logits ~N(0,1) + Zipf(1.1) bias, "
                     "one block hidden 2048 / 128 experts top-8 / inter 768 / Q4_K"),
        "value": GROUPED_TOKENS / (us * 1e-6), "unit": "tokens/s", "us_per_batch": us,
        "l2": "flushed (256 MiB write) between timed batches",
        "experts_touched": touched, "gpu_launches_per_batch": int(launches), "stage_us": stage_us,
        "hbm": {"algorithmic_bytes": weight_bytes + act_bytes,
                "achieved_gbs": (weight_bytes + act_bytes) / (us * 1e-6) / 1e9,
                "frac": (weight_bytes + act_bytes) / (us * 1e-6) / 1e9 / peaks["hbm_gbs"],
                "peak_gbs": peaks["hbm_gbs"], "peak_source": peaks["source"]},
        "tensor": {"flops": GROUPED_FLOPS, "achieved_tflops": tflops,
                   "frac_of_measured_bf16": tflops / measured_tflops()},
        "roofline": {"bound": "hbm", "kernel": "grouped_gemm_kernel<0> (Q4_K gate/up, tcgen05)",
                     "achieved": gu_bytes / (gu_us * 1e-6) / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gu_bytes / (gu_us * 1e-6) / 1e9 / peaks["hbm_gbs"],
                     "bytes_per_launch": gu_bytes, "avg_launch_us": gu_us},
        "e2e": {"value": GROUPED_TOKENS / (e2e_us * 1e-6), "unit": "tokens/s",
                "h2d_bytes_per_step": int(bits.nbytes + logits.nbytes),
                "d2h_bytes_per_step": int(GROUPED_TOKENS * (H + 2 * K_TOP) * 4)},
    }


# Benchmark configuration 3's MoE path (Qwen3.5-MoE-style): 48 layers, H 2048, 512 experts top-10,
# I 512, sigmoid-gated shared expert I 512 (Q8_0), Q4_K gate/up, down Q5_K / Q6_K alternating.
CFG3 = {"layers": 48, "hidden": 2048, "inter": 512, "experts": 512, "top_k": 10, "shared_inter": 512}


def cfg3_layer_bytes(down_type: int) -> int:
    """Algorithmic bytes of one configuration-3 MoE block per token: F32 router, 10 routed
    experts (gate + up Q4_K, down Q5_K or Q6_K), the shared expert (Q8_0) and its gate row."""
    Hc, Ic = CFG3["hidden"], CFG3["inter"]
    q4 = Ic * (Hc // 256) * 144
    down = Hc * (Ic // 256) * (176 if down_type == 13 else 210)
    shared = 3 * Ic * (Hc // 32) * 34
    return CFG3["experts"] * Hc * 4 + CFG3["top_k"] * (2 * q4 + down) + shared + Hc * 4 + 2 * Hc * 4


def measure_config3(device: int, stream, steps: int, cpu_seconds: float | None, layers: int | None = None) -> dict:
    """Configuration 3's MoE path: a 48-layer decode chain of Qwen3.5-MoE blocks (moe_chain35_kernel),
    weights synthesised in HBM from seed 0; tokens/s device-resident and end to end.  `layers`
    shortens the chain (a small process for profiling its kernels)."""
    import torch
    from pokitlms_b200 import backend as B
    from pokitlms_b200 import synth
    from pokitlms_b200._lib import (DOWN, FFN_NORM, GATE, Q5_K, Q6_K, Q8_0, QWEN35, ROUTER, SHARED_DOWN,
                                    SHARED_GATE, SHARED_ROUTER, SHARED_UP, UP)
    c = dict(CFG3, layers=layers or CFG3["layers"])
    downs = [Q5_K if l % 2 == 0 else Q6_K for l in range(c["layers"])]
    be = B.CudaMoeBackend(layers=c["layers"], hidden=c["hidden"], inter=c["inter"], experts=c["experts"],
                          top_k=c["top_k"], flavour=QWEN35, expert_weights_scale=1.0, rms_epsilon=EPS,
                          down_type=Q5_K, layer_down_types=downs, shared_inter=c["shared_inter"],
                          shared_gate_type=Q8_0, shared_up_type=Q8_0, shared_down_type=Q8_0, device=device)
    ones = np.ones(c["hidden"], dtype=np.float32)
    for l in range(c["layers"]):
        be.upload_tensor(l, ROUTER, synth.router_weights(c["experts"], c["hidden"], SEED, l))
        be.upload_tensor(l, FFN_NORM, ones)
        be.upload_tensor(l, SHARED_ROUTER, synth.router_weights(1, c["hidden"], SEED, 1000 + l)[0])
        for t in (GATE, UP, DOWN, SHARED_GATE, SHARED_UP, SHARED_DOWN):
            be.synthesize_tensor(l, t, SEED, synth.stream_id(l, t))
    inputs = torch.from_numpy(np.stack([synth.activation(c["hidden"], SEED, 30_000 + i)
                                        for i in range(16)])).cuda()
    work = torch.empty(c["hidden"], device="cuda")
    for i in range(3):
        work.copy_(inputs[i])
        be.decode_layers(0, c["layers"], work, stream)
    be.synchronize(stream)
    l0 = be.stats()["kernel_launches"]
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(steps):
        work.copy_(inputs[i % 16], non_blocking=True)
        be.decode_layers(0, c["layers"], work, stream)
    b.record(stream)
    torch.cuda.synchronize()
    be.synchronize(stream)
    ms = a.elapsed_time(b) / steps
    launches = (be.stats()["kernel_launches"] - l0) // steps
    hin = np.stack([synth.activation(c["hidden"], SEED, 31_000 + i) for i in range(4)])
    hout = np.empty(c["hidden"], dtype=np.float32)
    be.decode_layers_host(0, c["layers"], hin[0], hout)
    t0 = time.perf_counter()
    e2e_steps = max(steps // 4, 5)
    for i in range(e2e_steps):
        be.decode_layers_host(0, c["layers"], hin[i % 4], hout)
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    work.copy_(inputs[0], non_blocking=True)
    phases = chain_phases(be, c["layers"], work, stream)
    be.close()
    tok_bytes = sum(cfg3_layer_bytes(d) for d in downs)
    peaks = measured_peaks()
    gbs = tok_bytes / (ms * 1e-3) / 1e9
    res = {
        "workload": (f"benchmark configuration 3's MoE path: {c['layers']} Qwen3.5-MoE blocks (hidden 2048, 512 experts "
                     "top-10, inter 512, sigmoid-gated Q8_0 shared expert, Q4_K gate/up, Q5_K/Q6_K down "
                     "alternating), decode batch 1; DeltaNet / attention layers outside the path"),
        "value": 1e3 / ms, "unit": "tokens/s", "ms_per_token": ms, "gpu_launches_per_token": int(launches),
        "hbm": {"bytes_per_token": tok_bytes, "achieved_gbs": gbs, "frac": gbs / peaks["hbm_gbs"],
                "peak_gbs": peaks["hbm_gbs"], "peak_source": peaks["source"]},
        "e2e": {"value": 1.0 / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": c["hidden"] * 4,
                "d2h_bytes_per_step": c["hidden"] * 4},
        "path": ("moe_chain35_kernel: one cooperative launch for the 48 blocks; Q4_K gate/up and Q5_K/Q6_K down on "
                 "integer mma.sync (u8/s8 x int8 activation pieces), the Q8_0 shared expert as FP32 dots of "
                 "tensor-map boxes"),
        "chain_phases": phases,
    }
    if cpu_seconds:
        res["cpu_baseline"] = cpu_config3_rate(cpu_seconds)
    return res


def cpu_config3_rate(target_seconds: float) -> dict:
    """The reference's CPU kernels and row executor (oracle/_ref) on configuration-3 blocks: two
    synthesised layers (Q5_K and Q6_K down) cycled over the 48 layer evaluations of each token."""
    sys.path.insert(0, str(ROOT / "tests"))
    import cases
    from oracle import oracle as O
    from pokitlms_b200 import synth
    c = CFG3
    layers = [cases.moe_layer(hidden=c["hidden"], inter=c["inter"], experts=c["experts"], top_k=c["top_k"],
                              seed=SEED, layer=l, flavour=1, down_type=(13 if l == 0 else 14),
                              shared_inter=c["shared_inter"], with_norm=True) for l in range(2)]
    if O.ref_available():
        kind, cores = "reference", min(6, max(2, (os.cpu_count() or 1) - 1))
        runners = [O.RefMoe(L) for L in layers]
        norm = O.ref_rms_norm

        def block(l, x):
            return runners[l % 2].forward(x)[0]
    else:
        kind, cores, norm = "port", 1, O.rms_norm

        def block(l, x):
            return O.moe_forward(layers[l % 2], x)[0]
    ones = np.ones(c["hidden"], dtype=np.float32)
    tokens, t0 = 0, time.perf_counter()
    while True:
        h = synth.activation(c["hidden"], SEED, 40_000 + tokens)
        for l in range(c["layers"]):
            h = (h + block(l, norm(h, ones, EPS))).astype(np.float32)
        tokens += 1
        el = time.perf_counter() - t0
        if el >= target_seconds:
            break
    return {"value": tokens / el, "unit": "tokens/s", "cores": cores, "kind": kind,
            "sample": f"{tokens} decode tokens x 48 MoE blocks (2 synthesised layers cycled), {el:.1f} s",
            **host_cpu()}


# Configuration 2 end to end: bytes one decoded token streams (experts and routers of 48
# layers, the attention projections, the LM head and one embedding row).
def decoder_token_bytes(shape) -> int:
    H, L = shape.hidden, shape.layers
    qd, kd = shape.q_heads * shape.head_dim, shape.kv_heads * shape.head_dim
    q4 = lambda rows, cols: rows * (cols // 256) * 144          # noqa: E731
    q6 = lambda rows, cols: rows * (cols // 256) * 210          # noqa: E731
    attn = q4(qd + 2 * kd, H) + q4(H, qd)
    experts = shape.top_k * (2 * q4(shape.expert_inter, H) + q4(H, shape.expert_inter))
    router = shape.experts * H * 4
    return L * (attn + experts + router) + q6(shape.vocab, H) + q6(1, H)


def decoder35_token_bytes(shape) -> int:
    """Bytes one Qwen3.5-MoE hybrid token step reads (weights, the DeltaNet
    states read and written, routed experts as 10 distinct slices)."""
    from pokitlms_b200._lib import BLOCK
    H = shape.hidden
    qd, kd = shape.q_heads * shape.head_dim, shape.kv_heads * shape.head_dim
    mat = lambda t, rows, cols: rows * (cols // BLOCK[t][0]) * BLOCK[t][1]   # noqa: E731
    a = shape.attn_type
    hv, vw, ch = shape.ssm_time_step_rank, shape.ssm_inner_size, shape.conv_channels
    state = hv * shape.ssm_state_size * (vw // hv) * 4
    total = mat(shape.output_type, shape.vocab, H) + mat(shape.embed_type, 1, H)
    for l in range(shape.layers):
        if shape.attention_layer(l):
            total += mat(a, 2 * qd + 2 * kd, H) + mat(a, H, qd)
        else:
            total += mat(a, ch + vw + 2 * hv, H) + mat(a, H, vw) + ch * shape.ssm_conv_kernel * 4 + 2 * state
        I, Is = shape.expert_inter, shape.shared_inter
        total += shape.experts * H * 4 + H * 4
        total += shape.top_k * (2 * mat(shape.expert_type, I, H) + mat(shape.down_type(l), H, I))
        total += 2 * mat(shape.shared_type, Is, H) + mat(shape.shared_type, H, Is)
    return total


def measure_decoder(device: int, stream, new_tokens: int = 128, layers: int = 48, hybrid: bool = False) -> dict:
    """Benchmark configuration 2 end to end: the whole synthetic Qwen3-30B-A3B-shaped
    decoder (48 layers, GQA 32/4 x 128, RoPE theta 1e6, FP16 KV ring, MoE 128 experts
    top-8, Q4_K experts and attention, Q6_K embedding and LM head, vocabulary 151,936),
    weights synthesised in HBM from seed 0, greedy decoding of `new_tokens` tokens after a
    32-token uniform-random prompt through pokit_cuda_decoder_generate_tokens (the
    reference's metric: generated tokens / decode time, host wall clock).  With `hybrid`,
    configuration 3's Qwen3.5-MoE hybrid (gguf.Qwen35MoeShape) the same way."""
    import torch
    from pokitlms_b200 import backend as B
    from pokitlms_b200 import gguf
    shape = gguf.Qwen35MoeShape(layers=layers) if hybrid else gguf.Qwen3MoeShape(layers=layers)
    dec = B.CudaDecoder(shape, device=device)
    dec.synthesize_model()
    prompt = np.random.default_rng([0, 0x7072]).integers(0, shape.vocab, 32)
    dec.generate_tokens(prompt, 8)                                   # warm-up, graphs captured
    ids, st = dec.generate_tokens(prompt, new_tokens)
    e2e = st["generated_tokens"] / (st["decode_time_ns"] * 1e-9)
    # Device-resident: token steps back to back (each samples the next on the device).
    dec.generate_tokens(prompt, 1)
    steps = min(new_tokens, shape.context - 40)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    dec.run_steps(steps, stream)
    b.record(stream)
    torch.cuda.synchronize()
    step_us = a.elapsed_time(b) * 1e3 / steps
    launches = dec.launches_per_step()
    graphs, why = dec.step_graphs()
    dec.close()
    peaks = measured_peaks()
    tb = decoder35_token_bytes(shape) if hybrid else decoder_token_bytes(shape)
    gbs = tb / (step_us * 1e-6) / 1e9
    what = ("benchmark configuration 3 end to end: {n}-layer synthetic Qwen3.5-MoE hybrid (Gated DeltaNet and "
            "gated full attention 3:1, MoE 512 experts top-10 + Q8_0 shared expert, Q6_K LM head over vocabulary "
            "151,936), 32-token prompt, greedy decode" if hybrid else
            "benchmark configuration 2 end to end: {n}-layer synthetic Qwen3-30B-A3B-shaped decoder "
            "(attention + MoE + Q6_K LM head over vocabulary 151,936), 32-token prompt, greedy decode")
    return {
        "workload": what.format(n=layers),
        "value": 1e6 / step_us, "unit": "tokens/s", "us_per_token": step_us,
        "e2e": {"value": e2e, "unit": "tokens/s", "generated": int(st["generated_tokens"]),
                "how": "pokit_cuda_decoder_generate_tokens: generated tokens / decode time (host clock), "
                       "prompt ids in, generated ids out", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 4},
        "hbm": {"bytes_per_token": tb, "achieved_gbs": gbs, "frac": gbs / peaks["hbm_gbs"],
                "peak_gbs": peaks["hbm_gbs"], "peak_source": peaks["source"]},
        "gpu_launches_per_token": int(launches),
        "step_graphs": graphs, **({"capture_refused": why} if why else {}),
        "first_ids": [int(i) for i in ids[:8]],
    }


def measured_tflops() -> float:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        for k in ("bf16_tflops", "bf16_tflops_burst"):
            if k in d:
                return float(d[k])
    return 1590.0


# Benchmark configuration 5's MoE path: Qwen3-235B-A22B-shaped, decode batch 64.
CFG5 = {"hidden": 4096, "inter": 1536, "experts": 128, "top_k": 8, "layers": 94, "tokens": 64}
CFG5_WORKLOAD = ("qwen3-235b-a22b-shaped MoE expert path: 94 MoE FFN layers (hidden 4096, 128 experts top-8 "
                 "renormalised, inter 1536, Q4_K experts, F32 router), decode batch 64")


def run_expert_parallel(args, rank: int, world: int, local: int, barrier, max_over_ranks,
                        shape: dict | None = None, emit: bool = True, steps: int | None = None,
                        warmup: int | None = None) -> dict:
    """Expert-parallel decode.  Default shape: configuration 2 with one token per
    rank per step (--workload ep-decode); `shape` = CFG5 runs configuration 5
    (64 tokens per step whatever the rank count), with a parity object (the
    all-reduced block output of layer 0 on the last step's rows against one
    whole-pool handle on rank 0, and whether every rank holds the same bits)
    and, for N > 1, the exchange step timed both ways (NCCL all-reduce of the
    [64, 4096] partial against the two all-to-alls of the same bytes that a
    dispatch/combine design would make).  Returns the line; prints it on rank 0
    when `emit`."""
    import argparse as _ap
    args = _ap.Namespace(**{**vars(args), **({"steps": steps} if steps else {}),
                            **({"warmup": warmup} if warmup else {})})
    import torch
    import torch.distributed as dist
    from pokitlms_b200 import synth
    from pokitlms_b200._lib import DOWN, FFN_NORM, GATE, ROUTER, UP
    from pokitlms_b200.ep import ExpertParallelMoe
    cfg5 = shape is not None
    Hs = shape["hidden"] if cfg5 else H
    Is = shape["inter"] if cfg5 else I
    layers = (args.layers if args.layers != LAYERS else shape["layers"]) if cfg5 else args.layers
    T = shape["tokens"] if cfg5 else world
    peer = world > 1 and args.ep_combine == "peer"
    ep = ExpertParallelMoe(rank=rank, world=world, layers=layers, hidden=Hs, inter=Is, experts=E, top_k=K_TOP,
                           rms_epsilon=EPS, device=local, exchange_tokens=T if peer else None)
    be = ep.backend
    ones = np.ones(Hs, dtype=np.float32)
    for l in range(layers):
        be.upload_tensor(l, ROUTER, synth.router_weights(E, Hs, SEED, l))
        be.upload_tensor(l, FFN_NORM, ones)
        for t in (GATE, UP, DOWN):
            be.synthesize_tensor(l, t, SEED, synth.stream_id(l, t))
    n_in = args.steps + args.warmup
    n_distinct = min(n_in, 16)
    inputs = torch.from_numpy(np.stack([np.stack([synth.activation(Hs, SEED + j, i) for j in range(T)])
                                        for i in range(n_distinct)])).cuda()      # [16][T][H]
    static_in = torch.empty(T, Hs, device="cuda")
    hidden = torch.empty(T, Hs, device="cuda")
    x = torch.empty(T, Hs, device="cuda")
    part = torch.empty(T, Hs, device="cuda")
    # Configuration 5 routes by per-layer synthetic logits N(0, 1): with random
    # weights the residual stream of this synthetic model collapses onto one
    # direction within a few layers, after which every token of the batch would
    # pick the same 8 experts; caller logits keep the spread of a real batch
    # (64 x 8 routes over 128 experts, nearly all experts touched per layer).
    route_logits = None
    if cfg5:
        rng = np.random.default_rng([SEED, 0x6c67])
        route_logits = torch.from_numpy(rng.standard_normal((layers, T, E), dtype=np.float32)).cuda()

    def body():
        hidden.copy_(static_in)
        for l in range(layers):
            # rms_norm with ffn_norm = 1 (src/rms_norm.cpp:9-27; torch's fused
            # kernel), then the block.
            xn = torch.nn.functional.rms_norm(hidden, (Hs,), eps=EPS)
            ep.forward_batch(l, xn, part, logits=None if route_logits is None else route_logits[l])
            hidden.add_(part)

    # Eager warm-up (sizes the batch scratch, sets kernel attributes), then the
    # whole step -- 48 blocks and their all-reduces -- captured once and
    # replayed: a step is otherwise bound by host-side launch cost.
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for i in range(3):
            static_in.copy_(inputs[i])
            body()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    l0 = be.stats()["kernel_launches"]
    static_in.copy_(inputs[0])
    body()
    torch.cuda.synchronize()
    launches_per_step = be.stats()["kernel_launches"] - l0
    graph = None
    try:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            body()
        torch.cuda.synchronize()
    except Exception as exc:   # capture refused: run eagerly and say so
        graph = None
        print(f"[bench] rank {rank}: CUDA graph capture failed ({exc}); timing eager steps", file=sys.stderr)
    barrier()

    def step(i):
        static_in.copy_(inputs[i % n_distinct], non_blocking=True)
        if graph is not None:
            graph.replay()
        else:
            body()

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)
    cur = torch.cuda.current_stream()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(cur)
    for i in range(args.steps):
        step(args.warmup + i)
    ev1.record(cur)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    be.synchronize()
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    gpu_launches = launches_per_step * args.steps
    ms_per_step = ms / args.steps

    # End to end: the step's hidden states from pinned host memory, the result back.
    host_in = inputs[:8].cpu().pin_memory()
    host_out = torch.empty(T, Hs).pin_memory()
    e2e_steps = max(args.steps // 2, 5)
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        static_in.copy_(host_in[i % host_in.shape[0]], non_blocking=True)
        if graph is not None:
            graph.replay()
        else:
            body()
        host_out.copy_(hidden, non_blocking=True)
        torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    # Device time of each kernel of one layer's batched block on this rank's shard
    # (local to the rank: no collective), on the last step's normalised rows.
    x.copy_(torch.nn.functional.rms_norm(hidden, (Hs,), eps=EPS))
    names = (["route", "group", "pack_x", "gate_up_gemm", "pack_act", "down_gemm", "combine"] if cfg5 else
             ["router", "route", "group", "pack_x", "gate_up_gemm", "pack_act", "down_gemm", "combine"])
    st = be.time_batch(0, x, part, logits=route_logits[0] if cfg5 else None, reps=20)
    stage_us = {"layer": 0, **{n_: round(v, 2) for n_, v in zip(names, st)}}
    parity = None
    if cfg5:
        from pokitlms_b200 import backend as B
        lg0 = route_logits[0]
        # Seeded rows (normalised N(0, 1)), not the synthetic model's late hidden state.
        xp = torch.from_numpy(np.stack([synth.activation(Hs, SEED + 7, 90_000 + t) for t in range(T)])).cuda()
        x.copy_(torch.nn.functional.rms_norm(xp, (Hs,), eps=EPS))
        ep.forward_batch(0, x, part, logits=lg0)          # the whole block's output on every rank
        torch.cuda.synchronize()
        sig = part.view(torch.int32).to(torch.int64).sum().reshape(1)
        sigs = [torch.zeros_like(sig) for _ in range(world)]
        if world > 1:
            dist.all_gather(sigs, sig)
        else:
            sigs = [sig]
        same = all(int(v) == int(sig) for v in sigs)
        if rank == 0:
            full = B.CudaMoeBackend(layers=1, hidden=Hs, inter=Is, experts=E, top_k=K_TOP, rms_epsilon=EPS,
                                    device=local)
            full.upload_tensor(0, ROUTER, synth.router_weights(E, Hs, SEED, 0))
            for t in (GATE, UP, DOWN):
                full.synthesize_tensor(0, t, SEED, synth.stream_id(0, t))
            ref = torch.empty_like(part)
            full.forward_batch(0, x, ref, logits=lg0)
            full.synchronize()
            full.close()
            err = ((part - ref).abs().amax(dim=1) / ref.pow(2).mean(dim=1).sqrt()).max()
            parity = {"tokens": T, "max_err_over_rms": float(err), "bar": 1e-3, "ranks_bitwise_equal": same,
                      "finite": bool(torch.isfinite(part).all().item() and torch.isfinite(ref).all().item()),
                      "reference": ("layer 0 on 64 seeded normalised rows with the step's logits: the expert-"
                                    "parallel sum against one whole-pool handle on rank 0")}
        barrier()
    exchange = None
    if world > 1:
        buf = torch.randn(T * Hs, device="cuda")
        out = torch.empty_like(buf)

        def timed(fn, reps=20):
            fn()
            torch.cuda.synchronize()
            barrier()
            ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ea.record()
            for _ in range(reps):
                fn()
            eb.record()
            torch.cuda.synchronize()
            return max_over_ranks(ea.elapsed_time(eb) * 1e3 / reps)

        def a2a2():
            dist.all_to_all_single(out, buf)
            dist.all_to_all_single(buf, out)

        exchange = {"bytes": T * Hs * 4, "all_reduce_us": timed(lambda: dist.all_reduce(buf)),
                    "all_to_all_x2_us": timed(a2a2),
                    "how": "NCCL, CUDA events on the rank, max over ranks, 20 back to back"}
    barrier()
    graph_used = graph is not None
    graph = None                      # release the graph (it holds NCCL calls) before the group goes
    torch.cuda.synchronize()
    peaks = measured_peaks()
    expert_bytes = 3 * Is * (Hs // 256) * 144
    if cfg5:
        # Distinct experts the step's routes touch on this rank: all of its shard in practice
        # (64 tokens x 8 routes over 128 experts), read once per layer.
        per_rank_bytes = ep.expert_count * expert_bytes
    else:
        per_rank_bytes = K_TOP * expert_bytes
    per_rank_gbs = per_rank_bytes / (ms_per_step / 1e3 / layers) / 1e9
    line = {
            "metric": METRIC, "value": T * args.steps / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "strong" if cfg5 else "weak", "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic (seed 0): Q4_K experts synthesised in HBM per shard, F32 router N(0,0.02)",
            "config": {"workload": (CFG5_WORKLOAD if cfg5 else WORKLOAD + f", expert parallel: {world} tokens "
                                    "per step (one per rank)"),
                       "tokens_per_step": T,
                       "routing": ("per-layer synthetic logits N(0,1) (caller logits)" if cfg5 else
                                   "the layer's F32 router"),
                       "layers": layers, "hidden": Hs, "experts": E, "top_k": K_TOP, "inter": Is,
                       "expert_type": "Q4_K", "parallelism": f"ep{world} (experts {E // world} per GPU, "
                       + ("combine over NVLink peer memory in the block's last kernel)" if peer else
                          "NCCL all-reduce combine)"), "cuda_graph": graph_used,
                       "l2": "no flush: each rank streams its shard's routed experts every layer"},
            "roofline": {"bound": "hbm", "kernel": "moe block per rank (grouped path + all-reduce)",
                         "achieved": per_rank_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": per_rank_gbs / peaks["hbm_gbs"], "traffic": None,
                         "bytes_per_block": per_rank_bytes,
                         "note": ("per rank and layer: the shard's expert slices the step reads (config 5: the "
                                  "whole shard; else 8 slices, distinct experts assumed) / (step time / layers)")},
            "e2e": {"value": T * e2e_steps / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": T * Hs * 4,
                    "d2h_bytes_per_step": T * Hs * 4},
            "gpu_launches": int(gpu_launches), "clocks": clocks, "cpu_baseline": None,
            **({"stage_us": stage_us} if stage_us else {}),
            **({"parity": parity} if parity else {}),
            **({"exchange": exchange} if exchange else {}),
    }
    if emit and rank == 0:
        print(json.dumps(line))
    ep.close()
    return line


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="pokit", choices=["pokit", "reference"])
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-config5", action="store_true", help="skip the configuration-5 object of the line")
    ap.add_argument("--ep-combine", default="nccl", choices=["peer", "nccl"],
                    help="N > 1: sum the shards' outputs in the block's last kernel over NVLink peer memory "
                         "(peer) or with an NCCL all-reduce (nccl)")
    ap.add_argument("--workload", default="decode", choices=["decode", "chain", "decoder", "decoder3", "grouped", "config3", "config5",
                             "ep-decode"],
                    help="decoder: only configuration 2's whole decoder (one GPU; --layers shortens it); "
                         "decoder3: only configuration 3's whole hybrid decoder (one GPU; --layers shortens it); "
                         "chain: only the decode chain of the headline (one GPU; --layers shortens it; a small "
                         "process for profiling moe_chain_kernel); "
                         "grouped: only the configuration-4 measurement (one GPU; a small process for "
                         "profiling the grouped kernels); config3: only the configuration-3 chain (one "
                         "GPU; --layers shortens it); config5: configuration 5 (94 layers, hidden "
                         "4096, batch 64) through the expert-parallel path on 1..N GPUs; ep-decode: configuration "
                         "2 with one token per rank per step through expert parallelism")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    import torch.distributed as dist
    from pokitlms_b200 import backend as B

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    layers = args.layers
    if args.workload == "grouped":
        if rank == 0:
            print(json.dumps({"metric": "configuration-4 grouped-expert batch tokens/s", "n_gpus": 1,
                              **measure_grouped(local, torch.cuda.current_stream())}))
        if world > 1:
            dist.destroy_process_group()
        return
    if args.workload in ("decoder", "decoder3"):
        if rank == 0:
            hybrid = args.workload == "decoder3"
            print(json.dumps({"metric": f"configuration-{3 if hybrid else 2} decoder tokens/s", "n_gpus": 1,
                              **measure_decoder(local, torch.cuda.current_stream(),
                                                layers=args.layers, hybrid=hybrid)}))
        if world > 1:
            dist.destroy_process_group()
        return
    if args.workload == "config3":
        if rank == 0:
            short = args.layers if args.layers != LAYERS else None
            print(json.dumps({"metric": "configuration-3 MoE chain tokens/s", "n_gpus": 1,
                              **measure_config3(local, torch.cuda.current_stream(), max(args.steps, 5),
                                                None if args.no_cpu_baseline else args.cpu_seconds,
                                                layers=short)}))
        if world > 1:
            dist.destroy_process_group()
        return
    if args.workload == "config5":
        run_expert_parallel(args, rank, world, local, barrier, max_over_ranks, shape=CFG5)
        if world > 1:
            dist.destroy_process_group()
        return
    if args.workload == "ep-decode":
        run_expert_parallel(args, rank, world, local, barrier, max_over_ranks)
        if world > 1:
            dist.destroy_process_group()
        return
    # N >= 1: every rank decodes its own sequence on its own copy of the model
    # (independent replicas: 16.3 GB fits one GPU's HBM), no data-path collective.
    be = B.CudaMoeBackend(layers=layers, hidden=H, inter=I, experts=E, top_k=K_TOP,
                          rms_epsilon=EPS, device=local)
    build_model(be, layers)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    from pokitlms_b200 import synth
    n_in = args.steps + args.warmup
    inputs = torch.from_numpy(np.stack([synth.activation(H, SEED + rank, i) for i in range(n_in)])).cuda()
    work = torch.empty(H, device="cuda")

    def step(i):
        work.copy_(inputs[i], non_blocking=True)
        be.decode_layers(0, layers, work, stream)

    for i in range(args.warmup):
        step(i)
    be.synchronize(stream)
    torch.cuda.synchronize()
    launches_before = be.stats()["kernel_launches"]

    sampler = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for i in range(args.steps):
        step(args.warmup + i)
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    be.synchronize(stream)
    ms = ev0.elapsed_time(ev1)
    ms_max = max_over_ranks(ms)
    gpu_launches = be.stats()["kernel_launches"] - launches_before
    tokens_per_s = world * args.steps / (ms_max / 1e3)
    ms_per_step = ms_max / args.steps

    # End to end through the C ABI host entry, pinned host buffers.
    host_in = torch.from_numpy(np.stack([synth.activation(H, SEED + rank, 50_000 + i)
                                         for i in range(64)])).pin_memory()
    host_out = torch.empty(H, dtype=torch.float32).pin_memory()
    e2e_steps = max(args.steps // 2, 10)
    for i in range(3):
        be.decode_layers_host(0, layers, host_in[i].numpy(), host_out.numpy())
    barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        be.decode_layers_host(0, layers, host_in[i % 64].numpy(), host_out.numpy())
    t1 = time.perf_counter()
    barrier()
    e2e_s = max_over_ranks(t1 - t0)
    e2e_rate = world * e2e_steps / e2e_s

    # Dominant kernel: the decode chain runs as one launch of moe_chain_kernel
    # per token.  Its average launch duration: CUDA events around launches back
    # to back (no host copies between them), after the timed region.
    reps = 50
    ka, kb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    be.decode_layers(0, layers, work, stream)
    ka.record(stream)
    for _ in range(reps):
        be.decode_layers(0, layers, work, stream)
    kb.record(stream)
    torch.cuda.synchronize()
    chain_us = ka.elapsed_time(kb) * 1e3 / reps
    phases = chain_phases(be, layers, work, stream)

    peaks = measured_peaks()
    block_s = ms_per_step / 1e3 / layers
    block_achieved = BLOCK_BYTES / block_s / 1e9
    routed_gbs = ROUTED_BYTES / block_s / 1e9
    chain_bytes = BLOCK_BYTES * layers
    achieved = chain_bytes / (chain_us / 1e6) / 1e9
    gu = phases["gate_up_us"]
    phases["gate_up_gbs"] = GATE_UP_BYTES / (gu * 1e-6) / 1e9
    phases["gate_up_frac"] = phases["gate_up_gbs"] / peaks["hbm_gbs"]

    # Replicas run the same weights: the same input must give the same bits on
    # every rank (and rank 0's is the single-GPU result).
    probe = synth.activation(H, SEED, 424_242)
    probe_out = np.empty(H, dtype=np.float32)
    be.decode_layers_host(0, layers, probe, probe_out)
    sig = torch.tensor([int(probe_out.view(np.int32).astype(np.int64).sum())], dtype=torch.int64, device="cuda")
    sigs = [torch.zeros_like(sig) for _ in range(world)]
    if world > 1:
        dist.all_gather(sigs, sig)
    else:
        sigs = [sig]
    parity = {"replicas_bitwise_equal": all(int(v) == int(sig) for v in sigs), "ranks": world,
              "probe": f"one {layers}-layer chain on a common seeded input, bit signature gathered from every rank",
              "finite": bool(np.all(np.isfinite(probe_out)))}

    chain_only = args.workload == "chain"
    one_gpu = world == 1 and not chain_only
    decoder = measure_decoder(local, stream) if one_gpu else None
    decoder3 = measure_decoder(local, stream, hybrid=True) if one_gpu else None
    grouped = measure_grouped(local, stream) if one_gpu else None
    config3 = (measure_config3(local, stream, steps=max(args.steps // 10, 20),
                               cpu_seconds=None if (args.no_cpu_baseline or rank != 0) else 6.0)
               if one_gpu else None)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, kind, cores, sample = cpu_reference_rate(args.cpu_seconds)
        cpu = {"value": v, "unit": "tokens/s", "cores": cores, "kind": kind, "sample": sample, **host_cpu()}
        # One configuration-4 token is one block evaluation of the same shape.
        if grouped is not None:
            grouped["cpu_baseline"] = {"value": v * LAYERS, "unit": "tokens/s", "cores": cores, "kind": kind,
                                       "sample": sample + "; one config-4 token = one of those block evaluations"}

    # Configuration 5 (expert parallel over all ranks, strong scaling): the
    # replica model is released first (the whole-pool config-5 model is 128 GB
    # on one GPU).
    be.close()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    config5 = None
    if not chain_only and not args.no_config5:
        config5 = run_expert_parallel(args, rank, world, local, barrier, max_over_ranks, shape=CFG5, emit=False,
                                      steps=20, warmup=3)
        for k in ("metric", "n_gpus", "higher_is_better", "vs_baseline", "dtype", "cpu_baseline"):
            config5.pop(k, None)

    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": tokens_per_s, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seed 0): Q4_K experts synthesised in HBM, F32 router N(0,0.02)",
            "config": {"workload": WORKLOAD, "layers": layers, "hidden": H, "experts": E,
                       "top_k": K_TOP, "inter": I, "expert_type": "Q4_K",
                       "parallelism": ("single GPU" if world == 1 else
                                       f"{world} independent replicas: each GPU decodes its own sequence on its "
                                       "own copy of the 16.3 GB model, no data-path collective; expert "
                                       "parallelism is the config5 object"),
                       "l2": "no flush: each step streams 1.07 GB of distinct weights (> 126 MB L2)"},
            "routed_expert_gbs": routed_gbs,
            "routed_expert_frac_of_peak": routed_gbs / peaks["hbm_gbs"],
            "roofline": {"bound": "hbm", "kernel": "moe_chain_kernel (48 MoE blocks, one cooperative launch)",
                         "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / peaks["hbm_gbs"], "peak_source": peaks["source"],
                         "bytes_per_launch": chain_bytes, "avg_launch_us": chain_us,
                         "traffic": ncu_traffic_bytes(layers),
                         "traffic_source": TRAFFIC_SOURCE},
            "block_roofline": {"bound": "hbm", "kernel": "moe block (one layer of the chain kernel)",
                               "achieved": block_achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                               "frac": block_achieved / peaks["hbm_gbs"], "bytes_per_block": BLOCK_BYTES},
            "chain_phases": phases,
            "e2e": {"value": e2e_rate, "unit": "tokens/s", "h2d_bytes_per_step": H * 4,
                    "d2h_bytes_per_step": H * 4},
            "gpu_launches": int(gpu_launches),
            "clocks": clocks,
            "cpu_baseline": cpu,
            **({"decoder": decoder} if decoder is not None else {}),
            **({"config3_decoder": decoder3} if decoder3 is not None else {}),
            **({"grouped": grouped} if grouped is not None else {}),
            **({"config3": config3} if config3 is not None else {}),
            "parity": parity,
            **({"config5": config5} if config5 is not None else {}),
        }))
    if world > 1:
        # Every graph that held NCCL calls is gone with its frame; collect any
        # cycle still holding one before the communicators go.
        import gc
        gc.collect()
        torch.cuda.synchronize()
        barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
