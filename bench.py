#!/usr/bin/env python
"""Benchmark: the OLMoE-1B-7B-shaped MoE hot path on B200.

One step = one pass of T tokens through the 16 MoE blocks of an OLMoE-1B-7B-
shaped model (hidden 2048, 64 experts, top-8, SwiGLU intermediate 1024, bf16
weights ~N(0, 0.02), seeded; inputs ~N(0, 1)).  Each block is the engine's MoE
block, x += MoE(rmsnorm(x)) (rabbit2.c:512-542).  The default T = 1 is batch-1
decode; --tokens 4096 is the prefill-sized layer call.

  value  tokens/s over the whole job, device-timed with CUDA events, inputs and
         weights resident in HBM (16 layers x 805 MB of weights per step, so the
         working set is ~100x the 126 MB L2: no flush needed);
  e2e    the same metric through the engine-facing C call with host buffers
         (rbt_moe_block: pinned host x in, x and routing out, per layer);
  roofline of the dominant kernel, from per-stage CUDA-event timing in a
         separate profiled pass, against MEASURED_PEAKS.json;
  cpu_baseline the reference's own CPU MoE layer (rabbit2.c compiled, through
         oracle/_ref) on the host cores, on a bounded sample.

--impl reference times only that CPU path (rank 0) and prints its line.
--workload model-decode / model-prefill time the whole forward() of an
OLMoE-1B-7B-shaped model on one GPU instead (rbt_model_forward per generated
token, config 3; rbt_model_prefill for one prompt, config 4's unit of work).
Multi-GPU (torchrun, N ranks): expert parallelism.  Rank g holds experts
[g*64/N, (g+1)*64/N) of every layer and its own T tokens; each layer is one
rbt_moe_ep_block_device call per GPU: local routing, each token's row stored once
into every GPU that owns one of its experts (peer memory over NVLink), the
experts, the partial rows stored back, and the combine in rank order -- no host
synchronisation, the 16 layers one CUDA graph.  value = N*T tokens / max-over-ranks
step time (weak scaling: T tokens per GPU); the line carries a parity check of
rank 0's tokens against the CPU oracle and the per-stage time of a layer.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

D, H, E, K, LAYERS = 2048, 1024, 64, 8, 16
METRIC = "olmoe_moe_stack_tok_per_s"
UNIT = "tok/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="rabbit2_b200", choices=["rabbit2_b200", "reference"])
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--routing", default="natural", choices=["natural", "zipf"])
    ap.add_argument("--path", type=int, default=0, help="0 auto, 1 GEMV, 2 tcgen05 GEMM")
    ap.add_argument("--profile-steps", type=int, default=5)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="moe", choices=["moe", "model-decode", "model-prefill", "model-batch"],
                    help="moe: the MoE stack (the metric's config); model-decode: the whole forward() of an "
                         "OLMoE-1B-7B-shaped model, batch-1 greedy decode (config 3); model-prefill: the same "
                         "model's prompt of --prompt tokens in one rbt_model_prefill call (config 4, one sequence); "
                         "model-batch: 64 sequences at context 2048 decoded together with the Zipf router "
                         "bias (config 5; expert-parallel under torchrun)")
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--gen", type=int, default=256)
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the other configs' keys of the line (N=1: moe_T16, moe_T4096, model_prefill, "
                         "model_decode with its reference-engine baseline, model_batch_decode; N>1: "
                         "moe_T16_ep, moe_T4096_ep, model_batch_decode)")
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def workload_desc(args):
    return {"workload": f"olmoe1b7b_moe_stack_{args.layers}L_T{args.tokens}_{args.routing}",
            "tokens_per_step_per_gpu": args.tokens, "layers": args.layers, "dim": D, "expert_hidden": H,
            "n_experts": E, "top_k": K, "weights": "bf16 ~N(0,0.02) seeded, .rbt2 expert blobs",
            "inputs": "f32 ~N(0,1) seeded", "routing": args.routing,
            "l2": "working set 16 x 805 MB weights per step >> 126 MB L2 (no flush needed)",
            "parallelism": f"ep{args.gpus}" if args.gpus > 1 else "single"}


# ----------------------------------------------------------------------------- CPU reference

def host_layers(n, seed0, device):
    """Host copies (router bf16 bits, expert blobs) of n seeded OLMoE layers."""
    from rabbit2_b200 import workload
    out = []
    for l in range(n):
        router, experts, stride = workload.device_layer(D, H, E, seed=seed0 + l, device=device)
        out.append(workload.host_copy(router, experts) + (stride,))
        del router, experts
    return out


def cpu_reference_run(args, seconds=None, steps=None, warmup=0, device="cuda"):
    """Time the reference CPU MoE block (oracle/_ref, else the C restatement).

    A step is the bench step's work on a bounded sample of its tokens: one layer
    call per layer over `sample` tokens (weights of 2 distinct layers, cycled:
    each is 805 MB, far beyond any CPU cache).  Returns (tok/s, info)."""
    from oracle.oracle import MoeLayerHost, Oracle, Reference, available_reference
    from rabbit2_b200 import workload
    if available_reference():
        lib, kind = Reference(), "reference"
        kernel = "avx2" if lib.set_kernel(True) else "scalar"
    else:
        lib, kind, kernel = Oracle(), "port", "scalar"
    ncores = len(os.sched_getaffinity(0))
    sample = min(args.tokens, ncores)
    threads = max(1, min(sample, ncores))
    layers = host_layers(2, seed0=1, device=device)
    bias = workload.zipf_bias(E, 1.2, seed=0) if args.routing == "zipf" else None
    hosts = [MoeLayerHost(D, H, E, K, 1, 0, r, e, s, ffn_norm=np.ones(D, np.float32), router_bias=bias)
             for (r, e, s) in layers]
    x = np.random.default_rng(1000).standard_normal((sample, D)).astype(np.float32)

    def one_step():
        y = x
        for l in range(args.layers):
            y, _ = lib.moe_block(hosts[l % 2], y, nthreads=threads)
        return y

    for _ in range(warmup):
        one_step()
    t0, n = time.perf_counter(), 0
    while True:
        one_step()
        n += 1
        el = time.perf_counter() - t0
        if (steps is not None and n >= steps) or (seconds is not None and el >= seconds):
            break
    value = sample * n / el
    info = {"kind": kind, "cores": threads,
            "sample": f"{n} steps x {args.layers} MoE blocks x {sample} token(s), rabbit2.c --kernel {kernel}, "
                      f"{threads} thread(s) of {ncores} host cores; {el:.1f} s",
            "host_cpu": cpu_model()}
    return value, info, el / n * 1e3


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args, rank):
    if rank != 0:
        return
    try:
        import torch
        device = "cuda" if torch.cuda.is_available() else "cpu"
    except ImportError:
        device = "cpu"
    value, info, ms = cpu_reference_run(args, steps=args.steps, warmup=args.warmup, device=device)
    cfg = workload_desc(args)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": cfg,
            "cpu_baseline": dict(info, value=value, unit=UNIT),
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU

class ClockSampler:
    """SM clock and throttle-reason samples taken while the timed region runs.

    A host thread polls NVML every ~2 ms from just before the first timed launch until the
    closing synchronize, so even a timed region of a few milliseconds is sampled under load.
    The GPU is found by its PCI bus id, so the index order of NVML and CUDA does not matter.
    Falls back to `nvidia-smi -lms 200` where NVML is not importable.
    """
    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4), ("hw_power_brake_slowdown", 0x80))

    def __init__(self, device_index, period_s=0.002):
        self.device_index, self.period = device_index, period_s
        self.samples, self.max_mhz, self.error = [], None, None

    def _handle(self, nvml):
        import torch
        p = torch.cuda.get_device_properties(self.device_index)
        bus = getattr(p, "pci_bus_id", None)
        if bus is not None:
            busid = "%08X:%02X:%02X.0" % (getattr(p, "pci_domain_id", 0), bus, getattr(p, "pci_device_id", 0))
            try:
                return nvml.nvmlDeviceGetHandleByPciBusId_v2(busid)
            except Exception:
                pass
        return nvml.nvmlDeviceGetHandleByIndex(self.device_index)

    def _poll(self, nvml, h):
        while not self._stop.is_set():
            try:
                mhz = nvml.nvmlDeviceGetClockInfo(h, nvml.NVML_CLOCK_SM)
                mask = nvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((float(mhz), int(mask)))
            except Exception as exc:  # keep the bench going; report why there are no samples
                self.error = repr(exc)
                return
            self._stop.wait(self.period)

    def __enter__(self):
        import threading
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml as nvml
            nvml.nvmlInit()
            h = self._handle(nvml)
            self.max_mhz = float(nvml.nvmlDeviceGetMaxClockInfo(h, nvml.NVML_CLOCK_SM))
            self._thread = threading.Thread(target=self._poll, args=(nvml, h), daemon=True)
            self._thread.start()
        except Exception as exc:
            self.error = repr(exc)
            self._smi = None
            try:
                self._smi = subprocess.Popen(
                    ["nvidia-smi", "-i", str(self.device_index), "--query-gpu=clocks.sm,clocks.max.sm,"
                     "clocks_event_reasons.active", "--format=csv,noheader,nounits", "-lms", "200"],
                    stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            except OSError:
                pass
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)
            return
        smi = getattr(self, "_smi", None)
        if smi is None:
            return
        smi.terminate()
        try:
            out, _ = smi.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            smi.kill()
            out, _ = smi.communicate()
        for line in out.splitlines():
            parts = [p.strip() for p in line.split(",")]
            try:
                self.samples.append((float(parts[0]), int(parts[2], 16)))
                self.max_mhz = float(parts[1])
            except (ValueError, IndexError):
                pass

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["no clock samples: %s" % self.error]}
        reasons = sorted({n for _, m in self.samples for n, bit in self.REASONS if m & bit})
        return {"sm_mhz": statistics.median(s for s, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples),
                "sm_mhz_min": min(s for s, _ in self.samples), "source": "nvml" if self._thread else "nvidia-smi"}


# DRAM bytes (read + write) per launch of the dominant kernel, from one ncu capture of the same
# workload (natural routing); the profile summary named beside each figure holds the capture.
MEASURED_TRAFFIC = {
    ("decode_fused", 1): (101.294080e6 + 3.348480e6, "profiles/decode_fused_olmoe_T1.md"),
    ("gate_up", 4096): (843.422976e6 + 124.197632e6, "profiles/prefill_tc_olmoe_T4096.md"),
}


def stage_cost(T, U, S):
    """Algorithmic HBM bytes and FLOPs per launch of each stage (bf16 weights, f32 activations)."""
    w = 2
    bytes_ = {"rmsnorm": T * D * 4 * 2 + D * 4,
              "router": E * D * w + T * D * 4 + T * K * 8,
              "gate_up": U * 2 * H * D * w + T * D * 4 + S * H * 4,
              "down": U * H * D * w + S * H * 4 + S * D * 4,
              "combine": S * D * 4 + T * D * 4 * 2 + S * 8,
              "gather": T * D * 4 + S * D * 4,
              # the one-token kernel: router + the U experts' three matrices + x in and out
              "decode_fused": E * D * w + U * 3 * H * D * w + T * D * 4 * 2}
    flops = {"router": 2 * T * E * D, "gate_up": 4 * S * H * D, "down": 2 * S * H * D,
             "decode_fused": T * (2 * E * D + 6 * K * H * D)}
    return bytes_, flops


def run_ep(args, rank, world, local_rank):
    """Expert-parallel step over `world` GPUs, one process each (rbt_moe_ep_*): rank g
    holds experts [g*64/N, (g+1)*64/N) of every layer and its own T tokens; each layer
    is one library call per GPU (route, peer-memory dispatch over NVLink, experts,
    return, combine; no host synchronisation), the 16 layers one CUDA graph."""
    import torch
    import torch.distributed as dist

    from oracle.oracle import MoeLayerHost, Oracle
    from rabbit2_b200 import ep, moe, workload

    dev = torch.device("cuda", local_rank)
    T, L = args.tokens, args.layers
    epr = E // world
    e0 = rank * epr
    stride = workload.layer_stride(D, H)
    ctx = moe.MoeContext(D, E, K, H, L, moe.DT_BF16, 0, stride, device=local_rank)
    ctx.set_path(args.path)
    ctx.ep_init(rank, world, T)
    ones = torch.ones(D, device=dev)
    keep = []
    bias = workload.zipf_bias(E, 1.2, seed=0) if args.routing == "zipf" else None
    full0 = None
    for l in range(L):
        router, experts, _ = workload.device_layer(D, H, E, seed=1 + l, device=dev)
        local = experts[e0:e0 + epr].clone()
        if l == 0 and rank == 0:
            full0 = workload.host_copy(router, experts)
        del experts
        ctx.bind_layer(l, router, local, ones)
        keep.append((router, local))
        if bias is not None:
            ctx.set_router_bias(l, bias)
    ctx.reserve(world * T)
    ep.connect(ctx)
    x0 = workload.inputs(T, D, seed=1000 + rank, device=dev)
    x = torch.empty_like(x0)
    st = torch.cuda.Stream(device=dev)

    def step():
        x.copy_(x0)
        for l in range(L):
            ctx.ep_block_device(l, x, stream=st)

    # parity before timing: rank 0's first tokens through layer 0 against the CPU oracle
    parity = None
    n_chk = min(8, T)
    xc = x0[:n_chk].clone()
    rc = torch.empty(n_chk, K, dtype=torch.int32, device=dev)
    with torch.cuda.stream(st):
        ctx.ep_block_device(0, xc if rank == 0 else x0[:0], rc if rank == 0 else None, T=n_chk if rank == 0 else 0,
                            stream=st)
    torch.cuda.synchronize()
    status = ctx.status()
    if rank == 0:
        r_h, e_h = full0
        host = MoeLayerHost(D, H, E, K, moe.DT_BF16, 0, r_h, e_h, stride, ffn_norm=np.ones(D, np.float32),
                            router_bias=bias)
        want, want_r = Oracle().moe_block(host, x0[:n_chk].cpu().numpy(), nthreads=8)
        got = xc.cpu().numpy()
        xin = x0[:n_chk].cpu().numpy()
        parity = {"checked": True, "tokens": n_chk, "layer": 0,
                  "routing_equal": bool(np.array_equal(rc.cpu().numpy(), want_r)),
                  "max_rel_err": float(np.abs((got - xin) - (want - xin)).max() / np.abs(want - xin).max()),
                  "status": status, "against": "oracle/ MoE block (CPU), all 64 experts"}
    del full0

    with torch.cuda.stream(st):
        for _ in range(max(args.warmup, 3)):
            step()
    torch.cuda.synchronize()
    # routed slots per expert of one step: each rank's local counts, gathered
    hist = torch.zeros(E, dtype=torch.int64, device=dev)
    U_sum = 0
    with torch.cuda.stream(st):
        x.copy_(x0)
        for l in range(L):
            ctx.ep_block_device(l, x, stream=st)
            torch.cuda.synchronize()
            loc = torch.zeros(E, dtype=torch.int64, device=dev)
            loc[e0:e0 + epr] = torch.from_numpy(ctx.expert_histogram()[:epr].astype(np.int64)).to(dev)
            dist.all_reduce(loc)
            hist += loc
            U_sum += int((loc > 0).sum())
    U = U_sum / L
    ctx.profile(timing=0, reset=True)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        step()
    launches_per_step = ctx.profile(reset=True)["launches"]
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(st):
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        with ClockSampler(local_rank) as clocks:
            ev0.record(st)
            for _ in range(args.steps):
                g.replay()
            ev1.record(st)
            torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / args.steps
    bad = ctx.status()
    t = torch.tensor([ms, float(bad != 0)], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, any_bad = float(t[0].item()), bool(t[1].item())
    value = world * T / (ms / 1e3)

    # per-stage device time: a second graph with event nodes at every stage boundary
    ctx.profile(timing=1, reset=True)
    gp = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gp, stream=st):
        step()
    stage_ms = {}
    with torch.cuda.stream(st):
        for _ in range(args.profile_steps):
            gp.replay()
            torch.cuda.synchronize()
            for n, v in ctx.profile()["stage_ms"].items():
                stage_ms[n] = stage_ms.get(n, 0.0) + v
    ctx.profile(timing=0, reset=True)
    del gp
    stage_us_per_layer = {n: v / args.profile_steps / L * 1e3 for n, v in stage_ms.items() if v > 0}

    # e2e: this rank's tokens from pinned host memory in, the block output back, every step
    xh = x0.cpu().pin_memory()
    oh = torch.empty_like(xh).pin_memory()

    def host_step():
        with torch.cuda.stream(st):
            x.copy_(xh, non_blocking=True)
            for l in range(L):
                ctx.ep_block_device(l, x, stream=st)
            oh.copy_(x, non_blocking=True)
        st.synchronize()

    for _ in range(max(args.warmup, 3)):
        host_step()
    dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        host_step()
    e2e_ms = (time.perf_counter() - t0) * 1e3 / args.steps
    t = torch.tensor([e2e_ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())
    e2e = {"value": world * T / (e2e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": T * D * 4,
           "d2h_bytes_per_step": T * D * 4,
           "how": "rbt_moe_ep_block_device per layer on this rank's tokens copied in from pinned host memory, "
                  "output copied back, wall clock, max over ranks (per-rank bytes)"}

    hbm, bf16, src = peaks()
    layer_ms = ms / L
    layer_bytes = world * E * D * 2 + U * 3 * H * D * 2 + world * T * D * 4 * 2 + world * T * K * 8
    layer_flops = world * T * (2 * E * D + 6 * K * H * D)
    gbs = layer_bytes / world / (layer_ms / 1e3) / 1e9
    tfs = layer_flops / world / (layer_ms / 1e3) / 1e12
    tensor_bound = tfs / bf16 > gbs / hbm
    roofline = {"bound": "tensor" if tensor_bound else "hbm", "kernel": "ep_layer",
                "achieved": tfs if tensor_bound else gbs, "peak": bf16 if tensor_bound else hbm,
                "unit": "TFLOP/s" if tensor_bound else "GB/s",
                "frac": (tfs / bf16) if tensor_bound else (gbs / hbm), "peak_source": src, "traffic": None,
                "timing": "CUDA events around the timed graph replays (the 16 layers' library calls), max over "
                          "ranks; per GPU: the job's algorithmic bytes or flops of a layer / N / layer time",
                "layer": {"us_per_layer": layer_ms * 1e3, "algorithmic_bytes_job": layer_bytes,
                          "algorithmic_flops_job": layer_flops, "distinct_experts_per_layer": U,
                          "experts_per_gpu": epr,
                          "stage_us_per_layer": stage_us_per_layer}}
    out = None
    if rank == 0:
        out = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
               "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": workload_desc(args),
               "clocks": clocks.summary(), "e2e": e2e, "gpu_launches": launches_per_step * args.steps,
               "roofline": roofline, "expert_histogram": hist.cpu().tolist(), "parity": parity,
               "ep_status_error": any_bad}
    del g
    torch.cuda.synchronize()
    ctx.close()
    return out


def run_ours(args, rank, world, local_rank):
    if world > 1:
        return run_ep(args, rank, world, local_rank)
    import torch
    import torch.distributed as dist
    from rabbit2_b200 import moe, workload

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    T, L = args.tokens, args.layers
    stride = workload.layer_stride(D, H)
    ctx = moe.MoeContext(D, E, K, H, L, moe.DT_BF16, 0, stride, device=local_rank)
    ctx.set_path(args.path)
    ones = torch.ones(D, device=dev)
    keep = []
    bias = workload.zipf_bias(E, 1.2, seed=0) if args.routing == "zipf" else None
    for l in range(L):
        router, experts, _ = workload.device_layer(D, H, E, seed=1 + l, device=dev)
        ctx.bind_layer(l, router, experts, ones)
        keep.append((router, experts))
        if bias is not None:
            ctx.set_router_bias(l, bias)
    ctx.reserve(T)
    x0 = workload.inputs(T, D, seed=1000 + rank, device=dev)
    x = torch.empty_like(x0)

    def step():
        st = torch.cuda.current_stream()
        x.copy_(x0)
        for l in range(L):
            ctx.block_device(l, x, stream=st)

    def barrier():
        if world > 1:
            dist.barrier()

    # eager warm-up, and the routed-expert statistics of every layer
    s = torch.cuda.Stream(device=dev)
    hist = np.zeros(E, np.int64)
    U_sum = 0
    with torch.cuda.stream(s):
        for _ in range(max(args.warmup, 3)):
            step()
        x.copy_(x0)
        for l in range(L):
            ctx.block_device(l, x, stream=s)
            h = ctx.expert_histogram()
            hist += h
            U_sum += int((h > 0).sum())
    torch.cuda.synchronize()
    U = U_sum / L

    # the timed step is a CUDA graph of the 16 layer calls (5 kernels each)
    ctx.profile(timing=0, reset=True)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    launches_per_step = ctx.profile(reset=True)["launches"]
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        with ClockSampler(local_rank) as clocks:
            ev0.record(s)
            for _ in range(args.steps):
                g.replay()
            ev1.record(s)
            torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / args.steps
    barrier()
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = world * T / (ms / 1e3)

    # e2e through the engine-facing host call: pinned x in, x + routing out, per layer
    xh = torch.empty((T, D), dtype=torch.float32, pin_memory=True)
    rh = torch.empty((T, K), dtype=torch.int32, pin_memory=True)
    x0h = x0.cpu()
    lib, handle = ctx.lib, ctx.handle

    def host_step():
        xh.copy_(x0h)
        for l in range(L):
            if not lib.rbt_moe_block(handle, l, xh.data_ptr(), T, rh.data_ptr(), K):
                raise moe.RbtMoeError(lib.rbt_moe_last_error().decode())

    for _ in range(max(args.warmup, 3)):
        host_step()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        host_step()
    e2e_ms = (time.perf_counter() - t0) * 1e3 / args.steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e = {"value": world * T / (e2e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": L * T * D * 4,
           "d2h_bytes_per_step": L * (T * D * 4 + T * K * 4),
           "how": "rbt_moe_block per layer (host x in, x and routing out, synchronous), pinned host memory, "
                  "wall clock"}

    # profiled replays: a second graph with event-record nodes at every stage boundary
    ctx.profile(timing=1, reset=True)
    gp = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gp):
        step()
    prof_launch = ctx.profile(timing=-1)["stage_launches"]
    stage_ms = {}
    with torch.cuda.stream(s):
        for _ in range(args.profile_steps):
            gp.replay()
            torch.cuda.synchronize()
            for n, v in ctx.profile()["stage_ms"].items():
                stage_ms[n] = stage_ms.get(n, 0.0) + v
    ctx.profile(timing=0, reset=True)
    del gp
    S = T * K
    bytes_per, flops_per = stage_cost(T, U, S)
    per_launch_ms = {n: stage_ms[n] / (prof_launch[n] * args.profile_steps)
                     for n in bytes_per if prof_launch.get(n)}
    dom = max(per_launch_ms, key=lambda n: per_launch_ms[n] * prof_launch[n])
    timing = "CUDA events recorded as nodes of a captured graph of the step"
    if set(per_launch_ms) == {dom}:
        # one kernel per layer: the timed graph itself gives its launch duration, free of
        # the event nodes (which also break the launch overlap between layers)
        per_launch_ms[dom] = ms / prof_launch[dom]
        timing = "CUDA events around the timed graph replays; the step is one kernel per layer"
    traffic = MEASURED_TRAFFIC.get((dom, T)) if args.routing == "natural" else None
    hbm, bf16, src = peaks()
    layer_bytes = E * D * 2 + U * 3 * H * D * 2 + T * D * 4 * 2 + T * K * 8
    layer_flops = T * (2 * E * D + 6 * K * H * D)
    layer_ms = ms / L
    t_dom = per_launch_ms[dom] / 1e3
    gbs = bytes_per[dom] / t_dom / 1e9
    tfs = flops_per.get(dom, 0) / t_dom / 1e12
    tensor_bound = tfs / bf16 > gbs / hbm
    roofline = {"bound": "tensor" if tensor_bound else "hbm", "kernel": dom,
                "achieved": tfs if tensor_bound else gbs, "peak": bf16 if tensor_bound else hbm,
                "unit": "TFLOP/s" if tensor_bound else "GB/s",
                "frac": (tfs / bf16) if tensor_bound else (gbs / hbm), "peak_source": src,
                "traffic": traffic[0] if traffic else None,
                "traffic_source": traffic[1] if traffic else None,
                "algorithmic_bytes_per_launch": bytes_per[dom], "algorithmic_flops_per_launch": flops_per.get(dom, 0),
                "avg_launch_ms": per_launch_ms[dom],
                "stage_ms_per_launch": per_launch_ms,
                "stage_share": {n: per_launch_ms[n] * prof_launch[n] / sum(per_launch_ms[k] * prof_launch[k]
                                                                            for k in per_launch_ms)
                                for n in per_launch_ms},
                "timing": timing,
                "layer": {"us_per_layer": layer_ms * 1e3, "algorithmic_bytes": layer_bytes,
                          "algorithmic_flops": layer_flops,
                          "hbm_frac": layer_bytes / (layer_ms / 1e3) / 1e9 / hbm,
                          "tensor_frac": layer_flops / (layer_ms / 1e3) / 1e12 / bf16,
                          "distinct_experts_per_layer": U}}
    out = None
    if rank == 0:
        out = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
               "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": workload_desc(args),
               "clocks": clocks.summary(), "e2e": e2e, "gpu_launches": launches_per_step * args.steps,
               "roofline": roofline, "expert_histogram": hist.tolist()}
    del g
    ctx.close()
    return out


# ----------------------------------------------------------------------------- configs 3 and 4

def olmoe_model(args, ctx_len, ep=None, device=0):
    """A random-init OLMoE-1B-7B-shaped model (args.layers layers, vocab 50304, bf16
    weights ~N(0, 0.02) from a seeded GPU generator, norms 1): assembled as the bytes
    of its .rbt2 file in host memory (the engine's own view of the model, which the
    reference engine can run), then uploaded from there into an RbtModel with a KV
    cache of ctx_len positions.  ep = (rank, n_ranks, max_tokens): the model is that
    rank of an expert-parallel group, and only its experts are written into the
    image and uploaded (the same draws as the whole model's).  Returns (cfg, model,
    image)."""
    import torch

    from rabbit2_b200 import model as model_mod
    from rabbit2_b200.rbt2fmt import BLOB_ALIGN, DT_BF16, HEADER_BYTES, ModelConfig, layout, pack_header
    cfg = ModelConfig(vocab=50304, dim=D, n_layers=args.layers, n_heads=16, n_kv_heads=16, head_dim=128,
                      n_experts=E, top_k=K, expert_hidden=H, max_seq=max(4096, ctx_len), dtype=DT_BF16, qk_norm=1,
                      norm_topk=0, rope_theta=10000.0, rms_eps=1e-5)
    lay = layout(cfg)
    image = torch.empty(-(-lay["total"] // BLOB_ALIGN) * BLOB_ALIGN, dtype=torch.uint8)
    image[:HEADER_BYTES] = torch.frombuffer(bytearray(pack_header(cfg)), dtype=torch.uint8)
    dev = torch.device("cuda", device)
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    e0, n_local = 0, E
    if ep is not None:
        n_local = E // ep[1]
        e0 = ep[0] * n_local

    def put_mat(off, rows, cols, first=0, n=None):  # drawn on the GPU, rows [first, first+n) into the image
        n = rows if n is None else n
        t = (torch.randn(rows, cols, generator=g, device=dev) * 0.02).to(torch.bfloat16)[first:first + n]
        off += first * cols * 2
        image[off:off + n * cols * 2].copy_(t.view(torch.uint8).reshape(-1))

    def put_ones(off, n):
        image[off:off + 4 * n].view(torch.float32).fill_(1.0)

    put_mat(lay["tok_emb"], cfg.vocab, D)
    for ly in lay["layers"]:
        put_ones(ly["attn_norm"], D)
        for name in ("wq", "wk", "wv"):
            put_mat(ly[name], 16 * 128, D)
        put_mat(ly["wo"], D, 16 * 128)
        put_ones(ly["q_norm"], 16 * 128)
        put_ones(ly["k_norm"], 16 * 128)
        put_ones(ly["ffn_norm"], D)
        put_mat(ly["router"], E, D)
        assert lay["expert_stride"] == 3 * H * D * 2
        put_mat(ly["experts"], E, 3 * H * D, e0, n_local)
    put_ones(lay["final_norm"], D)
    put_mat(lay["lm_head"], cfg.vocab, D)
    torch.cuda.synchronize(dev)
    m = model_mod.ModelContext(cfg, ctx=ctx_len, device=device)
    if ep is not None:
        m.moe().ep_init(*ep)
    base = image.data_ptr()
    lib, h = m.lib, m.handle
    m._call(lib.rbt_model_load_globals, h, base + lay["tok_emb"], base + lay["final_norm"], base + lay["lm_head"])
    for l, ly in enumerate(lay["layers"]):
        ptrs = [base + ly[n] for n in ("attn_norm", "wq", "wk", "wv", "wo", "q_norm", "k_norm", "ffn_norm", "router")]
        m._call(lib.rbt_model_load_layer, h, l, *ptrs, base + ly["experts"] + e0 * lay["expert_stride"])
    return cfg, m, image


def run_model_prefill(args, built=None):
    """Config 4's unit of work on one GPU: one sequence of --prompt uniform-random
    tokens through the whole model in one rbt_model_prefill call (host tokens in,
    the last token's logits and every routing row out).  value = prompt tokens
    per second of wall clock around the call, averaged over --steps calls after
    --warmup (each call rewrites the same cache positions)."""
    cfg, m, _ = built if built is not None else olmoe_model(args, args.prompt)
    prompt = np.random.default_rng(1).integers(0, cfg.vocab, size=args.prompt)
    import torch
    nw = max(1, args.warmup)
    for w in range(nw):
        if w == nw - 1:  # the last warm-up call is the one an ncu run with --profile-from-start off captures
            torch.cuda.cudart().cudaProfilerStart()
        m.prefill(prompt, 0, logit_rows=1)
    torch.cuda.cudart().cudaProfilerStop()
    times = []
    with ClockSampler(0) as clocks:
        for _ in range(args.steps):
            t0 = time.perf_counter()
            m.prefill(prompt, 0, logit_rows=1)
            times.append(time.perf_counter() - t0)
    if built is None:
        m.close()
    dt = statistics.mean(times)
    T, L = args.prompt, cfg.n_layers
    nq = nkv = 16 * 128
    flops = {"attention projections": 2 * T * L * (nq + 2 * nkv + nq) * D,
             "attention scores and values (causal)": 2 * 2 * L * 16 * 128 * T * (T + 1) / 2,
             "moe": T * L * (2 * E * D + 6 * K * H * D), "lm_head (last token)": 2 * cfg.vocab * D}
    total = sum(flops.values())
    _, tf, src = peaks()
    return {"metric": "olmoe1b7b_full_model_prefill_tok_per_s", "value": T / dt, "unit": "tok/s", "n_gpus": 1,
            "steps": args.steps, "warmup": max(1, args.warmup), "ms_per_step": dt * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config4_olmoe1b7b_full_model_prefill_one_sequence", "layers": L,
                       "prompt": T, "vocab": cfg.vocab, "dim": D, "heads": 16, "head_dim": 128,
                       "n_experts": E, "top_k": K, "expert_hidden": H,
                       "weights": "bf16 ~N(0,0.02) seeded (norms 1)",
                       "timing": "wall clock per rbt_model_prefill call"},
            "clocks": clocks.summary(),
            "roofline": {"bound": "tensor", "achieved": total / dt / 1e12, "peak": tf, "unit": "TFLOP/s",
                         "frac": total / dt / 1e12 / tf, "peak_source": src, "flops_per_step": total,
                         "flops_parts": flops, "traffic": None}}


def run_model_decode(args, built=None):
    """Config 3: the whole forward() (rbt_model_forward: attention, MoE, lm_head) of a
    random-init OLMoE-1B-7B-shaped model on one GPU -- a uniform-random prompt of
    --prompt tokens, then --gen greedy tokens with the KV cache, as the engine's
    --gen loop does (logits to the host, argmax there).  value = generated tokens
    per second of wall clock around the calls (host round trip per token
    included); prefill_tok_s is the prompt fed token by token."""
    cfg, m, _ = built if built is not None else olmoe_model(args, args.prompt + args.gen)
    prompt = np.random.default_rng(1).integers(0, cfg.vocab, size=args.prompt)
    # warm-up: graph capture and first launches (positions are rewritten below); the
    # last warm-up token is the one an ncu run with --profile-from-start off captures
    import torch
    nw = min(3, args.prompt)
    for p in range(nw):
        if p == nw - 1:
            torch.cuda.cudart().cudaProfilerStart()
        m.forward(int(prompt[p]), p, logits=True)
    torch.cuda.cudart().cudaProfilerStop()
    t0 = time.perf_counter()
    for p in range(args.prompt):
        logits, _ = m.forward(int(prompt[p]), p, logits=p == args.prompt - 1)
    t1 = time.perf_counter()
    ids, pos = [], args.prompt
    with ClockSampler(0) as clocks:
        t2 = time.perf_counter()
        for _ in range(args.gen):
            nxt = int(np.argmax(logits))
            ids.append(nxt)
            logits, _ = m.forward(nxt, pos)
            pos += 1
        t3 = time.perf_counter()
    if built is None:
        m.close()
    hbm, _, src = peaks()
    dt = (t3 - t2) / args.gen
    nq = nkv = 16 * 128
    avg_ctx = args.prompt + (args.gen + 1) / 2
    per_token = {"attention weights": cfg.n_layers * (nq + 2 * nkv + nq) * D * 2,
                 "moe weights": cfg.n_layers * (E * D * 2 + K * 3 * H * D * 2),
                 "lm_head": cfg.vocab * D * 2,
                 "kv cache (f32, mean context)": cfg.n_layers * avg_ctx * nkv * 4 * 2}
    total = sum(per_token.values())
    return {"metric": "olmoe1b7b_full_model_decode_tok_per_s", "value": 1.0 / dt, "unit": "tok/s", "n_gpus": 1,
            "steps": args.gen, "warmup": 3, "ms_per_step": dt * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config3_olmoe1b7b_full_model_batch1_decode", "layers": cfg.n_layers,
                       "prompt": args.prompt, "gen": args.gen, "vocab": cfg.vocab, "dim": D, "heads": 16,
                       "head_dim": 128, "n_experts": E, "top_k": K, "expert_hidden": H,
                       "weights": "bf16 ~N(0,0.02) seeded (norms 1)", "timing": "wall clock per forward call"},
            "prefill_tok_s": args.prompt / (t1 - t0), "clocks": clocks.summary(),
            "gpu_launches": (2 + 4 * cfg.n_layers) * args.gen,
            "roofline": {"bound": "hbm", "achieved": total / dt / 1e9, "peak": hbm, "unit": "GB/s",
                         "frac": total / dt / 1e9 / hbm, "peak_source": src, "bytes_per_token": total,
                         "bytes_per_token_parts": per_token, "traffic": None},
            "generated_ids_head": ids[:8]}


def run_model_batch(args, rank=0, world=1, local_rank=0, seqs=64, ctx_len=2048, steps=10, warmup=3,
                    prefill_tokens=4096):
    """Config 5: batched decode of `seqs` concurrent sequences per GPU at context
    ctx_len, the router biased by a Zipf(1.2) expert popularity (the same prior on
    every layer), one rbt_model_decode_batch call per step (one token of every
    sequence: host tokens and positions in, greedy ids and routing rows out).  Each
    sequence's KV cache is first filled by rbt_model_prefill_seq with
    ctx_len - warmup - steps uniform-random tokens, so the timed steps run at
    positions up to ctx_len - 1.  With N > 1 ranks the model is expert-parallel
    (rank g holds experts [g*64/N, (g+1)*64/N) and its own `seqs` sequences; every
    MoE block goes through the group).  value = N * seqs tokens / max-over-ranks
    wall time per call; the per-expert histogram counts the routed slots of the
    timed steps (summed over layers and ranks).  Before the caches are filled, the same
    model (natural routing) times config 4's split: one prompt of `prefill_tokens`
    tokens per GPU through rbt_model_prefill, every MoE block through the group
    (the `prefill` key: N * prefill_tokens tokens / max-over-ranks wall time per call)."""
    import torch
    import torch.distributed as dist

    from rabbit2_b200 import ep as ep_mod
    from rabbit2_b200 import workload
    m_args = argparse.Namespace(**vars(args))
    m_args.layers = LAYERS
    prompt_len = ctx_len - warmup - steps
    epcfg = (rank, world, max(prompt_len, seqs, prefill_tokens)) if world > 1 else None
    cfg, m, image = olmoe_model(m_args, max(ctx_len, prefill_tokens), ep=epcfg, device=local_rank)
    del image
    try:
        if world > 1:
            ep_mod.connect(m.moe())
            m.moe().ep_set_timeout(30_000_000_000)  # the ranks' first calls (cuBLAS set-up) start apart
        prompt = np.random.default_rng(200 + rank).integers(0, cfg.vocab, size=prefill_tokens)
        for _ in range(2):
            m.prefill(prompt, 0, logit_rows=1)
        if world > 1:
            dist.barrier()
        with ClockSampler(local_rank) as p_clocks:
            t0 = time.perf_counter()
            for _ in range(3):
                m.prefill(prompt, 0, logit_rows=1)
            p_dt = (time.perf_counter() - t0) / 3
        if world > 1:
            t = torch.tensor([p_dt], device=f"cuda:{local_rank}")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            p_dt = float(t.item())
        prefill = {"metric": "olmoe1b7b_full_model_prefill_tok_per_s", "value": world * prefill_tokens / p_dt,
                   "unit": "tok/s", "ms_per_call": p_dt * 1e3, "calls": 3, "warmup": 2,
                   "config": {"workload": "config4_split_one_prompt_per_gpu", "prompt_per_gpu": prefill_tokens,
                              "parallelism": f"ep{world}" if world > 1 else "single GPU", "routing": "natural",
                              "timing": "wall clock per rbt_model_prefill call, max over ranks"},
                   "clocks": p_clocks.summary()}
        bias = workload.zipf_bias(E, 1.2, seed=0)
        for l in range(cfg.n_layers):
            m.set_router_bias(l, bias)
        m.set_sequences(seqs)
        rng = np.random.default_rng(100 + rank)
        t0 = time.perf_counter()
        for i in range(seqs):
            m.prefill_seq(i, rng.integers(0, cfg.vocab, size=prompt_len), 0, logit_rows=0)
        t_fill = time.perf_counter() - t0
        toks = rng.integers(0, cfg.vocab, size=seqs)
        pos = np.full(seqs, prompt_len, np.int32)
        for w in range(warmup):
            if w == warmup - 1:  # the last untimed step is the one an ncu run with
                torch.cuda.cudart().cudaProfilerStart()  # --profile-from-start off captures
            toks, _, _ = m.decode_batch(toks, pos)
            pos += 1
        torch.cuda.cudart().cudaProfilerStop()
        routed = []
        if world > 1:
            dist.barrier()
        with ClockSampler(local_rank) as clocks:
            t0 = time.perf_counter()
            for _ in range(steps):
                toks, _, rt = m.decode_batch(toks, pos)
                pos += 1
                routed.append(rt)
            dt = (time.perf_counter() - t0) / steps
        # per step and layer: each expert's routed slots (this rank's rows)
        counts = np.stack([[np.bincount(rt[:, l].reshape(-1), minlength=E) for l in range(cfg.n_layers)]
                           for rt in routed])
        hist = counts.sum(axis=0)
        if world > 1:
            c = torch.from_numpy(counts).to(f"cuda:{local_rank}")
            dist.all_reduce(c)
            counts = c.cpu().numpy()
        if world > 1:
            t = torch.tensor([dt], device=f"cuda:{local_rank}")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dt = float(t.item())
            h = torch.from_numpy(hist).to(f"cuda:{local_rank}")
            dist.all_reduce(h)
            hist = h.cpu().numpy()
    finally:
        m.close()
    per_expert = hist.sum(axis=0)
    hbm, _, src = peaks()
    nq = nkv = 16 * 128
    mean_ctx = prompt_len + warmup + (steps + 1) / 2
    touched = float((counts > 0).sum()) / steps  # distinct experts of a step, summed over layers (whole job)
    per_step = {"attention weights": cfg.n_layers * (nq + 2 * nkv + nq) * D * 2,
                "kv cache (f32, every sequence)": seqs * cfg.n_layers * mean_ctx * nkv * 4 * 2,
                "router weights": cfg.n_layers * E * D * 2,
                "expert weights (distinct experts of the step / N)": touched / world * 3 * H * D * 2,
                "lm_head": cfg.vocab * D * 2}
    total = sum(per_step.values())
    return {"metric": "olmoe1b7b_batched_decode_tok_per_s", "value": world * seqs / dt, "unit": "tok/s",
            "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": dt * 1e3,
            "higher_is_better": True, "scaling": "weak",
            "config": {"workload": "config5_olmoe1b7b_batched_decode_zipf", "sequences_per_gpu": seqs,
                       "ctx": ctx_len, "positions_timed": [prompt_len + warmup, prompt_len + warmup + steps - 1],
                       "layers": cfg.n_layers, "routing": "zipf(1.2) router bias, every layer",
                       "parallelism": f"ep{world}" if world > 1 else "single GPU",
                       "timing": "wall clock per rbt_model_decode_batch call (host tokens in, greedy ids and "
                                 "routing rows out), max over ranks",
                       "l2": "KV caches of 34 GB per GPU >> 126 MB L2"},
            "kv_fill_s": t_fill, "clocks": clocks.summary(), "prefill": prefill,
            "roofline": {"bound": "hbm", "achieved": total / dt / 1e9, "peak": hbm, "unit": "GB/s",
                         "frac": total / dt / 1e9 / hbm, "peak_source": src, "bytes_per_step_per_gpu": total,
                         "bytes_parts": per_step, "traffic": None},
            "expert_histogram": per_expert.tolist(),
            "expert_imbalance_max_over_mean": float(per_expert.max() / max(per_expert.mean(), 1e-9))}


# ----------------------------------------------------------------------------- the other configs, N = 1

def reference_engine_decode(built, prompt_tokens=4, gen=4):
    """The reference engine's own decode loop (rabbit2.c compiled as is, through
    oracle/_ref: forward() per token, argmax between) on the same model bytes the GPU
    model was uploaded from: `prompt_tokens` prompt tokens, then `gen` greedy tokens,
    --kernel avx2 (its faster kernel), one thread (the engine is single-threaded).
    The GPU model decodes the same prompt, and the greedy ids are compared."""
    from oracle.oracle import Reference, available_reference
    if not available_reference():
        return {"unavailable": "oracle/_ref not built (the reference source was absent at build time)"}
    cfg, m, image = built
    prompt = np.random.default_rng(2).integers(0, cfg.vocab, size=prompt_tokens)
    ref = Reference()
    t0 = time.perf_counter()
    ids, t_prompt, t_gen = ref.decode_image(image.data_ptr(), image.numel(), prompt, gen, avx2=True)
    wall = time.perf_counter() - t0
    got = []
    logits = None
    for p, tok in enumerate(prompt):
        logits, _ = m.forward(int(tok), p)
    for i in range(gen):
        nxt = int(np.argmax(logits))
        got.append(nxt)
        if i + 1 < gen:
            logits, _ = m.forward(nxt, prompt_tokens + i)
    return {"value": gen / t_gen, "unit": "tok/s", "kind": "reference", "cores": 1,
            "prompt_tok_s": prompt_tokens / t_prompt, "host_cpu": cpu_model(),
            "greedy_ids_equal": got == ids.tolist(), "greedy_ids": ids.tolist(),
            "sample": f"the engine's decode loop (oracle/_ref, --kernel avx2, 1 thread) on the same "
                      f"{cfg.n_layers}-layer model: {prompt_tokens} prompt tokens then {gen} greedy tokens, "
                      f"{wall:.1f} s"}


def run_extras(args):
    """The other BASELINE configs as keys of the N = 1 line, each measured here with
    its own clocks: the MoE stack at T = 4096 (the prefill-sized layer call whose
    GEMMs carry the bf16 target), config 4's unit (one 4096-token prompt through the
    whole model) and config 3 (batch-1 decode of 256 tokens after a 512-token
    prompt, with the reference engine timed beside it)."""
    import argparse as ap
    import copy

    import torch
    out = {}
    a16 = copy.copy(args)
    a16.tokens, a16.steps, a16.warmup, a16.profile_steps = 16, 50, 5, 2
    l16 = run_ours(a16, 0, 1, 0)
    out["moe_T16"] = {k: l16[k] for k in ("metric", "value", "unit", "ms_per_step", "steps", "warmup", "config",
                                          "clocks", "e2e", "roofline")}
    torch.cuda.empty_cache()
    a = copy.copy(args)
    a.tokens, a.steps, a.warmup, a.profile_steps = 4096, 5, 3, 2
    line = run_ours(a, 0, 1, 0)
    torch.cuda.empty_cache()
    rf = line["roofline"]
    _, flops = stage_cost(4096, rf["layer"]["distinct_experts_per_layer"], 4096 * K)
    _, bf16, src = peaks()
    gemm = {n: flops[n] / (rf["stage_ms_per_launch"][n] / 1e3) / 1e12 / bf16
            for n in ("gate_up", "down") if n in rf["stage_ms_per_launch"]}
    out["moe_T4096"] = {"metric": METRIC, "value": line["value"], "unit": UNIT, "ms_per_step": line["ms_per_step"],
                        "steps": a.steps, "warmup": a.warmup, "config": line["config"], "clocks": line["clocks"],
                        "e2e": line["e2e"], "gpu_launches": line["gpu_launches"], "roofline": rf,
                        "gemm_frac_of_bf16": gemm, "layer_frac_of_bf16": rf["layer"]["tensor_frac"],
                        "peak_source": src}
    m_args = ap.Namespace(**vars(args))
    m_args.layers = LAYERS
    built = olmoe_model(m_args, 4096)
    try:
        p_args = copy.copy(m_args)
        p_args.prompt, p_args.steps, p_args.warmup = 4096, 3, 1
        out["model_prefill"] = run_model_prefill(p_args, built)
        d_args = copy.copy(m_args)
        d_args.prompt, d_args.gen = 512, 256
        out["model_decode"] = run_model_decode(d_args, built)
        out["model_decode"]["cpu_baseline"] = reference_engine_decode(built)
    finally:
        built[1].close()
    del built
    torch.cuda.empty_cache()
    out["model_batch_decode"] = run_model_batch(args)
    return out


def main():
    args = parse()
    if args.workload == "model-decode":
        print(json.dumps(run_model_decode(args)), flush=True)
        return
    if args.workload == "model-prefill":
        print(json.dumps(run_model_prefill(args)), flush=True)
        return
    if args.workload == "model-batch" and int(os.environ.get("WORLD_SIZE", "1")) == 1:
        print(json.dumps(run_model_batch(args, steps=args.steps, warmup=max(3, args.warmup))), flush=True)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    args.gpus = world
    if args.impl == "reference":
        run_reference(args, rank)
        return
    import datetime

    import torch
    import torch.distributed as dist
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        line = run_ours(args, rank, world, local_rank)
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            v, info, _ = cpu_reference_run(args, seconds=args.cpu_seconds, device="cuda")
            line["cpu_baseline"] = dict(info, value=v, unit=UNIT)
        if world == 1 and not args.no_extras and args.tokens == 1:
            line.update(run_extras(args))
        if world > 1 and not args.no_extras:
            # config 4's split (4096 tokens per GPU through the expert-parallel stack)
            # and config 5 (64 sequences per GPU), every rank taking part
            import copy
            torch.cuda.empty_cache()
            a16 = copy.copy(args)
            a16.tokens, a16.steps, a16.warmup, a16.profile_steps = 16, 20, 3, 1
            r16 = run_ep(a16, rank, world, local_rank)
            torch.cuda.empty_cache()
            a4 = copy.copy(args)
            a4.tokens, a4.steps, a4.warmup, a4.profile_steps = 4096, 3, 3, 1
            r4 = run_ep(a4, rank, world, local_rank)
            torch.cuda.empty_cache()
            r5 = run_model_batch(args, rank, world, local_rank)
            if rank == 0:
                rf = r4["roofline"]
                line["moe_T4096_ep"] = {k: r4[k] for k in ("metric", "value", "unit", "ms_per_step", "steps",
                                                          "warmup", "config", "clocks", "parity",
                                                          "ep_status_error")}
                line["moe_T4096_ep"]["roofline"] = rf
                line["moe_T16_ep"] = {k: r16[k] for k in ("metric", "value", "unit", "ms_per_step", "steps",
                                                          "warmup", "config", "clocks", "parity", "roofline",
                                                          "ep_status_error")}
                line["model_batch_decode"] = r5
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
