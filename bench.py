#!/usr/bin/env python
"""MoE decode benchmark of the B200 expert path (BASELINE.json metric:
"MoE decode tokens/s; expert-GEMV HBM GB/s (% of 8 TB/s)").

Workload (N=1 line): BASELINE config 2 -- one full-width MoE layer at batch-1
decode: hidden 3072, 512 experts, expert FFN 768, top-8 routing over
Zipf(1.1)-skewed router logits, one always-on shared expert, gate/up/down Q2_K
from N(0, 0.02) weights, f32 activations ~ N(0, 1), all experts HBM-resident.
A step = one token through the layer: route, fused gate/up GEMV + SwiGLU +
shared expert, down GEMV, weighted combine -- one launch of the fused layer
kernel (four launches on the per-op path). The timed loop cycles
through 32 independently generated copies of the layer (38 GB), so every step
reads expert weights that the L2 (126 MB) no longer holds.

  python bench.py [--gpus N --steps K --warmup W]       # this implementation
  python bench.py --impl reference [...]                 # CPU reference arm

N > 1 (under torchrun): expert-parallel decode -- every layer copy's 512
experts are split over the N GPUs (512 / N each, the shared expert on every
GPU), every GPU brings its own batch-1 token per step, and each step is one
launch per GPU of the layer kernel with the exchange inside it (tokens
gathered, down rows returned and summed over NVLink peer memory); value = all
ranks' tokens / max-over-ranks time. Rank 0 checks its outputs against a
full copy of the layer decoded on its own GPU and reports the difference.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

H, F, E, K_TOP = 3072, 768, 512, 8
Q2_K = 10
EXPERT_BYTES = 768 * (3072 // 256) * 84          # one Q2_K expert matrix: 774,144 B
GATEUP_BYTES = (K_TOP + 1) * 2 * EXPERT_BYTES     # per gate/up launch (8 routed + shared)
DOWN_BYTES = (K_TOP + 1) * EXPERT_BYTES
STEP_BYTES = GATEUP_BYTES + DOWN_BYTES            # 20,901,888 B per token
METRIC = "MoE decode tokens/s; expert-GEMV HBM GB/s (% of 8 TB/s) at 1/2/4/8 B200"
WORKLOAD = "config2: full-width MoE layer (H=3072, E=512, F=768, top-8 Zipf(1.1) + shared expert, Q2_K), batch-1 decode"


def parse():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100000)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--impl", choices=["mine", "reference"], default="mine")
    ap.add_argument("--layers", type=int, default=32, help="independent layer copies cycled by the timed loop")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="bounded CPU-baseline sample")
    ap.add_argument("--e2e-steps", type=int, default=2000)
    ap.add_argument("--config", type=int, choices=[1, 2, 3, 4, 5], default=2,
                    help="BASELINE config; 2 (default) is the headline line, 1/3/4/5 print their own lines")
    ap.add_argument("--prompt", type=int, default=512, help="prefill tokens per rank (config 4)")
    ap.add_argument("--stack-layers", type=int, default=48, help="layers of the config-3/4 stack (48 in BASELINE)")
    ap.add_argument("--kernel-shares", action="store_true",
                    help="config 4: also print each kernel's share of the device time (torch profiler, rank 0)")
    ap.add_argument("--ep-exchange", choices=["p2p", "nccl"], default="p2p",
                    help="config 4 dispatch/combine: peer-memory kernels (default) or NCCL all-to-all")
    ap.add_argument("--batch", type=int, default=1, help="decode tokens per step (configs 3 and 5)")
    ap.add_argument("--launch", choices=["stack", "layer"], default="stack",
                    help="config 2 on one GPU: 512 steps per persistent launch (stack) or one launch per step "
                         "replayed from CUDA graphs (layer)")
    return ap.parse_args()


def zipf_logits(n_tok, seed, alpha=1.1):
    rng = np.random.default_rng(seed)
    perm = rng.permutation(E)
    base = -alpha * np.log(perm + 1.0)
    return (base[None, :] + rng.normal(0.0, 1.0, size=(n_tok, E))).astype(np.float32)


def token_pool(n, seed):
    rng = np.random.default_rng(seed)
    x = rng.normal(0.0, 1.0, size=(n, H)).astype(np.float32)
    return x, zipf_logits(n, seed + 1)


# ---------------------------------------------------------------------------
# CPU side: the oracle's llama.cpp-semantics layer on the host cores
# ---------------------------------------------------------------------------
def cpu_layer_sample(seconds, n_threads, layer_seed=0, pool_seed=1234):
    """Time the CPU restatement of llama.cpp's MoE layer (Q8_K activations,
    generic vec_dot) on config 2, weights generated for the experts the sampled
    tokens route to. Returns (tokens/s, steps, seconds)."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle as O
    n_pool = 16
    x, logits = token_pool(n_pool, pool_seed)
    ids, _ = O.topk_softmax(logits, K_TOP)
    used = sorted(set(ids.reshape(-1).tolist()))
    rb_h, rb_f = O.row_size(Q2_K, H), O.row_size(Q2_K, F)
    W = {r: np.zeros((E, F if r != "down" else H, rb_h if r != "down" else rb_f), np.uint8) for r in ("gate", "up", "down")}
    for i, r in enumerate(("gate", "up", "down")):
        rows, cols = (F, H) if r != "down" else (H, F)
        for e in used:
            O.fill_quantized(Q2_K, W[r][e], e * rows, rows, cols, seed=layer_seed * 1000003 + i, n_threads=n_threads)
    shared = {}
    for i, r in enumerate(("gate", "up", "down")):
        rows, cols = (F, H) if r != "down" else (H, F)
        buf = np.zeros((rows, O.row_size(Q2_K, cols)), np.uint8)
        O.fill_quantized(Q2_K, buf, 0, rows, cols, seed=layer_seed * 1000003 + 7 + i, n_threads=n_threads)
        shared[r] = buf
    L = dict(H=H, F=F, E=E, k=K_TOP, type_gate=Q2_K, type_up=Q2_K, type_down=Q2_K, gate=W["gate"], up=W["up"],
             down=W["down"], shared_type=Q2_K, shared_gate=shared["gate"], shared_up=shared["up"],
             shared_down=shared["down"])
    O.moe_layer(L, x[:1], logits[:1], n_threads=n_threads)       # warm
    steps, t0 = 0, time.perf_counter()
    while True:
        i = steps % n_pool
        O.moe_layer(L, x[i:i + 1], logits[i:i + 1], n_threads=n_threads)
        steps += 1
        el = time.perf_counter() - t0
        if el >= seconds and steps >= 3:
            break
    return steps / el, steps, el


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    per_step_s = None
    tps, steps, el = cpu_layer_sample(min(args.cpu_seconds, 20.0), cores)
    per_step_s = 1.0 / tps
    line = {
        "impl": "reference", "metric": METRIC, "value": round(tps, 3), "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": steps, "warmup": 1, "ms_per_step": round(per_step_s * 1e3, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": WORKLOAD, "global_batch": 1, "parallelism": "host cores"},
        "cpu_baseline": {"value": round(tps, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{steps} decode tokens of one config-2 layer ({el:.1f} s), CPU restatement of "
                                   "llama.cpp's MUL_MAT_ID (oracle/, Q8_K activations), not llama.cpp itself"},
        "e2e": {"value": round(tps, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "llama.cpp is not present on this machine; the reference arm times this repo's CPU restatement "
                "of its MUL_MAT_ID path",
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU side
# ---------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id):
        self.gpu = gpu_id
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0, t1):
        rows = [l for (t, l) in self.lines if t0 <= t <= t1] or [l for (_, l) in self.lines]
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            f = [c.strip() for c in r.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def run_mine(args):
    import torch
    import torch.distributed as dist
    import importlib
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        return run_mine_ep(args)
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    pkg = importlib.import_module("a6000-custom-kernels_b200")
    mc = pkg.moe_cache
    mc.configure(enabled=True)
    R = args.layers
    layers = [pkg.MoELayer(H, F, E, K_TOP, {"gate": Q2_K, "up": Q2_K, "down": Q2_K}, shared=True, device=dev,
                           seed=rank * 1000 + l, name=f"blk.{l}") for l in range(R)]
    P = 64
    xs_np, lg_np = token_pool(P, 1234 + rank)
    xs = torch.from_numpy(xs_np).to(dev).view(P, 1, H)
    lgs = torch.from_numpy(lg_np).to(dev).view(P, 1, E)
    outs = torch.empty((P, 1, H), device=dev)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize()

    def step(i):
        layers[i % R].decode(xs[i % P], lgs[i % P], outs[i % P], stream=stream)

    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, R)):
            step(i)
    torch.cuda.synchronize()
    assert mc.device_error(stream) == 0

    # CUDA graphs of the timed sequence: G-step chunks plus a remainder, so the
    # timed region is exactly K steps
    G = 512
    K = args.steps
    graphs = {}

    def graph_for(n, start):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for j in range(n):
                step(start + j)
        return g

    use_stack = args.launch == "stack"
    if use_stack:
        # G steps per persistent launch: the layer list repeats every G steps
        # (G is a multiple of the 32 layer copies and of the 64 tokens)
        def stack_for(n):
            return pkg.Stack([layers[j % R] for j in range(n)], [xs[j % P] for j in range(n)],
                             [lgs[j % P] for j in range(n)], [outs[j % P] for j in range(n)], stream=stream)
        st_full = stack_for(G) if K >= G else None
        st_rem = stack_for(K % G) if K % G else None

        class _Run:
            def __init__(self, st):
                self.st = st

            def replay(self):
                self.st.run(stream)
        full = _Run(st_full) if st_full is not None else None
        rem = _Run(st_rem) if st_rem is not None else None
    else:
        full = graph_for(G, 0) if K >= G else None
        rem = graph_for(K % G, 0) if K % G else None
    # warm the graphs / stacks (W warm-up steps already ran eagerly)
    with torch.cuda.stream(stream):
        if full is not None:
            full.replay()
        if rem is not None:
            rem.replay()
    torch.cuda.synchronize()

    clocks = ClockSampler("GPU-" + str(torch.cuda.get_device_properties(dev).uuid))
    clocks.start()
    # keep the GPU busy while the sampler starts
    t_end = time.time() + 0.5
    with torch.cuda.stream(stream):
        while time.time() < t_end:
            (full or rem).replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wall0 = time.time()
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for _ in range(K // G):
            full.replay()
        if rem is not None:
            rem.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    wall1 = time.time()
    if world > 1:
        dist.barrier()
    clocks.stop()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    assert mc.device_error(stream) == 0
    value = world * K / (ms / 1e3)

    # ---- dominant kernel: the fused gate/up GEMV, timed per launch -------------
    kern = time_gateup_kernel(pkg, layers, xs, dev, stream, n=min(max(K, 256), 4096))

    # ---- end to end through the public API with host buffers ------------------
    e2e = run_e2e(pkg, layers, xs_np, lg_np, dev, stream, args.e2e_steps)
    if world > 1:
        t = torch.tensor([e2e["seconds"]], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e["seconds"] = float(t.item())
    e2e_value = world * e2e["steps"] / e2e["seconds"]

    peaks = {}
    try:
        peaks = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    peak = peaks.get("hbm_gbs")
    peak_src = "of measured" if peak else "of fallback"
    peak = peak or 6650.0
    fused = layers[0].fused(1)
    if use_stack:
        k_us = 1e3 * ms / K
        k_bytes = STEP_BYTES
        k_name = "moe_stack_kernel<Q2_K,Q2_K>: 512 layer steps per persistent launch (route, gate/up+SwiGLU+shared, down, combine per step)"
        k_how = f"timed region: {K} steps in {-(-K // G)} persistent launches, per-step time"
        tfile = "stack_kernel_traffic.json"
    elif fused:
        # one launch per step: the timed region's per-step time is the layer
        # kernel's launch-to-launch time (an upper bound of its duration)
        k_us = 1e3 * ms / K
        k_bytes = STEP_BYTES
        k_name = "moe_layer_kernel<Q2_K,Q2_K,1>: whole layer in one launch (route, gate/up+SwiGLU+shared, down, combine)"
        k_how = f"timed region: {K} back-to-back launches in CUDA graphs, per-step time"
        tfile = "layer_kernel_traffic.json"
    else:
        k_us, k_bytes = kern["us"], GATEUP_BYTES
        k_name = "moe_gemv_kernel<Q2_K> fused gate/up+SwiGLU+shared"
        k_how = kern["how"]
        tfile = "gemv_gateup_traffic.json"
    achieved = k_bytes / (k_us * 1e-6) / 1e9
    traffic = None
    tpath = os.path.join(REPO, "profiles", tfile)
    if os.path.exists(tpath):
        try:
            traffic = json.load(open(tpath)).get("bytes_per_launch")
        except (OSError, ValueError):
            traffic = None

    cpu = None
    if rank == 0 and world == 1 and args.cpu_seconds > 0:
        cores = os.cpu_count() or 1
        tps, steps, el = cpu_layer_sample(args.cpu_seconds, cores)
        cpu = {"value": round(tps, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"{steps} batch-1 decode tokens of one config-2 layer ({el:.1f} s) through the CPU "
                         "restatement of llama.cpp's MUL_MAT_ID (oracle/), all host threads"}

    if rank == 0:
        ck = clocks.summary(wall0, wall1)
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": round(ms / K, 6), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": WORKLOAD, "global_batch": world, "seq_len": 1,
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                       "layers_cycled": R, "l2": f"inputs larger than L2: {R} layer copies "
                                                 f"({R * 3 * E * EXPERT_BYTES / 1e9:.1f} GB) cycled",
                       "graph": ("persistent launches of 512 steps" if use_stack else "CUDA graphs of 512-step chunks")},
            "layer_gbs": round(STEP_BYTES * value / world / 1e9, 1),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_src,
                         "frac_of_8TBs": round(achieved / 8000.0, 4), "traffic": traffic,
                         "kernel": k_name, "bytes_per_launch": k_bytes, "us_per_launch": round(k_us, 3),
                         "timing": k_how},
            "per_op_gemv": {"kernel": "moe_gemv_kernel<Q2_K> (ggml_cuda_moe_cache_mul_mat_vec_q, the drop-in op)",
                            "gateup_us": round(kern["us"], 3), "gateup_bytes": GATEUP_BYTES,
                            "gateup_gbs": round(GATEUP_BYTES / (kern["us"] * 1e-6) / 1e9, 1),
                            "down_us": round(kern.get("down_us", 0.0), 3), "down_bytes": DOWN_BYTES,
                            "timing": kern["how"]},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 2), "unit": "tokens/s", "h2d_bytes_per_step": e2e["h2d"],
                    "d2h_bytes_per_step": e2e["d2h"], "steps": e2e["steps"]},
            "gpu_launches": -(-K // G) if use_stack else (1 if fused else 4) * K,
            "clocks": ck,
        }
        print(json.dumps(line), flush=True)
    for L in layers:
        L._ws.clear()
    del full, rem
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_mine_ep(args):
    """Config 2 with the experts sharded over the ranks (see the module
    docstring). Timed like the one-GPU line: K steps replayed from CUDA graphs,
    barrier + synchronize around the timed region, max over ranks."""
    import datetime
    import importlib
    import torch
    import torch.distributed as dist
    world = int(os.environ["WORLD_SIZE"])
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    pkg = importlib.import_module("a6000-custom-kernels_b200")
    ep = importlib.import_module("a6000-custom-kernels_b200.ep")
    mc = pkg.moe_cache
    mc.configure(enabled=True)
    R = args.layers
    lo, hi = ep.expert_range(E, rank, world)
    layers, check_full = [], None
    for l in range(R):
        # the same full layer on every rank (same seeds), sliced to this rank's experts
        full = pkg.MoELayer(H, F, E, K_TOP, {"gate": Q2_K, "up": Q2_K, "down": Q2_K}, shared=True, device=dev,
                            seed=l, name=f"blk.{l}")
        layers.append(ep.EPMoELayer(full, rank, world))
        if l == 0 and rank == 0:
            check_full = full
        del full
    torch.cuda.synchronize()
    ex = ep.DecodeExchange(H, E, K_TOP, rank, world).connect()
    P = 64
    xs_np, lg_np = token_pool(P, 1234 + rank)
    xs = torch.from_numpy(xs_np).to(dev).view(P, 1, H)
    lgs = torch.from_numpy(lg_np).to(dev).view(P, 1, E)
    outs = torch.empty((P, 1, H), device=dev)
    stream = torch.cuda.Stream(device=dev)

    def step(i):
        layers[i % R].decode_p2p(ex, xs[i % P], lgs[i % P], outs[i % P], stream=stream)

    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, R)):
            step(i)
    torch.cuda.synchronize()
    assert mc.device_error(stream) == 0

    # in-run check (rank 0): layer copy 0 on this GPU alone, same token
    check = None
    with torch.cuda.stream(stream):
        layers[0].decode_p2p(ex, xs[0], lgs[0], outs[0], stream=stream)
    torch.cuda.synchronize()
    if rank == 0:
        ref = check_full.decode(xs[0], lgs[0])
        torch.cuda.synchronize()
        check = float((outs[0] - ref).abs().max() / ref.abs().max())
        del check_full, ref

    G = 512
    K = args.steps

    def graph_for(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for j in range(n):
                step(j)
        return g

    full_g = graph_for(G) if K >= G else None
    rem = graph_for(K % G) if K % G else None
    with torch.cuda.stream(stream):
        if full_g is not None:
            full_g.replay()
        if rem is not None:
            rem.replay()
    torch.cuda.synchronize()
    dist.barrier()
    clocks = ClockSampler("GPU-" + str(torch.cuda.get_device_properties(dev).uuid))
    clocks.start()
    time.sleep(0.3)
    dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wall0 = time.time()
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for _ in range(K // G):
            full_g.replay()
        if rem is not None:
            rem.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    wall1 = time.time()
    dist.barrier()
    clocks.stop()
    ms = ev0.elapsed_time(ev1)
    t = torch.tensor([ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    assert mc.device_error(stream) == 0
    value = world * K / (ms / 1e3)

    # end to end: per step, H2D of the token and logits, the layer, D2H of the output
    hx = torch.from_numpy(xs_np).pin_memory()
    hl = torch.from_numpy(lg_np).pin_memory()
    hout = torch.empty((P, H), dtype=torch.float32).pin_memory()
    dx, dl, dout = torch.empty((1, H), device=dev), torch.empty((1, E), device=dev), torch.empty((1, H), device=dev)
    n_e2e = min(args.e2e_steps, 1000)

    def one(i):
        with torch.cuda.stream(stream):
            dx.copy_(hx[i % P:i % P + 1], non_blocking=True)
            dl.copy_(hl[i % P:i % P + 1], non_blocking=True)
            layers[i % R].decode_p2p(ex, dx, dl, dout, stream=stream)
            hout[i % P:i % P + 1].copy_(dout, non_blocking=True)
        stream.synchronize()

    for i in range(20):
        one(i)
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(n_e2e):
        one(i)
    e1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / 1e3], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_value = world * n_e2e / float(t.item())

    # expert bytes this rank streams per step: its experts picked by any rank's
    # token (each once) plus the shared expert, 3 matrices each
    pools = [token_pool(P, 1234 + r)[1] for r in range(world)]
    per_step = []
    for i in range(P):
        picks = set()
        for r in range(world):
            picks |= set(np.argsort(-pools[r][i], kind="stable")[:K_TOP].tolist())
        mine = sum(1 for e in picks if lo <= e < hi)
        per_step.append((mine + 1) * 3 * EXPERT_BYTES)
    bytes_rank0 = float(np.mean(per_step))
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    peak = peaks.get("hbm_gbs") or 6650.0
    k_us = 1e3 * ms / K
    achieved = bytes_rank0 / (k_us * 1e-6) / 1e9
    if rank == 0:
        ck = clocks.summary(wall0, wall1)
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": round(ms / K, 6), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": WORKLOAD + f"; experts sharded {E // world} per GPU, one token per GPU per step",
                       "global_batch": world, "seq_len": 1, "parallelism": f"ep{world}",
                       "layers_cycled": R, "l2": f"inputs larger than L2: {R} layer copies "
                                                 f"({R * 3 * E * EXPERT_BYTES / world / 1e9:.1f} GB per GPU) cycled",
                       "graph": "CUDA graphs of 512-step chunks",
                       "exchange": "inside the layer kernel: peer stores over NVLink (CUDA IPC), no NCCL on the data path"},
            "layer_gbs_rank0": round(achieved, 1),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": "of measured",
                         "traffic": None, "bytes_per_launch": round(bytes_rank0),
                         "kernel": "moe_layer2_kernel<Q2_K,Q2_K> with the expert-parallel exchange (rank 0)",
                         "us_per_launch": round(k_us, 3),
                         "timing": f"timed region: {K} back-to-back launches in CUDA graphs, per-step time"},
            "parity_check": {"rank0_max_rel_err_vs_one_gpu": check,
                             "what": "rank 0's token through layer copy 0 sharded over all GPUs vs the same layer "
                                     "whole on rank 0's GPU"},
            "cpu_baseline": None,
            "e2e": {"value": round(e2e_value, 2), "unit": "tokens/s", "h2d_bytes_per_step": (H + E) * 4 * world,
                    "d2h_bytes_per_step": H * 4 * world, "steps": n_e2e},
            "gpu_launches": world * K,
            "clocks": ck,
        }
        print(json.dumps(line), flush=True)
    del full_g, rem
    torch.cuda.synchronize()
    dist.barrier()
    ex.close()
    for L in layers:
        L._ws.clear()
    dist.destroy_process_group()


def time_gateup_kernel(pkg, layers, xs, dev, stream, n):
    """Per-launch duration of the fused gate/up GEMV and of the down GEMV on the
    benchmark's own layers and tokens: graphs of n launches each, bracketed by
    external CUDA events per launch; mean of the per-launch intervals."""
    import torch
    mc = pkg.moe_cache
    R = len(layers)
    P = xs.shape[0]
    bufs = []
    for L in layers:
        ids, _ = L.routing_of(1)
        h = torch.empty((1, K_TOP, F), device=dev)
        hs = torch.empty((1, F), device=dev)
        y = torch.empty((1, K_TOP, H), device=dev)
        ys = torch.empty((1, H), device=dev)
        fd = mc.fusion_device(gate=L.w["gate"], glu_op=0, shared_up=L.shared["up"], shared_gate=L.shared["gate"],
                              shared_dst=hs, shared_stride_col_dst=F)
        fd2 = mc.fusion_device(shared_up=L.shared["down"], shared_dst=ys, shared_stride_col_dst=H)
        bufs.append((ids, h, hs, y, ys, fd, fd2))

    def gateup(i):
        L = layers[i % R]
        ids, h, hs, y, ys, fd, fd2 = bufs[i % R]
        mc.mul_mat_vec_q(L.desc_t["up"], xs[i % P], mc.F32, ids, h, ncols_dst=1, nchannels_y=1, nchannels_dst=K_TOP,
                         stride_col_y=H, stride_col_dst=K_TOP * F, stride_channel_y=0, stride_channel_dst=F,
                         ids_stride=K_TOP, fusion_gate=L.desc_t["gate"], fusion_dev=fd, stream=stream)

    def down(i):
        L = layers[i % R]
        ids, h, hs, y, ys, fd, fd2 = bufs[i % R]
        mc.mul_mat_vec_q(L.desc_t["down"], h, mc.F32, ids, y, ncols_dst=1, nchannels_y=K_TOP, nchannels_dst=K_TOP,
                         stride_col_y=K_TOP * F, stride_channel_y=F, stride_col_dst=K_TOP * H, stride_channel_dst=H,
                         ids_stride=K_TOP, fusion_dev=fd2, stream=stream)

    out = {}
    for name, fn in (("gateup", gateup), ("down", down)):
        with torch.cuda.stream(stream):
            for i in range(R):
                fn(i)
        torch.cuda.synchronize()
        try:
            evs = [(torch.cuda.Event(enable_timing=True, external=True),
                    torch.cuda.Event(enable_timing=True, external=True)) for _ in range(n)]
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for i in range(n):
                    evs[i][0].record(stream)
                    fn(i)
                    evs[i][1].record(stream)
            with torch.cuda.stream(stream):
                g.replay()
            torch.cuda.synchronize()
            per = [a.elapsed_time(b) for a, b in evs]
            us = 1e3 * statistics.mean(per)
            how = (f"CUDA events around each of {n} launches (external event nodes in one CUDA graph), "
                   f"{R} layer copies cycled")
            del g
        except (TypeError, RuntimeError):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for i in range(n):
                    fn(i)
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                g.replay()
                ev0.record(stream)
                g.replay()
                ev1.record(stream)
            torch.cuda.synchronize()
            us = 1e3 * ev0.elapsed_time(ev1) / n
            how = f"CUDA events around a graph of {n} back-to-back launches (includes launch gaps)"
            del g
        out[name] = (us, how)
    assert mc.device_error(stream) == 0
    return {"us": out["gateup"][0], "how": out["gateup"][1], "down_us": out["down"][0]}


def run_e2e(pkg, layers, xs_np, lg_np, dev, stream, steps):
    """Public API end to end: per step, H2D of the token's activations and router
    logits from pinned host memory, MoELayer.decode (one moe_b200_layer_decode
    call), D2H of the layer output into pinned host memory. The steps go back
    to back with no host wait between them (the inputs of consecutive steps
    are independent tokens): copies in, calls and copies out on three streams
    ordered by events, so a step's copies overlap its neighbours' calls; G
    steps are captured once into a CUDA graph and replayed, so the host's
    per-call overhead does not set the pace. Every step's output is on the
    host when the timed region ends."""
    import torch
    R = len(layers)
    P = xs_np.shape[0]
    G = 64
    hx = torch.from_numpy(xs_np).pin_memory()
    hl = torch.from_numpy(lg_np).pin_memory()
    hout = torch.empty((P, H), dtype=torch.float32).pin_memory()
    D = 4                                   # device buffers in rotation
    dx = torch.empty((D, 1, H), device=dev)
    dl = torch.empty((D, 1, E), device=dev)
    dout = torch.empty((D, 1, H), device=dev)

    # copies in on s_in, calls on `stream`, copies out on s_out, ordered by
    # events over the D buffers: step i + 1's input crosses while step i runs
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in range(D)]     # step's input landed
    ev_done = [torch.cuda.Event() for _ in range(D)]   # step's call done (its buffers read and written)
    ev_out = [torch.cuda.Event() for _ in range(D)]    # step's output copied out

    def one(i):
        j = i % D
        with torch.cuda.stream(s_in):
            if i >= D:
                s_in.wait_event(ev_done[j])
            dx[j].copy_(hx[i % P:i % P + 1], non_blocking=True)
            dl[j].copy_(hl[i % P:i % P + 1], non_blocking=True)
            ev_in[j].record(s_in)
        stream.wait_event(ev_in[j])
        if i >= D:
            stream.wait_event(ev_out[j])
        layers[i % R].decode(dx[j], dl[j], dout[j], stream=stream)
        ev_done[j].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_done[j])
            hout[i % P:i % P + 1].copy_(dout[j], non_blocking=True)
            ev_out[j].record(s_out)

    def block():
        fork = torch.cuda.Event()
        fork.record(stream)
        s_in.wait_event(fork)
        s_out.wait_event(fork)
        for i in range(G):
            one(i)
        stream.wait_stream(s_in)
        stream.wait_stream(s_out)

    with torch.cuda.stream(stream):
        block()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        block()
    reps = max(1, steps // G)
    with torch.cuda.stream(stream):
        graph.replay()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for _ in range(reps):
            graph.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    return {"seconds": ev0.elapsed_time(ev1) / 1e3, "steps": reps * G, "h2d": (H + E) * 4, "d2h": H * 4}


# ---------------------------------------------------------------------------
# Other BASELINE configs (their own JSON lines; the headline is config 2)
# ---------------------------------------------------------------------------
STACK_TYPES = (Q2_K, 11, 12, 14)              # Q2_K, Q3_K, Q4_K, Q6_K
STACK_P = (0.40, 0.30, 0.15, 0.15)            # ~0.47 B/weight: ~77 GiB for 48 layers
BYTES_PER_W = {2: 18 / 32, 10: 84 / 256, 11: 110 / 256, 12: 144 / 256, 14: 210 / 256}


def stack_types(n_layers, seed=3):
    """Per-layer types drawn by seed: one draw for the gate/up pair (llama.cpp's
    quantization mixes give ffn_gate and ffn_up the same type) and one for down."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n_layers):
        gu, dn = (int(t) for t in rng.choice(STACK_TYPES, size=2, p=STACK_P))
        out.append({"gate": gu, "up": gu, "down": dn})
    return out


def run_other_config(args):
    """Config 1: one small Q4_0 layer (32 copies cycled). Config 3: the
    48-layer stack, one decode step = every layer in turn with a residual add,
    batch 1..64 (chunks of 8 tokens per layer launch above 8)."""
    import torch
    import importlib
    pkg = importlib.import_module("a6000-custom-kernels_b200")
    mc = pkg.moe_cache
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(device=dev)
    B = args.batch
    if args.config == 1:
        H1, F1, E1, R = 2048, 512, 64, 32
        mc.configure(enabled=True)
        layers = [pkg.MoELayer(H1, F1, E1, 8, {"gate": 2, "up": 2, "down": 2}, shared=False, device=dev, seed=l,
                               name=f"c1.{l}") for l in range(R)]
        rng = np.random.default_rng(11)
        P = 64
        xs = torch.from_numpy(rng.normal(0, 1, (P, B, H1)).astype(np.float32)).to(dev)
        lgs = torch.from_numpy(rng.normal(0, 1, (P, B, E1)).astype(np.float32)).to(dev)
        outs = torch.empty((P, B, H1), device=dev)
        step_bytes = []
        lg_np = lgs.cpu().numpy()
        for i in range(P):
            picks = set(np.argsort(-lg_np[i], axis=1, kind="stable")[:, :8].reshape(-1).tolist())
            step_bytes.append(len(picks) * 3 * F1 * H1 * BYTES_PER_W[2])

        def step(i):
            layers[i % R].decode(xs[i % P], lgs[i % P], outs[i % P], stream=stream)
        launches = 1 if layers[0].fused(B) else 4
        workload = f"config1: H=2048, E=64, F=512, top-8 over N(0,1) logits, Q4_0, no shared expert; batch {B}"
        n_layers_step = 1
        mean_bytes = float(np.mean(step_bytes))
    else:
        n_layers = args.stack_layers
        types = stack_types(n_layers)
        mc.configure(enabled=True)
        # weights N(0, 0.005) before quantization: with no normalization
        # between layers the residual chain x + out stays finite over 48
        # layers (at 0.02 the SwiGLU's square growth overflows it)
        layers = [pkg.MoELayer(H, F, E, K_TOP, types[l], shared=True, device=dev, seed=7000 + l, sigma=0.005,
                               name=f"blk.{l}") for l in range(n_layers)]
        P = 16
        rng = np.random.default_rng(33)
        xs = torch.from_numpy(rng.normal(0, 1, (P, B, H)).astype(np.float32)).to(dev)
        lg_np = np.zeros((n_layers, P, B, E), np.float32)
        for l in range(n_layers):
            perm = np.random.default_rng(1000 + l).permutation(E)
            base = -1.1 * np.log(perm + 1.0)
            lg_np[l] = base[None, None, :] + rng.normal(0, 1, (P, B, E))
        lgs = torch.from_numpy(lg_np).to(dev)
        xbuf = torch.empty((B, H), device=dev)
        obuf = torch.empty((B, H), device=dev)
        chunks = [(c, min(B, c + 8)) for c in range(0, B, 8)]
        step_bytes = []
        for i in range(P):
            tot = 0.0
            for l in range(n_layers):
                picks = set(np.argsort(-lg_np[l, i], axis=1, kind="stable")[:, :8].reshape(-1).tolist())
                for r, t in types[l].items():
                    rows, cols = (F, H) if r != "down" else (H, F)
                    tot += (len(picks) + 1) * rows * cols * BYTES_PER_W[t]
            step_bytes.append(tot)

        def step(i):
            with torch.cuda.stream(stream):
                xbuf.copy_(xs[i % P])
                for l in range(n_layers):
                    for c0, c1 in chunks:
                        layers[l].decode(xbuf[c0:c1], lgs[l, i % P, c0:c1], obuf[c0:c1], stream=stream)
                    xbuf.add_(obuf)
        fused = all(L.fused(c1 - c0) for L in layers for c0, c1 in chunks)
        launches = n_layers * len(chunks) * (1 if fused else 4)
        gib = sum(sum(L.w[r].numel() for r in ("gate", "up", "down")) for L in layers) / 2 ** 30
        workload = (f"config{args.config}: {n_layers}-layer stack of config-2 layers, per-tensor types from "
                    f"{{Q2_K,Q3_K,Q4_K,Q6_K}} drawn by seed (gate/up pair, down) ({gib:.1f} GiB of experts), per-layer Zipf(1.1) routing, "
                    f"shared expert, f32 residual; batch {B}")
        n_layers_step = n_layers
        mean_bytes = float(np.mean(step_bytes))

    K = args.steps
    W = max(args.warmup, 3)
    with torch.cuda.stream(stream):
        for i in range(W):
            step(i)
    torch.cuda.synchronize()
    G = 64 if n_layers_step > 1 else 512
    stack_mode = B == 1 and args.launch == "stack"
    if stack_mode and args.config == 1:
        # batch 1: 512 independent layer steps (the 32 copies cycled) in one
        # persistent launch of the stack kernel
        st = pkg.Stack([layers[j % R] for j in range(G)], [xs[j % P] for j in range(G)],
                       [lgs[j % P] for j in range(G)], [outs[j % P] for j in range(G)], stream=stream)
        st.run(stream)
        torch.cuda.synchronize()
        assert mc.device_error(stream) == 0
        # in-run check: the stack's outputs equal the per-step layer decode
        first = outs[:8].clone()
        with torch.cuda.stream(stream):
            for i in range(8):
                step(i)
        torch.cuda.synchronize()
        stack_diff = float((first - outs[:8]).abs().max())
        reps = max(1, K // G)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(reps):
                st.run(stream)
            ev1.record(stream)
        torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1)
        K = reps * G
        launches = 1.0 / G
        extra = {"timing": f"persistent launches of {G} layer steps (stack kernel), device events",
                 "stack_vs_per_layer_max_abs_diff": stack_diff}
    elif stack_mode:
        # batch 1: G steps x n_layers layers in one persistent launch of the
        # mixed-type stack kernel (each layer its own gate/up and down types);
        # within a step the layers chain through x_next, a step starts from
        # its own token
        chain = [torch.empty((1, H), device=dev) for _ in range(2)]

        def stack_of(n_steps):
            Ls, X, Lg, O_, XN = [], [], [], [], []
            for j in range(n_steps):
                for l in range(n_layers):
                    e = j * n_layers + l
                    Ls.append(layers[l])
                    X.append(xs[j % P] if l == 0 else chain[(e - 1) % 2])
                    Lg.append(lgs[l, j % P])
                    O_.append(obuf)
                    XN.append(chain[e % 2])
            return pkg.Stack(Ls, X, Lg, O_, x_nexts=XN, stream=stream)
        # in-run check: one step through the stack equals the per-layer path bit for bit
        st1 = stack_of(1)
        st1.run(stream)
        with torch.cuda.stream(stream):
            step(0)
        torch.cuda.synchronize()
        assert mc.device_error(stream) == 0
        stack_diff = float((chain[(n_layers - 1) % 2] - xbuf).abs().max())
        st = stack_of(G)
        st.run(stream)
        torch.cuda.synchronize()
        reps = max(1, K // G)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(reps):
                st.run(stream)
            ev1.record(stream)
        torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1)
        K = reps * G
        launches = 1.0 / G
        extra = {"timing": f"persistent launches of {G} steps x {n_layers} layers (mixed-type stack kernel), device events",
                 "stack_vs_per_layer_max_abs_diff": stack_diff}
    else:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for j in range(G):
                step(j)
        with torch.cuda.stream(stream):
            g.replay()
        torch.cuda.synchronize()
        reps = max(1, K // G)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(reps):
                g.replay()
            ev1.record(stream)
        torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1)
        K = reps * G
        extra = {"timing": f"CUDA graphs of {G} steps, device events"}
        del g
    assert mc.device_error(stream) == 0
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    peak = peaks.get("hbm_gbs") or 6650.0
    gbs = mean_bytes * K / (ms / 1e3) / 1e9
    line = {"metric": METRIC, "value": round(B * K / (ms / 1e3), 2), "unit": "tokens/s", "n_gpus": 1, "steps": K,
            "warmup": W, "ms_per_step": round(ms / K, 6), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": workload, "global_batch": B, "layers_per_step": n_layers_step},
            "expert_gbs": round(gbs, 1), "frac_of_measured_hbm": round(gbs / peak, 4),
            "bytes_per_step": round(mean_bytes), "gpu_launches": round(launches * K), **extra}
    print(json.dumps(line), flush=True)
    for L in layers:
        L._ws.clear()


def zipf_gumbel_logits(gen, base, n, device):
    """n router-logit rows for one layer: log Zipf(1.1) weights of the layer's
    expert permutation plus Gumbel(0, 1) noise, so the top-8 of a row is a
    sample of 8 experts without replacement from Zipf(1.1)."""
    import torch
    u = torch.rand((n, base.shape[0]), generator=gen, device=device).clamp_(1e-12, 1.0 - 1e-7)
    return base[None, :] - torch.log(-torch.log(u))


def run_config5(args):
    """Config 5 (tiered-cache stress): the config-3 stack (48 layers, per-tensor
    types drawn by seed) with every expert tensor in pinned host memory behind
    an HBM pool capped at 128 of 512 experts per tensor, seeded from a routing
    frequency table sampled from the same distribution (4096 tokens per
    layer). Each decode step routes a fresh token with fresh logits drawn as
    Gumbel-top-8 over log Zipf(1.1) with the layer's own expert permutation,
    runs every layer (residual added), then the cache's promotion step -- on
    the GPU, so steps are captured in CUDA graphs of 50 with their fresh
    inputs refilled on the device before each replay (inside the timed
    region). Experts the pool misses are read zero-copy over the host link."""
    import importlib
    import tempfile
    import torch
    pkg = importlib.import_module("a6000-custom-kernels_b200")
    mc = pkg.moe_cache
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(device=dev)
    n_layers = args.stack_layers
    types = stack_types(n_layers)
    POOL = 128
    bases = []
    lines = []
    rng = np.random.default_rng(55)
    for l in range(n_layers):
        perm = np.random.default_rng(1000 + l).permutation(E)
        base = -1.1 * np.log(perm + 1.0)
        bases.append(base)
        # routing-frequency table: 4096 sampled tokens of this layer
        g = -np.log(-np.log(np.clip(rng.random((4096, E)), 1e-12, 1 - 1e-7)))
        picks = np.argpartition(-(base[None, :] + g), K_TOP, axis=1)[:, :K_TOP]
        cnt = np.bincount(picks.reshape(-1), minlength=E)
        hot = sorted(range(E), key=lambda e: (-cnt[e], e))[:POOL]
        for r in ("gate", "up", "down"):
            lines.append(f"blk.{l}.ffn_{r}_exps.weight " + ",".join(str(e) for e in hot))
    fd_, seed_path = tempfile.mkstemp(suffix=".seed")
    os.write(fd_, ("\n".join(lines) + "\n").encode())
    os.close(fd_)
    mc.configure(enabled=True, slots=POOL, budget_gb=1e6, seed_path=seed_path)
    t_build = time.time()
    layers = [pkg.MoELayer(H, F, E, K_TOP, types[l], shared=True, device=dev, host=True, seed=7000 + l, sigma=0.005,
                           name=f"blk.{l}") for l in range(n_layers)]
    t_build = time.time() - t_build
    host_gib = sum(sum(L.w[r].numel() for r in ("gate", "up", "down")) for L in layers) / 2 ** 30
    mean_expert = float(np.mean([L.w[r][0].numel() for L in layers for r in ("gate", "up", "down")]))
    base_d = torch.tensor(np.stack(bases), dtype=torch.float32, device=dev)
    C = 50
    lg = torch.empty((n_layers, C, 1, E), device=dev)
    xin = torch.empty((C, 1, H), device=dev)
    xbuf = torch.empty((1, H), device=dev)
    obuf = torch.empty((1, H), device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(77)

    def refill():
        for l in range(n_layers):
            lg[l, :, 0].copy_(zipf_gumbel_logits(gen, base_d[l], C, dev))
        xin.normal_(generator=gen)

    def step(j):
        xbuf.copy_(xin[j])
        for l in range(n_layers):
            layers[l].decode(xbuf, lg[l, j], obuf, stream=stream)
            xbuf.add_(obuf)
        mc.step(stream)

    # warm-up: eager steps register every tensor (seeded pools) and settle the cache
    W = max(args.warmup, 3)
    with torch.cuda.stream(stream):
        for i in range(W):
            if i % C == 0:
                refill()
            step(i % C)
    torch.cuda.synchronize()
    assert mc.device_error(stream) == 0
    # the promotion pass alone (device time), eager
    evs = []
    with torch.cuda.stream(stream):
        refill()
        for j in range(20):
            xbuf.copy_(xin[j])
            for l in range(n_layers):
                layers[l].decode(xbuf, lg[l, j], obuf, stream=stream)
                xbuf.add_(obuf)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            mc.step(stream)
            e1.record(stream)
            evs.append((e0, e1))
    torch.cuda.synchronize()
    pass_us = 1e3 * float(np.mean([a.elapsed_time(b) for a, b in evs]))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for j in range(C):
            step(j)
    torch.cuda.synchronize()
    K = max(C, min(args.steps, 2000)) // C * C
    s0 = mc.stats()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler("GPU-" + str(torch.cuda.get_device_properties(dev).uuid))
    clocks.start()
    time.sleep(0.3)
    wall0 = time.time()
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for _ in range(K // C):
            refill()
            g.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    wall1 = time.time()
    clocks.stop()
    ms = ev0.elapsed_time(ev1)
    s1 = mc.stats()
    assert mc.device_error(stream) == 0
    hits, misses = s1["hits"] - s0["hits"], s1["misses"] - s0["misses"]
    promos, evicts = s1["promotions"] - s0["promotions"], s1["evictions"] - s0["evictions"]
    line = {"metric": METRIC, "value": round(K / (ms / 1e3), 2), "unit": "tokens/s", "n_gpus": 1, "steps": K,
            "warmup": W, "ms_per_step": round(ms / K, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"config5: {n_layers}-layer config-3 stack ({host_gib:.1f} GiB of experts in pinned "
                                   f"host memory), HBM pool {POOL} of {E} experts per tensor seeded from a sampled "
                                   f"frequency table, fresh Gumbel-top-8 Zipf(1.1) routing every step, batch 1",
                       "global_batch": 1, "layers_per_step": n_layers, "pool_slots": POOL},
            "hit_rate": round(hits / max(1, hits + misses), 4),
            "hits_per_step": round(hits / K, 1), "misses_per_step": round(misses / K, 1),
            "promotions_per_step": round(promos / K, 2), "evictions_per_step": round(evicts / K, 2),
            "resident_experts": s1["resident"],
            "hbm_expert_bytes_per_step": round(hits / K * mean_expert),
            "host_link_bytes_per_step": round((misses + promos) / K * mean_expert),
            "promotion_pass_us": round(pass_us, 2),
            "gpu_launches": K * (n_layers * 2 + 2),
            "timing": f"CUDA graphs of {C} steps (decode of every layer + residual + promotion step), inputs "
                      f"refilled on the device before each replay, device events",
            "build_seconds": round(t_build, 1), "clocks": clocks.summary(wall0, wall1)}
    print(json.dumps(line), flush=True)
    for L in layers:
        L._ws.clear()
    os.unlink(seed_path)


def run_config4(args):
    """Config 4: expert-parallel prefill through the config-3 stack (48
    layers, per-tensor types from {Q2_K,Q3_K,Q4_K,Q6_K} drawn by seed). Every
    rank holds 512 / N experts of each layer and prefills its own prompt of
    --prompt tokens: route, dispatch all-to-all (NCCL), tensor-core expert
    prefill on the rows it received, return all-to-all, shared expert,
    weighted combine, residual add. N = 1 runs the single-GPU layer prefill
    (no exchange). value = all ranks' prompt tokens / max-over-ranks time."""
    import datetime
    import importlib
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    pkg = importlib.import_module("a6000-custom-kernels_b200")
    ep = importlib.import_module("a6000-custom-kernels_b200.ep")
    mc = pkg.moe_cache
    mc.configure(enabled=True)
    n_layers, B = args.stack_layers, args.prompt
    types = stack_types(n_layers)
    lo, hi = ep.expert_range(E, rank, world)
    layers = []
    for l in range(n_layers):
        L = pkg.MoELayer(H, F, hi - lo, K_TOP, types[l], shared=True, device=dev, seed=7000 + 97 * l + rank,
                         name=f"blk.{l}")
        layers.append(ep.EPMoELayer(L, rank, world, local=True, n_experts=E) if world > 1 else L)
    rng = np.random.default_rng(33 + rank)
    P = 2
    xs_host = torch.from_numpy(rng.normal(0, 1, (P, B, H)).astype(np.float32)).pin_memory()
    lg_np = np.zeros((n_layers, B, E), np.float32)
    touched = 0
    for l in range(n_layers):
        perm = np.random.default_rng(1000 + l).permutation(E)
        lg_np[l] = (-1.1 * np.log(perm + 1.0))[None, :] + rng.normal(0, 1, (B, E))
        picks = np.argsort(-lg_np[l], axis=1, kind="stable")[:, :K_TOP]
        touched += len(set(picks.reshape(-1).tolist())) * sum(
            (F * H) * BYTES_PER_W[t] for t in types[l].values())
    lgs = torch.from_numpy(lg_np).to(dev)
    ex = None
    if world > 1 and args.ep_exchange == "p2p":
        ex = ep.PeerExchange(H, B * K_TOP, rank, world).connect()
    x = torch.empty((B, H), device=dev)
    out = torch.empty((B, H), device=dev)
    res_host = torch.empty((B, H), dtype=torch.float32).pin_memory()
    stream = torch.cuda.current_stream(dev)

    xs_dev = xs_host.to(dev)

    def step(i, e2e=False):
        # a fresh prompt every step (the residual adds overwrite x): from HBM,
        # or for the end-to-end number from pinned host memory
        x.copy_(xs_host[i % P] if e2e else xs_dev[i % P], non_blocking=True)
        for l in range(n_layers):
            if ex is not None:
                ep.prefill_p2p(layers[l], ex, x, lgs[l], out, stream=stream)
            else:
                layers[l].prefill(x, lgs[l], out, stream=stream)
            x.add_(out)
        if e2e:
            res_host.copy_(x, non_blocking=True)

    W = max(args.warmup, 3)
    K = max(1, min(args.steps, 20))
    for i in range(W):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for i in range(K):
        step(i)
    ev1.record(stream)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    # end to end: each step copies its prompt in from pinned host memory and the result back
    if world > 1:
        dist.barrier()
    ev2, ev3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev2.record(stream)
    for i in range(K):
        step(i, e2e=True)
    ev3.record(stream)
    torch.cuda.synchronize()
    ms_e2e = ev2.elapsed_time(ev3)
    if args.kernel_shares and rank == 0:
        # device time per kernel over two steps (CUPTI timestamps; the kernels
        # run back to back as in the timed loop, nothing is serialized)
        import collections
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for i in range(2):
                step(i)
            torch.cuda.synchronize()
        agg = collections.defaultdict(lambda: [0, 0.0])
        for e in prof.events():
            if e.device_type.name == "CUDA":
                a = agg[e.name.split("(")[0].replace("void ", "")[:48]]
                a[0] += 1
                a[1] += e.device_time_total
        tot = sum(v[1] for v in agg.values())
        print("kernel shares over 2 steps (us per layer):", file=sys.stderr)
        for name, (c, t) in sorted(agg.items(), key=lambda kv: -kv[1][1])[:12]:
            print(f"  {name:48s} {c:6d} launches {t / 2 / n_layers:8.1f} us {100 * t / tot:5.1f} %", file=sys.stderr)
    assert mc.device_error() == 0
    if world > 1:
        t = torch.tensor([ms, ms_e2e], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_e2e = float(t[0]), float(t[1])
    tok = world * B * K
    # launches per layer: routing 1; gate + up 5 (one grouping, quantize and
    # gather, two MMQ), GLU 1, down 4; the shared expert the same 10; combine 1
    launches = n_layers * (1 + 10 + 10 + 1) * K
    if rank == 0:
        gib = sum(sum(L.w[r].numel() for r in ("gate", "up", "down")) for L in layers) / 2 ** 30
        line = {"metric": "MoE prefill tokens/s (expert-parallel)", "value": round(tok / (ms / 1e3), 2),
                "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": round(ms / K, 4),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
                "data": "synthetic",
                "config": {"workload": f"config4: {n_layers}-layer config-3 stack ({gib:.1f} GiB of experts on rank 0), "
                                       f"{B}-token prompt per rank, 512 experts over {world} GPU(s) "
                                       f"({hi - lo} on rank 0), per-layer Zipf(1.1) top-8, shared expert, "
                                       f"f32 residual; dispatch/combine "
                                       + ("by peer-memory stores over NVLink (no host round trip)"
                                          if ex is not None else "by NCCL all-to-all") if world > 1 else
                                       f"config4 on one GPU: {n_layers}-layer config-3 stack, {B}-token prompt, "
                                       f"all 512 experts local (layer prefill, no exchange)",
                           "global_batch": tok // K, "layers_per_step": n_layers,
                           "parallelism": f"ep{world}"},
                "expert_gbs_rank0": round(touched * K / (ms / 1e3) / 1e9, 1),
                "e2e": {"value": round(tok / (ms_e2e / 1e3), 2), "unit": "tokens/s",
                        "h2d_bytes_per_step": B * H * 4, "d2h_bytes_per_step": B * H * 4},
                "gpu_launches": launches, "timing": "eager steps, device events, max over ranks"}
        print(json.dumps(line), flush=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    if ex is not None:
        ex.close()
    for L in layers:
        L._ws.clear()
    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse()
    if args.kernel_shares and int(os.environ.get("WORLD_SIZE", "1")) > 1:
        # the profiled steps would run on one rank only: its exchange waits
        # would wait for dispatches the other ranks never send
        sys.exit("--kernel-shares profiles a one-GPU run; run it without torchrun")
    if args.impl == "reference":
        run_reference(args)
    elif args.config == 2:
        run_mine(args)
    elif args.config == 4:
        run_config4(args)
    elif args.config == 5:
        run_config5(args)
    else:
        run_other_config(args)


if __name__ == "__main__":
    main()
