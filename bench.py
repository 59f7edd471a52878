"""Benchmark of the B200 MoE hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 1]

A step is one MoE layer forward (router -> top-k -> dispatch -> 4-bit SwiGLU
experts -> combine) over one batch of seeded synthetic tokens.  The default
workload is BASELINE config 1: one Qwen3-30B-A3B MoE layer (E=128, top-8,
H=2048, I=768, 4-bit group-64 experts, 8-bit router), batched prefill of
T=512 tokens.  Config 0 (decode of one token) is selectable with --config 0.

* value     tokens/s of the whole job, inputs resident in HBM, device-timed
            (CUDA events, barrier + synchronize both sides, max over ranks).
            Steps rotate over 4 resident layers (1.36 GB of weights, far more
            than the 126 MB L2), so no step reads the previous step's weights
            from L2.
* e2e       the same metric through the host entry points (obs_moe_forward_host_async
            + obs_moe_host_join): every step copies its input from pinned host memory
            and its output back; successive steps pipeline (step i+1's input copy and
            step i-1's output copy overlap step i), as a serving loop would.
* roofline  the dominant kernel (the gate/up grouped GEMM at T=512, the fused
            decode layer at T=1), algorithmic bytes per launch / its mean
            CUDA-event duration on the launching stream, against the measured
            HBM copy bandwidth in MEASURED_PEAKS.json.
* cpu_baseline  the C oracle (oracle/, all host threads) on the same layer.

--impl reference runs the reference's own kernels (shaders/*.metal compiled
for the CPU into oracle/_ref) on the host cores over a bounded token sample.
Multi-GPU (torchrun): every rank runs its own T-token batch against its own
copy of the layers (data-parallel replicas; weak scaling), timed on the device,
max over ranks.  --ep instead splits the experts E/N per GPU and exchanges the
routed rows over NVLink peer memory (expert parallelism).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "project-obsidian_b200"))

H, I, E, K = 2048, 768, 128, 8
EXPERT_BYTES = 2_654_208        # one expert: 3 projections of 4-bit codes + bf16 scales/biases
GATEUP_BYTES = 2 * 884_736      # the gate and up projections of one expert
ROUTER_BYTES = 278_528
N_ROT = 4                       # resident layers the steps rotate over
# DRAM bytes (read + write) per launch of the dominant kernel, from one ncu capture of the same
# workload (the committed profile summaries); other workloads report null
NCU_TRAFFIC = {("gemm_gateup", 512): 246_949_888 + 4_585_472, ("decode_fused", 1): 21_645_056}
CONFIGS = {
    0: dict(T=1, name="config0: Qwen3-30B-A3B MoE layer, decode of 1 token"),
    1: dict(T=512, name="config1: Qwen3-30B-A3B MoE layer, batched prefill of T=512 tokens"),
    2: dict(T=None, name="config2: 48-layer MoE stack, decode of B independent tokens per step", stack=True),
    3: dict(T=4096, name="config3: 48-layer MoE stack, prefill of T=4096 tokens, Zipf(1.1) expert bias",
            stack=True),
}
LAYER_FLOPS = 2 * K * 4_718_592  # per token and layer (router excluded)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=1, choices=sorted(CONFIGS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=32, help="config 2: tokens per decode step (1, 8, 32, 128)")
    ap.add_argument("--layers", type=int, default=48, help="configs 2 and 3: layers in the stack")
    ap.add_argument("--tokens", type=int, default=0, help="configs 0 and 1: override T (a sweep point, not a BASELINE config)")
    ap.add_argument("--ep", action="store_true",
                    help="N > 1: expert parallelism (E/N experts per GPU) instead of N data-parallel replicas")
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class Clocks:
    """SM clock and throttle reasons sampled through NVML every ~2 ms on a
    background thread while the timed region runs."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, index: int):
        import threading

        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._h = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            return
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for name, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(0.002)

    def stop(self):
        if self._h is None:
            return None
        self._stop.set()
        self._t.join(timeout=2)
        if not self.samples:
            return None
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def cpu_baseline(L_host, x_host, T):
    """The C oracle on the host cores (all threads), the same layer and tokens."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    n = os.cpu_count() or 1
    t0 = time.perf_counter()
    O.moe_layer(L_host, x_host, nthreads=n)
    dt = time.perf_counter() - t0
    return {"value": T / dt, "unit": "tokens/s", "cores": n, "kind": "port",
            "sample": f"the full {T}-token layer once through oracle/obs_oracle.c ({dt:.2f} s)"}


def zipf_bias(beta, seed=11):
    """Config 3's per-expert logit bias: beta * log(r_e^-1.1) over a seeded rank
    permutation r (1 = hottest)."""
    import numpy as np

    r = np.random.default_rng(seed).permutation(E) + 1
    return (beta * -1.1 * np.log(r)).astype(np.float32)


def run_stack(args, rank, world, local):
    """Configs 2 and 3: a stack of MoE layers on a residual stream,
    r <- r + MoE_l(RMSNorm(r)) for every layer (obs_moe_stack_forward); a step is
    one pass of the batch through all layers, captured in one CUDA graph."""
    import numpy as np
    import torch

    import obsmoe

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        # NCCL carries only barriers and small reductions here; no NVLink multicast
        # (NVLS) objects next to the peer buffers the expert exchange writes into
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    cfg = CONFIGS[args.config]
    nl = args.layers
    T = args.batch if args.config == 2 else cfg["T"]
    decode = args.config == 2
    path = obsmoe.PATH_AUTO if decode else obsmoe.PATH_PREFILL
    ep = world > 1 and args.ep  # default for N > 1: data-parallel replicas, every GPU holds all experts
    shape = obsmoe.MoeShape(H, I, E, K, n_layers=nl, max_tokens=max(T, 16),
                            ep_world=world if ep else 1, ep_rank=rank if ep else 0)
    ctx = obsmoe.MoeContext(shape, local)
    if ep:
        handles = [None] * world
        dist.all_gather_object(handles, ctx.ep_handle())
        ctx.ep_connect(handles)
    for l in range(nl):
        ctx.synth_layer(l, 0)
    r0 = torch.empty((T, H), dtype=torch.int16, device="cuda")
    obsmoe.synth_activations(rank, 0, 0, T, H, r0)
    stream = torch.cuda.current_stream()
    bias, beta, imbalance = None, None, None
    if args.config == 3:
        # calibrate beta so the hottest expert gets ~10x the mean load (layer 0's routing)
        logits = torch.empty((T, E), dtype=torch.float32, device="cuda")
        ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
        wts = torch.empty((T, K), dtype=torch.float32, device="cuda")
        xn = torch.empty_like(r0)
        ctx.rmsnorm(r0, xn, T)
        ctx.gate_gpu(0, xn, logits, T)
        best = None
        for b in np.linspace(0.0, 8.0, 81):
            bt = torch.from_numpy(zipf_bias(b)).cuda()
            ctx.route(logits, T, ids, wts, bias=bt)
            load = np.bincount(ids.cpu().numpy().ravel(), minlength=E)
            ratio = load.max() / load.mean()
            if best is None or abs(ratio - 10.0) < abs(best[1] - 10.0):
                best = (float(b), float(ratio))
        beta, imbalance = best
        bias = torch.from_numpy(zipf_bias(beta)).cuda()
    r = torch.empty_like(r0)

    def step():
        r.copy_(r0)
        ctx.moe_stack_forward(0, nl, r, T, bias=bias, path=path, stream=stream)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    step()
    barrier()
    ctx.check_device()
    n0 = obsmoe.kernel_launches()
    step()
    launches_per_step = obsmoe.kernel_launches() - n0
    cap = torch.cuda.Stream()
    cap.wait_stream(stream)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(cap):
        with torch.cuda.graph(g, stream=cap):
            r.copy_(r0)
            ctx.moe_stack_forward(0, nl, r, T, bias=bias, path=path, stream=cap)
    stream.wait_stream(cap)
    barrier()
    for _ in range(max(args.warmup, 3)):
        g.replay()
    barrier()
    ctx.check_device()
    clocks = Clocks(local)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    ev0.record(stream)
    for _ in range(args.steps):
        g.replay()
    ev1.record(stream)
    barrier()
    ms = ev0.elapsed_time(ev1)
    clk = clocks.stop()
    ctx.check_device()
    ms_t = torch.tensor([ms], device="cuda")
    if dist is not None:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    step_s = ms / args.steps / 1e3
    value = world * T / step_s

    # e2e: the residual batch from pinned host memory, the stack, the result back
    rh = r0.cpu().pin_memory()
    oh = torch.empty_like(rh).pin_memory()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        r.copy_(rh, non_blocking=True)
        ctx.moe_stack_forward(0, nl, r, T, bias=bias, path=path, stream=stream)
        oh.copy_(r, non_blocking=True)
    e1.record(stream)
    barrier()
    ems_t = torch.tensor([e0.elapsed_time(e1)], device="cuda")
    if dist is not None:
        dist.all_reduce(ems_t, op=dist.ReduceOp.MAX)
    e2e_value = world * T * args.steps / (float(ems_t.item()) / 1e3)

    # per-layer routing of this step (distinct experts), replayed eagerly layer by layer
    hbm, bf16, peak_kind = peaks()
    logits = torch.empty((T, E), dtype=torch.float32, device="cuda")
    ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
    wts = torch.empty((T, K), dtype=torch.float32, device="cuda")
    xn = torch.empty_like(r0)
    rr = r0.clone()
    U, loads = [], []
    for l in range(nl):
        ctx.rmsnorm(rr, xn, T)
        ctx.gate_gpu(l, xn, logits, T)
        ctx.route(logits, T, ids, wts, bias=bias)
        every = ids.cpu().numpy().ravel()
        if ep:
            parts = [None] * world
            dist.all_gather_object(parts, every)
            every = np.concatenate(parts)
        U.append(len(np.unique(every)))
        loads.append(np.bincount(every, minlength=E))
        ctx.moe_stack_forward(l, 1, rr, T, bias=bias, path=path, stream=stream)
    torch.cuda.synchronize()
    load = np.sum(loads, axis=0)
    if decode:
        # HBM roofline: every routed expert's weights, the router and the activations, per layer
        per_gpu_bytes = (sum(U) * EXPERT_BYTES / world + nl * ROUTER_BYTES + nl * 2 * T * H * 2 * 2)
        achieved = per_gpu_bytes / step_s / 1e9
        roof = {"bound": "hbm", "kernel": f"whole {nl}-layer decode step (router, top-k, 4-bit mat-vecs, combine, "
                f"RMSNorm per layer)", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                "algorithmic_bytes_per_launch": per_gpu_bytes, "traffic": None}
    else:
        flops = nl * T * LAYER_FLOPS  # per GPU (weak scaling: each GPU's T tokens)
        achieved = flops / step_s / 1e12
        roof = {"bound": "tensor", "kernel": f"whole {nl}-layer prefill step (grouped tcgen05 GEMMs dominate)",
                "achieved": achieved, "peak": bf16, "unit": "TFLOP/s", "frac": achieved / bf16,
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json bf16_tflops)",
                "algorithmic_flops_per_launch": flops, "traffic": None}
    line = {
        "metric": "MoE stack tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded; BASELINE config distributions; weights generated on the device)",
        "config": {"workload": cfg["name"], "layers": nl, "T": T, "E": E, "K": K, "H": H, "I": I,
                   "parallelism": (f"expert parallel x{world} (NVLink peer all-to-all)" if ep else
                                   f"data parallel x{world} (replicas)" if world > 1 else "single GPU"),
                   "l2": f"inputs larger than L2: {nl} resident layers ({nl * 340} MB) per step",
                   "path": "decode (mat-vec)" if decode and T <= 2 and not ep else "prefill (tcgen05 grouped GEMM)",
                   "zipf_beta": beta, "load_max_over_mean_layer0": imbalance,
                   "load_max_over_mean_all_layers": float(load.max() / load.mean())},
        "roofline": roof, "distinct_experts_per_layer": float(np.mean(U)),
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": T * H * 2,
                "d2h_bytes_per_step": T * H * 2},
        "gpu_launches": launches_per_step * args.steps, "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O

        # bounded sample: 2 layers and at most 32 tokens through the C oracle, scaled to the stack
        nlo, Ts = 2, min(T, 32)
        Ls = [O.synth_layer(0, l, E=E, H=H, I=I, K=K) for l in range(nlo)]
        rs = r0[:Ts].cpu().numpy().view(np.uint16)
        n = os.cpu_count() or 1
        t0 = time.perf_counter()
        O.moe_stack(Ls, rs, bias=None if bias is None else bias.cpu().numpy(), nthreads=n)
        dt = (time.perf_counter() - t0) * nl / nlo
        line["cpu_baseline"] = {"value": Ts / dt, "unit": "tokens/s", "cores": n, "kind": "port",
                                "sample": f"{Ts} tokens through {nlo} layers of oracle/obs_oracle.c, "
                                          f"time scaled to {nl} layers"}
    if dist is not None:
        dist.barrier()  # no rank frees its peer-mapped buffer while another may still use it
    ctx.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line))


def run_reference(args, rank, world):
    """The reference's own kernels on the host cores (oracle/_ref)."""
    cfg = CONFIGS[args.config]
    T = cfg["T"] if cfg["T"] is not None else args.batch
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    if O.ref_lib() is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libobs_refshaders.so was not built"}))
        return
    n = os.cpu_count() or 1
    Ts = min(T, 64)  # bounded sample: one step is Ts tokens of the workload
    L = O.synth_layer(0, 0, E=E, H=H, I=I, K=K)
    x = O.synth_x(0, 0, Ts, H)
    for _ in range(args.warmup):
        O.ref_moe_prefill(L, x, nthreads=n)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.ref_moe_prefill(L, x, nthreads=n)
    dt = time.perf_counter() - t0
    value = Ts * args.steps / dt
    sample = (f"{Ts} of the {T} tokens per step through the reference's shaders/*.metal kernels compiled "
              f"for the CPU (oracle/_ref), strung as src/forward.rs:164-232, {n} threads")
    metric = "MoE layer tokens/s"
    if cfg.get("stack"):  # one layer timed, scaled to the stack's layer count
        value /= args.layers
        metric = "MoE stack tokens/s"
        sample += f"; one layer per step, time scaled to {args.layers} layers"
    print(json.dumps({
        "impl": "reference", "metric": metric, "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded, BASELINE config distributions)",
        "config": {"workload": cfg["name"], "T": T, "E": E, "K": K, "H": H, "I": I, "sample_tokens": Ts},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": n, "kind": "reference", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if CONFIGS[args.config].get("stack"):
        return run_stack(args, rank, world, local)

    import numpy as np
    import torch

    import obsmoe

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        # NCCL carries only barriers and small reductions here; no NVLink multicast
        # (NVLS) objects next to the peer buffers the expert exchange writes into
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    cfg = dict(CONFIGS[args.config])
    if args.tokens:
        cfg["T"], cfg["name"] = args.tokens, cfg["name"].split(",")[0] + f", T={args.tokens} tokens (sweep)"
    T = cfg["T"]
    # N GPUs: each routes its own T tokens; by default every GPU holds all experts
    # (data-parallel replicas), with --ep E/N experts per GPU and an NVLink exchange
    ep = world > 1 and args.ep
    path = obsmoe.PATH_DECODE if T <= 2 and not ep else obsmoe.PATH_PREFILL
    shape = obsmoe.MoeShape(H, I, E, K, n_layers=N_ROT, max_tokens=max(T, 16),
                            ep_world=world if ep else 1, ep_rank=rank if ep else 0)
    ctx = obsmoe.MoeContext(shape, local)
    if ep:
        handles = [None] * world
        dist.all_gather_object(handles, ctx.ep_handle())
        ctx.ep_connect(handles)
    for l in range(N_ROT):
        ctx.synth_layer(l, 0)  # layer l of seed 0 (config 2's per-layer seeding)
    xs = [torch.empty((T, H), dtype=torch.int16, device="cuda") for _ in range(N_ROT)]
    for l, x in enumerate(xs):
        obsmoe.synth_activations(rank, l, 0, T, H, x)
    out = torch.empty((T, H), dtype=torch.int16, device="cuda")
    stream = torch.cuda.current_stream()

    def step(i):
        l = i % N_ROT
        ctx.moe_forward(l, xs[l], out, T, path=path, stream=stream)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for i in range(max(args.warmup, 3)):
        step(i)
    ctx.check_device()
    # one CUDA graph per resident layer: a step replays the layer's whole
    # forward (router .. combine) without host launch gaps
    n0 = obsmoe.kernel_launches()
    step(0)
    launches_per_step = obsmoe.kernel_launches() - n0
    graphs = []
    cap = torch.cuda.Stream()
    cap.wait_stream(stream)
    with torch.cuda.stream(cap):
        for l in range(N_ROT):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                ctx.moe_forward(l, xs[l], out, T, path=path, stream=cap)
            graphs.append(g)
    stream.wait_stream(cap)
    for i in range(max(args.warmup, 3)):
        graphs[i % N_ROT].replay()
    barrier()
    ctx.check_device()
    # ------------------------------------------------------------ timed region
    clocks = Clocks(local)
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for i in range(args.steps):
        graphs[i % N_ROT].replay()
    ev1.record(stream)
    barrier()
    ms = ev0.elapsed_time(ev1)
    clk = clocks.stop()
    ctx.check_device()
    # stage times from a separate, eager pass (events between the stages)
    ctx.profile(True)
    for i in range(args.steps):
        step(i)
    torch.cuda.synchronize()
    prof = ctx.profile_read()
    ctx.profile(False)
    ms_t = torch.tensor([ms], device="cuda")
    if dist is not None:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    value = world * T * args.steps / (ms / 1e3)

    # ---------------------------------------------------------------- e2e
    # every step copies its input in from pinned host memory and its output back, through the
    # pipelined host entry: step i+1's input copy and step i-1's output copy overlap step i
    xh = [torch.empty((T, H), dtype=torch.int16).pin_memory() for _ in range(N_ROT)]
    for l in range(N_ROT):
        xh[l].copy_(xs[l].cpu())
    oh = [torch.empty((T, H), dtype=torch.int16).pin_memory() for _ in range(2)]

    def host_step(i):
        if ep:  # the pipelined entry is single-GPU: expert parallelism copies in and out per call
            ctx.moe_forward_host(i % N_ROT, xh[i % N_ROT], oh[i % 2], T, path=path, stream=stream)
        else:
            ctx.moe_forward_host_async(i % N_ROT, xh[i % N_ROT], oh[i % 2], T, path=path, stream=stream)

    for i in range(3):
        host_step(i)
    ctx.host_join(stream)
    stream.synchronize()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        host_step(i)
    ctx.host_join(stream)  # the last step's result is in host memory before e1
    e1.record(stream)
    stream.synchronize()
    barrier()
    ems_t = torch.tensor([e0.elapsed_time(e1)], device="cuda")
    if dist is not None:
        dist.all_reduce(ems_t, op=dist.ReduceOp.MAX)
    e2e_value = world * T * args.steps / (float(ems_t.item()) / 1e3)

    # ------------------------------------------------ roofline of the top kernel
    hbm, bf16, peak_kind = peaks()
    # distinct experts per step (U), from the same routing the timed steps used
    ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
    wts = torch.empty((T, K), dtype=torch.float32, device="cuda")
    logits = torch.empty((T, E), dtype=torch.float32, device="cuda")
    U, R = [], []
    e_lo, e_hi = (rank * E // world, (rank + 1) * E // world) if ep else (0, E)
    for l in range(N_ROT):
        ctx.gate_gpu(l, xs[l], logits, T, stream=stream)
        ctx.route(logits, T, ids, wts, stream=stream)
        mine = ids.cpu().numpy().ravel()
        if ep:  # this GPU's experts see every rank's rows routed to them
            every = [None] * world
            dist.all_gather_object(every, mine)
            mine = np.concatenate(every)
        local_ids = mine[(mine >= e_lo) & (mine < e_hi)]
        U.append(len(np.unique(local_ids)))
        R.append(len(local_ids))
    U_mean, R_mean = sum(U) / len(U), sum(R) / len(R)
    if path == obsmoe.PATH_PREFILL:
        top = "gemm_gateup"
        # gate+up weights of the U routed experts (this GPU's), the routed rows read, h written
        alg = U_mean * GATEUP_BYTES + R_mean * H * 2 + R_mean * I * 2
        kname = "k_gemm<kEpiSwiglu> (tcgen05 grouped gate/up GEMM + SwiGLU)"
    elif prof["decode_fused"][1]:
        top = "decode_fused"
        # the whole decode layer in one launch: router weights, all three projections
        # of the U routed experts, x read, out written
        alg = ROUTER_BYTES + U_mean * EXPERT_BYTES + 2 * T * H * 2
        kname = ("k_decode_fused (whole decode layer: router, top-k, 4-bit gate/up and down mat-vec, "
                 "combine; one cooperative launch)")
    else:
        top = "decode_gateup"
        alg = U_mean * GATEUP_BYTES + T * H * 2 + T * K * I * 2
        kname = "k_decode_gateup (4-bit gate/up mat-vec)"
    kms, kn = prof[top]
    k_avg_s = kms / max(kn, 1) / 1e3
    achieved = alg / k_avg_s / 1e9
    stage_us = {k: round(v[0] / max(v[1], 1) * 1e3, 2) for k, v in prof.items() if v[1]}
    layer_bytes = U_mean * EXPERT_BYTES + ROUTER_BYTES + 2 * T * H * 2
    line = {
        "metric": "MoE layer tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded; BASELINE config distributions; weights generated on the device)",
        "config": {"workload": cfg["name"], "T": T, "E": E, "K": K, "H": H, "I": I, "weights": "4-bit g64 (router 8-bit)",
                   "parallelism": (f"expert parallel x{world} (NVLink peer all-to-all)" if ep else
                                   f"data parallel x{world} (replicas)" if world > 1 else "single GPU"),
                   "l2": f"inputs larger than L2: steps rotate over {N_ROT} resident layers ({N_ROT * 340} MB)",
                   "path": "prefill (tcgen05 grouped GEMM)" if path == obsmoe.PATH_PREFILL else "decode (mat-vec)"},
        "roofline": {"bound": "hbm", "kernel": kname, "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                     "algorithmic_bytes_per_launch": alg,
                     "traffic": NCU_TRAFFIC.get((top, T)) if world == 1 else None,
                     "kernel_us": k_avg_s * 1e6},
        "layer_hbm_gbs": layer_bytes / (ms / args.steps / 1e3) / 1e9,
        "layer_tflops": 2 * T * K * 4_718_592 / (ms / args.steps / 1e3) / 1e12,
        "stage_us": stage_us, "distinct_experts": U_mean,
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": T * H * 2,
                "d2h_bytes_per_step": T * H * 2},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O

        Lh = O.synth_layer(0, 0, E=E, H=H, I=I, K=K)
        line["cpu_baseline"] = cpu_baseline(Lh, xs[0].cpu().numpy().view(np.uint16), T)
    if dist is not None:
        dist.barrier()  # no rank frees its peer-mapped buffer while another may still use it
    ctx.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line))


if __name__ == "__main__":
    main()
