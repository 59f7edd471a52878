"""Benchmark of the B200 MoE hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 3]

The default workload is BASELINE config 3, the largest single-GPU configuration:
a 48-layer Qwen3-30B-A3B MoE stack (E=128, top-8, H=2048, I=768, 4-bit
group-64 experts, 8-bit router; 16.3 GB of weights resident in HBM), prefill of
T=4096 tokens per GPU with a Zipf(1.1) expert bias on the router logits (the
hottest expert gets ~10x the mean load).  A step is one pass of the batch
through all 48 layers, r <- r + MoE_l(RMSNorm(r)) (obs_moe_stack_forward),
replayed from one CUDA graph.  Configs 0 (one-layer decode of 1 token), 1
(one-layer prefill of 512 tokens) and 2 (48-layer decode of B tokens) are
selectable with --config; on one GPU the default line also carries configs 0
and 1 (`config0`, `config1`), each timed for about half a second.

* value     tokens/s of the whole job, inputs resident in HBM, device-timed
            (CUDA events on the launching stream, barrier + synchronize on both
            sides, max over ranks).  The 48 resident layers (16.3 GB) are far
            larger than the 126 MB L2.
* e2e       the same metric with every step's input copied in from pinned host
            memory and its result copied back inside the timed region.
* roofline  the dominant kernel: for prefill the gate/up grouped GEMM
            (k_gemm<kEpiSwiglu>), algorithmic FLOPs per launch (6,291,456 per
            routed row) over its mean CUDA-event duration in an eager pass of
            one step, against the measured sustained bf16 peak (the kernel runs
            inside a seconds-long step; the burst fraction is also given); the
            whole-stack fraction beside it.  For decode the fused decode layer
            against the measured HBM copy bandwidth.
* cpu_baseline  the C oracle (oracle/, all host threads) on a bounded sample.

Multi-GPU (torchrun): every rank routes its own batch (weak scaling) and the
experts are split E/N per GPU (expert parallelism: routed rows travel to the
rank holding their expert and back over NVLink peer memory); the line reports
all-to-all bytes per GPU per layer and the per-GPU load.  --replicas instead
runs N independent replicas that each hold every expert.

--impl reference times the reference's own kernels (shaders/*.metal compiled
for the CPU into oracle/_ref, strung as src/forward.rs:164-232) on the host
cores, on the same config: each step is a 256-token slice of the same batch
through one layer with the same expert bias, scaled to the stack's layers.
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
GATEUP_FLOPS_PER_ROW = 2 * 2 * I * H   # gate + up of one routed (token, expert) row
LAYER_FLOPS = 2 * K * 4_718_592        # per token and layer (router excluded)
N_ROT = 4                       # resident layers the single-layer configs rotate over
# DRAM bytes (read + write) per launch of the dominant kernel, from one ncu capture of the same
# workload (the committed profile summaries); other workloads report null
NCU_TRAFFIC = {("gemm_gateup", 512): 246_949_888 + 4_585_472, ("decode_fused", 1): 21_645_056,
               # layer 0 of config 3 (T=4096, Zipf bias) captured in a 2-layer stack: the same launch
               ("gemm_gateup_cfg3", 4096): 462_567_680 + 38_029_568}
CONFIGS = {
    0: dict(T=1, name="config0: Qwen3-30B-A3B MoE layer, decode of 1 token"),
    1: dict(T=512, name="config1: Qwen3-30B-A3B MoE layer, batched prefill of T=512 tokens"),
    2: dict(T=None, name="config2: 48-layer MoE stack, decode of B independent tokens per step", stack=True),
    3: dict(T=4096, name="config3: 48-layer MoE stack, prefill of T=4096 tokens, Zipf(1.1) expert bias",
            stack=True),
    4: dict(T=None, name="config4: full Qwen3-30B-A3B forward (random init), prefill of 2048 tokens per sequence "
                         "then greedy decode of 128 tokens at batch B, 4096-token bf16 KV caches", full=True),
}
# config 4: the model around the MoE path (Qwen3MoeConfig)
VOCAB, NQ, NKV, HD, KV_SEQ, PREFILL, DECODE = 151936, 32, 4, 128, 4096, 2048, 128
ATTN_BYTES = (NQ + 2 * NKV) * HD * (H // 8) * 4 + (NQ + 2 * NKV) * HD * (H // 64) * 4 \
    + H * (NQ * HD // 8) * 4 + H * (NQ * HD // 64) * 4  # q/k/v/o codes + scales + biases, one layer
HEAD_BYTES = VOCAB * (H // 8) * 4 + VOCAB * (H // 64) * 4  # lm_head codes + scales + biases
REF_PUBLISHED_DECODE = 3.71  # tokens/s, full-model decode at batch 1 (Apple M4, experts paged from SSD)
EXTRA_SECONDS = 0.5   # timed region of the extra config 0 / config 1 measurements


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=3, choices=sorted(CONFIGS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="config 3 on one GPU: skip the config 0/1 keys")
    ap.add_argument("--batch", type=int, default=0,
                    help="config 2: tokens per decode step (1, 8, 32, 128; default 32); config 4: sequences "
                         "decoded together (1 or 16; default 1)")
    ap.add_argument("--layers", type=int, default=48, help="configs 2 and 3: layers in the stack")
    ap.add_argument("--tokens", type=int, default=0,
                    help="configs 0 and 1: override T (a sweep point, not a BASELINE config)")
    ap.add_argument("--decode-max", type=int, default=0,
                    help="largest T the decode (mat-vec) path takes under OBS_PATH_AUTO (0: the library's default)")
    ap.add_argument("--ref-tokens", type=int, default=256, help="reference arm: tokens per step (a slice of T)")
    ap.add_argument("--placement", default="balanced", choices=["balanced", "contiguous"],
                    help="expert parallelism: experts placed on the GPUs by the routed loads of a separate "
                         "calibration batch (balanced), or GPU g holding experts [g*E/G, (g+1)*E/G)")
    ap.add_argument("--replicas", action="store_true",
                    help="N > 1: N data-parallel replicas (every GPU holds all experts) instead of expert parallelism")
    return ap.parse_args()


def peaks():
    """(HBM GB/s, bf16 TF/s burst, bf16 TF/s sustained, source)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), \
            "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


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


class Ranks:
    """The process group (NCCL) of a multi-GPU run: barriers, max over ranks and
    gathering the host-side statistics -- the data path never goes through it."""

    def __init__(self, world):
        self.dist = None
        if world > 1:
            import datetime

            import torch.distributed as dist

            # no NVLink multicast (NVLS) objects next to the peer buffers the expert exchange writes into
            os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
            self.dist = dist

    def barrier(self):
        import torch

        if self.dist is not None:
            self.dist.barrier()
        torch.cuda.synchronize()

    def max(self, v: float) -> float:
        import torch

        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        if self.dist is not None:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def gather(self, obj):
        if self.dist is None:
            return [obj]
        out = [None] * self.dist.get_world_size()
        self.dist.all_gather_object(out, obj)
        return out

    def close(self):
        if self.dist is not None:
            self.dist.barrier()
            self.dist.destroy_process_group()


def zipf_bias_device(beta):
    import torch

    import synthetic

    return torch.from_numpy(synthetic.zipf_bias(beta, E)).cuda()


def calibrate_beta(ctx, r0, T):
    """beta of config 3's Zipf bias so the hottest expert of layer 0 gets ~10x the mean load."""
    import numpy as np
    import torch

    logits = torch.empty((T, E), dtype=torch.float32, device="cuda")
    ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
    wts = torch.empty((T, K), dtype=torch.float32, device="cuda")
    xn = torch.empty_like(r0)
    ctx.rmsnorm(r0, xn, T)
    ctx.gate_gpu(0, xn, logits, T)
    best = None
    for b in np.linspace(0.0, 8.0, 81):
        ctx.route(logits, T, ids, wts, bias=zipf_bias_device(float(b)))
        load = np.bincount(ids.cpu().numpy().ravel(), minlength=E)
        ratio = load.max() / load.mean()
        if best is None or abs(ratio - 10.0) < abs(best[1] - 10.0):
            best = (float(b), float(ratio))
    return best


def layer_loads(ctx, r_in, nl, T, bias, path, stream):
    """Routed rows per expert of this rank's T tokens at every layer of the stack (the residual
    stream advanced through each layer), [nl][E], and the ids of each layer."""
    import numpy as np
    import torch

    logits = torch.empty((T, E), dtype=torch.float32, device="cuda")
    ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
    wts = torch.empty((T, K), dtype=torch.float32, device="cuda")
    xn = torch.empty_like(r_in)
    rr = r_in.clone()
    counts, all_ids = [], []
    for l in range(nl):
        ctx.rmsnorm(rr, xn, T)
        ctx.gate_gpu(l, xn, logits, T)
        ctx.route(logits, T, ids, wts, bias=bias)
        mine = ids.cpu().numpy().ravel()
        all_ids.append(mine)
        counts.append(np.bincount(mine, minlength=E))
        ctx.moe_stack_forward(l, 1, rr, T, bias=bias, path=path, stream=stream)
    torch.cuda.synchronize()
    return counts, all_ids


def run_stack(args, rank, world, local, ranks):
    """Configs 2 and 3: a stack of MoE layers on a residual stream; a step is one
    pass of the batch through every layer, captured in one CUDA graph."""
    import numpy as np
    import torch

    import obsmoe

    cfg = CONFIGS[args.config]
    nl = args.layers
    T = args.batch if args.config == 2 else cfg["T"]
    decode = args.config == 2
    path = obsmoe.PATH_AUTO if decode else obsmoe.PATH_PREFILL
    ep = world > 1 and not args.replicas
    shape = obsmoe.MoeShape(H, I, E, K, n_layers=nl, max_tokens=max(T, 16), decode_max_tokens=args.decode_max,
                            ep_world=world if ep else 1, ep_rank=rank if ep else 0)
    ctx = obsmoe.MoeContext(shape, local)
    decode_max = args.decode_max if args.decode_max > 0 else 4  # the library's default
    if ep:
        ctx.ep_connect(ranks.gather(ctx.ep_handle()))
    for l in range(nl):
        ctx.synth_layer(l, 0)
    r0 = torch.empty((T, H), dtype=torch.int16, device="cuda")
    obsmoe.synth_activations(rank, 0, 0, T, H, r0)
    stream = torch.cuda.current_stream()
    bias, beta, imbalance0 = None, None, None
    if args.config == 3:
        beta, imbalance0 = calibrate_beta(ctx, r0, T)
        beta = ranks.gather(beta)[0]  # every rank uses rank 0's bias
        bias = zipf_bias_device(beta)
    placement = None
    if ep and args.placement == "balanced":
        # per-layer expert loads of a separate calibration batch (other seeded tokens), summed over
        # the ranks; the same plan on every rank; the layers are generated again for the new placement
        rcal = torch.empty_like(r0)
        obsmoe.synth_activations(rank, 0, T, T, H, rcal)
        cal, _ = layer_loads(ctx, rcal, nl, T, bias, path, stream)
        tot = np.sum(ranks.gather(np.stack(cal)), axis=0)
        placement = [obsmoe.plan_placement(tot[l], world) for l in range(nl)]
        for l in range(nl):
            ctx.ep_set_placement(l, placement[l])
            ctx.synth_layer(l, 0)
        ranks.barrier()
    r = torch.empty_like(r0)

    def step(s=stream):
        r.copy_(r0)
        ctx.moe_stack_forward(0, nl, r, T, bias=bias, path=path, stream=s)

    step()
    ranks.barrier()
    ctx.check_device()
    n0 = obsmoe.kernel_launches()
    step()
    ranks.barrier()
    launches_per_step = obsmoe.kernel_launches() - n0
    cap = torch.cuda.Stream()
    cap.wait_stream(stream)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(cap):
        with torch.cuda.graph(g, stream=cap):
            step(cap)
    stream.wait_stream(cap)
    ranks.barrier()
    for _ in range(max(args.warmup, 3)):
        g.replay()
    ranks.barrier()
    ctx.check_device()
    # ---------------------------------------------------------------- timed region
    clocks = Clocks(local)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ranks.barrier()
    ev0.record(stream)
    for _ in range(args.steps):
        g.replay()
    ev1.record(stream)
    ranks.barrier()
    clk = clocks.stop()
    ms = ranks.max(ev0.elapsed_time(ev1))
    ctx.check_device()
    step_s = ms / args.steps / 1e3
    value = world * T / step_s

    # ---------------------------------------------------------------- e2e
    # every step: the residual batch in from pinned host memory, the stack, the result back
    rh = r0.cpu().pin_memory()
    oh = torch.empty_like(rh).pin_memory()
    ranks.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        r.copy_(rh, non_blocking=True)
        ctx.moe_stack_forward(0, nl, r, T, bias=bias, path=path, stream=stream)
        oh.copy_(r, non_blocking=True)
    e1.record(stream)
    ranks.barrier()
    e2e_value = world * T * args.steps / (ranks.max(e0.elapsed_time(e1)) / 1e3)

    # ------------------------------------------- stage times: one eager step, events per launch
    ctx.profile(True)
    step()
    ranks.barrier()
    prof = ctx.profile_read()
    ctx.profile(False)
    stage_us = {k: round(v[0] / max(v[1], 1) * 1e3, 2) for k, v in prof.items() if v[1]}

    # ---------------------------------- per-layer routing of this step (the same inputs), eagerly
    _, step_ids = layer_loads(ctx, r0, nl, T, bias, path, stream)
    U, loads, local_rows, sent_rows = [], [], [], []
    EL = E // world if ep else E
    for l in range(nl):
        mine = step_ids[l]
        # gpu_of[e]: the GPU holding expert e at this layer
        gpu_of = np.arange(E) // EL
        if placement is not None:
            gpu_of[np.asarray(placement[l])] = np.arange(E) // EL
        if ep:  # rows this rank sends to other ranks: once per (token, rank); outputs back per (token, expert)
            dest = gpu_of[mine].reshape(T, K)
            sent_rows.append((sum(int(np.sum(np.any(dest == d, axis=1))) for d in range(world) if d != rank),
                              int(np.sum(dest != rank))))
        every = np.concatenate(ranks.gather(mine)) if ep else mine
        U.append(len(np.unique(every)))
        cnt = np.bincount(every, minlength=E)
        loads.append(cnt)
        local_rows.append(int(cnt[gpu_of == rank].sum()) if ep else int(cnt.sum()))
    load = np.sum(loads, axis=0)
    hbm, bf16, bf16_sus, peak_kind = peaks()
    if decode:
        # HBM roofline: every routed expert's weights, the router and the activations, per layer
        per_gpu_bytes = (sum(U) * EXPERT_BYTES / world + nl * ROUTER_BYTES + nl * 2 * T * H * 2 * 2)
        achieved = per_gpu_bytes / step_s / 1e9
        roof = {"bound": "hbm", "kernel": f"whole {nl}-layer decode step (router, top-k, 4-bit mat-vecs, combine, "
                f"RMSNorm per layer)", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                "peak_source": f"{peak_kind} copy bandwidth (MEASURED_PEAKS.json hbm_gbs)",
                "algorithmic_bytes_per_launch": per_gpu_bytes, "traffic": None}
    else:
        # the gate/up grouped GEMM: FLOPs of the rows it processed in this step / its event time
        gu_ms, gu_n = prof["gemm_gateup"]
        gu_flops = float(np.mean(local_rows)) * GATEUP_FLOPS_PER_ROW  # per launch (one per layer)
        gu_s = gu_ms / max(gu_n, 1) / 1e3
        achieved = gu_flops / gu_s / 1e12
        stack_tf = nl * T * LAYER_FLOPS / step_s / 1e12
        roof = {"bound": "tensor",
                "kernel": "k_gemm<kEpiSwiglu> (tcgen05 grouped gate/up GEMM + SwiGLU), mean over the step's layers",
                "achieved": achieved, "peak": bf16_sus, "unit": "TFLOP/s", "frac": achieved / bf16_sus,
                "peak_source": f"{peak_kind} sustained bf16 (MEASURED_PEAKS.json bf16_tflops_sustained: the kernel "
                               f"runs inside a {step_s * 1e3:.0f} ms step)",
                "frac_of_burst_peak": achieved / bf16, "burst_peak": bf16,
                "algorithmic_flops_per_launch": gu_flops, "kernel_us": gu_s * 1e6,
                "traffic": NCU_TRAFFIC.get(("gemm_gateup_cfg3", T)) if world == 1 else None,
                "whole_stack": {"achieved": stack_tf, "frac": stack_tf / bf16_sus,
                                "flops_per_step": nl * T * LAYER_FLOPS}}
    line = {
        "metric": "MoE stack tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded; BASELINE config distributions; weights generated on the device)",
        "config": {"workload": cfg["name"], "layers": nl, "T": T, "E": E, "K": K, "H": H, "I": I,
                   "parallelism": (f"expert parallel x{world} (NVLink peer stores)" if ep else
                                   f"data parallel x{world} (replicas)" if world > 1 else "single GPU"),
                   "l2": f"inputs larger than L2: {nl} resident layers ({nl * 340} MB) per step",
                   "path": "decode (mat-vec)" if decode and T <= decode_max and not ep else
                           "prefill (tcgen05 grouped GEMM)",
                   "zipf_beta": beta},
        "roofline": roof, "stage_us": stage_us, "distinct_experts_per_layer": float(np.mean(U)),
        "load": {"expert_max_over_mean_layer0": imbalance0,
                 "expert_max_over_mean_all_layers": float(load.max() / load.mean())},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": T * H * 2,
                "d2h_bytes_per_step": T * H * 2},
        "gpu_launches": launches_per_step * args.steps, "clocks": clk,
    }
    if ep:
        rows_per_gpu = ranks.gather(float(np.mean(local_rows)))
        sent = ranks.gather([float(np.mean([r[0] for r in sent_rows])), float(np.mean([r[1] for r in sent_rows]))])
        line["ep"] = {"experts_per_gpu": EL,
                      "placement": ("balanced: per-layer greedy plan (obs_ep_plan_placement) from the routed "
                                    "loads of a separate seeded calibration batch" if placement is not None else
                                    "contiguous: GPU g holds experts [g*E/G, (g+1)*E/G)"),
                      "rows_per_gpu_per_layer": rows_per_gpu,
                      "gpu_rows_max_over_mean": float(max(rows_per_gpu) / np.mean(rows_per_gpu)),
                      "a2a_bytes_per_gpu_per_layer": {"dispatch": [s[0] * H * 2 for s in sent],
                                                      "combine": [s[1] * H * 2 for s in sent],
                                                      "row_bytes": H * 2},
                      "note": "over NVLink: a token row goes to another GPU once per (token, GPU) however many of "
                              "its experts live there; outputs come back once per (token, expert) pair; rows and "
                              "outputs that stay on their GPU do not move"}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O

        # bounded sample: 2 layers and at most 64 tokens through the C oracle, scaled to the stack
        nlo, Ts = 2, min(T, 64)
        Ls = [O.synth_layer(0, l, E=E, H=H, I=I, K=K) for l in range(nlo)]
        rs = r0[:Ts].cpu().numpy().view(np.uint16)
        n = os.cpu_count() or 1
        t0 = time.perf_counter()
        O.moe_stack(Ls, rs, bias=None if bias is None else bias.cpu().numpy(), nthreads=n)
        dt = (time.perf_counter() - t0) * nl / nlo
        line["cpu_baseline"] = {"value": Ts / dt, "unit": "tokens/s", "cores": n, "kind": "port",
                                "sample": f"{Ts} tokens through {nlo} layers of oracle/obs_oracle.c, "
                                          f"time scaled to {nl} layers"}
    ranks.barrier()  # no rank frees its peer-mapped buffer while another may still use it
    del g
    ctx.close()
    return line


def run_layer(args, cfg_id, rank, world, local, ranks, steps, warmup, tokens=0, cpu=True):
    """Configs 0 and 1: one MoE layer per step, steps rotating over N_ROT resident
    layers, each replayed from a CUDA graph of its forward."""
    import numpy as np
    import torch

    import obsmoe

    cfg = dict(CONFIGS[cfg_id])
    if tokens:
        cfg["T"], cfg["name"] = tokens, cfg["name"].split(",")[0] + f", T={tokens} tokens (sweep)"
    T = cfg["T"]
    ep = world > 1 and not args.replicas
    path = obsmoe.PATH_DECODE if T <= 2 and not ep else obsmoe.PATH_PREFILL
    shape = obsmoe.MoeShape(H, I, E, K, n_layers=N_ROT, max_tokens=max(T, 16),
                            ep_world=world if ep else 1, ep_rank=rank if ep else 0)
    ctx = obsmoe.MoeContext(shape, local)
    if ep:
        ctx.ep_connect(ranks.gather(ctx.ep_handle()))
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

    for i in range(max(warmup, 3)):
        step(i)
    ctx.check_device()
    n0 = obsmoe.kernel_launches()
    step(0)
    launches_per_step = obsmoe.kernel_launches() - n0
    # one graph per layer, and one graph of N_ROT consecutive steps (layers 0..N_ROT-1, the way
    # a decode loop over layers runs): the timed region replays the latter, then single steps
    # for the remainder, so it runs exactly `steps` forwards
    graphs = []
    cap = torch.cuda.Stream()
    cap.wait_stream(stream)
    with torch.cuda.stream(cap):
        for l in range(N_ROT):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                ctx.moe_forward(l, xs[l], out, T, path=path, stream=cap)
            graphs.append(g)
        g_rot = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_rot, stream=cap):
            for l in range(N_ROT):
                ctx.moe_forward(l, xs[l], out, T, path=path, stream=cap)
    stream.wait_stream(cap)
    for i in range(max(warmup, 3)):
        graphs[i % N_ROT].replay()
    g_rot.replay()
    ranks.barrier()
    ctx.check_device()
    # ------------------------------------------------------------ timed region
    clocks = Clocks(local)
    ranks.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for i in range(steps // N_ROT):
        g_rot.replay()
    for i in range(steps % N_ROT):
        graphs[i].replay()
    ev1.record(stream)
    ranks.barrier()
    clk = clocks.stop()
    ms = ranks.max(ev0.elapsed_time(ev1))
    ctx.check_device()
    # stage times from a separate, eager pass (events between the stages)
    ctx.profile(True)
    for i in range(min(steps, 200)):
        step(i)
    torch.cuda.synchronize()
    prof = ctx.profile_read()
    ctx.profile(False)
    value = world * T * steps / (ms / 1e3)

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
    ranks.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        host_step(i)
    ctx.host_join(stream)  # the last step's result is in host memory before e1
    e1.record(stream)
    stream.synchronize()
    ranks.barrier()
    e2e_value = world * T * steps / (ranks.max(e0.elapsed_time(e1)) / 1e3)

    # ------------------------------------------------ roofline of the top kernel
    hbm, _, _, peak_kind = peaks()
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
            mine = np.concatenate(ranks.gather(mine))
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
    if top == "decode_fused" and launches_per_step == 1:
        # the timed region is that one kernel per step: its per-step time (CUDA events over the
        # graph replays) bounds the launch's duration better than the eager, event-bracketed pass
        k_avg_s = min(k_avg_s, ms / steps / 1e3)
    achieved = alg / k_avg_s / 1e9
    stage_us = {k: round(v[0] / max(v[1], 1) * 1e3, 2) for k, v in prof.items() if v[1]}
    layer_bytes = U_mean * EXPERT_BYTES + ROUTER_BYTES + 2 * T * H * 2
    line = {
        "metric": "MoE layer tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": steps, "warmup": max(warmup, 3), "ms_per_step": ms / steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded; BASELINE config distributions; weights generated on the device)",
        "config": {"workload": cfg["name"], "T": T, "E": E, "K": K, "H": H, "I": I,
                   "weights": "4-bit g64 (router 8-bit)",
                   "parallelism": (f"expert parallel x{world} (NVLink peer stores)" if ep else
                                   f"data parallel x{world} (replicas)" if world > 1 else "single GPU"),
                   "l2": f"inputs larger than L2: steps rotate over {N_ROT} resident layers ({N_ROT * 340} MB)",
                   "path": "prefill (tcgen05 grouped GEMM)" if path == obsmoe.PATH_PREFILL else "decode (mat-vec)"},
        "roofline": {"bound": "hbm", "kernel": kname, "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "peak_source": f"{peak_kind} copy bandwidth (MEASURED_PEAKS.json hbm_gbs)",
                     "algorithmic_bytes_per_launch": alg,
                     "traffic": NCU_TRAFFIC.get((top, T)) if world == 1 else None,
                     "kernel_us": k_avg_s * 1e6},
        "layer_hbm_gbs": layer_bytes / (ms / steps / 1e3) / 1e9,
        "layer_tflops": 2 * T * K * 4_718_592 / (ms / steps / 1e3) / 1e12,
        "stage_us": stage_us, "distinct_experts": U_mean,
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": T * H * 2,
                "d2h_bytes_per_step": T * H * 2},
        "gpu_launches": launches_per_step * steps,
        "clocks": clk,
    }
    if cpu and rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O

        Lh = O.synth_layer(0, 0, E=E, H=H, I=I, K=K)
        xh0 = xs[0].cpu().numpy().view(np.uint16)
        n = os.cpu_count() or 1
        t0 = time.perf_counter()
        O.moe_layer(Lh, xh0, nthreads=n)
        dt = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": T / dt, "unit": "tokens/s", "cores": n, "kind": "port",
                                "sample": f"the full {T}-token layer once through oracle/obs_oracle.c ({dt:.2f} s)"}
    ranks.barrier()
    del graphs
    ctx.close()
    return line


class RandLinear4:
    """Random weights of one MLX 4-bit group-64 linear layer on the device: uniform codes, bf16
    scales U(lo, hi) and biases -8*scale + N(0, 1e-3) (the expert weights' distribution)."""

    def __init__(self, torch, gen, rows, in_f, lo=0.002, hi=0.02):
        self.w = torch.randint(-2 ** 31, 2 ** 31 - 1, (rows, in_f // 8), dtype=torch.int32, device="cuda",
                               generator=gen)
        sc = torch.empty((rows, in_f // 64), device="cuda").uniform_(lo, hi, generator=gen)
        self.s = sc.to(torch.bfloat16)
        self.b = (-8.0 * sc + 1e-3 * torch.randn(sc.shape, device="cuda", generator=gen)).to(torch.bfloat16)


def run_full(args, rank, world, local, ranks):
    """Config 4: the whole model through the library's entry points -- embed, 48 x (attention
    block, then RMSNorm + MoE + residual), final norm + lm_head + greedy token -- with random
    weights generated on the device.  Each of B sequences is prefilled with 2048 random tokens
    (256-token chunks, eager, timed as the prefill rate), then 128 greedy decode steps of all B
    sequences at once are timed, each step one CUDA graph replay.  N > 1: N replicas."""
    import types

    import numpy as np
    import torch

    import obsmoe

    cfg = CONFIGS[args.config]
    B, nl, C = args.batch, args.layers, 256
    stream = torch.cuda.current_stream()
    shape = obsmoe.MoeShape(H, I, E, K, n_layers=nl, max_tokens=C, decode_max_tokens=args.decode_max)
    ctx = obsmoe.MoeContext(shape, local)
    ctx.attn_init(NQ, NKV, HD, KV_SEQ, B, 1e7)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(4 + 1000 * rank)
    ones = lambda n: torch.ones(n, dtype=torch.bfloat16, device="cuda")  # noqa: E731
    for l in range(nl):
        ctx.synth_layer(l, 0)
        q, k, v = (RandLinear4(torch, gen, n * HD, H) for n in (NQ, NKV, NKV))
        o = RandLinear4(torch, gen, H, NQ * HD)
        w = types.SimpleNamespace(q_w=q.w, q_s=q.s, q_b=q.b, k_w=k.w, k_s=k.s, k_b=k.b, v_w=v.w, v_s=v.s, v_b=v.b,
                                  o_w=o.w, o_s=o.s, o_b=o.b, in_norm=ones(H), q_norm=ones(HD), k_norm=ones(HD))
        ctx.load_attn(l, w, on_device=True)
    emb, lm = RandLinear4(torch, gen, VOCAB, H, 0.001, 0.01), RandLinear4(torch, gen, VOCAB, H, 0.001, 0.01)
    ctx.load_head(VOCAB, types.SimpleNamespace(embed_w=emb.w, embed_s=emb.s, embed_b=emb.b, lm_w=lm.w, lm_s=lm.s,
                                               lm_b=lm.b, norm_w=ones(H)), on_device=True)
    del emb, lm
    torch.cuda.synchronize()
    xa = torch.empty((C, H), dtype=torch.int16, device="cuda")
    xb = torch.empty_like(xa)

    def layers(n, seqs, pos, st):
        """The residual rows xa[:n] through every layer (ping-pong through xb); ends in xa."""
        x, y = xa, xb
        for l in range(nl):
            ctx.attn_forward(l, x, y, n, seqs, pos, stream=st)
            ctx.moe_stack_forward(l, 1, y, n, path=obsmoe.PATH_AUTO, stream=st)
            x, y = y, x
        return x

    # ---- prefill: every sequence's 2048 random tokens, 256 at a time; its last row gives its first token
    prompts = torch.randint(0, VOCAB, (B, PREFILL), dtype=torch.int32, device="cuda", generator=gen)
    ids = torch.empty(B, dtype=torch.int32, device="cuda")
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ranks.barrier()
    p0.record(stream)
    for sq in range(B):
        seq_c = torch.full((C,), sq, dtype=torch.int32, device="cuda")
        for c0 in range(0, PREFILL, C):
            pos_c = torch.arange(c0, c0 + C, dtype=torch.int32, device="cuda")
            ctx.embed(prompts[sq, c0:c0 + C], C, xa, stream=stream)
            last = layers(C, seq_c, pos_c, stream)
        ctx.lm_head(last[C - 1:C], 1, ids[sq:sq + 1], stream=stream)
    p1.record(stream)
    ranks.barrier()
    prefill_s = ranks.max(p0.elapsed_time(p1)) / 1e3
    ctx.check_device()

    # ---- decode: one token of every sequence per step, positions 2048, 2049, ...
    seqs = torch.arange(B, dtype=torch.int32, device="cuda")
    pos = torch.full((B,), PREFILL, dtype=torch.int32, device="cuda")

    def dstep(st):
        ctx.embed(ids, B, xa, stream=st)
        ctx.lm_head(layers(B, seqs, pos, st)[:B], B, ids, stream=st)
        pos.add_(1)

    # one eager step that also records the distinct experts each layer routes to (the HBM bytes)
    logits = torch.empty((B, E), dtype=torch.float32, device="cuda")
    rids = torch.empty((B, K), dtype=torch.int32, device="cuda")
    rw = torch.empty((B, K), dtype=torch.float32, device="cuda")
    xn = torch.empty((B, H), dtype=torch.int16, device="cuda")
    U = []
    ctx.embed(ids, B, xa, stream=stream)
    x, y = xa, xb
    for l in range(nl):
        ctx.attn_forward(l, x, y, B, seqs, pos, stream=stream)
        ctx.rmsnorm(y[:B], xn, B, stream=stream)
        ctx.gate_gpu(l, xn, logits, B, stream=stream)
        ctx.route(logits, B, rids, rw, stream=stream)
        U.append(len(np.unique(rids.cpu().numpy())))
        ctx.moe_stack_forward(l, 1, y, B, path=obsmoe.PATH_AUTO, stream=stream)
        x, y = y, x
    ctx.lm_head(x[:B], B, ids, stream=stream)
    pos.add_(1)
    n0 = obsmoe.kernel_launches()
    dstep(stream)
    torch.cuda.synchronize()
    launches_per_step = obsmoe.kernel_launches() - n0
    cap = torch.cuda.Stream()
    cap.wait_stream(stream)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(cap):
        with torch.cuda.graph(g, stream=cap):
            dstep(cap)
    stream.wait_stream(cap)
    for _ in range(max(args.warmup, 3) - 2):
        g.replay()
    ranks.barrier()
    ctx.check_device()
    clocks = Clocks(local)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ranks.barrier()
    ev0.record(stream)
    for _ in range(DECODE):
        g.replay()
    ev1.record(stream)
    ranks.barrier()
    clk = clocks.stop()
    ms = ranks.max(ev0.elapsed_time(ev1))
    ctx.check_device()
    step_s = ms / DECODE / 1e3
    last_pos = int(pos[0].item())
    # e2e: the same steps with each step's tokens read back to pinned host memory (a serving loop)
    ids_host = torch.empty(B, dtype=torch.int32).pin_memory()
    pos.fill_(last_pos - DECODE)  # rewrite the last 128 positions of the caches
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ranks.barrier()
    e0.record(stream)
    for _ in range(DECODE):
        g.replay()
        ids_host.copy_(ids, non_blocking=True)
    e1.record(stream)
    ranks.barrier()
    e2e_s = ranks.max(e0.elapsed_time(e1)) / 1e3 / DECODE
    finite = bool(torch.isfinite(xa[:B].view(torch.bfloat16).float()).all().item())
    del g
    ctx.check_device()

    # HBM roofline of a decode step: every layer's attention weights, its router and routed
    # experts, the KV cache rows read (mean position of the timed steps), the lm_head
    hbm, _, _, peak_kind = peaks()
    mean_pos = last_pos - DECODE / 2
    kv_bytes = nl * B * 2 * NKV * (mean_pos + 1) * HD * 2
    step_bytes = nl * (ATTN_BYTES + ROUTER_BYTES) + sum(U) * EXPERT_BYTES + kv_bytes + HEAD_BYTES
    achieved = step_bytes / step_s / 1e9
    value = world * B / step_s
    line = {
        "metric": "full-model decode tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": DECODE, "warmup": max(args.warmup, 3), "ms_per_step": step_s * 1e3, "higher_is_better": True,
        "scaling": "weak", "dtype": "bf16",
        "vs_baseline": value / REF_PUBLISHED_DECODE if B == 1 and world == 1 else None,
        "vs_baseline_note": "the reference's published full-model decode, 3.71 tokens/s at batch 1 on an Apple M4 "
                            "with experts paged from SSD (other hardware)",
        "data": "synthetic (random weights generated on the device: MoE layers seeded as configs 2/3, attention and "
                "head uniform 4-bit codes; random prompt tokens)",
        "config": {"workload": cfg["name"], "batch": B, "layers": nl, "prefill_tokens": PREFILL,
                   "decode_tokens": DECODE, "kv_cache": KV_SEQ, "vocab": VOCAB,
                   "parallelism": f"data parallel x{world} (replicas)" if world > 1 else "single GPU",
                   "l2": f"inputs larger than L2: {nl} resident layers per step",
                   "moe_path": "decode (fused layer)" if B <= 4 else "grouped GEMM"},
        "prefill": {"tokens_per_s": world * B * PREFILL / prefill_s, "seconds": prefill_s,
                    "note": "eager, 256-token chunks, attention by 16-row mat-vec projections"},
        "roofline": {"bound": "hbm", "kernel": "whole decode step (attention, MoE, lm_head)", "achieved": achieved,
                     "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_source": f"{peak_kind} copy bandwidth (MEASURED_PEAKS.json hbm_gbs)",
                     "algorithmic_bytes_per_launch": step_bytes, "distinct_experts_per_layer": float(np.mean(U)),
                     "traffic": None},
        "e2e": {"value": world * B / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": B * 4},
        "gpu_launches": launches_per_step * DECODE, "clocks": clk, "finite": finite,
    }
    ranks.barrier()
    return line


def extra_summary(line):
    """The keys of a config 0 / config 1 line that the default line carries."""
    keep = ("value", "unit", "ms_per_step", "steps", "roofline", "stage_us", "e2e", "gpu_launches", "clocks",
            "layer_hbm_gbs", "layer_tflops", "distinct_experts")
    out = {k: line[k] for k in keep if k in line}
    out["workload"] = line["config"]["workload"]
    out["path"] = line["config"]["path"]
    return out


def run_reference(args, rank, world):
    """The reference's own kernels on the host cores (oracle/_ref), on the same config."""
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    import synthetic

    cfg = CONFIGS[args.config]
    if cfg.get("full"):
        print(json.dumps({"impl": "reference", "unavailable": "config 4 (the full forward after a 2048-token "
                          "prefill) has no bounded CPU sample: the reference's host kernels cover the MoE path "
                          "only, and a CPU prefill of 2048 tokens through 48 layers takes hours"}))
        return
    T = cfg["T"] if cfg["T"] is not None else args.batch
    if O.ref_lib() is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libobs_refshaders.so was not built"}))
        return
    n = os.cpu_count() or 1
    Ts = min(T, args.ref_tokens)
    L = O.synth_layer(0, 0, E=E, H=H, I=I, K=K)
    # the same inputs as our arm: rank 0's residual batch; the layer input is its RMSNorm
    r = O.synth_x(0, 0, T, H)
    x = O.rmsnorm_layer(r)
    bias = synthetic.zipf_bias(synthetic.CONFIG3_BETA, E) if args.config == 3 else None

    def ref_step(i):
        lo = (i * Ts) % T
        O.ref_moe_prefill(L, x[lo:lo + Ts], residual=r[lo:lo + Ts], bias=bias, nthreads=n)

    for i in range(args.warmup):
        ref_step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        ref_step(i)
    dt = time.perf_counter() - t0
    value = Ts * args.steps / dt
    metric = "MoE layer tokens/s"
    sample = (f"{Ts} of the {T} tokens per step (slice i*{Ts} mod {T}; each token's work is independent of "
              f"the others') through the reference's shaders/*.metal kernels compiled for the CPU (oracle/_ref), "
              f"strung as src/forward.rs:164-232, {n} threads")
    config = {"workload": cfg["name"], "T": T, "E": E, "K": K, "H": H, "I": I}
    if cfg.get("stack"):  # one layer per step, time scaled to the stack's layers
        value /= args.layers
        metric = "MoE stack tokens/s"
        config["layers"] = args.layers
        sample += f"; one layer per step, time scaled to {args.layers} layers"
    if bias is not None:
        sample += "; the Zipf expert bias added to the reference's logits before its top-k kernel"
    print(json.dumps({
        "impl": "reference", "metric": metric, "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded, BASELINE config distributions)",
        "config": config,
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": n, "kind": "reference", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def main():
    args = parse()
    if args.batch <= 0:
        args.batch = 1 if args.config == 4 else 32
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    import torch

    torch.cuda.set_device(local)
    ranks = Ranks(world)
    if CONFIGS[args.config].get("full"):
        line = run_full(args, rank, world, local, ranks)
    elif CONFIGS[args.config].get("stack"):
        line = run_stack(args, rank, world, local, ranks)
        if args.config == 3 and world == 1 and not args.no_extras:
            # the decode target (config 0) and config 1, each timed for ~EXTRA_SECONDS
            line["config0"] = extra_summary(run_layer(args, 0, rank, world, local, ranks,
                                                      steps=int(EXTRA_SECONDS / 27e-6), warmup=20, cpu=False))
            line["config1"] = extra_summary(run_layer(args, 1, rank, world, local, ranks,
                                                      steps=int(EXTRA_SECONDS / 130e-6), warmup=10, cpu=False))
    else:
        line = run_layer(args, args.config, rank, world, local, ranks, args.steps, args.warmup, tokens=args.tokens)
    ranks.close()
    if rank == 0:
        print(json.dumps(line))


if __name__ == "__main__":
    main()
