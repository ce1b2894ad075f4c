#!/usr/bin/env python
"""MoE-layer forward benchmark (metric: MoE-layer tokens/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c5] [--impl ours|reference]

One step = one MixtureOfExperts.Forward of the config's whole token batch
(whole-job: all ranks' tokens).  Under torchrun (N > 1) each rank owns T/N
tokens; the default workload is config c5 (65536 tokens x d 4096,
256 routed experts + 1 shared, hidden 2048, top-8, FP4 experts, bf16
activations, Zipf(1.0) router bias), the configuration the metric is quoted
on at 1/2/4/8 GPUs.  Inputs are seeded synthetic data of the config's shape
(no dataset exists for this path); every input exceeds the 126 MB L2 (x is
512 MiB, the expert weights 4.85 GB), so no L2 flush is needed between steps.

Rank 0 prints one JSON line.  `value` is device-resident throughput (CUDA
events on the launching stream, max over ranks); `e2e` is the same metric
through the C-ABI call with pinned host buffers, host<->device copies inside
the timed region; `roofline` is the dominant kernel (the grouped expert
GEMMs) timed live by the library's per-phase CUDA events; `cpu_baseline` is
the CPU oracle (a C float64 restatement of the reference algorithm, all host
cores) on a seeded token sample.

`--impl reference` times the reference's CPU algorithm instead (the oracle
port; the Go reference cannot be built here) on the same config, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--config", default="c5")
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--mode", default="auto", choices=["auto", "ep", "replicas"],
                   help="multi-GPU mode: expert parallel (routed experts sharded by index; token rows and the "
                        "per-expert counts exchanged by peer stores over NVLink) or token-sharded replicas of the "
                        "whole layer")
    p.add_argument("--replicas", default="auto",
                   help="expert parallel: hot experts held on every rank ('auto': chosen from the config's expected "
                        "expert popularity, '0': none -- routed experts purely owned by index, or a number: the "
                        "hottest experts chosen the same way, at most that many)")
    p.add_argument("--op", default="forward", choices=["forward", "block", "backward"],
                   help="forward: MixtureOfExperts.Forward (gtmoe_forward); block: the block's feed-forward step "
                        "x + Forward(RMSNorm(x)) (gtmoe_forward_block, one GPU); backward: a training step's "
                        "mixture part, Forward then Backward (gtmoe_backward: input and router gradients, "
                        "frozen compressed experts; float64, one GPU)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-seconds", type=float, default=15.0)
    return p.parse_args()


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            j = json.load(f)
        return {"hbm_gbs": j["hbm_gbs"], "bf16_tflops": j["bf16_tflops"],
                "bf16_tflops_sustained": j.get("bf16_tflops_sustained", j["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ----------------------------------------------------------------- clocks

CLOCK_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


def physical_gpu_index(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        parts = [p for p in vis.split(",") if p.strip()]
        try:
            return int(parts[local_rank])
        except (ValueError, IndexError):
            return local_rank
    return local_rank


class ClockSampler:
    def __init__(self):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={CLOCK_FIELDS}", "--format=csv,noheader,nounits",
                                       "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self, gpu_index: int):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.flush()
        self.f.seek(0)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f.read().splitlines():
            parts = [q.strip() for q in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                if int(parts[0]) != gpu_index:
                    continue
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.f.name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------- CPU oracle

def oracle_spec(cfg, host):
    from oracle import oracle as O

    wr, rb = host[("router",)]
    router = O.Layer(O.FLOAT64, cfg.n_routed, cfg.d, np.ascontiguousarray(wr).reshape(-1), None,
                     np.ascontiguousarray(rb, np.float64))
    experts = []
    for e in range(cfg.n_shared + cfg.n_routed):
        layers = []
        for which, (rows, width) in enumerate([(cfg.h, cfg.d), (cfg.h, cfg.d), (cfg.d, cfg.h)]):
            codes, scales = host[(e, which)]
            layers.append(O.Layer(cfg.precision, rows, width, codes, scales, None))
        experts.append(tuple(layers))
    return O.MoESpec(d=cfg.d, h=cfg.h, n_shared=cfg.n_shared, n_routed=cfg.n_routed, k=cfg.k, router=router,
                     experts=experts)


def time_oracle(spec, x_all, budget_s: float, threads: int, min_tokens: int = 2):
    """Runs the oracle on a seeded token sample sized for ~budget_s seconds;
    returns (tokens/s, tokens, seconds)."""
    from oracle import oracle as O

    rng = np.random.default_rng(123)
    T = x_all.shape[0]
    probe = np.sort(rng.choice(T, size=min(min_tokens, T), replace=False))
    t0 = time.perf_counter()
    O.moe_forward(spec, x_all[probe], probe.astype(np.int64), threads=threads)
    per_tok = max((time.perf_counter() - t0) / len(probe), 1e-6)
    n = int(min(T, max(min_tokens, budget_s / per_tok)))
    sample = np.sort(rng.choice(T, size=n, replace=False))
    t0 = time.perf_counter()
    O.moe_forward(spec, x_all[sample], sample.astype(np.int64), threads=threads)
    dt = time.perf_counter() - t0
    return n / dt, n, dt


def time_oracle_backward(spec, x_all, g_all, budget_s: float, min_tokens: int = 2):
    """Forward + Backward of the oracle on a seeded token sample sized for
    ~budget_s seconds; returns (tokens/s, tokens, seconds)."""
    from oracle import oracle as O

    rng = np.random.default_rng(321)
    T = x_all.shape[0]
    probe = np.sort(rng.choice(T, size=min(min_tokens, T), replace=False))
    t0 = time.perf_counter()
    O.moe_backward(spec, x_all[probe], g_all[probe])
    per_tok = max((time.perf_counter() - t0) / len(probe), 1e-6)
    n = int(min(T, max(min_tokens, budget_s / per_tok)))
    sample = np.sort(rng.choice(T, size=n, replace=False))
    t0 = time.perf_counter()
    O.moe_backward(spec, x_all[sample], g_all[sample])
    dt = time.perf_counter() - t0
    return n / dt, n, dt


# ------------------------------------------------------------------ main

def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and not (world == 1 and args.gpus == 1):
        print(f"bench.py: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)

    from gotransformers_b200 import synthetic

    cfg = synthetic.CONFIGS[args.config]
    metric = "MoE-layer tokens/s"
    if args.impl == "reference":
        return run_reference(args, cfg, rank, world, local_rank, metric)

    import torch
    import torch.distributed as dist

    from gotransformers_b200 import _lib
    from gotransformers_b200 import moe as M

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
    mode = args.mode
    if mode == "auto":
        mode = "replicas" if world == 1 else "ep"

    T_total = cfg.T
    if T_total % world:
        raise SystemExit(f"{T_total} tokens do not split over {world} ranks")
    T_local = T_total // world
    if world > 1 and mode == "ep":
        nccl_id = bytearray(128)
        if rank == 0:
            import ctypes

            _lib.check(_lib.lib().gtmoe_ep_unique_id((ctypes.c_char * 128).from_buffer(nccl_id)))
        obj = [bytes(nccl_id)]
        dist.broadcast_object_list(obj, src=0)
        moe = M.MixtureOfExperts(cfg.d, cfg.h, cfg.n_shared, cfg.n_routed, cfg.k, weight_precision=cfg.precision,
                                 device=local_rank, ep_ranks=world, ep_rank=rank, nccl_id=obj[0])
        reps = bench_replicas(args, cfg, world)
        if reps:
            moe.set_replicas(reps)
    else:
        moe = M.MixtureOfExperts(cfg.d, cfg.h, cfg.n_shared, cfg.n_routed, cfg.k, weight_precision=cfg.precision,
                                 device=local_rank)
    want_cpu = rank == 0 and world == 1 and not args.no_cpu_baseline
    host = synthetic.load_config_on_gpu(cfg, moe, keep_host=want_cpu, device=local_rank)
    x = synthetic.make_x_on_gpu(cfg, T=T_local, offset_rows=rank * T_local, device=local_rank)
    out = torch.empty((T_local, cfg.d), dtype=torch.bfloat16, device=dev)
    if args.op == "block":
        if world > 1:
            raise SystemExit("--op block runs on one GPU")
        # the block's FeedForwardNorm: seeded RMSNorm weights around 1
        moe.set_norm(1.0 + 0.1 * synthetic.normal(cfg.weight_seed, synthetic.STREAM_NORM, cfg.d), 1e-6)
        out = torch.empty_like(x)  # the block's output has the input's dtype (x is the residual)
    grads = None
    if args.op == "backward":
        if world > 1:
            raise SystemExit("--op backward runs on one GPU")
        moe.set_training(True)
        # seeded N(0,1) output gradients; the input gradients in float32;
        # the router's gradients accumulate into float64 storage
        gen = torch.Generator(device=dev).manual_seed(cfg.act_seed + 17)
        dout = torch.randn((T_local, cfg.d), generator=gen, device=dev, dtype=torch.float32)
        grads = {"dout": dout, "dx": torch.empty_like(dout),
                 "gw": torch.zeros((cfg.n_routed, cfg.d), dtype=torch.float64, device=dev),
                 "gb": torch.zeros((cfg.n_routed,), dtype=torch.float64, device=dev)}

    def step(xx, oo, g=None):
        if args.op == "block":
            moe.forward_block(xx, out=oo, want_routing=False)
        else:
            moe.forward(xx, out=oo, want_routing=False)
        if args.op == "backward":
            g = g or grads
            moe.backward(g["dout"], input_gradients=g["dx"], router_weight_grad=g["gw"], router_bias_grad=g["gb"])
    # a dedicated stream: torch's default (legacy) stream has handle 0, which
    # the C ABI reads as "the handle's own stream"
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    moe.set_stream(stream.cuda_stream)

    def barrier():
        if world > 1:
            dist.barrier()

    # clocks: nvidia-smi starts sampling before the warm-up steps, so that it
    # is running through the whole timed region, and stops right after it
    sampler = ClockSampler()
    for _ in range(args.warmup):
        step(x, out)
    torch.cuda.synchronize(dev)
    barrier()

    L = _lib.lib()
    import ctypes

    launches = ctypes.c_int64()
    _lib.check(L.gtmoe_read_timing(moe.handle, None, 0, None, ctypes.byref(launches)))  # restarts the count
    torch.cuda.synchronize(dev)
    barrier()
    # decode-shaped batches touch less than a few L2s of weights: write a
    # buffer larger than L2 between steps (outside each step's events)
    flush = decode_shaped(cfg)
    flush_buf = torch.empty((512 << 20) // 4, dtype=torch.int32, device=dev) if flush else None
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps if flush else 1)]
    torch.cuda.nvtx.range_push("timed")  # lets ncu list exactly the timed launches (--nvtx-include timed/)
    if flush:
        for i in range(args.steps):
            flush_buf.fill_(i)
            evs[i][0].record(stream)
            step(x, out)
            evs[i][1].record(stream)
    else:
        evs[0][0].record(stream)
        for _ in range(args.steps):
            step(x, out)
        evs[0][1].record(stream)
    evs[-1][1].synchronize()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize(dev)
    barrier()
    clocks = sampler.stop(physical_gpu_index(local_rank))
    ms = sum(a.elapsed_time(b) for a, b in evs) / args.steps
    _lib.check(L.gtmoe_read_timing(moe.handle, None, 0, None, ctypes.byref(launches)))  # kernels in the timed steps

    # the split of a step into phases: a separate pass with the library's
    # per-phase CUDA events (which run the forward without graph replay)
    phase_ms = (ctypes.c_double * _lib.N_PHASES)()
    calls, plaunch = ctypes.c_int64(), ctypes.c_int64()
    _lib.check(L.gtmoe_set_timing(moe.handle, 1))
    for i in range(min(args.steps, 5)):
        if flush:
            flush_buf.fill_(i)
        # ranks start each step together, so a rank's count-exchange phase
        # holds the exchange itself, not another rank's host lag
        barrier()
        step(x, out)
    _lib.check(L.gtmoe_read_timing(moe.handle, phase_ms, _lib.N_PHASES, ctypes.byref(calls), ctypes.byref(plaunch)))
    _lib.check(L.gtmoe_set_timing(moe.handle, 0))
    phases = {n: phase_ms[i] / max(calls.value, 1) for i, n in enumerate(_lib.PHASES)}
    bwd_ms = None
    if grads is not None:
        # the backward alone: events around gtmoe_backward after each forward
        bev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(min(args.steps, 5))]
        for a_ev, b_ev in bev:
            moe.forward(x, out=out, want_routing=False)
            a_ev.record(stream)
            moe.backward(grads["dout"], input_gradients=grads["dx"], router_weight_grad=grads["gw"],
                         router_bias_grad=grads["gb"])
            b_ev.record(stream)
        bev[-1][1].synchronize()
        bwd_ms = sum(a_ev.elapsed_time(b_ev) for a_ev, b_ev in bev) / len(bev)

    # end to end through the C ABI with pinned host buffers
    x_host = x.cpu().pin_memory()
    out_host = torch.empty((T_local, cfg.d), dtype=out.dtype).pin_memory()
    g_host = None
    if grads is not None:
        g_host = {"dout": grads["dout"].cpu().pin_memory(), "dx": grads["dx"].cpu().pin_memory(),
                  "gw": grads["gw"], "gb": grads["gb"]}
    for _ in range(2):
        step(x_host, out_host, g_host)
    barrier()
    e2e_steps = max(3, args.steps // 2)
    eevs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            for _ in range(e2e_steps if flush else 1)]
    if flush:
        for i in range(e2e_steps):
            flush_buf.fill_(i)
            eevs[i][0].record(stream)
            step(x_host, out_host, g_host)
            eevs[i][1].record(stream)
    else:
        eevs[0][0].record(stream)
        for _ in range(e2e_steps):
            step(x_host, out_host, g_host)
        eevs[0][1].record(stream)
    eevs[-1][1].synchronize()
    barrier()
    e2e_ms = sum(a.elapsed_time(b) for a, b in eevs) / e2e_steps

    # expert rows this rank ran: its tokens through the shared experts plus the
    # rows routed to the experts it owns
    sent_bytes = recv_bytes = 0
    if world > 1 and mode == "ep":
        # each rank's load counts its own tokens; an owned expert's rows come
        # from all ranks, a replicated expert's only from this rank's tokens
        own = moe.last_expert_load()
        load = torch.from_numpy(own).to(dev)
        dist.all_reduce(load)
        glob = load.cpu().numpy()
        el = cfg.n_routed // world
        rep = set(getattr(moe, "replicas", ()))
        mine = [e for e in range(rank * el, (rank + 1) * el) if e not in rep]
        my_rows = cfg.n_shared * T_local + int(glob[mine].sum()) + int(sum(own[e] for e in rep))
        # token rows (and the same number of output rows back) that crossed NVLink
        row_b = cfg.d * 2
        sent_bytes = row_b * int(sum(own[e] for e in range(cfg.n_routed) if e not in rep and e // el != rank))
        recv_bytes = row_b * int(sum(glob[e] - own[e] for e in mine))
    else:
        my_rows = (cfg.n_shared + cfg.k) * T_local
    per_rank = [[ms, e2e_ms, float(my_rows), float(sent_bytes), float(recv_bytes)] + [phases[n] for n in _lib.PHASES]]
    NP = 5  # per-rank values before the phases
    if world > 1:
        t = torch.tensor(per_rank[0], dtype=torch.float64, device=dev)
        allv = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(allv, t)
        per_rank = [v.tolist() for v in allv]
        ms = max(v[0] for v in per_rank)
        e2e_ms = max(v[1] for v in per_rank)
        phases = {n: max(v[NP + i] for v in per_rank) for i, n in enumerate(_lib.PHASES)}

    peaks = measured_peaks()
    # dominant kernel: the grouped gate/up GEMM (2/3 of the expert FLOPs and
    # weight bytes), on the rank where it took longest, with its own rows
    ig, idn = NP + _lib.PHASES.index("expert_gate_up"), NP + _lib.PHASES.index("expert_down")
    kname, col = max((("expert_gate_up", ig), ("expert_down", idn)), key=lambda kv: phases[kv[0]])
    slow = max(per_rank, key=lambda v: v[col])
    kms, rows = slow[col], slow[2]
    traffic_ent = profiled_traffic(kname, cfg.name, T_local)
    traffic = traffic_ent["bytes"] if traffic_ent else None
    simt = cfg.precision in (0, 1)  # Float64 / Float32 experts run on the SIMT kernels (no tensor path)
    if decode_shaped(cfg) or simt:
        # weight streaming (decode) or FFMA kernels: bytes of the touched
        # experts' layers (codes + block scales) plus the activation rows in
        # and out (bf16 on the decode path, float32 on the SIMT path), over the
        # kernel's time
        touched = int((moe.last_expert_load() > 0).sum()) + cfg.n_shared
        kbytes = kernel_bytes(cfg, kname, rows, touched, act_bytes=4 if simt else 2)
        achieved = kbytes / (kms * 1e-3) / 1e9 if kms > 0 else 0.0
        roofline = {"kernel": kname, "bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                    "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": traffic,
                    "peak_source": f"{peaks['source']} HBM copy bandwidth",
                    "algorithmic_bytes_per_launch": int(kbytes), "touched_experts": touched,
                    "avg_ms": round(kms, 4), "traffic_source": traffic_ent}
        if simt:
            roofline["note"] = ("Float32 experts: FFMA kernels; the layer's weights and rows fit in L2, so this "
                                "is a warm-L2 rate against the HBM copy peak")
    else:
        kflops = rows * (4.0 if kname == "expert_gate_up" else 2.0) * cfg.d * cfg.h
        achieved = kflops / (kms * 1e-3) / 1e12 if kms > 0 else 0.0
        roofline = {"kernel": kname, "bound": "tensor", "achieved": round(achieved, 2),
                    "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s",
                    "frac": round(achieved / peaks["bf16_tflops_sustained"], 4), "traffic": traffic,
                    "peak_source": f"{peaks['source']} bf16 sustained (kernel timed inside a long step loop)",
                    "algorithmic_flops_per_launch": kflops, "avg_ms": round(kms, 4),
                    "algorithmic_bytes_per_launch": int(kernel_bytes(cfg, kname, rows, cfg.n_shared + cfg.n_routed)),
                    "traffic_source": traffic_ent}

    if bwd_ms is not None:
        # float64 work of the backward per work row (the grouped GEMM stages):
        # the gate and up pre-activations recomputed (2 d h multiply-adds), the
        # routed row's output (d h), dH = dY Wd (d h), dX = dG Wg + dU Wu
        # (2 d h): 12 d h FLOPs per routed row, 10 d h per shared row; the
        # router term (2 T d E for the logits, T E d for its gradients) is added
        bflops = (12.0 * cfg.k + 10.0 * cfg.n_shared) * T_local * cfg.d * cfg.h + 4.0 * T_local * cfg.d * cfg.n_routed
        roofline = {"kernel": "backward (gtmoe_backward: bwd_gemm_kernel stages + router terms)", "bound": "fp64",
                    "achieved": round(bflops / (bwd_ms * 1e-3) / 1e12, 4), "unit": "TFLOP/s", "peak": None,
                    "frac": None, "traffic": None, "avg_ms": round(bwd_ms, 4),
                    "algorithmic_flops_per_launch": bflops,
                    "note": "float64 SIMT tiles (64 rows of one expert x 64 outputs), within summation rounding "
                            "of the reference's float64 arithmetic; no measured FP64 peak on this pool, so no "
                            "fraction is given",
                    "forward_roofline": roofline}

    cpu_baseline = None
    if want_cpu and grads is not None:
        # the oracle's numpy restatement of Forward + Backward on a seeded token sample
        spec = oracle_spec(cfg, host)
        x_cpu = x.to(torch.float64).cpu().numpy()
        g_cpu = grads["dout"].to(torch.float64).cpu().numpy()
        v, n, dt = time_oracle_backward(spec, x_cpu, g_cpu, args.cpu_seconds)
        cpu_baseline = {"value": round(v, 3), "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
                        "sample": f"{n} seeded tokens of {cfg.name} ({dt:.1f} s), float64 numpy restatement of "
                                  f"the reference's Forward + Backward (oracle.moe_backward; BLAS threads)"}
    elif want_cpu:
        spec = oracle_spec(cfg, host)
        x_cpu = x.to(torch.float64).cpu().numpy()
        threads = os.cpu_count() or 1
        v, n, dt = time_oracle(spec, x_cpu, args.cpu_seconds, threads)
        cpu_baseline = {"value": round(v, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
                        "sample": f"{n} seeded tokens of {cfg.name} ({dt:.1f} s), C float64 restatement of "
                                  f"the reference CPU path; row independence makes a token sample valid"
                                  + ("; the MoE forward only (without the block's RMSNorm and residual)"
                                     if args.op == "block" else "")}

    if rank == 0:
        value = T_total / (ms * 1e-3)
        line = {
            "metric": metric, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) bf16 activations, N(0,1/fan_in) weights quantised by the reference "
                    "quantiser, Zipf router bias)",
            "config": {**workload_config(cfg, world, mode, getattr(moe, "replicas", [])),
                       **({"op": "block step: x + Forward(RMSNorm(x)), gtmoe_forward_block"} if args.op == "block"
                          else {}),
                       **({"op": "training step of the mixture: Forward then Backward (gtmoe_backward, float64 "
                                 "input and router gradients, frozen compressed experts)"}
                          if args.op == "backward" else {})},
            "e2e": {"value": round(T_total / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": int(x_host.numel() * x_host.element_size()),
                    "d2h_bytes_per_step": int(out_host.numel() * out_host.element_size())},
            "roofline": roofline,
            "cpu_baseline": cpu_baseline,
            "phases_ms": {k: round(v, 4) for k, v in phases.items()},
            **({"ranks": [{"ms": round(v[0], 4), "expert_rows": int(v[2]), "push_bytes": int(v[3]),
                           "received_bytes": int(v[4]), "return_bytes": int(v[4]),
                           "phases_ms": {n: round(v[NP + i], 4) for i, n in enumerate(_lib.PHASES)}}
                          for v in per_rank]} if world > 1 else {}),
            "gpu_launches": int(launches.value),
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    moe.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def bench_replicas(args, cfg, world: int) -> list:
    """Hot experts held on every expert-parallel rank (--replicas)."""
    from gotransformers_b200 import synthetic

    if world < 2 or args.replicas == "0" or args.mode == "replicas":
        return []
    cap = 16 if args.replicas == "auto" else int(args.replicas)
    return synthetic.choose_replicas(cfg, world, max_replicas=cap)


def workload_config(cfg, world: int, mode: str, replicas=()) -> dict:
    """The `config` object of both arms' JSON lines."""
    prec = ["Float64", "Float32", "Int8", "FP4"][cfg.precision]
    return {"workload": f"{cfg.name}: {cfg.T} tokens x d {cfg.d}, {cfg.n_routed} routed + {cfg.n_shared} shared "
                        f"SwiGLU experts (hidden {cfg.h}), top-{cfg.k}, {prec} experts, "
                        f"{'bf16' if cfg.x_bf16 else 'float64'} activations",
            "tokens": cfg.T, "d_model": cfg.d, "hidden": cfg.h, "n_routed": cfg.n_routed,
            "n_shared": cfg.n_shared, "top_k": cfg.k, "precision": prec,
            "parallelism": (f"{mode}{world}" + (f" + {len(replicas)} hot-expert replicas" if replicas else "")
                            if world > 1 else "single"),
            **({"replicated_experts": list(replicas)} if replicas else {}),
            "l2": l2_note(cfg)}


def kernel_bytes(cfg, kernel: str, rows: int, touched: int, act_bytes: int = 2) -> float:
    """Algorithmic bytes of one expert-kernel launch: the touched experts'
    weights of that kernel (codes + one float32 scale per 16 values) plus its
    activation rows read and written."""
    bpv = {0: 8.0, 1: 4.0, 2: 1.0 + 4 / 16, 3: 0.5 + 4 / 16}[cfg.precision]
    n_layers, k_in, n_out = (2, cfg.d, cfg.h) if kernel == "expert_gate_up" else (1, cfg.h, cfg.d)
    return touched * n_layers * cfg.h * cfg.d * bpv + rows * (k_in + n_out) * act_bytes


def decode_shaped(cfg) -> bool:
    """A few tokens per expert: the forward streams expert weights (HBM-bound)."""
    return cfg.T <= 64


def l2_note(cfg) -> str:
    """Why no L2 flush is needed between steps: the step's inputs exceed L2."""
    l2 = 126 << 20
    xb = cfg.T * cfg.d * (2 if cfg.x_bf16 else 8)
    code = {0: 8.0, 1: 4.0, 2: 1.0 + 4 / 16, 3: 0.5 + 4 / 16}[cfg.precision]
    wb = (cfg.n_routed + cfg.n_shared) * 3 * cfg.d * cfg.h * code
    if decode_shaped(cfg):
        verdict = "512 MiB buffer written between steps (L2 flushed), each step timed by its own events"
    else:
        verdict = "no flush" if xb + wb > l2 else "weights and activations fit in L2: not flushed (warm-L2 figure)"
    return f"x {xb / 2**20:.0f} MiB, expert weights {wb / 1e9:.2f} GB, L2 126 MiB: {verdict}"


def profiled_traffic(kernel: str, config: str, T_local: int):
    """DRAM bytes per launch of `kernel` from the committed ncu summary
    (profiles/traffic.json) when it was captured on this run's token count;
    None otherwise (no capture, or an expert-parallel rank, whose launches
    hold other rows than a single-GPU run's)."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        j = json.load(f)
    ent = j.get(f"{kernel}:{config}")
    if not ent:
        return None
    if int(ent["tokens"]) != int(T_local):
        return None
    return {"bytes": int(ent["bytes_per_launch"]), "source": ent["source"],
            **({"scaled_from": ent["scaled_from"]} if "scaled_from" in ent else {})}


def host_spec_and_sample(cfg, n_tokens: int, threads: int, seed: int = 7):
    """The config's router and expert weights made on the host by the
    oracle's restatement of the seeded generator and the reference quantiser
    (no GPU library), and the activations of a seeded sample of n_tokens
    tokens.  Returns (spec, x_sample float64, token indices)."""
    from gotransformers_b200 import synthetic
    from oracle import oracle as O

    E, S, d, h = cfg.n_routed, cfg.n_shared, cfg.d, cfg.h
    rb = synthetic.zipf_router_bias(E, cfg.k, cfg.zipf_s, cfg.weight_seed) if cfg.zipf_s else np.zeros(E)
    wr = O.synth_rows(O.FLOAT64, E, d, cfg.weight_seed, synthetic.STREAM_ROUTER, 1.0 / np.sqrt(d), threads)
    router = O.Layer(O.FLOAT64, E, d, wr.values, None, np.ascontiguousarray(rb, np.float64))
    experts = []
    for e in range(S + E):
        experts.append(tuple(
            O.synth_rows(cfg.precision, rows, width, cfg.weight_seed, synthetic.expert_stream(e, which),
                         1.0 / np.sqrt(width), threads)
            for which, (rows, width) in enumerate([(h, d), (h, d), (d, h)])))
    spec = O.MoESpec(d=d, h=h, n_shared=S, n_routed=E, k=cfg.k, router=router, experts=experts)
    rng = np.random.default_rng(seed)
    tokens = np.sort(rng.choice(cfg.T, size=min(n_tokens, cfg.T), replace=False))
    x = np.stack([synthetic.normal(cfg.act_seed, synthetic.STREAM_X, d, offset=int(t) * d) for t in tokens])
    if cfg.x_bf16:
        x = synthetic.bf16_round(x)
    return spec, np.ascontiguousarray(x), tokens


def run_reference(args, cfg, rank, world, local_rank, metric):
    """The reference's CPU algorithm (the C float64 oracle port; the Go
    reference has no toolchain here) on all host cores, rank 0 only, on the
    same config as the GPU arm.  Its inputs are made on the host by the
    oracle (seeded generator + reference quantiser); neither the GPU library
    nor the GPU is used.  Each step runs a bounded seeded token sample (row
    independence, mixtureofexperts_test.go:83-100, makes a sample valid)."""
    if rank != 0:
        return
    from oracle import oracle as O

    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    spec, x_all, tokens = host_spec_and_sample(cfg, min(cfg.T, 4096), threads)
    prep_s = time.perf_counter() - t0
    # size each step for ~ (two minutes / steps)
    t0 = time.perf_counter()
    O.moe_forward(spec, x_all[:2], tokens[:2].astype(np.int64), threads=threads)
    per_tok = max((time.perf_counter() - t0) / 2, 1e-6)
    budget = 120.0 / max(args.steps + args.warmup, 1)
    n = int(min(len(tokens), max(2, budget / per_tok)))
    xs, ids = x_all[:n], tokens[:n].astype(np.int64)
    for _ in range(args.warmup):
        O.moe_forward(spec, xs, ids, threads=threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        O.moe_forward(spec, xs, ids, threads=threads)
        times.append(time.perf_counter() - t0)
    ms = 1e3 * sum(times) / len(times)
    value = n / (ms * 1e-3)
    mode = args.mode if args.mode != "auto" else ("ep" if world > 1 else "replicas")
    config = workload_config(cfg, world, mode, bench_replicas(args, cfg, world) if mode == "ep" else [])
    config["sample_tokens"] = n
    line = {
        "impl": "reference", "metric": metric, "value": round(value, 3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (the GPU arm's seeded generator and reference quantiser, run on the host by the oracle)",
        "config": config,
        "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{n} seeded tokens of {cfg.name} per step; C float64 restatement of the "
                                   f"reference CPU path (no Go toolchain on this image); inputs made on the host "
                                   f"in {prep_s:.0f} s (not timed)"},
        "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
