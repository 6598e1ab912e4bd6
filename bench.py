#!/usr/bin/env python
"""Benchmark of the DeepSeek-V3/R1 MoE block on B200 (libmoe_cuda.so).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

One JSON line on rank 0.  A "step" is one decode step of one MoE layer over
one batch of synthetic tokens.  Workloads (the reference's headline configs):
  decode_b64_zipf  (default) config 3: 64 tokens, router skewed by a Zipf(1.1)
                   per-expert bias, 256 experts sharded over N GPUs
  decode_b1        config 2: one token on one GPU
Weights are random-init N(0, 0.02) quantized to Q4_K gate/up and Q6_K down on
the device; inputs N(0, 1) from a fixed seed.  Between timed steps a 256 MiB
buffer is written to flush the 126 MB L2.  On one GPU the default run then
measures the other configs too (one expert per call, one token, the 4096-token
prefill, the 58-layer stack at batch 1, the dense FFN layers 0-2 and the output
head with the top-p sampler at one token) and reports them under "configs";
--no-extra skips them.

--impl reference times the reference's own CPU path (quant.c dequant + fp32
dots + route(), built in place under oracle/_ref) on this host's cores, on a
bounded sample of tokens of the same workload.
"""
from __future__ import annotations

import argparse
import glob
import json
import os
import re
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from flash_deepseek_b200.workloads import token_pool, zipf_logit_bias  # noqa: E402

METRIC = "MoE decode tokens/s at 1/2/4/8 B200; expert matvec HBM GB/s vs 8 TB/s peak"
H, I, E, K = 7168, 2048, 256, 8
Q4_ROW = H // 256 * 144
GATE_BYTES = I * Q4_ROW                      # 8,257,536
DOWN_Q6_BYTES = H * (I // 256) * 210         # 12,042,240
EXPERT_BYTES = 2 * GATE_BYTES + DOWN_Q6_BYTES
ROUTER_BYTES = E * H * 4 + E * 4
WORKLOADS = {
    "decode_b64_zipf": dict(B=64, zipf=True, name="config3_decode_b64_zipf"),
    "decode_b1": dict(B=1, zipf=False, name="config2_decode_b1"),
}
# the other headline configs (one expert, the 58-layer stack, prefill), measured by run_extra()
EXTRA = {
    "expert1": dict(B=1, name="config1_single_q4k_expert"),
    "stack_b1": dict(B=1, name="config4_stack58_b1"),
    "stack_b8": dict(B=8, name="config4_stack58_b8"),
    "stack_b32": dict(B=32, name="config4_stack58_b32"),
    "prefill4096": dict(B=4096, name="config5_prefill4096_1layer"),
    "dense_b1": dict(B=1, name="dense_ffn_layers0to2_b1"),
    "head_b1": dict(B=1, name="lm_head_sample_b1"),
}
VOCAB = 129280              # VOCAB_SIZE of DeepSeek-V3
DENSE_I = 18432             # DENSE_INTERMEDIATE (infer.m:59)
DENSE_LAYERS = 3            # FIRST_MOE_LAYER (infer.m:46)
Q4_DOWN_BYTES = H * (I // 256) * 144         # 8,257,536


TC_MIN_TOKENS = 9           # an expert with this many tokens or more runs on the tcgen05 kernels (MOE_TC + 1)
NVLINK_GBS = 900.0          # NVLink 5, per direction per GPU (nominal)
NVLINK_MEASURED_GBS = 770.0  # peer copy per direction measured on this pool's B200 boxes
N_POOL = 4


def workload_config(W, NE, world, b_loc):
    """The `config` object of both arms' JSON lines."""
    return {"workload": W["name"], "global_batch": W["B"], "tokens_per_gpu": b_loc, "hidden": H,
            "intermediate": I, "experts": NE, "top_k": K, "gate_up": "Q4_K", "down": "Q6_K",
            "router_skew": "zipf(1.1) logit bias" if W["zipf"] else "none",
            "parallelism": f"ep{world}", "l2": "flushed: 256 MiB write between timed steps",
            "tokens": f"numpy default_rng(1234) N(0,1), {N_POOL} batches in turn"}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def traffic_from_profiles(kernel: str, workload: str, alg_bytes: float):
    """Per-launch DRAM bytes from a committed ncu summary, if there is one.
    The captures run a smaller case of the same kernel (fewer experts); their
    traffic is scaled to this launch by the algorithmic bytes of both."""
    for p in sorted(glob.glob(os.path.join(ROOT, "profiles", f"{kernel}__{workload}*.txt"))):
        txt = open(p).read()
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", txt)
        a = re.search(r"algorithmic_bytes_per_launch:\s*([0-9.eE+]+)", txt)
        if m and a:
            return float(m.group(1)) * alg_bytes / float(a.group(1))
    return None


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed
    region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.proc, self.lines = gpu, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------- CPU path
def cpu_reference(workload: str, steps: int, warmup: int, seconds: float = 20.0):
    """The reference's CPU expert path (oracle/_ref: quant.c + route() of the
    reference, plain-C dots in place of Accelerate) on sampled tokens."""
    import ctypes as C
    from oracle import oracle as O
    W = WORKLOADS[workload]
    threads = len(os.sched_getaffinity(0))
    if not O.ref_available():
        O.build()
    R = O.ref()
    router = O.normal(0, O.stream(0, 0, O.KIND_ROUTER), E * H, 0.006, threads=threads).reshape(E, H)
    bias = O.normal(0, O.stream(0, 0, O.KIND_BIAS), E, 0.01, threads=threads)
    lbias = zipf_logit_bias() if W["zipf"] else np.zeros(E, np.float32)
    # the GPU arm's token batches, one token at a time in the same order
    n_tok = max(1, steps + warmup)
    pool = token_pool(W["B"], N_POOL)
    xs = np.stack([pool[(i // W["B"]) % N_POOL][i % W["B"]] for i in range(n_tok)])
    need = set()
    for t in range(n_tok):
        lg = (router.astype(np.float64) @ xs[t].astype(np.float64) + lbias).astype(np.float32)
        idx, _ = O.ref_route(lg, bias, K=8)
        need |= set(idx.tolist())
    blobs = {e: O.gen_expert(0, 0, e, H, I, O.TYPE_Q6_K, threads=threads) for e in sorted(need)}
    blobs[E] = O.gen_expert(0, 0, E, H, I, O.TYPE_Q6_K, threads=threads)
    dummy = np.zeros(EXPERT_BYTES, np.uint8)
    table = (C.c_void_p * (E + 1))()
    for e in range(E + 1):
        table[e] = (blobs.get(e, dummy)).ctypes.data
    out = np.empty(H, np.float32)
    times = []
    for t in range(n_tok):
        t0 = time.perf_counter()
        rc = R.ref_moe_token_cpu(table, 1, router, lbias, bias, xs[t], 8, out, None, None, threads)
        dt = time.perf_counter() - t0
        if rc != 0:
            raise RuntimeError(f"ref_moe_token_cpu failed ({rc})")
        if t >= warmup:
            times.append(dt)
        if sum(times) > seconds and len(times) >= 2:
            break
    tok_s = len(times) / sum(times)
    return dict(value=tok_s, unit="tokens/s", cores=threads, kind="reference",
                sample=f"{len(times)} tokens of {W['name']}, one at a time as infer.m decodes "
                       f"(quant.c dequant of 8 routed + 1 shared expert, fp32 dots, route())")


# ----------------------------------------------------------------- GPU path
def run_ours(args):
    import torch
    import flash_deepseek_b200 as F
    from flash_deepseek_b200 import ep

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
        pg = dist
    W = dict(WORKLOADS[args.workload])
    if args.batch:
        W["B"] = args.batch
    B = W["B"]
    # tokens of this rank: an even share, or (batch < GPUs) one token on the
    # first B ranks and none elsewhere
    t0_loc, b_loc = ep.local_tokens(B, world, rank)
    uid = ep.share_unique_id(pg, rank, F.get_unique_id) if world > 1 else None
    cfg = F.MoeConfig(n_layers=1, max_tokens=max(1, b_loc), n_experts=args.experts)
    moe = F.MoE(cfg, device=local, rank=rank, world_size=world, unique_id=uid)
    moe.init_layer_synthetic(0, seed=0, down_type=F.TYPE_Q6_K)
    if W["zipf"]:
        moe.set_logit_bias(0, zipf_logit_bias(n=args.experts))

    dev = torch.device("cuda", local)
    stream = torch.cuda.ExternalStream(moe.stream, device=dev)
    n_pool = N_POOL
    pool_h = [torch.from_numpy(x) for x in token_pool(B, n_pool)]
    pool = [p[t0_loc:t0_loc + b_loc].contiguous().to(dev) for p in pool_h]
    out = torch.empty(max(1, b_loc), H, device=dev)
    steps_total = args.warmup + args.steps
    idx_all = torch.empty(steps_total, max(1, b_loc), K, dtype=torch.int32, device=dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    def barrier():
        torch.cuda.synchronize()
        if pg:
            pg.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if not pg:
            return v
        t = torch.tensor([v], dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t[0])

    clk = Clocks(local).__enter__()
    t_wait = time.time()
    while not clk.lines and time.time() - t_wait < 5.0:
        time.sleep(0.05)
    # ---- device-resident leg (value).  The library replays each call
    # signature as a CUDA graph from its second call on; two untimed passes
    # over the input pool capture them before the warm-up proper.
    for s in range(2 * n_pool):
        moe.forward_device(0, pool[s % n_pool], b_loc, out)
    for s in range(args.warmup):
        with torch.cuda.stream(stream):
            flush.zero_()
        moe.forward_device(0, pool[s % n_pool], b_loc, out, d_idx=idx_all[s])
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    phases = []
    barrier()
    launches0 = moe.kernel_launches
    n_clk0 = len(clk.lines)
    for s in range(args.steps):
        with torch.cuda.stream(stream):
            flush.zero_()
        ev[s][0].record(stream)
        moe.forward_device(0, pool[(args.warmup + s) % n_pool], b_loc, out, d_idx=idx_all[args.warmup + s])
        ev[s][1].record(stream)
    barrier()
    moe.check_error()  # a bounded device wait that gave up would surface here
    clk_lines_timed = clk.lines[n_clk0:]
    launches = moe.kernel_launches - launches0
    step_ms = [a.elapsed_time(b) for a, b in ev]
    total_ms = max_over_ranks(sum(step_ms))
    value = B * args.steps / (total_ms / 1e3)

    # ---- per-kernel durations: a separate pass with CUDA events between the
    # kernels (direct launches, no graph), same inputs and L2 flush
    n_ph = min(args.steps, 50)
    moe.set_timing(n_ph)
    for s in range(n_ph):
        with torch.cuda.stream(stream):
            flush.zero_()
        moe.forward_device(0, pool[(args.warmup + s) % n_pool], b_loc, out)
    barrier()
    phases = [moe.timing(back) for back in range(n_ph)]
    moe.set_timing(0)

    # ---- roofline of the dominant kernel (gate/up GEMV) on this rank: the
    # experts it holds that any token of the global batch routes to
    idx_loc = idx_all[args.warmup:, :b_loc].cpu()
    if pg:
        sizes = [None] * world
        pg.all_gather_object(sizes, idx_loc.numpy())
        idx_g = np.concatenate([x for x in sizes if x.size], axis=1)
    else:
        idx_g = idx_loc.numpy()
    NE = args.experts
    # algorithmic bytes per launch, split between the GEMVs and the tcgen05
    # kernels: an expert with more than TC_MIN_TOKENS - 1 tokens on this rank
    # runs on tcgen05 (the shared expert with this rank's b_loc tokens too)
    gu_bytes, dn_bytes, gu_tc, dn_tc, active = [], [], [], [], []
    for s in range(args.steps):
        mine = ep.expert_owner(idx_g[s], NE, world) == rank
        n_act = len(ep.experts_hit(idx_g[s], NE, world, rank)) + 1
        cnt = np.bincount(idx_g[s][mine].reshape(-1), minlength=NE)
        ntok = [int(c) for c in cnt if c > 0] + [b_loc]
        active.append(n_act)
        g = [0, 0]   # gate/up bytes: GEMV, tcgen05
        dd = [0, 0]
        for n in ntok:
            tc = 1 if n >= TC_MIN_TOKENS else 0
            g[tc] += 2 * GATE_BYTES + n * H * 4 + n * I * 4
            dd[tc] += DOWN_Q6_BYTES + n * (I * 4 + H * 4)
        gu_bytes.append(g[0])
        gu_tc.append(g[1])
        dn_bytes.append(dd[0])
        dn_tc.append(dd[1])
    # expert-parallel exchange and the per-GPU critical path, from the
    # global routing of every timed step (all ranks compute the same figures)
    nv = None
    crit = None
    if world > 1:
        row_b = H * 4 + (2 + 2 * K) * 4        # a dispatched token row: fp32 activations + routing metadata
        part_b = H * 4                          # a returned partial sum (fp32)
        starts = [ep.local_tokens(B, world, r)[0] for r in range(world)]
        counts_r = [ep.local_tokens(B, world, r)[1] for r in range(world)]
        send = np.zeros((args.steps, world))
        recv = np.zeros((args.steps, world))
        hbm = np.zeros((args.steps, world))
        for s_ in range(args.steps):
            own = ep.expert_owner(idx_g[s_], NE, world)  # [B, K] owning rank of every routed expert
            for r in range(world):
                n_exp = len(ep.experts_hit(idx_g[s_], NE, world, r))
                hbm[s_, r] = n_exp * EXPERT_BYTES + ((NE * H * 4 + NE * 4 + EXPERT_BYTES) if counts_r[r] else 0)
            for tkn in range(B):
                src = next(r for r in range(world) if starts[r] <= tkn < starts[r] + counts_r[r])
                for dst in set(own[tkn].tolist()) - {src}:
                    send[s_, src] += row_b      # dispatch: token row to the expert owner
                    recv[s_, dst] += row_b
                    send[s_, dst] += part_b     # combine: partial sum back to the token's rank
                    recv[s_, src] += part_b
        ex_ms = float(np.mean([p["dispatch"] + p["combine_a2a"] for p in phases]))
        ex_ms = max_over_ranks(ex_ms)
        crit_link = float(np.maximum(send, recv).max(1).mean())   # busiest direction of the busiest rank
        nv = {"bytes_per_step_busiest_rank": round(crit_link), "dispatch_plus_combine_ms": round(ex_ms, 5),
              "achieved_gbs": round(crit_link / (ex_ms / 1e3) / 1e9, 2) if ex_ms > 0 else None,
              "frac_of_900": round(crit_link / (ex_ms / 1e3) / 1e9 / NVLINK_GBS, 5) if ex_ms > 0 else None,
              "frac_of_measured_770": round(crit_link / (ex_ms / 1e3) / 1e9 / NVLINK_MEASURED_GBS, 5)
              if ex_ms > 0 else None,
              "send_bytes_per_rank": [round(x) for x in send.mean(0)],
              "recv_bytes_per_rank": [round(x) for x in recv.mean(0)],
              "note": "exchange phases include waiting for the busiest rank's experts"}
        crit_b = float(hbm.max(1).mean())
        crit = {"bytes_per_step_busiest_rank": round(crit_b),
                "achieved_gbs": round(crit_b / (total_ms / args.steps / 1e3) / 1e9, 1),
                "frac": round(crit_b / (total_ms / args.steps / 1e3) / 1e9 / peaks()[0], 4),
                "aggregate_frac": round(float(hbm.sum(1).mean()) / (total_ms / args.steps / 1e3) / 1e9 /
                                        (peaks()[0] * world), 4)}
    gu_ms = float(np.mean([p["gateup"] for p in phases]))
    dn_ms = float(np.mean([p["down"] for p in phases]))
    gut_ms = float(np.mean([p["gateup_tc"] for p in phases]))
    dnt_ms = float(np.mean([p["down_tc"] for p in phases]))
    peak, peak_kind = peaks()
    ach = float(np.mean(gu_bytes)) / (gu_ms / 1e3) / 1e9
    ach_dn = float(np.mean(dn_bytes)) / (dn_ms / 1e3) / 1e9

    def tc_roof(nbytes, ms, kernel):
        if ms <= 0 or nbytes <= 0:
            return None
        a = nbytes / (ms / 1e3) / 1e9
        return {"kernel": kernel, "achieved": round(a, 1), "frac": round(a / peak, 4),
                "algorithmic_bytes_per_launch": round(nbytes), "launch_ms": round(ms, 5)}
    step_bytes = float(np.mean([a * EXPERT_BYTES for a in active])) + NE * H * 4 + NE * 4
    traffic = traffic_from_profiles("k_gateup", args.workload, float(np.mean(gu_bytes)))
    traffic_dn = traffic_from_profiles("k_down", args.workload, float(np.mean(dn_bytes)))

    # ---- end-to-end leg through the C ABI with host buffers
    h_pin = [p[t0_loc:t0_loc + max(1, b_loc)].contiguous().pin_memory() for p in pool_h]
    o_pin = torch.empty(max(1, b_loc), H, dtype=torch.float32).pin_memory()
    h_np = [p.numpy() for p in h_pin]
    ev2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    idx_np = np.empty((max(1, b_loc), K), np.int32)
    w_np = np.empty((max(1, b_loc), K), np.float32)
    lib = moe.lib
    o_np = o_pin.numpy()
    for s in range(args.warmup):
        lib.moe_forward(moe.ctx, 0, h_np[s % n_pool].ctypes.data, b_loc, o_np.ctypes.data, idx_np.ctypes.data,
                        w_np.ctypes.data)
    barrier()
    for s in range(args.steps):
        with torch.cuda.stream(stream):
            flush.zero_()
        ev2[s][0].record(stream)
        rc = lib.moe_forward(moe.ctx, 0, h_np[(args.warmup + s) % n_pool].ctypes.data, b_loc, o_np.ctypes.data,
                             idx_np.ctypes.data, w_np.ctypes.data)
        ev2[s][1].record(stream)
        if rc != 0:
            raise RuntimeError(moe.lib.moe_last_error(moe.ctx))
    barrier()
    moe.check_error()
    e2e_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in ev2))
    clk.__exit__(None, None, None)
    if len(clk_lines_timed) < 3:   # timed region shorter than the sampling period
        clk_lines_timed = clk.lines
    clk.lines = clk_lines_timed
    e2e = B * args.steps / (e2e_ms / 1e3)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_reference(args.workload, steps=20, warmup=1, seconds=15.0)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "exact tensor-core products of the Q4_K/Q6_K integers (sub-block scales folded in) with "
                     "fp16 hi/lo (22-bit) or int8-plane (21-bit) activations, fp32 accumulation (tcgen05 for "
                     "experts with 9+ tokens, mma.sync GEMVs for the rest)",
            "data": "synthetic: random-init N(0,0.02) weights quantized on device, N(0,1) tokens",
            "config": workload_config(W, NE, world, b_loc),
            "roofline": {"bound": "hbm", "kernel": "k_gateup (grouped Q4_K gate/up GEMV + SwiGLU; experts with at "
                                                   "most 8 tokens, the largest kernel of the step)",
                         "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(ach / peak, 4), "peak_source": peak_kind,
                         "frac_of_8TBs": round(ach / 8000.0, 4),
                         "traffic": traffic,
                         "algorithmic_bytes_per_launch": round(float(np.mean(gu_bytes))),
                         "launch_ms": round(gu_ms, 5)},
            "roofline_down": {"kernel": "k_down (grouped Q6_K down GEMV)", "achieved": round(ach_dn, 1),
                              "frac": round(ach_dn / peak, 4), "traffic": traffic_dn,
                              "algorithmic_bytes_per_launch": round(float(np.mean(dn_bytes))),
                              "launch_ms": round(dn_ms, 5)},
            "roofline_tc": {"gateup": tc_roof(float(np.mean(gu_tc)), gut_ms,
                                              "k_tc_gather + k_experts_tc<0> (busy experts' gate/up on tcgen05)"),
                            "down": tc_roof(float(np.mean(dn_tc)), dnt_ms,
                                            "k_experts_tc<2> (busy experts' Q6_K down on tcgen05)")},
            "roofline_phases": {
                "gateup": round(float(np.mean(gu_bytes) + np.mean(gu_tc)) / ((gu_ms + gut_ms) / 1e3) / 1e9 / peak, 4),
                "down": round(float(np.mean(dn_bytes) + np.mean(dn_tc)) / ((dn_ms + dnt_ms) / 1e3) / 1e9 / peak, 4),
                "note": "all weight and activation bytes of the phase over the phase's time, fraction of measured HBM"},
            "step_hbm": {"weight_bytes_per_step": round(step_bytes),
                         "achieved_gbs": round(step_bytes / (total_ms / args.steps / 1e3) / 1e9, 1),
                         "active_experts_per_step": round(float(np.mean(active)), 2)},
            "phase_ms": {k: round(float(np.mean([p[k] for p in phases])), 5) for k in phases[0]},
            "nvlink": nv,
            "step_hbm_critical_path": crit,
            "e2e": {"value": round(e2e, 2), "unit": "tokens/s", "h2d_bytes_per_step": B * H * 4,
                    "d2h_bytes_per_step": B * H * 4 + B * K * 8},
            "gpu_launches": int(launches),
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
        }
    moe.close()
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    return line if rank == 0 else None


def run_extra(args):
    """Configs 1, 4 and 5 on one GPU (informational lines; the default bench
    line is config 3).
      expert1      one Q4_K expert (gate/up/down Q4_K) per call, routing given
                   (moe_experts_forward_device, K = 1), 256 distinct experts in
                   turn so that no call finds its weights in L2
      stack_b*     the 58-layer stack (RMSNorm + MoE + residual per layer,
                   down Q6_K / Q4_K alternating) through moe_forward_stack_device:
                   20 layers are resident (about 137 GB) and a step runs them
                   20 + 20 + 18 times; every layer's weights exceed L2, so the
                   re-use changes nothing but the memory needed
      prefill4096  4096 tokens through one layer per moe_prefill_device call
                   (tcgen05 GEMMs over fp16-dequantized weight tiles)
      dense_b1     one token through the three dense FFN layers (0-2) per
                   step, moe_dense_forward_device per layer
      head_b1      one token through lm_head (129280 x 7168 fp16) and the
                   top-p sampler (temp 0.6, top_p 0.95)"""
    import torch
    import flash_deepseek_b200 as F
    W = EXTRA[args.workload]
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if int(os.environ.get("WORLD_SIZE", "1")) > 1 and not (args.workload == "prefill4096" or
                                                             args.workload.startswith("stack")):
        raise SystemExit(f"--workload {args.workload} runs on one GPU")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(local)
    g = torch.Generator(device="cpu").manual_seed(1234)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    peak, peak_kind = peaks()
    clk = Clocks(local).__enter__()
    extra = {}
    if args.workload == "expert1":
        cfg = F.MoeConfig(n_layers=1, max_tokens=1, top_k=1)
        moe = F.MoE(cfg)
        moe.init_layer_synthetic(0, seed=0, down_type=F.TYPE_Q4_K)
        x = torch.randn(1, H, generator=g).to(dev)
        out = torch.empty_like(x)
        idx = torch.arange(E, dtype=torch.int32, device=dev).reshape(E, 1)
        w1 = torch.ones(E, 1, dtype=torch.float32, device=dev)
        stream = torch.cuda.ExternalStream(moe.stream, device=dev)
        for e in range(args.warmup):
            moe.experts_forward_device(0, x, 1, idx[e % E], w1[e % E], 1, out)
        n = args.steps
        torch.cuda.synchronize()
        l0 = moe.kernel_launches
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for e in range(n):
            moe.experts_forward_device(0, x, 1, idx[e % E], w1[e % E], 1, out)
        b.record(stream)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b)
        launches = moe.kernel_launches - l0
        per_call = ms / n
        bytes_call = 3 * GATE_BYTES + H * 4 + I * 4 * 2 + H * 4
        value = n / (ms / 1e3)
        roof = {"bound": "hbm", "kernel": "whole call (route given, gate/up, prep, down, combine)",
                "achieved": round(bytes_call / (per_call / 1e3) / 1e9, 1), "peak": peak, "unit": "GB/s",
                "frac": round(bytes_call / (per_call / 1e3) / 1e9 / peak, 4), "peak_source": peak_kind,
                "algorithmic_bytes_per_launch": bytes_call, "traffic": None}
        unit, ms_step = "expert calls/s", per_call
        e2e = None
    elif args.workload.startswith("stack"):
        # one GPU holds 20 of the 58 layers (137 GB) and runs them in the order
        # 0-19, 0-19, 0-17; with expert parallelism every rank holds its
        # n_experts / world experts of every layer (all 58 at 8 GPUs, ~51 GB)
        from flash_deepseek_b200 import ep
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        pg = None
        if world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
            pg = dist
        B = W["B"]
        layer_gb = (E / world * 26.6 + 28.6 + 7.4) / 1e3  # experts of this rank + shared + router, GB
        n_res = min(58, max(1, int(140 / layer_gb)))
        seq, left = [], 58
        while left > 0:
            seq.append((0, min(n_res, left)))
            left -= seq[-1][1]
        t0, bl = ep.local_tokens(B, world, rank)
        uid = ep.share_unique_id(pg, rank, F.get_unique_id) if world > 1 else None
        cfg = F.MoeConfig(n_layers=n_res, max_tokens=max(1, -(-B // world)))  # the same capacity on every rank
        moe = F.MoE(cfg, device=local, rank=rank, world_size=world, unique_id=uid)
        for l in range(n_res):
            moe.init_layer_synthetic(l, seed=0, down_type=F.TYPE_Q6_K if l % 2 == 0 else F.TYPE_Q4_K)
        hs = [torch.randn(B, H, generator=g)[t0:t0 + bl].contiguous().to(dev) for _ in range(4)]
        hid = torch.empty(max(1, bl), H, device=dev)
        stream = torch.cuda.ExternalStream(moe.stream, device=dev)

        def sync_all():
            torch.cuda.synchronize()
            if pg:
                pg.barrier()
            torch.cuda.synchronize()

        def step(i):
            if bl:
                hid[:bl].copy_(hs[i % 4])
            for f0, nl in seq:
                moe.forward_stack_device(f0, nl, hid, bl, stream=moe.stream)
        with torch.cuda.stream(stream):
            for i in range(args.warmup):
                step(i)
        sync_all()
        # one untimed step that records the routed experts every rank read in
        # each of the 58 layer calls: the weight bytes of each call per rank
        hits = torch.zeros(n_res, dtype=torch.int32, device=dev)
        moe.record_expert_hits(hits)
        call_bytes = []
        if bl:
            hid[:bl].copy_(hs[0])
        with torch.cuda.stream(stream):
            for f0, nl in seq:
                moe.forward_stack_device(f0, nl, hid, bl, stream=moe.stream)
                torch.cuda.synchronize()
                hv = hits.cpu().tolist()
                for l in range(f0, f0 + nl):
                    eb = 2 * GATE_BYTES + (DOWN_Q6_BYTES if l % 2 == 0 else Q4_DOWN_BYTES)  # shared: same down type
                    call_bytes.append(hv[l] * eb + ((ROUTER_BYTES + eb) if bl else 0))
        moe.record_expert_hits(None)
        call_bytes = torch.tensor(call_bytes, dtype=torch.float64)
        if pg:
            allb = [torch.zeros_like(call_bytes) for _ in range(world)]
            pg.all_gather(allb, call_bytes)
            allb = torch.stack(allb)
        else:
            allb = call_bytes[None]
        crit_b = float(allb.max(0).values.sum())   # per-GPU critical path: the busiest rank of every layer
        agg_b = float(allb.sum())
        sync_all()
        l0 = moe.kernel_launches
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        with torch.cuda.stream(stream):
            for i in range(args.steps):
                ev[i][0].record(stream)
                step(i)
                ev[i][1].record(stream)
        sync_all()
        ms = sum(x.elapsed_time(y) for x, y in ev)
        if pg:
            t = torch.tensor([ms], dtype=torch.float64)
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            ms = float(t[0])
        launches = moe.kernel_launches - l0
        ms_step = ms / args.steps
        value = B * args.steps / (ms / 1e3)
        unit = "tokens/s"
        # per-GPU critical path: in every layer call the rank that reads the most
        # weight bytes (routed experts it was sent tokens for, plus router and
        # shared expert where it holds tokens), summed over the 58 calls
        sec = ms_step / 1e3
        roof = {"bound": "hbm", "kernel": "whole 58-layer step, per-GPU critical path (busiest rank per layer)",
                "achieved": round(crit_b / sec / 1e9, 1), "peak": peak, "unit": "GB/s",
                "frac": round(crit_b / sec / 1e9 / peak, 4), "peak_source": peak_kind,
                "algorithmic_bytes_per_step": crit_b, "traffic": None,
                "aggregate": {"bytes_per_step": agg_b, "achieved": round(agg_b / sec / 1e9, 1),
                              "peak": peak * world, "frac": round(agg_b / sec / 1e9 / (peak * world), 4)}}
        e2e = None
        if world == 1:
            h_pin = hs[0].cpu().pin_memory().numpy()
            lib = moe.lib
            buf = h_pin.copy()
            lib.moe_forward_stack(moe.ctx, 0, n_res, buf.ctypes.data, B)
            torch.cuda.synchronize()
            t_0 = time.perf_counter()
            n_e2e = max(2, args.steps // 4)
            for i in range(n_e2e):
                buf[:] = h_pin
                for f0, nl in seq:
                    rc = lib.moe_forward_stack(moe.ctx, f0, nl, buf.ctypes.data, B)
                    if rc != 0:
                        raise RuntimeError(lib.moe_last_error(moe.ctx))
            e2e_s = time.perf_counter() - t_0
            e2e = {"value": round(B * n_e2e / e2e_s, 2), "unit": "tokens/s", "h2d_bytes_per_step": 3 * B * H * 4,
                   "d2h_bytes_per_step": 3 * B * H * 4, "timer": "host wall clock (synchronous calls)"}
        extra = {"layers_resident": n_res, "layer_calls_per_step": 58, "tokens_per_rank": bl,
                 "parallelism": f"ep{world}"}
        if rank != 0:
            clk.__exit__(None, None, None)
            moe.close()
            return None
    elif args.workload == "dense_b1":
        # the three dense FFN layers of one decode token (infer.m:1852-1868):
        # fp16 weights, 792.7 MB per layer, 2.38 GB per step (> L2: no flush)
        cfg = F.MoeConfig(n_layers=DENSE_LAYERS, max_tokens=1)
        moe = F.MoE(cfg, device=local)
        for l in range(DENSE_LAYERS):
            moe.init_dense_synthetic(l, DENSE_I, seed=0, w_sigma=0.02)
        xs = [torch.randn(1, H, generator=g).to(dev) for _ in range(N_POOL)]
        out = torch.empty(1, H, device=dev)
        stream = torch.cuda.ExternalStream(moe.stream, device=dev)

        def step(i):
            for l in range(DENSE_LAYERS):
                moe.dense_forward_device(l, xs[i % N_POOL], 1, out, stream=moe.stream)
        with torch.cuda.stream(stream):
            for i in range(args.warmup):
                step(i)
        torch.cuda.synchronize()
        n = args.steps
        l0 = moe.kernel_launches
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            a.record(stream)
            for i in range(n):
                step(i)
            b.record(stream)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b)
        launches = moe.kernel_launches - l0
        ms_step = ms / n
        value = n / (ms / 1e3)
        unit = "tokens/s"
        bytes_step = DENSE_LAYERS * 3 * DENSE_I * H * 2 + DENSE_LAYERS * (2 * H * 4 + 2 * DENSE_I * 4)
        roof = {"bound": "hbm", "kernel": "whole step (3 layers x k_dense_gateup + k_dense_down)",
                "achieved": round(bytes_step / (ms_step / 1e3) / 1e9, 1), "peak": peak, "unit": "GB/s",
                "frac": round(bytes_step / (ms_step / 1e3) / 1e9 / peak, 4), "peak_source": peak_kind,
                "algorithmic_bytes_per_step": bytes_step, "traffic": None}
        # end to end: moe_dense_forward per layer from pinned host memory
        h_pin = xs[0].cpu().pin_memory().numpy()
        o_pin = torch.empty(1, H).pin_memory().numpy()
        lib = moe.lib
        for l in range(DENSE_LAYERS):
            lib.moe_dense_forward(moe.ctx, l, h_pin.ctypes.data, 1, o_pin.ctypes.data)
        n_e2e = max(2, n // 4)
        t_0 = time.perf_counter()
        for i in range(n_e2e):
            for l in range(DENSE_LAYERS):
                if lib.moe_dense_forward(moe.ctx, l, h_pin.ctypes.data, 1, o_pin.ctypes.data) != 0:
                    raise RuntimeError(lib.moe_last_error(moe.ctx))
        e2e_s = time.perf_counter() - t_0
        e2e = {"value": round(n_e2e / e2e_s, 2), "unit": "tokens/s", "h2d_bytes_per_step": DENSE_LAYERS * H * 4,
               "d2h_bytes_per_step": DENSE_LAYERS * H * 4, "timer": "host wall clock (synchronous calls)"}
        extra = {"intermediate": DENSE_I, "layers": DENSE_LAYERS, "experts": 0,
                 "l2": "not flushed: 2.38 GB of weights per step cycle through the 126 MB L2"}
    elif args.workload == "head_b1":
        # one decode token through the output head and the sampler
        # (infer.m:1937-1941, 419-456): fp16 [129280 x 7168] = 1.85 GB per step
        cfg = F.MoeConfig(n_layers=1, max_tokens=1)
        moe = F.MoE(cfg, device=local)
        moe.init_lm_head_synthetic(VOCAB, seed=0, w_sigma=0.02)
        xs = [torch.randn(1, H, generator=g).to(dev) for _ in range(N_POOL)]
        logits = torch.empty(1, VOCAB, device=dev)
        tok = torch.empty(1, dtype=torch.int32, device=dev)
        stream = torch.cuda.ExternalStream(moe.stream, device=dev)
        state = 0xA1B2C3D4

        def step(i):
            moe.lm_head_device(xs[i % N_POOL], 1, logits, stream=moe.stream)
            moe.sample_device(logits, 1, VOCAB, 0.6, 0.95, (state + i) & 0xFFFFFFFF, tok, stream=moe.stream)
        with torch.cuda.stream(stream):
            for i in range(args.warmup):
                step(i)
        torch.cuda.synchronize()
        n = args.steps
        l0 = moe.kernel_launches
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(n)]
        with torch.cuda.stream(stream):
            for i in range(n):
                ev[i][0].record(stream)
                moe.lm_head_device(xs[i % N_POOL], 1, logits, stream=moe.stream)
                ev[i][1].record(stream)
                moe.sample_device(logits, 1, VOCAB, 0.6, 0.95, (state + i) & 0xFFFFFFFF, tok, stream=moe.stream)
                ev[i][2].record(stream)
        torch.cuda.synchronize()
        head_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / n
        samp_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / n
        ms = sum(e[0].elapsed_time(e[2]) for e in ev)
        launches = moe.kernel_launches - l0
        ms_step = ms / n
        value = n / (ms / 1e3)
        unit = "tokens/s"
        head_bytes = VOCAB * H * 2 + H * 4 + VOCAB * 4
        roof = {"bound": "hbm", "kernel": "k_lm_head (the sampler, k_sample, is latency-bound: see phase_ms)",
                "achieved": round(head_bytes / (head_ms / 1e3) / 1e9, 1), "peak": peak, "unit": "GB/s",
                "frac": round(head_bytes / (head_ms / 1e3) / 1e9 / peak, 4), "peak_source": peak_kind,
                "algorithmic_bytes_per_launch": head_bytes, "traffic": None}
        extra = {"vocab": VOCAB, "temp": 0.6, "top_p": 0.95, "experts": 0,
                 "l2": "not flushed: 1.85 GB of weights per step", "phase_ms": {"lm_head": round(head_ms, 4),
                                                                                 "sample": round(samp_ms, 4)}}
        # end to end: moe_lm_head (hidden in, logits out) then moe_sample (logits in, token out)
        import ctypes as C
        h_pin = xs[0].cpu().pin_memory().numpy()
        lg_pin = torch.empty(1, VOCAB).pin_memory().numpy()
        t_pin = np.empty(1, np.int32)
        lib = moe.lib
        st = C.c_uint32(state)
        n_e2e = max(2, n // 4)
        t_0 = None
        for i in range(n_e2e + 1):
            if i == 1:
                t_0 = time.perf_counter()
            if (lib.moe_lm_head(moe.ctx, h_pin.ctypes.data, 1, lg_pin.ctypes.data) != 0 or
                    lib.moe_sample(moe.ctx, lg_pin.ctypes.data, 1, VOCAB, 0.6, 0.95, C.byref(st),
                                   t_pin.ctypes.data) != 0):
                raise RuntimeError(lib.moe_last_error(moe.ctx))
        e2e_s = time.perf_counter() - t_0
        e2e = {"value": round(n_e2e / e2e_s, 2), "unit": "tokens/s", "h2d_bytes_per_step": H * 4 + VOCAB * 4,
               "d2h_bytes_per_step": VOCAB * 4 + 4, "timer": "host wall clock (synchronous calls)"}
    else:  # prefill4096: one moe_prefill_device call (tcgen05 GEMMs) per step and rank
        from flash_deepseek_b200 import ep
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        pg = None
        if world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
            pg = dist
        B = int(os.environ.get("MOE_PREFILL_TOKENS", "4096"))
        NE = args.experts
        t0, bl = ep.local_tokens(B, world, rank)  # this rank's share of the global batch
        uid = ep.share_unique_id(pg, rank, F.get_unique_id) if world > 1 else None
        cfg = F.MoeConfig(n_layers=1, max_tokens=64, n_experts=NE)
        moe = F.MoE(cfg, device=dev.index, rank=rank, world_size=world, unique_id=uid)
        moe.init_layer_synthetic(0, seed=0, down_type=F.TYPE_Q6_K)
        xs = [torch.randn(B, H, generator=g)[t0:t0 + bl].contiguous().to(dev) for _ in range(2)]
        out = torch.empty(max(1, bl), H, device=dev)
        stream = torch.cuda.ExternalStream(moe.stream, device=dev)

        def sync_all():
            torch.cuda.synchronize()
            if pg:
                pg.barrier()
            torch.cuda.synchronize()

        for i in range(max(1, args.warmup)):
            moe.prefill_device(0, xs[i % 2], bl, out)
        sync_all()
        n = max(1, args.steps)
        l0 = moe.kernel_launches
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        with torch.cuda.stream(stream):
            for i in range(n):
                flush.zero_()
                ev[i][0].record(stream)
                moe.prefill_device(0, xs[i % 2], bl, out)
                ev[i][1].record(stream)
        sync_all()
        ms = sum(a.elapsed_time(b) for a, b in ev)
        if pg:
            t = torch.tensor([ms], dtype=torch.float64)
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            ms = float(t[0])
        launches = moe.kernel_launches - l0
        ms_step = ms / n
        value = B * n / (ms / 1e3)
        unit = "tokens/s"
        flops = 2.0 * B * (K + 1) * (3 * H * I) + 2.0 * B * NE * H
        tf = flops / world / (ms_step / 1e3) / 1e12  # per GPU
        pk = 1642.1
        try:
            with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
                pk = float(json.load(f)["bf16_tflops"])
        except Exception:
            pass
        roof = {"bound": "tensor", "kernel": "whole step (router, route, plan, gather, tcgen05 gate/up and down "
                "GEMMs, combine" + (", NCCL dispatch and combine" if world > 1 else "") + "), per GPU",
                "achieved": round(tf, 2), "peak": pk, "unit": "TFLOP/s", "frac": round(tf / pk, 4),
                "peak_source": "measured dense bf16 burst (fp16 MMA, same rate)", "flops_per_step": flops,
                "traffic": None}
        e2e = None
        extra = {"tokens_per_call": B, "tokens_per_rank": bl, "path": "moe_prefill_device (tcgen05)",
                 "parallelism": f"ep{world}"}
        if rank != 0:
            clk.__exit__(None, None, None)
            moe.close()
            return None
    clk.__exit__(None, None, None)
    line = {"metric": METRIC, "value": round(value, 2), "unit": unit,
            "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": ("fp16 operands (dequantized weights, activations) on tcgen05, fp32 accumulation"
                      if args.workload == "prefill4096" else
                      "fp16 weights, fp32 activations, fp32 accumulation" if args.workload in ("dense_b1", "head_b1")
                      else
                      "int8 tensor-core products of Q4_K/Q6_K integers and 21-bit activation planes (exact), fp32 "
                      "accumulation"),
            "data": ("synthetic: random-init N(0,0.02) weights rounded to fp16 on device, N(0,1) tokens"
                     if args.workload in ("dense_b1", "head_b1") else
                     "synthetic: random-init N(0,0.02) weights quantized on device, N(0,1) tokens"),
            "config": dict({"workload": W["name"], "global_batch": W["B"], "hidden": H, "intermediate": I,
                            "experts": E, "parallelism": "ep1"}, **extra),
            "roofline": roof, "e2e": e2e, "gpu_launches": int(launches), "clocks": clk.summary()}
    moe.close()
    return line


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    W = WORKLOADS[args.workload]
    cpu = cpu_reference(args.workload, steps=args.steps, warmup=args.warmup, seconds=60.0)
    # the GPU arm's config at this world size (its per-GPU token share)
    from flash_deepseek_b200 import ep
    b_loc = ep.local_tokens(W["B"], world, 0)[1]
    line = {
        "impl": "reference", "metric": METRIC, "value": round(cpu["value"], 4), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 / cpu["value"], 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic: the GPU arm's weights (same generator and seed) and its token batches, token by token",
        "config": workload_config(W, E, world, b_loc),
        "cpu_baseline": cpu,
        "e2e": {"value": round(cpu["value"], 4), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--workload", default="decode_b64_zipf", choices=sorted(WORKLOADS) + sorted(EXTRA))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--no-extra", action="store_true",
                    help="default workload only: skip the other configurations measured after it")
    ap.add_argument("--experts", type=int, default=E,
                    help="routed experts (default 256); smaller values only to keep ncu captures small")
    ap.add_argument("--batch", type=int, default=0,
                    help="tokens per step of decode_b64_zipf / decode_b1 (default: the workload's); other "
                         "values only to size ncu captures (with --experts, the same pairs per expert)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        if args.workload in EXTRA:
            print(json.dumps({"impl": "reference", "unavailable": "the reference arm times configs 2 and 3"}))
            return
        run_reference(args)
        return
    line = run_extra(args) if args.workload in EXTRA else run_ours(args)
    if line is None:
        return
    if (args.workload == "decode_b64_zipf" and int(os.environ.get("WORLD_SIZE", "1")) == 1 and not args.no_extra
            and args.experts == E and not args.batch):
        line["configs"] = other_configs(args)
    print(json.dumps(line), flush=True)


def other_configs(args):
    """The other headline configurations, measured in the same run on the same
    GPU after the default one (each in its own context, with its own warm-up,
    timed loop, L2 handling and clock sampling, as its --workload line would
    be): config 2 (one token), config 1 (one expert per call), config 5 (4096-
    token prefill), config 4 (the 58-layer stack at batch 1), the dense FFN
    layers 0-2 and the output head with the sampler at batch 1."""
    keep = ("metric", "value", "unit", "ms_per_step", "steps", "warmup", "dtype", "roofline", "roofline_down",
            "roofline_tc", "roofline_phases",
            "phase_ms", "e2e", "gpu_launches", "clocks", "config")
    out = {}
    for wl, steps in (("decode_b1", 100), ("expert1", 256), ("prefill4096", 3), ("stack_b1", 3), ("dense_b1", 100),
                      ("head_b1", 100)):
        a = argparse.Namespace(**vars(args))
        a.workload, a.steps, a.warmup, a.no_cpu = wl, steps, 3, True
        try:
            ln = run_extra(a) if wl in EXTRA else run_ours(a)
            out[wl] = {k: ln[k] for k in keep if k in ln}
        except Exception as e:  # reported in the line; the default measurement stands
            out[wl] = {"error": repr(e)[:300]}
    return out


if __name__ == "__main__":
    main()
