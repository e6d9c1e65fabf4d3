"""Benchmark: W2A16 g128 MoE decode layers on B200 (device-timed), with e2e, roofline and a CPU baseline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--case stack|layer|batched|int8|config0|config2|gemv]

Default case ("stack"), the same workload at every N: the decode step of BASELINE config 4 -- a stack of L=48
distinct MoE layers (M=1, H=4096, I=1536, E=256 experts per layer, top-8, W2A16 g128 with per-group zero points,
f16 scales), each layer's input the previous layer's output, a fresh routing for every layer of every step. At
N=1 all 256 experts of every layer sit on the one GPU, so each layer is BASELINE config 1; at N>1 (one process per
GPU under torchrun) the experts are split 1/N per rank and every layer ends with the library's peer all-reduce of
the partial outputs over NVLink. A "step" is one pass through the L layers. `value` is the whole job's GB/s of
algorithmic layer bytes (every routed expert's codes, scales and zero points, plus x and y) over the device time
of the step (max over ranks). The step with config 4's INT8 dense [4096 -> 4096] projection after every layer is
timed as well and reported under "with_dense". No expert is reused within a window of 4 layers, and all layers
together (62 GB at N=1) are far larger than L2, so no layer reads its weights out of L2.

The JSON line also carries the dominant kernel's roofline, e2e through the public API with pinned host buffers
(each step copies its input activation and routing in and its output back), SM clocks sampled during the timed
region, and, on rank 0 at N=1, the CPU baseline (the oracle port of the reference's torch path). ``--impl
reference`` times the reference's CPU path alone and prints its own line.

Other cases (profiling drivers; one GPU): ``layer`` runs `--calls` config-1 layers over an arena of
`--experts` experts (a small arena keeps an ncu capture small); ``batched`` times config 3's token counts on the
per-token and batched paths; ``int8`` times the INT8 dense GEMV cycling 16 distinct weight matrices; ``config0``
and ``config2`` time those configurations' layers (config 2 also with the INT8 dense after it); ``gemv`` times
config 1 through the three entry forms (the reference's two-GEMV composite on the drop-in GEMV, the fused layer on
int64 address tables, the fused layer on the slot arena).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "W2A16 MoE layer µs & HBM GB/s (% of ~8 TB/s) at 1/2/4/8 B200 vs host-CPU torch"
SHAPE = dict(E=256, H=4096, I=1536, top_k=8, M=1)
LAYERS = 48
DTYPE = ("2-bit codes x 16-bit block fixed-point activations (one power-of-two exponent per 128 x values, "
         "per 32 h values) -> exact int32 group sums -> fp32 accumulation -> bf16 output")


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def measured_traffic(name: str):
    """DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) of the named kernel, from the
    committed ncu summary profiles/<name>.json (written from one ncu capture); None when absent."""
    path = os.path.join(ROOT, "profiles", name + ".json")
    if not os.path.exists(path):
        return None
    try:
        return int(json.load(open(path))["traffic_bytes_per_launch"])
    except (ValueError, KeyError):
        return None


def layer_bytes(H: int, I: int, k: int, M: int, zeros: bool = True) -> int:
    """Algorithmic bytes of one layer: every routed expert's gate_up and down codes, f16 scales and (with zeros)
    zero points, plus x and y (bf16)."""
    per = (H // 16) * 2 * I * 4 + (H // 128) * 2 * I * 2 + (I // 16) * H * 4 + (I // 128) * H * 2
    if zeros:
        per += (H // 128) * (2 * I // 4) + (I // 128) * (H // 4)
    return per * k * M + 2 * M * H * 2


# ----------------------------------------------------------------------------- routing pool
def routing_pool(P: int, E: int, k: int, window: int, seed: int):
    """P routings (top-k of softmax(N(0,1)) renormalised), redrawn until no expert repeats within
    `window` consecutive draws."""
    g = torch.Generator().manual_seed(seed)
    ids = torch.empty(P, k, dtype=torch.int32)
    ws = torch.empty(P, k, dtype=torch.float32)
    recent = []
    for i in range(P):
        banned = set(x for r in recent for x in r)
        while True:
            logits = torch.randn(E, generator=g)
            if banned:
                logits[list(banned)] = -float("inf")
            p = torch.softmax(logits, -1)
            w, idx = torch.topk(p, k)
            if not (set(idx.tolist()) & banned):
                break
        ids[i] = idx.to(torch.int32)
        ws[i] = w / w.sum()
        recent.append(idx.tolist())
        if len(recent) > window - 1:
            recent.pop(0)
    return ids, ws


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.idx), "-lms", "100"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.15)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- timing helpers
def capture(fn, P: int):
    """A CUDA graph of fn(0) .. fn(P-1) (warmed once on the capture stream)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        fn(0)
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=s):
            for i in range(P):
                fn(i)
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    return g


def time_replays(g, reps: int, barrier=None):
    """Device time (ms) of `reps` back-to-back replays, and of each replay (CUDA events on the current stream)."""
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(reps + 1)]
    if barrier:
        barrier()
    torch.cuda.synchronize()
    evs[0].record()
    for r in range(reps):
        g.replay()
        evs[r + 1].record()
    torch.cuda.synchronize()
    each = [evs[r].elapsed_time(evs[r + 1]) for r in range(reps)]
    return evs[0].elapsed_time(evs[reps]), each


def pct(xs, q):
    xs = sorted(xs)
    return xs[min(len(xs) - 1, int(round(q * (len(xs) - 1))))]


# ----------------------------------------------------------------------------- CPU baseline
def cpu_baseline(arena, x, ids, w, budget_s: float):
    import oracle as O
    experts = O.routed_experts_from_arena(arena, ids)
    sec, n = O.time_cpu_layer(x.cpu(), experts, ids.cpu().reshape(1, -1), w.cpu().reshape(1, -1), budget_s)
    return sec, n, O.cpu_info()


def stack_workload(E: int, world: int) -> str:
    """The workload string of the default case (both arms)."""
    return (f"config4 stack of {LAYERS} MoE layers, each config 1 (M=1 H=4096 I=1536 E=256 top-8 W2A16 g128 zp "
            f"f16 scales), experts {E // world} per GPU")


# ----------------------------------------------------------------------------- the layer stack, any N
def run_stack(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import torch.distributed as dist
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    try:
        _run_stack(args, world, rank, dev)
    except BaseException:
        # A rank that fails says why and leaves at once: waiting in a barrier here would only hold it until the
        # other ranks' next collective times out, and the launcher ends the other ranks when this one exits.
        import traceback
        traceback.print_exc()
        sys.stderr.flush()
        sys.stdout.flush()
        os._exit(1)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _run_stack(args, world: int, rank: int, dev: torch.device):
    import torch.distributed as dist
    import __graft_entry__ as graft
    import oracle as O
    pkg = graft.load_package()
    ep = pkg.expert_parallel
    E, H, I, k, M = (SHAPE[n] for n in ("E", "H", "I", "top_k", "M"))
    L = LAYERS
    lo, hi = ep.expert_range(E, world, rank)
    slots = ep.local_slot_table(E, world, rank, dev)
    t0 = time.time()
    arenas = []
    for l in range(L):
        a = pkg.synth.make_arena(hi - lo, H, I, seed=7919 * l + lo, zeros=True, scale_dtype=torch.float16,
                                 device=dev)
        arenas.append(pkg.ExpertArena(a.codes13, a.scales13, a.codes2, a.scales2, a.zeros13, a.zeros2, slots))
    dense = [pkg.synth.make_int8_dense(H, H, seed=104729 + l, device=dev) for l in range(L)]
    ar = ep.PeerAllReduce(M * H, dev) if world > 1 else None
    P = 8                                              # steps (routings) cycled by the timed graph
    ids_all, w_all = routing_pool(P * L, E, k, window=4, seed=0)
    ids_d = ids_all.reshape(P, L, M, k).to(dev)
    w_d = w_all.reshape(P, L, M, k).to(dev)
    x_d = pkg.synth.make_activation(P * M, H, seed=0, device=dev).reshape(P, M, H)
    bufs = [torch.empty(M, H, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    setup_s = time.time() - t0
    barrier = (lambda: dist.barrier()) if world > 1 else None

    def moe(x, l, i, out):
        y = pkg.moe_decode_layer(x, ids_d[i, l], w_d[i, l], arenas[l], out=out if ar is None else None)
        return ar(y) if ar is not None else y

    def step_unfused(i, with_dense=False, x0=None):
        x = x_d[i] if x0 is None else x0
        for l in range(L):
            y = moe(x, l, i, bufs[l & 1])
            x = pkg.int8_gemv(y, dense[l][0], dense[l][1]) if with_dense else y
        return x

    def step(i, with_dense=False, x0=None):
        """N=1: each layer writes into the next one's input buffer. N>1: the exchange folded into the kernels --
        every layer pushes its partial into every rank's buffer and the next layer (or the INT8 projection) sums
        the ranks' partials while it converts its activation; one all-reduce closes the step without the dense."""
        x = x_d[i] if x0 is None else x0
        if ar is None:
            return step_unfused(i, with_dense, x)
        if with_dense:
            for l in range(L):
                ar.layer(x, ids_d[i, l], w_d[i, l], arenas[l], y_to_peers=True)
                x = ar.int8(dense[l][0], dense[l][1], M, out=bufs[l & 1])
            return x
        return ep.ep_stack_step(ar, x, ids_d[i], w_d[i], arenas, out=bufs[0])

    # correctness of one layer of the stack: GPU output vs the fp32 oracle (partials all-reduced over ranks)
    y0 = moe(x_d[0], 0, 0, bufs[0])
    ref = O.moe_layer_from_arena(arenas[0], x_d[0], ids_d[0, 0], w_d[0, 0]).to(dev)
    if world > 1:
        dist.all_reduce(ref)
    err = O.max_rel_err(y0.float().cpu(), ref.cpu())
    fused_same = None
    if ar is not None:                       # the folded exchange against (layer, all-reduce) per layer, bit for bit
        a0 = step_unfused(0).clone()
        b0 = step(0).clone()
        a1 = step_unfused(1, True).clone()
        b1 = step(1, True).clone()
        torch.cuda.synchronize()
        fused_same = bool(torch.equal(a0, b0) and torch.equal(a1, b1))

    for i in range(max(args.warmup, 3)):
        step(i % P)
    torch.cuda.synchronize()
    steps = max(1, args.steps)
    reps, rem = divmod(steps, P)
    g = capture(lambda i: step(i), P) if reps else None
    g_rem = capture(lambda i: step(i), rem) if rem else None
    with ClockSampler(dev.index or 0) as clk:
        ms, each = time_replays(g, reps, barrier) if reps else (0.0, [])
        if g_rem is not None:                          # the last steps % P steps (exactly `steps` steps in all)
            ms_rem, _ = time_replays(g_rem, 1, barrier)
            ms += ms_rem
    del g, g_rem
    tm = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
    us_step = float(tm.item()) * 1e3 / steps
    us_layer = us_step / L
    per_layer = [e * 1e3 / (P * L) for e in each] or [us_layer]

    gd = capture(lambda i: step(i, with_dense=True), P)
    reps_d = max(1, reps // 2)
    msd, _ = time_replays(gd, reps_d, barrier)
    del gd
    tmd = torch.tensor([msd], device=dev)
    if world > 1:
        dist.all_reduce(tmd, op=dist.ReduceOp.MAX)
    us_step_dense = float(tmd.item()) * 1e3 / (reps_d * P)

    # e2e: every step copies its input activation and its L layers' routing in from pinned host memory and its
    # output back, around the public-API calls (a CUDA graph of P steps, as a decode loop replays graphs)
    xh = x_d.cpu().pin_memory()
    rh = torch.cat([ids_d.view(P, -1).view(torch.uint8).cpu(), w_d.view(P, -1).view(torch.uint8).cpu()], 1).pin_memory()
    out_h = torch.empty(P, M, H, dtype=torch.bfloat16).pin_memory()
    x_in = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
    r_in = torch.empty(rh.shape[1], dtype=torch.uint8, device=dev)
    nid = ids_d[0].numel() * 4
    ids_in = r_in[:nid].view(torch.int32).view(L, M, k)
    w_in = r_in[nid:].view(torch.float32).view(L, M, k)

    def e2e_step(i):
        x_in.copy_(xh[i], non_blocking=True)
        r_in.copy_(rh[i], non_blocking=True)
        x = x_in
        if ar is None:
            for l in range(L):
                x = pkg.moe_decode_layer(x, ids_in[l], w_in[l], arenas[l], out=bufs[l & 1])
        else:
            x = ep.ep_stack_step(ar, x, ids_in, w_in, arenas, out=bufs[0])
        out_h[i].copy_(x, non_blocking=True)

    ge = capture(e2e_step, P)
    reps_e = max(1, reps)
    t_host = time.perf_counter()
    mse, _ = time_replays(ge, reps_e, barrier)
    host_ms = (time.perf_counter() - t_host) * 1e3
    del ge
    tme = torch.tensor([max(mse, host_ms)], device=dev)
    if world > 1:
        dist.all_reduce(tme, op=dist.ReduceOp.MAX)
    e2e_us_step = float(tme.item()) * 1e3 / (reps_e * P)
    h2d = x_in.numel() * 2 + r_in.numel()
    d2h = M * H * 2
    ar_flag = 0
    if ar is not None:
        try:
            ar.check()
        except RuntimeError:
            ar_flag = 1

    bpl = layer_bytes(H, I, k, M)
    gbs = bpl * L / (us_step * 1e-6) / 1e9
    peak, peak_kind = peaks()
    if rank != 0:
        return
    cpu = None
    if world == 1:
        sec, n_cpu, info = cpu_baseline(arenas[0], x_d[0], ids_d[0, 0], w_d[0, 0], args.cpu_budget)
        cpu = {"value": round(bpl / sec / 1e9, 3), "unit": "GB/s", "cores": info["torch_threads"], "kind": "port",
               "us_per_layer": round(sec * 1e6, 1),
               "sample": f"{n_cpu} layers of config 1 (8 routed experts dequantised in fp32 + matmuls, torch CPU)",
               "cpu_model": info["cpu_model"], "cpu_count": info["cpu_count"]}
    per_gpu = gbs / world
    line = {
        "metric": METRIC, "value": round(gbs, 1), "unit": "GB/s", "n_gpus": world, "steps": steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(us_step / 1e3, 6), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": DTYPE,
        "data": "synthetic (seeded; BASELINE config 1 / config 4 distributions)",
        "config": {"workload": stack_workload(E, world),
                   "global_batch": M, "seq_len": 1,
                   "parallelism": "single GPU" if world == 1 else f"ep{world} (exchange folded into the layer kernels)",
                   "l2": f"inputs larger than L2 ({(hi - lo) * L} local experts, {bpl * L * world // 2**20} MB of "
                         "routed weights per step; no expert reused within 4 layers)",
                   "layers": L, "graph_steps": P},
        "us_per_layer": round(us_layer, 3), "us_per_layer_p50": round(pct(per_layer, 0.5), 3),
        "us_per_layer_p99": round(pct(per_layer, 0.99), 3),
        "percentiles_over": f"{len(per_layer)} graph replays of {P} steps x {L} layers (mean layer time per replay)",
        "bytes_per_layer": bpl, "hbm_frac": round(per_gpu / peak, 4), "hbm_peak_gbs": peak,
        "roofline": {"bound": "hbm", "achieved": round(per_gpu, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(per_gpu / peak, 4), "traffic": measured_traffic("fused_layer_config1"),
                     "kernel": "fused_layer_kernel (gate_up+SiLU*mul, grid barrier, down+weighted top-k sum): one "
                               "cooperative launch per layer; achieved = algorithmic layer bytes / device time per "
                               "layer" + ("" if world == 1 else " / N GPUs (includes the exchange)"),
                     "peak_kind": peak_kind},
        "e2e": {"value": round(bpl * L / (e2e_us_step * 1e-6) / 1e9, 1), "unit": "GB/s",
                "us_per_layer": round(e2e_us_step / L, 3), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "how": "CUDA graph of steps, each: pinned-host H2D of x and the L layers' routing, L moe_decode_layer "
                       "calls" + ("" if world == 1 else " + peer all-reduces") + ", D2H of the output (max of device "
                       "events and host wall clock)"},
        "with_dense": {"us_per_step": round(us_step_dense, 2), "us_per_layer": round(us_step_dense / L, 3),
                       "gbs": round((bpl + (H // 4) * H * 4 + H * 2) * L / (us_step_dense * 1e-6) / 1e9, 1),
                       "what": "config 4 step: every MoE layer followed by the INT8 dense [4096 -> 4096] GEMV "
                               "(replicated on every rank)"},
        "gpu_launches": steps * L if world == 1 else steps * (L + 1),
        "clocks": clk.summary(),
        "check_max_rel_err": err,
        "setup_s": round(setup_s, 1),
    }
    if cpu:
        line["cpu_baseline"] = cpu
    if ar is not None:
        line["exchange"] = {"impl": "folded into the layer kernels (w2a16_moe_decode_layer_slots_ep: partials pushed "
                                    "into every rank's buffer over NVLink, summed by the next layer / projection), "
                                    "one w2a16_allreduce_peers_bf16 closing the step",
                            "equals_layer_allreduce_bit_for_bit": fused_same, "device_error": ar_flag}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- profiling cases (one GPU)
def run_case_layer(args):
    """`--calls` config-1 layers over an arena of `--experts` experts (no expert reused within 4 calls), the
    last one checked against the oracle. The command that ncu captures use."""
    import __graft_entry__ as graft
    import oracle as O
    pkg = graft.load_package()
    dev = torch.device("cuda", 0)
    E, H, I, k, M = args.experts, SHAPE["H"], SHAPE["I"], SHAPE["top_k"], args.M
    arena = pkg.synth.make_arena(E, H, I, seed=0, zeros=True, scale_dtype=torch.float16, device=dev)
    ids_pool, w_pool = routing_pool(args.calls * M, E, k, window=min(4, max(1, E // (2 * k))), seed=0)
    x = pkg.synth.make_activation(args.calls * M, H, seed=0, device=dev)
    ids, ws = ids_pool.to(dev), w_pool.to(dev)
    y = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
    for c in range(args.calls):
        sl = slice(c * M, (c + 1) * M)
        pkg.moe_decode_layer(x[sl], ids[sl], ws[sl], arena, out=y)
    torch.cuda.synchronize()
    sl = slice((args.calls - 1) * M, args.calls * M)
    err = O.max_rel_err(y.float().cpu(), O.moe_layer_from_arena(arena, x[sl], ids[sl], ws[sl]))
    print(json.dumps({"case": "layer", "experts": E, "M": M, "calls": args.calls, "max_rel_err": err}))
    return 0 if err < 1e-2 else 1


def run_case_batched(args):
    """Config 3's token counts: the layer per call (CUDA-graph replay of `--calls` calls, fresh uniform routing per
    call) on the per-token path and on the batched tensor-core path; bytes per layer count each distinct routed
    expert once. The last call of each path is checked against the oracle."""
    import __graft_entry__ as graft
    import oracle as O
    pkg = graft.load_package()
    dev = torch.device("cuda", 0)
    E, H, I, k = SHAPE["E"], SHAPE["H"], SHAPE["I"], SHAPE["top_k"]
    arena = pkg.synth.make_arena(E, H, I, seed=0, zeros=True, scale_dtype=torch.float16, device=dev, gen_device=dev)
    per_expert = arena.bytes_per_expert()
    rc = 0
    for M in args.tokens:
        P = args.calls
        x = pkg.synth.make_activation(P * M, H, seed=M, device=dev, gen_device=dev).reshape(P, M, H)
        ids, w = pkg.synth.route_softmax(P * M, E, k, seed=M, device=dev, gen_device=dev, uniform_logits=True)
        ids = ids.reshape(P, M, k).contiguous()
        w = w.reshape(P, M, k).contiguous()
        distinct = sum(int(torch.unique(ids[c]).numel()) for c in range(P)) / P
        res = {}
        for name, batched in (("batched", True), ("per-token", False)):
            if batched and M < 16:
                continue
            y = torch.empty(P, M, H, dtype=torch.bfloat16, device=dev)
            g = capture(lambda c: pkg.moe_decode_layer(x[c], ids[c], w[c], arena, batched=batched, out=y[c]), P)
            times = [time_replays(g, 1)[0] * 1e3 / P for _ in range(3)]
            us = sorted(times)[1]
            del g
            rel = O.max_rel_err(y[P - 1].float().cpu(), O.moe_layer_by_expert(arena, x[P - 1], ids[P - 1], w[P - 1]))
            res[name] = us
            rc |= 0 if rel < 1e-2 else 1
            print(json.dumps({"case": "batched", "M": M, "path": name, "us_per_layer": round(us, 1),
                              "distinct_experts": round(distinct, 1),
                              "gbs_distinct": round(distinct * per_expert / us / 1e3, 1), "max_rel_err": rel}))
    return rc


def run_case_gemv(args):
    """Config 1 (E=256, M=1, top-8) through the three entry forms a caller has, CUDA-graph replay over 16 routings
    (no expert reused within 4 calls, the 1.3 GB arena > L2), µs per layer:
      `two_gemv`  -- the reference's `_apply_gemv` composite on the drop-in `moe_gemv_int2_tab` (gate_up GEMV,
                     silu*mul and the top-k sum in torch, down GEMV with the routed weight), as the shim of the
                     integration notes runs it;
      `table`     -- `apply_gemv` on the reference's int64 address tables (one fused launch, register mode);
      `slots`     -- `moe_decode_layer` on the slot arena (one fused launch, copy-engine mode)."""
    import __graft_entry__ as graft
    import oracle as O
    import torch.nn.functional as F
    pkg = graft.load_package()
    dev = torch.device("cuda", 0)
    E, H, I, k = 256, SHAPE["H"], SHAPE["I"], SHAPE["top_k"]
    arena = pkg.synth.make_arena(E, H, I, seed=0, zeros=True, scale_dtype=torch.float16, device=dev)
    P = 16
    ids_pool, w_pool = routing_pool(P, E, k, window=4, seed=0)
    ids, ws = ids_pool.to(dev).reshape(P, 1, k), w_pool.to(dev).reshape(P, 1, k)
    x = pkg.synth.make_activation(P, H, seed=0, device=dev).reshape(P, 1, H)
    wt13, st13, sw13, ss13 = pkg.make_tables(arena.codes13, arena.scales13)
    wt2, st2, sw2, ss2 = pkg.make_tables(arena.codes2, arena.scales2)
    zt13, zs13 = pkg.make_zero_table(arena.zeros13)
    zt2, zs2 = pkg.make_zero_table(arena.zeros2)
    tabs = ((wt13, st13, sw13, ss13), (wt2, st2, sw2, ss2), 2 * I, H, H, I, False)
    y = torch.empty(P, 1, H, dtype=torch.bfloat16, device=dev)

    def two_gemv(i):
        gu = pkg.moe_gemv_int2_tab(x[i], wt13, st13, ids[i], ws[i], 2 * I, H, sw13, ss13, k, False,
                                   scale_bf16=False, ztab=zt13, stride_zg=zs13)
        h = (F.silu(gu[:, :I].float()) * gu[:, I:].float()).to(torch.bfloat16)
        dn = pkg.moe_gemv_int2_tab(h, wt2, st2, ids[i], ws[i], H, I, sw2, ss2, 1, True,
                                   scale_bf16=False, ztab=zt2, stride_zg=zs2)
        y[i].copy_(dn.float().sum(0, keepdim=True))

    forms = {"two_gemv": two_gemv,
             "table": lambda i: y[i].copy_(pkg.apply_gemv(x[i], ids[i], ws[i], tabs, None, zero_tabs=(zt13, zt2))),
             "slots": lambda i: pkg.moe_decode_layer(x[i], ids[i], ws[i], arena, out=y[i])}
    out = {"case": "gemv", "E": E, "H": H, "I": I, "top_k": k, "M": 1}
    for name, fn in forms.items():
        g = capture(fn, P)
        times = [time_replays(g, 1)[0] * 1e3 / P for _ in range(5)]
        del g
        torch.cuda.synchronize()
        ref = O.moe_layer_from_arena(arena, x[P - 1], ids[P - 1], ws[P - 1])
        out[name] = {"us_per_layer": round(sorted(times)[2], 2),
                     "max_rel_err": O.max_rel_err(y[P - 1].float().cpu(), ref)}
    print(json.dumps(out))
    return 0 if all(out[n]["max_rel_err"] < 1e-2 for n in forms) else 1


def run_case_int8(args):
    """The INT8 dense [4096 -> 4096] GEMV (config 2/4) over 16 distinct weight matrices cycled (269 MB > L2):
    µs per call and GB/s of algorithmic bytes (weights + scales + x + y), CUDA-graph replay; checked once."""
    import __graft_entry__ as graft
    import oracle as O
    pkg = graft.load_package()
    dev = torch.device("cuda", 0)
    K = N = SHAPE["H"]
    mats = [pkg.synth.make_int8_dense(K, N, seed=3 + i, device=dev) for i in range(16)]
    x = pkg.synth.make_activation(16, K, seed=5, device=dev)
    ys = torch.empty(16, N, dtype=torch.bfloat16, device=dev)

    def call(i):
        q, s = mats[i % 16]
        pkg.int8_gemv(x[i % 16:i % 16 + 1], q, s, out=ys[i % 16:i % 16 + 1])

    P = 64
    g = capture(call, P)
    times = [time_replays(g, 1)[0] * 1e3 / P for _ in range(5)]
    us = sorted(times)[2]
    del g
    q, s = mats[15]
    ref = O.int8_gemv(x[15:16].float().cpu(), q.cpu(), s.float().cpu())
    err = O.max_rel_err(ys[15:16].float().cpu(), ref)
    nbytes = K * N + N * 2 + K * 2 + N * 2
    peak, kind = peaks()
    print(json.dumps({"case": "int8", "K": K, "N": N, "us_per_call": round(us, 3), "gbs": round(nbytes / us / 1e3, 1),
                      "hbm_frac": round(nbytes / us / 1e3 / peak, 4), "peak_kind": kind, "max_rel_err": err,
                      "l2": "16 distinct weight matrices cycled (269 MB > L2)"}))
    return 0 if err < 1e-2 else 1


def run_case_config(args):
    """BASELINE config 0 (H=2048, I=768, E=64, top-8, M=1) or config 2 (config-1 shapes, S=184 of 256 experts
    resident in a random permutation of arena rows, Zipf(1.1) routing, misses masked through slot -1, plus the
    INT8 dense [4096 -> 4096]): the layer per call in a CUDA graph of `--calls` calls with a fresh routing each
    (and the dense after each layer for config 2), bytes = the routed experts that are resident; the last call
    checked against the oracle."""
    import __graft_entry__ as graft
    import oracle as O
    pkg = graft.load_package()
    dev = torch.device("cuda", 0)
    k, M, P = 8, 1, max(args.calls, 8)
    if args.case == "config0":
        E, H, I, S = 64, 2048, 768, 64
        slots = None
        pop = None
    else:
        E, H, I, S = 256, 4096, 1536, 184
        pop = pkg.synth.zipf_popularity(E, 1.1, seed=2)
        slots = pkg.synth.resident_slots(pop, S, seed=2)
    arena = pkg.synth.make_arena(S, H, I, seed=7, zeros=True, scale_dtype=torch.float16, device=dev, gen_device=dev,
                                 slots=slots)
    if pop is None:
        routes = [pkg.synth.route_softmax(M, E, k, seed=100 + c, device=dev, gen_device=dev) for c in range(P)]
    else:
        routes = [pkg.synth.route_zipf(M, E, k, pop, seed=100 + c, device=dev) for c in range(P)]
    ids = torch.stack([r[0] for r in routes])
    w = torch.stack([r[1] for r in routes])
    x = pkg.synth.make_activation(P * M, H, seed=3, device=dev, gen_device=dev).reshape(P, M, H)
    y = torch.empty(P, M, H, dtype=torch.bfloat16, device=dev)
    g = capture(lambda c: pkg.moe_decode_layer(x[c], ids[c], w[c], arena, out=y[c]), P)
    us = sorted(time_replays(g, 1)[0] * 1e3 / P for _ in range(3))[1]
    del g
    st = arena.slots.cpu()
    resident = [[int(e) for e in ids[c, 0].tolist() if int(st[e]) >= 0] for c in range(P)]
    nbytes = sum(len(r) for r in resident) / P * arena.bytes_per_expert() + 2 * M * H * 2
    err = O.max_rel_err(y[P - 1].float().cpu(), O.moe_layer_from_arena(arena, x[P - 1], ids[P - 1], w[P - 1]))
    peak, kind = peaks()
    line = {"case": args.case, "E": E, "S": S, "H": H, "I": I, "M": M, "top_k": k, "us_per_layer": round(us, 3),
            "resident_routed_per_call": round(sum(len(r) for r in resident) / P, 2),
            "gbs": round(nbytes / us / 1e3, 1), "hbm_frac": round(nbytes / us / 1e3 / peak, 4), "peak_kind": kind,
            "max_rel_err": err}
    rc = 0 if err < 1e-2 else 1
    if args.case == "config2":
        q, sc = pkg.synth.make_int8_dense(H, H, seed=11, device=dev, gen_device=dev)
        z = torch.empty(P, M, H, dtype=torch.bfloat16, device=dev)

        def both(c):
            pkg.moe_decode_layer(x[c], ids[c], w[c], arena, out=y[c])
            pkg.int8_gemv(y[c], q, sc, out=z[c])
        g = capture(both, P)
        us2 = sorted(time_replays(g, 1)[0] * 1e3 / P for _ in range(3))[1]
        del g
        ref = O.int8_gemv(y[P - 1].float().cpu(), q.cpu(), sc.float().cpu())
        err2 = O.max_rel_err(z[P - 1].float().cpu(), ref)
        line.update({"us_layer_plus_dense": round(us2, 3), "dense_max_rel_err": err2})
        rc |= 0 if err2 < 1e-2 else 1
    print(json.dumps(line))
    return rc


# ----------------------------------------------------------------------------- reference arm
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle as O
    E, H, I, k, M = (SHAPE[n] for n in ("E", "H", "I", "top_k", "M"))
    # only the routed experts are materialised on the host (the reference dequantises those)
    ids_pool, w_pool = routing_pool(max(args.steps, 1), E, k, window=4, seed=0)
    g = torch.Generator().manual_seed(0)
    experts = {}
    for e in ids_pool[0].tolist():
        gg = torch.Generator().manual_seed(1000 + e)
        c13 = torch.randint(-(2 ** 31), 2 ** 31, (H // 16, 2 * I), dtype=torch.int32, generator=gg)
        s13 = (torch.randn(H // 128, 2 * I, generator=gg).abs() * 0.02).half()
        z13 = torch.randint(0, 256, (H // 128, 2 * I // 4), dtype=torch.uint8, generator=gg)
        c2 = torch.randint(-(2 ** 31), 2 ** 31, (I // 16, H), dtype=torch.int32, generator=gg)
        s2 = (torch.randn(I // 128, H, generator=gg).abs() * 0.02).half()
        z2 = torch.randint(0, 256, (I // 128, H // 4), dtype=torch.uint8, generator=gg)
        experts[e] = (c13, s13, z13, c2, s2, z2)
    x = torch.randn(1, H, generator=g).to(torch.bfloat16)
    bps = layer_bytes(H, I, k, M)
    torch.set_num_threads(os.cpu_count() or 1)
    for _ in range(max(args.warmup, 1)):
        O.moe_layer_routed_only(x, experts, ids_pool[:1], w_pool[:1])
    n = max(1, args.steps)
    t0 = time.perf_counter()
    for i in range(n):
        O.moe_layer_routed_only(x, experts, ids_pool[:1], w_pool[:1])
    sec = (time.perf_counter() - t0) / n
    info = O.cpu_info()
    gbs = bps / sec / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": n, "warmup": max(args.warmup, 1), "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded; BASELINE config 1 distributions)",
        # the same workload string as this bench's own arm at the launch's N; each sampled layer timed on the host
        "config": {"workload": stack_workload(E, max(1, args.gpus)), "global_batch": M, "seq_len": 1,
                   "parallelism": "host CPU (the reference's torch formulation, all host threads)", "layers": LAYERS},
        "us_per_layer": round(sec * 1e6, 1),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": info["torch_threads"], "kind": "port",
                         "sample": f"{n} layers: 8 routed experts dequantised in fp32 + matmuls (torch CPU)",
                         "cpu_model": info["cpu_model"], "cpu_count": info["cpu_count"]},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--case", choices=["stack", "layer", "batched", "int8", "config0", "config2", "gemv"],
                    default="stack")
    ap.add_argument("--cpu-budget", type=float, default=10.0, help="seconds of CPU baseline sampling")
    ap.add_argument("--experts", type=int, default=256, help="case layer: experts in the arena")
    ap.add_argument("--calls", type=int, default=6, help="case layer / batched: calls")
    ap.add_argument("--M", type=int, default=1, help="case layer: tokens per call")
    ap.add_argument("--tokens", type=int, nargs="+", default=[4, 16, 64], help="case batched: token counts")
    args = ap.parse_args()
    if args.impl == "reference":
        # bounded CPU work: each step is one layer of the reference formulation (~0.1-1 s)
        args.steps = max(1, min(args.steps, 20))
        run_reference(args)
        return 0
    if args.case == "layer":
        return run_case_layer(args)
    if args.case == "batched":
        return run_case_batched(args)
    if args.case == "int8":
        return run_case_int8(args)
    if args.case == "gemv":
        return run_case_gemv(args)
    if args.case in ("config0", "config2"):
        return run_case_config(args)
    run_stack(args)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
