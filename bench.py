#!/usr/bin/env python3
"""bench.py — expert-FFN decode throughput on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl warp|reference]
                    [--config cfg4|cfg3|cfg1]

One step = one decode token through the config's MoE stack (per layer:
RMSNorm, router, top-k, routed VQ3R experts, Q4 shared expert, route-ordered
combine, residual; attention is an identity residual, as the config states).
The default workload is BASELINE.json configs[3], the 600B-class block quoted
at 1/2/4/8 GPUs: hidden 7168, 256 routed experts (inter 2048) + 1 shared, top-8,
8 layers, decode batch 1.  Weights are seeded synthetic (random-code recipe of
the reference's make_test_container.py), resident in HBM.

Prints ONE JSON line (rank 0).  value = packed weight GB/s of the whole job
(bytes of every routed record, shared expert and router a step reads, over the
device-timed step), tokens_per_s beside it.  The reference arm (--impl
reference) times the reference's own CPU expert path (oracle/_ref, compiled
from the reference sources; the oracle port when that library is absent) on
the host cores.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "expert-FFN packed GB/s (% HBM peak) and decode tok/s at 1/2/4/8 B200"

CONFIGS = {
    "cfg4": dict(workload="600B-class MoE block decode (BASELINE.json configs[3])",
                 hidden=7168, inter=2048, E=256, K=8, layers=8, shared_inter=2048, seed=2,
                 zipf=1.1),
    "cfg5": dict(workload="trillion-class MoE decode, resident across GPUs "
                          "(BASELINE.json configs[4])",
                 hidden=7168, inter=2048, E=384, K=16, layers=60, shared_inter=2048, seed=3,
                 zipf=None, min_gpus=3),
    "cfg3": dict(workload="48B-class MoE decode stack (BASELINE.json configs[2])",
                 hidden=2304, inter=1024, E=256, K=8, layers=26, shared_inter=1024, seed=1,
                 zipf=None),
    "cfg2": dict(workload="trunk dequant-matvec sweep (BASELINE.json configs[1])", trunk=True,
                 hidden=7168, inter=0, E=0, K=0, layers=0, shared_inter=0, seed=5),
    "cfg1": dict(workload="single MoE layer decode (BASELINE.json configs[0])",
                 hidden=2304, inter=1024, E=32, K=8, layers=1, shared_inter=1024, seed=0,
                 zipf=None),
}


def load_peaks(kind="hbm_gbs"):
    """(peak, "measured"|"fallback"): HBM GB/s, or dense 16-bit TFLOP/s."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        if kind in d:
            return float(d[kind]), "measured"
    return (6650.0 if kind == "hbm_gbs" else 1590.0), "fallback"


# ---------------------------------------------------------------- clocks --

class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
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
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------- model --

def stack_bytes(cfg):
    """Resident bytes of the config's whole stack (records, shared expert,
    router), for deciding whether it fits one GPU."""
    from warp_b200 import container as C
    H, I, E, L = cfg["hidden"], cfg["inter"], cfg["E"], cfg["layers"]
    rec = C.record_layout(H, I)[5]
    shared = 3 * cfg["shared_inter"] * H * 0.5625
    return L * (E * rec + shared + 4 * E * H)


def build_model(cfg, device, ep_rank=0, ep_size=1, ep_mode=0):
    """The config's layers on this device.  Expert-parallel ranks hold only
    the experts they own (ep.owned_experts) in mode 0, every expert in mode
    1; router, codebooks and shared expert are the whole layer's on every
    rank (same seeds everywhere)."""
    import math
    import torch
    from warp_b200 import ep, synth
    H, E = cfg["hidden"], cfg["E"]
    experts = ep.owned_experts(E, ep_rank, ep_size) if ep_size > 1 and ep_mode == 0 else None
    u = synth.zipf_direction(H, cfg["seed"]) if cfg.get("zipf") else None
    model = []
    for l in range(cfg["layers"]):
        seed = cfg["seed"] * 1000 + l
        bank = synth.random_bank(E, H, cfg["inter"], seed, device=device, layer=l,
                                 experts=experts)
        if u is not None:
            router, _ = synth.zipf_router(E, H, seed + 500, u, synth.ZIPF_A * math.sqrt(H),
                                          s=cfg["zipf"], device=device)
        else:
            router = synth.router_matrix(E, H, seed + 500, device=device)
        shared = synth.shared_expert(H, cfg["shared_inter"], seed + 700, device=device)
        model.append(synth.SyntheticLayer(bank, router, shared))
    torch.cuda.synchronize()
    return model, u


class Stack:
    """The decode stack: per layer h = h + MoE(RMSNorm(h)) for T tokens.

    One CUDA graph per step.  Expert-parallel, each layer inside it is
    RMSNorm, warp_moe_layer_forward_ep into the slots, the NCCL all-reduce
    of the slots (captured into the same graph, so a step makes no host
    round trip), warp_moe_layer_combine."""

    def __init__(self, model, K, device, T=1, ep_rank=0, ep_size=1, ep_mode=0):
        import torch
        self.model, self.K, self.T = model, K, T
        self.ep_rank, self.ep_size = ep_rank, ep_size
        self.ep = ep_size > 1
        self.moes = [lay.moe(K, max_tokens=T, ep_rank=ep_rank, ep_size=ep_size, ep_mode=ep_mode)
                     for lay in model]
        H = model[0].bank.hidden
        self.h = torch.zeros(T, H, device=device)
        self.bufs = [torch.zeros(T, H, device=device) for _ in range(2)]
        self.xn = torch.zeros(T, H, device=device)
        self.slots = [m.slots(T, device) for m in self.moes] if self.ep else None
        self.graph = None
        self.out = self.bufs[(len(self.moes) - 1) % 2]

    # -- eager pieces
    def _pre(self, i, cur, routes=None):
        from warp_b200 import ops
        if self.ep:
            ops.rmsnorm(cur, out=self.xn)
            r = self.moes[i].forward_ep(self.xn, self.slots[i], want_route=routes is not None)
        else:
            # RMSNorm fused into the layer's kernels: h + MoE(RMSNorm(h))
            r = self.moes[i].forward_block(cur, out=self.bufs[i % 2],
                                           want_route=routes is not None)
            r = r[1:] if routes is not None else None
        if routes is not None:
            routes.append(r[0].cpu())

    def _post(self, i, cur):
        self.moes[i].combine(self.slots[i], residual=cur, out=self.bufs[i % 2])

    def _reduce(self, i):
        from warp_b200 import ep
        ep.all_reduce_slots(self.slots[i])

    def step(self, routes=None):
        """One eager step (routes: a list that receives each layer's top-k)."""
        cur = self.h
        for i in range(len(self.moes)):
            self._pre(i, cur, routes)
            if self.ep:
                self._reduce(i)
                self._post(i, cur)
            cur = self.bufs[i % 2]
        return cur

    def capture(self):
        import torch
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                self.step()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.step()
        self.graph = g

    def replay(self):
        self.graph.replay()

    def release(self):
        self.graph = None

    def collect(self):
        for m in self.moes:
            m.collect()


# ------------------------------------------------------- CPU (reference) --

def cpu_reference(cfg, seconds, want_lib="ref"):
    """Bounded CPU sample: (GB/s, tok/s, cores, kind, sample, bytes/token)."""
    one, per_tok, cores, kind, pool, done = cpu_layer(cfg, want_lib)
    import numpy as np
    rng = np.random.default_rng(cfg["seed"] + 99)
    xs = rng.standard_normal((64, cfg["hidden"])).astype(np.float32)
    one(xs[0])                                            # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        one(xs[n % 64])
        n += 1
        dt = time.perf_counter() - t0
        if dt >= seconds and n >= 3:
            break
    done()
    gbs = per_tok * n / dt / 1e9
    tok_s = n / dt / cfg["layers"]
    sample = (f"{n} tokens through one {cfg['E']}-expert layer at config shapes "
              f"({dt:.1f} s; records aliased over a pool of {pool} distinct); tok/s scaled "
              f"to the {cfg['layers']}-layer stack")
    return gbs, tok_s, cores, kind, sample, per_tok


def cpu_layer(cfg, want_lib="ref"):
    """One layer of the reference's own expert path on the host cores: router matvec,
    waste_qwen_moe_route, experts_staged over the top-k records, the Q4
    shared expert through ffn, route-ordered sum — for tokens through one
    layer, repeated for `seconds`.  The layer's 256 records alias a pool of
    32 distinct random records (528 MB at cfg4 shapes, far above the host
    caches), so the memory traffic is that of distinct experts.
    Returns (run one token through the layer, packed bytes per token, cores,
    kind, pool size, release)."""
    import ctypes

    import numpy as np

    from oracle import oracle as O
    from warp_b200 import container as C

    hidden, inter, E, K = cfg["hidden"], cfg["inter"], cfg["E"], cfg["K"]
    rng = np.random.default_rng(cfg["seed"])
    pool = 32
    rec_bytes = C.record_layout(hidden, inter)[5]
    recs = []
    for e in range(pool):
        blocks = [rng.integers(0, 256, C.index_bytes(M, N), dtype=np.uint8)
                  for M, N in ((inter, hidden), (inter, hidden), (hidden, inter))]
        scales = [rng.uniform(0.01, 0.05, n).astype(np.float16).view(np.uint16)
                  for n in (inter, inter, hidden)]
        recs.append(np.frombuffer(C.write_record(0, e, 0, blocks, scales, hidden, inter),
                                  np.uint8).copy())
    books_f16 = rng.uniform(-0.3, 0.3, (9, 256, 8)).astype(np.float16).view(np.uint16)
    books, booksT = C.books_decode(books_f16)
    router = (rng.standard_normal((E, hidden)) * 0.02).astype(np.float32)
    sh = {}
    si = cfg["shared_inter"]
    for k, (M, N) in (("gate", (si, hidden)), ("up", (si, hidden)), ("down", (hidden, si))):
        W = (rng.standard_normal((M, N)) * 0.02).astype(np.float32)
        sh[k] = O.quant_q(W, 32, 4)
    per_tok = K * C.packed_bytes_per_expert(hidden, inter) + 4 * E * hidden + \
        sum(q.size + 2 * s.size for q, s in sh.values())

    use_ref = want_lib == "ref" and O.ref_available()
    if use_ref:
        R = O.ref(0)
        cores = R.ref_threads()
        kind = "reference"
        h = R.ref_moe_new(O._p(booksT), 9, hidden, inter, K)
        logits = np.empty(E, np.float32)
        idx = np.empty(K, np.int32)
        w = np.empty(K, np.float32)
        acc = np.empty((K, hidden), np.float32)
        out = np.empty(hidden, np.float32)
        sout = np.empty(hidden, np.float32)

        def one(x):
            R.ref_matvec_f32(O._p(logits), O._p(router), O._p(x), E, hidden)
            R.ref_qwen_route(O._p(logits), E, K, 1, O._p(idx), O._p(w))
            sel = (ctypes.c_void_p * K)(*[recs[i % pool].ctypes.data for i in idx])
            R.ref_moe_experts(h, ctypes.cast(sel, ctypes.c_void_p), O._p(w), O._p(x),
                              O._p(acc), O._p(out), 0)
            R.ref_shared_expert(h, O._p(sh["gate"][0]), O._p(sh["gate"][1]), O._p(sh["up"][0]),
                                O._p(sh["up"][1]), O._p(sh["down"][0]), O._p(sh["down"][1]),
                                32, 4, O._p(x), O._p(sout))
    else:
        cores = 1
        kind = "port"
        shd = {"gate_w": sh["gate"][0], "gate_s": sh["gate"][1], "up_w": sh["up"][0],
               "up_s": sh["up"][1], "down_w": sh["down"][0], "down_s": sh["down"][1],
               "group": 32, "bits": 4, "inter": si}
        allrecs = [recs[e % pool] for e in range(E)]

        def one(x):
            O.moe_layer(x, hidden, inter, E, K, 1, router, allrecs, booksT, shd)

    def done():
        if use_ref:
            R.ref_moe_free(h)

    return one, per_tok, cores, kind, pool, done


def host_info():
    model = ""
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    model = ln.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"cpu": model, "logical_cpus": os.cpu_count()}


# ------------------------------------------------------------------ main --

def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def run_reference(args, cfg):
    ws, rank, local = dist_env()
    if rank != 0:
        return
    import numpy as np
    one, per_tok, cores, kind, pool, done = cpu_layer(cfg)
    rng = np.random.default_rng(cfg["seed"] + 99)
    xs = rng.standard_normal((64, cfg["hidden"])).astype(np.float32)
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        for l in range(cfg["layers"]):       # one token through the whole stack
            one(xs[(i * cfg["layers"] + l) % 64])
        if i >= args.warmup:
            times.append(time.perf_counter() - t0)
    done()
    sec = sum(times) / len(times)
    tok_s = 1.0 / sec
    gbs = per_tok * cfg["layers"] / sec / 1e9
    sample = (f"one token through the {cfg['layers']}-layer stack per step, each layer "
              f"{cfg['E']} experts aliased over a pool of {pool} distinct records")
    line = {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000.0 / tok_s, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "tokens_per_s": round(tok_s, 3),
        "config": {"workload": cfg["workload"], "hidden": cfg["hidden"], "inter": cfg["inter"],
                   "experts": cfg["E"], "top_k": cfg["K"], "layers": cfg["layers"],
                   "decode_batch": 1, "parallelism": "host cores",
                   "routing": f"softmax top-{cfg['K']} over a plain N(0, 0.02) router (no "
                              "Zipf skew; the routed bytes per token are the same)",
                   "records": f"the {cfg['E']} experts of a layer alias a pool of {pool} "
                              "distinct random records (above the host caches)"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": kind,
                         "sample": sample},
        "host": host_info(),
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def route_stats(routes, layers, ws, T, K, ep_mode=0):
    """Distinct experts per (step, layer) and the rank load balance, from the
    top-k of every layer of every step (routes: per step, per layer [T][K]).
    A route is computed by the rank holding its expert (mode 0) or by rank
    (route index) % ws (mode 1)."""
    import numpy as np
    distinct, owned0, imbalance = [], [], []
    for step in routes:
        d = 0
        for l in range(layers):
            idx = np.asarray(step[l]).reshape(-1)
            d += len(np.unique(idx))
            who = idx % ws if ep_mode == 0 else np.arange(idx.size) % ws
            per_rank = np.bincount(who, minlength=ws)
            owned0.append(per_rank[0])
            imbalance.append(per_rank.max() / max(per_rank.mean(), 1e-9))
        distinct.append(d)
    return (float(np.mean(distinct)), float(np.mean(owned0)), float(np.mean(imbalance)))


def run_warp(args, cfg):
    import math
    import torch
    ws, rank, local = dist_env()
    if ws > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    from warp_b200 import ffi, synth
    lib = ffi.load()
    if not lib.warp_device_ok(local):
        raise SystemExit("bench: this device is not an sm_100 part")
    if ws < cfg.get("min_gpus", 1):
        raise SystemExit(f"bench: {args.config} needs at least {cfg['min_gpus']} GPUs")

    # expert-parallel over the ranks; T decode tokens per step (default 1,
    # the config's decode batch, whatever the GPU count)
    T = args.batch if args.batch > 0 else 1
    ep_size = ws
    # routes dealt over a replicated bank when the whole stack fits one GPU,
    # else experts sharded by id (the split that keeps a larger model resident)
    ep_mode = args.ep_mode if args.ep_mode >= 0 else (1 if stack_bytes(cfg) < 120e9 else 0)
    if ws == 1:
        ep_mode = 0
    model, u = build_model(cfg, device, rank, ep_size, ep_mode)
    stack = Stack(model, cfg["K"], device, T, rank, ep_size, ep_mode)
    H, K = cfg["hidden"], cfg["K"]
    n_tok = args.warmup + args.steps
    # every rank sees the same tokens (the expert-parallel premise)
    if u is not None:
        tokens = synth.zipf_tokens(n_tok, T, H, u, synth.ZIPF_A * math.sqrt(H), 1234, device=device)
    else:
        tokens = torch.randn(n_tok, T, H, generator=torch.Generator().manual_seed(1234))
        tokens = tokens.to(device)

    # launches per step (eager, counted by the library)
    c0 = lib.warp_launch_count()
    stack.h.copy_(tokens[0])
    stack.step()
    torch.cuda.synchronize()
    launches_per_step = lib.warp_launch_count() - c0
    for moe in stack.moes:
        moe.status()

    # per-phase timing: the same step captured with CUDA events recorded (as
    # graph nodes) around every phase of every layer; device times
    for moe in stack.moes:
        moe.set_timing(True)
    stack.capture()
    n_prof = min(args.steps, 20)
    for i in range(n_prof):
        stack.h.copy_(tokens[i % n_tok])
        stack.replay()
        stack.collect()
    torch.cuda.synchronize()
    phase_ms, forwards = {}, 0
    for moe in stack.moes:
        n, ms_ = moe.timings()
        forwards += n
        for k, v in ms_.items():
            phase_ms[k] = phase_ms.get(k, 0.0) + v
    stack.release()                      # release the timing graphs before their events
    torch.cuda.synchronize()
    for moe in stack.moes:
        moe.set_timing(False)

    stack.capture()
    for i in range(args.warmup):
        stack.h.copy_(tokens[i])
        stack.replay()
    torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
    t0.record()
    for i in range(args.steps):
        stack.h.copy_(tokens[args.warmup + i])
        stack.replay()
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / args.steps

    # the same replay held for at least a second of device time, so the clock
    # sampler sees the GPU under sustained load (reported beside `value`,
    # which stays the K-step figure)
    n_sus = max(args.steps, int(math.ceil(1000.0 * args.sustain_s / max(ms, 1e-3))))
    if ws > 1:
        t = torch.tensor([n_sus], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        n_sus = int(t[0])
        torch.distributed.barrier()
    s0 = torch.cuda.Event(enable_timing=True)
    s1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s0.record()
    for i in range(n_sus):
        stack.h.copy_(tokens[args.warmup + i % args.steps])
        stack.replay()
    s1.record()
    torch.cuda.synchronize()
    ms_sus = s0.elapsed_time(s1) / n_sus

    # end to end: host tokens in pinned memory -> device -> step -> host out
    hin = torch.empty(T, H, pin_memory=True)
    hout = torch.empty(T, H, pin_memory=True)
    host_tokens = tokens.cpu()
    if ws > 1:
        torch.distributed.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for i in range(args.steps):
        hin.copy_(host_tokens[args.warmup + i])
        stack.h.copy_(hin, non_blocking=True)
        stack.replay()
        hout.copy_(stack.out, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    ms_e2e = e0.elapsed_time(e1) / args.steps
    clk = clocks.stop()

    # the routes the timed steps took (same tokens, eager, after timing)
    routes = []
    for i in range(args.steps):
        stack.h.copy_(tokens[args.warmup + i])
        r = []
        stack.step(routes=r)
        routes.append(r)
    torch.cuda.synchronize()
    distinct, owned0, imbalance = route_stats(routes, cfg["layers"], ws, T, K, ep_mode)

    if ws > 1:
        t = torch.tensor([ms, ms_e2e, ms_sus], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, ms_e2e, ms_sus = float(t[0]), float(t[1]), float(t[2])

    # packed bytes a step reads, whole job: the distinct expert records the
    # step's routes touch, each rank's router, and the shared expert once per
    # rank that computes it for some token
    lay = model[0]
    rec_b = lay.bank.packed_bytes_per_expert()
    sh_b = sum(lay.shared[k + "_w"].numel() + 2 * lay.shared[k + "_s"].numel()
               for k in ("gate", "up", "down"))
    rt_b = 4 * lay.router.numel()
    # the shared expert is read once per step (its rows and column blocks
    # are split over the ranks), the router by every rank
    per_step_bytes = distinct * rec_b + cfg["layers"] * (sh_b + ws * rt_b)
    gbs = per_step_bytes / (ms / 1e3) / 1e9
    gbs_e2e = per_step_bytes / (ms_e2e / 1e3) / 1e9
    tok_s = T * 1000.0 / ms
    peak, peak_kind = load_peaks()

    inter = cfg["inter"]
    # rank 0's gate/up launch: its owned routes of a layer, on average
    gu_bytes = owned0 * 2 * inter * H * 3 / 8
    dn_bytes = owned0 * H * inter * 3 / 8
    gu_ms = phase_ms["gate_up_gather"] / forwards
    dn_ms = phase_ms["down_gather"] / forwards
    gu_gbs = gu_bytes / (gu_ms / 1e3) / 1e9
    dn_gbs = dn_bytes / (dn_ms / 1e3) / 1e9
    traffic = None
    tp = os.path.join(ROOT, "profiles", "vq_gather_traffic.json")
    if os.path.exists(tp) and ws == 1 and T == 1:
        with open(tp) as f:
            tj = json.load(f)
        if tj.get("config") == args.config:
            traffic = tj.get("gate_up_bytes_per_launch")

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        gbs_c, tok_c, cores, kind, sample, _ = cpu_reference(cfg, seconds=args.cpu_seconds)
        cpu = {"value": round(gbs_c, 3), "unit": "GB/s", "cores": cores, "kind": kind,
               "sample": sample, "tokens_per_s": round(tok_c, 3), "host": host_info()}

    if rank == 0:
        par = "single GPU" if ws == 1 else (
            f"ep{ws} (" + ("routes dealt over a bank replicated on every GPU" if ep_mode == 1
                           else "experts sharded by id") +
            "; shared expert split in column blocks; NCCL slot all-reduce in the step graph)")
        routing = (f"softmax top-{K}; Zipf({cfg['zipf']}) skew of the top-1 expert over a "
                   "random popularity order" if cfg.get("zipf") else f"softmax top-{K}")
        line = {
            "metric": METRIC, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "strong" if ws > 1 and args.batch <= 0 else "weak",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random VQ3R codes, N(0,0.02) Q4 shared expert and router)",
            "tokens_per_s": round(tok_s, 2),
            "hbm_frac": round(gbs / ws / peak, 4),
            "config": {"workload": cfg["workload"], "hidden": H, "inter": inter,
                       "experts": cfg["E"], "top_k": K, "layers": cfg["layers"],
                       "decode_batch": T, "shared": "Q4 g32", "routing": routing,
                       "parallelism": par,
                       "distinct_experts_per_step": round(distinct, 2),
                       "rank_load_imbalance": round(imbalance, 3),
                       "l2": "inputs larger than L2 (%.2f GB of weights per step)"
                             % (per_step_bytes / 1e9)},
            "roofline": {"bound": "hbm", "kernel": "vq_gather (gate/up)",
                         "achieved": round(gu_gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gu_gbs / peak, 4), "traffic": traffic,
                         "peak_source": peak_kind,
                         "launch_ms": round(gu_ms, 5), "bytes_per_launch": int(gu_bytes),
                         "down_gather": {"achieved": round(dn_gbs, 1),
                                         "launch_ms": round(dn_ms, 5),
                                         "bytes_per_launch": int(dn_bytes)},
                         "phase_ms_per_layer": {k: round(v / forwards, 5)
                                                for k, v in phase_ms.items()}},
            "e2e": {"value": round(gbs_e2e, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": T * H * 4, "d2h_bytes_per_step": T * H * 4,
                    "ms_per_step": round(ms_e2e, 4)},
            "gpu_launches": int(launches_per_step * args.steps),
            "clocks": clk,
            "sustained": {"steps": n_sus, "ms_per_step": round(ms_sus, 4),
                          "seconds": round(n_sus * ms_sus / 1e3, 2),
                          "value": round(per_step_bytes / (ms_sus / 1e3) / 1e9, 2),
                          "note": "the timed step replayed for >= 1 s with clocks "
                                  "sampled throughout"},
        }
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    stack.release()
    torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def run_trunk(args, cfg):
    """Config 2: warp_mvq_matvec on Q4 g32 and Q8 per-row weights (N(0, 0.02),
    quantized as convert.py does) of 2304x2304, 7168x7168 and 7168x18432
    (out x in), bf16 activations N(0, 1) at batch 1, 4, 16 and 64 (the engine's
    prefill chunk), fp32 output.
    Each timed iteration reads another copy of the weights (copies total
    well above L2), so every byte comes from HBM.  One JSON line; value = the
    7168x18432 Q4 batch-1 case."""
    import math
    import torch
    from warp_b200 import ffi, ops, synth
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    lib = ffi.load()
    gen = torch.Generator(device=device).manual_seed(cfg["seed"])
    peak, pk = load_peaks()
    cases = []
    launches = 0
    for bits in (4, 8):
        for out, inn in ((2304, 2304), (7168, 7168), (7168, 18432)):
            group = 32 if bits == 4 else inn
            W = torch.randn(out, inn, generator=gen, device=device) * 0.02
            q, sc = synth.quantize_q(W, group, bits)
            del W
            nbytes = q.numel() + 2 * sc.numel()
            ncopy = max(2, math.ceil(320e6 / nbytes))
            qs = [q.clone() for _ in range(ncopy)]
            ss = [sc.clone() for _ in range(ncopy)]
            for batch in (1, 4, 16, 64):
                X = torch.randn(batch, inn, generator=gen, device=device).bfloat16()
                Y = torch.empty(batch, out, device=device)
                rb = (inn + group - 1) // group * group * bits // 8
                st = ctypes_stream()

                def call(i):
                    ffi.check(lib.warp_mvq_matvec(ptr(qs[i % ncopy]), ptr(ss[i % ncopy]), ptr(X), 1,
                                                  ptr(Y), batch, out, inn, group, bits, rb, st))
                for i in range(args.warmup):
                    call(i)
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                c0 = lib.warp_launch_count()
                e0.record()
                for i in range(args.steps):
                    call(args.warmup + i)
                e1.record()
                torch.cuda.synchronize()
                launches += lib.warp_launch_count() - c0
                us = e0.elapsed_time(e1) * 1e3 / args.steps
                gbs = nbytes / (us * 1e-6) / 1e9
                cases.append({"fmt": f"Q{bits}" + (" g32" if bits == 4 else " per-row"),
                              "shape": f"{out}x{inn}", "batch": batch, "us": round(us, 2),
                              "packed_gbs": round(gbs, 1), "hbm_frac": round(gbs / peak, 4)})
            del qs, ss
            torch.cuda.empty_cache()
    head = [c for c in cases if c["fmt"] == "Q4 g32" and c["shape"] == "7168x18432"
            and c["batch"] == 1][0]
    line = {"metric": "trunk dequant-matvec packed GB/s (config 2)", "value": head["packed_gbs"],
            "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "dtype": "Q4/Q8 weights, bf16 x, f32 accumulate",
            "data": "synthetic N(0,0.02) weights, N(0,1) activations",
            "config": {"workload": cfg["workload"], "l2": "weight copies rotated, > 2x L2"},
            "roofline": {"bound": "hbm", "kernel": "mvq_kernel", "achieved": head["packed_gbs"],
                         "peak": peak, "unit": "GB/s", "frac": head["hbm_frac"],
                         "peak_source": pk},
            "cases": cases, "gpu_launches": int(launches)}
    print(json.dumps(line), flush=True)


def ptr(t):
    import ctypes
    return ctypes.c_void_p(t.data_ptr())


def ctypes_stream():
    import ctypes
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def run_prefill(args, cfg):
    """Prefill of T tokens per step through the config's stack on one GPU:
    per layer h = h + MoE(RMSNorm(h)) with warp_moe_layer_prefill (the
    tensor-core grouped GEMMs).  Prints one JSON line with tokens/s, packed
    GB/s over the distinct expert records the step's routes touch, and the
    tensor FLOP/s of the gate/up GEMMs against the dense 16-bit peak."""
    import math
    import numpy as np
    import torch
    ws, rank, local = dist_env()
    if ws > 1:
        raise SystemExit("bench --prefill runs on one GPU")
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    from warp_b200 import ffi, ops, synth
    lib = ffi.load()
    T, K, H, E = args.prefill, cfg["K"], cfg["hidden"], cfg["E"]
    inter, si, L = cfg["inter"], cfg["shared_inter"], cfg["layers"]
    model, u = build_model(cfg, device)
    moes = [lay.moe(K, max_tokens=1, prefill_tokens=T) for lay in model]
    n_tok = args.warmup + args.steps
    if u is not None:
        tokens = synth.zipf_tokens(n_tok, T, H, u, synth.ZIPF_A * math.sqrt(H), 4321, device=device)
    else:
        tokens = torch.randn(n_tok, T, H, generator=torch.Generator().manual_seed(4321))
        tokens = tokens.to(device)
    h = torch.zeros(T, H, device=device)
    xn = torch.zeros(T, H, device=device)
    bufs = [torch.zeros(T, H, device=device) for _ in range(2)]

    def step(routes=None):
        cur = h
        for i, m in enumerate(moes):
            ops.rmsnorm(cur, out=xn)
            r = m.prefill(xn, residual=cur, out=bufs[i % 2], want_route=routes is not None)
            if routes is not None:
                routes.append(r[1].cpu())
            cur = bufs[i % 2]
        return cur

    def capture():
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step()
        return g

    c0 = lib.warp_launch_count()
    h.copy_(tokens[0])
    step()
    torch.cuda.synchronize()
    launches = lib.warp_launch_count() - c0
    for m in moes:
        m.status()
    for m in moes:
        m.set_timing(True)
    g = capture()
    for i in range(min(args.steps, 10)):
        h.copy_(tokens[i % n_tok])
        g.replay()
        for m in moes:
            m.collect()
    torch.cuda.synchronize()
    phase, fw = {}, 0
    for m in moes:
        n, ms_ = m.timings()
        fw += n
        for k, v in ms_.items():
            phase[k] = phase.get(k, 0.0) + v
    g = None
    torch.cuda.synchronize()
    for m in moes:
        m.set_timing(False)
    g = capture()
    for i in range(args.warmup):
        h.copy_(tokens[i])
        g.replay()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for i in range(args.steps):
        h.copy_(tokens[args.warmup + i])
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    clk = clocks.stop()
    g = None
    distinct = []
    for i in range(min(args.steps, 4)):
        h.copy_(tokens[args.warmup + i])
        r = []
        step(routes=r)
        distinct.append(sum(len(np.unique(x.numpy())) for x in r))
    dist_mean = float(np.mean(distinct))
    lay = model[0]
    rec_b = lay.bank.packed_bytes_per_expert()
    sh_b = sum(lay.shared[k + "_w"].numel() + 2 * lay.shared[k + "_s"].numel()
               for k in ("gate", "up", "down"))
    rt_b = 4 * lay.router.numel()
    step_bytes = dist_mean * rec_b + L * (sh_b + rt_b)
    routed_flops = 2.0 * T * K * 3 * inter * H
    step_flops = L * (routed_flops + 2.0 * T * 3 * si * H + 2.0 * T * E * H)
    per = {k: v / fw for k, v in phase.items()}
    gu_ms = per["gate_up_gather"]
    gu_flops = 2.0 * T * K * 2 * inter * H
    tpk, tkind = load_peaks("bf16_tflops")
    hpk, hkind = load_peaks("hbm_gbs")
    line = {
        "metric": "expert-FFN prefill tokens/s (tcgen05 grouped GEMMs)", "value": round(T * 1000.0 / ms, 1),
        "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "dtype": "f16 operands, f32 accumulate",
        "data": "synthetic", "packed_gbs": round(step_bytes / (ms / 1e3) / 1e9, 1),
        "tflops": round(step_flops / (ms / 1e3) / 1e12, 1),
        "config": {"workload": cfg["workload"] + f" prefill {T} tokens", "hidden": H,
                   "inter": inter, "experts": E, "top_k": K, "layers": L, "prefill_tokens": T,
                   "distinct_experts_per_step": dist_mean},
        "roofline": {"bound": "tensor", "kernel": "pf_gemm_kernel (routed gate/up + SwiGLU)",
                     "achieved": round(gu_flops / (gu_ms / 1e3) / 1e12, 1), "peak": tpk,
                     "unit": "TFLOP/s", "frac": round(gu_flops / (gu_ms / 1e3) / 1e12 / tpk, 4),
                     "peak_source": tkind, "launch_ms": round(gu_ms, 4),
                     "phase_ms_per_layer": {k: round(v, 4) for k, v in per.items()},
                     "hbm_gbs_gate_up": round(dist_mean / L * rec_b * 2 / 3 / (gu_ms / 1e3) / 1e9, 1),
                     "hbm_peak": hpk},
        "gpu_launches": int(launches * args.steps), "clocks": clk,
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="warp", choices=("warp", "reference"))
    ap.add_argument("--config", default="cfg4", choices=sorted(CONFIGS))
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--ep-mode", type=int, default=-1,
                    help="N > 1: 0 experts sharded by id, 1 routes dealt over a replicated "
                         "bank (default: 1 when the stack fits one GPU)")
    ap.add_argument("--sustain-s", type=float, default=1.0,
                    help="seconds of device time the sustained loop runs (0: K steps)")
    ap.add_argument("--layers", type=int, default=0,
                    help="override the config's layer count (profiling runs)")
    ap.add_argument("--batch", type=int, default=0,
                    help="decode tokens per step (default: one per GPU)")
    ap.add_argument("--prefill", type=int, default=0,
                    help="time prefill of this many tokens per step instead of decode")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    cfg = dict(CONFIGS[args.config])
    if args.layers > 0:
        cfg["layers"] = args.layers
        cfg["workload"] += f" [{args.layers} layers]"
    if args.impl == "reference":
        run_reference(args, cfg)
    elif cfg.get("trunk"):
        run_trunk(args, cfg)
    elif args.prefill > 0:
        run_prefill(args, cfg)
    else:
        run_warp(args, cfg)


if __name__ == "__main__":
    main()
