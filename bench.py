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
    "cfg4": dict(workload="600B-class MoE block decode, batch 1 (BASELINE.json configs[3])",
                 hidden=7168, inter=2048, E=256, K=8, layers=8, shared_inter=2048, seed=2),
    "cfg3": dict(workload="48B-class MoE decode stack, batch 1 (BASELINE.json configs[2])",
                 hidden=2304, inter=1024, E=256, K=8, layers=26, shared_inter=1024, seed=1),
    "cfg1": dict(workload="single MoE layer decode, batch 1 (BASELINE.json configs[0])",
                 hidden=2304, inter=1024, E=32, K=8, layers=1, shared_inter=1024, seed=0),
}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


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

def build_model(cfg, device, layers=None):
    import torch
    from warp_b200 import synth
    L = cfg["layers"] if layers is None else layers
    model = []
    for l in range(L):
        seed = cfg["seed"] * 1000 + l
        bank = synth.random_bank(cfg["E"], cfg["hidden"], cfg["inter"], seed, device=device,
                                 layer=l)
        router = synth.router_matrix(cfg["E"], cfg["hidden"], seed + 500, device=device)
        shared = synth.shared_expert(cfg["hidden"], cfg["shared_inter"], seed + 700,
                                     device=device)
        model.append(synth.SyntheticLayer(bank, router, shared))
    torch.cuda.synchronize()
    return model


class Stack:
    """The decode stack: per layer h = h + MoE(RMSNorm(h))."""

    def __init__(self, model, K, device):
        import torch
        self.model = model
        self.moes = [lay.moe(K) for lay in model]
        H = model[0].bank.hidden
        self.h = torch.zeros(1, H, device=device)
        self.bufs = [torch.zeros(1, H, device=device) for _ in range(2)]
        self.xn = torch.zeros(1, H, device=device)
        self.graph = None

    def step(self):
        from warp_b200 import ops
        cur = self.h
        for i, moe in enumerate(self.moes):
            ops.rmsnorm(cur, out=self.xn)
            nxt = self.bufs[i % 2]
            moe.forward(self.xn, residual=cur, out=nxt)
            cur = nxt
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
            self.out = self.step()
        self.graph = g

    def packed_bytes(self, K):
        return sum(lay.packed_bytes(K) for lay in self.model)


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
                   "decode_batch": 1, "parallelism": "host cores"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": kind,
                         "sample": sample},
        "host": host_info(),
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_warp(args, cfg):
    import torch
    ws, rank, local = dist_env()
    if ws > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    from warp_b200 import ffi
    lib = ffi.load()
    if not lib.warp_device_ok(local):
        raise SystemExit("bench: this device is not an sm_100 part")

    model = build_model(cfg, device)
    stack = Stack(model, cfg["K"], device)
    H = cfg["hidden"]
    gen = torch.Generator(device="cpu").manual_seed(1234 + rank)
    n_tok = args.warmup + args.steps
    tokens = torch.randn(n_tok, 1, H, generator=gen).to(device)

    # launches per step (eager, counted by the library)
    c0 = lib.warp_launch_count()
    stack.h.copy_(tokens[0])
    stack.step()
    torch.cuda.synchronize()
    launches_per_step = lib.warp_launch_count() - c0
    for moe in stack.moes:
        moe.status()

    # per-kernel timing: a second graph of the same step with CUDA events
    # recorded (as graph nodes) around every phase of every layer, replayed
    # on the launching stream; device times, no host in between
    for moe in stack.moes:
        moe.set_timing(True)
    stack.capture()
    n_prof = min(args.steps, 20)
    for i in range(n_prof):
        stack.h.copy_(tokens[i % n_tok])
        stack.graph.replay()
        for moe in stack.moes:
            moe.collect()
    torch.cuda.synchronize()
    phase_ms, forwards = {}, 0
    for moe in stack.moes:
        n, ms = moe.timings()
        forwards += n
        for k, v in ms.items():
            phase_ms[k] = phase_ms.get(k, 0.0) + v
    stack.graph = None                  # release the timing graph before its events
    torch.cuda.synchronize()
    for moe in stack.moes:
        moe.set_timing(False)

    stack.capture()
    for i in range(args.warmup):
        stack.h.copy_(tokens[i])
        stack.graph.replay()
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
        stack.graph.replay()
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / args.steps

    # end to end: host token in pinned memory -> device -> step -> host out
    hin = torch.empty(1, H, pin_memory=True)
    hout = torch.empty(1, H, pin_memory=True)
    host_tokens = tokens.cpu()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for i in range(args.steps):
        hin.copy_(host_tokens[args.warmup + i])
        stack.h.copy_(hin, non_blocking=True)
        stack.graph.replay()
        hout.copy_(stack.out, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    ms_e2e = e0.elapsed_time(e1) / args.steps
    clk = clocks.stop()

    if ws > 1:
        t = torch.tensor([ms, ms_e2e], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, ms_e2e = float(t[0]), float(t[1])

    per_step_bytes = stack.packed_bytes(cfg["K"]) * ws
    gbs = per_step_bytes / (ms / 1e3) / 1e9
    gbs_e2e = per_step_bytes / (ms_e2e / 1e3) / 1e9
    tok_s = ws * 1000.0 / ms
    peak, peak_kind = load_peaks()

    from warp_b200 import container as C
    K, hid, inter = cfg["K"], cfg["hidden"], cfg["inter"]
    gu_bytes = K * 2 * inter * hid * 3 // 8                 # gate+up codes per launch
    dn_bytes = K * hid * inter * 3 // 8
    gu_ms = phase_ms["gate_up_gather"] / forwards
    dn_ms = phase_ms["down_gather"] / forwards
    gu_gbs = gu_bytes / (gu_ms / 1e3) / 1e9
    dn_gbs = dn_bytes / (dn_ms / 1e3) / 1e9
    traffic = None
    tp = os.path.join(ROOT, "profiles", "vq_gather_traffic.json")
    if os.path.exists(tp):
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
        line = {
            "metric": METRIC, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random VQ3R codes, N(0,0.02) Q4 shared expert and router)",
            "tokens_per_s": round(tok_s, 2),
            "hbm_frac": round(gbs / ws / peak, 4),
            "config": {"workload": cfg["workload"], "hidden": hid, "inter": inter,
                       "experts": cfg["E"], "top_k": K, "layers": cfg["layers"],
                       "decode_batch": 1, "shared": "Q4 g32",
                       "parallelism": "replicas" if ws > 1 else "single GPU",
                       "l2": "inputs larger than L2 (%.2f GB of weights per step)"
                             % (per_step_bytes / ws / 1e9)},
            "roofline": {"bound": "hbm", "kernel": "vq_gather (gate/up)",
                         "achieved": round(gu_gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gu_gbs / peak, 4), "traffic": traffic,
                         "peak_source": peak_kind,
                         "launch_ms": round(gu_ms, 5), "bytes_per_launch": gu_bytes,
                         "down_gather": {"achieved": round(dn_gbs, 1),
                                         "launch_ms": round(dn_ms, 5),
                                         "bytes_per_launch": dn_bytes},
                         "phase_ms_per_layer": {k: round(v / forwards, 5)
                                                for k, v in phase_ms.items()}},
            "e2e": {"value": round(gbs_e2e, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": H * 4, "d2h_bytes_per_step": H * 4,
                    "ms_per_step": round(ms_e2e, 4)},
            "gpu_launches": int(launches_per_step * args.steps),
            "clocks": clk,
        }
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    stack.graph = None
    if ws > 1:
        torch.distributed.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="warp", choices=("warp", "reference"))
    ap.add_argument("--config", default="cfg4", choices=sorted(CONFIGS))
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--layers", type=int, default=0,
                    help="override the config's layer count (profiling runs)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    cfg = dict(CONFIGS[args.config])
    if args.layers > 0:
        cfg["layers"] = args.layers
        cfg["workload"] += f" [{args.layers} layers]"
    if args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_warp(args, cfg)


if __name__ == "__main__":
    main()
