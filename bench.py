"""Benchmark of the fused LR-AttnRes depth-routing read, forward + backward.

One step = forward + backward of the LRID read over one batch (BASELINE
config 2: S=9 sources, N=8x2048 tokens per GPU, d=1024, rank 64, 1 head, bf16,
static query ~ N(0, 0.02), logit scale 1/8), plus, at N>1 GPUs, the NCCL
all-reduce of the query gradient. Work is token-sharded: every rank holds its
own 16384-token batch (weak scaling).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0). `value` is whole-job tokens/s with inputs
resident in HBM (the step captured in a CUDA graph, replayed K times; inputs
are 320 MB per rank, larger than the 126 MB L2, so no flush is needed); `e2e`
repeats the step through the public Python API with pinned host buffers and
host<->device copies inside the timed region. `--impl reference` times the CPU
oracle (a double-precision C restatement of the reference's PyTorch path) on
the host cores instead.
"""
import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "lr-attnres_b200"))
sys.path.insert(0, ROOT)

METRIC = "AttnRes fwd+bwd tokens/s and % HBM roofline at 1/2/4/8 B200 vs ref Triton & CPU"
UNIT = "tokens/s"

CONFIGS = {
    # BASELINE config 2 (the metric's configuration)
    "config2": dict(S=9, B=8, T=2048, D=1024, R=64, H=1, scale=1 / 8, query="static"),
    # BASELINE config 3 (gated hybrid query), reported with --config config3
    "config3": dict(S=13, B=16, T=2048, D=2048, R=64, H=4, scale=1 / 4, query="gated"),
    # keys projected from the values in-op (rms_norm(V) @ W_k^T, tcgen05)
    "config4": dict(S=17, B=32, T=4096, D=2048, R=64, H=1, scale=1 / 8, query="static", kv=True),
    # small case for ncu captures (inputs still > L2)
    "small": dict(S=9, B=4, T=2048, D=1024, R=64, H=1, scale=1 / 8, query="static"),
    # config-4 shapes at 8192 tokens for ncu captures of the key-from-value kernels (570 MB of values)
    "small_kv": dict(S=17, B=2, T=4096, D=2048, R=64, H=1, scale=1 / 8, query="static", kv=True),
}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", choices=sorted(CONFIGS), default="config2")
    p.add_argument("--e2e-steps", type=int, default=12)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--profile", action="store_true",
                   help="short run for ncu: warmup + steps eager launches, no e2e/cpu legs")
    return p.parse_args()


def algorithmic_bytes(c, esz=2):
    """Each input read once, each output written once (per token)."""
    S, D, R = c["S"], c["D"], c["R"]
    if c.get("kv"):
        # forward reads V, writes out; backward reads V and g, writes dV (keys stay internal)
        return S * D * esz + D * esz, S * D * esz + D * esz + S * D * esz
    q_tok = R * esz if c["query"] != "static" else 0
    fwd = S * (D + R) * esz + q_tok + D * esz
    bwd = D * esz + S * (D + R) * esz + q_tok + S * (D + R) * esz + q_tok
    return fwd, bwd


# ---------------------------------------------------------------------------
# clocks sampling (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def start(self):
        """Starts nvidia-smi and waits for its first sample, so that sampling
        covers the whole timed region that follows (nvidia-smi can take a
        fraction of a second to start)."""
        self.first = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.first = self.proc.stdout.readline()
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            return None
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        lines = out.strip().splitlines()
        if not lines and self.first:
            lines = [self.first]  # a region shorter than one sampling period
        for line in lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# reference arm: the CPU oracle on the host cores
# ---------------------------------------------------------------------------
def cpu_oracle_rate(c, target_s=12.0, max_tokens=4096):
    """cpu_baseline leg: the oracle's fwd+bwd rate on a bounded token sample."""
    from oracle import oracle

    n = min(max_tokens, c["B"] * c["T"])
    v, k, g, kw = _oracle_inputs(c, n)
    tokens, t0 = 0, time.perf_counter()
    while True:
        oracle.lrid_forward(v, k, c["H"], c["scale"], True, **kw)
        oracle.lrid_backward(v, k, c["H"], c["scale"], True, g, **kw)
        tokens += n
        el = time.perf_counter() - t0
        if el >= target_s:
            break
    return (tokens / el, oracle.num_threads(),
            f"{n} tokens of the workload per call, {tokens} tokens in {el:.1f} s (fp64 C oracle, OpenMP)")


def _oracle_inputs(c, n, seed=0):
    S, D, R, H = c["S"], c["D"], c["R"], c["H"]
    rng = np.random.default_rng(seed)
    v = rng.standard_normal((S, n, D), dtype=np.float32)
    k = rng.standard_normal((S, n, R), dtype=np.float32)
    g = rng.standard_normal((n, D), dtype=np.float32)
    kw = {"query": (rng.standard_normal((H, R // H)) * 0.02).astype(np.float32)}
    if c["query"] == "gated":
        kw.update(gate=np.full(H, 0.1, np.float32),
                  query_dynamic=rng.standard_normal((n, H, R // H), dtype=np.float32))
    return v, k, g, kw


def run_reference(args, c):
    """Reference arm: the CPU oracle (fp64 C restatement of the reference's
    PyTorch path, all host threads) over a token sample of the workload per
    step, sized so that warmup + steps take about a minute."""
    from oracle import oracle

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    H = c["H"]
    v, k, g, kw = _oracle_inputs(c, 256)
    t0 = time.perf_counter()
    oracle.lrid_forward(v, k, H, c["scale"], True, **kw)
    oracle.lrid_backward(v, k, H, c["scale"], True, g, **kw)
    rate = 256 / (time.perf_counter() - t0)
    budget = min(10.0, 60.0 / max(1, args.steps + args.warmup))
    n = int(min(c["B"] * c["T"], max(32, rate * budget)))
    v, k, g, kw = _oracle_inputs(c, n)
    for i in range(args.warmup + args.steps):
        if i == args.warmup:
            t0 = time.perf_counter()
        oracle.lrid_forward(v, k, H, c["scale"], True, **kw)
        oracle.lrid_backward(v, k, H, c["scale"], True, g, **kw)
    el = time.perf_counter() - t0
    value = n * max(1, args.steps) / el
    cores = oracle.num_threads()
    sample = f"{n} of {c['B'] * c['T']} tokens per step, {args.steps} steps in {el:.2f} s (fp64 C oracle, OpenMP {cores} threads)"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * c["B"] * c["T"] / value, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": config_block(c, args),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def profiled_traffic_per_token():
    """DRAM bytes per token of each kernel, from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "lrid_kernels_config2_small.md")
    out = {}
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_token:"):
                _, kernel, value = [x.strip() for x in line.split(":")]
                out[kernel] = float(value)
    except OSError:
        pass
    return out


def config_block(c, args):
    return {
        "workload": f"{args.config}: LRID read fwd+bwd, S={c['S']}, N={c['B']}x{c['T']} tokens per GPU, "
                    f"d={c['D']}, R={c['R']}, H={c['H']}, {c['query']} query, bf16",
        "tokens_per_gpu": c["B"] * c["T"], "global_tokens": c["B"] * c["T"] * args.gpus,
        "parallelism": f"token-sharded x{args.gpus}",
        "l2": "inputs larger than L2 (no flush)",
    }


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def make_inputs(c, device, torch, seed):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    S, B, T, D, R, H = c["S"], c["B"], c["T"], c["D"], c["R"], c["H"]
    bf = torch.bfloat16
    x = {
        "values": [torch.randn(B, T, D, device=device, dtype=bf, generator=g) for _ in range(S)],
        "keys": ([torch.randn(B, T, R, device=device, dtype=bf, generator=g) for _ in range(S)]
                 if not c.get("kv") else None),
        "weight": ((torch.randn(R, D, device=device, generator=g) / D ** 0.5).to(bf) if c.get("kv") else None),
        "query": (torch.randn(H, R // H, device=device, generator=g) * 0.02).to(bf),
        "grad": torch.randn(B, T, D, device=device, dtype=bf, generator=g),
        "gate": None, "qdyn": None,
    }
    if c["query"] == "gated":
        x["gate"] = torch.full((H,), 0.1, device=device, dtype=bf)
        x["qdyn"] = torch.randn(B, T, H, R // H, device=device, dtype=bf, generator=g)
    return x


def main():
    args = parse()
    c = CONFIGS[args.config]
    if args.impl == "reference":
        return run_reference(args, c)

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=device)

    import attnres_b200  # noqa: F401  (registers torch.ops.attnres.*)

    ops = torch.ops.attnres
    x = make_inputs(c, device, torch, seed=1234 + rank)
    H, scale = c["H"], c["scale"]
    gated = c["query"] == "gated"
    q, gate, qdyn = x["query"], x["gate"], x["qdyn"]

    kv = bool(c.get("kv"))

    def fwd():
        if kv:
            return ops.lrid_kv_read(x["values"], x["weight"], q, gate, qdyn, None, H, scale, True, 0, True)
        return ops.lrid_read(x["values"], x["keys"], q, gate, qdyn, None, H, scale, True, 0)

    def bwd(*fo):
        if kv:
            out, inv, keys, vinv, alpha = fo
            r = ops.lrid_kv_read_backward(x["values"], x["weight"], keys, vinv, alpha, q, gate, qdyn, None,
                                          x["grad"], out, inv, H, scale, True, 0, True)
            # (dV, dW, dq, dgate, ...) -> keep dq / dgate at the same positions as the plain read
            return r[0], r[1], r[2], r[3]
        out, inv = fo
        return ops.lrid_read_backward(x["values"], x["keys"], q, gate, qdyn, None, x["grad"], out, inv,
                                      H, scale, True, 0)

    from attnres_b200.sharding import allreduce_param_grads

    def allreduce(dq, dgate):
        # the only cross-GPU step: one bucketed NCCL all-reduce of the summed grads
        if world > 1:
            allreduce_param_grads([dq] + ([dgate] if gated else []) + ([dw] if kv else []))

    stream = torch.cuda.Stream(device)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]

    if args.profile:
        with torch.cuda.stream(stream):
            for _ in range(args.warmup + args.steps):
                bwd(*fwd())
        torch.cuda.synchronize()
        if rank == 0:
            print(json.dumps({"profile_run": True, "config": args.config}), flush=True)
        return

    # ---- capture fwd and bwd as two CUDA graphs (static buffers) ----------
    with torch.cuda.stream(stream):
        for _ in range(3):  # allocator warm-up outside capture
            res = bwd(*fwd())
    torch.cuda.synchronize()
    g_fwd, g_bwd = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_fwd, stream=stream):
        fo = fwd()
    with torch.cuda.graph(g_bwd, stream=stream):
        res = bwd(*fo)
    dq, dgate = res[2], res[3]
    dw = res[1] if kv else None
    torch.cuda.synchronize()

    sampler = ClockSampler(local)
    sampler.start()
    # The gradient all-reduce of step k runs on its own stream, overlapping the
    # forward of step k+1 (which does not read it); the backward of step k+1,
    # which rewrites the gradient buffers, waits for it.
    comm = torch.cuda.Stream(device)
    bwd_done = [torch.cuda.Event() for _ in range(2)]
    comm_done = [torch.cuda.Event() for _ in range(2)]

    def step(i, fe=None, be=None):
        if fe:
            fe[0].record(stream)
        g_fwd.replay()
        if fe:
            fe[1].record(stream)
        if world > 1 and i > 0:
            stream.wait_event(comm_done[(i - 1) % 2])
        if be:
            be[0].record(stream)
        g_bwd.replay()
        if be:
            be[1].record(stream)
        if world > 1:
            bwd_done[i % 2].record(stream)
            comm.wait_event(bwd_done[i % 2])
            with torch.cuda.stream(comm):
                allreduce(dq, dgate)
                comm_done[i % 2].record(comm)

    def drain(last):
        if world > 1:
            stream.wait_event(comm_done[last % 2])

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i)
        drain(args.warmup - 1)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    # per-kernel CUDA-event timing on the launching stream
    fwd_events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(args.steps)]
    bwd_events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(args.steps)]
    with torch.cuda.stream(stream):
        ev[0].record(stream)
        for i in range(args.steps):
            step(i, fwd_events[i], bwd_events[i])
        drain(args.steps - 1)
        ev[1].record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    ms = ev[0].elapsed_time(ev[1]) / args.steps
    fwd_ms = float(np.mean([a.elapsed_time(b) for a, b in fwd_events]))
    bwd_ms = float(np.mean([a.elapsed_time(b) for a, b in bwd_events]))
    t = torch.tensor([ms, fwd_ms, bwd_ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, fwd_ms, bwd_ms = (float(v) for v in t.tolist())

    tokens = c["B"] * c["T"]
    value = tokens * world / (ms * 1e-3)
    fwd_b, bwd_b = algorithmic_bytes(c)
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except Exception:
        pass
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    traffic = profiled_traffic_per_token()
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    bwd_gbs = tokens * bwd_b / (bwd_ms * 1e-3) / 1e9
    fwd_gbs = tokens * fwd_b / (fwd_ms * 1e-3) / 1e9
    step_gbs = tokens * (fwd_b + bwd_b) / (ms * 1e-3) / 1e9

    # ---- e2e: public API, pinned host buffers, copies inside timed region --
    e2e = None
    if args.e2e_steps > 0 and not kv:
        e2e = run_e2e(args, c, x, device, torch, dist, world)

    proj = None
    if kv:
        # the tcgen05 key projection alone, for its TFLOP/s against the tensor peak
        from attnres_b200.ops import _kv_project

        with torch.cuda.stream(stream):
            _kv_project(x["values"], x["weight"], True)
        torch.cuda.synchronize()
        g_proj = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_proj, stream=stream):
            _kv_project(x["values"], x["weight"], True)
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            g_proj.replay()
            p0.record(stream)
            for _ in range(10):
                g_proj.replay()
            p1.record(stream)
        torch.cuda.synchronize()
        pms = p0.elapsed_time(p1) / 10
        flops = 2.0 * c["S"] * tokens * c["D"] * c["R"]
        tpeak = float(peaks.get("bf16_tflops", 1590.0))
        pbytes = c["S"] * tokens * (c["D"] + c["R"]) * 2
        proj = {"kernel": "keyproj_tc_kernel (tcgen05)", "ms": pms, "tflops": flops / pms / 1e9,
                "peak_tflops": tpeak, "frac_tensor": flops / pms / 1e9 / tpeak,
                "gbs": pbytes / pms / 1e6, "frac_hbm": pbytes / pms / 1e6 / hbm}

    # a9: the block-summary op (running block sum + scaled source) on rows of
    # this config, 4x its token count so the four arrays (537 MB at config 2)
    # are far larger than L2
    aux = None
    if not kv:
        xs = torch.randn(4 * c["B"], c["T"], c["D"], device=device, dtype=torch.bfloat16)
        ps = torch.randn_like(xs)
        bsum = torch.ops.attnres.block_summary
        with torch.cuda.stream(stream):
            bsum(ps, xs, None, 0.25)
        torch.cuda.synchronize()
        g_sum = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_sum, stream=stream):
            bsum(ps, xs, None, 0.25)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            for _ in range(3):
                g_sum.replay()
            s0.record(stream)
            for _ in range(20):
                g_sum.replay()
            s1.record(stream)
        torch.cuda.synchronize()
        sms = s0.elapsed_time(s1) / 20
        sbytes = 4 * xs.numel() * 2
        aux = {"block_summary": {"kernel": "summary_fwd_kernel (a9: sum = partial + x, source = sum * c)",
                                 "elements": xs.numel(), "ms": sms, "achieved_gbs": sbytes / sms / 1e6,
                                 "frac": sbytes / sms / 1e6 / hbm, "bytes": sbytes}}
        # cached-logit phase 2 (LRID key, one query) on the same 4x rows: forward
        # and backward, each timed alone
        R = c["R"]
        pk = torch.randn(xs.shape[0], xs.shape[1], R, device=device, dtype=torch.bfloat16)
        q2 = torch.randn(R, device=device, dtype=torch.bfloat16) * 0.1
        lse2 = torch.randn(xs.shape[0], xs.shape[1], device=device)
        p2 = torch.ops.attnres.phase2
        p2b = torch.ops.attnres.phase2_backward

        def p2f():
            return p2(0, ps, pk, None, q2, xs, lse2, c["scale"], True, None, 0.0, False)

        def p2g(o):
            return p2b(0, ps, pk, None, q2, xs, lse2, c["scale"], True, None, 0.0, False, o[0], o[1], ps, True,
                       False)

        with torch.cuda.stream(stream):
            o2 = p2f()
            p2g(o2)
        torch.cuda.synchronize()
        gf, gb = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(gf, stream=stream):
            o2 = p2f()
        with torch.cuda.graph(gb, stream=stream):
            p2g(o2)
        ev2 = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        with torch.cuda.stream(stream):
            for _ in range(3):
                gf.replay()
                gb.replay()
            ev2[0].record(stream)
            for _ in range(10):
                gf.replay()
            ev2[1].record(stream)
            for _ in range(10):
                gb.replay()
            ev2[2].record(stream)
        torch.cuda.synchronize()
        fms, bms = ev2[0].elapsed_time(ev2[1]) / 10, ev2[1].elapsed_time(ev2[2]) / 10
        ntok = xs.shape[0] * xs.shape[1]
        fb = ntok * (3 * c["D"] + R) * 2 + ntok * 4
        bb = ntok * (5 * c["D"] + 2 * R) * 2 + ntok * 8
        aux["phase2"] = {"kernel": "phase2_fwd_kernel / phase2_bwd_kernel (LRID key, key norm)", "tokens": ntok,
                         "fwd_ms": fms, "fwd_frac": fb / fms / 1e6 / hbm, "bwd_ms": bms,
                         "bwd_frac": bb / bms / 1e6 / hbm, "fwd_bytes": fb, "bwd_bytes": bb}
        del xs, ps, pk, o2

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not kv:
        r, cores, sample = cpu_oracle_rate(c, target_s=12.0)
        cpu = {"value": r, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample}

    # per step: forward kernel, backward kernel, fixed-order reduce of dq (+ dgate)
    launches_per_step = 3 + (1 if gated else 0)
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) values/keys/grads, query N(0,0.02))",
            "config": config_block(c, args),
            "roofline": {
                "kernel": ("backward (read backward + projection backward)" if kv else "backward LRID read (lrid_stream_kernel for this row shape)"), "bound": "hbm",
                "achieved": bwd_gbs, "peak": hbm, "unit": "GB/s", "frac": bwd_gbs / hbm,
                "peak_source": f"{peak_src} MEASURED_PEAKS.json hbm_gbs" if peak_src == "measured" else "fallback 6650 GB/s",
                "traffic": (traffic.get("backward", 0) * tokens) if (traffic and args.config == "config2") else None,
                "traffic_source": "ncu dram read+write per token x tokens, profiles/lrid_kernels_config2_small.md",
                "algorithmic_bytes_per_token": bwd_b, "kernel_ms": bwd_ms,
                "forward": {"achieved": fwd_gbs, "frac": fwd_gbs / hbm, "kernel_ms": fwd_ms,
                            "algorithmic_bytes_per_token": fwd_b},
                "step": {"achieved": step_gbs, "frac": step_gbs / hbm},
                "projection": proj,
            },
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
            "aux": aux,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_e2e(args, c, x, device, torch, dist, world):
    """Same step through the public API with host buffers: every step's inputs
    are copied in from pinned host memory, the read runs forward + backward
    with autograd, and out/dV/dK/dq (+ dgate/dq_dynamic) are copied back to
    pinned host memory. Steps are pipelined the way a user overlaps transfers
    with CUDA streams: copy-in of step k+1 (stream h2d), compute of step k
    (current stream) and copy-out of step k-1 (stream d2h) run concurrently,
    with the device input buffers double-buffered. PCIe is full duplex, so the
    step rate is bound by the larger of the two copy directions. The timed
    region runs from the first copy-in to the last copy-out."""
    import attnres_b200 as A

    S = c["S"]
    gated = x["qdyn"] is not None
    host = {
        "values": [v.cpu().pin_memory() for v in x["values"]],
        "keys": [k.cpu().pin_memory() for k in x["keys"]],
        "grad": x["grad"].cpu().pin_memory(),
        "query": x["query"].float().cpu().pin_memory(),
    }
    if gated:
        host["qdyn"] = x["qdyn"].cpu().pin_memory()
        host["gate"] = x["gate"].float().cpu().pin_memory()
    out_host = {
        "out": torch.empty_like(host["grad"]).pin_memory(),
        "dV": [torch.empty_like(v).pin_memory() for v in host["values"]],
        "dK": [torch.empty_like(k).pin_memory() for k in host["keys"]],
        "dq": torch.empty_like(host["query"]).pin_memory(),
    }
    if gated:
        out_host["dqd"] = torch.empty_like(host["qdyn"]).pin_memory()
        out_host["dgate"] = torch.empty_like(host["gate"]).pin_memory()

    def flat(h):
        return [*h["values"], *h["keys"], h["grad"], h["query"]] + ([h["qdyn"], h["gate"]] if gated else [])

    h2d = sum(t.numel() * t.element_size() for t in flat(host))
    d2h = sum(t.numel() * t.element_size() for t in
              [out_host["out"], *out_host["dV"], *out_host["dK"], out_host["dq"]] +
              ([out_host["dqd"], out_host["dgate"]] if gated else []))
    dev = [{k: ([torch.empty_like(t, device=device) for t in v] if isinstance(v, list)
                else torch.empty_like(v, device=device)) for k, v in host.items()} for _ in range(2)]
    comp = torch.cuda.current_stream(device)
    h2d_s, d2h_s = torch.cuda.Stream(device), torch.cuda.Stream(device)

    def run(nsteps, e0=None, e1=None):
        done = []
        if e0 is not None:
            e0.record(h2d_s)
        for k in range(nsteps):
            b = dev[k % 2]
            with torch.cuda.stream(h2d_s):
                if k >= 2:
                    h2d_s.wait_event(done[k - 2])  # step k-2 has finished reading this buffer set
                for d_t, h_t in zip(flat(b), flat(host)):
                    d_t.copy_(h_t, non_blocking=True)
                ready = torch.cuda.Event()
                ready.record(h2d_s)
            comp.wait_event(ready)
            vs = [t.detach().requires_grad_(True) for t in b["values"]]
            ks = [t.detach().requires_grad_(True) for t in b["keys"]]
            q = b["query"].detach().requires_grad_(True)
            if gated:
                qd = b["qdyn"].detach().requires_grad_(True)
                gt = b["gate"].detach().requires_grad_(True)
                out = A.lrid_attention_residual_read_gated(vs, ks, q, gt, qd, c["H"], c["scale"], True)
            else:
                out = A.lrid_attention_residual_read(vs, ks, q, c["H"], c["scale"], True)
            out.backward(b["grad"])
            if world > 1:
                dist.all_reduce(q.grad)
            ev = torch.cuda.Event()
            ev.record(comp)
            done.append(ev)
            results = [(out_host["out"], out.detach()), (out_host["dq"], q.grad)]
            results += [(out_host["dV"][i], vs[i].grad) for i in range(S)]
            results += [(out_host["dK"][i], ks[i].grad) for i in range(S)]
            if gated:
                results += [(out_host["dqd"], qd.grad), (out_host["dgate"], gt.grad)]
            with torch.cuda.stream(d2h_s):
                d2h_s.wait_event(ev)
                for h_t, d_t in results:
                    d_t.record_stream(d2h_s)  # the allocator keeps it until the copy is done
                    h_t.copy_(d_t, non_blocking=True)
        comp.wait_stream(d2h_s)
        comp.wait_stream(h2d_s)
        if e1 is not None:
            e1.record(comp)

    run(3)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    run(args.e2e_steps, e0, e1)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.e2e_steps
    t = torch.tensor([ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    return {"value": c["B"] * c["T"] * world / (ms * 1e-3), "unit": UNIT, "ms_per_step": ms,
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "pipelined": "copy-in k+1 | compute k | copy-out k-1 on three streams"}


if __name__ == "__main__":
    main()
