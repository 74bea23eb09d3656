"""Verify-step benchmark (driver contract: one JSON line from rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
                    [--workload verify|accept|q4gemm|attn|c1] [--case c5|c3]

Default workload: the north-star path, BASELINE config 5 -- one speculative
verify step of a Llama-3-70B-shape q4_0 target (80 layers, hidden 8192, GQA
64/8, FFN 28672, vocab 128256) over B=64 sequences with a 32-node draft tree
each and 4096 tokens of context in 16-token fp16 KV pages: the target forward
over all 2048 tree nodes, greedy tree acceptance and the KV commit of the
accepted paths, through velo_cuda_verify_step.  Under torchrun the N ranks are
one tensor-parallel group over the same batch ("scaling": "strong").

value  = accepted tokens/s = sum_b (accepted_len_b + 1) per step / device time
         of the step (CUDA events on the context stream, max over ranks);
e2e    = the same metric through the host-buffer C ABI call (inputs copied
         from pinned memory, results copied back, every step), wall clock;
roofline: the dominant kernel (the w1/w3 SwiGLU q4_0 GEMM) -- its algorithmic
         FLOPs per launch over its measured duration inside the step, against
         the measured sustained bf16 peak -- plus the whole step against its
         floor (GEMM FLOPs at peak + KV bytes at HBM bandwidth);
cpu_baseline: the CPU port of llama_cpu.rs (oracle/) timed on this host at
         N=1 and extrapolated to the step.

--workload accept is BASELINE config 2 (the acceptance microbench; replicas
under torchrun, "scaling": "weak"); q4gemm / attn / c1 time single kernels or
config 1.
"""
import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "velo-core_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import numpy as np  # noqa: E402

BASELINE_METRIC = "accepted tokens/sec & µs per verify step (device-timed) at 1/2/4/8 B200"
HBM_FALLBACK_GBS = 6650.0


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return HBM_FALLBACK_GBS, "fallback"


def load_traffic(name):
    """Per-launch DRAM bytes of the dominant kernel from a committed ncu
    summary (profiles/<name>.json), or None."""
    try:
        with open(os.path.join(ROOT, "profiles", name + ".json")) as f:
            return json.load(f).get("dram_bytes_per_launch")
    except Exception:
        return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    def __init__(self, device_index, period=0.02):
        self.samples = []
        self.period = period
        self.idx = device_index
        self._stop = threading.Event()
        self._t = None
        self.max_mhz = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None
            return self
        self._sample()
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def _sample(self):
        nv = self._nv
        try:
            mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
            reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            self.samples.append((mhz, reasons))
        except Exception:
            pass

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(self.period)

    def __exit__(self, *a):
        if self._nv is None:
            return
        self._stop.set()
        if self._t:
            self._t.join()
        self._sample()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        nv = self._nv
        names = {
            "gpu_idle": getattr(nv, "nvmlClocksEventReasonGpuIdle", 0x1),
            "sw_power_cap": getattr(nv, "nvmlClocksEventReasonSwPowerCap", 0x4),
            "hw_slowdown": getattr(nv, "nvmlClocksEventReasonHwSlowdown", 0x8),
            "sw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
            "hw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
            "hw_power_brake_slowdown": getattr(nv, "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80),
        }
        seen = set()
        for _, r in self.samples:
            for n, bit in names.items():
                if r & bit and n != "gpu_idle":
                    seen.add(n)
        return {"sm_mhz": statistics.median(m for m, _ in self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": sorted(seen),
                "samples": len(self.samples)}


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def accepted_tokens(acc):
    return int(np.sum(acc.astype(np.int64) + 1))


# ---------------------------------------------------------------- reference arm
def run_reference(args):
    """CPU implementation of the same step (the oracle port of the reference's
    CPU path + the acceptance spec) on this host's cores."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    import vo
    import synthetic
    threads = os.cpu_count() or 1
    B, k, V, T = 64, 8, 32000, 0.8
    tgt, drf, tok, u = synthetic.acceptance_inputs(B, k, V, T)
    # size each step so the whole run stays within ~2 minutes
    t0 = time.perf_counter()
    vo.accept(tgt[:8], drf[:8], tok[:8], u[:8], T, n_threads=threads)
    per_seq = (time.perf_counter() - t0) / 8
    budget = 120.0 / max(1, args.steps + args.warmup)
    bs = int(max(1, min(B, budget / max(per_seq, 1e-9))))
    toks, secs = 0, 0.0
    for s in range(args.warmup + args.steps):
        lo = (s * bs) % B
        idx = np.arange(lo, lo + bs) % B
        t0 = time.perf_counter()
        acc, _ = vo.accept(tgt[idx], drf[idx], tok[idx], u[idx], T, n_threads=threads)
        dt = time.perf_counter() - t0
        if s >= args.warmup:
            toks += accepted_tokens(acc)
            secs += dt
    value = toks / secs
    line = {
        "impl": "reference", "metric": BASELINE_METRIC, "value": value,
        "unit": "accepted tokens/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * secs / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded Philox, BASELINE config 2 distributions)",
        "config": {"workload": "acceptance microbench (BASELINE config 2)", "B": B, "k": k,
                   "V": V, "temperature": T, "parallelism": "replicas"},
        "cpu_baseline": {"value": value, "unit": "accepted tokens/s", "cores": threads,
                         "kind": "port",
                         "sample": f"{bs} of {B} sequences per step (k=8, V=32000), "
                                   f"{threads} threads over sequences"},
        "e2e": {"value": value, "unit": "accepted tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- CUDA arm
def run_cuda(args):
    import torch
    import torch.distributed as dist
    import synthetic
    import velo_cuda

    ws, rank, local = dist_env()
    if args.gpus != ws and ws > 1:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {ws}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    B, k, V, T = 64, 8, 32000, 0.8
    n_sets = 2
    sets = []
    for sidx in range(n_sets):
        tgt, drf, tok, u = synthetic.acceptance_inputs(B, k, V, T, seed=rank * 16 + sidx)
        sets.append(tuple(torch.from_numpy(a).to(dev) for a in
                          (tgt, drf, tok.view(np.int32), u)))
    acc = torch.empty(B, dtype=torch.int32, device=dev)
    bonus = torch.empty(B, dtype=torch.int32, device=dev)
    ctx = velo_cuda.Context(device=local)
    # a real (non-default) stream shared by torch and the context, so the
    # CUDA events below bracket exactly the launches of the timed steps
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)

    def step(i):
        t, d, tk, uu = sets[i % n_sets]
        ctx.accept_device(t, d, tk, uu, T, acc, bonus)

    # accepted tokens per step of each input set (deterministic)
    tok_per_set = []
    for sidx in range(n_sets):
        step(sidx)
        torch.cuda.synchronize()
        tok_per_set.append(accepted_tokens(acc.cpu().numpy()))
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        start.record(stream)
        for i in range(args.steps):
            step(i)
        end.record(stream)
        torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    ms = start.elapsed_time(end)
    toks = sum(tok_per_set[i % n_sets] for i in range(args.steps))
    if ws > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        tt = torch.tensor([toks], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.SUM)
        toks = float(tt.item())
    ms_per_step = ms / args.steps
    value = toks / (ms / 1e3)

    # ---- e2e through the host-buffer C ABI (pinned host memory) ----------
    host = []
    for sidx in range(n_sets):
        hs = []
        for a in sets[sidx]:
            h = torch.empty(a.shape, dtype=a.dtype, pin_memory=True)
            h.copy_(a)
            hs.append(h.numpy())
        host.append(hs)
    ctx.set_stream(None)
    e2e_steps = max(3, min(args.steps, 50))
    for i in range(2):
        t, d, tk, uu = host[i % n_sets]
        ctx.accept(t, d, tk.view(np.uint32), uu, T)
    if ws > 1:
        dist.barrier()
    t0 = time.perf_counter()
    e2e_toks = 0
    for i in range(e2e_steps):
        t, d, tk, uu = host[i % n_sets]
        a, _ = ctx.accept(t, d, tk.view(np.uint32), uu, T)
        e2e_toks += accepted_tokens(a)
    e2e_s = time.perf_counter() - t0
    if ws > 1:
        t = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
        tt = torch.tensor([e2e_toks], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.SUM)
        e2e_toks = float(tt.item())
    h2d = sum(x.nbytes for x in host[0])
    d2h = 2 * B * 4

    line = None
    if rank == 0:
        peak, peak_kind = load_peaks()
        alg_bytes = B * V * 4 * ((k + 1) + k)  # every logit read once
        achieved = alg_bytes / (ms_per_step * 1e-3) / 1e9
        clocks = clk.summary()
        line = {
            "metric": BASELINE_METRIC, "value": value, "unit": "accepted tokens/s",
            "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_per_step, "us_per_step": ms_per_step * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded Philox, BASELINE config 2 distributions)",
            "config": {"workload": "acceptance microbench (BASELINE config 2)", "B": B, "k": k,
                       "V": V, "temperature": T,
                       "l2": "2 alternating input sets of 139 MB (> 126 MB L2)",
                       "parallelism": f"replicas x{ws} (sequences sharded, no collective)"},
            "accepted_per_step": toks / args.steps / ws,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": load_traffic("accept_c2"),
                         "algorithmic_bytes": alg_bytes, "kernel": "accept_stream_kernel<false> + accept_finish_kernel<false>"},
            "clocks": clocks,
            "e2e": {"value": e2e_toks / e2e_s, "unit": "accepted tokens/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": e2e_steps, "ms_per_step": 1e3 * e2e_s / e2e_steps},
            "gpu_launches": 2 * args.steps,  # stream + finish kernels per step
        }
    ctx.close()
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- tree acceptance
TREE_C3 = [-1, 0, 0, 0, 0, 1, 1, 2, 2, 3, 3, 4, 4, 5, 5, 6]


def tree_walk_rows(par, plen, path):
    """Vocabulary rows the tree walk reads per sequence (the spec's passes):
    per visited node its target row, plus its draft row when it has
    children; two rows per rejected child (the residual pass); one more row
    pass for the draw when the final distribution is p (leaf, or no
    rejection)."""
    rows = 0
    N = len(par)
    for i in range(plen):
        v = path[i]
        kids = [c for c in range(N) if par[c] == v]
        rows += 1 + (1 if kids else 0)
        nxt = path[i + 1] if i + 1 < plen else None
        rej = sum(1 for c in kids if nxt is None or c < nxt)
        rows += 2 * rej
        if nxt is None and rej == 0:
            rows += 1
    return rows


def run_accept_tree(args):
    """Rejection sampling over config-3-shaped draft trees (16 nodes,
    branching 4,2,2 breadth-first), B=64, V=32000, T=0.8, target ~ N(0,2^2),
    draft = target + N(0,0.5^2), children drawn from their parent's draft
    distribution: one velo_cuda_accept_tree_device launch per step."""
    import torch
    import velo_cuda
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    B, V, T = 64, 32000, 0.8
    N = len(TREE_C3)
    par = np.tile(np.array(TREE_C3, np.int32), (B, 1))
    sets = []
    for sidx in range(2):  # two input sets of 2 x 64 x 16 x 32000 x 4 B = 262 MB (> L2)
        g = np.random.Generator(np.random.Philox(key=100 + sidx))
        tgt = g.normal(0, 2.0, (B, N, V)).astype(np.float32)
        drf = (tgt[:, :N - 1] + g.normal(0, 0.5, (B, N - 1, V))).astype(np.float32)
        tok = np.zeros((B, N), np.uint32)
        import synthetic
        for b in range(B):
            c = np.cumsum(synthetic.softmax64(drf[b] / T), axis=-1)
            for n in range(1, N):
                tok[b, n] = min(int((c[par[b, n]] < g.random()).sum()), V - 1)
        u = g.random((B, N)).astype(np.float32)
        sets.append((tgt, drf, tok, u))
    ctx = velo_cuda.Context(device=0)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    dsets = [tuple(torch.from_numpy(np.ascontiguousarray(a)).to(dev) for a in
                   (t, d, k.view(np.int32), u)) for t, d, k, u in sets]
    dpar = torch.from_numpy(par).to(dev)
    path = torch.empty((B, N), dtype=torch.int32, device=dev)
    plen = torch.empty(B, dtype=torch.int32, device=dev)
    bonus = torch.empty(B, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()

    def step(i):
        t, d, k, u = dsets[i % 2]
        ctx.accept_tree_device(t, d, k, dpar, u, T, path, plen, bonus)

    toks, rows = [], []
    for i in range(2):
        step(i)
        torch.cuda.synchronize()
        pl, pa = plen.cpu().numpy(), path.cpu().numpy()
        toks.append(int(pl.sum()))  # accepted nodes + bonus = path_len per sequence
        rows.append(sum(tree_walk_rows(par[b], int(pl[b]), pa[b]) for b in range(B)))
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        e0.record(stream)
        for i in range(args.steps):
            step(i)
        e1.record(stream)
        torch.cuda.synchronize()
    ctx.sync()
    ms = e0.elapsed_time(e1) / args.steps
    tok_step = sum(toks[i % 2] for i in range(args.steps)) / args.steps
    row_step = sum(rows[i % 2] for i in range(args.steps)) / args.steps
    alg = row_step * V * 4
    hbm, peak_kind = load_peaks()
    ctx.set_stream(None)
    e2e_steps = max(3, min(args.steps, 50))
    w0 = time.perf_counter()
    for i in range(e2e_steps):
        t, d, k, u = sets[i % 2]
        ctx.accept_tree(t, d, k, par, u, T)
    wall = time.perf_counter() - w0
    line = {"workload": "rejection sampling over draft trees: B=64 config-3 trees (16 nodes, "
                        "branching 4,2,2), V=32000, T=0.8 (velo_cuda_accept_tree_device)",
            "metric": BASELINE_METRIC, "value": tok_step / (ms / 1e3), "unit": "accepted tokens/s",
            "us_per_step": ms * 1e3, "accepted_per_step": tok_step,
            "roofline": {"bound": "hbm", "achieved": alg / (ms * 1e-3) / 1e9, "peak": hbm,
                         "unit": "GB/s", "frac": alg / (ms * 1e-3) / 1e9 / hbm, "peak_kind": peak_kind,
                         "algorithmic_bytes": alg,
                         "note": "bytes of the vocabulary rows the walk must read (stats, residual and "
                                 "draw passes); the walk is sequential per sequence, one CTA each"},
            "e2e": {"value": sum(toks[i % 2] for i in range(e2e_steps)) / wall, "unit": "accepted tokens/s",
                    "h2d_bytes_per_step": sum(a.nbytes for a in sets[0]) + par.nbytes,
                    "d2h_bytes_per_step": (B * N + 2 * B) * 4},
            "clocks": clk.summary()}
    ctx.close()
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- q4_0 GEMM workload
Q4_SHAPES_C3 = [  # (name, N, K, mode) of one Llama-2-7B layer + LM head at M = 32 x 16 nodes
    ("wqkv", 3 * 4096, 4096, 1), ("wo", 4096, 4096, 2), ("w1w3", 2 * 11008, 4096, 3),
    ("w2", 4096, 11008, 2), ("output", 32000, 4096, 0)]
Q4_SHAPES_C5 = [  # one Llama-3-70B layer (GQA 64/8) + LM head at M = 64 x 32 nodes, one GPU
    ("wqkv", 8192 + 2 * 1024, 8192, 1), ("wo", 8192, 8192, 2), ("w1w3", 2 * 28672, 8192, 3),
    ("w2", 8192, 28672, 2), ("output", 128256, 8192, 0)]


def run_q4gemm(args):
    """tcgen05 q4_0 GEMMs at BASELINE config 3 shapes (M = 512 verify rows), or
    config 5 shapes with --case c5 (M = 2048).  Weights of `layers` distinct
    layers (> L2 in total) are cycled so no launch finds its weight tile in L2."""
    import torch
    import synthetic
    import velo_cuda
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    c5 = args.case == "c5"
    shapes = Q4_SHAPES_C5 if c5 else Q4_SHAPES_C3
    M, layers = (2048, 4) if c5 else (512, 8)
    ctx = velo_cuda.Context(device=0)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    kmax = max(K for _, _, K, _ in shapes)
    x = torch.from_numpy(synthetic.rng(0, 20).normal(0, 1, (M, kmax)).astype(np.float16)).to(dev)
    res = []
    for name, N, K, mode in shapes:
        ws = []
        for l in range(layers if name != "output" else 2):
            raw = torch.randint(0, 256, (N, K // 32, 18), dtype=torch.uint8, device=dev)
            raw[:, :, 1] &= 0x3B  # keep the f16 scales finite and modest
            w = torch.empty(velo_cuda.q4_0_repacked_bytes(N, K), dtype=torch.uint8, device=dev)
            if mode == 3:
                ctx.q4_0_repack(raw[: N // 2], N, K, w, src_b=raw[N // 2:])
            else:
                ctx.q4_0_repack(raw, N, K, w)
            ws.append(w)
        ncol = N // 2 if mode == 3 else N
        y = torch.zeros((M, ncol), dtype=torch.float16 if mode in (1, 3) else torch.float32,
                        device=dev)
        xk = x[:, :K].contiguous()
        for i in range(max(3, args.warmup)):
            ctx.gemm_q4_0(ws[i % len(ws)], xk, M, N, K, y, ncol, mode)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(args.steps):
            ctx.gemm_q4_0(ws[i % len(ws)], xk, M, N, K, y, ncol, mode)
        e1.record(stream)
        torch.cuda.synchronize()
        ctx.sync()
        us = e0.elapsed_time(e1) * 1e3 / args.steps
        flops = 2.0 * M * N * K
        res.append({"gemm": name, "M": M, "N": N, "K": K, "us": us,
                    "tflops": flops / us / 1e6})
        del ws
        torch.cuda.empty_cache()
    peak = 1665.7
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["bf16_tflops"])
    except Exception:
        pass
    tot_us = sum(r["us"] for r in res[:-1])
    tot_fl = sum(2.0 * r["M"] * r["N"] * r["K"] for r in res[:-1])
    line = {"workload": f"q4_0 tcgen05 GEMM at BASELINE config {'5' if c5 else '3'} shapes (M={M})",
            "per_gemm": res, "layer_us": tot_us, "layer_tflops": tot_fl / tot_us / 1e6,
            "roofline": {"bound": "tensor", "achieved": tot_fl / tot_us / 1e6, "peak": peak,
                         "unit": "TFLOP/s", "frac": tot_fl / tot_us / 1e6 / peak,
                         "peak_kind": "measured bf16 burst (f16 operands here)"}}
    ctx.close()
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- tree attention workload
def _attn_device_inputs(B, N, Hq, Hkv, ctx, kv_int8, seed, dev):
    """Config-4 / config-3 attention inputs built on the device (seeded torch
    generator): K/V ~ N(0,1) (int8: per-token-per-head trunc quantisation,
    f16 scale), random page permutation, random draft trees of depth <= 6."""
    import torch
    import synthetic
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    npg = [(int(c) + 15) // 16 for c in ctx]
    total = sum(npg) + 1
    perm = torch.randperm(total, generator=g, device=dev).to(torch.int32)
    max_pages = max(npg)
    pt = torch.zeros((B, max_pages), dtype=torch.int32, device=dev)
    off = 0
    for b in range(B):
        pt[b, :npg[b]] = perm[off:off + npg[b]]
        off += npg[b]
    pools, scales = [], []
    for _ in range(2):
        if kv_int8:
            pool = torch.empty((total, Hkv, 16, 128), dtype=torch.int8, device=dev)
            sc = torch.empty((total, Hkv, 16), dtype=torch.float16, device=dev)
            step = 4096
            for p0 in range(0, total, step):
                x = torch.randn((min(step, total - p0), Hkv, 16, 128), generator=g, device=dev)
                mx = x.abs().amax(-1)
                inv = torch.where(mx > 0, 127.0 / mx, torch.zeros_like(mx))
                pool[p0:p0 + x.shape[0]] = torch.trunc(x * inv[..., None]).to(torch.int8)
                sc[p0:p0 + x.shape[0]] = (mx / 127.0).half()
            pools.append(pool)
            scales.append(sc.view(torch.int16))
        else:
            pools.append(torch.randn((total, Hkv, 16, 128), generator=g, device=dev).half())
            scales.append(None)
    q = torch.randn((B, N, Hq, 128), generator=g, device=dev).half()
    nk = torch.randn((B, N, Hkv, 128), generator=g, device=dev).half()
    nv = torch.randn((B, N, Hkv, 128), generator=g, device=dev).half()
    gg = synthetic.rng(seed, 35)
    par = torch.from_numpy(np.stack([synthetic.random_tree(N, 6, gg) for _ in range(B)])).to(dev)
    ctx_t = torch.tensor(ctx, dtype=torch.int32, device=dev)
    depth_sum = 0
    for row in par.cpu().numpy():
        d = np.zeros(N, np.int64)
        for n in range(1, N):
            d[n] = d[row[n]] + 1
        depth_sum += int((d + 1).sum())
    return dict(q=q, k=pools[0], v=pools[1], ks=scales[0], vs=scales[1], pt=pt, ctx=ctx_t,
                nk=nk, nv=nv, par=par, total=total, depth_sum=depth_sum)


def run_attn(args):
    """Tree-masked paged attention at BASELINE config 4 (INT8 KV, B=128, 64
    nodes, 32/8 heads, ctx U{512..8192}), one config-3 layer (f16 KV, B=32,
    16 nodes, 32/32 heads, ctx 2048) and one config-5 layer (f16 KV, B=64, 32
    nodes, 64/8 heads, ctx 4096).  Pools total > L2, so launches stream their
    KV from HBM."""
    import torch
    import velo_cuda
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    ctx = velo_cuda.Context(device=0)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except Exception:
        pass
    hbm = float(peaks.get("hbm_gbs", HBM_FALLBACK_GBS))
    tfl = float(peaks.get("bf16_tflops", 1590.0))
    res = []
    cfgs = [("config4_int8", 128, 64, 32, 8, None, True),
            ("config3_layer_f16", 32, 16, 32, 32, 2048, False),
            ("config5_layer_f16", 64, 32, 64, 8, 4096, False),
            # one rank's heads of the config-5 layer under tensor parallelism (4 and 8 GPUs)
            ("config5_tp4_layer_f16", 64, 32, 16, 2, 4096, False),
            ("config5_tp8_layer_f16", 64, 32, 8, 1, 4096, False)]
    for name, B, N, Hq, Hkv, fixed_ctx, i8 in cfgs:
        if args.case and args.case != name:
            continue
        if fixed_ctx is None:
            ctx_l = [int(c) for c in synthetic_ctx(B)]
        else:
            ctx_l = [fixed_ctx] * B
        d = _attn_device_inputs(B, N, Hq, Hkv, ctx_l, i8, 0, dev)
        out = torch.empty((B, N, Hq, 128), dtype=torch.float16, device=dev)
        call = lambda: ctx.tree_attention(d["q"], d["k"], d["v"], d["ks"], d["vs"], d["pt"],
                                          d["ctx"], d["nk"], d["nv"], d["par"], Hkv,
                                          1 if i8 else 0, out)
        for _ in range(max(3, args.warmup)):
            call()
        torch.cuda.synchronize()
        ctx.sync()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = max(5, min(args.steps, 100))
        e0.record(stream)
        for _ in range(n):
            call()
        e1.record(stream)
        torch.cuda.synchronize()
        ctx.sync()
        us = e0.elapsed_time(e1) * 1e3 / n
        tok = sum(ctx_l)
        elt = 1 if i8 else 2
        kv_bytes = tok * Hkv * 128 * elt * 2 + (tok * Hkv * 2 * 2 if i8 else 0)
        io_bytes = B * N * Hq * 128 * 2 * 2 + B * N * Hkv * 128 * 2 * 2
        alg_bytes = kv_bytes + io_bytes
        flops = 2.0 * 2.0 * 128 * Hq * (N * tok + d["depth_sum"])
        res.append({"case": name, "B": B, "nodes": N, "heads": f"{Hq}/{Hkv}",
                    "kv": "int8" if i8 else "f16", "ctx_tokens": tok, "us": us,
                    "alg_bytes": alg_bytes, "gbs": alg_bytes / us / 1e3,
                    "hbm_frac": alg_bytes / us / 1e3 / hbm, "tflops": flops / us / 1e6,
                    "tensor_frac": flops / us / 1e6 / tfl})
        del d
        torch.cuda.empty_cache()
    ctx.close()
    print(json.dumps({"workload": "tree-masked paged attention (BASELINE configs 4, 3 and 5)",
                      "per_case": res, "hbm_peak_gbs": hbm, "bf16_peak_tflops": tfl}), flush=True)
    return 0


# ---------------------------------------------------------------- full verify step
C3_META = dict(n_vocab=32000, n_embd=4096, n_layer=32, n_head=32, n_head_kv=32, n_ff=11008,
               head_dim=128, rope_freq_base=10000.0, norm_eps=1e-5)
C3_TREE = [-1, 0, 0, 0, 0, 1, 1, 2, 2, 3, 3, 4, 4, 5, 5, 6]  # (4,2,2) breadth-first to 16 nodes


C5_META = dict(n_vocab=128256, n_embd=8192, n_layer=80, n_head=64, n_head_kv=8, n_ff=28672,
               head_dim=128, rope_freq_base=500000.0, norm_eps=1e-5)
# branching (4, 2, 2, 2, ...) filled breadth-first to 32 nodes
C5_TREE = ([-1, 0, 0, 0, 0] + [1 + i // 2 for i in range(8)] + [5 + i // 2 for i in range(16)]
           + [13 + i // 2 for i in range(3)])


def _q4_device(w, keep_on_device=False):
    """q4_0 bytes of a device f32 matrix [rows][cols] (the rule of
    synthetic.quantize_q4_0, on the GPU): uint8 [rows][cols/32*18], on the host
    (numpy) or left on the device."""
    import torch
    rows, cols = w.shape
    xb = w.view(rows, cols // 32, 32)
    idx = xb.abs().argmax(-1, keepdim=True)
    m = torch.gather(xb, -1, idx)[..., 0]
    d = m / -8.0
    inv = torch.where(d != 0, 1.0 / d, torch.zeros_like(d))
    q = torch.clamp(torch.trunc(xb * inv[..., None] + 8.5), 0, 15).to(torch.uint8)
    out = torch.empty((rows, cols // 32, 18), dtype=torch.uint8, device=w.device)
    out[..., 0:2] = d.half().view(torch.uint8).view(rows, cols // 32, 2)
    out[..., 2:] = q[..., 0::2] | (q[..., 1::2] << 4)
    out = out.view(rows, -1)
    return out if keep_on_device else out.cpu().numpy()


def c5_shard_tensors(meta, tp, rank, seed=0):
    """This rank's shards of a Llama-3-70B-shape model:
    random N(0, 0.02^2) matrices quantised to q4_0 and an f32 embedding, all
    generated on the device and handed to the loader as device tensors (no
    host copy of the 39 GB of weights).  Shard shapes follow sharding.rs
    (column split of q/k/v/w1/w3/output, row split of wo/w2)."""
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(seed * 1000 + rank)
    H, V, F, L = meta["n_embd"], meta["n_vocab"], meta["n_ff"] // tp, meta["n_layer"]
    Dq, Dk, Vl = meta["n_head"] // tp * 128, meta["n_head_kv"] // tp * 128, V // tp

    def q4(rows, cols):
        w = torch.randn((rows, cols), generator=g, device="cuda") * 0.02
        q = _q4_device(w, keep_on_device=True)
        del w
        return (2, q, rows, cols)

    def norm():
        return (0, 1.0 + 0.1 * torch.randn(H, generator=g, device="cuda"), 1, H)

    t = {"token_embd.weight": (0, torch.randn((V, H), generator=g, device="cuda") * 0.02, V, H),
         "output_norm.weight": norm(), "output.weight": q4(Vl, H)}
    for l in range(L):
        p = f"layers.{l}."
        t[p + "attention_norm.weight"] = norm()
        t[p + "attention.wq.weight"] = q4(Dq, H)
        t[p + "attention.wk.weight"] = q4(Dk, H)
        t[p + "attention.wv.weight"] = q4(Dk, H)
        t[p + "attention.wo.weight"] = q4(H, Dq)
        t[p + "ffn_norm.weight"] = norm()
        t[p + "feed_forward.w1.weight"] = q4(F, H)
        t[p + "feed_forward.w2.weight"] = q4(H, F)
        t[p + "feed_forward.w3.weight"] = q4(F, H)
    return t


def c3_model_tensors(meta, seed=0):
    """Llama-2-7B-shape random-init weights N(0, 0.02^2) quantised to q4_0
    generated and quantised on the GPU."""
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    H, V, F, L = meta["n_embd"], meta["n_vocab"], meta["n_ff"], meta["n_layer"]
    Dq, Dk = meta["n_head"] * 128, meta["n_head_kv"] * 128

    def q4(rows, cols):
        return (2, _q4_device(torch.randn((rows, cols), generator=g, device="cuda") * 0.02), rows, cols)

    def norm():
        return (0, (1.0 + 0.1 * torch.randn(H, generator=g, device="cuda")).cpu().numpy(), 1, H)

    t = {"token_embd.weight": q4(V, H), "output_norm.weight": norm(), "output.weight": q4(V, H)}
    for l in range(L):
        p = f"layers.{l}."
        t[p + "attention_norm.weight"] = norm()
        t[p + "attention.wq.weight"] = q4(Dq, H)
        t[p + "attention.wk.weight"] = q4(Dk, H)
        t[p + "attention.wv.weight"] = q4(Dk, H)
        t[p + "attention.wo.weight"] = q4(H, Dq)
        t[p + "ffn_norm.weight"] = norm()
        t[p + "feed_forward.w1.weight"] = q4(F, H)
        t[p + "feed_forward.w2.weight"] = q4(H, F)
        t[p + "feed_forward.w3.weight"] = q4(F, H)
    return t


def host_q4(rows, cols, g, scale=0.0025):
    """Random q4_0 bytes [rows][cols/32*18] made on the host without the GPU
    (random nibbles, every block scale `scale`): the CPU port's timing does
    not depend on the values, and generating 1.5 GB of normals would take
    longer than timing it."""
    nb = cols // 32
    raw = np.frombuffer(g.bytes(rows * nb * 18), np.uint8).reshape(rows, nb, 18).copy()
    raw[:, :, 0:2] = np.frombuffer(np.float16(scale).tobytes(), np.uint8)
    return raw.reshape(rows, nb * 18)


def cpu_sample_tensors(meta, n_layer, seed=0):
    """Oracle tensor list of a model with the config's layer shapes but
    `n_layer` layers (q4_0 matrices and embedding, f32 norms of 1)."""
    g = np.random.Generator(np.random.Philox(key=seed + 77))
    H, V, F = meta["n_embd"], meta["n_vocab"], meta["n_ff"]
    Dq, Dk = meta["n_head"] * 128, meta["n_head_kv"] * 128
    ones = np.ones(H, np.float32)
    out = [(2, host_q4(V, H, g)), (0, ones), (2, host_q4(V, H, g))]
    for _ in range(n_layer):
        out += [(0, ones), (2, host_q4(Dq, H, g)), (2, host_q4(Dk, H, g)), (2, host_q4(Dk, H, g)),
                (2, host_q4(H, Dq, g)), (0, ones), (2, host_q4(F, H, g)), (2, host_q4(H, F, g)),
                (2, host_q4(F, H, g))]
    return out


def cpu_token_model(meta, ctx_len):
    """forward_one of the CPU port (oracle restatement of llama_cpu.rs, one
    thread) at position ctx_len - 1 (attention over ctx_len cached positions),
    timed on 1- and 2-layer models of the config's shapes and extrapolated to
    all n_layer layers: t = t1 + (n_layer - 1) * (t2 - t1).  Returns
    (seconds per token over all layers, seconds of the 2-layer sample,
    the 2-layer tensors)."""
    import vo
    ts = {}
    keep = None
    for nl in (1, 2):
        tl = cpu_sample_tensors(meta, nl)
        m = vo.Model(dict(meta, n_layer=nl, n_ctx=ctx_len), tl)
        m.forward_one(1, ctx_len - 1)  # page the weights in
        t0 = time.perf_counter()
        m.forward_one(1, ctx_len - 1)
        ts[nl] = time.perf_counter() - t0
        del m
        if nl == 2:
            keep = tl
    per_layer = max(ts[2] - ts[1], 0.0)
    return ts[1] + (meta["n_layer"] - 1) * per_layer, ts[2], keep


def verify_case(case):
    c5 = case != "c3"
    meta = dict(C5_META if c5 else C3_META)
    tree = C5_TREE if c5 else C3_TREE
    B, ctx_len = (64, 4096) if c5 else (32, 2048)
    wl = ("BASELINE config 5: Llama-3-70B-shape verify step in q4_0 (80 layers, hidden 8192, "
          "64/8 heads, FFN 28672, vocab 128256), B=64 sequences, 32-node draft tree each "
          "(branching 4,2,2,.. breadth-first), context 4096 in 16-token fp16 KV pages" if c5 else
          "BASELINE config 3: Llama-2-7B-shape verify step in q4_0 (32 layers, hidden 4096, 32 heads, "
          "FFN 11008, vocab 32000), B=32 sequences, 16-node draft tree each (branching 4,2,2 "
          "breadth-first), context 2048 in 16-token fp16 KV pages")
    return c5, meta, tree, B, ctx_len, wl


def verify_counts(meta, B, N, ctx_len, tp):
    """Per-step algorithmic work of the verify step on one rank of `tp`."""
    H, F, V, L = meta["n_embd"], meta["n_ff"], meta["n_vocab"], meta["n_layer"]
    Dq, Dk = meta["n_head"] * 128, meta["n_head_kv"] * 128
    M = B * N
    params = L * (H * (Dq + 2 * Dk) + Dq * H + 3 * H * F) + V * H
    return dict(M=M, flops=2.0 * M * params / tp, params=params,
                ffn_up_flops=2.0 * M * (2 * F // tp) * H,
                kv_bytes=B * ctx_len * L * Dk * 2 * 2 / tp, w_bytes=params * 18 / 32 / tp)


def run_verify(args):
    """The verify step (the north-star path) through velo_cuda_verify_step:
    target forward over every draft-tree node of B sequences (q4_0 tcgen05
    GEMMs, tree-masked paged attention over fp16 pages), greedy tree
    acceptance (GreedySampler + find_best_path) and the KV commit of the
    accepted paths.  Default: BASELINE config 5; --case c3 for config 3.
    Under torchrun the ranks form one tensor-parallel group (column / row
    split as sharding.rs, bf16 NCCL all-reduce after o_proj and down_proj,
    vocabulary-sharded LM head): the job is the same batch at every N, so
    "scaling" is "strong".  Inputs (weights, KV pages) are resident in HBM and
    each step streams ~40 GB of weights and ~86 GB of KV (config 5), far more
    than the 126 MB L2."""
    import torch
    import torch.distributed as dist
    import velo_cuda
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    nid = None
    if ws > 1:
        from datetime import timedelta
        dist.init_process_group("gloo", timeout=timedelta(seconds=300))
        box = [velo_cuda.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        nid = box[0]

    def max_over_ranks(vals):
        if ws == 1:
            return list(vals)
        t = torch.tensor(list(vals), dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return [float(x) for x in t]

    c5, meta, tree, B, ctx_len, wl = verify_case(args.case)
    N = len(tree)
    per_seq = (ctx_len + N + 15) // 16
    cnt = verify_counts(meta, B, N, ctx_len, ws)
    M = cnt["M"]
    t0 = time.time()
    tensors = c5_shard_tensors(meta, ws, rank) if c5 else c3_model_tensors(meta)
    torch.cuda.synchronize()
    gen_s = time.time() - t0
    ctx = velo_cuda.Context(device=local, total_pages=B * per_seq, max_slots=B,
                            max_pages_per_slot=per_seq, tp_rank=rank, tp_size=ws, nccl_id=nid)
    t0 = time.time()
    ctx.load_model(meta, tensors, shards=c5)
    load_s = time.time() - t0
    del tensors
    torch.cuda.empty_cache()
    for b in range(B):
        ctx.bind_slot(b, np.arange(b * per_seq, (b + 1) * per_seq))
    g = np.random.Generator(np.random.Philox(7))
    tokens = g.integers(0, meta["n_vocab"], (B, N)).astype(np.uint32)
    parents = np.tile(np.array(tree, np.int32), (B, 1))
    slots = np.arange(B, dtype=np.uint32)
    ctxl = np.full(B, ctx_len, np.int32)
    stream = torch.cuda.Stream()
    ctx.set_stream(stream.cuda_stream)

    def step():
        r = ctx.verify_step(slots, ctxl, tokens, parents, commit=True, n_vocab=meta["n_vocab"])
        return int((r["accepted_len"] + 1).sum())

    for _ in range(args.warmup):
        step()
    # ---- device-timed steps (CUDA events on the context stream) ----------
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    acc_tok = 0
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            acc_tok += step()
        e1.record(stream)
        torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    ms = max_over_ranks([e0.elapsed_time(e1) / args.steps])[0]
    acc_per_step = acc_tok / args.steps
    # ---- end to end: the host-buffer C ABI call, wall clock --------------
    e2e_steps = max(3, min(args.steps, 10))
    if ws > 1:
        dist.barrier()
    w0 = time.perf_counter()
    e2e_tok = 0
    for _ in range(e2e_steps):
        e2e_tok += step()
    wall = max_over_ranks([time.perf_counter() - w0])[0]
    # ---- phase profile of two more steps (events between the phases) -----
    ctx.profile(True)
    prof_steps = 2
    for _ in range(prof_steps):
        step()
    phases, nsteps = ctx.profile_read()
    ctx.profile(False)
    names = list(phases)
    phase_ms = dict(zip(names, max_over_ranks([phases[n] / max(nsteps, 1) for n in names])))
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
        peak_kind = "measured"
    except Exception:
        peak_kind = "fallback"
    tfl = float(peaks.get("bf16_tflops_sustained", 1400.0))
    hbm = float(peaks.get("hbm_gbs", HBM_FALLBACK_GBS))
    floor_ms = (cnt["flops"] / (tfl * 1e12) + cnt["kv_bytes"] / (hbm * 1e9)) * 1e3
    up_ms = phase_ms["gemm_ffn_up"] / meta["n_layer"]  # one launch per layer
    up_tflops = cnt["ffn_up_flops"] / (up_ms * 1e-3) / 1e12
    gemm_ms = sum(phase_ms[k] for k in ("gemm_qkv", "gemm_o", "gemm_ffn_up", "gemm_ffn_down",
                                        "lm_head"))
    H2D = (2 * M + 2 * B + B * per_seq) * 4  # tokens, parents, ctx_len, slots, page-table rows
    D2H = (2 * B + 2 * M) * 4                # path lengths, bonus tokens, paths, expected tokens
    L = meta["n_layer"]
    sum_path = ctx.tp_sum_path()
    # per layer 8 kernels, plus our sum kernels: 2 (peer, fused) or 2 x 5 (ce: signal,
    # wait, add, signal, wait per sum)
    launches = 2 + (8 + {"peer": 2, "fused": 2, "ce": 10}.get(sum_path, 0)) * L + 2 + (2 if ws == 1 else 3) + 1
    traffic = None
    if ws == 1:
        traffic = load_traffic("q4gemm_swiglu_c5" if c5 else "q4gemm_swiglu_c3")
    line = {
        "metric": BASELINE_METRIC, "value": acc_per_step / (ms / 1e3),
        "unit": "accepted tokens/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "us_per_step": ms * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "f16 operands (q4_0 weights dequantised to f16 in the GEMM), f32 accumulation, f16 KV",
        "data": "synthetic: random-init N(0,0.02^2) weights quantised to q4_0 on the device"
                + ("; each rank generates its own shards" if c5 else "")
                + "; random draft-tree tokens (seeded Philox); KV pages zero-filled (the timing "
                  "does not depend on their values)",
        "config": {"workload": wl, "B": B, "nodes": N, "ctx": ctx_len, "rows": M,
                   "parallelism": f"tp{ws}" if ws > 1 else "tp1 (single GPU)",
                   "tp_sum": {"ce": "column blocks cross NVLink as copy-engine copies (CUDA IPC); "
                                    "the owner's kernel adds, copies back",
                              "fused": "row-split GEMM epilogue pushes each column block to its owner "
                                       "over NVLink (CUDA IPC); the owner's kernel adds and broadcasts",
                              "peer": "one kernel over NVLink peer memory (CUDA IPC)",
                              "nccl": "NCCL bf16 all-reduce", "none": None}[sum_path],
                   "l2": f"inputs > L2: {cnt['w_bytes'] / 1e9:.1f} GB of weights and "
                         f"{cnt['kv_bytes'] / 1e9:.1f} GB of KV streamed per step and rank"},
        "accepted_per_step": acc_per_step,
        "roofline": {"bound": "tensor", "achieved": up_tflops, "peak": tfl, "unit": "TFLOP/s",
                     "frac": up_tflops / tfl, "traffic": traffic, "peak_kind": peak_kind
                     + " bf16 sustained (the GEMM runs inside a long step)",
                     "kernel": "q4_gemm_ta_swiglu_kernel (w1/w3 + SwiGLU, the largest share of the "
                               "step), one launch per layer",
                     "algorithmic_flops_per_launch": cnt["ffn_up_flops"],
                     "us_per_launch": up_ms * 1e3,
                     "all_gemms_tflops": cnt["flops"] / (gemm_ms * 1e-3) / 1e12 if gemm_ms else None,
                     "step_floor_ms": floor_ms, "step_frac_of_floor": floor_ms / ms,
                     "step_floor_note": "GEMM FLOPs at the sustained bf16 peak + KV bytes at the "
                                        "measured HBM bandwidth, per rank"},
        "phase_ms_per_step": phase_ms,
        "clocks": clk.summary(),
        "e2e": {"value": e2e_tok / e2e_steps / (wall / e2e_steps), "unit": "accepted tokens/s",
                "h2d_bytes_per_step": H2D, "d2h_bytes_per_step": D2H, "steps": e2e_steps,
                "ms_per_step": wall / e2e_steps * 1e3,
                "path": "velo_cuda_verify_step with host buffers (inputs packed into pinned memory "
                        "and copied in, paths / bonus tokens / expected tokens copied back, every "
                        "step), wall clock, max over ranks"},
        "gpu_launches": launches * args.steps,
        "model_gen_s": gen_s, "load_s": load_s,
    }
    ctx.close()
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        t_tok, t2, _ = cpu_token_model(meta, ctx_len)
        cpu_step = t_tok * M  # the reference runs forward_one once per tree node
        line["cpu_baseline"] = {
            "value": acc_per_step / cpu_step, "unit": "accepted tokens/s", "cores": 1,
            "kind": "port", "ms_per_step": cpu_step * 1e3,
            "sample": f"forward_one of the CPU port (llama_cpu.rs restatement, one thread) at "
                      f"position {ctx_len - 1} on 1- and 2-layer models of the config's shapes "
                      f"(2 layers: {t2:.2f} s), extrapolated to {meta['n_layer']} layers "
                      f"({t_tok:.1f} s per token); a verify step is {M} such calls "
                      f"(B x nodes), extrapolated linearly"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def run_reference_verify(args):
    """--impl reference for the verify step: the CPU port of the reference's
    path (oracle restatement of llama_cpu.rs forward_one, the CPU backend the
    CUDA one replaces) on all host threads, one forward_one per thread (one
    tree node each) on a 2-layer model of the config's shapes per step;
    the full step (B x nodes forward_one calls of all layers) is extrapolated
    from it.  Rank 0 alone runs it."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    import threading as th
    import vo
    c5, meta, tree, B, ctx_len, wl = verify_case(args.case)
    N = len(tree)
    M = B * N
    threads = max(1, min(os.cpu_count() or 1, M))
    t_tok, t2, tl = cpu_token_model(meta, ctx_len)
    scale = t_tok / t2  # all layers over the 2-layer sample, single thread
    models = [vo.Model(dict(meta, n_layer=2, n_ctx=ctx_len), tl) for _ in range(threads)]

    def one(mm):
        mm.forward_one(1, ctx_len - 1)

    secs = []
    for s_ in range(args.warmup + args.steps):
        ts = [th.Thread(target=one, args=(mm,)) for mm in models]
        t0 = time.perf_counter()
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        dt = time.perf_counter() - t0
        if s_ >= args.warmup:
            secs.append(dt)
    sample_s = statistics.mean(secs)
    rounds = -(-M // threads)
    step_s = sample_s * scale * rounds
    acc_per_step = float(B)  # random-token drafts are rejected at the root; each sequence emits one
    value = acc_per_step / step_s
    line = {
        "impl": "reference", "metric": BASELINE_METRIC, "value": value,
        "unit": "accepted tokens/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32 (q4_0 weights dequantised per row)",
        "data": "synthetic (random q4_0 weights, zero KV of the config's context)",
        "config": {"workload": wl, "B": B, "nodes": N, "ctx": ctx_len, "rows": M,
                   "parallelism": f"{threads} host threads, one tree node each"},
        "cpu_baseline": {"value": value, "unit": "accepted tokens/s", "cores": threads,
                         "kind": "port",
                         "sample": f"per step {threads} concurrent forward_one calls (one per "
                                   f"thread) of the CPU port on a 2-layer model of the config's "
                                   f"shapes at position {ctx_len - 1}, {sample_s:.2f} s; scaled by "
                                   f"{scale:.1f} to all {meta['n_layer']} layers (single-thread "
                                   f"1- vs 2-layer timing) and by {rounds} rounds to the step's "
                                   f"{M} nodes; {acc_per_step:.0f} accepted tokens per step (one "
                                   f"per sequence, as the CUDA arm measures on random drafts)"},
        "e2e": {"value": value, "unit": "accepted tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- tiny fp32 pair (config 1)
C1_K, C1_PROMPT, C1_NEW = 4, 64, 128


class _Timed:
    """A draft / target model whose every call is bracketed by CUDA events on
    the contexts' stream (device time of the call, host gaps inside it
    included)."""

    def __init__(self, model, stream):
        import torch
        self.m, self.stream, self.ev, self.torch = model, stream, [], torch

    def _call(self, fn, *a):
        e0 = self.torch.cuda.Event(enable_timing=True)
        e1 = self.torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        out = fn(*a)
        e1.record(self.stream)
        self.ev.append((e0, e1))
        return out

    def draft(self, context, n):
        return self._call(self.m.draft, context, n)

    def verify(self, context, drafted):
        return self._call(self.m.verify, context, drafted)


class _OracleGreedyTarget:
    """The CPU port's target for the session baseline (chain verify, commit)."""

    def __init__(self, model):
        self.m, self.cached = model, 0

    def verify(self, context, drafted):
        import vo
        from speculative import VerifyStep
        for i in range(self.cached, len(context) - 1):
            self.m.forward_one(int(context[i]), i)
        pos = len(context) - 1
        nodes = np.array([context[-1]] + list(drafted), np.uint32)
        lg = self.m.verify_tree(nodes, np.arange(-1, len(nodes) - 1, dtype=np.int32), pos)
        exp = [vo.greedy(lg[i])[0] for i in range(len(drafted))]
        acc = 0
        while acc < len(drafted) and drafted[acc] == exp[acc]:
            acc += 1
        self.m.commit_path(list(range(acc + 1)), pos)
        self.cached = pos + acc + 1
        return [VerifyStep(e) for e in exp]


class _OracleGreedyDraft:
    def __init__(self, model):
        self.m, self.tokens = model, []

    def draft(self, context, n):
        import vo
        from speculative import NextTokenPrediction
        common = 0
        for a, b in zip(self.tokens, context[:-1]):
            if a != b:
                break
            common += 1
        self.tokens = self.tokens[:common]
        for i in range(common, len(context) - 1):
            self.m.forward_one(int(context[i]), i)
            self.tokens.append(int(context[i]))
        out, last = [], int(context[-1])
        for _ in range(n):
            lg = self.m.forward_one(last, len(self.tokens))
            self.tokens.append(last)
            last = vo.greedy(lg)[0]
            out.append(NextTokenPrediction(last))
        return out


def c1_cpu_baseline():
    """The CPU port (oracle restatement of llama_cpu.rs, one thread) running the
    whole greedy session of config 1: accepted tokens/s."""
    import synthetic
    import vo
    from speculative import SpeculativeDecoder
    tm, tw, dm, dw = synthetic.c1_pair(0)
    prompt = [int(t) for t in synthetic.rng(0, 91).integers(0, tm["n_vocab"], C1_PROMPT)]
    dl, tl = synthetic.oracle_tensor_list(dm, dw), synthetic.oracle_tensor_list(tm, tw)
    secs, toks, reps = 0.0, 0, 0
    while secs < 10.0:
        t0 = time.perf_counter()
        out = SpeculativeDecoder(C1_K, C1_K).generate(
            _OracleGreedyDraft(vo.Model(dict(dm, n_ctx=512), dl)),
            _OracleGreedyTarget(vo.Model(dict(tm, n_ctx=512), tl)), prompt, C1_NEW)
        secs += time.perf_counter() - t0
        toks += len(out.tokens)
        reps += 1
    return {"value": toks / secs, "unit": "accepted tokens/s", "cores": 1, "kind": "port",
            "sample": f"{reps} whole greedy sessions ({C1_PROMPT}-token prompt incl. prefill, "
                      f"k={C1_K}, {C1_NEW} new tokens), single-threaded like llama_cpu.rs, "
                      f"{secs:.1f} s"}


def run_c1(args):
    """BASELINE config 1 on the fp32 path: the tiny Llama pair (target 2 layers,
    draft 1 layer; hidden 256, 4 x 64 heads, FFN 688, vocab 4096, f32 weights
    N(0, 0.02^2)), batch 1, 64-token prompt, linear speculation k = 4, sessions
    of 128 new tokens, greedy and T = 1.0.  A step is one session round: the
    draft's k one-token decode steps and the target's verify step (forward over
    k + 1 nodes, acceptance, KV commit), every call through the host-buffer C
    ABI.  Independent replicas under torchrun."""
    import torch
    import torch.distributed as dist
    import synthetic
    import velo_cuda
    from speculative import CudaDraft, CudaTarget, SpeculativeDecoder
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    if ws > 1:
        from datetime import timedelta
        dist.init_process_group("gloo", timeout=timedelta(seconds=300))
    tm, tw, dm, dw = synthetic.c1_pair(0)
    V = tm["n_vocab"]
    prompt = [int(t) for t in synthetic.rng(0, 91).integers(0, V, C1_PROMPT)]
    pages = (C1_PROMPT + C1_NEW + C1_K + 16) // 16 + 1
    stream = torch.cuda.Stream()
    ctxs = []
    for meta, w in ((tm, tw), (dm, dw)):
        c = velo_cuda.Context(device=local, kv_dtype=velo_cuda.KV_F32, total_pages=pages,
                              max_slots=1, max_pages_per_slot=pages)
        c.load_model(meta, w)
        c.bind_slot(0, np.arange(pages))
        c.set_stream(stream.cuda_stream)
        ctxs.append(c)
    tctx, dctx = ctxs
    rounds = max(3, min(args.steps, 400))

    def run_mode(T):
        rng = np.random.Generator(np.random.Philox(5))
        rec = []  # per round: (new tokens, drafted, accepted, draft event, verify event)
        wall = 0.0
        while len(rec) < args.warmup + rounds:
            draft = CudaDraft(dctx, 0, V, T, rng)
            target = CudaTarget(tctx, 0, V, T, draft, rng)
            td, tt = _Timed(draft, stream), _Timed(target, stream)
            sess = SpeculativeDecoder(C1_K, C1_K).begin(prompt)
            target.prefill(sess.context)
            draft.prefill(sess.context)
            generated = 0
            while generated < C1_NEW and len(rec) < args.warmup + rounds:
                s0, d0 = sess.stats.accepted_tokens, sess.stats.drafted_tokens
                w0 = time.perf_counter()
                got = sess.draft(td, tt, C1_NEW - generated)
                new = len(got) + (1 if sess.take_rejected_token() is not None else 0)
                wall_r = time.perf_counter() - w0
                if len(rec) >= args.warmup:
                    wall += wall_r
                generated += new
                rec.append((new, sess.stats.drafted_tokens - d0, sess.stats.accepted_tokens - s0,
                            td.ev[-1], tt.ev[-1]))
        torch.cuda.synchronize()
        timed = rec[args.warmup:]
        d_ms = [r[3][0].elapsed_time(r[3][1]) for r in timed]
        v_ms = [r[4][0].elapsed_time(r[4][1]) for r in timed]
        toks = sum(r[0] for r in timed)
        acc = sum(r[2] for r in timed)
        drafted = sum(r[1] for r in timed)
        return dict(tokens=toks, draft_ms=sum(d_ms), verify_ms=sum(v_ms), wall=wall,
                    acceptance_rate=acc / max(drafted, 1), rounds=len(timed),
                    us_per_verify=statistics.mean(v_ms) * 1e3, us_per_draft=statistics.mean(d_ms) * 1e3)

    if ws > 1:
        dist.barrier()
    with ClockSampler(local) as clk:
        g = run_mode(0.0)
        t1 = run_mode(1.0)
    dev_s = (g["draft_ms"] + g["verify_ms"]) / 1e3
    vals = [g["tokens"] / dev_s, g["tokens"] / g["wall"], dev_s, g["wall"]]
    if ws > 1:
        t = torch.tensor([dev_s, g["wall"]], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_s, wall = float(t[0]), float(t[1])
        vals = [ws * g["tokens"] / dev_s, ws * g["tokens"] / wall, dev_s, wall]
    L, Ld, H, F, D = tm["n_layer"], dm["n_layer"], tm["n_embd"], tm["n_ff"], tm["head_dim"]
    Hq = tm["n_head"]
    layer_w = (H * (Hq + 2 * tm["n_head_kv"]) * D + Hq * D * H + 3 * H * F) * 4
    step_bytes = L * layer_w + V * H * 4  # every f32 weight of the target read once per verify
    ctx_mean = C1_PROMPT + C1_NEW / 2
    step_bytes += L * ctx_mean * tm["n_head_kv"] * D * 4 * 2
    hbm, peak_kind = load_peaks()
    v_s = g["verify_ms"] / 1e3 / g["rounds"]
    # launches per round: verify step (tree ancestors, embed, 8 per layer, norm + head,
    # argmax + walk, commit) and k draft decode steps (the same sequence at L = 1)
    launches_round = (2 + 8 * L + 2 + 2 + 1) + C1_K * (2 + 8 * Ld + 2 + 2 + 1)
    N = C1_K + 1
    h2d = (N * 8 + 8 + pages * 4) + C1_K * (8 + 8 + pages * 4)
    d2h = (8 + N * 4) + C1_K * (8 + 4)
    line = {
        "metric": BASELINE_METRIC, "value": vals[0], "unit": "accepted tokens/s",
        "n_gpus": ws, "steps": g["rounds"], "warmup": args.warmup,
        "ms_per_step": dev_s * 1e3 / g["rounds"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "BASELINE config 1: tiny fp32 Llama pair (target 2 layers, draft 1; "
                               "hidden 256, 4x64 heads, FFN 688, vocab 4096), batch 1, 64-token "
                               "prompt, k=4, sessions of 128 new tokens",
                   "parallelism": f"{ws} replicas" if ws > 1 else "single GPU",
                   "l2": "weights (10.5 MB) are L2-resident by design: latency-bound"},
        "us_per_verify_step": g["us_per_verify"], "us_per_draft_k4": g["us_per_draft"],
        "acceptance_rate": g["acceptance_rate"],
        "t1": {"accepted_tokens_per_s": t1["tokens"] / ((t1["draft_ms"] + t1["verify_ms"]) / 1e3),
               "us_per_verify_step": t1["us_per_verify"], "us_per_draft_k4": t1["us_per_draft"],
               "acceptance_rate": t1["acceptance_rate"], "rounds": t1["rounds"]},
        "e2e": {"value": vals[1], "unit": "accepted tokens/s (wall clock of the Python session "
                                          "loop over the host-buffer C ABI)",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "roofline": {"bound": "hbm", "achieved": step_bytes / v_s / 1e9, "peak": hbm, "unit": "GB/s",
                     "frac": step_bytes / v_s / 1e9 / hbm, "traffic": None,
                     "peak_kind": peak_kind,
                     "note": "verify step: target f32 weights + mean-context KV bytes / step time; "
                             "the step is launch-latency-bound (weights live in L2)"},
        "gpu_launches": launches_round * g["rounds"],
        "clocks": clk.summary(),
    }
    for c in ctxs:
        c.close()
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = c1_cpu_baseline()
        print(json.dumps(line), flush=True)
    return 0


def synthetic_ctx(B, seed=0):
    """Per-sequence context lengths U{512..8192}."""
    import synthetic
    return synthetic.rng(seed, 36).integers(512, 8193, B)


def cpu_baseline():
    """The CPU port (oracle) on this host, full C2 batch repeated ~10 s."""
    import vo
    import synthetic
    threads = os.cpu_count() or 1
    B, k, V, T = 64, 8, 32000, 0.8
    tgt, drf, tok, u = synthetic.acceptance_inputs(B, k, V, T)
    toks, secs, reps = 0, 0.0, 0
    while secs < 10.0 or reps < 1:
        t0 = time.perf_counter()
        acc, _ = vo.accept(tgt, drf, tok, u, T, n_threads=threads)
        secs += time.perf_counter() - t0
        toks += accepted_tokens(acc)
        reps += 1
    return {"value": toks / secs, "unit": "accepted tokens/s", "cores": threads, "kind": "port",
            "sample": f"{reps} full steps of config 2 (64 sequences, k=8, V=32000), "
                      f"{threads} threads over sequences, {secs:.1f} s"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--impl", default="cuda", choices=["cuda", "reference"])
    ap.add_argument("--workload", default="verify", choices=["verify", "accept", "accept_tree", "q4gemm", "attn", "c1"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--case", default="", help="one case of a multi-case workload "
                                               "(verify: c5 [default] or c3)")
    args = ap.parse_args()
    quick = args.workload == "verify"  # 0.05-0.4 s per step: a few dozen steps
    if args.steps is None:
        args.steps = 20 if quick else 2000
    if args.warmup is None:
        args.warmup = 3 if quick else 20
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        if args.workload == "verify":
            return run_reference_verify(args)
        return run_reference(args)
    if args.workload == "accept_tree":
        return run_accept_tree(args)
    if args.workload == "q4gemm":
        return run_q4gemm(args)
    if args.workload == "attn":
        return run_attn(args)
    if args.workload == "verify":
        return run_verify(args)
    if args.workload == "c1":
        return run_c1(args)
    return run_cuda(args)


if __name__ == "__main__":
    sys.exit(main())
