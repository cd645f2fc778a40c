#!/usr/bin/env python
"""RACE attention fwd+bwd throughput on B200 (tokens/s) and % of HBM roofline.

Workload (the reference's long-context scaling config): B=1, H=1, d=64, K=2,
L=5, 2^20 tokens per GPU, q/k/v/dO ~ N(0,1) from seed 0, one sequence
sharded along the tokens over the GPUs (weak scaling: every GPU holds 2^20
tokens; bucket states are all-reduced over NCCL).  The headline line is the
non-causal float32 layer; causal and bfloat16 variants are measured in the
same run and reported under "variants".

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one forward + backward of the layer over the resident inputs.
Inputs (256 MiB per tensor in fp32) are larger than the 126 MB L2, so no L2
flush is needed between steps.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

D, K, L = 64, 2, 5
S = L << K
TOKENS = 1 << 20
METRIC = "RACE attn fwd+bwd tokens/s at N=1M (d=64, K=2, L=5)"
STRONG_TOKENS = 1 << 26          # the 64M-token sequence, sharded over the GPUs
VARIANT_STEPS = 200              # timed steps of each variant (the headline uses --steps)


# --------------------------------------------------------------------------- helpers
def load_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.idx = device_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
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
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, val in zip(names, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "samples": len(sm),
                "reasons": sorted(reasons)}


def cpu_model():
    try:
        out = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
        for ln in out.splitlines():
            if ln.startswith("Model name:"):
                return ln.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# --------------------------------------------------------------------------- our arm
class Layer:
    """Preallocated buffers + the C-ABI calls of one fwd+bwd step."""

    def __init__(self, causal, dtype, tokens, group, device, seed, normalize=0, batch=1, heads=1,
                 bits=K, tables=L):
        from race_attention_b200 import _lib
        from race_attention_b200.functional import Buffers, make_desc, query
        self.lib = _lib.load()
        self.causal, self.dtype, self.group = causal, dtype, group
        g = torch.Generator(device=device).manual_seed(seed)
        # [M=1, B, T, H, d] as the modules lay the Linear outputs out
        shape = (1, batch, tokens, heads, D)
        rnd = lambda: torch.randn(shape, generator=g, device=device, dtype=torch.float32).to(dtype)
        self.q, self.k, self.v, self.dout = rnd(), rnd(), rnd(), rnd()
        g0 = torch.Generator(device=device).manual_seed(0)   # identical planes on every rank
        self.planes = torch.randn((1, bits * tables, D), generator=g0, device=device)
        self.scale = torch.tensor(1.0, device=device)
        self.desc = make_desc(shape, dtype, bits, tables, causal, 1e-6, 0, True, normalize,
                              _lib.RACE_FLAG_STRICT_TMA)
        self.sizes = query(self.desc)
        self.buf = Buffers(self.sizes, device)
        self.out = torch.empty(shape, dtype=dtype, device=device)
        self.dq, self.dk, self.dv = (torch.empty(shape, dtype=dtype, device=device) for _ in range(3))
        self.dscale = torch.empty((), device=device)
        self.state = self.buf.floats(self.sizes.state_bytes)
        self.gstate = self.buf.floats(self.sizes.gstate_bytes)
        self.ws = self.buf.workspace()
        self.tokens = tokens

    def phases(self):
        """The step as its four C-ABI phases (+ collectives when sharded)."""
        from race_attention_b200._lib import check
        from race_attention_b200.functional import _ptr, _rt, _stream
        from race_attention_b200 import sequence_parallel as sp
        lib, d = self.lib, self.desc
        q, k, v, o = _rt(self.q), _rt(self.k), _rt(self.v), _rt(self.out)
        P, sc, st, gs, ws, n = (_ptr(self.planes), _ptr(self.scale), _ptr(self.state),
                                _ptr(self.gstate), _ptr(self.ws), self.ws.numel())
        total = self.buf.floats(self.sizes.total_bytes) if self.causal else None
        gtotal = self.buf.floats(self.sizes.total_bytes) if self.causal else None

        def f_reduce():
            check(lib.race_forward_reduce(d, k, v, P, sc, st, _ptr(total), ws, n, _stream()))
            if self.group is not None:
                add = lambda off: check(lib.race_add_offset(d, st, _ptr(off), 0, _stream()))
                sp.exchange_forward_state(self.state, total, self.causal, self.group, add)

        def f_readout():
            check(lib.race_forward_readout(d, q, k, v, P, sc, st, o, ws, n, _stream()))

        def b_q():
            check(lib.race_backward_q(d, q, k, v, P, sc, st, _rt(self.dout), _rt(self.dq),
                                      _ptr(self.dscale), gs, _ptr(gtotal), ws, n, _stream()))
            if self.group is not None:
                slots = self.gstate[: self.state.numel()] if self.causal else self.gstate
                add = lambda off: check(lib.race_add_offset(d, gs, _ptr(off), 1, _stream()))
                sp.exchange_backward_state(slots, gtotal, self.causal, self.group, add)

        def b_kv():
            # dscale stays rank-local (this rank's tokens), as the C ABI defines it: a
            # training step sums it with the model's other parameter gradients
            check(lib.race_backward_kv(d, q, k, v, P, sc, st, gs, _rt(self.dout), _rt(self.dk),
                                       _rt(self.dv), _ptr(self.dscale), ws, n, _stream()))

        return [("forward_reduce", f_reduce), ("forward_readout", f_readout),
                ("backward_q", b_q), ("backward_kv", b_kv)]

    def step(self):
        for _, fn in self.phases():
            fn()

    def kernels_per_step(self):
        # nc: reduce+sum, readout, bwd_q+sum+dscale, bwd_kv+dscale
        # causal: totals+scan, fwd, bwd_q+scan+dscale, bwd_kv+dscale
        n = 8
        if self.group is not None and self.causal:
            n += 2   # the two offset adds
        return n

    def phase_bytes(self):
        """Algorithmic HBM bytes per token of each phase (I/O of the function)."""
        e = torch.tensor([], dtype=self.dtype).element_size() * D
        if self.causal:
            return {"forward_reduce": 2 * e, "forward_readout": 4 * e, "backward_q": 5 * e,
                    "backward_kv": 6 * e}
        return {"forward_reduce": 2 * e, "forward_readout": 2 * e, "backward_q": 3 * e,
                "backward_kv": 4 * e}


# Measured DRAM bytes (read + write) of the dominant phase's main kernel per
# launch and token.  fp32 entries: one step captured at 2^19 tokens with
#   ncu --set full --clock-control none -k regex:k_t5_ (or k_c5_) python bench.py
#       --variants noncausal_f32 (or causal_f32) --tokens 524288 --steps 2 --warmup 3
#       --no-e2e --no-cpu --no-strong --no-shapes
# bf16 entries: ncu --metrics gpu__time_duration.sum,dram__bytes_read.sum,
# dram__bytes_write.sum --clock-control none -k regex:'k_t5_|k_c5_' python bench.py
# --variants noncausal_bf16,causal_bf16 --tokens 262144 --steps 2 --warmup 3
# --no-e2e --no-cpu --no-strong --no-shapes (2^18 tokens).
TRAFFIC_PER_TOKEN = {
    (False, "f32", "backward_kv"): (268.58e6 + 221.34e6) / 2 ** 19,
    (False, "f32", "backward_q"): (268.51e6 + 105.29e6) / 2 ** 19,
    (False, "bf16", "backward_kv"): (67.18e6 + 18.79e6) / 2 ** 18,
    (False, "bf16", "backward_q"): (67.17e6 + 3.48e6) / 2 ** 18,
    (True, "f32", "backward_kv"): (381.16e6 + 229.57e6) / 2 ** 19,
    (True, "f32", "backward_q"): (337.17e6 + 144.85e6) / 2 ** 19,
    (True, "bf16", "backward_kv"): (124.33e6 + 33.24e6) / 2 ** 18,
    (True, "bf16", "backward_q"): (102.28e6 + 20.94e6) / 2 ** 18,
}


def timed(fn, steps, warmup, group, device):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(device)
    if group is not None:
        torch.distributed.barrier(group)
    torch.cuda.synchronize(device)
    stream = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1)
    if group is not None:
        t = torch.tensor([ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX, group=group)
        ms = float(t.item())
        torch.distributed.barrier(group)
    return ms / steps


def phase_times(layer, steps, device):
    """Average per-phase device time (CUDA events on the launching stream)."""
    stream = torch.cuda.current_stream(device)
    names = [n for n, _ in layer.phases()]
    acc = {n: 0.0 for n in names}
    for _ in range(steps):
        evs = []
        for name, fn in layer.phases():
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            evs.append((name, a, b))
        torch.cuda.synchronize(device)
        for name, a, b in evs:
            acc[name] += a.elapsed_time(b)
    return {n: acc[n] / steps for n in names}


def e2e_rate(causal, dtype, tokens, steps, device, group=None, pipelined=True):
    """Same metric through a public API with pinned HOST buffers: H2D of q, k,
    v, dO and D2H of out, dq, dk, dv inside the timed region, every step.
    pipelined: ``streaming.fwd_bwd_host`` (token chunks, copies on side
    streams overlapping the kernels and each other); otherwise the autograd
    path (``race_attention`` + ``backward``) with whole-tensor copies on the
    launching stream.  Every rank runs its own shard of the sequence; the time
    is taken with CUDA events on the launching stream (which waits for the
    copy streams) and the maximum over ranks is used."""
    from race_attention_b200 import race_attention
    from race_attention_b200.streaming import fwd_bwd_host
    world = 1 if group is None else torch.distributed.get_world_size(group)
    rank = 0 if group is None else torch.distributed.get_rank(group)
    g = torch.Generator().manual_seed(1 + rank)
    shape = (1, tokens, 1, D)
    host = [torch.randn(shape, generator=g).to(dtype).pin_memory() for _ in range(4)]
    outs = [torch.empty(shape, dtype=dtype).pin_memory() for _ in range(4)]
    planes = torch.randn((1, K * L, D), generator=torch.Generator().manual_seed(0)).to(device)
    lt = torch.zeros((), device=device, requires_grad=True)

    def step_autograd():
        q, k, v, do = (h.to(device, non_blocking=True) for h in host)
        for t in (q, k, v):
            t.requires_grad_(True)
        out = race_attention(q, k, v, planes, K, L, lt.exp().clamp(1e-2, 20.0), causal=causal,
                             group=group)
        out.backward(do)
        for dst, src in zip(outs, (out, q.grad, k.grad, v.grad)):
            dst.copy_(src.detach(), non_blocking=True)
        lt.grad = None

    def step_pipelined():
        sc = lt.exp().clamp(1e-2, 20.0)
        *_, ds = fwd_bwd_host(*host, planes, K, L, sc.detach(), causal=causal, device=device,
                              outputs=outs, group=group)
        # the temperature gradient through exp().clamp(), as autograd would give it
        torch.autograd.backward(sc, ds)
        lt.grad = None

    step = step_pipelined if pipelined else step_autograd
    step()
    dt = timed(step, steps, 0, group, device) / 1e3
    nbytes = tokens * D * torch.tensor([], dtype=dtype).element_size() * 4
    return {"value": world * tokens / dt, "unit": "tokens/s", "h2d_bytes_per_step": nbytes,
            "d2h_bytes_per_step": nbytes, "steps": steps, "per_rank_shard_tokens": tokens,
            "api": ("race_attention_b200.streaming.fwd_bwd_host (pinned host buffers, "
                    "chunked copies overlapping the kernels)") if pipelined else
                   "race_attention autograd on device copies of pinned host buffers"}


def cpu_rate(causal, tokens, budget_s=20.0, iters_max=50, iters_min=3):
    """Reference op sequence on the host cores (float32, all threads), on the
    full workload: at least ``iters_min`` steps, then until ``budget_s``."""
    from oracle import torch_ref
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, tokens, D, generator=g).requires_grad_(True) for _ in range(3))
    dout = torch.randn(1, tokens, D, generator=g)
    planes_T = torch.randn(K * L, D, generator=g).T
    protos = torch_ref.protos_T(K)
    scale = torch.tensor(1.0)
    torch_ref.fwd_bwd(q, k, v, planes_T, K, L, scale, protos, dout, causal)   # warm-up
    times = []
    t_start = time.perf_counter()
    while len(times) < iters_min or (len(times) < iters_max and
                                     (time.perf_counter() - t_start) < budget_s):
        t0 = time.perf_counter()
        torch_ref.fwd_bwd(q, k, v, planes_T, K, L, scale, protos, dout, causal)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {"value": tokens / med, "unit": "tokens/s", "cores": threads, "kind": "port",
            "cpu": cpu_model(),
            "sample": f"{'causal' if causal else 'non-causal'} fp32 fwd+bwd, B1 H1 T={tokens} "
                      f"d{D} K{K} L{L}, torch CPU restatement of the reference op sequence, "
                      f"median of {len(times)}"}


def run_ours(args):
    world, rank, local = dist_env()
    group = None
    if world > 1:
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", device_id=torch.device("cuda", local))
        group = torch.distributed.group.WORLD
    device = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(device)
    peak, peak_kind = load_peak()

    # (causal, dtype, normalize): the last is the global-normalised causal mode
    configs = [(False, torch.float32, 0), (True, torch.float32, 0), (False, torch.bfloat16, 0),
               (True, torch.bfloat16, 0), (True, torch.float32, 1)]
    if args.variants:   # profiling runs: a subset of the variants (the first listed leads)
        names = {"noncausal_f32": 0, "causal_f32": 1, "noncausal_bf16": 2, "causal_bf16": 3,
                 "global_f32": 4}
        configs = [configs[names[v]] for v in args.variants.split(",")]
    results = []
    head = None
    clocks = None
    for i, (causal, dtype, norm) in enumerate(configs):
        layer = Layer(causal, dtype, args.tokens, group, device, seed=1000 + rank, normalize=norm)
        sampler = ClockSampler(device.index) if (i == 0 and rank == 0) else None
        steps = args.steps if i == 0 else min(args.steps, VARIANT_STEPS)
        if sampler:
            sampler.__enter__()
        ms = timed(layer.step, steps, args.warmup, group, device)
        if sampler:
            sampler.__exit__()
            clocks = sampler.summary()
        total_tokens = args.tokens * world
        esize = torch.tensor([], dtype=dtype).element_size()
        rec = {"causal": causal, "dtype": "f32" if dtype == torch.float32 else "bf16",
               "value": total_tokens / (ms / 1e3), "ms_per_step": ms,
               "step_roofline_frac": (args.tokens * 11 * D * esize / (ms / 1e3) / 1e9) / peak}
        if norm:
            rec["normalize"] = "global"
        rec["steps"] = steps
        if world == 1:
            ph = phase_times(layer, max(3, min(args.steps, VARIANT_STEPS) // 2), device)
            pb = layer.phase_bytes()
            rec["phases_ms"] = ph
            dom = max(ph, key=ph.get)
            ach = pb[dom] * args.tokens / (ph[dom] / 1e3) / 1e9
            tr = None if norm else TRAFFIC_PER_TOKEN.get((causal, rec["dtype"], dom))
            rec["roofline"] = {"bound": "hbm", "kernel": dom, "achieved": ach, "peak": peak,
                               "unit": "GB/s", "frac": ach / peak,
                               "traffic": None if tr is None else tr * args.tokens,
                               "peak_kind": peak_kind}
            if tr is not None:
                rec["roofline"]["traffic_note"] = (
                    "DRAM read+write bytes per launch from one ncu capture at 2^19 (fp32) or "
                    "2^18 (bf16) tokens, scaled by tokens; reads equal the algorithmic bytes, writes of the last "
                    "tiles are still in L2 when a launch ends")
        rec["gpu_launches_per_step"] = layer.kernels_per_step()
        results.append(rec)
        if i == 0:
            head = (layer, rec)
        else:
            del layer
        torch.cuda.empty_cache()

    strong = None if args.no_strong else strong_scaling(args, world, group, device)
    shapes = baseline_shapes(args, device) if (world == 1 and not args.no_shapes) else None
    parity = sharded_parity(group, device) if world > 1 else None

    layer, rec = head
    line = {
        "metric": METRIC, "value": rec["value"], "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": rec["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: q,k,v,dO ~ N(0,1), hyperplanes ~ N(0,1), seed 0",
        "config": {"workload": "single non-causal RACE layer fwd+bwd, sequence-sharded",
                   "batch": 1, "heads": 1, "tokens_per_gpu": args.tokens,
                   "tokens_total": args.tokens * world, "head_dim": D, "K": K, "L": L,
                   "temperature": 1.0, "parallelism": f"seq{world}",
                   "l2": "inputs larger than L2 (q,k,v,dO 256 MiB each in fp32), no flush"},
        "gpu_launches": rec["gpu_launches_per_step"] * args.steps,
        "clocks": clocks,
        "variants": results[1:],
        "step_roofline_frac": rec["step_roofline_frac"],
        "dscale": "rank-local per step (each rank's tokens); a training step sums it with the "
                  "model's other parameter gradients, so the timed step runs 2 collectives",
    }
    if strong is not None:
        line["strong_64M"] = strong
    if shapes is not None:
        line["baseline_shapes"] = shapes
    if parity is not None:
        line["sharded_parity"] = parity
    if world == 1:
        line["roofline"] = rec["roofline"]
        line["phases_ms"] = rec["phases_ms"]
    del layer
    torch.cuda.empty_cache()
    if not args.no_e2e:
        line["e2e"] = e2e_rate(False, torch.float32, args.tokens, args.e2e_steps, device, group)
        line["e2e_autograd"] = e2e_rate(False, torch.float32, args.tokens, args.e2e_steps, device,
                                        group, pipelined=False)
    if world > 1:
        torch.distributed.barrier()
    if rank == 0 and not args.no_cpu and world == 1:
        line["cpu_baseline"] = cpu_rate(False, args.tokens)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def strong_scaling(args, world, group, device):
    """One fixed 64M-token sequence (STRONG_TOKENS) sharded over the ranks:
    2^26 / N tokens per GPU, non-causal fp32 fwd+bwd, the same 2 collectives
    per step.  Efficiency against N = 1 is (t1 / tN) / N across the lines of
    a 1/2/4/8 sweep."""
    tokens = STRONG_TOKENS // world
    need = tokens * D * 4 * 8 + (1 << 30)          # 8 token tensors + state / slack
    free, _ = torch.cuda.mem_get_info(device)
    ok = torch.tensor([1.0 if free > need else 0.0], device=device)
    if group is not None:
        torch.distributed.all_reduce(ok, op=torch.distributed.ReduceOp.MIN, group=group)
    if ok.item() < 1.0:
        return {"skipped": f"needs {need / 2**30:.0f} GiB per GPU, {free / 2**30:.0f} GiB free"}
    layer = Layer(False, torch.float32, tokens, group, device, seed=2000 + (0 if group is None
                                                                             else dist_env()[1]))
    steps = 10
    ms = timed(layer.step, steps, 3, group, device)
    del layer
    torch.cuda.empty_cache()
    return {"tokens_total": STRONG_TOKENS, "tokens_per_gpu": tokens, "steps": steps,
            "ms_per_step": ms, "value": STRONG_TOKENS / (ms / 1e3), "unit": "tokens/s",
            "scaling": "strong"}


def baseline_shapes(args, device):
    """The BASELINE configs' own layer shapes on one GPU (many independent
    (b, h) streams: the replica case, no collective): C3 ViT (B 256, H 6,
    785 tokens, K4 L4 = 64 buckets, fp32, non-causal), C2 (B 4, H 12, 16384
    tokens, bf16, causal), C4 (B 1, H 12, 65536 tokens, bf16, causal).
    tokens/s counts B * T per layer call; head-tokens/s counts B * H * T."""
    res = []
    for name, b, t, h, bits, tables, causal, dtype in (
            ("C3_vit", 256, 785, 6, 4, 4, False, torch.float32),
            ("C2_causal", 4, 16384, 12, 2, 5, True, torch.bfloat16),
            ("C4_long_causal", 1, 65536, 12, 2, 5, True, torch.bfloat16)):
        layer = Layer(causal, dtype, t, None, device, seed=3000, batch=b, heads=h, bits=bits,
                      tables=tables)
        ms = timed(layer.step, 20, 3, None, device)
        res.append({"config": name, "batch": b, "heads": h, "tokens": t, "K": bits, "L": tables,
                    "causal": causal, "dtype": "f32" if dtype == torch.float32 else "bf16",
                    "ms_per_step": ms, "tokens_per_s": b * t / (ms / 1e3),
                    "head_tokens_per_s": b * h * t / (ms / 1e3)})
        del layer
        torch.cuda.empty_cache()
    return res


def sharded_parity(group, device):
    """Correctness of the sequence-sharded path on this run's GPUs: two
    streams of 20480 tokens (non-causal and causal, fp32) through
    race_attention(group=...), every rank holding its contiguous token range;
    rank 0 gathers out, dq, dk, dv and compares them with the same sequence
    run unsharded on its own GPU.  Returns the worst relative L2 per mode."""
    from race_attention_b200 import race_attention
    world = torch.distributed.get_world_size(group)
    rank = torch.distributed.get_rank(group)
    T = 20480
    g = torch.Generator(device=device).manual_seed(77)
    full = [torch.randn((1, 2, T, 1, D), generator=g, device=device) for _ in range(4)]
    planes = torch.randn((1, K * L, D), generator=g, device=device)
    per = T // world
    res = {}
    for causal in (False, True):
        def run(xs, grp):
            leaves = [x.clone().requires_grad_(True) for x in xs[:3]]
            out = race_attention(*leaves, planes, K, L, 1.1, causal=causal, group=grp)
            out.backward(xs[3])
            return [out.detach()] + [x.grad.detach() for x in leaves]
        shard = [x[:, :, rank * per:(rank + 1) * per].contiguous() for x in full]
        got = run(shard, group)
        gathered = []
        for t in got:
            parts = [torch.empty_like(t) for _ in range(world)]
            torch.distributed.all_gather(parts, t.contiguous(), group=group)
            gathered.append(torch.cat(parts, dim=2))
        if rank == 0:
            ref = run(full, None)
            errs = [float((a - b).norm() / b.norm()) for a, b in zip(gathered, ref)]
            res["causal" if causal else "noncausal"] = max(errs)
    torch.distributed.barrier(group)
    if rank == 0:
        res["streams"], res["tokens"] = 2, T
    return res if rank == 0 else None


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    tokens = args.tokens
    from oracle import torch_ref
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, tokens, D, generator=g).requires_grad_(True) for _ in range(3))
    dout = torch.randn(1, tokens, D, generator=g)
    planes_T = torch.randn(K * L, D, generator=g).T
    protos = torch_ref.protos_T(K)
    scale = torch.tensor(1.0)
    for _ in range(min(args.warmup, 3)):
        torch_ref.fwd_bwd(q, k, v, planes_T, K, L, scale, protos, dout, False)
    # every step is the full 2^20-token workload; the run stops after --steps
    # steps or once 60 s have been timed, whichever comes first
    done = 0
    t0 = time.perf_counter()
    while done < args.steps and (done < 3 or time.perf_counter() - t0 < 60.0):
        torch_ref.fwd_bwd(q, k, v, planes_T, K, L, scale, protos, dout, False)
        done += 1
    dt = (time.perf_counter() - t0) / done
    val = tokens / dt
    sample = (f"non-causal fp32 fwd+bwd, B1 H1 T={tokens} (the full workload) d{D} K{K} L{L}: "
              f"torch CPU restatement of the reference op sequence, {done} timed steps")
    line = {
        "metric": METRIC, "value": val, "unit": "tokens/s", "n_gpus": world, "steps": done,
        "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "impl": "reference",
        "data": "synthetic: q,k,v,dO ~ N(0,1), seed 0",
        "config": {"workload": "single non-causal RACE layer fwd+bwd, sequence-sharded",
                   "batch": 1, "heads": 1, "tokens_per_gpu": args.tokens, "head_dim": D,
                   "K": K, "L": L, "parallelism": f"seq{world}",
                   "l2": "host run"},
        "cpu_baseline": {"value": val, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "cpu": cpu_model(), "sample": sample},
        "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1200)   # ~1.1 s timed at 2^20 tokens
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--tokens", type=int, default=TOKENS)
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--no-strong", action="store_true")
    ap.add_argument("--no-shapes", action="store_true")
    ap.add_argument("--variants", default="",
                    help="comma list of noncausal_f32, causal_f32, noncausal_bf16, causal_bf16, "
                         "global_f32 (default: all, headline first); for profiling runs")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
