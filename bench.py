"""Benchmark of the quantized-MoE expert hot path on B200 (and the reference CPU arm).

Workload (one "step"): batch-1 decode of one token through the 48 MoE FFN layers of a
Qwen3-30B-A3B-shaped decoder: hidden 2048, 128 experts, top-8
softmax routing with renormalisation, expert intermediate 768, Q4_K gate/up, Q6_K down,
f32 router; each layer is QuestWend's ffn_norm + build_moe graph (rms_norm * ffn_norm
weight -> router mul_mat -> route -> 3x mul_mat_id -> swiglu -> weighted sum) plus the
residual add, chained so layer l+1 routes on layer l's output.  Attention, norms and the output head are outside the hot
path and not run.  All 48 x 128 x 3 expert matrices are resident in HBM (18.8 GB), so a
step streams ~1.17 GB of distinct expert weights, far more than the 126 MB L2: inputs
are larger than L2, no flush is needed.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl qwb|reference]

Prints one JSON line (rank 0).  `value` is decode tokens/s of the whole job.  At N = 1 the
step is the fused single-GPU layer (qwb_moe_ffn).  At N > 1 the experts are sharded over
the ranks (expert parallelism: rank r holds experts [r*128/N, (r+1)*128/N) of every layer)
and a step decodes N tokens, one per rank ("scaling": "weak"): every rank holds all N
tokens' hidden states, routes them (replicated router) and runs its own experts over the
pairs routed to them (one qwb_moe_ep_layer call per layer), and one NCCL all-reduce per
layer sums the partial outputs (questwend_b200.expert_parallel).  `ep_nrmse` compares one
such layer with the fused single-GPU layer on the same tokens (the run fails above 1e-5).
`ep_config4` (every N) runs the 235B-A22B layer shape (hidden 4096, expert FFN 1536) the
same way at decode batches of 1, 8 and 64 tokens with the aggregate HBM roofline.  `e2e` is
the same metric through the public C ABI with
the token's hidden state copied from pinned host memory and the layer output copied back
every step.  `roofline` is the gate/up GEMV kernel (the largest weight stream per layer)
at N = 1 and the whole step's aggregate HBM bytes over N x peak at N > 1.
`cpu_baseline` times the reference's own ggml CPU backend (oracle/_ref, built from the
reference sources) on one layer of the same shapes, scaled to 48 layers.

`prefill` (rank 0): the prefill grouped-GEMM sweep of MUL_MAT_ID on
Q4_K experts (hidden 4096, 128 experts, top-8, expert intermediate 1536; gate/up shape
[4096 -> 1536] with one activation row per token and down shape [1536 -> 4096] with one
per (token, slot)), n_tokens in {512, 2048, 8192}, routing from Gumbel-perturbed
Zipf(1.1) expert popularity.  TFLOPS = 2 * T * 8 * K * M / time: `tflops` for the whole
qwb_mul_mat_id call (activation quantisation, expert sort, B-tile gather, GEMM), `gemm_tflops`
for the tensor-core kernel alone (event marks around it).  The weights of all 128 experts
(453 MB per matrix) exceed L2.  Its `roofline` compares the GEMM kernel with the measured
dense bf16 peak; its `cpu_baseline` times the reference CPU backend on T = 512, gate shape.

`decode_mmid` (rank 0): the large-model expert shape (hidden 4096 -> expert FFN 1536,
128 Q4_K experts, top-8) as a decode-batch MUL_MAT_ID at T = 1, 8, 64 tokens, the path a
ggml backend takes for a decode graph's MUL_MAT_ID nodes (weight streaming: each selected
expert row read once for all its tokens).  GB/s counts the distinct expert weights per
call; `frac` is against the measured HBM copy bandwidth, for the whole call (`us`) and for
the streaming kernel alone (`kernel_us`).

`gathers` (rank 0): GET_ROWS on a 151936 x 4096 embedding table stored as
Q4_K / Q6_K / Q8_0 with index streams of n = 1, 512, 8192 (uniform, 50 % repeats; bytes =
n x (row + 16 KB f32 written + index)) - and the decoder's Q6_K output head [2048 -> 151936]
(255 MB) as quantized MUL_MAT at T = 1 and 8 tokens.
"""
from __future__ import annotations

import argparse
import functools
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

H, F, E, K_USED, LAYERS = 2048, 768, 128, 8, 48
# dram__bytes_read.sum + dram__bytes_write.sum of one gate/up decode launch, from an ncu
# capture of this kernel at these shapes (one token, 4-layer stack: the same launch shape)
GATEUP_TRAFFIC_BYTES = 14_179_584
Q4_K, Q6_K = 12, 14
ROW_GU = H // 256 * 144        # bytes per gate/up row
ROW_D = F // 256 * 210         # bytes per down row
EXPERT_GU = F * ROW_GU         # 884,736 B
EXPERT_D = H * ROW_D           # 1,290,240 B
UNIQUE = 32                    # distinct quantized experts per role, tiled over 128 x 48


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], "measured"
    except Exception:
        return 6650.0, "fallback"


Q8_0 = 8


def synth_blocks(t, n_rows, K, rng):
    """n_rows rows of K weights as valid ggml blocks of type t: uniformly random quantized
    codes with fp16 scales sized so the dequantized weights are of the magnitude of a
    quantized N(0, 0.02) matrix (|w| <~ 0.02-0.04).  The kernels' work and bytes do not
    depend on the values; these only keep every output finite."""
    def f16(lo, hi, n):
        return rng.uniform(lo, hi, n).astype(np.float16).view(np.uint8).reshape(n, 2)
    if t == Q4_K:  # d, dmin fp16 | 12 packed 6-bit scales / mins | 128 B nibbles
        nb = n_rows * (K // 256)
        b = rng.integers(0, 256, (nb, 144), dtype=np.uint8)
        b[:, 0:2] = f16(1.5e-5, 2.5e-5, nb)
        b[:, 2:4] = f16(1.5e-4, 2.5e-4, nb)
    elif t == Q6_K:  # 128 B low bits | 64 B high bits | 16 int8 scales | d fp16
        nb = n_rows * (K // 256)
        b = rng.integers(0, 256, (nb, 210), dtype=np.uint8)
        b[:, 192:208] = rng.integers(-64, 64, (nb, 16), dtype=np.int8).view(np.uint8)
        b[:, 208:210] = f16(0.8e-5, 1.2e-5, nb)
    else:  # Q8_0: d fp16 | 32 int8
        nb = n_rows * (K // 32)
        b = rng.integers(0, 256, (nb, 34), dtype=np.uint8)
        b[:, 0:2] = f16(1.2e-4, 1.8e-4, nb)
    return b.reshape(-1)


def quantized_experts(seed=0):
    """UNIQUE distinct expert matrices per role (gate/up Q4_K [H -> F], down Q6_K [F -> H])
    of synthetic quantized blocks (synth_blocks)."""
    out = []
    for role in range(3):
        rng = np.random.default_rng(seed * 1000 + role)
        t, rows, K = (Q4_K, F, H) if role < 2 else (Q6_K, H, F)
        out.append(synth_blocks(t, UNIQUE * rows, K, rng))
    return out


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms while running."""

    def __init__(self, index):
        self.index, self.proc, self.lines = index, None, []

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
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
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
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
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_info():
    """Host CPU model, logical CPU count and the ISA extensions the reference build uses."""
    model, isa = None, []
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if model is None and ln.startswith("model name"):
                    model = ln.split(":", 1)[1].strip()
                if ln.startswith("flags"):
                    fl = set(ln.split(":", 1)[1].split())
                    isa = [x for x in ("avx2", "fma", "f16c", "avx512f", "avx512bw", "avx512_vnni",
                                       "avx512_bf16", "amx_tile", "amx_int8") if x in fl]
                    break
    except OSError:
        pass
    return {"model": model, "logical_cpus": os.cpu_count(), "isa": isa}


def host_threads():
    """Threads the host can run at once for this process: the CPUs in its affinity mask,
    capped by a cgroup CPU quota when one is set (spinning ggml worker threads beyond
    what the quota allows slow the CPU backend down instead of speeding it up)."""
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    try:
        with open("/sys/fs/cgroup/cpu.max") as f:
            quota, period = f.read().split()[:2]
        if quota != "max":
            n = min(n, max(1, int(int(quota) // int(period))))
    except (OSError, ValueError):
        pass
    return max(1, n)


def stats(ms):
    a = np.asarray(ms, dtype=np.float64)
    return {"median": float(np.median(a)), "p10": float(np.percentile(a, 10)),
            "p90": float(np.percentile(a, 90)), "n": int(a.size)}


@functools.lru_cache(maxsize=1)
def _cpu_decode_inputs():
    g, u, d = quantized_experts()
    reps = E // UNIQUE
    gate, up, down = (np.tile(a, reps) for a in (g, u, d))
    rng = np.random.default_rng(1)
    rw = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    x = rng.standard_normal((1, H)).astype(np.float32)
    nw = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    return gate, up, down, rw, x, nw


def cpu_decode_layer_times(threads, samples, warm=3):
    """ms of each of `samples` evaluations of one MoE layer (config-1 shapes: ffn_norm,
    router, top-8, Q4_K gate/up, Q6_K down, weighted sum) on the reference's ggml CPU
    backend (oracle/_ref) with `threads` threads, after `warm` untimed evaluations."""
    import oracle as O
    if not O.ref_available():
        return None
    O.set_ref_threads(threads)
    gate, up, down, rw, x, nw = _cpu_decode_inputs()
    O.moe_layer(x, rw, Q4_K, gate, up, Q6_K, down, F, E, K_USED, impl="ref", iters=warm + samples,
                norm_w=nw, norm_eps=1e-6)
    return O.ref_last_times()[warm:]


def cpu_prefill_times(threads, samples, warm=1):
    """ms of each of `samples` reference CPU MUL_MAT_ID calls at T = 512, gate/up shape of
    the prefill sweep (Q4_K, hidden 4096 -> 1536, 128 experts, top-8, Zipf routing)."""
    import oracle as O
    if not O.ref_available():
        return None
    O.set_ref_threads(threads)
    T = PF_TOKENS[0]
    ids = zipf_ids(T, E, K_USED, seed=T)
    x = np.random.default_rng(3).standard_normal((T, 1, PF_H)).astype(np.float32)
    w = np.tile(prefill_experts()[0], E // PF_UNIQUE)
    O.mul_mat_id(Q4_K, w, PF_H, PF_F, E, x, ids, impl="ref", iters=warm + samples)
    return O.ref_last_times()[warm:]


def run_cpu_leg(args):
    """--cpu-leg: the reference CPU timings for the GPU arm's cpu_baseline, in a process of
    its own (no CUDA context, no torch threads): decode layer and prefill call, with all
    host threads and with one."""
    nproc = host_threads()
    out = {"cpu": cpu_info()}
    for name, threads, n in (("decode", nproc, 300), ("decode_1t", 1, 60)):
        t = cpu_decode_layer_times(threads, n)
        out[name] = None if t is None else dict(stats(t), threads=threads)
    if not args.no_prefill:
        for name, threads, n in (("prefill", nproc, 8), ("prefill_1t", 1, 2)):
            t = cpu_prefill_times(threads, n)
            out[name] = None if t is None else dict(stats(t), threads=threads)
    print(json.dumps(out))


def cpu_leg_subprocess(no_prefill):
    """Runs --cpu-leg in a fresh interpreter and returns its JSON (None on failure)."""
    cmd = [sys.executable, os.path.abspath(__file__), "--cpu-leg"] + (["--no-prefill"] if no_prefill else [])
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
        return json.loads(r.stdout.strip().splitlines()[-1])
    except Exception as ex:  # the baseline is reported, never required
        print(f"cpu leg failed: {ex}", file=sys.stderr)
        return None


def run_reference(args):
    """--impl reference: the reference's own CPU path, all host threads, same workload.
    A step = 5 evaluations of one MoE layer (config-1 shapes) scaled by the 48 layers."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle as O
    threads = host_threads()
    if not O.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref not built (needs the reference sources)"}))
        return
    cpu_decode_layer_times(threads, 5)  # first-touch of the 340 MB expert tables, thread pool start
    for _ in range(args.warmup):
        cpu_decode_layer_times(threads, 5, warm=1)
    per_step = [float(np.mean(cpu_decode_layer_times(threads, 5, warm=1))) * LAYERS for _ in range(args.steps)]
    ms = float(np.mean(per_step))
    tok_s = 1000.0 / ms
    sample = (f"one MoE layer (config-1 shapes, Q4_K gate/up, Q6_K down) x 5 evaluations per step, "
              f"scaled x{LAYERS} layers")
    print(json.dumps({
        "impl": "reference", "metric": "decode_tokens_per_s", "value": tok_s, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "step_ms": stats(per_step),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "q4_K/q6_K x q8_K -> f32",
        "data": "synthetic", "config": workload_config(args.gpus),
        "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": threads, "kind": "reference",
                         "sample": sample, "cpu": cpu_info()},
        "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


PF_H, PF_F, PF_UNIQUE, PF_TOKENS = 4096, 1536, 8, (512, 2048, 8192)


def zipf_ids(T, n_exp, n_used, seed, s=1.1):
    """top-n_used of log Zipf(s) popularity (seeded expert ranks) + Gumbel noise."""
    r = np.random.default_rng(seed)
    pop = 1.0 / np.arange(1, n_exp + 1, dtype=np.float64) ** s
    logits = np.log(pop[r.permutation(n_exp)])[None, :] + r.gumbel(size=(T, n_exp))
    return np.argsort(-logits, axis=1, kind="stable")[:, :n_used].astype(np.int32)


@functools.lru_cache(maxsize=1)
def prefill_experts(seed=7):
    """PF_UNIQUE distinct Q4_K experts for the gate/up shape [PF_H -> PF_F] and the down
    shape [PF_F -> PF_H] of synthetic quantized blocks (synth_blocks)."""
    out = []
    for role in range(2):
        rng = np.random.default_rng(seed * 1000 + role)
        rows, k = (PF_F, PF_H) if role == 0 else (PF_H, PF_F)
        out.append(synth_blocks(Q4_K, PF_UNIQUE * rows, k, rng))
    return out


MMID_TOKENS = (1, 8, 64)  # decode batches of the large-model expert shape


def decode_mmid_sweep(q, lib, dev, tokens=MMID_TOKENS, n_pools=8):
    """Decode-batch MUL_MAT_ID (large-model expert shape: hidden 4096 -> expert FFN 1536,
    128 Q4_K experts, top-8 of uniform random routing) at T = 1, 8, 64 tokens: the
    weight-streaming path qwb_mul_mat_id takes for few tokens per expert.  Timed from CUDA
    graph replays of 8 calls; call i reads pool i of 8 identical expert pools, so the
    bytes touched between two reads of a pool exceed L2 (and the calls are not L2 hits).
    GB/s counts the distinct expert weights a call streams (experts touched x 3.54 MB)."""
    import ctypes as C

    import torch

    from questwend_b200 import _lib as L
    experts = prefill_experts()[0]  # gate/up shape [PF_H -> PF_F], PF_UNIQUE distinct matrices
    reps = E // PF_UNIQUE
    per = experts.size // PF_UNIQUE
    base = torch.from_numpy(experts).to(dev)
    n_call = 8
    pools = []
    for _ in range(n_pools):
        buf = torch.empty(base.numel() * reps, dtype=torch.uint8, device=dev)
        buf.view(reps, -1).copy_(base.expand(reps, -1))
        pools.append(q.QTensor(buf, Q4_K, (PF_H, PF_F, E, 1)))
    hbm, kind = peaks()
    rng = np.random.default_rng(11)
    s = torch.cuda.Stream()
    points = []
    for T in tokens:
        ids_np = np.stack([rng.permutation(E)[:K_USED] for _ in range(T)]).astype(np.int32)
        ids = torch.from_numpy(ids_np).to(dev)
        b = torch.randn((T, 1, PF_H), device=dev)
        out = torch.empty((T, K_USED, PF_F), device=dev)
        for i in range(3):
            q.mul_mat_id(pools[i % n_pools], b, ids, out)
        torch.cuda.synchronize()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
            for i in range(n_call):
                q.mul_mat_id(pools[i % n_pools], b, ids, out)
        # per-kernel marks: a one-call graph with event records around the kernels
        L.check("qwb_profile_enable", lib.qwb_profile_enable(8))
        g1 = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s), torch.cuda.graph(g1, stream=s):
            lib.qwb_profile_reset()
            q.mul_mat_id(pools[0], b, ids, out)
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        calls, kern = [], []
        for _ in range(10):
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            calls.append(e0.elapsed_time(e1) / n_call)
            for p_ in pools[1:4]:  # evict pool 0 before the marked call
                p_.data[: 64 << 20].add_(0)
            g1.replay()
            torch.cuda.synchronize()
            n = lib.qwb_profile_count() - 1
            ms = (C.c_float * max(n, 1))()
            tg = (C.c_int32 * max(n, 1))()
            L.check("qwb_profile_read", lib.qwb_profile_read(ms, tg, n))
            kern.append(sum(m for m, t in zip(ms[:n], tg[:n]) if t == 6))
        L.check("qwb_profile_enable", lib.qwb_profile_enable(0))
        del g, g1
        assert torch.isfinite(out).all()
        wbytes = len(np.unique(ids_np)) * per
        c_ms, k_ms = float(np.median(calls)), float(np.median(kern))
        points.append({"tokens": T, "experts_touched": int(len(np.unique(ids_np))), "weight_mb": wbytes / 1e6,
                       "us": 1e3 * c_ms, "gbs": wbytes / (c_ms * 1e-3) / 1e9, "frac": wbytes / (c_ms * 1e-3) / 1e9 / hbm,
                       "kernel_us": 1e3 * k_ms,
                       "kernel_gbs": wbytes / (k_ms * 1e-3) / 1e9 if k_ms > 0 else None,
                       "kernel_frac": wbytes / (k_ms * 1e-3) / 1e9 / hbm if k_ms > 0 else None})
    del pools
    torch.cuda.empty_cache()
    return {"config": {"workload": "C4 decode-batch MUL_MAT_ID, Q4_K x Q8_K, weight streaming", "hidden": PF_H,
                       "expert_ffn": PF_F, "experts": E, "top_k": K_USED, "routing": "uniform random",
                       "tokens": list(tokens),
                       "l2": f"{n_pools} pools of all 128 experts, call i reads pool i mod {n_pools}"},
            "peak": hbm, "peak_kind": kind, "points": points}


VOCAB, EMB = 151936, 4096  # embedding table rows x width; the decoder's output head is VOCAB x H
GATHER_N = (1, 512, 8192)


def _graph_time(fn, n_call=8, reps=10):
    """Median ms per call of fn(i), i = 0..n_call-1, from CUDA graph replays."""
    import torch
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    for i in range(3):
        fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
        for i in range(n_call):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ts = []
    for _ in range(reps):
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1) / n_call)
    del g
    return float(np.median(ts))


def gathers_sweep(q, dev):
    """GET_ROWS on the embedding table and the decoder's output head.
    GET_ROWS on a 151936 x 4096 table stored as Q4_K / Q6_K / Q8_0 (350 / 510 / 661 MB)
    with index streams of n = 1, 512, 8192 rows, uniform random with 50 % repeats; 8 index
    sets rotate between calls so the rows read are not L2 hits.  Bytes = n x (row bytes +
    16,384 B written + 4 B index).  Output head: qwb_mul_mat of the Q6_K [2048 -> 151936]
    matrix (255 MB) at T = 1 and 8 tokens.  Tables: 512 distinct synthetic rows tiled."""
    import torch
    hbm, kind = peaks()
    rng = np.random.default_rng(5)
    out = {"peak": hbm, "peak_kind": kind, "get_rows": [], "output_head": []}
    for t in (Q4_K, Q6_K, Q8_0):
        rows = synth_blocks(t, 512, EMB, rng)
        rb = rows.size // 512
        tab = torch.empty(VOCAB * rb, dtype=torch.uint8, device=dev)
        reps = -(-VOCAB // 512)
        src = torch.from_numpy(rows).to(dev).view(1, -1).expand(reps, -1).reshape(-1)
        tab.copy_(src[:VOCAB * rb])
        T = q.QTensor(tab, t, (EMB, VOCAB, 1, 1))
        for n in GATHER_N:
            sets = []
            for _ in range(8):
                base = rng.integers(0, VOCAB, max(1, (n + 1) // 2))
                idx = np.concatenate([base, rng.choice(base, n - base.size)]) if n > 1 else base
                sets.append(torch.from_numpy(rng.permutation(idx).astype(np.int32)).to(dev))
            dst = torch.empty((1, 1, n, EMB), device=dev)
            ms = _graph_time(lambda i: q.get_rows(T, sets[i % 8], dst))
            nbytes = n * (rb + EMB * 4 + 4)
            out["get_rows"].append({"type": {12: "Q4_K", 14: "Q6_K", 8: "Q8_0"}[t], "n": n, "us": 1e3 * ms,
                                    "gbs": nbytes / (ms * 1e-3) / 1e9, "frac": nbytes / (ms * 1e-3) / 1e9 / hbm})
        del tab, T
    # the decoder's output head: Q6_K [H = 2048 -> VOCAB]
    rows = synth_blocks(Q6_K, 512, H, rng)
    rb = rows.size // 512
    heads = []
    for _ in range(2):  # two copies: consecutive calls read different 255 MB matrices
        w = torch.empty(VOCAB * rb, dtype=torch.uint8, device=dev)
        w.copy_(torch.from_numpy(rows).to(dev).view(1, -1).expand(-(-VOCAB // 512), -1).reshape(-1)[:VOCAB * rb])
        heads.append(q.QTensor(w, Q6_K, (H, VOCAB, 1, 1)))
    for Tt in (1, 8):
        x = torch.randn((Tt, H), device=dev)
        y = torch.empty((Tt, VOCAB), device=dev)
        ms = _graph_time(lambda i: q.mul_mat(heads[i % 2], x, y))
        nbytes = VOCAB * rb
        out["output_head"].append({"tokens": Tt, "weight_mb": nbytes / 1e6, "us": 1e3 * ms,
                                   "gbs": nbytes / (ms * 1e-3) / 1e9, "frac": nbytes / (ms * 1e-3) / 1e9 / hbm})
    del heads
    torch.cuda.empty_cache()
    return out


def slab_sweep(q, dev, iters=20):
    """Expert pool writes: the expert cache's slab uploads (core/expert_cache.cpp:637-723,
    :1357-1377) for one config-2 layer group, 8 experts x (gate, up: 884,736 B Q4_K; down:
    1,290,240 B Q6_K) = 24 slabs of 24.5 MB, from one page-locked staging buffer into random
    slots of three 64-slot pools (qwb_pool_write_slabs, one call per pool).  GB/s of slab
    bytes, against one plain host-to-device copy of the same staging buffer measured in the
    same run (the host link's copy rate).  Then the device byte audit of the 24 slots
    (qwb_pool_audit_slabs), compare only and with the FNV-1a 64 checksums (a diagnostic
    whose serial chains take milliseconds).  The audit times include the ctypes calls."""
    import ctypes as C

    import torch

    from questwend_b200 import _lib as L
    lib = q.lib()
    rng = np.random.default_rng(11)
    roles = ((Q4_K, H, F), (Q4_K, H, F), (Q6_K, F, H))
    slab = [q.ops.row_size(t, k) * m for t, k, m in roles]
    n_slots, n_exp = 64, K_USED
    pools = [q.QTensor(torch.zeros(n_slots * sb, dtype=torch.uint8, device=dev), t, (k, m, n_slots, 1))
             for (t, k, m), sb in zip(roles, slab)]
    group = sum(slab) * n_exp
    stage = torch.from_numpy(np.concatenate([synth_blocks(t, m, k, rng) for t, k, m in roles] * n_exp)).pin_memory()
    assert stage.numel() == group
    # staging order: expert-major (gate, up, down of expert 0, then expert 1, ...)
    offs = np.cumsum([0] + [sb for _ in range(n_exp) for sb in slab])[:-1].reshape(n_exp, 3)
    descs = [p.desc() for p in pools]
    calls = []
    for it in range(iters + 3):
        per_pool = []
        for r in range(3):
            slots = rng.choice(n_slots, n_exp, replace=False)
            arr = (L.SlabCopy * n_exp)()
            for e in range(n_exp):
                arr[e].src = stage.data_ptr() + int(offs[e, r])
                arr[e].slot = int(slots[e])
            per_pool.append((arr, slots))
        calls.append(per_pool)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)

    def upload(i):
        for r in range(3):
            L.check("qwb_pool_write_slabs", lib.qwb_pool_write_slabs(C.byref(descs[r]), slab[r], calls[i][r][0],
                                                                     n_exp, stream))
    for i in range(3):
        upload(i)
    dst = torch.empty(group, dtype=torch.uint8, device=dev)
    for _ in range(3):
        dst.copy_(stage, non_blocking=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for i in range(3, iters + 3):
        upload(i)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / iters
    e0.record()
    for _ in range(iters):
        dst.copy_(stage, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    ms_link = e0.elapsed_time(e1) / iters
    # every written slot holds its staged slab (last iteration)
    last = calls[iters + 2]
    for r in range(3):
        got = pools[r].data.view(n_slots, slab[r])[torch.from_numpy(last[r][1]).to(dev)]
        want = torch.stack([stage[int(offs[e, r]):int(offs[e, r]) + slab[r]] for e in range(n_exp)]).to(dev)
        assert torch.equal(got, want)
    # device byte audit of the 24 slots against the staging buffer (page-locked host memory):
    # compare only, then with both FNV-1a 64 checksums
    audit_ms = []
    for sums in (False, True):
        e0.record()
        audits = [q.pool_audit_slabs(pools[r], [stage.data_ptr() + int(offs[e, r]) for e in range(n_exp)],
                                     last[r][1], checksums=sums) for r in range(3)]
        e1.record()
        torch.cuda.synchronize()
        assert all(a["equal"] for rec in audits for a in rec)
        audit_ms.append(e0.elapsed_time(e1))
    link = group / (ms_link * 1e-3) / 1e9
    return {"config": {"workload": "C2 layer group: 8 experts x (gate, up Q4_K, down Q6_K) slabs",
                       "slabs": 3 * n_exp, "bytes": group, "pool_slots": n_slots,
                       "source": "one page-locked staging buffer"},
            "ms": ms, "gbs": group / (ms * 1e-3) / 1e9, "link_gbs": link,
            "frac_of_link": (group / (ms * 1e-3) / 1e9) / link,
            "audit_compare_ms": audit_ms[0], "audit_checksums_ms": audit_ms[1], "audit_equal": True}


def prefill_sweep(q, lib, dev, warmup, iters, cpu=None, tokens=PF_TOKENS, parts=("q4k", "q8_0", "q6k")):
    """cpu: the --cpu-leg JSON (reference CPU timings), or None.  tokens / parts: a subset
    of the sweep (profiling runs); the headline keys need the full Q4_K sweep."""
    import ctypes as C

    import torch

    from questwend_b200 import _lib as L
    experts = prefill_experts()
    reps = E // PF_UNIQUE
    pools = []
    for role, (k, rows) in enumerate(((PF_H, PF_F), (PF_F, PF_H))):
        base = torch.from_numpy(experts[role]).to(dev)
        buf = torch.empty(base.numel() * reps + 16, dtype=torch.uint8, device=dev)
        buf[:-16].view(reps, -1).copy_(base.expand(reps, -1))
        pools.append((q.QTensor(buf[:-16], Q4_K, (k, rows, E, 1)), k, rows))
    L.check("qwb_profile_enable", lib.qwb_profile_enable(8))
    gen = torch.Generator(device=dev)
    gen.manual_seed(99)
    points = []
    for T in (tokens if "q4k" in parts else ()):
        ids = torch.from_numpy(zipf_ids(T, E, K_USED, seed=T)).to(dev)
        for name, (W, k, rows) in zip(("gate_up", "down"), pools):
            nb = 1 if name == "gate_up" else K_USED
            b = torch.randn((T, nb, k), generator=gen, device=dev)
            out = torch.empty((T, K_USED, rows), device=dev)
            for _ in range(max(3, warmup)):
                q.mul_mat_id(W, b, ids, out)
            torch.cuda.synchronize()
            tot, gemm = [], []
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            for _ in range(iters):
                lib.qwb_profile_reset()
                e0.record()
                q.mul_mat_id(W, b, ids, out)
                e1.record()
                torch.cuda.synchronize()
                tot.append(e0.elapsed_time(e1))
                n = lib.qwb_profile_count() - 1
                ms = (C.c_float * max(n, 1))()
                tg = (C.c_int32 * max(n, 1))()
                L.check("qwb_profile_read", lib.qwb_profile_read(ms, tg, n))
                gemm.append(sum(m for m, t in zip(ms[:n], tg[:n]) if t == 5))
            assert torch.isfinite(out).all()
            fl = 2.0 * T * K_USED * k * rows
            t_ms, g_ms = float(np.median(tot)), float(np.median(gemm))
            points.append({"tokens": T, "shape": name, "ms": t_ms, "tflops": fl / (t_ms * 1e-3) / 1e12,
                           "gemm_ms": g_ms, "gemm_tflops": fl / (g_ms * 1e-3) / 1e12 if g_ms > 0 else None})
    L.check("qwb_profile_enable", lib.qwb_profile_enable(0))
    # Q8_0 experts (the sweep's second weight type), gate/up shape, and Q6_K experts, down
    # shape: the integer tensor-core kernel
    q8_points = []
    rng = np.random.default_rng(17)
    q8base = torch.from_numpy(synth_blocks(Q8_0, PF_UNIQUE * PF_F, PF_H, rng)).to(dev)
    q8buf = torch.empty(q8base.numel() * reps, dtype=torch.uint8, device=dev)
    q8buf.view(reps, -1).copy_(q8base.expand(reps, -1))
    W8 = q.QTensor(q8buf, Q8_0, (PF_H, PF_F, E, 1))
    for T in (tokens if "q8_0" in parts else ()):
        ids = torch.from_numpy(zipf_ids(T, E, K_USED, seed=T)).to(dev)
        b = torch.randn((T, 1, PF_H), generator=gen, device=dev)
        out = torch.empty((T, K_USED, PF_F), device=dev)
        q.mul_mat_id(W8, b, ids, out)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        tot = []
        for _ in range(3):
            e0.record()
            q.mul_mat_id(W8, b, ids, out)
            e1.record()
            torch.cuda.synchronize()
            tot.append(e0.elapsed_time(e1))
        assert torch.isfinite(out).all()
        fl = 2.0 * T * K_USED * PF_H * PF_F
        t_ms = float(np.median(tot))
        # the library's rule: 128-token tcgen05 tiles at >= 256 routed pairs per expert
        path = ("tcgen05 kind::i8 grouped GEMM" if T * K_USED >= 256 * min(T * K_USED, E)
                else "int8 tensor cores (mma.sync)")
        q8_points.append({"tokens": T, "shape": "gate_up", "type": "Q8_0", "ms": t_ms,
                          "tflops": fl / (t_ms * 1e-3) / 1e12, "path": path})
    del W8, q8buf, q8base
    # Q6_K experts, down shape [PF_F -> PF_H] (the Q4_K_M mix's down projections)
    q6base = torch.from_numpy(synth_blocks(Q6_K, PF_UNIQUE * PF_H, PF_F, rng)).to(dev)
    q6buf = torch.empty(q6base.numel() * reps, dtype=torch.uint8, device=dev)
    q6buf.view(reps, -1).copy_(q6base.expand(reps, -1))
    W6 = q.QTensor(q6buf, Q6_K, (PF_F, PF_H, E, 1))
    for T in (tokens if "q6k" in parts else ()):
        ids = torch.from_numpy(zipf_ids(T, E, K_USED, seed=T)).to(dev)
        b = torch.randn((T, K_USED, PF_F), generator=gen, device=dev)
        out = torch.empty((T, K_USED, PF_H), device=dev)
        q.mul_mat_id(W6, b, ids, out)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        tot = []
        for _ in range(3):
            e0.record()
            q.mul_mat_id(W6, b, ids, out)
            e1.record()
            torch.cuda.synchronize()
            tot.append(e0.elapsed_time(e1))
        assert torch.isfinite(out).all()
        fl = 2.0 * T * K_USED * PF_H * PF_F
        t_ms = float(np.median(tot))
        # the library's rule: 128-token tcgen05 tiles at >= 96 routed pairs per expert
        path = ("tcgen05 kind::i8 grouped GEMM" if T * K_USED >= 96 * min(T * K_USED, E)
                else "int8 tensor cores (mma.sync)")
        q8_points.append({"tokens": T, "shape": "down", "type": "Q6_K", "ms": t_ms,
                          "tflops": fl / (t_ms * 1e-3) / 1e12, "path": path})
    del W6, q6buf, q6base
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak, pkind = json.load(f)["bf16_tflops"], "measured bf16 burst"
    except Exception:
        peak, pkind = 1590.0, "fallback"
    if "q4k" not in parts or tuple(tokens) != PF_TOKENS:
        return {"points": points, "int8_points": q8_points}
    top = [p for p in points if p["tokens"] == PF_TOKENS[-1] and p["shape"] == "gate_up"][0]
    res = {"config": {"workload": "C3 prefill grouped GEMM, MUL_MAT_ID Q4_K x Q8_K", "hidden": PF_H,
                      "expert_ffn": PF_F, "experts": E, "top_k": K_USED, "routing": "Zipf(1.1) + Gumbel",
                      "tokens": list(PF_TOKENS), "l2": "weights 453 MB per matrix > L2"},
           "points": points, "int8_points": q8_points,
           "roofline": {"bound": "tensor", "kernel": f"grouped GEMM, gate/up shape, T={PF_TOKENS[-1]}",
                        "achieved": top["gemm_tflops"], "peak": peak, "peak_kind": pkind, "unit": "TFLOP/s",
                        "frac": top["gemm_tflops"] / peak if top["gemm_tflops"] else None, "traffic": None}}
    gate_pts = [p for p in points if p["shape"] == "gate_up"]
    res.update({"metric": "prefill_tflops", "value": top["tflops"], "unit": "TFLOP/s",
                "value_what": f"whole qwb_mul_mat_id call, Q4_K gate/up shape, T={PF_TOKENS[-1]}",
                "gemm_tflops": top["gemm_tflops"],
                "by_tokens": {str(p["tokens"]): p["tflops"] for p in gate_pts}})
    if cpu and cpu.get("prefill"):
        c, T = cpu["prefill"], PF_TOKENS[0]
        fl = 2.0 * T * K_USED * PF_H * PF_F
        res["cpu_baseline"] = {"value": fl / (c["median"] * 1e-3) / 1e12, "unit": "TFLOP/s", "cores": c["threads"],
                               "kind": "reference", "cpu": cpu.get("cpu"),
                               "sample": f"reference ggml CPU mul_mat_id, T={T}, gate shape, median of {c['n']} calls "
                                         f"({c['median']:.1f} ms)"}
        if cpu.get("prefill_1t"):
            c1 = cpu["prefill_1t"]
            res["cpu_baseline"]["value_1_thread"] = fl / (c1["median"] * 1e-3) / 1e12
    return res


# the 235B-A22B expert-parallel layer: hidden 4096, expert FFN 1536, 128 experts, top-8
EP4_H, EP4_F, EP4_TOKENS, EP4_LAYERS, EP4_UNIQUE = 4096, 1536, (1, 8, 64), 24, 8


def ep_layers(q, dev, base, shapes, n_layers, n_exp, lo, n, unique):
    """n_layers MoE layers of which this rank holds experts [lo, lo + n): global expert e of
    layer l is distinct image ((e mod unique) - l) mod unique of `base` (one image per
    expert and role in its own memory); router and ffn_norm weights from one seed, the
    same on every rank."""
    import torch

    from questwend_b200.expert_parallel import ExpertShard
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234)
    hid = shapes[0][2]
    layers = []
    for layer in range(n_layers):
        mats = []
        for role, (t, rows, K) in enumerate(shapes):
            idx = torch.tensor([((lo + i) % unique - layer) % unique for i in range(n)], device=dev)
            rows_img = base[role].view(unique, -1).index_select(0, idx).reshape(-1)
            buf = torch.empty(rows_img.numel() + 16, dtype=torch.uint8, device=dev)
            buf[:-16].copy_(rows_img)
            mats.append(q.QTensor(buf[:-16], t, (K, rows, n, 1)))
        rw = torch.randn((n_exp, hid), generator=gen, device=dev) * 0.02
        nw = 1.0 + 0.1 * torch.randn(hid, generator=gen, device=dev)
        layers.append((rw, nw, ExpertShard(mats[0], mats[1], mats[2], lo, n)))
    return layers


def ep_run(layers, x, n_used, steps, warmup, world, comm=None):
    """Time the expert-parallel stack (one qwb_moe_ep_layer call and one all-reduce per
    layer: the peer-memory one when `comm` is given, else NCCL's) captured in a CUDA
    graph.  Returns (per-step ms stats, mean ms, the selections of every layer, the stack
    output, the graph, the collective-only ms per step, NCCL's collective-only ms)."""
    import torch
    import torch.distributed as dist

    from questwend_b200.expert_parallel import moe_layer
    T, hid = x.shape
    outs = [torch.empty((T, hid), device=x.device) for _ in layers]

    def step():
        y, sels = x, []
        for (rw, nw, shard), o in zip(layers, outs):
            y, sel, _ = moe_layer(y, rw, shard, n_used, norm_w=nw, norm_eps=1e-6, out=o, comm=comm)
            sels.append(sel)
        return y, sels

    for _ in range(2):  # eager: sizes the workspace, configures the kernels
        y, _ = step()
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()
    if world > 1:
        dist.barrier()
    graph = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream()
    cs.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cs):
        with torch.cuda.graph(graph, stream=cs):
            y, sels = step()
    torch.cuda.synchronize()
    for _ in range(max(3, warmup)):
        graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    evs[0].record()
    for i in range(steps):
        graph.replay()
        evs[i + 1].record()
    torch.cuda.synchronize()
    ms = evs[0].elapsed_time(evs[-1]) / steps
    st = stats([evs[i].elapsed_time(evs[i + 1]) for i in range(steps)])
    def coll_alone(use_comm):
        # the collectives alone: the same all-reduces (one per layer, (T, H) f32) in a graph
        bufs = [torch.zeros((T, hid), device=x.device) for _ in layers]
        red = (lambda b: comm.all_reduce(b)) if use_comm else (lambda b: dist.all_reduce(b))
        cgraph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(cs):
            for bf in bufs:
                red(bf)
            torch.cuda.synchronize()
            with torch.cuda.graph(cgraph, stream=cs):
                for bf in bufs:
                    red(bf)
        torch.cuda.synchronize()
        for _ in range(3):
            cgraph.replay()
        torch.cuda.synchronize()
        dist.barrier()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record()
        for _ in range(steps):
            cgraph.replay()
        c1.record()
        torch.cuda.synchronize()
        del cgraph
        return c0.elapsed_time(c1) / steps

    coll_ms = nccl_ms = 0.0
    if world > 1:
        coll_ms = coll_alone(comm is not None)
        nccl_ms = coll_alone(False) if comm is not None else coll_ms
    return st, ms, sels, y, graph, coll_ms, nccl_ms


def ep_step_bytes(sels, n_exp, expert_bytes, router_bytes, world):
    """Algorithmic HBM bytes of one step over all ranks: every expert some token selected
    is read once (by its owner), and every rank reads its router replica."""
    return sum(int(np.unique(s.cpu().numpy()).size) * expert_bytes + world * router_bytes for s in sels)


def ep_check(q, dev, base, shapes, n_exp, unique, layer0, x, y_ep, n_used):
    """nRMS of one expert-parallel layer's output against the fused single-GPU layer
    (qwb_moe_ffn with all experts of the layer) on the same input."""
    import torch
    full = ep_layers(q, dev, base, shapes, 1, n_exp, 0, n_exp, unique)[0]
    rw, nw, sh = full
    assert torch.equal(rw, layer0[0]) and torch.equal(nw, layer0[1])
    want, _, _ = q.moe_ffn(x, rw, sh.gate, sh.up, sh.down, n_used, residual=x, norm_w=nw, norm_eps=1e-6)
    got, ref = y_ep.cpu().numpy(), want.cpu().numpy()
    return float(np.sqrt(np.mean((got - ref) ** 2)) / max(np.sqrt(np.mean(ref ** 2)), 1e-30))


def ep_fused_ms(q, layers, x, steps):
    """One GPU holding every expert: the same stack through qwb_moe_ffn (the batch-1 decode
    kernels at T = 1), ms per step, captured in a CUDA graph."""
    import torch
    outs = [torch.empty_like(x) for _ in layers]

    def step():
        y = x
        for (rw, nw, sh), o in zip(layers, outs):
            y, _, _ = q.moe_ffn(y, rw, sh.gate, sh.up, sh.down, K_USED, residual=y, out=o, norm_w=nw, norm_eps=1e-6)
        return y

    step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream()
    cs.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cs):
        with torch.cuda.graph(graph, stream=cs):
            step()
    torch.cuda.synchronize()
    for _ in range(3):
        graph.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    del graph
    return e0.elapsed_time(e1) / steps


def ep_config4_sweep(q, dev, world, rank, steps, warmup, comm=None):
    """The 235B-A22B layer (hidden 4096, expert FFN 1536, 128 experts, top-8; Q4_K gate/up,
    Q6_K down) expert-parallel over `world` GPUs: EP4_LAYERS layers per step (of the
    model's 94), decode batches of T in EP4_TOKENS tokens (total over the job), one
    qwb_moe_ep_layer call and one all-reduce per layer."""
    import torch
    import torch.distributed as dist

    from questwend_b200.expert_parallel import moe_layer, shard_range
    hbm, kind = peaks()
    shapes = ((Q4_K, EP4_F, EP4_H), (Q4_K, EP4_F, EP4_H), (Q6_K, EP4_H, EP4_F))
    rng = np.random.default_rng(4)
    base = [torch.from_numpy(synth_blocks(t, EP4_UNIQUE * rows, K, rng)).to(dev) for t, rows, K in shapes]
    lo, n = shard_range(E, world, rank)
    layers = ep_layers(q, dev, base, shapes, EP4_LAYERS, E, lo, n, EP4_UNIQUE)
    expert_bytes = 2 * EP4_F * (EP4_H // 256) * 144 + EP4_H * (EP4_F // 256) * 210
    router_bytes = E * EP4_H * 4
    points = []
    for T in EP4_TOKENS:
        x = torch.randn((T, EP4_H), generator=torch.Generator(device=dev).manual_seed(900 + T), device=dev)
        st, ms, sels, y, graph, coll_ms, nccl_ms = ep_run(layers, x, K_USED, steps, warmup, world, comm)
        del graph
        t = torch.tensor([ms, st["median"], coll_ms, nccl_ms], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, med, coll_ms, nccl_ms = t.tolist()
        nbytes = ep_step_bytes(sels, E, expert_bytes, router_bytes, world)
        # one layer's output against the fused single-GPU layer (rank 0), T = 8
        err = None
        if T == 8:
            y1, _, _ = moe_layer(x, layers[0][0], layers[0][2], K_USED, norm_w=layers[0][1], norm_eps=1e-6,
                                 comm=comm)
            torch.cuda.synchronize()
            if rank == 0:
                err = ep_check(q, dev, base, shapes, E, EP4_UNIQUE, layers[0], x, y1, K_USED)
        gbs = nbytes / (ms * 1e-3) / 1e9
        fused_ms = ep_fused_ms(q, layers, x, steps) if world == 1 else None
        points.append({"tokens": T, "ms_per_step": ms, "ms_per_layer": ms / EP4_LAYERS, "step_ms_median": med,
                       "fused_layer_ms_per_step": fused_ms,
                       "tokens_per_s": T * 1000.0 / ms,
                       "collective_ms_per_step": coll_ms if world > 1 else 0.0,
                       "nccl_allreduce_ms_per_step": nccl_ms if world > 1 else 0.0,
                       "kernel_ms_per_step": ms - coll_ms if world > 1 else ms,
                       "hbm_bytes_per_step": nbytes, "hbm_gbs_aggregate": gbs,
                       "roofline": {"bound": "hbm", "achieved": gbs, "peak": world * hbm,
                                    "peak_kind": f"{kind} x {world} GPUs", "unit": "GB/s",
                                    "frac": gbs / (world * hbm)},
                       "ep_nrmse": err})
    return {"workload": "qwen3-235b-a22b MoE FFN layer, expert-parallel decode", "layers": EP4_LAYERS,
            "collective": "peer-memory all-reduce (qwb_ep_allreduce_f32)" if comm is not None else "NCCL all-reduce",
            "hidden": EP4_H, "expert_ffn": EP4_F, "experts": E, "top_k": K_USED, "experts_per_gpu": n,
            "n_gpus": world, "collectives_per_step": EP4_LAYERS if world > 1 else 0,
            "note": "kernel_ms_per_step = step - the same all-reduces timed alone in a graph",
            "points": points}


def run_ep(args, world, rank, local):
    """N > 1: the 48-layer decode stack with the experts sharded over the ranks; every rank
    holds all N tokens (one per rank) and routes them; one all-reduce per layer."""
    import torch
    import torch.distributed as dist

    import questwend_b200 as q
    from questwend_b200.expert_parallel import PeerAllReduce, moe_layer, shard_range
    q.lib()
    dev = torch.device("cuda", local)
    lo, n = shard_range(E, world, rank)
    # the per-layer all-reduce over peer memory; messages up to the 235B layer at 64 tokens
    comm = PeerAllReduce(max_bytes=max(world * H, EP4_TOKENS[-1] * EP4_H) * 4)
    base = [torch.from_numpy(a).to(dev) for a in quantized_experts(seed=0)]
    shapes = ((Q4_K, F, H), (Q4_K, F, H), (Q6_K, H, F))
    n_layers = args.layers
    layers = ep_layers(q, dev, base, shapes, n_layers, E, lo, n, UNIQUE)
    # the step's batch: one token per rank, the same (N, H) rows on every rank
    x = torch.randn((world, H), generator=torch.Generator(device=dev).manual_seed(77), device=dev)
    with ClockSampler(local) as clk:
        st, ms_step, sels, y_graph, graph, coll_ms, nccl_ms = ep_run(layers, x, K_USED, args.steps, args.warmup,
                                                                     world, comm)
        # end to end: the batch from pinned host memory (every rank reads all N rows), the
        # rank's own token's output row back
        x_host = torch.randn((world, H), generator=torch.Generator().manual_seed(5)).pin_memory()
        y_host = torch.empty((1, H)).pin_memory()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(args.steps):
            x.copy_(x_host, non_blocking=True)
            graph.replay()
            y_host.copy_(y_graph[rank:rank + 1], non_blocking=True)
            torch.cuda.current_stream().synchronize()
        e1.record()
        torch.cuda.synchronize()
    ms_e2e = e0.elapsed_time(e1) / args.steps
    del graph
    flags, bad, cnt = q.read_status()
    times = torch.tensor([ms_step, ms_e2e, coll_ms, nccl_ms, st["median"], st["p10"], st["p90"], float(flags)],
                         device=dev)
    dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms_step, ms_e2e, coll_ms, nccl_ms, med, p10, p90, flags = times.tolist()
    expert_bytes = 2 * EXPERT_GU + EXPERT_D
    nbytes = ep_step_bytes(sels, E, expert_bytes, E * H * 4, world)
    # multi-GPU correctness: one layer against the fused single-GPU layer (rank 0 decides)
    y1, _, _ = moe_layer(x, layers[0][0], layers[0][2], K_USED, norm_w=layers[0][1], norm_eps=1e-6, comm=comm)
    torch.cuda.synchronize()
    err = ep_check(q, dev, base, shapes, E, UNIQUE, layers[0], x, y1, K_USED) if rank == 0 else 0.0
    bad_t = torch.tensor([1.0 if (err > 1e-5 or flags) else 0.0], device=dev)
    dist.all_reduce(bad_t, op=dist.ReduceOp.MAX)
    if bad_t.item():
        raise RuntimeError(f"expert-parallel output differs from the fused layer: nrmse {err:.3e}, flags {flags}")
    c4 = None if args.no_ep4 else ep_config4_sweep(q, dev, world, rank, max(20, args.steps // 10), args.warmup,
                                                   comm)
    torch.cuda.synchronize()
    dist.barrier()
    comm.close()
    hbm, kind = peaks()
    gbs = nbytes / (ms_step * 1e-3) / 1e9
    if rank == 0:
        cfg = workload_config(world, n_layers)
        cfg["parallelism"] = f"ep{world}"
        cfg["experts_per_gpu"] = n
        print(json.dumps({
            "metric": "decode_tokens_per_s", "value": world * 1000.0 / ms_step, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "step_ms": {"median": med, "p10": p10, "p90": p90, "n": args.steps},
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "q4_K/q6_K x q8_K -> f32", "data": "synthetic (seeded quantized blocks: random codes, scales sized like quantized N(0,0.02))",
            "config": cfg,
            "e2e": {"value": world * 1000.0 / ms_e2e, "unit": "tokens/s", "h2d_bytes_per_step": world * H * 4,
                    "d2h_bytes_per_step": H * 4},
            "collectives_per_step": n_layers,
            "collective": "peer-memory all-reduce (qwb_ep_allreduce_f32), one per layer",
            "collective_ms_per_step": coll_ms,
            "nccl_allreduce_ms_per_step": nccl_ms,
            "kernel_ms_per_step": ms_step - coll_ms,
            "gpu_launches": args.steps * 4 * n_layers,  # router, gate/up, down, all-reduce per layer
            "ep_nrmse": err,
            "device_errors": int(flags),
            "roofline": {"bound": "hbm", "kernel": "whole expert-parallel step, aggregate over the GPUs",
                         "achieved": gbs, "peak": world * hbm, "peak_kind": f"{kind} x {world} GPUs",
                         "unit": "GB/s", "frac": gbs / (world * hbm), "traffic": None,
                         "algorithmic_bytes": nbytes},
            "ep_config4": c4,
            "clocks": clk.summary(),
        }))
    dist.barrier()
    dist.destroy_process_group()


def run_ggml_leg(args):
    """--ggml-leg: the decode stack and a prefill stack through ggml itself, the way
    QuestWend runs them (ggml_backend_graph_compute on the whole graph), on two backends of
    the same B200: the stock ggml-cuda backend (the reference's own GPU path: MMVQ / MMQ
    kernels, Q8_1 activations), and libggml-qwb.so installed as the "cuda" backend beside
    it (build_moe subgraphs fused into qwb_moe_ffn, everything else handed to ggml-cuda).
    The host is the reference's own ggml library (compiled from its sources); weights are
    the bench's seeded synthetic blocks (UNIQUE images per role, expert e of layer l =
    image (e + l) mod UNIQUE).  Runs in a process of its own (it loads ggml's CUDA
    backends next to nothing else)."""
    import shutil
    import tempfile

    import oracle as O
    if not O.ref_available():
        print(json.dumps({"unavailable": "reference ggml (oracle/_ref) not built"}))
        return
    cuda_lib = os.path.join(ROOT, "oracle", "_ref", "cuda", "libggml-cuda.so")
    qwb_lib = os.path.join(ROOT, "questwend_b200", "libggml-qwb.so")
    if not (os.path.exists(cuda_lib) and os.path.exists(qwb_lib)):
        print(json.dumps({"unavailable": "reference ggml-cuda build or libggml-qwb.so missing"}))
        return
    inst = tempfile.mkdtemp()
    shutil.copy(qwb_lib, os.path.join(inst, "libggml-cuda-qwb.so"))
    os.symlink(cuda_lib, os.path.join(inst, "libggml-cuda.so"))
    os.symlink(os.path.join(ROOT, "questwend_b200", "libqwb.so"), os.path.join(inst, "libqwb.so"))
    g, u, d = quantized_experts(seed=0)
    rng = np.random.default_rng(2)
    L = args.layers
    rw = (rng.standard_normal((L, E, H)) * 0.02).astype(np.float32)
    nw = (1.0 + 0.1 * rng.standard_normal((L, H))).astype(np.float32)
    out = {"host": "reference ggml (ggml_backend_graph_compute on the whole stack graph)",
           "config": {"layers": L, "hidden": H, "experts": E, "top_k": K_USED, "expert_ffn": F,
                      "gate_up": "Q4_K", "down": "Q6_K"}, "points": []}
    for T, iters in ((1, max(args.steps, 5)), (PF_GGML_T, 3)):
        x = rng.standard_normal((T, H)).astype(np.float32)
        res = {}
        for name, path in (("stock_ggml_cuda", cuda_lib), ("qwb", os.path.join(inst, "libggml-cuda-qwb.so"))):
            r = O.backend_moe_stack(path, L, H, F, E, K_USED, T, Q4_K, g, u, Q6_K, d, UNIQUE, rw, nw, x,
                                    iters=iters)
            res[name] = r
            pt = {"backend": name, "tokens": T, "rc": r["rc"], "ms_per_pass": r["ms"],
                  "tokens_per_s": T * 1000.0 / r["ms"] if r["ms"] > 0 else None, "passes": iters}
            if name == "qwb":
                pt["stats_per_pass"] = dict(zip(("fused_layers", "own_nodes", "delegated_nodes", "delegated_runs"),
                                                [v / (iters + 1) for v in r["stats"][:4]]))
            out["points"].append(pt)
        if res["qwb"]["rc"] == 0 and res["stock_ggml_cuda"]["rc"] == 0:
            out["points"][-1]["nrmse_vs_stock"] = O.nrmse(res["qwb"]["out"], res["stock_ggml_cuda"]["out"])
    print(json.dumps(out))


def ggml_leg_subprocess(args):
    cmd = [sys.executable, os.path.abspath(__file__), "--ggml-leg", "--layers", str(args.layers),
           "--steps", str(min(args.steps, 50))]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
        return json.loads(r.stdout.strip().splitlines()[-1])
    except Exception as ex:  # reported, never required
        print(f"ggml leg failed: {ex}", file=sys.stderr)
        return None


PF_GGML_T = 2048  # the prefill batch of the decoder workload


def workload_config(n, n_layers=LAYERS):
    return {"workload": "qwen3-30b-a3b MoE FFN stack, batch-1 decode", "layers": n_layers, "hidden": H,
            "experts": E, "top_k": K_USED, "expert_ffn": F, "gate_up": "Q4_K", "down": "Q6_K",
            "router": "f32", "global_batch": n, "parallelism": f"replicas{n}" if n > 1 else "single",
            "l2": "inputs larger than L2 (1.17 GB of distinct expert weights per step)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="qwb", choices=["qwb", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="MoE layers per step (default 48; fewer only for profiling captures)")
    ap.add_argument("--no-prefill", action="store_true", help="skip the prefill sweep")
    ap.add_argument("--no-mmid", action="store_true", help="skip the decode-batch MUL_MAT_ID sweep")
    ap.add_argument("--no-gathers", action="store_true",
                    help="skip the GET_ROWS and output-head measurements")
    ap.add_argument("--no-slabs", action="store_true", help="skip the expert pool write (slab upload) measurement")
    ap.add_argument("--only-prefill", action="store_true",
                    help="run only the prefill sweep, without its CPU baseline (profiling runs)")
    ap.add_argument("--pf-tokens", default=",".join(str(t) for t in PF_TOKENS),
                    help="with --only-prefill: comma-separated token counts")
    ap.add_argument("--pf-parts", default="q4k,q8_0,q6k",
                    help="with --only-prefill: comma-separated subset of q4k, q8_0, q6k")
    ap.add_argument("--only-mmid", action="store_true",
                    help="run only the decode-batch MUL_MAT_ID sweep and print its JSON (profiling runs)")
    ap.add_argument("--mmid-tokens", default=",".join(str(t) for t in MMID_TOKENS),
                    help="comma-separated token counts of the decode-batch MUL_MAT_ID sweep")
    ap.add_argument("--mmid-pools", type=int, default=8,
                    help="expert pools (453 MB each) the sweep rotates through between calls")
    ap.add_argument("--cpu-leg", action="store_true",
                    help="internal: print the reference CPU timings used by cpu_baseline and exit")
    ap.add_argument("--ggml-leg", action="store_true",
                    help="internal: time the stack through ggml on the stock ggml-cuda backend and on "
                         "libggml-qwb.so, print the JSON and exit")
    ap.add_argument("--no-ggml", action="store_true", help="skip the ggml drop-in comparison")
    ap.add_argument("--no-ep4", action="store_true",
                    help="skip the 235B-A22B expert-parallel layer sweep (T = 1, 8, 64)")
    args = ap.parse_args()
    if args.cpu_leg:
        return run_cpu_leg(args)
    if args.ggml_leg:
        return run_ggml_leg(args)
    if args.impl == "reference":
        return run_reference(args)
    world0 = int(os.environ.get("WORLD_SIZE", "1"))
    # the reference CPU timings first, in a process of their own, before this one touches
    # the GPU (they are a reported baseline; the GPU timings below do not overlap them)
    cpu_leg = None
    if world0 == 1 and not args.no_cpu and not (args.only_mmid or args.only_prefill):
        cpu_leg = cpu_leg_subprocess(args.no_prefill)

    import torch
    import torch.distributed as dist

    import questwend_b200 as q
    from questwend_b200 import _lib as L

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        return run_ep(args, world, rank, local)
    lib = q.lib()
    mmid_tokens = tuple(int(t) for t in args.mmid_tokens.split(","))
    if args.only_mmid:
        print(json.dumps({"decode_mmid": decode_mmid_sweep(q, lib, torch.device("cuda", local), mmid_tokens, args.mmid_pools)}))
        return
    if args.only_prefill:
        pf_tokens = tuple(int(t) for t in args.pf_tokens.split(","))
        print(json.dumps({"prefill": prefill_sweep(q, lib, torch.device("cuda", local), args.warmup, 10,
                                                   tokens=pf_tokens, parts=tuple(args.pf_parts.split(",")))}))
        return

    # ---------------------------------------------------------------- weights
    g, u, d = quantized_experts(seed=0)
    dev = torch.device("cuda", local)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    reps = E // UNIQUE
    base = [torch.from_numpy(a).to(dev) for a in (g, u, d)]
    n_layers = args.layers
    layers = []
    for layer in range(n_layers):
        pools = []
        for role, (t, rows, K) in enumerate(((Q4_K, F, H), (Q4_K, F, H), (Q6_K, H, F))):
            buf = torch.empty(base[role].numel() * reps + 16, dtype=torch.uint8, device=dev)
            # rotate the unique experts per layer so consecutive layers differ
            rolled = torch.roll(base[role].view(UNIQUE, -1), shifts=layer % UNIQUE, dims=0).reshape(-1)
            buf[:-16].view(reps, -1).copy_(rolled.expand(reps, -1))
            pools.append(q.QTensor(buf[:-16], t, (K, rows, E, 1)))
        rw = torch.randn((E, H), generator=gen, device=dev) * 0.02
        nw = 1.0 + 0.1 * torch.randn(H, generator=gen, device=dev)
        layers.append((rw, nw, pools))
    xs = [torch.empty(H, device=dev) for _ in range(n_layers + 1)]
    xs[0].copy_(torch.randn(H, generator=gen, device=dev))
    sel = torch.empty((n_layers, K_USED), dtype=torch.int32, device=dev)
    wts = torch.empty((n_layers, K_USED), dtype=torch.float32, device=dev)
    descs = []
    for layer, (rw, nw, (pg, pu, pd)) in enumerate(layers):
        # l_out = build_moe(rms_norm(cur) * ffn_norm) + cur  (core/runtime.cpp:2979-2993)
        descs.append(q.ops.moe_ffn_desc(xs[layer].view(1, H), rw, pg, pu, pd, K_USED, xs[layer + 1].view(1, H),
                                        residual=xs[layer].view(1, H), selected=sel[layer], weights=wts[layer],
                                        norm_w=nw, norm_eps=1e-6))
    import ctypes as C
    need = lib.qwb_moe_ffn_workspace_size(C.byref(descs[0]))
    ws = q.ops.workspace(need)
    status = q.ops.status_block()

    def step(stream_ptr):
        for dsc in descs:
            rc = lib.qwb_moe_ffn(C.byref(dsc), ws.data_ptr(), ws.numel(), status.data_ptr(), stream_ptr)
            if rc:
                raise L.QwbError("qwb_moe_ffn", rc)

    # clocks and throttle reasons sampled from the eager warm-up to the end of the e2e loop
    clk = ClockSampler(local).__enter__()
    # eager warm-up, layer by layer with checks (also configures kernel attributes
    # outside capture)
    s_main = torch.cuda.current_stream()
    for layer, dsc in enumerate(descs):
        rc = lib.qwb_moe_ffn(C.byref(dsc), ws.data_ptr(), ws.numel(), status.data_ptr(),
                             C.c_void_p(s_main.cuda_stream))
        if rc:
            raise L.QwbError("qwb_moe_ffn", rc)
        try:
            torch.cuda.synchronize()
        except Exception as ex:
            raise RuntimeError(f"eager warm-up failed at layer {layer}") from ex
        flags, bad, cnt = q.read_status()
        xo = xs[layer + 1]
        if flags or not torch.isfinite(xo).all():
            raise RuntimeError(f"layer {layer}: device flags {flags} (value {bad}, count {cnt}), "
                               f"finite={bool(torch.isfinite(xo).all())}, selected={sel[layer].tolist()}")
    # two graphs of the same step: `graph` (timed) and `pgraph` (same kernels plus an
    # event record after each, for the per-kernel breakdown)
    graph = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream()
    cs.wait_stream(s_main)
    with torch.cuda.stream(cs):
        with torch.cuda.graph(graph, stream=cs):
            step(C.c_void_p(cs.cuda_stream))
    L.check("qwb_profile_enable", lib.qwb_profile_enable(n_layers * 4 + 4))
    pgraph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(cs):
        lib.qwb_profile_reset()
        with torch.cuda.graph(pgraph, stream=cs):
            step(C.c_void_p(cs.cuda_stream))
    n_rec = lib.qwb_profile_count()
    torch.cuda.synchronize()

    for _ in range(max(3, args.warmup)):
        graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    # an event after every replay: the step total and each step's time (median, p10, p90)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    torch.cuda.synchronize()
    evs[0].record()
    for i in range(args.steps):
        graph.replay()
        evs[i + 1].record()
    torch.cuda.synchronize()
    ms_step = evs[0].elapsed_time(evs[-1]) / args.steps
    step_ms = stats([evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps)])
    # per-kernel durations: replays of the profiled graph right after the timed region
    per_kernel = {}
    ms = (C.c_float * (n_rec - 1))()
    tags = (C.c_int32 * (n_rec - 1))()
    for _ in range(3):
        pgraph.replay()
        L.check("qwb_profile_read", lib.qwb_profile_read(ms, tags, n_rec - 1))
        for m, tg in zip(ms, tags):
            per_kernel.setdefault(int(tg), []).append(float(m))
    flags, bad, cnt = q.read_status()

    # ------------------------------------------------------------------ e2e
    x_host = torch.randn(H, generator=torch.Generator().manual_seed(5)).pin_memory()
    y_host = torch.empty(H).pin_memory()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(args.steps):
        xs[0].copy_(x_host, non_blocking=True)
        graph.replay()
        y_host.copy_(xs[n_layers], non_blocking=True)
        torch.cuda.current_stream().synchronize()
    e1.record()
    torch.cuda.synchronize()
    ms_e2e = e0.elapsed_time(e1) / args.steps
    clk.__exit__(None, None, None)

    times = torch.tensor([ms_step, ms_e2e], device=dev)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms_step, ms_e2e = times.tolist()

    # graph replays of the same step are identical: check the output is finite and sane
    out = xs[n_layers].float().cpu().numpy()
    assert np.isfinite(out).all()

    hbm, kind = peaks()
    gu = per_kernel.get(2, [])
    gu_ms = float(np.mean(gu)) if gu else None
    gu_bytes = K_USED * 2 * EXPERT_GU + K_USED * (H + 4 * 8 + 2 * 128)  # weights + q8 activation rows
    dn = per_kernel.get(3, [])
    dn_ms = float(np.mean(dn)) if dn else None
    step_bytes = n_layers * (K_USED * (2 * EXPERT_GU + EXPERT_D) + E * H * 4)
    achieved = gu_bytes / (gu_ms * 1e-3) / 1e9 if gu_ms else None
    result = {
        "metric": "decode_tokens_per_s", "value": world * 1000.0 / ms_step, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "q4_K/q6_K x q8_K -> f32", "data": "synthetic (seeded quantized blocks: random codes, scales sized like quantized N(0,0.02))",
        "config": workload_config(world, n_layers),
        "step_ms": step_ms,
        "decode_hbm_gbs": step_bytes / (ms_step * 1e-3) / 1e9,
        "decode_hbm_frac": step_bytes / (ms_step * 1e-3) / 1e9 / hbm,
        "roofline": {"bound": "hbm", "kernel": "moe gate/up GEMV (GLU) per layer", "achieved": achieved,
                     "peak": hbm, "peak_kind": kind, "unit": "GB/s",
                     "frac": achieved / hbm if achieved else None, "traffic": GATEUP_TRAFFIC_BYTES,
                     "traffic_source": "ncu capture of this kernel (dram bytes read + written per launch)",
                     "algorithmic_bytes": gu_bytes},
        "kernels_us": {"router": 1e3 * float(np.mean(per_kernel.get(1, [0]))), "gate_up": 1e3 * (gu_ms or 0),
                       "down": 1e3 * (dn_ms or 0)},
        "down_gbs": (K_USED * EXPERT_D) / (dn_ms * 1e-3) / 1e9 if dn_ms else None,
        "e2e": {"value": world * 1000.0 / ms_e2e, "unit": "tokens/s", "h2d_bytes_per_step": H * 4,
                "d2h_bytes_per_step": H * 4},
        "gpu_launches": args.steps * 3 * n_layers,
        "device_errors": flags,
        "clocks": clk.summary(),
    }
    if cpu_leg and cpu_leg.get("decode"):
        c = cpu_leg["decode"]
        result["cpu_baseline"] = {
            "value": 1000.0 / (c["median"] * n_layers), "unit": "tokens/s", "cores": c["threads"],
            "kind": "reference", "cpu": cpu_leg.get("cpu"),
            "sample": f"one MoE layer on the reference ggml CPU backend, median of {c['n']} evaluations "
                      f"after 3 untimed ({c['median']:.3f} ms; p10 {c['p10']:.3f}, p90 {c['p90']:.3f}), "
                      f"scaled x{n_layers} layers"}
        if cpu_leg.get("decode_1t"):
            c1 = cpu_leg["decode_1t"]
            result["cpu_baseline"]["value_1_thread"] = 1000.0 / (c1["median"] * n_layers)
            result["cpu_baseline"]["layer_ms_1_thread"] = c1["median"]
    del graph, pgraph
    if rank == 0 and not args.no_prefill:
        result["prefill"] = prefill_sweep(q, lib, dev, args.warmup, 10, cpu=cpu_leg)
    if rank == 0 and not args.no_mmid:
        result["decode_mmid"] = decode_mmid_sweep(q, lib, dev, mmid_tokens, args.mmid_pools)
    if rank == 0 and not args.no_gathers:
        result["gathers"] = gathers_sweep(q, dev)
    if rank == 0 and not args.no_slabs:
        result["slab_upload"] = slab_sweep(q, dev)
    if rank == 0 and not args.no_ep4:
        result["ep_config4"] = ep_config4_sweep(q, dev, 1, 0, max(20, args.steps // 10), args.warmup)
    if rank == 0 and not args.no_ggml:
        # the GPU memory this process holds is released first: the leg loads 2 x 16 GB stacks
        del layers, descs, ws, base
        torch.cuda.empty_cache()
        result["ggml_dropin"] = ggml_leg_subprocess(args)
    if rank == 0:
        print(json.dumps(result))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
