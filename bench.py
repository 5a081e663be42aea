#!/usr/bin/env python
"""Benchmark: Mixtral-style MoE training step on B200.

Workload (one step): 4 layers, d_model 1024, 16 heads (MHA, head_dim 64),
8 experts top-2 with SwiGLU FFN 1024->3584->1024, RMSNorm, vocab 32000,
global batch 8 x seq 2048 = 16384 tokens; bf16 compute, fp32 master weights,
Adam; synthetic token ids uniform in [0, 32000), weights N(0, 0.02), seed 4.
Metric: training tokens/s over the whole job (all ranks).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs one process per GPU (torchrun): the global batch is split over
ranks (data parallel) with the expert-parallel token exchange and gradient
all-reduce of the trainer over NCCL. Rank 0 prints one JSON line. At N = 1
the line also carries the other BASELINE configs, measured on the device
(`workloads`: the f32 MLP step, the transformer block, mixtral-tiny, and the
dense GEMM sweep), each beside its CPU-restatement timing.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "cat-nn-compiler_b200"))
sys.path.insert(0, ROOT)

CFG = dict(vocab=32000, hidden=1024, mid=3584, layers=4, heads=16, kv_heads=16, experts=8, top_k=2,
           global_batch=8, seq=2048, rope_theta=1e6, rms_eps=1e-5, lr=1e-4, seed=4)
METRIC = "MoE train tokens/s (config 5: 4L d1024 h16 E8 top-2 F3584 V32000, seq 2048, global batch 8)"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=30)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-workloads", action="store_true", help="N=1: skip the config 1/3/4 measurements")
    p.add_argument("--kernel-only", action="store_true",
                   help="run only one kernel at its config-5 shape for profiling (--kernel)")
    p.add_argument("--kernel", default="w13",
                   choices=["w13", "swiglu_fwd", "swiglu_bwd", "attn", "step_small", "gemm_tf32"],
                   help="w13: grouped expert GEMM (W13 forward shape); swiglu_fwd / swiglu_bwd: the expert GEMMs "
                        "with the SwiGLU epilogues; attn: tcgen05 flash attention fwd + bwd (B8 S2048 H16 hd64); "
                        "step_small: trainer steps at config-5 widths on 2 sequences (its HBM-bound kernels); "
                        "gemm_tf32: the TF32 tensor-core GEMM at 4096^3")
    p.add_argument("--batches", type=int, default=1,
                   help="distinct resident token batches the steps cycle through (1: every step trains the same batch)")
    p.add_argument("--reps", type=int, default=20)
    p.add_argument("--batch", type=int, default=2, help="--kernel step_small: sequences per step (1 layer)")
    p.add_argument("--attn-batch", type=int, default=8, help="--kernel attn: sequences (8: config 5 on one GPU)")
    return p.parse_args()


def peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def step_flops(cfg, tokens):
    """Algorithmic FLOPs of one training step: the GEMM and attention FLOPs of the forward, times 3
    (forward + the two backward products)."""
    d, F, V, S, L, k = cfg["hidden"], cfg["mid"], cfg["vocab"], cfg["seq"], cfg["layers"], cfg["top_k"]
    E = cfg["experts"]
    per_tok = L * (8 * d * d + 2 * d * (S + 1) + k * 6 * d * F + 2 * d * E) + 2 * d * V
    return 3 * per_tok * tokens


class Clocks:
    """nvidia-smi sampling during the timed region (clocks + throttle reasons)."""

    def __init__(self, gpu_index):
        self.proc = None
        self.path = f"/tmp/catnn_clocks_{os.getpid()}.csv"
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={gpu_index}",
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                mx.append(float(f[1]))
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def gemm_bytes(rows, E, F, d):
    """Algorithmic bytes of one grouped W13 launch: A [rows, d], B [E, d, 2F], C [rows, 2F], bf16."""
    return 2 * (rows * d + E * d * 2 * F + rows * 2 * F)


def traffic_from_profile(rows, E, F, d):
    """DRAM bytes per launch of the dominant kernel: the committed ncu
    capture at the one-GPU shape (profiles/gemm_grouped_w13.json), scaled by
    this launch's algorithmic bytes over the captured launch's (traffic
    grows with the rows and the local experts)."""
    try:
        j = json.load(open(os.path.join(ROOT, "profiles", "gemm_grouped_w13.json")))
        full = j["dram_bytes_per_launch_full_size"]
        return int(full * gemm_bytes(rows, E, F, d) / j["algorithmic_bytes_per_launch"])
    except Exception:
        return None


def oracle_env(split=False, threads=None):
    """Environment for timing the oracle the way the reference runs: loops the
    reference runs on one thread stay on one thread (ORACLE_SPLIT=0); threads
    only where its Rayon splits rows, capped at `threads`."""
    os.environ["ORACLE_SPLIT"] = "1" if split else "0"
    if threads is not None:
        os.environ["ORACLE_THREADS"] = str(int(threads))


def mix_cfg(cfg):
    from oracle import oracle as O
    return O.MixCfg(cfg["vocab"], cfg["hidden"], cfg["mid"], cfg["layers"], cfg["heads"], cfg["kv_heads"],
                    cfg["experts"], cfg["top_k"], cfg["rms_eps"], cfg["rope_theta"], None)


_GRAD_BUF = {}


def oracle_step_seconds(P, cfg, S, seed):
    """Wall time of the oracle's train::mixtral_step on one sequence of S
    tokens at config-5 widths (full forward + backward). The gradient buffer
    is allocated once per process and reused, as a training loop would."""
    import numpy as np
    from oracle import oracle as O
    tok = np.random.default_rng(seed).integers(0, cfg["vocab"], S)
    G = _GRAD_BUF.get(P.size)
    if G is None:
        G = _GRAD_BUF[P.size] = np.zeros_like(P)
    t0 = time.perf_counter()
    O.mixtral_step(mix_cfg(cfg), P, tok, 1, S, out=G)
    return time.perf_counter() - t0


def step_cost_model(t1, t2):
    """A step of S tokens costs fixed + S * marginal (parameter-sized
    gradient buffers once, then per-token GEMVs: the reference's MoE step has
    no batching). From samples of 1 and 2 tokens."""
    marginal = max(t2 - t1, 1e-9)
    fixed = max(t1 - marginal, 0.0)
    return fixed, marginal


def cpu_baseline_port(P_host, cfg, tokens_per_step):
    """The oracle (C++ restatement of train::mixtral_step) on a bounded sample
    at config-5 widths, on one host thread (the reference's step is
    sequential linear_seq loops): 1- and 2-token steps give the fixed and the
    per-token cost; tokens/s = T / (fixed + T * per-token) for the full
    T-token step."""
    oracle_env(split=False, threads=1)
    t1 = oracle_step_seconds(P_host, cfg, 1, 11)
    t2 = oracle_step_seconds(P_host, cfg, 2, 12)
    fixed, marg = step_cost_model(t1, t2)
    full = fixed + tokens_per_step * marg
    return {"value": tokens_per_step / full, "unit": "tokens/s", "cores": 1, "kind": "port",
            "sample": f"oracle train::mixtral_step (train.rs:261 restated) at config-5 widths on one thread: a 1-token "
                      f"step {t1:.2f} s and a 2-token step {t2:.2f} s give a fixed cost {fixed:.2f} s and {marg:.3f} s "
                      f"per token; the {tokens_per_step}-token step extrapolates to {full:.0f} s "
                      f"(linear in tokens; the attention's S^2 term, ~6% of the step's FLOPs at S=2048, is left out, "
                      f"which favours the CPU)"}


def dominant_kernel(local, pairs, E, warm, reps):
    """The grouped expert GEMM at this rank's config-5 W13 forward shape
    (`pairs` routed rows over E local experts, each padded to 128 rows, x 7168
    x 1024), timed with CUDA events on the launching stream. Returns (ms per
    launch, algorithmic FLOPs, rows, F, d)."""
    import numpy as np
    import torch
    from catnn_b200 import ops
    cfg = CFG
    F, d = cfg["mid"], cfg["hidden"]
    rng = np.random.default_rng(cfg["seed"])
    counts = np.bincount(rng.integers(0, E, pairs), minlength=E)
    padded = -(-counts // 128) * 128
    offs = np.concatenate([[0], np.cumsum(padded)]).astype(np.int32)
    rows = int(offs[-1])
    dev = f"cuda:{local}"
    A = torch.randn(rows, d, device=dev, dtype=torch.bfloat16)
    Bw = torch.randn(E, d, 2 * F, device=dev, dtype=torch.bfloat16)
    C = torch.empty(rows, 2 * F, device=dev, dtype=torch.bfloat16)
    off_t = torch.as_tensor(offs).to(dev)
    for _ in range(warm):
        ops.grouped_gemm(A, Bw, off_t, out=C)
    torch.cuda.synchronize(local)
    stream = torch.cuda.current_stream(local)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        ops.grouped_gemm(A, Bw, off_t, out=C)
    e1.record(stream)
    torch.cuda.synchronize(local)
    return e0.elapsed_time(e1) / reps, 2.0 * int(counts.sum()) * 2 * F * d, rows, F, d


FFMA_PEAK_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12  # nominal fp32 CUDA-core peak (148 SMs x 128 lanes x FMA x 1.965 GHz)


def graph_time_ms(fn, local, reps, warm=3):
    """Device time of fn per call: warm-up calls (every workspace reaches its
    size), then `reps` calls captured in one CUDA graph and replayed between
    CUDA events on the launching stream — the kernels' time without the
    Python/ctypes launch cost. Returns (ms per call, launches per call)."""
    import torch
    from catnn_b200 import ops
    ctx = ops.context(local)
    for _ in range(warm):
        fn()
    torch.cuda.synchronize(local)
    l0 = ctx.launch_count()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            fn()
    launches = (ctx.launch_count() - l0) // reps
    g.replay()  # first replay uploads the graph
    torch.cuda.synchronize(local)
    stream = torch.cuda.current_stream(local)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    g.replay()
    e1.record(stream)
    torch.cuda.synchronize(local)
    ms = e0.elapsed_time(e1) / reps
    del g
    return ms, launches


def gemm_sweep(local, peak):
    """Config 2: C = A·B with M = N = K in {1024, 4096, 8192}, A and B N(0,1)/sqrt(K)
    and N(0,1), bf16 operands, fp32 accumulation; forward (2K³) and forward +
    backward (dA = dC·Bᵀ, dB = Aᵀ·dC: 6K³). Device time of the kernels: the
    calls are captured in a CUDA graph and replayed (CUDA events)."""
    import torch
    from catnn_b200 import ops
    g = torch.Generator(device=f"cuda:{local}").manual_seed(1)
    out = {}
    for K in (1024, 4096, 8192):
        A = (torch.randn(K, K, generator=g, device=f"cuda:{local}") / K ** 0.5).to(torch.bfloat16)
        B = torch.randn(K, K, generator=g, device=f"cuda:{local}").to(torch.bfloat16)
        dC = torch.randn(K, K, generator=g, device=f"cuda:{local}").to(torch.bfloat16)
        C, dA, dB = (torch.empty(K, K, device=f"cuda:{local}", dtype=torch.bfloat16) for _ in range(3))
        reps = {1024: 50, 4096: 10, 8192: 4}[K]

        def fwd():
            ops.gemm(A, B, out=C)

        def fwdbwd():
            ops.gemm(A, B, out=C)
            ops.gemm(dC, B, trans_b=True, out=dA)
            ops.gemm(A, dC, trans_a=True, out=dB)
        A32, B32 = A.float(), B.float()
        C32 = torch.empty(K, K, device=f"cuda:{local}")

        def fwd_tf32():
            ops.gemm(A32, B32, out=C32, tf32=True)
        res = {}
        # kind::tf32 runs at half the kind::f16 rate: its roofline is half the measured bf16 peak
        for name, f, flops, pk in (("fwd", fwd, 2 * K ** 3, peak), ("fwd_bwd", fwdbwd, 6 * K ** 3, peak),
                                   ("fwd_tf32", fwd_tf32, 2 * K ** 3, peak / 2)):
            ms, _ = graph_time_ms(f, local, reps)
            tf = flops / (ms * 1e-3) / 1e12
            res[name] = {"ms": round(ms, 4), "tflops": round(tf, 1), "frac": round(tf / pk, 3)}
        out[str(K)] = res
        del A32, B32, C32
    return out


def cpu_seconds(fn):
    t0 = time.perf_counter()
    fn()
    return time.perf_counter() - t0


def workload_mlp(local, steps, cpu):
    """Config 1: the f32 MLP train step (batch 64, Linear 784->256, ReLU,
    Linear 256->10, softmax cross-entropy, SGD lr 0.05; Xavier-uniform weights,
    N(0,1) inputs, labels uniform in [0,10), seed 0) — train::mlp_step
    (train.rs:71) plus Sgd::put on the four tensors, replayed as a CUDA graph.
    Latency-bound (78 MFLOP per step)."""
    import numpy as np
    import torch
    from catnn_b200 import ops
    r = np.random.default_rng(0)
    a1, a2 = np.sqrt(6.0 / (784 + 256)), np.sqrt(6.0 / (256 + 10))
    host = [r.uniform(-a1, a1, (784, 256)).astype(np.float32), np.zeros(256, np.float32),
            r.uniform(-a2, a2, (256, 10)).astype(np.float32), np.zeros(10, np.float32)]
    x = r.standard_normal((64, 784)).astype(np.float32)
    lab = r.integers(0, 10, 64)
    dev = f"cuda:{local}"
    W = [torch.as_tensor(t).to(dev) for t in host]
    X, L = torch.as_tensor(x).to(dev), torch.as_tensor(lab.astype(np.int32)).to(dev)

    def step():
        loss, *grads = ops.mlp_step(*W, X, labels=L)
        for p, gr in zip(W, grads):
            ops.sgd_(p, gr, 0.05)
    ms, launches = graph_time_ms(step, local, max(steps, 12))
    flops = 3 * 2 * 64 * (784 * 256 + 256 * 10)
    out = {"metric": "f32 MLP train step time (config 1)", "value": ms * 1e3, "unit": "us/step",
           "higher_is_better": False, "dtype": "f32", "steps_per_graph": max(steps, 12),
           "gpu_launches_per_step": launches,
           "roofline": {"bound": "latency", "achieved": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                        "peak": FFMA_PEAK_TFLOPS, "frac": flops / (ms * 1e-3) / 1e12 / FFMA_PEAK_TFLOPS,
                        "peak_source": "nominal fp32 CUDA-core peak", "note": "78 MFLOP per step: launch-latency bound"}}
    if cpu:
        from oracle import oracle as O
        threads = os.cpu_count() or 1
        oracle_env(split=False, threads=threads)
        Wh = [t.copy() for t in host]

        def cpu12():
            nonlocal Wh
            for _ in range(12):
                _, *g = O.mlp_step(*Wh, x, labels=lab)
                Wh = [O.sgd_put(p, gg, 0.05) for p, gg in zip(Wh, g)]
        sec = cpu_seconds(cpu12) / 12
        out["cpu_baseline"] = {"value": sec * 1e6, "unit": "us/step", "cores": threads, "kind": "port",
                               "sample": "the full 12-step run: oracle mlp_step (cpu::linear rows over all host "
                                         "threads, as Rayon splits them; the adjoints sequential) + Sgd::put"}
    return out


def workload_block(local, cpu):
    """Config 3: one pre-LN causal transformer block forward + backward (batch
    8, seq 512, d_model 512, 8 heads of 64, GELU FFN 2048; inputs N(0,1),
    weights N(0, 0.02), injected dY N(0,1), seed 2), composed from the
    library's operators; the f32 parity path and the bf16 tensor-core path,
    each replayed as a CUDA graph. 83.8 GFLOP per forward + backward."""
    import numpy as np
    import torch
    from catnn_b200 import ops
    b, s, d, h, ff = 8, 512, 512, 8, 2048
    r = np.random.default_rng(2)
    W = {"g1": np.ones(d, np.float32), "be1": np.zeros(d, np.float32), "g2": np.ones(d, np.float32),
         "be2": np.zeros(d, np.float32), "c1": np.zeros(ff, np.float32), "c2": np.zeros(d, np.float32)}
    for k, shape in (("wq", (d, d)), ("wk", (d, d)), ("wv", (d, d)), ("wo", (d, d)), ("f1", (d, ff)), ("f2", (ff, d))):
        W[k] = (r.standard_normal(shape) * 0.02).astype(np.float32)
    x = r.standard_normal((b, s, d)).astype(np.float32)
    dy = r.standard_normal((b, s, d)).astype(np.float32)
    dev = f"cuda:{local}"
    per_tok = 8 * d * d + 2 * d * (s + 1) + 4 * d * ff
    flops = 3 * per_tok * b * s
    out = {"metric": "transformer block fwd+bwd (config 3)", "unit": "ms", "higher_is_better": False,
           "flops_per_step": flops}
    for name, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
        G = {k: torch.as_tensor(v).to(dev, dt if k in ("wq", "wk", "wv", "wo", "f1", "f2") else torch.float32)
             for k, v in W.items()}
        X, DY = torch.as_tensor(x).to(dev, dt), torch.as_tensor(dy).to(dev, dt)

        def step():
            ln1 = ops.layer_norm(X, G["g1"], G["be1"])
            att = ops.attention(ln1, G["wq"], G["wk"], G["wv"], G["wo"], h, causal=True)
            hh = ops.add(X, att)
            ln2 = ops.layer_norm(hh, G["g2"], G["be2"])
            u = ops.linear(ln2, G["f1"], G["c1"])
            gl = ops.gelu(u)
            ops.add(hh, ops.linear(gl, G["f2"], G["c2"]))
            dgl, _, _ = ops.linear_backward(gl, G["f2"], DY)
            du = ops.gelu_backward(u, dgl)
            dln2, _, _ = ops.linear_backward(ln2, G["f1"], du)
            dh, _, _ = ops.layer_norm_backward(hh, G["g2"], dln2)
            dh = ops.add(dh, DY)
            dln1, *_ = ops.attention_backward(ln1, G["wq"], G["wk"], G["wv"], G["wo"], dh, h, causal=True)
            dxa, _, _ = ops.layer_norm_backward(X, G["g1"], dln1)
            ops.add(dxa, dh)
        ms, launches = graph_time_ms(step, local, 5)
        tf = flops / (ms * 1e-3) / 1e12
        pk, _ = peaks()
        peak = pk.get("bf16_tflops", 1590.0) if name == "bf16" else FFMA_PEAK_TFLOPS
        out[name] = {"ms": ms, "tflops": tf, "gpu_launches_per_step": launches,
                     "roofline": {"bound": "tensor" if name == "bf16" else "fma", "achieved": tf, "peak": peak,
                                  "unit": "TFLOP/s", "frac": tf / peak,
                                  "peak_source": "measured bf16_tflops" if name == "bf16" else
                                  "nominal fp32 CUDA-core peak"}}
    out["value"] = out["bf16"]["ms"]
    if cpu:
        from oracle import oracle as O
        threads = os.cpu_count() or 1
        oracle_env(split=False, threads=threads)
        sec = cpu_seconds(lambda: O.block_fwd_bwd(W, x[:1], dy[:1], h))
        out["cpu_baseline"] = {"value": sec * b * 1e3, "unit": "ms", "cores": threads, "kind": "port",
                               "sample": f"oracle block fwd+bwd on 1 of the 8 sequences ({sec:.1f} s), x8 (the block "
                                         f"is linear in the batch); cpu::linear rows over all host threads as Rayon "
                                         f"splits them, attention and adjoints sequential as in the reference"}
    return out


def workload_tiny(local, steps, cpu):
    """Config 4: mixtral-tiny training (2 layers, d 256, 4 heads, 8 experts
    top-2, SwiGLU 256->512->256, RMSNorm, vocab 1024, seq 256, batch 4; SGD lr
    0.05, seed 3) through the native trainer; the f32 parity path (the one the
    parity tests pin to the oracle) and the bf16 path, each step replayed as a
    CUDA graph. 15.3 GFLOP per step."""
    import numpy as np
    import torch
    from catnn_b200.train import MoeConfig, MoeTrainer, init_params
    out = {"metric": "mixtral-tiny train tokens/s (config 4)", "unit": "tokens/s", "higher_is_better": True}
    dev = f"cuda:{local}"
    tokens = np.random.default_rng(3).integers(0, 1024, 4 * 256)
    d, F, V, S, L, k, E = 256, 512, 1024, 256, 2, 2, 8
    per_tok = L * (8 * d * d + 2 * d * (S + 1) + k * 6 * d * F + 2 * d * E) + 2 * d * V
    flops = 3 * per_tok * 1024
    for name, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
        cfg = MoeConfig.make(1024, 256, 512, 2, 4, 4, 8, 2, batch=4, seq=256, rope_theta=1e4, dtype=dt,
                             optimizer="sgd", lr=0.05)
        tr = MoeTrainer(cfg, device=local)
        tr.set_params(init_params(cfg, 3))
        tr.set_graphs(True)
        tok = torch.as_tensor(tokens.astype(np.int32)).to(dev)
        loss = torch.zeros(1, device=dev)
        for _ in range(3):
            tr.step(tok, update=True, loss_out=loss)
        torch.cuda.synchronize(local)
        stream = torch.cuda.current_stream(local)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = max(steps, 20)
        e0.record(stream)
        for _ in range(n):
            tr.step(tok, update=True, loss_out=loss)
        e1.record(stream)
        torch.cuda.synchronize(local)
        tr.check()
        ms = e0.elapsed_time(e1) / n
        tr.close()
        tf = flops / (ms * 1e-3) / 1e12
        out[name] = {"tokens_per_s": 1024 / (ms * 1e-3), "ms_per_step": ms, "tflops": tf}
    out["value"] = out["bf16"]["tokens_per_s"]
    pk, _ = peaks()
    out["roofline"] = {"bound": "latency", "achieved": out["bf16"]["tflops"], "peak": pk.get("bf16_tflops", 1590.0),
                       "unit": "TFLOP/s", "frac": out["bf16"]["tflops"] / pk.get("bf16_tflops", 1590.0),
                       "note": "15.3 GFLOP per step over ~200 launches: latency/launch bound"}
    if cpu:
        from oracle import oracle as O
        oracle_env(split=False, threads=1)
        oc = O.MixCfg(1024, 256, 512, 2, 4, 4, 8, 2, 1e-5, 1e4, None)
        cfg = MoeConfig.make(1024, 256, 512, 2, 4, 4, 8, 2, batch=4, seq=256, rope_theta=1e4, dtype=torch.float32,
                             optimizer="sgd", lr=0.05)
        P = init_params(cfg, 3)
        sec = cpu_seconds(lambda: O.mixtral_step(oc, P, tokens[:256], 1, 256))
        out["cpu_baseline"] = {"value": 256 / sec, "unit": "tokens/s", "cores": 1, "kind": "port",
                               "sample": f"oracle train::mixtral_step on 1 of the 4 sequences (256 tokens, {sec:.1f} s, "
                                         f"forward + backward, no update); the reference's step is sequential"}
    return out


def run_kernel_only(args):
    """One kernel at its config-5 per-launch shape, `args.reps` launches, for
    ncu captures (the printed timing is informational)."""
    import numpy as np
    import torch
    from catnn_b200 import ops
    torch.cuda.set_device(0)
    T = CFG["global_batch"] * CFG["seq"]
    F, d, E = CFG["mid"], CFG["hidden"], CFG["experts"]
    if args.kernel == "w13":
        ms, flops, rows, F, d = dominant_kernel(0, T * CFG["top_k"], E, 1, args.reps)
        print(json.dumps({"kernel": "k_gemm_tc grouped W13 forward", "rows": rows, "N": 2 * F, "K": d, "ms": ms,
                          "tflops": flops / (ms * 1e-3) / 1e12}), flush=True)
        return
    dev = "cuda:0"
    stream = torch.cuda.current_stream(0)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(fn, flops, name, **kw):
        fn()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.reps
        print(json.dumps({"kernel": name, "ms": ms, "tflops": flops / (ms * 1e-3) / 1e12, **kw}), flush=True)
    if args.kernel in ("swiglu_fwd", "swiglu_bwd"):
        rng = np.random.default_rng(CFG["seed"])
        counts = np.bincount(rng.integers(0, E, T * CFG["top_k"]), minlength=E)
        offs = np.concatenate([[0], np.cumsum(-(-counts // 128) * 128)]).astype(np.int32)
        rows = int(offs[-1])
        off = torch.as_tensor(offs).to(dev)
        X = (torch.randn(rows, d, device=dev) * 0.5).to(torch.bfloat16)
        W13 = (torch.randn(E, d, 2 * F, device=dev) / d ** 0.5).to(torch.bfloat16)
        ac, h = ops.moe_expert_swiglu(X, W13, off)
        if args.kernel == "swiglu_fwd":
            timed(lambda: ops.moe_expert_swiglu(X, W13, off), 2.0 * int(counts.sum()) * 2 * F * d,
                  "k_gemm_tc grouped W13 + SwiGLU epilogue", rows=rows)
        else:
            W2 = (torch.randn(E, F, d, device=dev) / F ** 0.5).to(torch.bfloat16)
            DY = torch.randn(rows, d, device=dev).to(torch.bfloat16)
            timed(lambda: ops.moe_expert_swiglu_backward(DY, W2, ac, off), 2.0 * int(counts.sum()) * F * d,
                  "k_gemm_tc grouped W2 dgrad + SwiGLU adjoint epilogue", rows=rows)
    elif args.kernel == "attn":
        B, S, H, hd = args.attn_batch, CFG["seq"], CFG["heads"], CFG["hidden"] // CFG["heads"]
        q, k, v, do = (torch.randn(B, S, H, hd, device=dev).to(torch.bfloat16) for _ in range(4))
        do = do.reshape(B, S, H * hd)
        o, lse = ops.attention_core(q, k, v, True)
        fwd = 2.0 * B * H * S * S * hd  # causal half of 4·B·H·S²·hd
        timed(lambda: ops.attention_core(q, k, v, True), fwd, "fa5 forward (causal)", batch=B)
        timed(lambda: ops.attention_core_backward(q, k, v, o, lse, do, True), 2.5 * fwd, "fa5 backward (causal)", batch=B)
    elif args.kernel == "gemm_tf32":
        K = 4096
        A = torch.randn(K, K, device=dev) / K ** 0.5
        B = torch.randn(K, K, device=dev)
        C = torch.empty(K, K, device=dev)
        timed(lambda: ops.gemm(A, B, trans_b=True, out=C, tf32=True), 2.0 * K ** 3, "k_gemm_tc tf32 (K-major A, B)", K=K)
    elif args.kernel == "step_small":
        from catnn_b200.train import MoeConfig, MoeTrainer, init_params
        mc = MoeConfig.make(CFG["vocab"], d, F, 1, CFG["heads"], CFG["kv_heads"], E, CFG["top_k"], batch=args.batch,
                            seq=CFG["seq"], rope_theta=CFG["rope_theta"], dtype=torch.bfloat16, optimizer="adam",
                            lr=CFG["lr"])
        tr = MoeTrainer(mc)
        tr.set_params(init_params(mc, CFG["seed"]))
        tok = torch.randint(0, CFG["vocab"], (args.batch * CFG["seq"],), device=dev, dtype=torch.int32)
        loss = torch.zeros(1, device=dev)
        timed(lambda: tr.step(tok, update=True, loss_out=loss), 0.0,
              f"trainer step, 1 layer, {args.batch * CFG['seq']} tokens")
        tr.close()


def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    from catnn_b200 import ops
    from catnn_b200.train import MoeConfig, MoeTrainer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    cfg = dict(CFG)
    B = cfg["global_batch"] // world
    T_local = B * cfg["seq"]
    T_global = cfg["global_batch"] * cfg["seq"]
    # the global batch on every rank: each trains its sequences and owns
    # experts/world experts (data + expert parallel; world 1: one GPU)
    mc = MoeConfig.make(cfg["vocab"], cfg["hidden"], cfg["mid"], cfg["layers"], cfg["heads"], cfg["kv_heads"],
                        cfg["experts"], cfg["top_k"], batch=cfg["global_batch"], seq=cfg["seq"],
                        rope_theta=cfg["rope_theta"], rms_eps=cfg["rms_eps"], dtype=torch.bfloat16, optimizer="adam",
                        lr=cfg["lr"])
    comm = None
    if world > 1:
        from catnn_b200.dist import Comm
        comm = Comm.from_process_group(local)
    tr = MoeTrainer(mc, device=local, comm=comm)
    tr.set_graphs(True)  # the step body replays as one CUDA graph after its first two runs (every rank)
    # weights N(0, 0.02), norms 1; identical on every rank (same seed)
    g = torch.Generator(device=f"cuda:{local}").manual_seed(cfg["seed"])
    P = torch.randn(tr.n_params, generator=g, device=f"cuda:{local}") * 0.02
    from catnn_b200.train import packed_layout
    L = packed_layout(mc)
    h = cfg["hidden"]
    for l in range(cfg["layers"]):
        base = L["layer0"] + l * L["layer_stride"]
        P[base + L["rms_attn"]:base + L["rms_attn"] + h] = 1.0
        P[base + L["rms_moe"]:base + L["rms_moe"] + h] = 1.0
    P[L["final_norm"]:L["final_norm"] + h] = 1.0
    tr.set_params(P)
    gt = torch.Generator(device=f"cuda:{local}").manual_seed(cfg["seed"] + 1000)
    pool = [torch.randint(0, cfg["vocab"], (T_global,), generator=gt, device=f"cuda:{local}", dtype=torch.int32)
            for _ in range(max(args.batches, 1))]
    tokens = pool[0]
    loss = torch.zeros(1, device=f"cuda:{local}")
    ctx = ops.context(local)
    stream = torch.cuda.current_stream(local)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(local)

    # the loss of the first step, before any update: the sharded forward is the
    # one-GPU forward, so this agrees across N up to the order of cross-rank sums
    tr.step(tokens, update=False, loss_out=loss)
    barrier()
    tr.check()
    loss_step0 = float(loss)
    for i in range(args.warmup):
        tr.step(pool[i % len(pool)], update=True, loss_out=loss)
    barrier()
    tr.check()
    clocks = Clocks(local)
    launches0 = ctx.launch_count()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        tr.step(pool[i % len(pool)], update=True, loss_out=loss)
    e1.record(stream)
    barrier()
    ms = e0.elapsed_time(e1) / args.steps
    launches = (ctx.launch_count() - launches0) // max(args.steps, 1)
    clk = clocks.stop()
    tr.check()
    last_loss = float(loss)
    # max over ranks
    t = torch.tensor([ms], device=f"cuda:{local}")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t)

    # end to end through the public host-buffer call: host tokens -> device,
    # step, loss -> host, every step
    host_pool = [t.cpu().numpy().astype(np.uint32) for t in pool]
    barrier()
    clocks_e2e = Clocks(local)
    e0.record(stream)
    for i in range(args.steps):
        tr.step_host(host_pool[i % len(host_pool)], update=True)
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    clk_e2e = clocks_e2e.stop()
    t = torch.tensor([e2e_ms], device=f"cuda:{local}")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t)

    # where a rank's step goes: device-clock stamps at the step's phase
    # boundaries (one extra profiled step, replayed as a graph like the timed
    # ones), per phase the max over ranks
    tr.set_profile(True)
    for i in range(3):
        tr.step(pool[i % len(pool)], update=True, loss_out=loss)
    phases = tr.timeline()
    tr.set_profile(False)
    barrier()
    # routing balance of that last step: (token, slot) pairs per expert, summed
    # over ranks, and the load of each rank's experts (what expert parallelism
    # waits on at its barriers), as max / mean
    E, K = cfg["experts"], cfg["top_k"]
    cnt = torch.zeros(cfg["layers"], E, device=f"cuda:{local}", dtype=torch.float64)
    for l in range(cfg["layers"]):
        idx = torch.topk(tr.activation("router_logits", l), K, dim=1).indices
        cnt[l] = torch.bincount(idx.flatten(), minlength=E).double()
    if world > 1:
        dist.all_reduce(cnt)
    per_rank = cnt.view(cfg["layers"], world, E // world).sum(2)
    routing = {"expert_max_over_mean": [round(float(x), 3) for x in (cnt.max(1).values / cnt.mean(1))],
               "rank_max_over_mean": [round(float(x), 3) for x in (per_rank.max(1).values / per_rank.mean(1))]}
    if world > 1:
        every = [None] * world
        dist.all_gather_object(every, phases)
    else:
        every = [phases]
    agg = {}
    for name, ms_ in every[0]:
        agg.setdefault(name, 0.0)
    for rk in every:
        seen = {}
        for name, ms_ in rk:
            seen[name] = seen.get(name, 0.0) + ms_
        for name, v in seen.items():
            agg[name] = max(agg.get(name, 0.0), v)
    phase_breakdown = {"ms_max_over_ranks": {k: round(v, 4) for k, v in agg.items()},
                       "step_ms_per_rank": [round(sum(v for _, v in rk), 4) for rk in every],
                       "how": "device clock (%globaltimer) stamped on the step's stream at phase boundaries; the time of "
                              "a phase includes the waits (barriers, peer flags) inside it; summed over layers"}

    # dominant kernel: the grouped expert GEMM (W13 forward shape), timed live
    pk, pk_kind = peaks()
    kms, kflops, rows, F, d = dominant_kernel(local, T_global * cfg["top_k"] // world, cfg["experts"] // world, 3,
                                              args.reps)
    achieved = kflops / (kms * 1e-3) / 1e12
    peak = pk.get("bf16_tflops", 1590.0)

    out = {
        "metric": METRIC,
        "value": T_global / (ms * 1e-3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (token ids uniform [0,32000), weights N(0,0.02), seed 4)"
                + (f"; {len(pool)} resident batches cycled" if len(pool) > 1 else ""),
        "config": {"workload": "config5_moe_train_step", "global_batch": cfg["global_batch"], "seq_len": cfg["seq"],
                   "tokens_per_step": T_global, "layers": 4, "d_model": 1024, "heads": 16, "experts": 8, "top_k": 2,
                   "ffn": 3584, "vocab": 32000, "optimizer": "adam (fp32 master)",
                   "parallelism": f"dp{world}+ep{world}" if world > 1 else "single",
                   "l2": "inputs larger than L2 (per-step working set > 10 GB, no flush needed)"},
        "e2e": {"value": T_global / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": T_global * 4 * world,
                "d2h_bytes_per_step": 4 * world, "ms_per_step": e2e_ms,
                "call": "catnn_moe_trainer_step_host (host tokens -> pinned staging -> device, step, loss -> host)",
                "clocks": {"sm_mhz": clk_e2e.get("sm_mhz"), "reasons": clk_e2e.get("reasons")}},
        "gpu_launches": int(launches),
        "tflops_per_step": step_flops(cfg, T_global) / 1e12,
        "model_tflops_achieved": step_flops(cfg, T_global) / (ms * 1e-3) / 1e12,
        "loss_step0": loss_step0,
        "phases": phase_breakdown,
        "routing": routing,
        "loss_last": last_loss,
        "roofline": {"bound": "tensor", "kernel": "k_gemm_tc grouped (expert W13 forward, rows=%d, N=%d, K=%d)"
                     % (rows, 2 * F, d), "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "peak_source": f"{pk_kind} bf16_tflops (burst, kernel timed alone)",
                     "traffic": traffic_from_profile(rows, cfg["experts"] // world, F, d),
                     "algorithmic_bytes": gemm_bytes(rows, cfg["experts"] // world, F, d), "launch_ms": kms},
        "clocks": clk,
    }
    if world == 1:
        # config 2 (dense GEMM fwd / fwd+bwd, bf16): the metric's "GEMM TFLOP/s and % of tensor peak"
        out["gemm_sweep"] = {"peak_tflops": peak, "peak_source": f"{pk_kind} bf16_tflops",
                             "timing": "device time, calls replayed as a CUDA graph", **gemm_sweep(local, peak)}
    P_host = tr.params().cpu().numpy() if (rank == 0 and world == 1 and not args.no_cpu_baseline) else None
    tr.close()
    if world == 1 and not args.no_workloads:
        cpu = not args.no_cpu_baseline
        out["workloads"] = {"config1_mlp": workload_mlp(local, args.steps, cpu),
                            "config3_block": workload_block(local, cpu),
                            "config4_mixtral_tiny": workload_tiny(local, args.steps, cpu)}
    if P_host is not None:
        out["cpu_baseline"] = cpu_baseline_port(P_host, cfg, T_global)
    if comm is not None:
        comm.close()
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


def _ref_worker(seed):
    """One bounded sample of the reference step (oracle restatement) in this
    worker process: the wall times of a 1-token and a 2-token step."""
    return (oracle_step_seconds(_SHARED["P"], CFG, 1, seed), oracle_step_seconds(_SHARED["P"], CFG, 2, seed + 1))


_SHARED = {}


def run_reference(args):
    """The reference's CPU path (its train::mixtral_step restated in C++ —
    Rust is not available here) on the host cores: one worker process per
    usable core, each running its own steps (the reference's step is
    sequential, so one core per step; independent steps in parallel are how
    a CPU host uses all its cores).

    Each round runs a 1-token and then a 2-token step in every worker (the
    warm-up rounds are discarded: their first touches of the gradient
    buffers fault pages in): the medians give the step's fixed cost and its
    per-token cost, and tokens/s = workers x T / (fixed + T x per-token) for
    the full T = 16384-token step — the fixed cost is charged once per step,
    as a real 16384-token step pays it."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import multiprocessing as mp

    import numpy as np
    cfg = CFG
    n = mix_cfg(cfg).layout()["total"]
    r = np.random.default_rng(cfg["seed"])
    P = (r.standard_normal(n, dtype=np.float32) * 0.02).astype(np.float32)
    _SHARED["P"] = P  # shared copy-on-write with the forked workers (no CUDA in this process)
    oracle_env(split=False, threads=1)  # inherited by the workers: one thread each, the reference's own threading
    try:
        avail = os.sysconf("SC_AVPHYS_PAGES") * os.sysconf("SC_PAGE_SIZE")
    except (ValueError, OSError):
        avail = 64 << 30
    cores = os.cpu_count() or 1
    workers = max(1, min(cores, int((avail - (8 << 30)) // (3 << 30))))
    T = cfg["global_batch"] * cfg["seq"]
    ctx = mp.get_context("fork")  # this process never initialises CUDA
    budget_s = 150.0
    with ctx.Pool(workers) as pool:
        tw = time.perf_counter()
        for i in range(max(1, min(args.warmup, 2))):
            pool.map(_ref_worker, [1000 * (i + 1) + 2 * w for w in range(workers)])
        t_round = (time.perf_counter() - tw) / max(1, min(args.warmup, 2))
        steps = max(1, min(args.steps, max(3, int(budget_s / max(t_round, 1e-3)))))
        t1s, t2s = [], []
        t0 = time.perf_counter()
        for st in range(steps):
            for a, b in pool.map(_ref_worker, [100000 * (st + 1) + 2 * w for w in range(workers)]):
                t1s.append(a)
                t2s.append(b)
        wall = time.perf_counter() - t0
    t1, t2 = statistics.median(t1s), statistics.median(t2s)
    fixed, marg = step_cost_model(t1, t2)
    full = fixed + T * marg
    value = workers * T / full
    sample = (f"{workers} worker processes (nproc {cores}), one thread each; per worker, 1-token steps (median "
              f"{t1:.2f} s over {len(t1s)}) and 2-token steps (median {t2:.2f} s over {len(t2s)}) of the oracle's "
              f"train::mixtral_step at config-5 widths give a fixed cost of {fixed:.2f} s and {marg:.3f} s per token; "
              f"a full {T}-token step extrapolates to {full:.0f} s per worker (linear in tokens; the attention's S^2 "
              f"term, ~6% of the FLOPs at S=2048, is left out, which favours the CPU)")
    out = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": steps,
           "steps_requested": args.steps,
           "warmup": args.warmup, "ms_per_step": full / workers * 1e3, "higher_is_better": True,
           "scaling": "strong", "vs_baseline": None, "dtype": "f32", "impl": "reference",
           "data": "synthetic (token ids uniform [0,32000), weights N(0,0.02), seed 4)",
           "config": {"workload": "config5_moe_train_step", "global_batch": 8, "seq_len": 2048,
                      "tokens_per_step": T, "parallelism": f"{workers} CPU processes", "nproc": cores},
           "sampling_wall_s": wall,
           "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": workers, "kind": "port", "sample": sample,
                            "fixed_s": fixed, "per_token_s": marg},
           "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def main():
    args = parse()
    if args.kernel_only:
        run_kernel_only(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
