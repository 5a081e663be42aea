"""Measured Mixtral training sweep beside the reference's modelled one.

The reference's ``catnn mixtral-train-sweep`` (crates/catnn-cli/src/main.rs:587)
prints, for N = 1/2/4/8 DGX Sparks, a step time and tokens/s *modelled* by
``spark_train::train_cost`` (crates/catnn-compile/src/spark_train.rs:226-271)
and never runs a training step. This module runs the measured counterpart on
B200s — ``bench.py`` at N = 1/2/4/8 (one process per GPU, the trainer's data
+ expert parallel step) — or reads its JSON lines, and prints both columns
in the reference's table layout (spark_train.rs:613-646).

  python -m catnn_b200.sweep [--gpus 1,2,4,8] [--steps 10] [--json FILE ...]

The modelled column restates ``train_cost`` for the plan the B200 run uses:
expert parallel EP = N over data parallel DP = N, no tensor or pipeline
parallelism, no checkpointing or offload, bf16 (DgxSparkSpec::official,
crates/catnn-core/src/architecture/spark.rs:40-73).
"""
import argparse
import json
import os
import subprocess
import sys

# DgxSparkSpec::official (spark.rs:40-55)
SPARK_MEMORY_BPS = 273.0e9
SPARK_CX7_BYTES_PER_S = 200.0e9 / 8.0
SPARK_FP4_FLOPS = 1.0e15
SPARK_BF16_FLOPS = SPARK_FP4_FLOPS * 0.25  # peak_flops(Bf16), spark.rs:67-73
SPARK_FP8_FLOPS = SPARK_FP4_FLOPS * 0.5


def param_count(cfg):
    """MixtralConfig::param_count (crates/catnn-core/src/spec/mixtral.rs:148-164),
    untied embeddings."""
    h, mid, v, layers = cfg["hidden"], cfg["mid"], cfg["vocab"], cfg["layers"]
    hd = h // cfg["heads"]
    q, kv = cfg["heads"] * hd, cfg["kv_heads"] * hd
    attn = layers * (h * q + h * kv + h * kv + q * h)
    norms = layers * 2 * h + h
    router = layers * h * cfg["experts"]
    experts = layers * cfg["experts"] * 3 * h * mid
    return v * h + v * h + attn + norms + router + experts


def active_param_count(cfg):
    """MixtralConfig::active_param_count (mixtral.rs:166-175): idle experts left out."""
    idle = cfg["layers"] * (cfg["experts"] - cfg["top_k"]) * 3 * cfg["hidden"] * cfg["mid"]
    return max(param_count(cfg) - idle, 0)


def spark_train_cost(cfg, ep, tp, pp, dp, seq, global_batch, mixed_fp8=False):
    """spark_train::train_cost (spark_train.rs:226-271) without checkpointing
    or NVMe offload: seconds per training step on DGX Sparks."""
    active = float(active_param_count(cfg))
    micro = max(global_batch // max(dp, 1), 1)
    tokens = micro * seq
    flops = 6.0 * active * tokens / max(ep * tp, 1)
    compute = flops / (SPARK_FP8_FLOPS if mixed_fp8 else SPARK_BF16_FLOPS)
    hbm = active * 2.0 * tokens * 2.0 / max(ep * tp, 1) / SPARK_MEMORY_BPS
    gbytes = 2.0 * param_count(cfg) / max(ep * tp * pp * dp, 1)
    ar = 2.0 * (dp - 1) / dp * gbytes / SPARK_CX7_BYTES_PER_S if dp > 1 else 0.0
    tp_ar = (4.0 * cfg["layers"] * 2.0 * (tp - 1) / tp * cfg["hidden"] * 2.0 / SPARK_CX7_BYTES_PER_S * tokens
             if tp > 1 else 0.0)
    stage = max(compute, hbm) / max(pp, 1)
    pipe = (pp + micro - 1) * stage
    return pipe + ar + tp_ar


def rows_for(cfg, results, seq, global_batch):
    """One table row per measured N: the Spark model for EP = DP = N beside
    the B200 measurement."""
    out = []
    for n in sorted(results):
        r = results[n]
        step = spark_train_cost(cfg, n, 1, 1, n, seq, global_batch)
        out.append({"n": n, "ep": n, "tp": 1, "pp": 1, "dp": n, "spark_step_s": step,
                    "spark_tok_s": global_batch * seq / step, "b200_step_s": r["ms_per_step"] / 1e3,
                    "b200_tok_s": r["value"], "b200_e2e_tok_s": (r.get("e2e") or {}).get("value"),
                    "loss_step0": r.get("loss_step0")})
    return out


def format_table(model, rows, seq, global_batch):
    s = ("model              N  mp    EP/TP/PP/DP  spark_step_s  spark_tok/s   b200_step_s   b200_tok/s  "
         "b200_e2e_tok/s   x_spark  loss_step0  seq  gbs\n")
    s += "-" * 150 + "\n"
    for r in rows:
        e2e = r["b200_e2e_tok_s"]
        s += (f"{model:<18} {r['n']:>2}  bf16  {r['ep']:>2}/{r['tp']:<2}/{r['pp']:<2}/{r['dp']:<2}  "
              f"{r['spark_step_s']:>12.4f} {r['spark_tok_s']:>12.1f} {r['b200_step_s']:>13.5f} {r['b200_tok_s']:>12.1f} "
              f"{(e2e if e2e is not None else float('nan')):>15.1f} {r['b200_tok_s'] / r['spark_tok_s']:>9.1f} "
              f"{(r['loss_step0'] if r['loss_step0'] is not None else float('nan')):>11.6f} {seq:>4} {global_batch:>4}\n")
    return s


def run_bench(n, steps, warmup, root):
    """bench.py at N GPUs (torchrun for N > 1); returns its JSON line."""
    bench = os.path.join(root, "bench.py")
    args = ["--gpus", str(n), "--steps", str(steps), "--warmup", str(warmup), "--no-cpu-baseline", "--no-workloads"]
    if n == 1:
        cmd = [sys.executable, bench] + args
    else:
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
               "--master-addr", "127.0.0.1", "--master-port", str(29600 + n), bench] + args
    r = subprocess.run(cmd, capture_output=True, text=True, check=True)
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    return json.loads(lines[-1])


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("--gpus", default="1,2,4,8")
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--json", nargs="*", help="bench.py JSON lines (files) to tabulate instead of running")
    args = p.parse_args(argv)
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    sys.path.insert(0, root)
    import bench
    c = bench.CFG
    cfg = {"vocab": c["vocab"], "hidden": c["hidden"], "mid": c["mid"], "layers": c["layers"], "heads": c["heads"],
           "kv_heads": c["kv_heads"], "experts": c["experts"], "top_k": c["top_k"]}
    results = {}
    if args.json:
        for path in args.json:
            for line in open(path):
                if line.startswith("{"):
                    d = json.loads(line)
                    if d.get("impl", "ours") != "reference" and "n_gpus" in d:
                        results[int(d["n_gpus"])] = d
    else:
        for n in (int(x) for x in args.gpus.split(",")):
            results[n] = run_bench(n, args.steps, args.warmup, root)
    rows = rows_for(cfg, results, c["seq"], c["global_batch"])
    print("Mixtral-style training sweep: measured on B200 beside the DGX Spark model (spark_train::train_cost)")
    print(f"config 5: {c['layers']}L d{c['hidden']} h{c['heads']} E{c['experts']} top-{c['top_k']} F{c['mid']} "
          f"V{c['vocab']}; bf16 compute, fp32 master + Adam; seq={c['seq']} global_batch={c['global_batch']}")
    print()
    print(format_table("config5", rows, c["seq"], c["global_batch"]), end="")
    print()
    print("executed: the full training step on B200 (data + expert parallel, NCCL + NVLink peer memory) at each N;")
    print("modelled: the Spark column, the reference's cost formula for EP = DP = N, TP = PP = 1, no checkpointing.")
    return rows


if __name__ == "__main__":
    main()
