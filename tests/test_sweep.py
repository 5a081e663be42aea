"""The measured-sweep entry point (catnn_b200.sweep) on CPU: the restated
parameter counts and Spark cost formula, and the table it prints from bench
JSON lines."""
import json

from catnn_b200 import sweep

MIXTRAL_8X7B = {"vocab": 32000, "hidden": 4096, "mid": 14336, "layers": 32, "heads": 32, "kv_heads": 8,
                "experts": 8, "top_k": 2}


def test_param_counts_match_mixtral_8x7b():
    # Mixtral 8x7B: 46.7 B parameters, 12.9 B active per token (top-2 of 8)
    assert abs(sweep.param_count(MIXTRAL_8X7B) / 1e9 - 46.70) < 0.01
    assert abs(sweep.active_param_count(MIXTRAL_8X7B) / 1e9 - 12.88) < 0.01


def test_spark_cost_terms():
    cfg = dict(MIXTRAL_8X7B)
    seq, gbs = 2048, 8
    act, tot = sweep.active_param_count(cfg), sweep.param_count(cfg)
    # one Spark: compute-bound stage, micro = 8 stages in the 1F1B pipe, no all-reduce
    compute = 6.0 * act * gbs * seq / 250e12
    hbm = act * 2.0 * gbs * seq * 2.0 / 273e9
    assert abs(sweep.spark_train_cost(cfg, 1, 1, 1, 1, seq, gbs) - gbs * max(compute, hbm)) < 1e-9 * compute
    # EP = DP = 4: a quarter of the work on micro-batches of 2 sequences, plus the gradient all-reduce
    micro = gbs // 4
    compute4 = 6.0 * act * micro * seq / 4 / 250e12
    hbm4 = act * 2.0 * micro * seq * 2.0 / 4 / 273e9
    ar = 2.0 * 3 / 4 * (2.0 * tot / 16) / 25e9
    got = sweep.spark_train_cost(cfg, 4, 1, 1, 4, seq, gbs)
    assert abs(got - (micro * max(compute4, hbm4) + ar)) < 1e-9 * got


def test_table_from_bench_lines(tmp_path, capsys):
    lines = [{"metric": "m", "value": 7.5e5 * n ** 0.8, "ms_per_step": 16384 / (7.5e5 * n ** 0.8) * 1e3, "n_gpus": n,
              "e2e": {"value": 7.4e5 * n ** 0.8}, "loss_step0": 10.5721} for n in (1, 2, 4, 8)]
    lines.append({"impl": "reference", "value": 5.0, "n_gpus": 1})
    f = tmp_path / "scale.jsonl"
    f.write_text("\n".join(json.dumps(l) for l in lines) + "\n")
    rows = sweep.main(["--json", str(f)])
    out = capsys.readouterr().out
    assert [r["n"] for r in rows] == [1, 2, 4, 8]
    assert "config5" in out and "spark_tok/s" in out and "b200_tok/s" in out
    for r in rows:
        assert r["spark_tok_s"] > 0 and abs(r["b200_tok_s"] - 7.5e5 * r["n"] ** 0.8) < 1e-6 * r["b200_tok_s"]
