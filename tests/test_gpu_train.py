"""End-to-end parity of the native MoE decoder training step against the
oracle's train::mixtral_step (train.rs:261-356): loss, every packed
gradient, and multi-step trajectories (SGD and Adam).

- fp32 path at the reference's own tiny fixture (MixtralConfig::tiny, seed
  7, tokens 1..8, B=2, S=4) and at config 4's full shape (4 SGD steps);
- bf16 tensor-core path at a reduced shape of the benchmark config, against
  the fp32 oracle at the bf16 tolerance (rtol 2e-2, atol 1e-3·scale).
"""
import numpy as np
import pytest
import torch

from gpu_util import bf16_round, close_bf16, close_f32, rel_l2
from oracle import oracle as O

pytestmark = pytest.mark.gpu

from catnn_b200.train import MoeConfig, MoeTrainer, init_params, packed_layout  # noqa: E402


def ocfg(c):
    return O.MixCfg(c.vocab, c.hidden, c.mid, c.layers, c.heads, c.kv_heads, c.experts, c.top_k, c.rms_eps, c.rope_theta,
                    c.window or None)


def groups(cfg):
    """(name, slice) per parameter tensor of the packed vector."""
    L = packed_layout(cfg)
    out = [("embed", slice(0, L["layer0"]))]
    names = ["rms_attn", "wq", "wk", "wv", "wo", "rms_moe", "gate", "w1", "w3", "w2"]
    for l in range(cfg.layers):
        base = L["layer0"] + l * L["layer_stride"]
        for i, n in enumerate(names):
            end = L[names[i + 1]] if i + 1 < len(names) else L["layer_stride"]
            out.append((f"L{l}.{n}", slice(base + L[n], base + end)))
    out.append(("final_norm", slice(L["final_norm"], L["lm_head"])))
    out.append(("lm_head", slice(L["lm_head"], L["total"])))
    return out


def tc_inputs(cfg, P):
    """The parameters as the bf16 path consumes them: every tensor-core GEMM
    weight (wq, wk, wv, wo, w1, w3, w2, LM head) rounded to bf16; the
    embedding table, RMSNorm weights and router gate stay fp32 (the gather,
    the norms and the fp32 router read the fp32 master)."""
    L = packed_layout(cfg)
    Q = P.copy()
    def rnd(sl):
        Q[sl] = bf16_round(Q[sl])
    for l in range(cfg.layers):
        base = L["layer0"] + l * L["layer_stride"]
        rnd(slice(base + L["wq"], base + L["rms_moe"]))   # wq, wk, wv, wo
        rnd(slice(base + L["w1"], base + L["layer_stride"]))  # w1, w3, w2
    rnd(slice(L["lm_head"], L["total"]))
    return Q


def run_compare(cfg, P, tokens, close, steps=1, exact=False, report=None, oracle_params=None):
    """exact=True also runs the oracle's f64 instantiation and passes it to
    `close` so an element the fp32 oracle itself rounds worse than the band
    allows is checked against the exact value."""
    tr = MoeTrainer(cfg)
    tr.set_params(P)
    tok = torch.as_tensor(tokens.astype(np.int32)).cuda()
    loss = torch.zeros(1, device="cuda")
    oc = ocfg(cfg)
    Pref = P.copy()
    to_oracle = oracle_params or (lambda p: p)
    m = np.zeros_like(P)
    v = np.zeros_like(P)
    for s in range(steps):
        tr.step(tok, update=False, loss_out=loss)
        torch.cuda.synchronize()
        tr.check()
        rl, rg = O.mixtral_step(oc, to_oracle(Pref), tokens, cfg.batch, cfg.seq)
        ex = O.mixtral_step(oc, Pref.astype(np.float64), tokens, cfg.batch, cfg.seq, f64=True) if exact else None
        close(loss, np.float32(rl), what=f"loss step {s}", exact=None if ex is None else ex[0])
        g = tr.grads().cpu().numpy()
        gscale = float(np.max(np.abs(rg)))  # a tensor whose gradient vanishes is measured on the model's scale
        for name, sl in groups(cfg):
            close(g[sl], rg[sl], what=f"grad {name} step {s}", exact=None if ex is None else ex[1][sl],
                  scale=max(gscale * 1e-2, float(np.max(np.abs(rg[sl])))))
        if report is not None:
            report.append({name: rel_l2(g[sl], rg[sl]) for name, sl in groups(cfg)})
        tr.step(tok, update=True, loss_out=loss)  # same step again, now with the update
        torch.cuda.synchronize()
        if cfg.optimizer == 0:
            Pref = O.sgd_put(Pref, rg, cfg.lr)
        else:
            Pref, m, v, _ = O.adam_put(Pref, rg, m, v, s, cfg.lr, cfg.beta1, cfg.beta2, cfg.adam_eps)
        close(tr.params().cpu().numpy(), Pref, what=f"params after step {s}", exact=None)
    tr.close()


def test_tiny_fixture_fp32():
    """MixtralConfig::tiny with seeded LCG weights (moe.rs:247), seed 7, tokens
    1..8, three SGD steps: loss, every gradient and the parameters at rtol 1e-5
    (floor 1e-5 of each tensor's scale), or at least as close to the f64 value
    as the fp32 oracle (LCG(-1,1) weights make this chain badly conditioned)."""
    cfg = MoeConfig.make(32, 32, 64, 2, 4, 2, 4, 2, batch=2, seq=4, window=8, rope_theta=1e4, dtype=torch.float32,
                         optimizer="sgd", lr=0.02)
    P = O.mixtral_seeded(ocfg(cfg), 7)
    run_compare(cfg, P, np.arange(1, 9), close_f32, steps=3, exact=True)


def test_mixtral_tiny_config4_fp32():
    """Config 4 at its full shape (mixtral-tiny: 2 layers, d256, 4 heads, 8
    experts top-2, SwiGLU 256->512->256, RMSNorm, vocab 1024, seq 256, batch 4;
    token ids uniform in [0, 1024), weights N(0, 0.02), SGD lr 0.05, 4 steps,
    seed 3), fp32 path against train::mixtral_step at rtol 1e-5 with the f64
    fallback, every step: loss, all gradients, parameters after the update."""
    cfg = MoeConfig.make(1024, 256, 512, 2, 4, 4, 8, 2, batch=4, seq=256, rope_theta=1e4, dtype=torch.float32,
                         optimizer="sgd", lr=0.05)
    P = init_params(cfg, 3)
    tokens = np.random.default_rng(3).integers(0, 1024, cfg.batch * cfg.seq)
    run_compare(cfg, P, tokens, close_f32, steps=4, exact=True)


@pytest.mark.parametrize("hidden,mid,layers,heads,batch,seq", [(256, 512, 2, 4, 2, 128), (1024, 1024, 1, 16, 1, 256)])
def test_moe_sweep_shape_bf16_adam(hidden, mid, layers, heads, batch, seq):
    """Reduced config 5 (bf16 compute, fp32 master, fp32 router, Adam) vs the fp32 oracle;
    the second case has config 5's width (d 1024, 16 heads of 64), which takes the
    width-specific kernels (fused RMSNorm backward, tcgen05 attention).

    Top-k routing is discontinuous: bf16 rounding of the attention branch
    (~0.2%) moves a few tokens across a near-tie, and those tokens then
    differ by O(1). So, as fd64.rs does for its MoE checks, the oracle replays
    the GPU's routing decisions (mixtral_step_frozen) for the tensor
    comparison, and the fraction of decisions that differ from the free
    oracle is bounded separately. The oracle reads the weights the tensor
    cores consume (tc_inputs)."""
    cfg = MoeConfig.make(2048, hidden, mid, layers, heads, heads, 8, 2, batch=batch, seq=seq, rope_theta=1e6,
                         dtype=torch.bfloat16, optimizer="adam", lr=1e-3)
    P = init_params(cfg, 4)
    tokens = np.random.default_rng(4).integers(0, 2048, cfg.batch * cfg.seq)
    tr = MoeTrainer(cfg)
    tr.set_params(P)
    tok = torch.as_tensor(tokens.astype(np.int32)).cuda()
    loss = torch.zeros(1, device="cuda")
    oc = ocfg(cfg)
    Pq = tc_inputs(cfg, P)
    losses = []
    for step in range(3):
        tr.step(tok, update=False, loss_out=loss)
        torch.cuda.synchronize()
        tr.check()
        idx = np.stack([np.stack([O.topk_softmax(r, cfg.top_k)[0] for r in tr.activation("router_logits", l).cpu().numpy()])
                        for l in range(cfg.layers)])
        g = tr.grads().cpu().numpy()
        if step == 0:
            rl, rg = O.mixtral_step_frozen(oc, Pq, tokens, cfg.batch, cfg.seq, idx)
            close_bf16(loss, np.float32(rl), what="loss")
            for name, sl in groups(cfg):
                e = rel_l2(g[sl], rg[sl])
                assert e <= 2e-2, (name, e)
                close_bf16(g[sl], rg[sl], what=f"grad {name}")
            # routing agreement with the free-running oracle's forward
            free = oracle_routing(cfg, Pq, tokens)
            flips = float(np.mean(np.any(np.sort(free, -1) != np.sort(idx, -1), -1)))
            assert flips <= 0.05, flips
        losses.append(float(loss))
        tr.step(tok, update=True, loss_out=loss)
    assert losses[-1] < losses[0], losses
    tr.close()


def oracle_routing(cfg, P, tokens):
    """Per-layer top-k of the oracle's own forward (no freezing)."""
    L = packed_layout(cfg)
    h, F, E, B, S = cfg.hidden, cfg.mid, cfg.experts, cfg.batch, cfg.seq
    hd = h // cfg.heads
    def g(l, key, shape):
        o = L["layer0"] + l * L["layer_stride"] + L[key]
        return P[o:o + int(np.prod(shape))].reshape(shape)
    x = O.embedding(tokens, P[:cfg.vocab * h].reshape(cfg.vocab, h))
    out = []
    for l in range(cfg.layers):
        xn = O.rmsnorm(x, g(l, "rms_attn", (h,)), cfg.rms_eps)
        x = x + O.gqa(xn.reshape(B, S, h), g(l, "wq", (h, cfg.heads * hd)), g(l, "wk", (h, cfg.kv_heads * hd)),
                      g(l, "wv", (h, cfg.kv_heads * hd)), g(l, "wo", (cfg.heads * hd, h)), cfg.heads, cfg.kv_heads,
                      cfg.rope_theta, cfg.window or None).reshape(B * S, h)
        xm = O.rmsnorm(x, g(l, "rms_moe", (h,)), cfg.rms_eps)
        idx, _, _ = O.route(xm, g(l, "gate", (h, E)), cfg.top_k)
        out.append(idx)
        x = x + O.moe(xm, g(l, "gate", (h, E)), g(l, "w1", (E, h, F)), g(l, "w3", (E, h, F)), g(l, "w2", (E, F, h)),
                      cfg.top_k)
    return np.stack(out)


def test_host_step_matches_device_step():
    cfg = MoeConfig.make(512, 128, 256, 1, 2, 2, 4, 2, batch=2, seq=64, dtype=torch.bfloat16, optimizer="adam")
    P = init_params(cfg, 5)
    tokens = np.random.default_rng(5).integers(0, 512, 128)
    a, b = MoeTrainer(cfg), MoeTrainer(cfg)
    a.set_params(P)
    b.set_params(P)
    la = [a.step_host(tokens) for _ in range(3)]
    tok = torch.as_tensor(tokens.astype(np.int32)).cuda()
    loss = torch.zeros(1, device="cuda")
    lb = []
    for _ in range(3):
        b.step(tok, loss_out=loss)
        lb.append(float(loss))
    assert la == lb, (la, lb)  # deterministic: same kernels, same order
    assert la[-1] < la[0]
    a.close()
    b.close()


def test_bad_token_is_reported():
    cfg = MoeConfig.make(64, 128, 256, 1, 2, 2, 4, 2, batch=1, seq=64, dtype=torch.bfloat16)
    tr = MoeTrainer(cfg)
    tr.set_params(init_params(cfg, 6))
    tok = torch.full((64,), 64, dtype=torch.int32, device="cuda")
    tr.step(tok, update=False)
    from catnn_b200.errors import ShapeMismatch
    with pytest.raises(ShapeMismatch):
        tr.check()
    tr.close()


def test_graph_replay_matches_eager():
    """The step replayed as a CUDA graph gives the eager step's results bit for
    bit (loss every step, then parameters, gradients and Adam state through
    updates), and its launches are still counted."""
    cfg = MoeConfig.make(2048, 256, 512, 2, 4, 4, 8, 2, batch=2, seq=128, rope_theta=1e6, dtype=torch.bfloat16,
                         optimizer="adam", lr=1e-3)
    P = init_params(cfg, 5)
    tok = torch.as_tensor(np.random.default_rng(5).integers(0, 2048, cfg.batch * cfg.seq).astype(np.int32)).cuda()
    a, b = MoeTrainer(cfg), MoeTrainer(cfg)
    a.set_params(P)
    b.set_params(P)
    b.set_graphs(True)
    la, lb = torch.zeros(1, device="cuda"), torch.zeros(1, device="cuda")
    n0 = b.ctx.launch_count()
    for upd in (True, True, True, False, False, False, True):
        a.step(tok, update=upd, loss_out=la)
        b.step(tok, update=upd, loss_out=lb)
        torch.cuda.synchronize()
        assert torch.equal(la, lb), (upd, float(la), float(lb))
    assert torch.equal(a.params(), b.params())
    assert torch.equal(a.grads(), b.grads())
    assert b.ctx.launch_count() - n0 > 7 * 100, "replayed launches are counted"
    a.check()
    b.check()
    a.close()
    b.close()


def test_step_timeline_phases():
    """catnn_moe_trainer_set_profile / _timeline: the device-clock stamps of a
    profiled step name every phase (per layer), are non-decreasing, and their
    sum is the step's device time; with graph replay the stamps are replayed
    too; profiling off leaves the step's results unchanged."""
    cfg = MoeConfig.make(1024, 256, 512, 2, 4, 4, 8, 2, batch=2, seq=128, rope_theta=1e4, dtype=torch.bfloat16,
                         optimizer="adam", lr=1e-3)
    P = init_params(cfg, 8)
    tok = torch.as_tensor(np.random.default_rng(8).integers(0, 1024, 256).astype(np.int32)).cuda()
    a, b = MoeTrainer(cfg), MoeTrainer(cfg)
    a.set_params(P)
    b.set_params(P)
    b.set_graphs(True)
    b.set_profile(True)
    la, lb = torch.zeros(1, device="cuda"), torch.zeros(1, device="cuda")
    for _ in range(4):  # eager, eager warm-up, capture, replay
        a.step(tok, update=True, loss_out=la)
        b.step(tok, update=True, loss_out=lb)
        torch.cuda.synchronize()
        assert torch.equal(la, lb)
    phases = b.timeline()
    names = [n for n, _ in phases]
    assert names[0] == "embedding" and names[-1] == "updates joined"
    assert names.count("fwd attention") == 2 and names.count("bwd moe") == 2
    assert all(ms >= 0 for _, ms in phases)
    total = sum(ms for _, ms in phases)
    assert 0 < total < 1000
    b.set_profile(False)
    b.step(tok, update=True, loss_out=lb)
    a.step(tok, update=True, loss_out=la)
    torch.cuda.synchronize()
    assert torch.equal(la, lb) and torch.equal(a.params(), b.params())
    a.close()
    b.close()
