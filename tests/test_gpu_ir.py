"""The reference's operator boundary driven as a graph on the GPU.

IR graphs run through ``ir.train_step`` — the one-device training runtime of
crates/catnn-rt/src/coord.rs (forward_one, loss_one, backward_one,
apply_pending) over ``eval_gpu`` / ``adjoint_of`` — with every activation,
cotangent, parameter and optimizer state resident on the device:

- an MLP IrGraph (linear, relu, linear, softmax cross-entropy) trained with
  SGD against the oracle's train::mlp_step + Sgd::put (train.rs:71-91);
- the Mixtral IR chain with its residual adds wired as residual_add nodes,
  against train::mixtral_step (train.rs:261-356): loss and every gradient of
  a step, then parameters after SGD steps;
- rematerialization: a step whose checkpointed activations are dropped after
  the forward and rebuilt by ensure_act (coord.rs:436-473) gives the same
  parameters bit for bit as the step that kept them (the reference's
  constrained_equals_unconstrained, train.rs:826).
fp32 path, rtol 1e-5 with a floor of 1e-5 of each tensor's scale, or at least
as close to the f64 value as the fp32 oracle.
"""
import numpy as np
import pytest
import torch

from gpu_util import close_f32, dev, host, rng
from oracle import oracle as O

pytestmark = pytest.mark.gpu

from catnn_b200 import ir  # noqa: E402
from catnn_b200.train import MoeConfig, init_params, packed_layout  # noqa: E402


def mlp_graph(w1, b1, w2, b2):
    g = ir.IrGraph("mlp")
    x = g.add("x", ir.OpenOp.identity(), is_input=True)
    h = g.add("fc1", ir.OpenOp.linear(784, 256), {"w": w1, "b": b1}, [x])
    a = g.add("relu", ir.OpenOp.relu(), {}, [h])
    y = g.add("fc2", ir.OpenOp.linear(256, 10), {"w": w2, "b": b2}, [a])
    g.outputs.append(y)
    return g


def test_mlp_graph_trains_like_mlp_step():
    r = rng(0)
    a1, a2 = np.sqrt(6.0 / (784 + 256)), np.sqrt(6.0 / (256 + 10))
    W = [r.uniform(-a1, a1, (784, 256)).astype(np.float32), np.zeros(256, np.float32),
         r.uniform(-a2, a2, (256, 10)).astype(np.float32), np.zeros(10, np.float32)]
    x = r.standard_normal((64, 784)).astype(np.float32)
    lab = r.integers(0, 10, 64)
    G = [dev(t) for t in W]
    g = mlp_graph(*G)
    st = ir.DeviceRt(g)
    st.feed(g, [dev(x)], dev(lab, torch.int32))
    handler = ir.DeviceHandler()
    ref = [t.copy() for t in W]
    for step in range(4):
        loss = ir.train_step(g, st, handler, opt="sgd", lr=0.05)
        rl, *rg = O.mlp_step(*ref, x, labels=lab)
        ref = [O.sgd_put(p, gg, 0.05) for p, gg in zip(ref, rg)]
        close_f32(loss, np.float32(rl), what=f"loss at step {step}")
    for name, got, want in zip(("w1", "b1", "w2", "b2"), G, ref):
        close_f32(got, want, what=f"{name} after 4 steps")
    kinds = {e.kind for e in handler.events}
    assert kinds == {"KernelStart", "KernelEnd"} and len(handler.events) >= 4 * 2 * 6


def ocfg(c):
    return O.MixCfg(c.vocab, c.hidden, c.mid, c.layers, c.heads, c.kv_heads, c.experts, c.top_k, c.rms_eps, c.rope_theta,
                    c.window or None)


def run_mixtral_graph(cfg, P, tokens, steps, lr, checkpointed=()):
    Pd = dev(P)
    g, tok = ir.mixtral_graph(cfg, Pd, cfg.batch, cfg.seq)
    st = ir.DeviceRt(g)
    n = cfg.batch * cfg.seq
    targets = np.array([tokens[(i + 1) % n] % cfg.vocab for i in range(n)])
    st.feed(g, [dev(tokens.reshape(cfg.batch, cfg.seq), torch.int32)], dev(targets, torch.int32))
    handler = ir.DeviceHandler()
    out = []
    for s in range(steps):
        loss = ir.train_step(g, st, handler, checkpointed=checkpointed, update=False)
        grads = ir.pack_grads(g, st, cfg)
        out.append((float(loss), host(grads)))
        ir.apply_pending(st, "sgd", lr)
    return Pd, out, st


@pytest.mark.parametrize("shape", ["tiny_fixture", "config4_reduced"])
def test_mixtral_graph_with_residuals_matches_mixtral_step(shape):
    if shape == "tiny_fixture":
        # MixtralConfig::tiny, seeded LCG weights (moe.rs:247), seed 7, tokens 1..8
        cfg = MoeConfig.make(32, 32, 64, 2, 4, 2, 4, 2, batch=2, seq=4, window=8, rope_theta=1e4, dtype=torch.float32,
                             optimizer="sgd", lr=0.02)
        P = O.mixtral_seeded(ocfg(cfg), 7)
        tokens = np.arange(1, 9)
    else:
        cfg = MoeConfig.make(1024, 256, 512, 2, 4, 4, 8, 2, batch=2, seq=64, rope_theta=1e4, dtype=torch.float32,
                             optimizer="sgd", lr=0.05)
        P = init_params(cfg, 3)
        tokens = rng(3).integers(0, 1024, cfg.batch * cfg.seq)
    Pd, out, _ = run_mixtral_graph(cfg, P, tokens, 2, cfg.lr)
    oc = ocfg(cfg)
    Pref = P.copy()
    for s, (loss, grads) in enumerate(out):
        rl, rg = O.mixtral_step(oc, Pref, tokens, cfg.batch, cfg.seq)
        el, eg = O.mixtral_step(oc, Pref.astype(np.float64), tokens, cfg.batch, cfg.seq, f64=True)
        close_f32(np.float32(loss), np.float32(rl), what=f"loss step {s}", exact=el)
        L = packed_layout(cfg)
        gscale = float(np.max(np.abs(rg)))
        bounds = sorted({0, L["layer0"], L["final_norm"], L["lm_head"], L["total"]} |
                        {L["layer0"] + l * L["layer_stride"] + L[k] for l in range(cfg.layers)
                         for k in ("rms_attn", "wq", "wk", "wv", "wo", "rms_moe", "gate", "w1", "w3", "w2")})
        for lo, hi in zip(bounds[:-1], bounds[1:]):
            sl = slice(lo, hi)
            close_f32(grads[sl], rg[sl], what=f"grad [{lo}, {hi}) step {s}", exact=eg[sl],
                      scale=max(gscale * 1e-2, float(np.max(np.abs(rg[sl])))))
        Pref = O.sgd_put(Pref, rg, cfg.lr)
    close_f32(Pd, Pref, what="parameters after 2 steps")


def test_rematerialized_step_is_bit_identical():
    """Dropping every layer's normalized inputs, attention and expert outputs
    after the forward (they are rebuilt with eval_gpu when the backward needs
    them) leaves the trajectory unchanged bit for bit."""
    cfg = MoeConfig.make(512, 128, 256, 2, 4, 2, 4, 2, batch=2, seq=32, rope_theta=1e4, dtype=torch.float32,
                         optimizer="sgd", lr=0.05)
    P = init_params(cfg, 9)
    tokens = rng(9).integers(0, 512, cfg.batch * cfg.seq)
    dropped = [f"L{l}.{k}" for l in range(cfg.layers) for k in ("rms_attn", "gqa", "res_attn", "rms_moe", "moe")]
    dropped += ["final_norm"]
    Pa, out_a, _ = run_mixtral_graph(cfg, P, tokens, 3, cfg.lr)
    Pb, out_b, st = run_mixtral_graph(cfg, P, tokens, 3, cfg.lr, checkpointed=dropped)
    assert st.rematerialized >= len(dropped)
    for (la, ga), (lb, gb) in zip(out_a, out_b):
        assert la == lb
        assert np.array_equal(ga, gb)
    assert torch.equal(Pa, Pb), "parameter drift between the stored and the rematerialized step"


def test_checkpointed_input_cannot_be_rematerialized():
    """coord.rs:454-457: a graph input dropped after the forward is a host
    value the device cannot rebuild."""
    from catnn_b200.errors import Fibration
    r = rng(1)
    G = [dev(r.standard_normal((784, 256)) * 0.05), dev(np.zeros(256)), dev(r.standard_normal((256, 10)) * 0.05),
         dev(np.zeros(10))]
    g = mlp_graph(*G)
    st = ir.DeviceRt(g)
    st.feed(g, [dev(r.standard_normal((8, 784)))], dev(r.integers(0, 10, 8), torch.int32))
    with pytest.raises(Fibration, match="checkpointed"):
        ir.train_step(g, st, ir.DeviceHandler(), checkpointed=["x"])
