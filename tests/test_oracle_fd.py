"""Finite-difference checks of the oracle's adjoints.

Two tiers, as in the reference:
* f32 FD with eps 1e-3 at the tolerances of adjoint.rs:984-1088;
* f64 central differences (eps 1e-6) on the f64 instantiation of the same
  loop nests at the tolerances of fd64.rs:1232-1250 (2e-6 rel for isolated
  ops, 2e-5 rel / 5e-3 abs for the tiny Mixtral end-to-end groups).
"""
import numpy as np
import pytest

from oracle import oracle as O


def lcg64(shape, seed):
    return O.lcg(int(np.prod(shape)), seed).astype(np.float64).reshape(shape)


def fd_max(p, analytic, f, eps, n_probe):
    """fd64.rs:39-71 — relative error counted only where |g| >= 1e-4."""
    p = p.copy()
    flat = p.reshape(-1)
    n = flat.size
    take = max(1, min(n_probe, n))
    step = max(1, n // take)
    max_rel = max_abs = 0.0
    for i in list(range(0, n, step))[:take]:
        old = flat[i]
        flat[i] = old + eps
        fp = f(p)
        flat[i] = old - eps
        fm = f(p)
        flat[i] = old
        num = (fp - fm) / (2 * eps)
        a = analytic.reshape(-1)[i]
        ab = abs(num - a)
        scale = max(abs(a), abs(num))
        if scale >= 1e-4:
            max_rel = max(max_rel, ab / scale)
        max_abs = max(max_abs, ab)
    return max_rel, max_abs


ISO = 2e-6


def test_fd64_linear():
    x, w = lcg64((3, 4), 1), lcg64((4, 5), 2)
    dy = np.ones((3, 5))
    _, dw, _ = O.linear_backward(x, w, dy, f64=True)
    rel, _ = fd_max(w, dw, lambda wp: O.linear(x, wp, parallel=False, f64=True).sum(), 1e-6, 20)
    assert rel < ISO


def test_fd64_relu_gelu():
    for fwd, bwd, seed in ((O.relu, O.relu_backward, 3), (O.gelu, O.gelu_backward, 4)):
        x = lcg64((8,), seed)
        dx = bwd(x, np.ones(8), f64=True)
        rel, _ = fd_max(x, dx, lambda xp: fwd(xp, f64=True).sum(), 1e-6, 8)
        assert rel < ISO


def test_fd64_softmax():
    z = lcg64((2, 5), 5)
    y = O.softmax_last(z, f64=True)
    coeff = np.array([(i % 5 + 1) for i in range(10)], np.float64).reshape(2, 5)
    dx = O.softmax_backward(y, coeff, f64=True)
    rel, _ = fd_max(z, dx, lambda zp: (O.softmax_last(zp, f64=True) * coeff).sum(), 1e-6, 10)
    assert rel < ISO


def test_fd64_mse_ce():
    p, t = lcg64((6,), 6), lcg64((6,), 7)
    _, d = O.mse_loss(p, t, f64=True)
    rel, _ = fd_max(p, d, lambda pp: O.mse_loss(pp, t, f64=True)[0], 1e-6, 6)
    assert rel < ISO
    z = lcg64((2, 4), 8)
    tg = np.array([1, 2])
    _, d = O.cross_entropy(z, tg, f64=True)
    rel, _ = fd_max(z, d, lambda zp: O.cross_entropy(zp, tg, f64=True)[0], 1e-6, 8)
    assert rel < ISO


def test_fd64_rmsnorm_layernorm():
    x = lcg64((2, 6), 9)
    w = np.ones(6)
    dy = np.ones((2, 6))
    dx, dw = O.rmsnorm_backward(x, w, dy, f64=True)
    assert fd_max(w, dw, lambda wp: O.rmsnorm(x, wp, f64=True).sum(), 1e-6, 6)[0] < ISO
    assert fd_max(x, dx, lambda xp: O.rmsnorm(xp, w, f64=True).sum(), 1e-6, 12)[0] < ISO
    g, b = lcg64((6,), 5), lcg64((6,), 6)
    coeff = lcg64((2, 6), 11)
    dx, dg, db = O.layer_norm_backward(x, g, coeff, f64=True)
    assert fd_max(g, dg, lambda gp: (O.layer_norm(x, gp, b, f64=True) * coeff).sum(), 1e-6, 6)[0] < ISO
    assert fd_max(x, dx, lambda xp: (O.layer_norm(xp, g, b, f64=True) * coeff).sum(), 1e-6, 12)[0] < ISO


def test_fd64_embedding():
    table = lcg64((8, 4), 10)
    ids = np.array([1, 3, 1])
    dw = O.embedding_backward(ids, np.ones((3, 4)), 8, f64=True)
    assert fd_max(table, dw, lambda tp: O.embedding(ids, tp, f64=True).sum(), 1e-6, 12)[0] < ISO


def test_fd64_swiglu():
    x, w1, w3, w2 = lcg64((2, 4), 11), lcg64((4, 6), 12), lcg64((4, 6), 13), lcg64((6, 4), 14)
    dx, d1, d3, d2 = O.swiglu_backward(x, w1, w3, w2, np.ones((2, 4)), f64=True)
    assert fd_max(w1, d1, lambda wp: O.swiglu(x, wp, w3, w2, f64=True).sum(), 1e-6, 12)[0] < ISO
    assert fd_max(w2, d2, lambda wp: O.swiglu(x, w1, w3, wp, f64=True).sum(), 1e-6, 12)[0] < ISO
    assert fd_max(x, dx, lambda xp: O.swiglu(xp, w1, w3, w2, f64=True).sum(), 1e-6, 8)[0] < ISO


def test_fd64_gqa_rope_window():
    x = lcg64((1, 6, 8), 15)
    wq, wk, wv, wo = lcg64((8, 8), 16), lcg64((8, 4), 17), lcg64((8, 4), 18), lcg64((8, 8), 19)
    y = O.gqa(x, wq, wk, wv, wo, 2, 1, 10000.0, 4, f64=True)
    coeff = np.array([0.25 + (i % 7) * 0.1 for i in range(y.size)]).reshape(y.shape)
    dx, dwq, dwk, dwv, dwo = O.gqa_backward(x, wq, wk, wv, wo, coeff, 2, 1, 10000.0, 4, f64=True)
    f = lambda **kw: (O.gqa(kw.get("x", x), kw.get("wq", wq), kw.get("wk", wk), kw.get("wv", wv), kw.get("wo", wo),
                            2, 1, 10000.0, 4, f64=True) * coeff).sum()
    assert fd_max(wq, dwq, lambda p: f(wq=p), 1e-6, 16)[0] < ISO
    assert fd_max(wk, dwk, lambda p: f(wk=p), 1e-6, 16)[0] < ISO
    assert fd_max(x, dx, lambda p: f(x=p), 1e-6, 16)[0] < ISO


def test_fd64_attention_causal_and_full():
    x = lcg64((1, 4, 8), 8)
    ws = [lcg64((8, 8), s) for s in (9, 10, 11, 12)]
    for causal in (False, True):
        coeff = lcg64((1, 4, 8), 21)
        dx, dwq, dwk, dwv, dwo = O.attention_backward(x, *ws, coeff, 2, causal=causal, f64=True)
        f = lambda xx, wq: (O.attention(xx, wq, ws[1], ws[2], ws[3], 2, causal=causal, f64=True) * coeff).sum()
        assert fd_max(ws[0], dwq, lambda p: f(x, p), 1e-6, 16)[0] < ISO
        assert fd_max(x, dx, lambda p: f(p, ws[0]), 1e-6, 16)[0] < ISO


def test_fd64_moe_gate_and_expert():
    """fd64.rs:806-847 with the router indices held fixed: probes are small
    enough (1e-6) that no top-k decision flips on these LCG inputs."""
    x, gate = lcg64((3, 4), 20), lcg64((4, 3), 21)
    w1s = np.stack([lcg64((4, 6), s) for s in (22, 25, 28)])
    w3s = np.stack([lcg64((4, 6), s) for s in (23, 26, 29)])
    w2s = np.stack([lcg64((6, 4), s) for s in (24, 27, 30)])
    dy = np.ones((3, 4))
    dx, dg, d1, d3, d2 = O.moe_backward(x, gate, w1s, w3s, w2s, dy, 2, f64=True)
    assert fd_max(gate, dg, lambda gp: O.moe(x, gp, w1s, w3s, w2s, 2, f64=True).sum(), 1e-6, 12)[0] < ISO
    assert fd_max(w1s, d1, lambda wp: O.moe(x, gate, wp, w3s, w2s, 2, f64=True).sum(), 1e-6, 12)[0] < ISO
    assert fd_max(x, dx, lambda xp: O.moe(xp, gate, w1s, w3s, w2s, 2, f64=True).sum(), 1e-6, 12)[0] < ISO


def test_fd64_tiny_mixtral_e2e():
    """fd64.rs:857 — tiny Mixtral, seed 3, tokens 1..8: loss gradient groups."""
    cfg = O.MixCfg.tiny()
    P = O.mixtral_seeded(cfg, 3).astype(np.float64)
    tokens = np.arange(1, 9)
    loss, G = O.mixtral_step(cfg, P, tokens, 2, 4, f64=True)
    L = cfg.layout()
    f = lambda Pp: O.mixtral_step(cfg, Pp, tokens, 2, 4, f64=True)[0]
    groups = {"embed": (L["embed"], 32 * 32), "lm_head": (L["lm_head"], 32 * 32),
              "wq0": (L["layer0"] + L["wq"], 32 * 32), "gate0": (L["layer0"] + L["gate"], 32 * 4),
              "w1_0": (L["layer0"] + L["w1"], 32 * 64), "final_norm": (L["final_norm"], 32)}
    for name, (off, n) in groups.items():
        sl = slice(off, off + n)

        def fg(sub, off=off, n=n):
            Q = P.copy()
            Q[off:off + n] = sub
            return f(Q)
        rel, ab = fd_max(P[sl].copy(), G[sl], fg, 1e-6, 8)
        assert rel < 2e-5 and ab < 5e-3, (name, rel, ab)


def test_fd32_reference_tolerances():
    """adjoint.rs:984-1088 — the f32 FD checks at the reference's tolerances."""
    x, w = O.lcg(6, 1).reshape(2, 3), O.lcg(6, 2).reshape(3, 2)
    _, dw, _ = O.linear_backward(x, w, np.ones((2, 2), np.float32))
    assert fd_max(w.astype(np.float32), dw, lambda p: float(O.linear(x, p).sum()), 1e-3, 4)[0] < 0.05
    x = O.lcg(8, 3).reshape(2, 4)
    wr = np.ones(4, np.float32)
    _, dwr = O.rmsnorm_backward(x, wr, np.ones((2, 4), np.float32))
    assert fd_max(wr, dwr, lambda p: float(O.rmsnorm(x, p).sum()), 1e-3, 4)[0] < 0.08
