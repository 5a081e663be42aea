"""ORACLE — test infrastructure only.

ctypes front-end to ``liboracle_catnn.so``, the C++ restatement of the
reference's CPU kernels (crates/catnn-compile/src/kernel/{cpu,moe,adjoint}.rs,
crates/catnn-core/src/lens/{optim,moe}.rs, crates/catnn-compile/src/train.rs).
Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` import this module, and only to check or time the reference
algorithm — never as a product code path.

Every function takes numpy arrays (float32 for the oracle proper, float64
for the ``f64=True`` shadow) and returns new arrays. The library is built by
``oracle/Makefile`` (``build()`` in ``__graft_entry__`` runs it).
"""
import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle_catnn.so")
_lib = None

I64 = C.c_int64
PF = C.POINTER(C.c_float)
PD = C.POINTER(C.c_double)
PU32 = C.POINTER(C.c_uint32)
PI64 = C.POINTER(C.c_int64)
VP = C.c_void_p


def build(force=False):
    """Compile the oracle with its Makefile (g++, -ffp-contract=off)."""
    if force or not os.path.exists(_LIB_PATH):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(_LIB_PATH)
        _lib.orc_checksum.restype = C.c_uint64
        _lib.orc_mse_loss.restype = C.c_float
        _lib.orc64_mse_loss.restype = C.c_double
        _lib.orc_adam_put.restype = C.c_uint64
        _lib.orc_powi.restype = C.c_float
        _lib.orc_powi.argtypes = [C.c_float, C.c_int]
        _lib.orc_mixtral_param_count.restype = I64
    return _lib


def _p(a):
    """Pointer to a contiguous numpy array (or NULL for None)."""
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle needs contiguous arrays"
    return a.ctypes.data_as(VP)


def _ft(f64):
    return np.float64 if f64 else np.float32


def _fn(name, f64):
    return getattr(lib(), ("orc64_" if f64 else "orc_") + name)


def _arr(x, f64=False):
    return np.ascontiguousarray(x, dtype=_ft(f64))


def _scalar(v, f64):
    return C.c_double(v) if f64 else C.c_float(v)


# ----------------------------------------------------------------- tensor.rs
def lcg(n, seed):
    out = np.empty(int(n), np.float32)
    lib().orc_lcg(_p(out), I64(n), C.c_uint64(seed))
    return out


def checksum(x):
    x = _arr(x)
    return int(lib().orc_checksum(_p(x), I64(x.size)))


# ----------------------------------------------------------------- cpu.rs
def matmul_seq(a, b):
    a, b = _arr(a), _arr(b)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), np.float32)
    lib().orc_matmul_seq(_p(a), _p(b), _p(c), I64(m), I64(k), I64(n))
    return c


def linear(x, w, b=None, parallel=True, f64=False):
    """cpu::linear (parallel=True, 8-lane order) or cpu::linear_seq."""
    x, w = _arr(x, f64), _arr(w, f64)
    b = None if b is None else _arr(b, f64)
    k = x.shape[-1]
    m = x.size // k
    n = w.shape[1]
    y = np.empty(x.shape[:-1] + (n,), _ft(f64))
    _fn("linear", f64)(_p(x), _p(w), _p(b), _p(y), I64(m), I64(k), I64(n), C.c_int(1 if parallel else 0))
    return y


def ref_linear(x, w, b=None):
    x, w = _arr(x), _arr(w)
    b = None if b is None else _arr(b)
    k = x.shape[-1]
    m = x.size // k
    n = w.shape[1]
    y = np.empty(x.shape[:-1] + (n,), np.float32)
    lib().orc_ref_linear(_p(x), _p(w), _p(b), _p(y), I64(m), I64(k), I64(n))
    return y


def _unary(name, x, f64=False):
    x = _arr(x, f64)
    y = np.empty_like(x)
    _fn(name, f64)(_p(x), _p(y), I64(x.size))
    return y


def relu(x, f64=False):
    return _unary("relu", x, f64)


def gelu(x, f64=False):
    return _unary("gelu", x, f64)


def softmax_last(x, f64=False):
    x = _arr(x, f64)
    y = np.empty_like(x)
    last = x.shape[-1]
    _fn("softmax_last", f64)(_p(x), _p(y), I64(x.size // last), I64(last))
    return y


def layer_norm(x, gamma, beta, eps=1e-5, f64=False):
    x, g, b = _arr(x, f64), _arr(gamma, f64), _arr(beta, f64)
    y = np.empty_like(x)
    last = x.shape[-1]
    _fn("layer_norm", f64)(_p(x), _p(g), _p(b), _p(y), I64(x.size // last), I64(last), _scalar(eps, f64))
    return y


def add(a, b):
    a, b = _arr(a), _arr(b)
    y = np.empty_like(a)
    if a.size == b.size:
        lib().orc_add(_p(a), _p(b), _p(y), I64(a.size))
    else:
        last = a.shape[-1]
        lib().orc_add_bias(_p(a), _p(b), _p(y), I64(a.size // last), I64(last))
    return y


def mul(a, b):
    a, b = _arr(a), _arr(b)
    y = np.empty_like(a)
    lib().orc_mul(_p(a), _p(b), _p(y), I64(a.size))
    return y


def attention(x, wq, wk, wv, wo, n_heads, causal=False, f64=False):
    x = _arr(x, f64)
    ws = [_arr(w, f64) for w in (wq, wk, wv, wo)]
    b, s, d = x.shape
    y = np.empty_like(x)
    _fn("attention", f64)(_p(x), *[_p(w) for w in ws], _p(y), I64(b), I64(s), I64(d),
                          I64(n_heads), I64(d // n_heads), C.c_int(1 if causal else 0))
    return y


# ----------------------------------------------------------------- moe.rs
def rmsnorm(x, w, eps=1e-5, f64=False):
    x, w = _arr(x, f64), _arr(w, f64)
    y = np.empty_like(x)
    last = x.shape[-1]
    _fn("rmsnorm", f64)(_p(x), _p(w), _p(y), I64(x.size // last), I64(last), _scalar(eps, f64))
    return y


def embedding(ids, table, f64=False):
    ids = np.ascontiguousarray(ids, np.uint32)
    t = _arr(table, f64)
    v, h = t.shape
    y = np.empty(ids.shape + (h,), _ft(f64))
    rc = _fn("embedding", f64)(_p(ids), I64(ids.size), _p(t), I64(v), I64(h), _p(y))
    if rc != 0:
        raise ValueError("shape mismatch: token id >= vocab")
    return y


def rope(q, theta):
    """Rotate q [B,S,heads,hd] in place copy; negative theta = adjoint."""
    q = _arr(q).copy()
    b, s, hh, hd = q.shape
    lib().orc_rope(_p(q), I64(b), I64(s), I64(hh), I64(hd), C.c_double(theta))
    return q


def gqa(x, wq, wk, wv, wo, n_heads, n_kv, theta, window=None, f64=False):
    x = _arr(x, f64)
    ws = [_arr(w, f64) for w in (wq, wk, wv, wo)]
    b, s, d = x.shape
    hd = wq.shape[1] // n_heads
    y = np.empty_like(x)
    _fn("gqa", f64)(_p(x), *[_p(w) for w in ws], _p(y), I64(b), I64(s), I64(d), I64(n_heads),
                    I64(n_kv), I64(hd), C.c_double(theta), I64(window or 0))
    return y


def gqa_core(q, k, v, window=None):
    """Attention core on rotated q [B,S,H,hd], k/v [B,S,Hkv,hd] -> ctx [B,S,H*hd]."""
    q, k, v = _arr(q), _arr(k), _arr(v)
    b, s, h, hd = q.shape
    kv = k.shape[2]
    ctx = np.empty((b, s, h * hd), np.float32)
    lib().orc_gqa_core(_p(q), _p(k), _p(v), _p(ctx), I64(b), I64(s), I64(h), I64(kv), I64(hd), I64(window or 0))
    return ctx


def swiglu(x, w1, w3, w2, f64=False):
    x, w1, w3, w2 = (_arr(a, f64) for a in (x, w1, w3, w2))
    h = x.shape[-1]
    t = x.size // h
    m = w1.shape[1]
    y = np.empty_like(x)
    _fn("swiglu", f64)(_p(x), _p(w1), _p(w3), _p(w2), _p(y), I64(t), I64(h), I64(m))
    return y


def topk_softmax(logits, k):
    logits = _arr(logits)
    n = logits.shape[-1]
    kk = min(k, n)
    idx = np.empty(kk, np.int64)
    w = np.empty(kk, np.float32)
    lib().orc_topk_softmax(_p(logits), I64(n), I64(k), _p(idx), _p(w))
    return idx, w


def route(x, gate, k):
    x, gate = _arr(x), _arr(gate)
    h = x.shape[-1]
    t = x.size // h
    e = gate.shape[1]
    idx = np.empty((t, k), np.int64)
    w = np.empty((t, k), np.float32)
    logits = np.empty((t, e), np.float32)
    lib().orc_route(_p(x), _p(gate), I64(t), I64(h), I64(e), I64(k), _p(idx), _p(w), _p(logits))
    return idx, w, logits


def moe(x, gate, w1s, w3s, w2s, k, f64=False):
    x, gate, w1s, w3s, w2s = (_arr(a, f64) for a in (x, gate, w1s, w3s, w2s))
    h = x.shape[-1]
    t = x.size // h
    e, _, m = w1s.shape
    y = np.empty_like(x)
    _fn("moe", f64)(_p(x), _p(gate), _p(w1s), _p(w3s), _p(w2s), _p(y), I64(t), I64(h), I64(m), I64(e), I64(k))
    return y


def lm_head(x, w):
    x, w = _arr(x), _arr(w)
    v, h = w.shape
    rows = x.size // h
    y = np.empty(x.shape[:-1] + (v,), np.float32)
    lib().orc_lm_head(_p(x), _p(w), _p(y), I64(rows), I64(h), I64(v))
    return y


# ----------------------------------------------------------------- adjoint.rs
def linear_backward(x, w, dy, f64=False):
    x, w, dy = _arr(x, f64), _arr(w, f64), _arr(dy, f64)
    k = x.shape[-1]
    m = x.size // k
    n = w.shape[1]
    dx, dw, db = np.empty_like(x), np.empty_like(w), np.empty(n, _ft(f64))
    _fn("linear_backward", f64)(_p(x), _p(w), _p(dy), _p(dx), _p(dw), _p(db), I64(m), I64(k), I64(n))
    return dx, dw, db


def relu_backward(x, dy, f64=False):
    x, dy = _arr(x, f64), _arr(dy, f64)
    dx = np.empty_like(x)
    _fn("relu_backward", f64)(_p(x), _p(dy), _p(dx), I64(x.size))
    return dx


def gelu_backward(x, dy, f64=False):
    x, dy = _arr(x, f64), _arr(dy, f64)
    dx = np.empty_like(x)
    _fn("gelu_backward", f64)(_p(x), _p(dy), _p(dx), I64(x.size))
    return dx


def softmax_backward(y, dy, f64=False):
    y, dy = _arr(y, f64), _arr(dy, f64)
    dx = np.empty_like(y)
    last = y.shape[-1]
    _fn("softmax_backward", f64)(_p(y), _p(dy), _p(dx), I64(y.size // last), I64(last))
    return dx


def mse_loss(pred, target, f64=False):
    p, t = _arr(pred, f64), _arr(target, f64)
    d = np.empty_like(p)
    loss = _fn("mse_loss", f64)(_p(p), _p(t), _p(d), I64(p.size))
    return float(loss), d


def cross_entropy(logits, targets, f64=False):
    z = _arr(logits, f64)
    tg = np.ascontiguousarray(targets, np.uint32)
    last = z.shape[-1]
    d = np.empty_like(z)
    loss = (C.c_double if f64 else C.c_float)()
    rc = _fn("cross_entropy", f64)(_p(z), _p(tg), _p(d), I64(z.size // last), I64(last), C.byref(loss))
    if rc != 0:
        raise ValueError("shape mismatch: target >= classes")
    return float(loss.value), d


def rmsnorm_backward(x, w, dy, eps=1e-5, f64=False):
    x, w, dy = _arr(x, f64), _arr(w, f64), _arr(dy, f64)
    dx, dw = np.empty_like(x), np.empty_like(w)
    last = x.shape[-1]
    _fn("rmsnorm_backward", f64)(_p(x), _p(w), _p(dy), _p(dx), _p(dw), I64(x.size // last), I64(last), _scalar(eps, f64))
    return dx, dw


def embedding_backward(ids, dy, vocab, f64=False):
    ids = np.ascontiguousarray(ids, np.uint32)
    dy = _arr(dy, f64)
    h = dy.shape[-1]
    dw = np.empty((vocab, h), _ft(f64))
    _fn("embedding_backward", f64)(_p(ids), I64(ids.size), _p(dy), _p(dw), I64(vocab), I64(h))
    return dw


def swiglu_backward(x, w1, w3, w2, dy, f64=False):
    x, w1, w3, w2, dy = (_arr(a, f64) for a in (x, w1, w3, w2, dy))
    h = x.shape[-1]
    t = x.size // h
    m = w1.shape[1]
    dx, d1, d3, d2 = np.empty_like(x), np.empty_like(w1), np.empty_like(w3), np.empty_like(w2)
    _fn("swiglu_backward", f64)(_p(x), _p(w1), _p(w3), _p(w2), _p(dy), _p(dx), _p(d1), _p(d3), _p(d2), I64(t), I64(h), I64(m))
    return dx, d1, d3, d2


def router_backward_ste(x, gate, d_weights, k):
    x, gate, dw = _arr(x), _arr(gate), _arr(d_weights)
    h = x.shape[-1]
    t = x.size // h
    e = gate.shape[1]
    dx, dg = np.empty_like(x), np.empty_like(gate)
    lib().orc_router_backward_ste(_p(x), _p(gate), _p(dw), _p(dx), _p(dg), I64(t), I64(h), I64(e), I64(k))
    return dx, dg


def moe_backward(x, gate, w1s, w3s, w2s, dy, k, f64=False):
    x, gate, w1s, w3s, w2s, dy = (_arr(a, f64) for a in (x, gate, w1s, w3s, w2s, dy))
    h = x.shape[-1]
    t = x.size // h
    e, _, m = w1s.shape
    dx, dg = np.empty_like(x), np.empty_like(gate)
    d1, d3, d2 = np.empty_like(w1s), np.empty_like(w3s), np.empty_like(w2s)
    _fn("moe_backward", f64)(_p(x), _p(gate), _p(w1s), _p(w3s), _p(w2s), _p(dy), _p(dx), _p(dg), _p(d1), _p(d3), _p(d2),
                             I64(t), I64(h), I64(m), I64(e), I64(k))
    return dx, dg, d1, d3, d2


def layer_norm_backward(x, gamma, dy, eps=1e-5, f64=False):
    x, g, dy = _arr(x, f64), _arr(gamma, f64), _arr(dy, f64)
    last = x.shape[-1]
    dx, dg, db = np.empty_like(x), np.empty_like(g), np.empty_like(g)
    _fn("layer_norm_backward", f64)(_p(x), _p(g), _p(dy), _p(dx), _p(dg), _p(db), I64(x.size // last), I64(last), _scalar(eps, f64))
    return dx, dg, db


def gqa_backward(x, wq, wk, wv, wo, dy, n_heads, n_kv, theta, window=None, f64=False):
    x, wq, wk, wv, wo, dy = (_arr(a, f64) for a in (x, wq, wk, wv, wo, dy))
    b, s, d = x.shape
    hd = wq.shape[1] // n_heads
    outs = [np.empty_like(a) for a in (x, wq, wk, wv, wo)]
    _fn("gqa_backward", f64)(_p(x), _p(wq), _p(wk), _p(wv), _p(wo), _p(dy), *[_p(o) for o in outs], I64(b), I64(s), I64(d),
                             I64(n_heads), I64(n_kv), I64(hd), C.c_double(theta), I64(window or 0))
    return tuple(outs)


def attention_backward(x, wq, wk, wv, wo, dy, n_heads, causal=False, f64=False):
    x, wq, wk, wv, wo, dy = (_arr(a, f64) for a in (x, wq, wk, wv, wo, dy))
    b, s, d = x.shape
    outs = [np.empty_like(a) for a in (x, wq, wk, wv, wo)]
    _fn("attention_backward", f64)(_p(x), _p(wq), _p(wk), _p(wv), _p(wo), _p(dy), *[_p(o) for o in outs], I64(b), I64(s),
                                   I64(d), I64(n_heads), I64(d // n_heads), C.c_int(1 if causal else 0))
    return tuple(outs)


def lm_head_backward(x, w, dy):
    x, w, dy = _arr(x), _arr(w), _arr(dy)
    v, h = w.shape
    dx, dw = np.empty_like(x), np.empty_like(w)
    lib().orc_lm_head_backward(_p(x), _p(w), _p(dy), _p(dx), _p(dw), I64(x.size // h), I64(h), I64(v))
    return dx, dw


# ----------------------------------------------------------------- optim.rs
def sgd_put(p, g, lr):
    p, g = _arr(p), _arr(g)
    out = np.empty_like(p)
    lib().orc_sgd_put(_p(p), _p(g), _p(out), I64(p.size), C.c_float(lr))
    return out


def adam_put(p, g, m, v, t_prev, lr, b1=0.9, b2=0.999, eps=1e-8):
    """Returns (p_new, m_new, v_new, t)."""
    p, g, m, v = _arr(p).copy(), _arr(g), _arr(m).copy(), _arr(v).copy()
    t = lib().orc_adam_put(_p(p), _p(g), _p(m), _p(v), I64(p.size), C.c_uint64(t_prev), C.c_float(lr),
                           C.c_float(b1), C.c_float(b2), C.c_float(eps))
    return p, m, v, int(t)


def powi(a, b):
    return float(lib().orc_powi(a, b))


# ----------------------------------------------------------------- train.rs
class MixCfg:
    """Mixtral-style shapes (crates/catnn-core/src/spec/mixtral.rs fields)."""

    def __init__(self, vocab, hidden, mid, layers, heads, kv_heads, experts, top_k, eps=1e-5, theta=1e4, window=None):
        self.vocab, self.hidden, self.mid, self.layers = vocab, hidden, mid, layers
        self.heads, self.kv_heads, self.experts, self.top_k = heads, kv_heads, experts, top_k
        self.eps, self.theta, self.window = eps, theta, window

    @classmethod
    def tiny(cls):
        """MixtralConfig::tiny() (mixtral.rs:107-130)."""
        return cls(32, 32, 64, 2, 4, 2, 4, 2, 1e-5, 10000.0, 8)

    def arr(self):
        return np.array([self.vocab, self.hidden, self.mid, self.layers, self.heads, self.kv_heads,
                         self.experts, self.top_k, self.window or 0], np.int64)

    def layout(self):
        out = np.empty(16, np.int64)
        a = self.arr()
        lib().orc_mixtral_layout(_p(a), _p(out))
        keys = ["embed", "final_norm", "lm_head", "total", "layer0", "layer_stride", "rms_attn", "wq", "wk", "wv",
                "wo", "rms_moe", "gate", "w1", "w3", "w2"]
        return dict(zip(keys, (int(v) for v in out)))


def mixtral_seeded(cfg, seed):
    a = cfg.arr()
    n = int(lib().orc_mixtral_param_count(_p(a)))
    P = np.empty(n, np.float32)
    lib().orc_mixtral_seeded(_p(a), C.c_uint64(seed), _p(P))
    return P


def mixtral_forward(cfg, P, tokens, batch, seq):
    a, P = cfg.arr(), _arr(P)
    tok = np.ascontiguousarray(tokens, np.uint32)
    logits = np.empty((batch * seq, cfg.vocab), np.float32)
    rc = lib().orc_mixtral_forward(_p(a), C.c_float(cfg.eps), C.c_double(cfg.theta), _p(P), _p(tok), I64(batch), I64(seq), _p(logits))
    if rc:
        raise ValueError("shape mismatch in mixtral forward")
    return logits


def mixtral_step(cfg, P, tokens, batch, seq, f64=False, out=None):
    """train.rs:261 mixtral_step -> (loss, packed grads). `out` (optional, same
    shape and dtype as P) receives the gradients instead of a new array."""
    a, P = cfg.arr(), _arr(P, f64)
    tok = np.ascontiguousarray(tokens, np.uint32)
    G = np.empty_like(P) if out is None else out
    assert G.shape == P.shape and G.dtype == P.dtype and G.flags["C_CONTIGUOUS"]
    loss = (C.c_double if f64 else C.c_float)()
    rc = _fn("mixtral_step", f64)(_p(a), C.c_float(cfg.eps), C.c_double(cfg.theta), _p(P), _p(tok), I64(batch), I64(seq),
                                  C.byref(loss), _p(G))
    if rc:
        raise ValueError("shape mismatch in mixtral step")
    return float(loss.value), G


def mixtral_step_frozen(cfg, P, tokens, batch, seq, forced):
    """mixtral_step with every layer's routing held fixed to `forced`
    ([layers, batch*seq, top_k] expert indices) — fd64.rs's frozen-index
    methodology for comparing across the discontinuous top-k."""
    a, P = cfg.arr(), _arr(P)
    tok = np.ascontiguousarray(tokens, np.uint32)
    fz = np.ascontiguousarray(forced, np.int64)
    assert fz.shape == (cfg.layers, batch * seq, cfg.top_k), fz.shape
    G = np.empty_like(P)
    loss = C.c_float()
    rc = lib().orc_mixtral_step_frozen(_p(a), C.c_float(cfg.eps), C.c_double(cfg.theta), _p(P), _p(tok), I64(batch),
                                       I64(seq), _p(fz), C.byref(loss), _p(G))
    if rc:
        raise ValueError("shape mismatch in mixtral step")
    return float(loss.value), G


def mlp_step(w1, b1, w2, b2, x, labels=None, y_mse=None):
    """train.rs:71 mlp_step; CE on labels when given, else MSE on y_mse."""
    w1, b1, w2, b2, x = (_arr(a) for a in (w1, b1, w2, b2, x))
    batch, din = x.shape
    hid, dout = w1.shape[1], w2.shape[1]
    ce = labels is not None
    lab = np.ascontiguousarray(labels if ce else np.zeros(batch), np.uint32)
    ym = _arr(y_mse) if not ce else None
    loss = C.c_float()
    dw1, db1, dw2, db2 = np.empty_like(w1), np.empty_like(b1), np.empty_like(w2), np.empty_like(b2)
    rc = lib().orc_mlp_step(_p(w1), _p(b1), _p(w2), _p(b2), _p(x), _p(ym), _p(lab), C.c_int(1 if ce else 0), I64(batch),
                            I64(din), I64(hid), I64(dout), C.byref(loss), _p(dw1), _p(db1), _p(dw2), _p(db2))
    if rc:
        raise ValueError("shape mismatch in mlp step")
    return float(loss.value), dw1, db1, dw2, db2


BLOCK_KEYS = ["g1", "be1", "wq", "wk", "wv", "wo", "g2", "be2", "f1", "c1", "f2", "c2"]


def block_fwd_bwd(W, x, dy, n_heads, eps=1e-5, f64=False):
    """Causal pre-LN transformer block fwd (+bwd when dy is given).

    W: dict of BLOCK_KEYS arrays. Returns (y, dx, grads dict). f64=True runs
    the same loop nests in double precision (the exact reference of the
    parity tests' fallback)."""
    x = _arr(x, f64)
    b, s, d = x.shape
    ff = W["f1"].shape[1]
    Wc = [_arr(W[k], f64) for k in BLOCK_KEYS]
    Gs = [np.empty_like(w) for w in Wc]
    Wp = (VP * 12)(*[w.ctypes.data for w in Wc])
    Gp = (VP * 12)(*[g.ctypes.data for g in Gs])
    y = np.empty_like(x)
    dx = np.empty_like(x)
    dyc = _arr(dy, f64) if dy is not None else None
    _fn("block_fwd_bwd", f64)(Wp, Gp, _p(x), _p(dyc), _p(y), _p(dx), I64(b), I64(s), I64(d), I64(n_heads), I64(ff),
                              _scalar(eps, f64))
    return y, (dx if dy is not None else None), dict(zip(BLOCK_KEYS, Gs))
