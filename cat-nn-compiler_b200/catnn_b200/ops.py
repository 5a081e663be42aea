"""Functional operators over device tensors, one per C-ABI entry point.

PyTorch is used only as the device allocator and stream source: every
computation below is a kernel of libcatnn_b200 launched on the current
torch stream of the tensor's device. Inputs must be contiguous CUDA
tensors; float32 selects the fp32 parity path and bfloat16 the
tensor-core path (norm weights, losses, router weights and optimizer state
stay float32).
"""
import ctypes as C

import torch

from . import _lib
from .errors import DTypeMismatch, InvalidArgument, ShapeMismatch

F32, BF16, TF32 = 0, 1, 2
ACT = {"none": 0, None: 0, "relu": 1, "gelu": 2}


class Context:
    """One libcatnn_b200 context per device (catnn_ctx_create)."""

    def __init__(self, device):
        self.device = device
        h = C.c_void_p()
        _lib.call("catnn_ctx_create", int(device), C.byref(h))
        self.handle = h

    def bind(self):
        s = torch.cuda.current_stream(self.device).cuda_stream
        _lib.call("catnn_ctx_set_stream", self.handle, C.c_void_p(s))
        return self.handle

    def launch_count(self):
        v = C.c_uint64()
        _lib.call("catnn_ctx_launch_count", self.handle, C.byref(v))
        return int(v.value)

    def synchronize(self):
        _lib.call("catnn_ctx_synchronize", self.handle)


_CTX = {}


def context(device=None):
    if device is None:
        device = torch.cuda.current_device()
    if isinstance(device, torch.device):
        device = device.index if device.index is not None else torch.cuda.current_device()
    if device not in _CTX:
        _CTX[device] = Context(device)
    return _CTX[device]


def _h(t):
    return context(t.device).bind()


def _p(t):
    if t is None:
        return None
    if not t.is_cuda:
        raise InvalidArgument("catnn_b200 operators take CUDA tensors")
    if not t.is_contiguous():
        raise InvalidArgument("catnn_b200 operators take contiguous tensors")
    return C.c_void_p(t.data_ptr())


def _dt(t):
    if t.dtype == torch.float32:
        return F32
    if t.dtype == torch.bfloat16:
        return BF16
    raise DTypeMismatch(f"unsupported dtype {t.dtype}")


def _same(*ts):
    d = ts[0].dtype
    for t in ts[1:]:
        if t is not None and t.dtype != d:
            raise DTypeMismatch(f"{d} vs {t.dtype}")


def _f32(t, what):
    if t is not None and t.dtype != torch.float32:
        raise DTypeMismatch(f"{what} must be float32")


# ------------------------------------------------------------------ dense
def gemm(a, b, trans_a=False, trans_b=False, out=None, out_dtype=None, bias=None, act="none", accumulate=False,
         tf32=False):
    """C = act(op(a)·op(b) + bias) (+C). tf32=True multiplies fp32 a, b on
    the tensor cores as TF32 (fp32 accumulation) instead of the fp32 path."""
    _same(a, b)
    if tf32 and a.dtype != torch.float32:
        raise DTypeMismatch("tf32 gemm takes fp32 operands")
    M, K = (a.shape[1], a.shape[0]) if trans_a else (a.shape[0], a.shape[1])
    Kb, N = (b.shape[1], b.shape[0]) if trans_b else (b.shape[0], b.shape[1])
    if K != Kb:
        raise ShapeMismatch(f"gemm K {K} vs {Kb}")
    if out is None:
        out = torch.empty(M, N, dtype=out_dtype or a.dtype, device=a.device)
    _f32(bias, "bias")
    _lib.call("catnn_gemm", _h(a), int(trans_a), int(trans_b), M, N, K, _p(a), a.shape[1], _p(b), b.shape[1], _p(out),
              N, TF32 if tf32 else _dt(a), _dt(out), _p(bias), ACT[act], int(accumulate))
    return out


def linear(x, w, b=None, act="none"):
    """cpu::linear (cpu.rs:135): y = act(x @ w + b), w [in, out]."""
    _same(x, w)
    _f32(b, "bias")
    k = x.shape[-1]
    if w.dim() != 2 or w.shape[0] != k:
        raise ShapeMismatch(f"linear K {k} vs {tuple(w.shape)}")
    n = w.shape[1]
    m = x.numel() // max(k, 1)
    y = torch.empty(*x.shape[:-1], n, dtype=x.dtype, device=x.device)
    _lib.call("catnn_linear_fwd", _h(x), _p(x), _p(w), _p(b), _p(y), m, k, n, ACT[act], _dt(x))
    return y


def linear_backward(x, w, dy, need_dx=True, need_dw=True, need_db=True):
    """adjoint::linear_backward (adjoint.rs:35) -> (dx, dw, db)."""
    _same(x, w, dy)
    k, n = w.shape
    m = x.numel() // k
    dx = torch.empty_like(x) if need_dx else None
    dw = torch.empty_like(w) if need_dw else None
    db = torch.empty(n, dtype=torch.float32, device=x.device) if need_db else None
    _lib.call("catnn_linear_bwd", _h(x), _p(x), _p(w), _p(dy), _p(dx), _p(dw), _p(db), m, k, n, _dt(x))
    return dx, dw, db


def lm_head(x, w):
    """moe::lm_head (moe.rs:325): x @ w.T, w [vocab, hidden]."""
    _same(x, w)
    v, h = w.shape
    rows = x.numel() // h
    y = torch.empty(*x.shape[:-1], v, dtype=x.dtype, device=x.device)
    _lib.call("catnn_lm_head_fwd", _h(x), _p(x), _p(w), _p(y), rows, h, v, _dt(x))
    return y


def lm_head_backward(x, w, dy):
    _same(x, w, dy)
    v, h = w.shape
    rows = x.numel() // h
    dx, dw = torch.empty_like(x), torch.empty_like(w)
    _lib.call("catnn_lm_head_bwd", _h(x), _p(x), _p(w), _p(dy), _p(dx), _p(dw), rows, h, v, _dt(x))
    return dx, dw


# ------------------------------------------------------------------ elementwise
def _unary(name, x):
    y = torch.empty_like(x)
    _lib.call(name, _h(x), _p(x), _p(y), x.numel(), _dt(x))
    return y


def relu(x):
    return _unary("catnn_relu_fwd", x)


def gelu(x):
    return _unary("catnn_gelu_fwd", x)


def relu_backward(x, dy):
    _same(x, dy)
    if x.numel() != dy.numel():
        raise ShapeMismatch("relu grad")
    dx = torch.empty_like(x)
    _lib.call("catnn_relu_bwd", _h(x), _p(x), _p(dy), _p(dx), x.numel(), _dt(x))
    return dx


def gelu_backward(x, dy):
    _same(x, dy)
    dx = torch.empty_like(x)
    _lib.call("catnn_gelu_bwd", _h(x), _p(x), _p(dy), _p(dx), x.numel(), _dt(x))
    return dx


def add(a, b):
    """cpu::add (cpu.rs:80): same length, or b broadcast over the last dim."""
    _same(a, b)
    if b.numel() != a.numel():
        last = a.shape[-1] if a.dim() else a.numel()
        if b.numel() != last:
            raise ShapeMismatch(f"add {tuple(a.shape)} vs {tuple(b.shape)}")
    y = torch.empty_like(a)
    _lib.call("catnn_add", _h(a), _p(a), _p(b), _p(y), a.numel(), b.numel(), _dt(a))
    return y


def mul(a, b):
    _same(a, b)
    if a.numel() != b.numel():
        raise ShapeMismatch("mul length")
    y = torch.empty_like(a)
    _lib.call("catnn_mul", _h(a), _p(a), _p(b), _p(y), a.numel(), _dt(a))
    return y


# ------------------------------------------------------------------ softmax / losses
def softmax_last(x):
    y = torch.empty_like(x)
    last = x.shape[-1] if x.dim() else 1
    _lib.call("catnn_softmax_fwd", _h(x), _p(x), _p(y), x.numel() // max(last, 1), last, _dt(x))
    return y


def softmax_backward(y, dy):
    _same(y, dy)
    dx = torch.empty_like(y)
    last = y.shape[-1]
    _lib.call("catnn_softmax_bwd", _h(y), _p(y), _p(dy), _p(dx), y.numel() // last, last, _dt(y))
    return dx


def cross_entropy(logits, targets, check=True):
    """adjoint::cross_entropy (adjoint.rs:123) -> (loss scalar tensor, dlogits)."""
    if targets.dtype != torch.int32 and targets.dtype != torch.uint32:
        targets = targets.to(torch.int32)
    last = logits.shape[-1]
    rows = logits.numel() // last
    if targets.numel() != rows:
        raise ShapeMismatch("ce targets")
    loss = torch.empty((), dtype=torch.float32, device=logits.device)
    d = torch.empty_like(logits)
    _lib.call("catnn_xent_fwdbwd", _h(logits), _p(logits), _p(targets.contiguous()), rows, last, _p(loss), _p(d),
              _dt(logits), int(check))
    return loss, d


def mse_loss(pred, target):
    _f32(pred, "pred")
    _f32(target, "target")
    if pred.numel() != target.numel():
        raise ShapeMismatch("mse")
    loss = torch.empty((), dtype=torch.float32, device=pred.device)
    d = torch.empty_like(pred)
    _lib.call("catnn_mse_fwdbwd", _h(pred), _p(pred), _p(target), pred.numel(), _p(loss), _p(d))
    return loss, d


# ------------------------------------------------------------------ norms
def layer_norm(x, gamma, beta, eps=1e-5):
    last = x.shape[-1]
    if gamma.numel() != last or beta.numel() != last:
        raise ShapeMismatch("ln gamma/beta length")
    _f32(gamma, "gamma")
    _f32(beta, "beta")
    y = torch.empty_like(x)
    _lib.call("catnn_layernorm_fwd", _h(x), _p(x), _p(gamma), _p(beta), _p(y), x.numel() // last, last, eps, _dt(x))
    return y


def layer_norm_backward(x, gamma, dy, eps=1e-5):
    last = x.shape[-1]
    if gamma.numel() != last or dy.numel() != x.numel():
        raise ShapeMismatch("layernorm grad")
    dx = torch.empty_like(x)
    dg = torch.empty(last, dtype=torch.float32, device=x.device)
    db = torch.empty(last, dtype=torch.float32, device=x.device)
    _lib.call("catnn_layernorm_bwd", _h(x), _p(x), _p(gamma), _p(dy), _p(dx), _p(dg), _p(db), x.numel() // last, last,
              eps, _dt(x))
    return dx, dg, db


def rmsnorm(x, w, eps=1e-5):
    last = x.shape[-1]
    if w.numel() != last:
        raise ShapeMismatch("rmsnorm weight")
    _f32(w, "rmsnorm weight")
    y = torch.empty_like(x)
    _lib.call("catnn_rmsnorm_fwd", _h(x), _p(x), _p(w), _p(y), x.numel() // last, last, eps, _dt(x))
    return y


def rmsnorm_backward(x, w, dy, eps=1e-5):
    last = x.shape[-1]
    if w.numel() != last:
        raise ShapeMismatch("rmsnorm w")
    dx = torch.empty_like(x)
    dw = torch.empty(last, dtype=torch.float32, device=x.device)
    _lib.call("catnn_rmsnorm_bwd", _h(x), _p(x), _p(w), _p(dy), _p(dx), _p(dw), x.numel() // last, last, eps, _dt(x))
    return dx, dw


# ------------------------------------------------------------------ embedding
def _ids(ids):
    if ids.dtype not in (torch.int32, torch.uint32):
        ids = ids.to(torch.int32)
    return ids.contiguous()


def embedding(ids, table):
    """moe::embedding (moe.rs:34): raises ShapeMismatch on id >= vocab."""
    ids = _ids(ids)
    v, h = table.shape
    y = torch.empty(*ids.shape, h, dtype=table.dtype, device=table.device)
    _lib.call("catnn_embedding_fwd", _h(table), _p(ids), ids.numel(), _p(table), v, h, _p(y), _dt(table))
    return y


def embedding_backward(ids, dy, vocab):
    """adjoint::embedding_backward (adjoint.rs:195): fp32 [vocab, hidden]."""
    ids = _ids(ids)
    h = dy.shape[-1]
    dw = torch.empty(vocab, h, dtype=torch.float32, device=dy.device)
    _lib.call("catnn_embedding_bwd", _h(dy), _p(ids), ids.numel(), _p(dy), _p(dw), vocab, h, _dt(dy))
    return dw


# ------------------------------------------------------------------ attention
def rope(x, theta, inverse=False):
    """In-place RoPE on x [B,S,heads,hd] (moe.rs:47; inverse = adjoint.rs:454)."""
    b, s, hh, hd = x.shape
    _lib.call("catnn_rope", _h(x), _p(x), b, s, hh, hd, float(theta), int(inverse), _dt(x))
    return x


def attention_core(q, k, v, causal=True, window=None):
    """q [B,S,H,hd], k/v [B,S,Hkv,hd] -> (o [B,S,H*hd], lse [B,H,S])."""
    _same(q, k, v)
    b, s, h, hd = q.shape
    hkv = k.shape[2]
    o = torch.empty(b, s, h * hd, dtype=q.dtype, device=q.device)
    lse = torch.empty(b, h, s, dtype=torch.float32, device=q.device)
    _lib.call("catnn_attention_fwd", _h(q), _p(q), _p(k), _p(v), _p(o), _p(lse), b, s, h, hkv, hd, int(causal),
              int(window or 0), _dt(q))
    return o, lse


def attention_core_backward(q, k, v, o, lse, dout, causal=True, window=None):
    b, s, h, hd = q.shape
    hkv = k.shape[2]
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    _lib.call("catnn_attention_bwd", _h(q), _p(q), _p(k), _p(v), _p(o), _p(lse), _p(dout), _p(dq), _p(dk), _p(dv), b, s,
              h, hkv, hd, int(causal), int(window or 0), _dt(q))
    return dq, dk, dv


def attention(x, wq, wk, wv, wo, n_heads, causal=False):
    """cpu::attention (cpu.rs:235); causal=True adds the j <= i mask."""
    _same(x, wq, wk, wv, wo)
    b, s, d = x.shape
    if d % n_heads:
        raise ShapeMismatch("attention head split")
    y = torch.empty_like(x)
    _lib.call("catnn_mha_fwd", _h(x), _p(x), _p(wq), _p(wk), _p(wv), _p(wo), _p(y), b, s, d, n_heads, int(causal), _dt(x))
    return y


def attention_backward(x, wq, wk, wv, wo, dy, n_heads, causal=False):
    """attention_backward (adjoint.rs:582) -> (dx, dwq, dwk, dwv, dwo)."""
    b, s, d = x.shape
    outs = [torch.empty_like(t) for t in (x, wq, wk, wv, wo)]
    _lib.call("catnn_mha_bwd", _h(x), _p(x), _p(wq), _p(wk), _p(wv), _p(wo), _p(dy), *[_p(o) for o in outs], b, s, d,
              n_heads, int(causal), _dt(x))
    return tuple(outs)


def gqa(x, wq, wk, wv, wo, n_heads, n_kv, theta, window=None):
    """moe::gqa (moe.rs:64): causal GQA with RoPE and optional window."""
    _same(x, wq, wk, wv, wo)
    b, s, d = x.shape
    hd = wq.shape[1] // n_heads
    y = torch.empty(b, s, wo.shape[1], dtype=x.dtype, device=x.device)
    _lib.call("catnn_gqa_fwd", _h(x), _p(x), _p(wq), _p(wk), _p(wv), _p(wo), _p(y), b, s, d, n_heads, n_kv, hd,
              float(theta), int(window or 0), _dt(x))
    return y


def gqa_backward(x, wq, wk, wv, wo, dy, n_heads, n_kv, theta, window=None):
    """gqa_backward (adjoint.rs:287) -> (dx, dwq, dwk, dwv, dwo)."""
    b, s, d = x.shape
    hd = wq.shape[1] // n_heads
    outs = [torch.empty_like(t) for t in (x, wq, wk, wv, wo)]
    _lib.call("catnn_gqa_bwd", _h(x), _p(x), _p(wq), _p(wk), _p(wv), _p(wo), _p(dy), *[_p(o) for o in outs], b, s, d,
              n_heads, n_kv, hd, float(theta), int(window or 0), _dt(x))
    return tuple(outs)


# ------------------------------------------------------------------ MoE
def router_topk(logits, k):
    """lens::moe::topk_softmax per row -> (idx int32 [T,k], w fp32 [T,k])."""
    _f32(logits, "logits")
    t, e = logits.shape
    idx = torch.empty(t, k, dtype=torch.int32, device=logits.device)
    w = torch.empty(t, k, dtype=torch.float32, device=logits.device)
    _lib.call("catnn_router_topk", _h(logits), _p(logits), t, e, k, _p(idx), _p(w))
    return idx, w


def moe_permute_map(idx, n_experts, align=1):
    """Stable counting sort of (token, slot) pairs by expert."""
    t, k = idx.shape
    dev = idx.device
    cap = t * k + n_experts * (align - 1)
    counts = torch.empty(n_experts, dtype=torch.int32, device=dev)
    offsets = torch.empty(n_experts + 1, dtype=torch.int32, device=dev)
    row_of = torch.empty(t * k, dtype=torch.int32, device=dev)
    src_of = torch.empty(cap, dtype=torch.int32, device=dev)
    _lib.call("catnn_moe_permute_map", _h(idx), _p(idx.contiguous()), t, n_experts, k, align, _p(counts), _p(offsets),
              _p(row_of), _p(src_of))
    return counts, offsets, row_of, src_of


def moe_permute(x, src_of, k):
    rows = src_of.numel()
    h = x.shape[-1]
    xp = torch.empty(rows, h, dtype=x.dtype, device=x.device)
    _lib.call("catnn_moe_permute", _h(x), _p(x), _p(src_of), rows, h, k, _p(xp), _dt(x))
    return xp


def moe_unpermute(yp, row_of, w, tokens, k):
    h = yp.shape[-1]
    y = torch.empty(tokens, h, dtype=yp.dtype, device=yp.device)
    _lib.call("catnn_moe_unpermute", _h(yp), _p(yp), _p(row_of), _p(w), tokens, k, h, _p(y), _dt(yp))
    return y


def grouped_gemm(a, b, offsets, trans_b=False, out=None, out_dtype=None):
    """Per-expert GEMM over expert-sorted rows (catnn_grouped_gemm):
    rows [off[g], off[g+1]) of a [rows, K] times b[g] ([K,N], or [N,K] with trans_b)."""
    _same(a, b)
    rows, k = a.shape
    g = b.shape[0]
    n = b.shape[1] if trans_b else b.shape[2]
    if out is None:
        out = torch.empty(rows, n, dtype=out_dtype or a.dtype, device=a.device)
    _lib.call("catnn_grouped_gemm", _h(a), int(trans_b), rows, n, k, g, _p(offsets), _p(a), _p(b), _p(out), _dt(a),
              _dt(out))
    return out


def interleave_w13(w1s, w3s):
    """[E, hidden, 2·mid] with each expert's w1 and w3 columns interleaved in
    blocks of 128 (the layout of the fused SwiGLU expert GEMMs)."""
    E, h, F = w1s.shape
    if F % 128:
        raise ShapeMismatch("interleaved w13: mid must be a multiple of 128")
    return torch.stack((w1s.reshape(E, h, F // 128, 128), w3s.reshape(E, h, F // 128, 128)), 3).reshape(E, h, 2 * F)


def moe_expert_swiglu(x, w13, offsets):
    """ac = x·w13 and h = silu(a)·c per expert group, the SwiGLU in the GEMM
    epilogue (catnn_moe_expert_swiglu_fwd; bf16). Returns (ac, h)."""
    _same(x, w13)
    rows, hidden = x.shape
    E, _, F2 = w13.shape
    ac = torch.empty(rows, F2, dtype=x.dtype, device=x.device)
    h = torch.empty(rows, F2 // 2, dtype=x.dtype, device=x.device)
    _lib.call("catnn_moe_expert_swiglu_fwd", _h(x), _p(x), _p(w13), _p(offsets), rows, hidden, F2 // 2, E, _p(ac), _p(h))
    return ac, h


def moe_expert_swiglu_backward(dy, w2, ac, offsets):
    """dac = [da | dc] from dh = dy·w2ᵀ per expert group and the saved ac
    (catnn_moe_expert_swiglu_bwd; bf16)."""
    _same(dy, w2, ac)
    rows, hidden = dy.shape
    E, F, _ = w2.shape
    dac = torch.empty(rows, 2 * F, dtype=dy.dtype, device=dy.device)
    _lib.call("catnn_moe_expert_swiglu_bwd", _h(dy), _p(dy), _p(w2), _p(ac), _p(offsets), rows, hidden, F, E, _p(dac))
    return dac


def swiglu(x, w1, w3, w2):
    """moe::swiglu (moe.rs:159)."""
    _same(x, w1, w3, w2)
    h = x.shape[-1]
    t = x.numel() // h
    mid = w1.shape[1]
    y = torch.empty_like(x)
    _lib.call("catnn_swiglu_fwd", _h(x), _p(x), _p(w1), _p(w3), _p(w2), _p(y), t, h, mid, _dt(x))
    return y


def swiglu_backward(x, w1, w3, w2, dy):
    """swiglu_backward (adjoint.rs:217) -> (dx, dw1, dw3, dw2)."""
    h = x.shape[-1]
    t = x.numel() // h
    mid = w1.shape[1]
    outs = [torch.empty_like(a) for a in (x, w1, w3, w2)]
    _lib.call("catnn_swiglu_bwd", _h(x), _p(x), _p(w1), _p(w3), _p(w2), _p(dy), *[_p(o) for o in outs], t, h, mid, _dt(x))
    return tuple(outs)


def moe(x, gate, w1s, w3s, w2s, top_k):
    """moe::moe (moe.rs:197); expert weights stacked [E, ...]."""
    _same(x, gate, w1s, w3s, w2s)
    h = x.shape[-1]
    t = x.numel() // h
    e, _, mid = w1s.shape
    y = torch.empty_like(x)
    _lib.call("catnn_moe_fwd", _h(x), _p(x), _p(gate), _p(w1s), _p(w3s), _p(w2s), _p(y), t, h, mid, e, top_k, _dt(x))
    return y


def moe_backward(x, gate, w1s, w3s, w2s, dy, top_k):
    """moe_backward (adjoint.rs:471) -> (dx, dgate, dw1s, dw3s, dw2s)."""
    h = x.shape[-1]
    t = x.numel() // h
    e, _, mid = w1s.shape
    outs = [torch.empty_like(a) for a in (x, gate, w1s, w3s, w2s)]
    _lib.call("catnn_moe_bwd", _h(x), _p(x), _p(gate), _p(w1s), _p(w3s), _p(w2s), _p(dy), *[_p(o) for o in outs], t, h, mid,
              e, top_k, _dt(x))
    return tuple(outs)


# ------------------------------------------------------------------ optimizers
def sgd_(p, g, lr, shadow=None):
    """Sgd::put in place (optim.rs:32): p -= lr * g."""
    _f32(p, "param")
    _f32(g, "grad")
    if p.numel() != g.numel():
        raise ShapeMismatch("sgd put")
    _lib.call("catnn_sgd", _h(p), _p(p), _p(g), p.numel(), float(lr), _p(shadow))
    return p


def adam_(p, g, m, v, t, lr, beta1=0.9, beta2=0.999, eps=1e-8, shadow=None):
    """Adam::put in place (optim.rs:95) at step count t (>= 1)."""
    _f32(p, "param")
    if not (p.numel() == g.numel() == m.numel() == v.numel()):
        raise ShapeMismatch("adam shapes")
    _lib.call("catnn_adam", _h(p), _p(p), _p(g), _p(m), _p(v), p.numel(), int(t), float(lr), float(beta1), float(beta2),
              float(eps), _dt(g), _p(shadow))
    return p


# ------------------------------------------------------------------ MLP step
def mlp_step(w1, b1, w2, b2, x, labels=None, y_mse=None):
    """train::mlp_step (train.rs:71) -> (loss tensor, dw1, db1, dw2, db2)."""
    batch, din = x.shape
    hid, dout = w1.shape[1], w2.shape[1]
    ce = labels is not None
    loss = torch.empty((), dtype=torch.float32, device=x.device)
    dw1, db1, dw2, db2 = (torch.empty_like(t) for t in (w1, b1, w2, b2))
    lab = _ids(labels) if ce else None
    _lib.call("catnn_mlp_step", _h(x), _p(w1), _p(b1), _p(w2), _p(b2), _p(x), _p(lab), _p(y_mse), int(ce), batch, din, hid,
              dout, _p(loss), _p(dw1), _p(db1), _p(dw2), _p(db2))
    return loss, dw1, db1, dw2, db2


def checksum(x):
    """FNV-1a over the f32 bits (tensor.rs:279), computed on the device."""
    _f32(x, "checksum input")
    v = C.c_uint64()
    _lib.call("catnn_checksum_f32", _h(x), _p(x), x.numel(), C.byref(v))
    return int(v.value)


# ------------------------------------------------------------------ kernel resources
class KernelShape(C.Structure):
    """catnn_kernel_shape (include/catnn_b200.h)."""
    _fields_ = [(n, C.c_int64) for n in ("rows", "width", "inner", "batch", "seq", "heads", "head_dim")]


class KernelResource(C.Structure):
    """catnn_kernel_resource (include/catnn_b200.h): KernelResource of
    crates/catnn-compile/src/kernel/resource.rs:28-44, measured."""
    _fields_ = [("kernel", C.c_char * 192), ("file", C.c_char * 32), ("registers_per_thread", C.c_int32),
                ("max_threads_per_block", C.c_int32), ("static_smem_bytes", C.c_int64),
                ("dynamic_smem_bytes", C.c_int64), ("local_bytes_per_thread", C.c_int64), ("grid", C.c_uint32 * 3),
                ("block", C.c_uint32 * 3), ("launch_arg_bytes", C.c_int64), ("code_bytes", C.c_int64),
                ("code_estimated", C.c_int32), ("binary_version", C.c_int32)]


def kernel_describe(op, dtype=torch.bfloat16, device=None, rows=0, width=0, inner=0, batch=0, seq=0, heads=0,
                    head_dim=0):
    """The resource record of the kernel that runs IR op `op` (resource::describe,
    resource.rs:159), as a dict."""
    shape = KernelShape(rows, width, inner, batch, seq, heads, head_dim)
    out = KernelResource()
    h = context(device).bind()
    _lib.call("catnn_kernel_describe", h, op.encode(), BF16 if dtype == torch.bfloat16 else F32, C.byref(shape),
              C.byref(out))
    d = {f: getattr(out, f) for f, _ in KernelResource._fields_}
    d["kernel"], d["file"] = out.kernel.decode(), out.file.decode()
    d["grid"], d["block"] = list(out.grid), list(out.block)
    return d
