"""The operator boundary of the reference, re-hosted on the GPU backend.

Mirrors, with the same names, argument meaning and errors:
- ``OpenOp`` — the op vocabulary (crates/catnn-core/src/category/morphism.rs:19-116)
- ``IrNode`` — op + named parameter ports (crates/catnn-compile/src/ir.rs:17-24)
- ``eval_gpu`` — the forward dispatcher ``eval_cpu`` (crates/catnn-compile/src/kernel/mod.rs:21)
- ``adjoint_of`` / ``Adjoint`` — reverse dispatcher (crates/catnn-compile/src/kernel/adjoint.rs:752-951)
- ``adjoint_needs_output`` (adjoint.rs:954)
- ``DeviceHandler.run_kernel`` / ``note_kernel`` (crates/catnn-rt/src/handler.rs:34-79)
- ``loss_and_grad`` / ``apply_update`` (crates/catnn-compile/src/pipeline.rs:448-471)

Parameters are device tensors keyed by the reference's port names ("w",
"b", "gamma", "beta", "wq".."wo", "gate", "e{i}.w1|w3|w2"). Every op runs a
libcatnn_b200 kernel; an op the backend does not build raises Unsupported.
"""
import time
from dataclasses import dataclass, field

import torch

from . import ops
from .errors import ShapeMismatch, UnknownComponent, UnknownPort, Unlawful, Unsupported, Wiring


@dataclass(frozen=True)
class OpenOp:
    kind: str
    attrs: tuple = ()

    def get(self, key, default=None):
        return dict(self.attrs).get(key, default)

    def name(self):
        return self.kind

    # constructors, one per reference variant
    @staticmethod
    def _mk(kind, **kw):
        return OpenOp(kind, tuple(sorted(kw.items())))

    identity = staticmethod(lambda: OpenOp._mk("identity"))
    relu = staticmethod(lambda: OpenOp._mk("relu"))
    gelu = staticmethod(lambda: OpenOp._mk("gelu"))
    add = staticmethod(lambda: OpenOp._mk("add"))
    mul = staticmethod(lambda: OpenOp._mk("mul"))
    matmul = staticmethod(lambda: OpenOp._mk("matmul"))
    residual_add = staticmethod(lambda: OpenOp._mk("residual_add"))
    mix = staticmethod(lambda: OpenOp._mk("mix"))

    @staticmethod
    def linear(in_features, out_features, bias=True):
        return OpenOp._mk("linear", in_features=in_features, out_features=out_features, bias=bias)

    @staticmethod
    def softmax(axis=-1):
        return OpenOp._mk("softmax", axis=axis)

    @staticmethod
    def layer_norm(eps_e6=10):
        return OpenOp._mk("layer_norm", eps_e6=eps_e6)

    @staticmethod
    def transpose(dim0, dim1):
        return OpenOp._mk("transpose", dim0=dim0, dim1=dim1)

    @staticmethod
    def reshape(out):
        return OpenOp._mk("reshape", out=tuple(out))

    @staticmethod
    def attention(n_heads, d_model, d_head):
        return OpenOp._mk("attention", n_heads=n_heads, d_model=d_model, d_head=d_head)

    @staticmethod
    def embedding(vocab, hidden):
        return OpenOp._mk("embedding", vocab=vocab, hidden=hidden)

    @staticmethod
    def rms_norm(eps_e6=10):
        return OpenOp._mk("rms_norm", eps_e6=eps_e6)

    @staticmethod
    def gqa_attention(n_heads, n_kv_heads, head_dim, d_model, sliding_window=None, rope_theta=10000):
        return OpenOp._mk("gqa_attention", n_heads=n_heads, n_kv_heads=n_kv_heads, head_dim=head_dim, d_model=d_model,
                          sliding_window=sliding_window, rope_theta=rope_theta)

    @staticmethod
    def swiglu(hidden, intermediate):
        return OpenOp._mk("swiglu", hidden=hidden, intermediate=intermediate)

    @staticmethod
    def router(n_experts, top_k):
        return OpenOp._mk("router", n_experts=n_experts, top_k=top_k)

    @staticmethod
    def moe(n_experts, top_k, hidden, intermediate):
        return OpenOp._mk("moe", n_experts=n_experts, top_k=top_k, hidden=hidden, intermediate=intermediate)

    @staticmethod
    def lm_head(hidden, vocab):
        return OpenOp._mk("lm_head", hidden=hidden, vocab=vocab)


@dataclass
class IrNode:
    name: str
    op: OpenOp
    params: dict = field(default_factory=dict)
    output_shape: tuple = ()


@dataclass
class Adjoint:
    dx: list
    dparams: dict


def _need(node, port):
    t = node.params.get(port)
    if t is None:
        raise UnknownPort(f"unknown port {port} on interface {node.name}")
    return t


def _eps(op):
    return float(op.get("eps_e6")) * 1e-6


def _experts(node, n):
    w1 = torch.stack([_need(node, f"e{e}.w1") for e in range(n)])
    w3 = torch.stack([_need(node, f"e{e}.w3") for e in range(n)])
    w2 = torch.stack([_need(node, f"e{e}.w2") for e in range(n)])
    return w1, w3, w2


def _token_ids(x):
    # mod.rs:86-87: ids come in as f32 and are rounded, clamped at 0
    return torch.clamp(torch.round(x), min=0).to(torch.int32) if x.is_floating_point() else x.to(torch.int32)


def eval_gpu(node, inputs):
    """Forward of one IR node on the GPU (kernel/mod.rs:21 eval_cpu)."""
    op = node.op
    k = op.kind
    if not inputs:
        if k == "identity":
            return torch.zeros(node.output_shape, device="cuda")
        raise Wiring(f"{node.name} has no inputs")
    x = inputs[0]
    if k in ("identity", "reshape", "transpose"):
        return x.clone()
    if k == "relu":
        return ops.relu(x)
    if k == "gelu":
        return ops.gelu(x)
    if k == "softmax":
        return ops.softmax_last(x)
    if k in ("add", "residual_add"):
        return ops.add(x, inputs[1]) if len(inputs) > 1 else x.clone()
    if k == "mul":
        return ops.mul(x, inputs[1]) if len(inputs) > 1 else x.clone()
    if k in ("linear", "matmul"):
        w = node.params.get("w")
        if w is None:
            if not node.params:
                raise UnknownComponent(node.name)
            w = next(iter(node.params.values()))
        return ops.linear(x, w, node.params.get("b"))
    if k == "layer_norm":
        return ops.layer_norm(x, _need(node, "gamma"), _need(node, "beta"), _eps(op))
    if k == "attention":
        return ops.attention(x, _need(node, "wq"), _need(node, "wk"), _need(node, "wv"), _need(node, "wo"),
                             op.get("n_heads"), causal=False)
    if k == "rms_norm":
        return ops.rmsnorm(x, _need(node, "w"), _eps(op))
    if k == "embedding":
        y = ops.embedding(_token_ids(x), _need(node, "w"))
        return y
    if k == "swiglu":
        return ops.swiglu(x, _need(node, "w1"), _need(node, "w3"), _need(node, "w2"))
    if k == "moe":
        w1, w3, w2 = _experts(node, op.get("n_experts"))
        return ops.moe(x, _need(node, "gate"), w1, w3, w2, op.get("top_k"))
    if k == "gqa_attention":
        return ops.gqa(x, _need(node, "wq"), _need(node, "wk"), _need(node, "wv"), _need(node, "wo"), op.get("n_heads"),
                       op.get("n_kv_heads"), float(op.get("rope_theta")), op.get("sliding_window"))
    if k == "lm_head":
        return ops.lm_head(x, _need(node, "w"))
    if k == "router":
        return x.clone()  # mod.rs:131: the router node passes its input through
    raise Unsupported(f"{k} is not part of the GPU hot path")


def adjoint_of(node, inputs, output, dy):
    """Reverse rule of one IR node (adjoint.rs:762 adjoint_of)."""
    if not inputs:
        raise Wiring(f"{node.name} adjoint has no inputs")
    x = inputs[0]
    op = node.op
    k = op.kind
    dparams = {}
    if k in ("identity", "reshape", "transpose"):
        dx = [dy.clone()]
    elif k == "relu":
        dx = [ops.relu_backward(x, dy)]
    elif k == "gelu":
        dx = [ops.gelu_backward(x, dy)]
    elif k == "softmax":
        dx = [ops.softmax_backward(output, dy)]
    elif k in ("add", "residual_add"):
        dx = [dy.clone()] if len(inputs) == 1 else [dy.clone(), dy.clone()]
    elif k == "mul":
        dx = [dy.clone()] if len(inputs) == 1 else [ops.mul(dy, inputs[1]), ops.mul(dy, x)]
    elif k in ("linear", "matmul"):
        w = _need(node, "w")
        gx, gw, gb = ops.linear_backward(x, w, dy, need_db="b" in node.params)
        dparams["w"] = gw
        if "b" in node.params:
            dparams["b"] = gb
        dx = [gx]
    elif k == "layer_norm":
        gx, gg, gb = ops.layer_norm_backward(x, _need(node, "gamma"), dy, _eps(op))
        _need(node, "beta")
        dparams.update(gamma=gg, beta=gb)
        dx = [gx]
    elif k == "attention":
        gx, gq, gk, gv, go = ops.attention_backward(x, _need(node, "wq"), _need(node, "wk"), _need(node, "wv"),
                                                    _need(node, "wo"), dy, op.get("n_heads"), causal=False)
        dparams.update(wq=gq, wk=gk, wv=gv, wo=go)
        dx = [gx]
    elif k == "rms_norm":
        gx, gw = ops.rmsnorm_backward(x, _need(node, "w"), dy, _eps(op))
        dparams["w"] = gw
        dx = [gx]
    elif k == "embedding":
        table = _need(node, "w")
        dparams["w"] = ops.embedding_backward(_token_ids(x), dy, table.shape[0])
        dx = [torch.zeros_like(x)]
    elif k == "swiglu":
        gx, g1, g3, g2 = ops.swiglu_backward(x, _need(node, "w1"), _need(node, "w3"), _need(node, "w2"), dy)
        dparams.update(w1=g1, w3=g3, w2=g2)
        dx = [gx]
    elif k == "gqa_attention":
        gx, gq, gk, gv, go = ops.gqa_backward(x, _need(node, "wq"), _need(node, "wk"), _need(node, "wv"), _need(node, "wo"),
                                              dy, op.get("n_heads"), op.get("n_kv_heads"), float(op.get("rope_theta")),
                                              op.get("sliding_window"))
        dparams.update(wq=gq, wk=gk, wv=gv, wo=go)
        dx = [gx]
    elif k == "moe":
        n = op.get("n_experts")
        w1, w3, w2 = _experts(node, n)
        gx, gg, g1, g3, g2 = ops.moe_backward(x, _need(node, "gate"), w1, w3, w2, dy, op.get("top_k"))
        dparams["gate"] = gg
        for e in range(n):
            dparams[f"e{e}.w1"], dparams[f"e{e}.w3"], dparams[f"e{e}.w2"] = g1[e], g3[e], g2[e]
        dx = [gx]
    elif k == "lm_head":
        gx, gw = ops.lm_head_backward(x, _need(node, "w"), dy)
        dparams["w"] = gw
        dx = [gx]
    elif k == "router":
        raise Unlawful("router adjoint is the straight-through estimator inside MoE, not a standalone op")
    else:
        raise Unsupported(f"{k} is not part of the GPU hot path")
    if len(dx) != len(inputs):
        raise Wiring(f"{node.name} adjoint produced {len(dx)} cotangents for {len(inputs)} inputs")
    return Adjoint(dx, dparams)


def adjoint_needs_output(op):
    return op.kind == "softmax"


def loss_and_grad(pred, target):
    """pipeline.rs:448: integer class targets -> cross-entropy, else MSE."""
    if target.is_floating_point():
        return ops.mse_loss(pred, target)
    return ops.cross_entropy(pred, target)


class AdamState:
    def __init__(self, p):
        self.m = torch.zeros_like(p)
        self.v = torch.zeros_like(p)
        self.t = 0


def apply_update(p, g, opt, lr, adam_state=None):
    """pipeline.rs:455 apply_update, in place on the device parameter.
    Returns (p, adam_state)."""
    if opt == "sgd":
        ops.sgd_(p, g, lr)
        return p, adam_state
    if opt == "adam":
        st = adam_state or AdamState(p)
        st.t += 1
        ops.adam_(p, g, st.m, st.v, st.t, lr)
        return p, st
    raise ValueError(f"unknown optimizer {opt}")


@dataclass
class Event:
    """handler.rs / sheaf.rs event: time, op, device, kind, checksum."""
    t: int
    op: str
    device: str
    kind: str
    checksum: int


class DeviceHandler:
    """GPU DeviceHandler (handler.rs:14-91): runs kernels on its device and
    records KernelStart/KernelEnd events with the output checksum."""

    def __init__(self, device_id="gpu0", device=0):
        self.device_id = device_id
        self.device = device
        self.events = []
        self._epoch = time.perf_counter_ns()

    def _now(self):
        return time.perf_counter_ns() - self._epoch

    def run_kernel(self, node, inputs):
        t0 = self._now()
        self.events.append(Event(t0, node.name, self.device_id, "KernelStart", 0))
        with torch.cuda.device(self.device):
            y = eval_gpu(node, inputs)
            chk = ops.checksum(y.float().contiguous()) if y.is_floating_point() else 0
        self.events.append(Event(max(self._now(), t0 + 1), node.name, self.device_id, "KernelEnd", chk))
        return y

    def note_kernel(self, name, checksum):
        t0 = self._now()
        self.events.append(Event(t0, name, self.device_id, "KernelStart", 0))
        self.events.append(Event(max(self._now(), t0 + 1), name, self.device_id, "KernelEnd", checksum))
