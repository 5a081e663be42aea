"""The operator boundary of the reference, re-hosted on the GPU backend.

Mirrors, with the same names, argument meaning and errors:
- ``OpenOp`` — the op vocabulary (crates/catnn-core/src/category/morphism.rs:19-116)
- ``IrNode`` — op + named parameter ports (crates/catnn-compile/src/ir.rs:17-24)
- ``eval_gpu`` — the forward dispatcher ``eval_cpu`` (crates/catnn-compile/src/kernel/mod.rs:21)
- ``adjoint_of`` / ``Adjoint`` — reverse dispatcher (crates/catnn-compile/src/kernel/adjoint.rs:752-951)
- ``adjoint_needs_output`` (adjoint.rs:954)
- ``DeviceHandler.run_kernel`` / ``note_kernel`` (crates/catnn-rt/src/handler.rs:34-79)
- ``loss_and_grad`` / ``apply_update`` (crates/catnn-compile/src/pipeline.rs:448-471)
- ``IrGraph`` (crates/catnn-compile/src/ir.rs:33-80) and the one-device
  training runtime of crates/catnn-rt/src/coord.rs: ``DeviceRt`` keeps every
  activation, cotangent, parameter and optimizer state device-resident
  (``act:{id}``, ``grad:{id}:from:{succ}``, ``grad:{id}``), ``train_step``
  runs forward_one / loss_one / backward_one / apply_pending
  (coord.rs:188-488), and ``ensure_act`` rematerializes checkpointed
  activations with ``eval_gpu`` (coord.rs:436-473).
- ``mixtral_graph`` — the Mixtral IR chain with its residual adds wired as
  two-input ``residual_add`` nodes, so the IR path trains the model of
  train::mixtral_step (crates/catnn-compile/src/train.rs:261-356).

Parameters are device tensors keyed by the reference's port names ("w",
"b", "gamma", "beta", "wq".."wo", "gate", "e{i}.w1|w3|w2"). Every op runs a
libcatnn_b200 kernel; an op the backend does not build raises Unsupported.
"""
import time
from dataclasses import dataclass, field

import torch

from . import ops
from .errors import Fibration, ShapeMismatch, UnknownComponent, UnknownPort, Unlawful, Unsupported, Wiring


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
    id: int = -1


@dataclass(frozen=True)
class IrEdge:
    src: int
    dst: int
    src_port: str = "Y"
    dst_port: str = "X"


class IrGraph:
    """DAG of IR nodes (ir.rs:33-80): nodes keyed by id, edges in insertion
    order (a node's inputs are its predecessors in edge order), graph inputs
    (fed by the host) and outputs (the last one is the prediction)."""

    def __init__(self, name):
        self.name = name
        self.nodes = {}
        self.edges = []
        self.inputs = []
        self.outputs = []

    def add(self, name, op, params=None, preds=(), is_input=False):
        nid = len(self.nodes)
        self.nodes[nid] = IrNode(name, op, dict(params or {}), (), nid)
        for p in preds:
            self.edges.append(IrEdge(p, nid))
        if is_input:
            self.inputs.append(nid)
        return nid

    def node(self, nid):
        return self.nodes.get(nid)

    def preds(self, nid):
        return [e.src for e in self.edges if e.dst == nid]

    def succs(self, nid):
        return [e.dst for e in self.edges if e.src == nid]

    def by_name(self, name):
        for n in self.nodes.values():
            if n.name == name:
                return n
        raise UnknownComponent(name)

    def topo(self):
        """Kahn's order, smallest ready id first (ir.rs:64-80 pops the largest
        of a sorted list; any topological order gives the same values)."""
        indeg = {k: 0 for k in self.nodes}
        for e in self.edges:
            indeg[e.dst] += 1
        ready = sorted(k for k, d in indeg.items() if d == 0)
        out = []
        while ready:
            n = ready.pop(0)
            out.append(n)
            for s in sorted(e.dst for e in self.edges if e.src == n):
                indeg[s] -= 1
                if indeg[s] == 0:
                    ready.append(s)
                    ready.sort()
        if len(out) != len(self.nodes):
            raise Wiring(f"{self.name} has a cycle")
        return out


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


# ------------------------------------------------------------ runtime


class DeviceRt:
    """One device's training state (crates/catnn-rt/src/coord.rs DeviceRt):
    every tensor stays on the GPU between kernels, keyed as the reference
    keys them: ``act:{id}`` (outputs), ``grad:{id}:from:{succ}`` (cotangents
    from each consumer), ``grad:{id}`` (the loss gradient of the output).
    ``params[id]`` maps port names to device tensors; gradients wait in
    ``pending`` until every node's backward ran; ``adam`` keeps each
    (node, port)'s moments."""

    def __init__(self, graph, device=0):
        self.device = device
        self.tensors = {}
        self.fed = {}
        self.params = {nid: dict(n.params) for nid, n in graph.nodes.items() if n.params}
        self.pending = {}
        self.adam = {}
        self.target = None
        self.loss = None
        self.reset()

    def reset(self):
        """Clear one step's activations and cotangents (parameters, optimizer
        state and the inputs stay)."""
        self.tensors = {f"act:{nid}": x for nid, x in self.fed.items()}
        self.fw_done, self.bw_done = set(), set()
        self.loss_done = self.dropped = self.updates_done = False
        self.rematerialized = 0

    def feed(self, graph, inputs, target):
        """The host's batch: the graph inputs' activations and the target."""
        for nid, x in zip(graph.inputs, inputs):
            self.fed[nid] = x
            self.tensors[f"act:{nid}"] = x
        self.target = target


def _node_op(node, state):
    if node.id in state.params:
        return IrNode(node.name, node.op, state.params[node.id], node.output_shape, node.id)
    return node


def forward_one(nid, state, handler, graph):
    """coord.rs:295-328: run one node once all its inputs are present."""
    if nid in state.fw_done:
        return False
    if nid in graph.inputs:
        if f"act:{nid}" in state.tensors:
            state.fw_done.add(nid)
            return True
        return False
    preds = graph.preds(nid)
    if any(f"act:{p}" not in state.tensors for p in preds):
        return False
    y = handler.run_kernel(_node_op(graph.node(nid), state), [state.tensors[f"act:{p}"] for p in preds])
    state.tensors[f"act:{nid}"] = y
    state.fw_done.add(nid)
    return True


def loss_one(graph, state):
    """coord.rs:330-348: loss and its gradient at the last output."""
    if state.loss_done:
        return False
    out = graph.outputs[-1]
    pred = state.tensors.get(f"act:{out}")
    if pred is None or state.target is None:
        return False
    loss, dy = loss_and_grad(pred, state.target)
    state.tensors[f"grad:{out}"] = dy
    state.loss = loss
    state.loss_done = True
    return True


def ensure_act(nid, state, graph):
    """coord.rs:436-473: an activation dropped after the forward is rebuilt
    from its (recursively rebuilt) inputs by the same forward kernel."""
    if f"act:{nid}" in state.tensors:
        return
    node = graph.node(nid)
    if nid in graph.inputs:
        raise Fibration(f"input {node.name} was checkpointed; the host value cannot be rematerialized")
    preds = graph.preds(nid)
    for p in preds:
        ensure_act(p, state, graph)
    with torch.cuda.device(state.device):
        state.tensors[f"act:{nid}"] = eval_gpu(_node_op(node, state), [state.tensors[f"act:{p}"] for p in preds])
    state.rematerialized += 1


def backward_one(nid, state, handler, graph):
    """coord.rs:350-434: once every consumer's cotangent arrived, sum them (in
    consumer order), run the node's adjoint, send each input its cotangent and
    park the parameter gradients."""
    if nid in state.bw_done:
        return False
    if nid in graph.inputs:
        if nid in state.fw_done:
            state.bw_done.add(nid)
            return True
        return False
    succs = graph.succs(nid)
    if not succs:
        dy = state.tensors.get(f"grad:{nid}")
        if dy is None:
            return False
    else:
        dy = None
        for s in succs:
            g = state.tensors.get(f"grad:{nid}:from:{s}")
            if g is None:
                return False
            dy = g if dy is None else ops.add(dy, g)
    preds = graph.preds(nid)
    for p in preds:
        ensure_act(p, state, graph)
    node = graph.node(nid)
    if adjoint_needs_output(node.op):
        ensure_act(nid, state, graph)
    inputs = [state.tensors[f"act:{p}"] for p in preds]
    output = state.tensors.get(f"act:{nid}", inputs[0])
    op = _node_op(node, state)
    handler.note_kernel(f"{op.name}.bwd", ops.checksum(dy.float().contiguous()) if dy.is_floating_point() else 0)
    with torch.cuda.device(state.device):
        adj = adjoint_of(op, inputs, output, dy)
    for p, dx in zip(preds, adj.dx):
        tag = f"grad:{p}:from:{nid}"
        prev = state.tensors.get(tag)
        state.tensors[tag] = dx if prev is None else ops.add(prev, dx)
    for port, g in adj.dparams.items():
        state.pending[(nid, port)] = g
    state.bw_done.add(nid)
    return True


def apply_pending(state, opt, lr):
    """coord.rs:475-488: every parked gradient updates its parameter in
    place (SGD or Adam, pipeline.rs:455)."""
    pending, state.pending = state.pending, {}
    for (nid, port), g in pending.items():
        slot = state.params.get(nid)
        if slot is None or port not in slot:
            continue
        p, st = apply_update(slot[port], g, opt, lr, state.adam.get((nid, port)))
        if st is not None:
            state.adam[(nid, port)] = st


def train_step(graph, state, handler, checkpointed=(), opt="sgd", lr=0.05, update=True):
    """One training step of an IR graph on one GPU (coord.rs:188-290
    training_device with every node placed on this device): forward in
    topological order, the loss, then — once the forward is complete — the
    activations of the `checkpointed` node names are dropped; the backward
    runs in reverse order (rematerializing what it needs), then the updates.
    Returns the loss (device scalar). With update=False the gradients stay in
    ``state.pending``."""
    order = graph.topo()
    state.reset()
    for nid in order:
        if not forward_one(nid, state, handler, graph):
            raise Wiring(f"{graph.node(nid).name} could not run: an input is missing")
    if not loss_one(graph, state):
        raise Wiring(f"{graph.name}: no target or no output for the loss")
    for name in checkpointed:
        state.tensors.pop(f"act:{graph.by_name(name).id}", None)
    state.dropped = True
    for nid in reversed(order):
        if not backward_one(nid, state, handler, graph):
            raise Wiring(f"{graph.node(nid).name}: a cotangent is missing")
    if update:
        apply_pending(state, opt, lr)
        state.updates_done = True
    return state.loss


def mixtral_graph(cfg, P, batch, seq):
    """The Mixtral decoder as an IR graph with its residuals wired explicitly.

    The reference's lowering (crates/catnn-core/src/spec/mixtral.rs:179-294)
    is a chain — embed, per layer rms_attn, gqa, rms_moe, moe, then
    final_norm, lm_head — without the residual adds that train::mixtral_step
    performs (train.rs:303-319). Here each layer also gets two
    ``residual_add`` nodes (x_mid = x + gqa(rms(x)), x_out = x_mid +
    moe(rms(x_mid))), so the IR path computes mixtral_step's model.

    P: the packed fp32 parameter vector on the device (MixtralWeights order,
    train.packed_layout); every port is a view of it, so in-place updates
    land in P. Returns (graph, ids of the token input node)."""
    from .train import packed_layout
    L = packed_layout(cfg)
    h, V, F, E = cfg.hidden, cfg.vocab, cfg.mid, cfg.experts
    hd = h // cfg.heads
    qd, kd = cfg.heads * hd, cfg.kv_heads * hd

    def view(off, *shape):
        n = 1
        for s in shape:
            n *= s
        return P[off:off + n].view(*shape)
    g = IrGraph("mixtral")
    eps_e6 = int(round(cfg.rms_eps * 1e6))
    tok = g.add("tokens", OpenOp.identity(), is_input=True)
    x = g.add("embed", OpenOp.embedding(V, h), {"w": view(L["embed"], V, h)}, [tok])
    for l in range(cfg.layers):
        b = L["layer0"] + l * L["layer_stride"]
        r1 = g.add(f"L{l}.rms_attn", OpenOp.rms_norm(eps_e6), {"w": view(b + L["rms_attn"], h)}, [x])
        at = g.add(f"L{l}.gqa", OpenOp.gqa_attention(cfg.heads, cfg.kv_heads, hd, h, cfg.window or None,
                                                     cfg.rope_theta),
                   {"wq": view(b + L["wq"], h, qd), "wk": view(b + L["wk"], h, kd), "wv": view(b + L["wv"], h, kd),
                    "wo": view(b + L["wo"], qd, h)}, [r1])
        xm = g.add(f"L{l}.res_attn", OpenOp.residual_add(), {}, [x, at])
        r2 = g.add(f"L{l}.rms_moe", OpenOp.rms_norm(eps_e6), {"w": view(b + L["rms_moe"], h)}, [xm])
        mp = {"gate": view(b + L["gate"], h, E)}
        for e in range(E):
            mp[f"e{e}.w1"] = view(b + L["w1"] + e * h * F, h, F)
            mp[f"e{e}.w3"] = view(b + L["w3"] + e * h * F, h, F)
            mp[f"e{e}.w2"] = view(b + L["w2"] + e * F * h, F, h)
        mo = g.add(f"L{l}.moe", OpenOp.moe(E, cfg.top_k, h, F), mp, [r2])
        x = g.add(f"L{l}.res_moe", OpenOp.residual_add(), {}, [xm, mo])
    fn = g.add("final_norm", OpenOp.rms_norm(eps_e6), {"w": view(L["final_norm"], h)}, [x])
    lm = g.add("lm_head", OpenOp.lm_head(h, V), {"w": view(L["lm_head"], V, h)}, [fn])
    g.outputs.append(lm)
    return g, tok


def pack_grads(graph, state, cfg):
    """The pending parameter gradients of a mixtral_graph step as one packed
    fp32 vector in MixtralWeights order (the layout of mixtral_step's G)."""
    from .train import packed_layout
    L = packed_layout(cfg)
    out = torch.zeros(L["total"], dtype=torch.float32, device=f"cuda:{state.device}")
    h, F, E = cfg.hidden, cfg.mid, cfg.experts
    for (nid, port), gr in state.pending.items():
        name = graph.node(nid).name
        if name in ("embed", "final_norm", "lm_head"):
            off = {"embed": L["embed"], "final_norm": L["final_norm"], "lm_head": L["lm_head"]}[name]
        else:
            layer, kind = name.split(".", 1)
            b = L["layer0"] + int(layer[1:]) * L["layer_stride"]
            if kind in ("rms_attn", "rms_moe"):
                off = b + L[kind]
            elif kind == "gqa":
                off = b + L[port]
            elif port == "gate":
                off = b + L["gate"]
            else:
                e, w = port.split(".")
                e = int(e[1:])
                off = b + L[w] + e * h * F
        out[off:off + gr.numel()] = gr.reshape(-1).float()
    return out
