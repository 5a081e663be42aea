"""Training steps over the GPU backend.

``MoeTrainer`` wraps the native Mixtral-style decoder trainer
(catnn_moe_trainer_* in include/catnn_b200.h): parameters, optimizer state
and activations live on the device; a step is forward, next-token
cross-entropy, backward and SGD/Adam, mirroring train::mixtral_step
(crates/catnn-compile/src/train.rs:261) with its residual adds.

Parameters cross the boundary as one packed fp32 vector in the reference's
MixtralWeights field order (moe.rs:227-244); see ``packed_layout``.
"""
import ctypes as C

import numpy as np
import torch

from . import _lib, ops


class MoeConfig(C.Structure):
    """catnn_moe_config (include/catnn_b200.h)."""

    _fields_ = [(n, C.c_int64) for n in ("vocab", "hidden", "mid", "layers", "heads", "kv_heads", "experts", "top_k",
                                          "window", "batch", "seq")] + [
        ("rms_eps", C.c_float), ("rope_theta", C.c_double), ("dtype", C.c_int), ("optimizer", C.c_int),
        ("lr", C.c_float), ("beta1", C.c_float), ("beta2", C.c_float), ("adam_eps", C.c_float)]

    @classmethod
    def make(cls, vocab, hidden, mid, layers, heads, kv_heads, experts, top_k, batch, seq, window=None, rms_eps=1e-5,
             rope_theta=1e4, dtype=torch.bfloat16, optimizer="adam", lr=1e-3, beta1=0.9, beta2=0.999, adam_eps=1e-8):
        return cls(vocab, hidden, mid, layers, heads, kv_heads, experts, top_k, int(window or 0), batch, seq, rms_eps,
                   rope_theta, 1 if dtype == torch.bfloat16 else 0, 1 if optimizer == "adam" else 0, lr, beta1, beta2,
                   adam_eps)


def packed_layout(cfg):
    """Offsets of the packed parameter vector (the oracle's MixLayout)."""
    h, V, F, E = cfg.hidden, cfg.vocab, cfg.mid, cfg.experts
    hd = h // cfg.heads
    qd, kd = cfg.heads * hd, cfg.kv_heads * hd
    o = {"embed": 0, "layer0": V * h}
    off = 0
    for name, n in (("rms_attn", h), ("wq", h * qd), ("wk", h * kd), ("wv", h * kd), ("wo", qd * h), ("rms_moe", h),
                    ("gate", h * E), ("w1", E * h * F), ("w3", E * h * F), ("w2", E * F * h)):
        o[name] = off
        off += n
    o["layer_stride"] = off
    o["final_norm"] = o["layer0"] + cfg.layers * off
    o["lm_head"] = o["final_norm"] + h
    o["total"] = o["lm_head"] + V * h
    return o


def init_params(cfg, seed, std=0.02):
    """BASELINE init: weights N(0, std), RMSNorm weights 1 (seeded numpy)."""
    L = packed_layout(cfg)
    r = np.random.default_rng(seed)
    P = (r.standard_normal(L["total"]) * std).astype(np.float32)
    h = cfg.hidden
    for l in range(cfg.layers):
        base = L["layer0"] + l * L["layer_stride"]
        P[base + L["rms_attn"]:base + L["rms_attn"] + h] = 1.0
        P[base + L["rms_moe"]:base + L["rms_moe"] + h] = 1.0
    P[L["final_norm"]:L["final_norm"] + h] = 1.0
    return P


class MoeTrainer:
    """The native trainer on one GPU, or — given a ``dist.Comm`` — one rank of
    the data-parallel + expert-parallel trainer (catnn_moe_trainer_create_ep):
    ``cfg.batch`` is then the global batch, steps take the global token
    array, and ``params()`` / ``grads()`` fill the replicated entries and this
    rank's experts of the packed vector (other experts' entries are zero);
    with a communicator they are collective (every rank calls them)."""

    def __init__(self, cfg, device=0, comm=None):
        self.cfg = cfg
        self.device = device
        self.comm = comm
        self.ctx = ops.context(device)
        h = C.c_void_p()
        with torch.cuda.device(device):
            if comm is None:
                _lib.call("catnn_moe_trainer_create", self.ctx.bind(), C.byref(cfg), C.byref(h))
            else:
                _lib.call("catnn_moe_trainer_create_ep", self.ctx.bind(), C.byref(cfg), comm.handle, C.byref(h))
        self.handle = h
        self.world = comm.world if comm is not None else 1
        self.rank = comm.rank if comm is not None else 0
        n = C.c_int64()
        _lib.call("catnn_moe_trainer_param_count", C.byref(cfg), C.byref(n))
        self.n_params = int(n.value)

    def close(self):
        if self.handle:
            _lib.call("catnn_moe_trainer_destroy", self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _bind(self):
        self.ctx.bind()

    def set_params(self, packed):
        if torch.is_tensor(packed):
            t = packed.detach().to(device=f"cuda:{self.device}", dtype=torch.float32).contiguous()
        else:
            t = torch.as_tensor(np.ascontiguousarray(packed, np.float32)).to(f"cuda:{self.device}")
        assert t.numel() == self.n_params, (t.numel(), self.n_params)
        self._bind()
        _lib.call("catnn_moe_trainer_set_params", self.handle, C.c_void_p(t.data_ptr()))
        torch.cuda.synchronize(self.device)

    def _get(self, name):
        out = torch.zeros(self.n_params, dtype=torch.float32, device=f"cuda:{self.device}")
        self._bind()
        _lib.call(name, self.handle, C.c_void_p(out.data_ptr()))
        return out

    def params(self):
        return self._get("catnn_moe_trainer_get_params")

    def grads(self):
        return self._get("catnn_moe_trainer_get_grads")

    def step(self, tokens, update=True, loss_out=None):
        """Device step; tokens: int32/uint32 CUDA tensor [batch*seq]."""
        self._bind()
        _lib.call("catnn_moe_trainer_step", self.handle, C.c_void_p(tokens.data_ptr()),
                  C.c_void_p(loss_out.data_ptr()) if loss_out is not None else None, int(update))
        return loss_out

    def step_host(self, tokens_np, update=True):
        """End-to-end step from host token ids to a host float loss."""
        tok = np.ascontiguousarray(tokens_np, np.uint32)
        loss = C.c_float()
        self._bind()
        _lib.call("catnn_moe_trainer_step_host", self.handle, tok.ctypes.data_as(C.c_void_p), C.byref(loss), int(update))
        return float(loss.value)

    ACTIVATIONS = {"x_in": 0, "x_mid": 1, "xm": 2, "ctx": 3, "router_logits": 4, "x_last": 5, "xf": 6}

    def activation(self, name, layer=0):
        """A saved activation of the last step, as an fp32 tensor."""
        c = self.cfg
        T, d = c.batch // self.world * c.seq, c.hidden
        cols = {"router_logits": c.experts}.get(name, d)
        out = torch.empty(T, cols, dtype=torch.float32, device=f"cuda:{self.device}")
        self._bind()
        _lib.call("catnn_moe_trainer_activation", self.handle, self.ACTIVATIONS[name], layer, C.c_void_p(out.data_ptr()))
        torch.cuda.synchronize(self.device)
        return out

    def set_graphs(self, enable=True):
        """Replay the step body as a CUDA graph (catnn_moe_trainer_set_graphs)."""
        self._bind()
        _lib.call("catnn_moe_trainer_set_graphs", self.handle, int(bool(enable)))

    def set_profile(self, enable=True):
        """Record device-clock stamps at the step's phase boundaries
        (catnn_moe_trainer_set_profile)."""
        self._bind()
        _lib.call("catnn_moe_trainer_set_profile", self.handle, int(bool(enable)))

    def timeline(self):
        """Phases of the last profiled step: [(name, milliseconds since the
        previous stamp)], from the device clock."""
        ns = (C.c_int64 * 64)()
        names = C.create_string_buffer(4096)
        count = C.c_int()
        self._bind()
        _lib.call("catnn_moe_trainer_timeline", self.handle, ns, 64, names, 4096, C.byref(count))
        labels = names.value.decode().split("\n")[:count.value]
        return [(labels[i], (ns[i] - ns[i - 1]) / 1e6) for i in range(1, count.value)]

    def check(self):
        self._bind()
        _lib.call("catnn_moe_trainer_check", self.handle)
