"""One rank of the multi-GPU parity check (run under torchrun by
tests/test_gpu_dist.py): the data-parallel + expert-parallel trainer on the
global batch, saving its loss, merged-view gradients and parameters."""
import argparse
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "cat-nn-compiler_b200"))
sys.path.insert(0, os.path.join(HERE, ".."))

from catnn_b200 import dist as D  # noqa: E402
from catnn_b200.train import MoeConfig, MoeTrainer, init_params  # noqa: E402

CONFIGS = {
    # fp32 path: vocab, hidden, mid, layers, heads, kv, experts, top_k, batch, seq
    # (SGD on the fp32 path: Adam's first step is lr·sign(g), which turns a
    # last-bit difference of a near-zero gradient into a full lr step)
    "f32": dict(args=(512, 64, 96, 2, 4, 2, 8, 2, 4, 32), dtype=torch.float32, opt="sgd", lr=5e-2),
    # (Adam with eps 1e-3 for the comparison: a gradient far below eps moves its
    # parameter in proportion to it, not by ±lr as with eps 1e-8, so rounding
    # noise in near-zero gradients does not become full-size steps)
    "bf16": dict(args=(2048, 256, 512, 2, 4, 4, 8, 2, 4, 128), dtype=torch.bfloat16, opt="adam", lr=1e-3,
                 adam_eps=1e-3),
    # config 5 at its full widths (the benchmark's model): only the losses are
    # saved (the packed vectors would be 1.7 GB each)
    "config5": dict(args=(32000, 1024, 3584, 4, 16, 16, 8, 2, 8, 2048), dtype=torch.bfloat16, opt="adam", lr=1e-4,
                    light=True),
}


def params(cfg, name, device):
    """init_params for the small configs; for config 5 the same draw on the
    device (torch's generator, seed 3) on every rank and in the reference."""
    if not CONFIGS[name].get("light"):
        return init_params(cfg, seed=3)
    from catnn_b200.train import packed_layout
    L = packed_layout(cfg)
    g = torch.Generator(device=device).manual_seed(3)
    P = torch.randn(L["total"], generator=g, device=device) * 0.02
    h = cfg.hidden
    for l in range(cfg.layers):
        base = L["layer0"] + l * L["layer_stride"]
        P[base + L["rms_attn"]:base + L["rms_attn"] + h] = 1.0
        P[base + L["rms_moe"]:base + L["rms_moe"] + h] = 1.0
    P[L["final_norm"]:L["final_norm"] + h] = 1.0
    return P


def config(name):
    c = CONFIGS[name]
    return MoeConfig.make(*c["args"], rope_theta=1e4, dtype=c["dtype"], optimizer=c["opt"], lr=c["lr"],
                          adam_eps=c.get("adam_eps", 1e-8))


def tokens(cfg, seed=9):
    return np.random.default_rng(seed).integers(0, cfg.vocab, cfg.batch * cfg.seq).astype(np.uint32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="f32")
    ap.add_argument("--out", required=True)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--graphs", action="store_true", help="replay the step as a CUDA graph")
    a = ap.parse_args()
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    try:
        comm = D.Comm.from_process_group(local)
        cfg = config(a.config)
        tr = MoeTrainer(cfg, local, comm=comm)
        tr.set_params(params(cfg, a.config, f"cuda:{local}"))
        light = CONFIGS[a.config].get("light", False)
        if a.graphs:
            # the first update step runs eagerly, the second is captured, later ones replay
            tr.set_graphs(True)
        tok = torch.as_tensor(tokens(cfg).astype(np.int32)).to(f"cuda:{local}")
        loss = torch.zeros(1, device=f"cuda:{local}")
        tr.step(tok, update=False, loss_out=loss)
        tr.check()
        out = {"loss0": loss.cpu().numpy()}
        if not light:
            out["grads0"] = tr.grads().cpu().numpy()
        losses = []
        for _ in range(a.steps):
            tr.step(tok, update=True, loss_out=loss)
            losses.append(float(loss.item()))
        tr.check()
        out["losses"] = np.array(losses, np.float32)
        if not light:
            out["params"] = tr.params().cpu().numpy()
            out["x_last"] = tr.activation("x_last").cpu().numpy()
        np.savez(os.path.join(a.out, f"rank{rank}.npz"), **out)
        if a.graphs:
            # replays of the captured steps: every device wait must still hold
            for upd in (True, True, False, False, True):
                tr.step(tok, update=upd, loss_out=loss)
            tr.check()
            assert np.isfinite(float(loss.item()))
        torch.cuda.synchronize()
        tr.close()
        comm.close()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
