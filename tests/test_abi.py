"""CPU checks of the drop-in boundary: libcatnn_b200.so loads without a GPU
and exports every entry point include/catnn_b200.h declares; the Python
binding covers the same set; the host-side operator mirror raises the
reference's errors before any kernel runs."""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER_DIR = os.path.join(ROOT, "include")


def declared_symbols():
    names = set()
    for f in os.listdir(HEADER_DIR):
        if f.endswith(".h"):
            src = open(os.path.join(HEADER_DIR, f)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names |= set(re.findall(r"\b(catnn_\w+)\s*\(", src))
    return names


@pytest.fixture(scope="module")
def libpath():
    from catnn_b200 import build
    return build.build()


def test_library_exports_every_declared_symbol(libpath):
    out = subprocess.run(["nm", "-D", "--defined-only", libpath], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (catnn_\w+)", out))
    missing = declared_symbols() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"


def test_library_loads_without_gpu(libpath):
    import catnn_b200
    lib = catnn_b200.load()
    assert lib.catnn_version() == 1
    assert lib.catnn_last_error() == b""


def test_binding_covers_header(libpath):
    from catnn_b200 import _lib
    assert declared_symbols() == set(_lib.SIGNATURES), (
        sorted(declared_symbols() ^ set(_lib.SIGNATURES)))


def test_ctx_create_reports_missing_device(libpath):
    """Without a GPU, context creation fails with a CUDA status and text, not a crash."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from catnn_b200 import ops
    from catnn_b200.errors import CatError
    with pytest.raises(CatError):
        ops.Context(0)


def test_ir_errors_match_reference():
    import torch
    from catnn_b200.errors import UnknownPort, Unlawful, Wiring, Unsupported
    from catnn_b200.ir import IrNode, OpenOp, adjoint_of, adjoint_needs_output, eval_gpu
    x = torch.zeros(2, 4)
    with pytest.raises(Unlawful):  # adjoint.rs:914-918
        adjoint_of(IrNode("r", OpenOp.router(4, 2)), [x], x, x)
    with pytest.raises(Wiring):  # adjoint.rs:768-770
        adjoint_of(IrNode("l", OpenOp.relu()), [], x, x)
    with pytest.raises(UnknownPort):  # mod.rs:55-59
        eval_gpu(IrNode("ln", OpenOp.layer_norm(10), {"beta": x}), [x])
    with pytest.raises(UnknownPort):
        adjoint_of(IrNode("rms", OpenOp.rms_norm(10)), [x], x, x)
    with pytest.raises(Unsupported):
        eval_gpu(IrNode("m", OpenOp.mix()), [x, x])
    assert adjoint_needs_output(OpenOp.softmax())
    assert not adjoint_needs_output(OpenOp.relu())


def test_packed_layout_matches_oracle_and_abi(libpath):
    """The packed parameter order crossing the ABI is the oracle's MixLayout."""
    import ctypes as C
    import torch
    from catnn_b200 import _lib
    from catnn_b200.train import MoeConfig, packed_layout
    from oracle import oracle as O
    for args in ((32, 32, 64, 2, 4, 2, 4, 2), (32000, 1024, 3584, 4, 16, 16, 8, 2), (1024, 256, 512, 2, 4, 4, 8, 2)):
        dt = torch.bfloat16 if args[1] % 64 == 0 else torch.float32  # bf16 path needs 64-multiples
        cfg = MoeConfig.make(*args, batch=1, seq=8, dtype=dt)
        ours = packed_layout(cfg)
        ref = O.MixCfg(*args).layout()
        for k in ("embed", "final_norm", "lm_head", "total", "layer0", "layer_stride", "rms_attn", "wq", "wk", "wv",
                  "wo", "rms_moe", "gate", "w1", "w3", "w2"):
            assert ours[k] == ref[k], (args, k, ours[k], ref[k])
        n = C.c_int64()
        _lib.call("catnn_moe_trainer_param_count", C.byref(cfg), C.byref(n))
        assert n.value == ref["total"]
    # config 5: about 435 M parameters (n_kv = 16)
    big = O.MixCfg(32000, 1024, 3584, 4, 16, 16, 8, 2).layout()["total"]
    assert 4.3e8 < big < 4.4e8


def test_build_records_kernel_resources():
    """The build's record behind catnn_kernel_describe: every source file has a
    measured cubin size, every kernel its -Xptxas -v registers, and the
    tensor-core GEMM and attention kernels fit the register file and spill
    at most a few bytes.

    The 64 K registers of an SM are four partitions of 16 K, one per warp
    scheduler, and a CTA's warps are spread over them: a 10-warp CTA (the
    GEMM, the attention backward) puts 3 warps on one partition, and so does
    a pair of 6-warp attention-forward CTAs, so each thread can have at most
    16384 / (3 · 32) -> 168 registers or the launch fails."""
    import json
    import os
    import catnn_b200.build as b
    b.build()
    info = json.load(open(b.INFO))
    srcs = {os.path.basename(s) for s in b.sources()} - {b.LAST}
    assert srcs <= set(info["cubin_bytes"]), srcs - set(info["cubin_bytes"])
    assert all(n > 0 for n in info["cubin_bytes"].values())
    ks = info["kernels"]
    assert len(ks) > 50
    gemm = [k for k in ks if "k_gemm_tc" in k]
    fa5 = [k for k in ks if ks[k]["file"] == "attention_fa5.cu"]
    assert gemm and fa5
    for name in gemm + fa5:
        assert 0 < ks[name]["registers"] <= 168 and ks[name]["spill_stores"] <= 8, (name, ks[name])
    inc = open(os.path.join(b.BUILD, "code_sizes.inc")).read()
    for f, n in info["cubin_bytes"].items():
        assert f'"{f}", {n}' in inc
