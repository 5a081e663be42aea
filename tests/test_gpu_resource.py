"""catnn_kernel_describe against the build's own record.

For each IR op the reference's resource::describe covers
(crates/catnn-compile/src/kernel/resource.rs:159-193), the query reports the
sm_100a kernel the op's launcher runs. Its registers and static shared
memory, read from the CUDA runtime, must equal what ptxas printed for that
kernel when the library was built (kernel_build_info.json); its code size is
the measured cubin of the kernel's source file (code_estimated = 0); the
launch geometry is the launcher's for the given shape.
"""
import json
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

from catnn_b200 import build as B  # noqa: E402
from catnn_b200 import ops  # noqa: E402
from catnn_b200.errors import Unsupported  # noqa: E402

SHAPES = {
    "linear": dict(rows=16384, width=3072, inner=1024),
    "matmul": dict(rows=4096, width=4096, inner=4096),
    "lm_head": dict(rows=16384, width=32000, inner=1024),
    "moe": dict(rows=33280, width=7168, inner=1024),
    "attention": dict(batch=8, seq=512, heads=8, head_dim=64, rows=4096, width=512),
    "gqa_attention": dict(batch=8, seq=2048, heads=16, head_dim=64, rows=16384, width=1024),
    "embedding": dict(rows=16384, width=1024),
    "rms_norm": dict(rows=16384, width=1024),
    "layer_norm": dict(rows=4096, width=512),
    "softmax": dict(rows=64, width=10),
    "cross_entropy": dict(rows=16384, width=32000),
    "relu": dict(rows=64, width=256),
    "gelu": dict(rows=4096, width=2048),
    "add": dict(rows=4096, width=512),
    "residual_add": dict(rows=16384, width=1024),
    "mul": dict(rows=64, width=256),
    "router": dict(rows=16384, width=8),
    "swiglu": dict(rows=33280, width=3584),
    "sgd": dict(rows=1, width=203530),
    "adam": dict(rows=1, width=437_000_000),
}


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("op", sorted(SHAPES))
def test_describe_matches_build_record(op, dtype):
    info = json.load(open(B.INFO))
    r = ops.kernel_describe(op, dtype, **SHAPES[op])
    rec = info["kernels"].get(r["kernel"])
    assert rec is not None, f"{op}: {r['kernel']} is not in the build record"
    assert rec["file"] == r["file"]
    assert r["registers_per_thread"] == rec["registers"], (op, r["registers_per_thread"], rec)
    assert r["static_smem_bytes"] == rec["static_smem"], (op, r["static_smem_bytes"], rec)
    assert r["code_estimated"] == 0 and r["code_bytes"] == info["cubin_bytes"][r["file"]]
    assert r["launch_arg_bytes"] > 0 and r["binary_version"] == 100
    threads = r["block"][0] * r["block"][1] * r["block"][2]
    assert 0 < threads <= r["max_threads_per_block"]
    assert all(g >= 1 for g in r["grid"])
    assert r["dynamic_smem_bytes"] + r["static_smem_bytes"] <= 232448


def test_describe_launch_geometry_follows_the_shape():
    props = torch.cuda.get_device_properties(0)
    big = ops.kernel_describe("lm_head", torch.bfloat16, rows=16384, width=32000, inner=1024)
    assert big["grid"][0] == props.multi_processor_count  # persistent: one CTA per SM
    small = ops.kernel_describe("linear", torch.bfloat16, rows=128, width=128, inner=64)
    assert small["grid"][0] == 1 and small["block"][0] == 320  # TMA, MMA and 8 epilogue warps
    fa = ops.kernel_describe("gqa_attention", torch.bfloat16, batch=8, seq=2048, heads=16, head_dim=64)
    assert fa["grid"] == [16, 8, 16] and "fa5" in fa["kernel"]  # heads, sequences, query tiles (slowest)
    rows = ops.kernel_describe("rms_norm", torch.float32, rows=300, width=256)
    assert rows["grid"][0] == 300


def test_describe_rejects_ops_without_a_kernel():
    with pytest.raises(Unsupported):
        ops.kernel_describe("mix", torch.bfloat16, rows=1, width=1)
    assert os.path.exists(B.INFO)
