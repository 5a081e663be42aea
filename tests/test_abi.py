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
