"""The allocation-free cross-entropy entry point (catnn_xent_fwdbwd_noalloc).

It is meant for callers that cannot allocate device memory mid-step; its
scratch is a fixed array inside the library. This file is collected last
so that a run stopping at the first failure has already run every other
test; it also passes alone in a fresh process. Both calls below go through
the C ABI and are compared with catnn_xent_fwdbwd on the same inputs.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from gpu_util import close_f32

pytestmark = pytest.mark.gpu


def _call(name, logits, targets, loss, d, check=1):
    from catnn_b200 import _lib, ops
    rows, vocab = logits.shape
    dt = 1 if logits.dtype == torch.bfloat16 else 0
    h = ops.context(logits.device).bind()
    _lib.call(name, h, C.c_void_p(logits.data_ptr()), C.c_void_p(targets.data_ptr()), rows, vocab,
              C.c_void_p(loss.data_ptr()), C.c_void_p(d.data_ptr()), dt, check)


def test_noalloc_matches_allocating_entry_point_twice():
    r = np.random.default_rng(0)
    for call, (rows, vocab, dtype) in enumerate([(3000, 2000, torch.float32), (1700, 32000, torch.bfloat16)]):
        z = torch.as_tensor(r.standard_normal((rows, vocab)).astype(np.float32) * 3).to("cuda", dtype)
        tg = torch.as_tensor(r.integers(0, vocab, rows).astype(np.int32)).cuda()
        l_ref, d_ref = torch.empty((), device="cuda"), torch.empty_like(z)
        l_na, d_na = torch.empty((), device="cuda"), torch.empty_like(z)
        _call("catnn_xent_fwdbwd", z, tg, l_ref, d_ref)
        _call("catnn_xent_fwdbwd_noalloc", z, tg, l_na, d_na)
        torch.cuda.synchronize()
        close_f32(l_na, l_ref.cpu().numpy(), what=f"loss, call {call}")
        close_f32(d_na.float(), d_ref.float().cpu().numpy(), what=f"dlogits, call {call}")


def test_noalloc_allocates_nothing_on_a_fresh_context():
    """On a context whose scratch buffer is empty (a fresh catnn_ctx), a call
    with 60000 rows would need 240 KB of scratch if it fell back to the
    context's allocator; after one warm call, further calls leave the
    device's free memory unchanged and still match the allocating entry
    point (run afterwards on the same context)."""
    from catnn_b200 import _lib, ops
    ctx = ops.Context(torch.cuda.current_device())  # fresh: no scratch yet
    try:
        r = np.random.default_rng(1)
        rows, vocab = 60000, 64
        z = torch.as_tensor(r.standard_normal((rows, vocab)).astype(np.float32)).cuda()
        tg = torch.as_tensor(r.integers(0, vocab, rows).astype(np.int32)).cuda()
        loss, d = torch.empty((), device="cuda"), torch.empty_like(z)
        h = ctx.bind()

        def call(name):
            _lib.call(name, h, C.c_void_p(z.data_ptr()), C.c_void_p(tg.data_ptr()), rows, vocab,
                      C.c_void_p(loss.data_ptr()), C.c_void_p(d.data_ptr()), 0, 1)
        call("catnn_xent_fwdbwd_noalloc")  # warm
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        for _ in range(3):
            call("catnn_xent_fwdbwd_noalloc")
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] == free0, "the allocation-free entry point changed device free memory"
        l_na, d_na = loss.clone(), d.clone()
        call("catnn_xent_fwdbwd")
        torch.cuda.synchronize()
        close_f32(l_na, loss.cpu().numpy(), what="loss on a fresh context")
        close_f32(d_na, d.cpu().numpy(), what="dlogits on a fresh context")
    finally:
        _lib.call("catnn_ctx_destroy", ctx.handle)


def test_noalloc_rejects_rows_over_its_limit_and_bad_targets():
    from catnn_b200.errors import ShapeMismatch
    z = torch.zeros(65537, 2, device="cuda")
    tg = torch.zeros(65537, dtype=torch.int32, device="cuda")
    with pytest.raises(ShapeMismatch, match="fixed limit"):
        _call("catnn_xent_fwdbwd_noalloc", z, tg, torch.empty((), device="cuda"), torch.empty_like(z))
    z = torch.zeros(4, 3, device="cuda")
    tg = torch.tensor([0, 1, 2, 3], dtype=torch.int32, device="cuda")
    with pytest.raises(ShapeMismatch):
        _call("catnn_xent_fwdbwd_noalloc", z, tg, torch.empty((), device="cuda"), torch.empty_like(z))
