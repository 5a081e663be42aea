"""Shared helpers for the GPU parity tests: seeded inputs, host<->device
moves and the tolerance checks written into every comparison.

Tolerances (from the parity contract):
- fp32 path: |gpu - ref| <= 1e-5·|ref| + 1e-5·max|ref|  (RTOL_F32 with a
  scale-aware floor: summation order differs from the reference's)
- bf16 path: |gpu - ref| <= 2e-2·|ref| + 1e-3·max(1, max|ref|)
- integer / index / permutation outputs and the bit-exact ops: equality.
Where a test also passes `exact` (the same algorithm in f64), an element
outside the band still passes if the GPU value is at least as close to the
exact value as the fp32 reference itself (long fp32 sums in the reference's
sequential order carry more rounding error than the band allows).
"""
import numpy as np
import torch

RTOL_F32 = 1e-5
RTOL_BF16, ATOL_BF16 = 2e-2, 1e-3


def dev(a, dtype=torch.float32):
    return torch.as_tensor(np.ascontiguousarray(a)).to(device="cuda", dtype=dtype).contiguous()


def host(t):
    return t.detach().float().cpu().numpy()


def close_f32(got, ref, rtol=RTOL_F32, floor=RTOL_F32, what="", exact=None, scale=None):
    got = host(got) if torch.is_tensor(got) else np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32)
    assert got.shape == ref.shape or got.size == ref.size, (what, got.shape, ref.shape)
    got = got.reshape(ref.shape)
    if scale is None:
        scale = float(np.max(np.abs(ref))) if ref.size else 0.0
    err = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    bound = rtol * np.abs(ref) + floor * max(scale, 1e-30)
    bad = err > bound
    if exact is not None:
        ex = np.asarray(exact, np.float64).reshape(ref.shape)
        bad &= np.abs(got - ex) > np.abs(ref.astype(np.float64) - ex) + bound
    assert not bad.any(), f"{what}: {int(bad.sum())}/{ref.size} out of tolerance; max err {err.max():.3e}, scale {scale:.3e}"


def close_bf16(got, ref, what="", atol=ATOL_BF16):
    """bf16 band: 2e-2·|ref| + atol·max(1, max|ref|).

    Composite blocks that round an intermediate to bf16 before a reduction
    (the SwiGLU activation feeding the W2 GEMM, then a weighted sum over the
    k expert slots that can cancel) pass a larger `atol`, stated at the call."""
    got = host(got) if torch.is_tensor(got) else np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32).reshape(got.shape)
    scale = max(1.0, float(np.max(np.abs(ref)))) if ref.size else 1.0
    err = np.abs(got.astype(np.float64) - ref)
    bound = RTOL_BF16 * np.abs(ref) + atol * scale
    bad = err > bound
    i = int(np.argmax(err - bound)) if ref.size else 0
    assert not bad.any(), (f"{what}: {int(bad.sum())}/{ref.size} out of tolerance; max err {err.max():.3e}, scale "
                           f"{scale:.3e}, worst got {got.reshape(-1)[i]:.5e} ref {ref.reshape(-1)[i]:.5e}")


U_BF16 = 2.0 ** -8  # unit roundoff of bf16 (8 significant bits, round to nearest)
U2_3 = U_BF16 ** 2 / 3  # variance of one bf16 rounding's relative error (uniform on [-u, u])
LAMBDA = 6.0  # standard deviations of a probabilistic rounding-error bound


def close_bf16_derived(got, ref, rounding_bound, what=""):
    """The bf16 band plus a derived bound: |got - ref| <= 2e-2·|ref| +
    1e-3·max(1, max|ref|) + rounding_bound, where rounding_bound is the
    effect, per element, of the bf16 roundings of intermediates that the
    tensor-core path stores and the fp32 reference keeps in fp32 (each test
    derives it from the exact intermediates and states which roundings it
    covers): LAMBDA standard deviations of the propagated first-order error,
    each rounding an independent relative error of variance u²/3 (the
    probabilistic rounding-error model; the worst-case sum of |terms| over a
    few hundred products is an order of magnitude looser)."""
    got = host(got) if torch.is_tensor(got) else np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float64).reshape(got.shape)
    rb = np.asarray(rounding_bound, np.float64).reshape(got.shape)
    scale = max(1.0, float(np.max(np.abs(ref)))) if ref.size else 1.0
    err = np.abs(got.astype(np.float64) - ref)
    bound = RTOL_BF16 * np.abs(ref) + ATOL_BF16 * scale + rb
    bad = err > bound
    i = int(np.argmax(err - bound)) if ref.size else 0
    assert not bad.any(), (f"{what}: {int(bad.sum())}/{ref.size} out of tolerance; max excess "
                           f"{float(np.max(err - bound)):.3e}, worst got {got.reshape(-1)[i]:.5e} ref "
                           f"{ref.reshape(-1)[i]:.5e} rounding bound {rb.reshape(-1)[i]:.3e}")


def rel_l2(got, ref):
    got = host(got) if torch.is_tensor(got) else np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float64).reshape(got.shape)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))


def bf16_round(a):
    """Round an fp32 array to bf16 and back (the inputs the bf16 path sees)."""
    return torch.as_tensor(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16).float().numpy()


def rng(seed):
    return np.random.default_rng(seed)
