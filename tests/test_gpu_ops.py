"""Per-operator parity of the CUDA kernels (through the C ABI) against the
oracle on identical seeded inputs. fp32 path at rtol 1e-5; the ops the
reference computes with one rounding per step (add, mul, SGD, Adam,
embedding gather/scatter, router indices, permutations, checksums) are
compared bit for bit."""
import numpy as np
import pytest
import torch

from gpu_util import LAMBDA, U2_3, bf16_round, close_bf16, close_bf16_derived, close_f32, dev, host, rng
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _lib():
    import catnn_b200
    catnn_b200.load()


from catnn_b200 import ops  # noqa: E402
from catnn_b200.errors import ShapeMismatch  # noqa: E402


@pytest.mark.parametrize("m,k,n", [(64, 784, 256), (64, 256, 10), (7, 13, 5), (1, 1, 1), (130, 257, 129)])
def test_linear_fwd_bwd_f32(m, k, n):
    r = rng(m * 1000 + n)
    x = r.standard_normal((m, k)).astype(np.float32)
    w = (r.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32)
    b = r.standard_normal(n).astype(np.float32)
    dy = r.standard_normal((m, n)).astype(np.float32)
    close_f32(ops.linear(dev(x), dev(w), dev(b)), O.linear(x, w, b), what="linear")
    close_f32(ops.linear(dev(x), dev(w), dev(b), act="relu"), O.relu(O.linear(x, w, b)), what="linear+relu")
    gx, gw, gb = ops.linear_backward(dev(x), dev(w), dev(dy))
    rx, rw, rb = O.linear_backward(x, w, dy)
    close_f32(gx, rx, what="dx")
    close_f32(gw, rw, what="dw")
    close_f32(gb, rb, what="db")


@pytest.mark.parametrize("T,d,E", [(16384, 1024, 8), (1000, 260, 5), (300, 64, 16), (257, 96, 32), (4096, 33, 3)])
def test_router_shaped_gemm_f32(T, d, E):
    """The MoE gate's three fp32 GEMMs at router shapes (N or K = experts):
    logits = x·gate, dx += dlog·gateᵀ, dgate = xᵀ·dlog — the narrow-N,
    short-K and split-K kernels — against the oracle's f32 linear with an
    exact f64 fallback (rtol 1e-5 band)."""
    r = rng(T + d + E)
    x = r.standard_normal((T, d)).astype(np.float32)
    gate = (r.standard_normal((d, E)) / np.sqrt(d)).astype(np.float32)
    dlog = r.standard_normal((T, E)).astype(np.float32)
    dx0 = r.standard_normal((T, d)).astype(np.float32)
    X, G, DL = dev(x), dev(gate), dev(dlog)
    lg = ops.gemm(X, G)
    close_f32(lg, O.linear(x, gate), what="logits", exact=x.astype(np.float64) @ gate)
    lgt = ops.gemm(X, dev(np.ascontiguousarray(gate.T)), trans_b=True)
    close_f32(lgt, O.linear(x, gate), what="logits (gate stored [E, d])", exact=x.astype(np.float64) @ gate)
    dx = dev(dx0)
    ops.gemm(DL, G, trans_b=True, out=dx, accumulate=True)
    ex = dx0 + dlog.astype(np.float64) @ gate.T.astype(np.float64)
    close_f32(dx, ex.astype(np.float32), what="dx += dlog·gateᵀ", exact=ex)
    dg = ops.gemm(X, DL, trans_a=True)
    exg = x.T.astype(np.float64) @ dlog
    close_f32(dg, O.linear(np.ascontiguousarray(x.T), dlog), what="dgate", exact=exg)
    dg2 = ops.gemm(X, DL, trans_a=True)
    assert torch.equal(dg, dg2), "split-K weight gradient must be deterministic"


def test_linear_kat_identity():
    y = ops.linear(dev([[1.0, 2.0]]), dev([[1.0, 0.0], [0.0, 1.0]]))
    assert host(y).tolist() == [[1.0, 2.0]]


def test_elementwise():
    r = rng(1)
    x = r.standard_normal(10007).astype(np.float32) * 3
    dy = r.standard_normal(10007).astype(np.float32)
    assert np.array_equal(host(ops.relu(dev(x))), O.relu(x))
    assert np.array_equal(host(ops.relu_backward(dev(x), dev(dy))), O.relu_backward(x, dy))
    close_f32(ops.gelu(dev(x)), O.gelu(x), what="gelu")
    close_f32(ops.gelu_backward(dev(x), dev(dy)), O.gelu_backward(x, dy), what="gelu'")
    assert np.array_equal(host(ops.add(dev(x), dev(dy))), O.add(x, dy))
    assert np.array_equal(host(ops.mul(dev(x), dev(dy))), O.mul(x, dy))
    a = x.reshape(-1, 1).repeat(4, 1)[:1000].reshape(250, 16)
    bias = dy[:16]
    assert np.array_equal(host(ops.add(dev(a), dev(bias))), O.add(a, bias))
    with pytest.raises(ShapeMismatch):
        ops.add(dev(a), dev(dy[:7]))
    # reference KATs
    assert host(ops.relu(dev([-1.0, 0.0, 2.0, -0.5]))).tolist() == [0.0, 0.0, 2.0, 0.0]
    assert host(ops.relu_backward(dev([-1.0, 2.0, 0.0]), dev([1.0, 1.0, 1.0]))).tolist() == [0.0, 1.0, 0.0]


@pytest.mark.parametrize("rows,last", [(64, 10), (33, 1024), (4, 32000), (3, 1)])
def test_softmax_and_ce(rows, last):
    r = rng(rows + last)
    z = (r.standard_normal((rows, last)) * 4).astype(np.float32)
    close_f32(ops.softmax_last(dev(z)), O.softmax_last(z), what="softmax", exact=O.softmax_last(z, f64=True))
    y = O.softmax_last(z)
    dy = r.standard_normal((rows, last)).astype(np.float32)
    close_f32(ops.softmax_backward(dev(y), dev(dy)), O.softmax_backward(y, dy), what="softmax'",
              exact=O.softmax_backward(y, dy, f64=True))
    tg = r.integers(0, last, rows)
    loss, d = ops.cross_entropy(dev(z), dev(tg, torch.int32))
    rl, rd = O.cross_entropy(z, tg)
    rl64, rd64 = O.cross_entropy(z, tg, f64=True)
    close_f32(loss, np.float32(rl), what="ce loss", exact=rl64)
    close_f32(d, rd, what="dlogits", exact=rd64)


def test_ce_rejects_bad_target():
    with pytest.raises(ShapeMismatch):
        ops.cross_entropy(dev(np.zeros((2, 3))), dev([0, 3], torch.int32))


def test_softmax_grad_row_sum_kat():
    y = ops.softmax_last(dev([[1.0, 2.0, 3.0]]))
    dx = ops.softmax_backward(y, dev([[1.0, 1.0, 1.0]]))
    assert abs(float(host(dx).sum())) < 1e-5


def test_mse():
    r = rng(3)
    p, t = r.standard_normal(37).astype(np.float32), r.standard_normal(37).astype(np.float32)
    loss, d = ops.mse_loss(dev(p), dev(t))
    rl, rd = O.mse_loss(p, t)
    close_f32(loss, np.float32(rl), what="mse")
    close_f32(d, rd, what="mse d")


@pytest.mark.parametrize("rows,last", [(16, 512), (5, 33), (300, 256), (2, 4096)])
def test_norms(rows, last):
    r = rng(rows * 7 + last)
    x = (r.standard_normal((rows, last)) * 2 + 0.5).astype(np.float32)
    g = r.standard_normal(last).astype(np.float32)
    b = r.standard_normal(last).astype(np.float32)
    dy = r.standard_normal((rows, last)).astype(np.float32)
    close_f32(ops.layer_norm(dev(x), dev(g), dev(b)), O.layer_norm(x, g, b), what="ln")
    gx, gg, gb = ops.layer_norm_backward(dev(x), dev(g), dev(dy))
    rx, rg, rb = O.layer_norm_backward(x, g, dy)
    ex, eg, eb = O.layer_norm_backward(x, g, dy, f64=True)
    close_f32(gx, rx, what="ln dx", exact=ex)
    close_f32(gg, rg, what="ln dgamma", exact=eg)
    close_f32(gb, rb, what="ln dbeta", exact=eb)
    close_f32(ops.rmsnorm(dev(x), dev(g)), O.rmsnorm(x, g), what="rms", exact=O.rmsnorm(x, g, f64=True))
    gx, gw = ops.rmsnorm_backward(dev(x), dev(g), dev(dy))
    rx, rw = O.rmsnorm_backward(x, g, dy)
    ex, ew = O.rmsnorm_backward(x, g, dy, f64=True)
    close_f32(gx, rx, what="rms dx", exact=ex)
    close_f32(gw, rw, what="rms dw", exact=ew)


def test_embedding_exact():
    r = rng(5)
    table = r.standard_normal((1024, 256)).astype(np.float32)
    ids = r.integers(0, 1024, 1000).astype(np.uint32)
    ids[:50] = 7  # heavy repeats
    y = ops.embedding(dev(ids, torch.int32), dev(table))
    assert np.array_equal(host(y), O.embedding(ids, table))
    dy = r.standard_normal((1000, 256)).astype(np.float32)
    dw = ops.embedding_backward(dev(ids, torch.int32), dev(dy), 1024)
    assert np.array_equal(host(dw), O.embedding_backward(ids, dy, 1024)), "scatter-add must be bit-exact (t order)"
    with pytest.raises(ShapeMismatch):
        ops.embedding(dev([0, 1024], torch.int32), dev(table))


def test_rope_matches_reference_angles():
    r = rng(6)
    q = r.standard_normal((2, 37, 3, 64)).astype(np.float32)
    for theta in (1e4, 1e6):
        g = ops.rope(dev(q).clone(), theta)
        close_f32(g, O.rope(q, theta), rtol=1e-6, floor=1e-6, what="rope")
        back = ops.rope(g, theta, inverse=True)
        close_f32(back, O.rope(O.rope(q, theta), -theta), rtol=1e-6, floor=1e-6, what="rope^-1")


@pytest.mark.parametrize("b,s,h,kv,hd,window", [(1, 6, 2, 1, 4, 4), (2, 33, 4, 2, 8, 8), (2, 130, 4, 4, 64, None),
                                                 (1, 70, 2, 2, 128, None)])
def test_gqa_fwd_bwd(b, s, h, kv, hd, window):
    r = rng(s * 10 + hd)
    d = h * hd
    x = r.standard_normal((b, s, d)).astype(np.float32)
    wq = (r.standard_normal((d, h * hd)) / np.sqrt(d)).astype(np.float32)
    wk = (r.standard_normal((d, kv * hd)) / np.sqrt(d)).astype(np.float32)
    wv = (r.standard_normal((d, kv * hd)) / np.sqrt(d)).astype(np.float32)
    wo = (r.standard_normal((h * hd, d)) / np.sqrt(d)).astype(np.float32)
    dy = r.standard_normal((b, s, d)).astype(np.float32)
    y = ops.gqa(*(dev(a) for a in (x, wq, wk, wv, wo)), h, kv, 1e4, window)
    close_f32(y, O.gqa(x, wq, wk, wv, wo, h, kv, 1e4, window), what="gqa",
              exact=O.gqa(x, wq, wk, wv, wo, h, kv, 1e4, window, f64=True))
    got = ops.gqa_backward(*(dev(a) for a in (x, wq, wk, wv, wo, dy)), h, kv, 1e4, window)
    ref = O.gqa_backward(x, wq, wk, wv, wo, dy, h, kv, 1e4, window)
    ex = O.gqa_backward(x, wq, wk, wv, wo, dy, h, kv, 1e4, window, f64=True)
    for name, g, rr, ee in zip(("dx", "dwq", "dwk", "dwv", "dwo"), got, ref, ex):
        close_f32(g, rr, what=f"gqa {name}", exact=ee)


@pytest.mark.parametrize("causal", [False, True])
def test_mha_fwd_bwd(causal):
    r = rng(11 + causal)
    b, s, d, h = 2, 40, 64, 4
    x = r.standard_normal((b, s, d)).astype(np.float32)
    ws = [(r.standard_normal((d, d)) * 0.1).astype(np.float32) for _ in range(4)]
    dy = r.standard_normal((b, s, d)).astype(np.float32)
    close_f32(ops.attention(dev(x), *(dev(w) for w in ws), h, causal), O.attention(x, *ws, h, causal), what="mha",
              exact=O.attention(x, *ws, h, causal, f64=True))
    got = ops.attention_backward(dev(x), *(dev(w) for w in ws), dev(dy), h, causal)
    ref = O.attention_backward(x, *ws, dy, h, causal)
    ex = O.attention_backward(x, *ws, dy, h, causal, f64=True)
    for name, g, rr, ee in zip(("dx", "dwq", "dwk", "dwv", "dwo"), got, ref, ex):
        close_f32(g, rr, what=f"mha {name}", exact=ee)


def test_router_topk_bit_exact():
    r = rng(12)
    logits = r.standard_normal((4096, 8)).astype(np.float32)
    logits[:64] = np.round(logits[:64])  # many ties
    logits[64:70] = 0.5
    idx, w = ops.router_topk(dev(logits), 2)
    ri = np.stack([O.topk_softmax(row, 2)[0] for row in logits])
    rw = np.stack([O.topk_softmax(row, 2)[1] for row in logits])
    assert np.array_equal(host(idx).astype(np.int64), ri)
    close_f32(w, rw, rtol=1e-6, floor=1e-7, what="router w")
    idx, w = ops.router_topk(dev([[1.0, 3.0, 0.0, 2.0]]), 2)
    assert host(idx).astype(int).tolist() == [[1, 3]]
    assert abs(float(host(w).sum()) - 1.0) < 1e-6


@pytest.mark.parametrize("align,T,E", [(1, 1000, 8), (128, 1000, 8), (1, 16384, 8), (128, 16384, 8), (128, 7000, 32)])
def test_permute_map_stable(align, T, E):
    """Counting-sort permutation (single-CTA below 4096 pairs, multi-CTA
    histogram / scan / stable place above) against numpy's stable sort."""
    r = rng(13 + T)
    k = 2
    logits = r.standard_normal((T, E)).astype(np.float32)
    idx, _ = ops.router_topk(dev(logits), k)
    counts, offsets, row_of, src_of = ops.moe_permute_map(idx, E, align)
    idx_h = host(idx).astype(np.int64).reshape(-1)
    order = np.argsort(idx_h, kind="stable")
    cnt = np.bincount(idx_h, minlength=E)
    assert host(counts).astype(int).tolist() == cnt.tolist()
    off = np.zeros(E + 1, np.int64)
    for e in range(E):
        off[e + 1] = off[e] + -(-cnt[e] // align) * align
    assert host(offsets).astype(int).tolist() == off.tolist()
    src = src_of.cpu().numpy()
    rows = []
    for e in range(E):
        blk = src[off[e]:off[e + 1]]
        rows.extend(blk[:cnt[e]].tolist())
        assert (blk[cnt[e]:] == -1).all()
    assert rows == order.tolist(), "rows of an expert must be its pairs in token order"
    ro = row_of.cpu().numpy()
    assert (src[ro] == np.arange(T * k)).all()


def test_swiglu_fwd_bwd():
    r = rng(14)
    x = r.standard_normal((9, 32)).astype(np.float32)
    w1, w3 = (r.standard_normal((32, 64)) * 0.2).astype(np.float32), (r.standard_normal((32, 64)) * 0.2).astype(np.float32)
    w2 = (r.standard_normal((64, 32)) * 0.2).astype(np.float32)
    dy = r.standard_normal((9, 32)).astype(np.float32)
    close_f32(ops.swiglu(*(dev(a) for a in (x, w1, w3, w2))), O.swiglu(x, w1, w3, w2), what="swiglu",
              exact=O.swiglu(x, w1, w3, w2, f64=True))
    got = ops.swiglu_backward(*(dev(a) for a in (x, w1, w3, w2, dy)))
    ref = O.swiglu_backward(x, w1, w3, w2, dy)
    ex = O.swiglu_backward(x, w1, w3, w2, dy, f64=True)
    for name, g, rr, ee in zip(("dx", "dw1", "dw3", "dw2"), got, ref, ex):
        close_f32(g, rr, what=f"swiglu {name}", exact=ee)


@pytest.mark.parametrize("T,H,F,E,k", [(64, 32, 64, 4, 2), (300, 64, 96, 8, 2)])
def test_moe_fwd_bwd_f32(T, H, F, E, k):
    r = rng(T + H)
    x = r.standard_normal((T, H)).astype(np.float32)
    gate = r.standard_normal((H, E)).astype(np.float32)
    w1s = (r.standard_normal((E, H, F)) * 0.1).astype(np.float32)
    w3s = (r.standard_normal((E, H, F)) * 0.1).astype(np.float32)
    w2s = (r.standard_normal((E, F, H)) * 0.1).astype(np.float32)
    dy = r.standard_normal((T, H)).astype(np.float32)
    close_f32(ops.moe(*(dev(a) for a in (x, gate, w1s, w3s, w2s)), k), O.moe(x, gate, w1s, w3s, w2s, k), what="moe",
              exact=O.moe(x, gate, w1s, w3s, w2s, k, f64=True))
    got = ops.moe_backward(*(dev(a) for a in (x, gate, w1s, w3s, w2s, dy)), k)
    ref = O.moe_backward(x, gate, w1s, w3s, w2s, dy, k)
    ex = O.moe_backward(x, gate, w1s, w3s, w2s, dy, k, f64=True)
    for name, g, rr, ee in zip(("dx", "dgate", "dw1", "dw3", "dw2"), got, ref, ex):
        close_f32(g, rr, what=f"moe {name}", exact=ee)


def test_optimizers_bit_exact():
    r = rng(15)
    p = r.standard_normal(100003).astype(np.float32)
    g = r.standard_normal(100003).astype(np.float32)
    pd = dev(p)
    ops.sgd_(pd, dev(g), 0.05)
    assert np.array_equal(host(pd), O.sgd_put(p, g, 0.05))
    assert host(ops.sgd_(dev([1.0, 2.0]), dev([1.0, -1.0]), 0.5)).tolist() == [0.5, 2.5]
    m, v = np.zeros_like(p), np.zeros_like(p)
    pd, md, vd = dev(p), dev(m), dev(v)
    rp = p
    for t in range(1, 4):
        gt = (g * t).astype(np.float32)
        ops.adam_(pd, dev(gt), md, vd, t, 1e-3)
        rp, m, v, tt = O.adam_put(rp, gt, m, v, t - 1, 1e-3)
        assert tt == t
    assert np.array_equal(host(pd), rp), "Adam must match optim.rs bit for bit"
    assert np.array_equal(host(md), m) and np.array_equal(host(vd), v)


def test_lm_head():
    r = rng(16)
    x = r.standard_normal((50, 64)).astype(np.float32)
    w = (r.standard_normal((300, 64)) * 0.1).astype(np.float32)
    dy = r.standard_normal((50, 300)).astype(np.float32)
    close_f32(ops.lm_head(dev(x), dev(w)), O.lm_head(x, w), what="lm_head")
    gx, gw = ops.lm_head_backward(dev(x), dev(w), dev(dy))
    rx, rw = O.lm_head_backward(x, w, dy)
    close_f32(gx, rx, what="lm dx")
    close_f32(gw, rw, what="lm dw")


def test_checksum_matches_reference():
    x = O.lcg(4097, 3)
    assert ops.checksum(dev(x)) == O.checksum(x)


def test_mlp_step_matches_oracle():
    r = rng(0)
    w1 = r.uniform(-np.sqrt(6 / 1040), np.sqrt(6 / 1040), (784, 256)).astype(np.float32)
    w2 = r.uniform(-np.sqrt(6 / 266), np.sqrt(6 / 266), (256, 10)).astype(np.float32)
    b1, b2 = np.zeros(256, np.float32), np.zeros(10, np.float32)
    x = r.standard_normal((64, 784)).astype(np.float32)
    lab = r.integers(0, 10, 64)
    loss, *grads = ops.mlp_step(dev(w1), dev(b1), dev(w2), dev(b2), dev(x), labels=dev(lab, torch.int32))
    rl, *rg = O.mlp_step(w1, b1, w2, b2, x, labels=lab)
    close_f32(loss, np.float32(rl), what="mlp loss")
    for name, g, rr in zip(("dw1", "db1", "dw2", "db2"), grads, rg):
        close_f32(g, rr, what=f"mlp {name}")


# ------------------------------------------------------------------ bf16 / tcgen05
@pytest.mark.parametrize("ta,tb", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("M,N,K", [(256, 512, 256), (200, 300, 136), (1024, 1024, 1024), (128, 64, 64)])
def test_gemm_bf16_tensor_core(ta, tb, M, N, K):
    r = rng(M + N + K + 2 * ta + tb)
    a = bf16_round((r.standard_normal((K, M) if ta else (M, K)) / np.sqrt(K)).astype(np.float32))
    b = bf16_round(r.standard_normal((N, K) if tb else (K, N)).astype(np.float32))
    ref = (a.T if ta else a).astype(np.float64) @ (b.T if tb else b).astype(np.float64)
    for out_dtype in (torch.float32, torch.bfloat16):
        c = ops.gemm(dev(a, torch.bfloat16), dev(b, torch.bfloat16), ta, tb, out_dtype=out_dtype)
        close_bf16(c, ref.astype(np.float32), what=f"gemm ta={ta} tb={tb} {out_dtype}")


def test_gemm_bf16_bias_act_accumulate():
    r = rng(21)
    M, N, K = 384, 256, 192
    a = bf16_round(r.standard_normal((M, K)).astype(np.float32) / 8)
    b = bf16_round(r.standard_normal((K, N)).astype(np.float32))
    bias = r.standard_normal(N).astype(np.float32)
    ref = a.astype(np.float64) @ b + bias
    c = ops.gemm(dev(a, torch.bfloat16), dev(b, torch.bfloat16), out_dtype=torch.float32, bias=dev(bias), act="relu")
    close_bf16(c, np.maximum(ref, 0).astype(np.float32), what="bias+relu")
    c0 = dev(r.standard_normal((M, N)).astype(np.float32))
    ref2 = host(c0) + a.astype(np.float64) @ b
    ops.gemm(dev(a, torch.bfloat16), dev(b, torch.bfloat16), out=c0, accumulate=True)
    close_bf16(c0, ref2.astype(np.float32), what="accumulate")


@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True)])
def test_gemm_bf16_split_k(ta, tb):
    """Few output tiles over a long K: the K range is cut into slices whose
    fp32 partials are added in slice order (bit-identical run to run), with
    bias, activation and accumulate applied once after the sum."""
    r = rng(31 + 2 * ta + tb)
    M, N, K = 256, 384, 4096
    a = bf16_round((r.standard_normal((K, M) if ta else (M, K)) / np.sqrt(K)).astype(np.float32))
    b = bf16_round(r.standard_normal((N, K) if tb else (K, N)).astype(np.float32))
    bias = r.standard_normal(N).astype(np.float32)
    ref = (a.T if ta else a).astype(np.float64) @ (b.T if tb else b).astype(np.float64) + bias
    A, B = dev(a, torch.bfloat16), dev(b, torch.bfloat16)
    c1 = ops.gemm(A, B, ta, tb, out_dtype=torch.float32, bias=dev(bias), act="relu")
    close_bf16(c1, np.maximum(ref, 0).astype(np.float32), what="split-K bias+relu")
    c2 = ops.gemm(A, B, ta, tb, out_dtype=torch.float32, bias=dev(bias), act="relu")
    assert torch.equal(c1, c2)
    c0 = dev(r.standard_normal((M, N)).astype(np.float32))
    ref2 = host(c0) + (ref - bias)
    ops.gemm(A, B, ta, tb, out=c0, accumulate=True)
    close_bf16(c0, ref2.astype(np.float32), what="split-K accumulate")
    cb = ops.gemm(A, B, ta, tb, out_dtype=torch.bfloat16)
    close_bf16(cb, (ref - bias).astype(np.float32), what="split-K bf16 out")


@pytest.mark.parametrize("K", [4096, 8192])
def test_gemm_config2_fwd_bwd_bf16(K):
    """Config 2 at its large sizes: C = A·B, dA = dC·Bᵀ, dB = Aᵀ·dC with
    M = N = K, A and B N(0,1)/sqrt(K), dC N(0,1) (seed 1), bf16 operands on
    the tcgen05 path with fp32 accumulation and fp32 outputs, against the fp32
    CUDA-core GEMM of the same (bf16-valued) operands at the bf16 band."""
    g = torch.Generator(device="cuda").manual_seed(1)
    A = (torch.randn(K, K, generator=g, device="cuda") / K ** 0.5).to(torch.bfloat16)
    B = (torch.randn(K, K, generator=g, device="cuda") / K ** 0.5).to(torch.bfloat16)
    dC = torch.randn(K, K, generator=g, device="cuda").to(torch.bfloat16)
    A32, B32, dC32 = A.float(), B.float(), dC.float()
    for what, got, ref in (("C", ops.gemm(A, B, out_dtype=torch.float32), ops.gemm(A32, B32)),
                           ("dA", ops.gemm(dC, B, trans_b=True, out_dtype=torch.float32), ops.gemm(dC32, B32, trans_b=True)),
                           ("dB", ops.gemm(A, dC, trans_a=True, out_dtype=torch.float32), ops.gemm(A32, dC32, trans_a=True))):
        # a sampled block keeps the host comparison short; the row/column
        # offsets cross tile and split boundaries
        rows, cols = slice(K // 2 - 700, K // 2 + 700), slice(K // 3 - 500, K // 3 + 500)
        close_bf16(got[rows, cols], host(ref[rows, cols]), what=f"config2 {what} K={K}")
        assert float((got - ref).abs().max()) <= 2e-2 * float(ref.abs().max()), what


U_TF32 = 2.0 ** -10  # the tensor cores read the top 19 bits of an fp32 operand


def tf32_bound(a, b, ta, tb):
    """Rigorous error bound of a TF32 product against the exact one: each
    operand loses at most a relative 2^-10 to the 10-bit mantissa and the
    fp32 accumulation of K terms at most K·2^-24, all of Σ_k |a_ik||b_kj|."""
    A = np.abs(a.T if ta else a).astype(np.float64)
    B = np.abs(b.T if tb else b).astype(np.float64)
    K = A.shape[1]
    return (2 * U_TF32 + U_TF32 ** 2 + K * 2.0 ** -24) * (A @ B)


@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True), (True, True)])
@pytest.mark.parametrize("M,N,K", [(512, 384, 1024), (200, 136, 100), (128, 256, 4096)])
def test_gemm_tf32_tensor_core(ta, tb, M, N, K):
    """fp32 operands multiplied as TF32 (kind::tf32) with fp32 accumulation:
    inside the rigorous TF32 bound and the bf16 contract band, and closer to
    the exact product than bf16 operands would be."""
    r = rng(7 * M + N + K + 2 * ta + tb)
    a = (r.standard_normal((K, M) if ta else (M, K)) / np.sqrt(K)).astype(np.float32)
    b = r.standard_normal((N, K) if tb else (K, N)).astype(np.float32)
    ref = (a.T if ta else a).astype(np.float64) @ (b.T if tb else b).astype(np.float64)
    got = host(ops.gemm(dev(a), dev(b), ta, tb, tf32=True))
    err = np.abs(got - ref)
    bound = tf32_bound(a, b, ta, tb)
    assert (err <= bound).all(), f"tf32 ta={ta} tb={tb}: worst excess {float((err - bound).max()):.3g}"
    close_bf16(got, ref.astype(np.float32), what=f"tf32 ta={ta} tb={tb}")
    bf = host(ops.gemm(dev(a, torch.bfloat16), dev(b, torch.bfloat16), ta, tb, out_dtype=torch.float32))
    assert np.sqrt(np.mean(err ** 2)) < 0.5 * np.sqrt(np.mean((bf - ref) ** 2))


def test_gemm_tf32_bias_act_accumulate_and_small_shapes():
    r = rng(77)
    M, N, K = 384, 256, 192
    a = r.standard_normal((M, K)).astype(np.float32) / 8
    b = r.standard_normal((K, N)).astype(np.float32)
    bias = r.standard_normal(N).astype(np.float32)
    ref = a.astype(np.float64) @ b + bias
    bound = tf32_bound(a, b, False, False)
    c = host(ops.gemm(dev(a), dev(b), bias=dev(bias), act="relu", tf32=True))
    assert (np.abs(c - np.maximum(ref, 0)) <= bound).all()
    c0 = dev(r.standard_normal((M, N)).astype(np.float32))
    ref2 = host(c0) + (ref - bias)
    ops.gemm(dev(a), dev(b), out=c0, accumulate=True, tf32=True)
    assert (np.abs(host(c0) - ref2) <= bound + 1e-6 * np.abs(ref2)).all()
    cb = ops.gemm(dev(a), dev(b), out_dtype=torch.bfloat16, tf32=True)
    close_bf16(cb, (ref - bias).astype(np.float32), what="tf32 bf16 out")
    # N < 16 and an unaligned leading dimension take the fp32 CUDA-core GEMM
    for m, k, n in ((64, 256, 10), (7, 13, 5)):
        x = r.standard_normal((m, k)).astype(np.float32)
        w = r.standard_normal((k, n)).astype(np.float32)
        close_f32(ops.gemm(dev(x), dev(w), tf32=True), O.matmul_seq(x, w), what=f"tf32 small {m}x{k}x{n}")
    with pytest.raises(Exception):
        ops.gemm(dev(a, torch.bfloat16), dev(b, torch.bfloat16), tf32=True)


@pytest.mark.parametrize("tb", [False, True])
def test_grouped_gemm_bf16_split_k(tb):
    """Two experts of 256 rows against K = 4096: M-grouped tiles cut in K."""
    r = rng(41 + tb)
    E, R, N, K = 2, 256, 512, 4096
    a = bf16_round((r.standard_normal((E * R, K)) / np.sqrt(K)).astype(np.float32))
    b = bf16_round(r.standard_normal((E, N, K) if tb else (E, K, N)).astype(np.float32))
    off = torch.tensor([0, R, 2 * R], dtype=torch.int32, device="cuda")
    out = ops.grouped_gemm(dev(a, torch.bfloat16), dev(b, torch.bfloat16), off, trans_b=tb, out_dtype=torch.float32)
    for g in range(E):
        bg = b[g].T if tb else b[g]
        ref = a[g * R:(g + 1) * R].astype(np.float64) @ bg.astype(np.float64)
        close_bf16(out[g * R:(g + 1) * R], ref.astype(np.float32), what=f"grouped split-K expert {g}")


@pytest.mark.parametrize("E,R,H,F", [(4, 256, 256, 512), (2, 384, 1024, 3584), (3, 128, 128, 128)])
def test_expert_swiglu_fused_epilogues(E, R, H, F):
    """The SwiGLU inside the expert GEMM epilogues against the unfused
    composition on the same bf16 operands: a and c equal the grouped GEMM's
    bf16 outputs bit for bit; h = silu(a)·c, da = dh·c·silu'(a) and
    dc = dh·silu(a) (dh = dy·w2ᵀ rounded to bf16, as the unfused path stores
    it) agree with the same expressions in fp32 on the rounded inputs to
    within one bf16 rounding (2^-8 relative) plus one fp32 ulp of the
    exponential, and are exact for nearly all elements."""
    r = rng(E * 1000 + F)
    rows = E * R
    X = dev(r.standard_normal((rows, H)) / 2, torch.bfloat16)
    W1 = dev(r.standard_normal((E, H, F)) / np.sqrt(H), torch.bfloat16)
    W3 = dev(r.standard_normal((E, H, F)) / np.sqrt(H), torch.bfloat16)
    W2 = dev(r.standard_normal((E, F, H)) / np.sqrt(F), torch.bfloat16)
    DY = dev(r.standard_normal((rows, H)), torch.bfloat16)
    off = torch.arange(0, rows + 1, R, dtype=torch.int32, device="cuda")
    ac, h = ops.moe_expert_swiglu(X, ops.interleave_w13(W1, W3).contiguous(), off)
    a_ref = ops.grouped_gemm(X, W1, off)
    c_ref = ops.grouped_gemm(X, W3, off)
    ac4 = ac.view(rows, F // 128, 2, 128)
    assert torch.equal(ac4[:, :, 0].reshape(rows, F), a_ref), "a must equal the grouped GEMM's output"
    assert torch.equal(ac4[:, :, 1].reshape(rows, F), c_ref), "c must equal the grouped GEMM's output"
    af, cf = a_ref.float(), c_ref.float()
    sig = 1.0 / (1.0 + torch.exp(-af))

    def within_one_rounding(got, ref, what):
        err = (got.float() - ref).abs()
        bound = 2.0 ** -8 * ref.abs() * (1 + 1e-4) + 1e-30
        assert bool((err <= bound).all()), f"{what}: max excess {float((err - bound).max()):.3e}"
        exact = float((got == ref.to(torch.bfloat16)).float().mean())
        assert exact > 0.99, f"{what}: only {exact:.4f} exactly rounded"
    within_one_rounding(h, af * sig * cf, "h")
    dac = ops.moe_expert_swiglu_backward(DY, W2, ac, off)
    g = ops.grouped_gemm(DY, W2, off, trans_b=True).float()
    d4 = dac.view(rows, F // 128, 2, 128)
    within_one_rounding(d4[:, :, 0].reshape(rows, F), g * cf * (sig + af * sig * (1 - sig)), "da")
    within_one_rounding(d4[:, :, 1].reshape(rows, F), g * (af * sig), "dc")


def test_moe_bf16_grouped_tensor_core():
    r = rng(22)
    T, H, F, E, k = 512, 128, 256, 4, 2
    x = bf16_round(r.standard_normal((T, H)).astype(np.float32))
    gate = bf16_round(r.standard_normal((H, E)).astype(np.float32) * 0.3)
    w1s = bf16_round((r.standard_normal((E, H, F)) / np.sqrt(H)).astype(np.float32))
    w3s = bf16_round((r.standard_normal((E, H, F)) / np.sqrt(H)).astype(np.float32))
    w2s = bf16_round((r.standard_normal((E, F, H)) / np.sqrt(F)).astype(np.float32))
    dy = bf16_round(r.standard_normal((T, H)).astype(np.float32))
    args = [dev(a, torch.bfloat16) for a in (x, gate, w1s, w3s, w2s)]
    # The bf16 path stores h = silu(a)·c and the output y in bf16 (a, c and the
    # expert outputs stay fp32). Probabilistic bound of those roundings (each an
    # independent relative error of variance u²/3, propagated through the
    # linear maps, LAMBDA standard deviations): var(yp) = u²/3·Σ_p h_p²·w2[p,:]²,
    # var(y) = Σ_k w_k²·var(yp_k) + u²/3·y².
    idx, wts, _ = O.route(x, gate, k)
    X64 = x.astype(np.float64)
    var_yp = np.zeros((T, k, H))
    y64 = np.zeros((T, H))
    for j in range(k):
        for e in range(E):
            rows = np.nonzero(idx[:, j] == e)[0]
            a = X64[rows] @ w1s[e].astype(np.float64)
            c = X64[rows] @ w3s[e].astype(np.float64)
            hh = a / (1.0 + np.exp(-a)) * c
            var_yp[rows, j] = U2_3 * hh ** 2 @ w2s[e].astype(np.float64) ** 2
            y64[rows] += wts[rows, j, None] * (hh @ w2s[e].astype(np.float64))
    bound = LAMBDA * np.sqrt((wts[:, :, None] ** 2 * var_yp).sum(1) + U2_3 * y64 ** 2)
    close_bf16_derived(ops.moe(*args, k), O.moe(x, gate, w1s, w3s, w2s, k), bound, what="moe bf16")
    got = ops.moe_backward(*args, dev(dy, torch.bfloat16), k)
    ref = O.moe_backward(x, gate, w1s, w3s, w2s, dy, k)
    bounds = moe_backward_rounding_bounds(x, gate, w1s, w3s, w2s, dy, idx, wts)
    for name, g, rr, bnd in zip(("dx", "dgate", "dw1", "dw3", "dw2"), got, ref, bounds):
        close_bf16_derived(g, rr, bnd, what=f"moe bf16 {name}")


def moe_backward_rounding_bounds(x, gate, w1s, w3s, w2s, dy, idx, wts):
    """Probabilistic bounds (LAMBDA standard deviations) of the bf16 roundings
    in the MoE adjoint's bf16 path (catnn_moe_bwd), from the exact values:
    dyp = w·dy stored bf16; dh = dyp·w2ᵀ (fp32) then da, dc stored bf16;
    dxp = da·w1ᵀ stored bf16, then + dc·w3ᵀ stored bf16 again; the token sum
    dx stored bf16; the router's dlogits rounded to bf16 before dlog·gateᵀ
    (added into dx, rounded again) and xᵀ·dlog; h stored bf16 for the w2
    gradient; every output stored bf16. Each rounding is an independent
    relative error of variance u²/3; errors that reach an output through two
    paths (dh into both da and dc) are combined before squaring."""
    T, H = x.shape
    E, _, F = w1s.shape
    k = idx.shape[1]
    X = x.astype(np.float64)
    DY = dy.astype(np.float64)
    v_dx = np.zeros((T, H))
    dx_sum = np.zeros((T, H))
    v_dw1, v_dw3, v_dw2 = np.zeros((E, H, F)), np.zeros((E, H, F)), np.zeros((E, F, H))
    dw1, dw3, dw2 = np.zeros((E, H, F)), np.zeros((E, H, F)), np.zeros((E, F, H))
    dwt = np.zeros((T, k))
    for j in range(k):
        for e in range(E):
            rows = np.nonzero(idx[:, j] == e)[0]
            W1, W3, W2 = (w.astype(np.float64) for w in (w1s[e], w3s[e], w2s[e]))
            xe, wt = X[rows], wts[rows, j, None]
            a, c = xe @ W1, xe @ W3
            sig = 1.0 / (1.0 + np.exp(-a))
            ga, gc = c * (sig + a * sig * (1 - sig)), a * sig  # da = dh·ga, dc = dh·gc
            hh = a * sig * c
            dwt[rows, j] = ((hh @ W2) * DY[rows]).sum(1)
            dyp = wt * DY[rows]
            dh = dyp @ W2.T
            v_dh = U2_3 * dyp ** 2 @ (W2 ** 2).T
            da, dc = dh * ga, dh * gc
            dxp1 = da @ W1.T
            dxp = dxp1 + dc @ W3.T
            # dh's error reaches dxp through both da and dc: combined coefficients
            v_dx[rows] += (v_dh[:, None, :] * (ga[:, None, :] * W1[None] + gc[:, None, :] * W3[None]) ** 2).sum(2)
            v_dx[rows] += U2_3 * ((da ** 2) @ (W1 ** 2).T + (dc ** 2) @ (W3 ** 2).T + dxp1 ** 2 + dxp ** 2)
            dx_sum[rows] += dxp
            dw1[e] += xe.T @ da
            dw3[e] += xe.T @ dc
            dw2[e] += hh.T @ dyp
            v_dw1[e] += (xe ** 2).T @ (ga ** 2 * v_dh + U2_3 * da ** 2)
            v_dw3[e] += (xe ** 2).T @ (gc ** 2 * v_dh + U2_3 * dc ** 2)
            v_dw2[e] += 2 * U2_3 * (hh ** 2).T @ (dyp ** 2)
    dlog = np.zeros((T, E))
    dot = (wts * dwt).sum(1, keepdims=True)
    np.put_along_axis(dlog, idx, wts * (dwt - dot), axis=1)
    G = gate.astype(np.float64)
    dx = dx_sum + dlog @ G.T
    v_dx += U2_3 * (dx_sum ** 2 + (dlog ** 2) @ (G ** 2).T + dx ** 2)
    dgate = X.T @ dlog
    v_dgate = (X ** 2).T @ (U2_3 * dlog ** 2) + U2_3 * dgate ** 2
    out = (v_dx, v_dgate, v_dw1 + U2_3 * dw1 ** 2, v_dw3 + U2_3 * dw3 ** 2, v_dw2 + U2_3 * dw2 ** 2)
    return tuple(LAMBDA * np.sqrt(v) for v in out)


def attention_rounding_bounds(q, k, v, do, causal, window):
    """Probabilistic bounds (LAMBDA standard deviations), per element, of the
    bf16 roundings the tensor-core flash attention makes and the fp32
    attention core does not: P rounded for P·V (forward) and Pᵀ·dO (dV), the
    output O rounded (it feeds D = rowsum(dO∘O), whose error enters every dS
    of the row, so that term is propagated as one correlated error per row),
    dS = P∘(dP - D) rounded for dS·K (dQ) and dSᵀ·Q (dK), and the outputs
    rounded; from the exact (f64) attention of the same inputs. Each
    rounding is an independent relative error of variance u²/3. Returns
    (bound_o, bound_dq, bound_dk, bound_dv) in the inputs' layouts."""
    b, s, h, hd = q.shape
    kv = k.shape[2]
    rep = h // kv
    Q, K, V = (t.astype(np.float64) for t in (q, k, v))
    Kr, Vr = np.repeat(K, rep, axis=2), np.repeat(V, rep, axis=2)
    dO = do.reshape(b, s, h, hd).astype(np.float64)
    scale = 1.0 / np.sqrt(hd)
    S = np.einsum("bihd,bjhd->bhij", Q, Kr) * scale
    i_, j_ = np.arange(s)[:, None], np.arange(s)[None, :]
    allowed = np.ones((s, s), bool)
    if causal:
        allowed &= j_ <= i_
    if window:
        allowed &= j_ > i_ - window
    S = np.where(allowed, S, -np.inf)
    P = np.exp(S - S.max(-1, keepdims=True))
    P /= P.sum(-1, keepdims=True)
    Ov = np.einsum("bhij,bjhd->bihd", P, Vr)
    dP = np.einsum("bihd,bjhd->bhij", dO, Vr)
    D = np.einsum("bihd,bihd->bhi", dO, Ov)
    dS = P * (dP - D[..., None])
    dq = np.einsum("bhij,bjhd->bihd", dS, Kr) * scale
    dk = np.einsum("bhij,bihd->bjhd", dS, Q) * scale
    dv = np.einsum("bhij,bihd->bjhd", P, dO)
    v_O = U2_3 * (np.einsum("bhij,bjhd->bihd", P ** 2, Vr ** 2) + Ov ** 2)
    v_D = np.einsum("bihd,bihd->bhi", dO ** 2, v_O)
    PK = np.einsum("bhij,bjhd->bihd", P, Kr)  # Σ_j P_ij K_j: how D's error reaches dq
    v_dq = scale ** 2 * (U2_3 * np.einsum("bhij,bjhd->bihd", dS ** 2, Kr ** 2)
                         + PK ** 2 * v_D.transpose(0, 2, 1)[..., None]) + U2_3 * dq ** 2
    v_dk = scale ** 2 * (U2_3 * np.einsum("bhij,bihd->bjhd", dS ** 2, Q ** 2)
                         + np.einsum("bhij,bihd,bhi->bjhd", P ** 2, Q ** 2, v_D))
    v_dv = U2_3 * np.einsum("bhij,bihd->bjhd", P ** 2, dO ** 2)
    # kv heads shared by `rep` query heads sum their variances; outputs rounded
    v_dk = v_dk.reshape(b, s, kv, rep, hd).sum(3) + U2_3 * dk.reshape(b, s, kv, rep, hd).sum(3) ** 2
    v_dv = v_dv.reshape(b, s, kv, rep, hd).sum(3) + U2_3 * dv.reshape(b, s, kv, rep, hd).sum(3) ** 2
    return tuple(LAMBDA * np.sqrt(v) for v in (v_O.reshape(b, s, h * hd), v_dq, v_dk, v_dv))


@pytest.mark.parametrize("b,s,h,kv,hd,causal,window", [(2, 200, 4, 4, 64, True, None), (1, 130, 4, 2, 64, True, 48),
                                                        (2, 96, 2, 2, 128, True, None), (1, 64, 2, 2, 64, False, None),
                                                        (1, 257, 2, 1, 128, True, 100), (1, 1024, 2, 1, 64, True, None),
                                                        (2, 384, 2, 2, 64, False, None), (1, 600, 4, 2, 64, True, 200)])
def test_attention_core_bf16_tensor_core(b, s, h, kv, hd, causal, window):
    """Flash attention on the tensor cores (tcgen05 + TMEM for head_dim 64,
    mma.sync for 128; forward and backward) vs the fp32 attention
    core (itself checked against the oracle's GQA above) on the same bf16
    inputs."""
    r = rng(s + hd)
    q = bf16_round(r.standard_normal((b, s, h, hd)).astype(np.float32))
    k = bf16_round(r.standard_normal((b, s, kv, hd)).astype(np.float32))
    v = bf16_round(r.standard_normal((b, s, kv, hd)).astype(np.float32))
    do = bf16_round(r.standard_normal((b, s, h * hd)).astype(np.float32))
    o32, l32 = ops.attention_core(dev(q), dev(k), dev(v), causal, window)
    o16, l16 = ops.attention_core(dev(q, torch.bfloat16), dev(k, torch.bfloat16), dev(v, torch.bfloat16), causal, window)
    bo, bdq, bdk, bdv = attention_rounding_bounds(q, k, v, do, causal, window)
    close_bf16_derived(o16, host(o32), bo, what="fa fwd o")
    close_f32(l16, host(l32), rtol=1e-3, floor=1e-4, what="fa fwd lse")
    if causal:  # moe.rs:100-133 is the causal core; compare with the oracle directly too
        close_bf16_derived(o16, O.gqa_core(q, k, v, window), bo, what="fa fwd vs oracle")
    g32 = ops.attention_core_backward(dev(q), dev(k), dev(v), o32, l32, dev(do), causal, window)
    g16 = ops.attention_core_backward(dev(q, torch.bfloat16), dev(k, torch.bfloat16), dev(v, torch.bfloat16), o16, l16,
                                      dev(do, torch.bfloat16), causal, window)
    from gpu_util import rel_l2
    for name, a16, a32, bnd in zip(("dq", "dk", "dv"), g16, g32, (bdq, bdk, bdv)):
        assert rel_l2(a16, host(a32)) < 1e-2, (name, rel_l2(a16, host(a32)))
        close_bf16_derived(a16, host(a32), bnd, what=f"fa bwd {name}")


# ------------------------------------------------------------------ BASELINE configs 1 and 3
def test_mlp_twelve_sgd_steps_match_oracle():
    """Config 1's run: the f32 MLP (784 -> 256 ReLU -> 10, softmax cross-entropy)
    trained for 12 SGD steps (lr 0.05) on the GPU and in the oracle from the
    same Xavier-uniform weights; all 12 losses and the final weights agree at
    the fp32 band (train.rs:71 mlp_step, optim.rs:32 Sgd::put)."""
    r = rng(0)
    a1, a2 = np.sqrt(6.0 / (784 + 256)), np.sqrt(6.0 / (256 + 10))
    w1 = r.uniform(-a1, a1, (784, 256)).astype(np.float32)
    w2 = r.uniform(-a2, a2, (256, 10)).astype(np.float32)
    b1, b2 = np.zeros(256, np.float32), np.zeros(10, np.float32)
    x = r.standard_normal((64, 784)).astype(np.float32)
    lab = r.integers(0, 10, 64)
    gw = [dev(t) for t in (w1, b1, w2, b2)]
    X, L = dev(x), dev(lab, torch.int32)
    ow = [t.copy() for t in (w1, b1, w2, b2)]
    for step in range(12):
        loss, *grads = ops.mlp_step(*gw, X, labels=L)
        for p, g in zip(gw, grads):
            ops.sgd_(p, g, 0.05)
        rl, *rg = O.mlp_step(*ow, x, labels=lab)
        ow = [O.sgd_put(p, g, 0.05) for p, g in zip(ow, rg)]
        close_f32(np.float32(float(loss)), np.float32(rl), what=f"loss at step {step}")
    for name, g, o in zip(("w1", "b1", "w2", "b2"), gw, ow):
        close_f32(g, o, what=f"{name} after 12 steps")


def test_transformer_block_fwd_bwd_f32():
    """Config 3 at its full shape: the pre-LN causal block (B8 S512 d512, 8
    heads of 64, GELU FFN 2048, both residuals; fp32 weights N(0, 0.02),
    LayerNorm gamma 1 / beta 0, inputs N(0, 1), injected dY N(0, 1), seed 2)
    composed from the GPU operators in the oracle's order, against the
    oracle's block at rtol 1e-5 (floor 1e-5 of each tensor's scale), with the
    f64 instantiation of the same loop nests as the exact fallback."""
    r = rng(2)
    b, s, d, h, ff = 8, 512, 512, 8, 2048
    W = {"g1": np.ones(d, np.float32), "be1": np.zeros(d, np.float32), "g2": np.ones(d, np.float32),
         "be2": np.zeros(d, np.float32), "c1": np.zeros(ff, np.float32), "c2": np.zeros(d, np.float32)}
    for k, shape in (("wq", (d, d)), ("wk", (d, d)), ("wv", (d, d)), ("wo", (d, d)), ("f1", (d, ff)), ("f2", (ff, d))):
        W[k] = (r.standard_normal(shape) * 0.02).astype(np.float32)
    x = r.standard_normal((b, s, d)).astype(np.float32)
    dy = r.standard_normal((b, s, d)).astype(np.float32)
    G = {k: dev(v) for k, v in W.items()}
    X, DY = dev(x), dev(dy)
    ln1 = ops.layer_norm(X, G["g1"], G["be1"])
    att = ops.attention(ln1, G["wq"], G["wk"], G["wv"], G["wo"], h, causal=True)
    hh = ops.add(X, att)
    ln2 = ops.layer_norm(hh, G["g2"], G["be2"])
    u = ops.linear(ln2, G["f1"], G["c1"])
    gl = ops.gelu(u)
    y = ops.add(hh, ops.linear(gl, G["f2"], G["c2"]))
    dgl, df2, dc2 = ops.linear_backward(gl, G["f2"], DY)
    du = ops.gelu_backward(u, dgl)
    dln2, df1, dc1 = ops.linear_backward(ln2, G["f1"], du)
    dh, dg2, dbe2 = ops.layer_norm_backward(hh, G["g2"], dln2)
    dh = ops.add(dh, DY)
    dln1, dwq, dwk, dwv, dwo = ops.attention_backward(ln1, G["wq"], G["wk"], G["wv"], G["wo"], dh, h, causal=True)
    dxa, dg1, dbe1 = ops.layer_norm_backward(X, G["g1"], dln1)
    dx = ops.add(dxa, dh)
    ry, rdx, rg = O.block_fwd_bwd(W, x, dy, h)
    ey, edx, eg = O.block_fwd_bwd(W, x, dy, h, f64=True)
    close_f32(y, ry, what="block y", exact=ey)
    close_f32(dx, rdx, what="block dx", exact=edx)
    got = {"g1": dg1, "be1": dbe1, "wq": dwq, "wk": dwk, "wv": dwv, "wo": dwo, "g2": dg2, "be2": dbe2, "f1": df1,
           "c1": dc1, "f2": df2, "c2": dc2}
    for k, g in got.items():
        close_f32(g, rg[k], what=f"block d{k}", exact=eg[k])
