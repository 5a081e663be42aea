// ORACLE — test infrastructure only (see cpu_kernels.hpp header).
//
// Optimizers (crates/catnn-core/src/lens/optim.rs) and the end-to-end
// training steps (crates/catnn-compile/src/train.rs), plus the two composed
// steps the benchmark configs name but no single reference entry point runs
// (the cross-entropy MLP and the causal pre-LN transformer block).
#pragma once
#include "adjoint_kernels.hpp"

namespace orc {

// optim.rs:32-43 — p - lr*g.
template <typename T> void sgd_put(const T* p, const T* g, T* out, i64 n, T lr) {
    for (i64 i = 0; i < n; ++i) out[i] = p[i] - lr * g[i];
}

// Binary exponentiation for an integer power, the published algorithm of
// LLVM's powi lowering (compiler-rt __powisf2): multiply r by a on each set
// bit while squaring a; 1/r for a negative exponent.
template <typename T> T powi(T a, int b) {
    bool recip = b < 0;
    T r = 1;
    for (;;) {
        if (b & 1) r *= a;
        b /= 2;
        if (b == 0) break;
        a *= a;
    }
    return recip ? (T)1 / r : r;
}

// optim.rs:95-119 — one Adam step from step count t_prev (t = t_prev + 1).
// m, v are updated in place; returns t.
template <typename T>
uint64_t adam_put(T* p, const T* g, T* m, T* v, i64 n, uint64_t t_prev, T lr, T b1, T b2, T eps) {
    uint64_t t = t_prev + 1;
    T b1t = (T)1.0 - powi(b1, (int)t);
    T b2t = (T)1.0 - powi(b2, (int)t);
    for (i64 i = 0; i < n; ++i) {
        T gi = g[i];
        T mi = b1 * m[i] + ((T)1.0 - b1) * gi;
        T vi = b2 * v[i] + ((T)1.0 - b2) * gi * gi;
        m[i] = mi;
        v[i] = vi;
        T mhat = mi / tmax(b1t, (T)1e-30);
        T vhat = vi / tmax(b2t, (T)1e-30);
        p[i] = p[i] - lr * mhat / (std::sqrt(vhat) + eps);
    }
    return t;
}

// ---------------------------------------------------------------- Mixtral

// Shapes of a Mixtral-style decoder (crates/catnn-core/src/spec/mixtral.rs).
struct MixCfg {
    i64 vocab, hidden, mid, layers, heads, kv_heads, experts, top_k;
    float eps;
    double theta;
    i64 window;  // <= 0: no sliding window
};

// Packed parameter layout shared by the oracle and the CUDA backend:
// embed [V,h]; per layer: rms_attn [h], wq [h,H*hd], wk [h,Hkv*hd],
// wv [h,Hkv*hd], wo [H*hd,h], rms_moe [h], gate [h,E], w1 [E,h,F],
// w3 [E,h,F], w2 [E,F,h]; then final_norm [h], lm_head [V,h].
struct MixLayout {
    i64 embed, final_norm, lm_head, total;
    i64 layer0, layer_stride;
    i64 rms_attn, wq, wk, wv, wo, rms_moe, gate, w1, w3, w2;  // offsets within a layer
    explicit MixLayout(const MixCfg& c) {
        i64 h = c.hidden, hd = c.hidden / c.heads, qd = c.heads * hd, kd = c.kv_heads * hd;
        embed = 0;
        layer0 = c.vocab * h;
        i64 o = 0;
        rms_attn = o; o += h;
        wq = o; o += h * qd;
        wk = o; o += h * kd;
        wv = o; o += h * kd;
        wo = o; o += qd * h;
        rms_moe = o; o += h;
        gate = o; o += h * c.experts;
        w1 = o; o += c.experts * h * c.mid;
        w3 = o; o += c.experts * h * c.mid;
        w2 = o; o += c.experts * c.mid * h;
        layer_stride = o;
        final_norm = layer0 + c.layers * layer_stride;
        lm_head = final_norm + h;
        total = lm_head + c.vocab * h;
    }
};

// moe.rs:247-285 — MixtralWeights::seeded: a seed chain s = s*A + 1 hands a
// fresh LCG seed to each tensor in the order embed, then per layer the
// experts' (w1, w3, w2) followed by wq, wk, wv, wo, gate, and finally the LM
// head; RMS weights are ones.
inline void mixtral_seeded(const MixCfg& c, uint64_t seed, float* P) {
    MixLayout L(c);
    i64 h = c.hidden, hd = c.hidden / c.heads, qd = c.heads * hd, kd = c.kv_heads * hd;
    uint64_t s = seed;
    auto next = [&]() { s = s * 6364136223846793005ull + 1ull; return s; };
    lcg_fill(P + L.embed, c.vocab * h, next());
    for (i64 l = 0; l < c.layers; ++l) {
        float* Lp = P + L.layer0 + l * L.layer_stride;
        for (i64 e = 0; e < c.experts; ++e) {
            lcg_fill(Lp + L.w1 + e * h * c.mid, h * c.mid, next());
            lcg_fill(Lp + L.w3 + e * h * c.mid, h * c.mid, next());
            lcg_fill(Lp + L.w2 + e * c.mid * h, c.mid * h, next());
        }
        for (i64 i = 0; i < h; ++i) Lp[L.rms_attn + i] = 1.0f;
        lcg_fill(Lp + L.wq, h * qd, next());
        lcg_fill(Lp + L.wk, h * kd, next());
        lcg_fill(Lp + L.wv, h * kd, next());
        lcg_fill(Lp + L.wo, qd * h, next());
        for (i64 i = 0; i < h; ++i) Lp[L.rms_moe + i] = 1.0f;
        lcg_fill(Lp + L.gate, h * c.experts, next());
    }
    for (i64 i = 0; i < h; ++i) P[L.final_norm + i] = 1.0f;
    lcg_fill(P + L.lm_head, c.vocab * h, next());
}

// moe.rs:288-323 — forward to logits [B*S, V] (residual adds included).
template <typename T>
int mixtral_forward(const MixCfg& c, const T* P, const uint32_t* tokens, i64 batch, i64 seq, T* logits) {
    MixLayout L(c);
    i64 h = c.hidden, n = batch * seq, hd = c.hidden / c.heads;
    std::vector<T> x(n * h), xn(n * h), a(n * h);
    if (embedding(tokens, n, P + L.embed, c.vocab, h, x.data())) return -1;
    for (i64 l = 0; l < c.layers; ++l) {
        const T* Lp = P + L.layer0 + l * L.layer_stride;
        rmsnorm(x.data(), Lp + L.rms_attn, xn.data(), n, h, (T)c.eps);
        gqa(xn.data(), Lp + L.wq, Lp + L.wk, Lp + L.wv, Lp + L.wo, a.data(), batch, seq, h, c.heads,
            c.kv_heads, hd, c.theta, c.window);
        add(x.data(), a.data(), x.data(), n * h);
        rmsnorm(x.data(), Lp + L.rms_moe, xn.data(), n, h, (T)c.eps);
        moe(xn.data(), Lp + L.gate, Lp + L.w1, Lp + L.w3, Lp + L.w2, a.data(), n, h, c.mid, c.experts, c.top_k);
        add(x.data(), a.data(), x.data(), n * h);
    }
    rmsnorm(x.data(), P + L.final_norm, xn.data(), n, h, (T)c.eps);
    lm_head(xn.data(), P + L.lm_head, logits, n, h, c.vocab);
    return 0;
}

// train.rs:261-356 — mixtral_step without checkpointing (the rematerialized
// path is bit-identical in the reference, train.rs:826). Targets are the
// next token with wrap-around, mod vocab. G receives the packed gradients.
// forced (optional, [layers][batch*seq][top_k]) freezes the routing of each
// layer (the fd64.rs methodology for checks across a discontinuous top-k).
template <typename T>
int mixtral_step(const MixCfg& c, const T* P, const uint32_t* tokens, i64 batch, i64 seq, T* loss, T* G,
                 const int64_t* forced = nullptr) {
    MixLayout L(c);
    i64 h = c.hidden, n = batch * seq, hd = c.hidden / c.heads;
    std::vector<uint32_t> targets(n);
    for (i64 i = 0; i < n; ++i) targets[i] = tokens[(i + 1) % n] % (uint32_t)c.vocab;
    std::vector<T> x(n * h);
    if (embedding(tokens, n, P + L.embed, c.vocab, h, x.data())) return -1;
    std::vector<std::vector<T>> xs{x}, s_xn, s_xm, s_attn;
    std::vector<T> tmp(n * h);
    for (i64 l = 0; l < c.layers; ++l) {
        const T* Lp = P + L.layer0 + l * L.layer_stride;
        std::vector<T> xn(n * h), attn(n * h), xm(n * h);
        rmsnorm(x.data(), Lp + L.rms_attn, xn.data(), n, h, (T)c.eps);
        gqa(xn.data(), Lp + L.wq, Lp + L.wk, Lp + L.wv, Lp + L.wo, attn.data(), batch, seq, h,
            c.heads, c.kv_heads, hd, c.theta, c.window);
        add(x.data(), attn.data(), x.data(), n * h);
        rmsnorm(x.data(), Lp + L.rms_moe, xm.data(), n, h, (T)c.eps);
        moe(xm.data(), Lp + L.gate, Lp + L.w1, Lp + L.w3, Lp + L.w2, tmp.data(), n, h, c.mid, c.experts, c.top_k,
            forced ? forced + l * n * c.top_k : nullptr);
        add(x.data(), tmp.data(), x.data(), n * h);
        s_xn.push_back(xn);
        s_xm.push_back(xm);
        s_attn.push_back(attn);
        xs.push_back(x);
    }
    std::vector<T> xf(n * h), logits(n * c.vocab), dlog(n * c.vocab);
    rmsnorm(x.data(), P + L.final_norm, xf.data(), n, h, (T)c.eps);
    lm_head(xf.data(), P + L.lm_head, logits.data(), n, h, c.vocab);
    if (cross_entropy(logits.data(), targets.data(), dlog.data(), n, c.vocab, loss)) return -1;
    std::fill(G, G + L.total, (T)0);
    std::vector<T> dxf(n * h), dx(n * h);
    lm_head_backward(xf.data(), P + L.lm_head, dlog.data(), dxf.data(), G + L.lm_head, n, h, c.vocab);
    rmsnorm_backward(x.data(), P + L.final_norm, dxf.data(), dx.data(), G + L.final_norm, n, h, (T)c.eps);
    std::vector<T> xmid(n * h), dxm(n * h), dxmid(n * h), dxn(n * h), dxin(n * h);
    for (i64 l = c.layers - 1; l >= 0; --l) {
        const T* Lp = P + L.layer0 + l * L.layer_stride;
        T* Gl = G + L.layer0 + l * L.layer_stride;
        add(xs[l].data(), s_attn[l].data(), xmid.data(), n * h);
        moe_backward(s_xm[l].data(), Lp + L.gate, Lp + L.w1, Lp + L.w3, Lp + L.w2, dx.data(), dxm.data(),
                     Gl + L.gate, Gl + L.w1, Gl + L.w3, Gl + L.w2, n, h, c.mid, c.experts, c.top_k,
                     forced ? forced + l * n * c.top_k : nullptr);
        rmsnorm_backward(xmid.data(), Lp + L.rms_moe, dxm.data(), dxmid.data(), Gl + L.rms_moe, n, h, (T)c.eps);
        add(dx.data(), dxmid.data(), dxmid.data(), n * h);  // dx_mid = dx + dxmid_moe
        gqa_backward(s_xn[l].data(), Lp + L.wq, Lp + L.wk, Lp + L.wv, Lp + L.wo, dxmid.data(), dxn.data(),
                     Gl + L.wq, Gl + L.wk, Gl + L.wv, Gl + L.wo, batch, seq, h, c.heads, c.kv_heads, hd,
                     c.theta, c.window);
        rmsnorm_backward(xs[l].data(), Lp + L.rms_attn, dxn.data(), dxin.data(), Gl + L.rms_attn, n, h, (T)c.eps);
        add(dxin.data(), dxmid.data(), dx.data(), n * h);  // dx = dxin_attn + dx_mid
    }
    embedding_backward(tokens, n, dx.data(), G + L.embed, c.vocab, h);
    return 0;
}

// ---------------------------------------------------------------- MLP

// train.rs:71-91 (mlp_step) with the loss chosen by `ce`: ce=0 is the
// reference's MSE step; ce=1 swaps in adjoint::cross_entropy (adjoint.rs:123)
// on integer labels — the benchmark's MLP config, composed from the same
// reference functions (cpu::linear, cpu::relu, linear_backward,
// relu_backward). Gradients dw1 [din,hid], db1, dw2 [hid,dout], db2.
template <typename T>
int mlp_step(const T* w1, const T* b1, const T* w2, const T* b2, const T* x, const T* y_mse,
             const uint32_t* labels, int ce, i64 batch, i64 din, i64 hid, i64 dout, T* loss, T* dw1,
             T* db1, T* dw2, T* db2) {
    std::vector<T> z1(batch * hid), h1(batch * hid), pred(batch * dout), dpred(batch * dout);
    std::vector<T> dh1(batch * hid), dz1(batch * hid), dx(batch * din);
    linear(x, w1, b1, z1.data(), batch, din, hid, 1);
    relu(z1.data(), h1.data(), batch * hid);
    linear(h1.data(), w2, b2, pred.data(), batch, hid, dout, 1);
    if (ce) {
        if (cross_entropy(pred.data(), labels, dpred.data(), batch, dout, loss)) return -1;
    } else {
        *loss = mse_loss(pred.data(), y_mse, dpred.data(), batch * dout);
    }
    linear_backward(h1.data(), w2, dpred.data(), dh1.data(), dw2, db2, batch, hid, dout);
    relu_backward(z1.data(), dh1.data(), dz1.data(), batch * hid);
    linear_backward(x, w1, dz1.data(), dx.data(), dw1, db1, batch, din, hid);
    return 0;
}

// ------------------------------------------------- transformer block (cfg 3)

// Pre-LN causal block composed from reference kernels:
//   h = x + attention(layer_norm(x; g1, be1))            (cpu.rs:235 + mask)
//   y = h + linear(gelu(linear(layer_norm(h; g2, be2), f1, c1)), f2, c2)
// with cpu::linear (8-lane order) for every projection and the adjoints of
// adjoint.rs for the backward, given an injected dy.
template <typename T> struct BlockW {
    const T *g1, *be1, *wq, *wk, *wv, *wo, *g2, *be2, *f1, *c1, *f2, *c2;
};
template <typename T> struct BlockG {
    T *g1, *be1, *wq, *wk, *wv, *wo, *g2, *be2, *f1, *c1, *f2, *c2;
};

template <typename T>
void block_fwd_bwd(const BlockW<T>& W, const T* x, const T* dy, T* y, T* dx, const BlockG<T>& G, i64 b, i64 s,
                   i64 d, i64 heads, i64 ff, T eps) {
    i64 n = b * s, hdim = d / heads;
    std::vector<T> ln1(n * d), att(n * d), hh(n * d), ln2(n * d), u(n * ff), gl(n * ff), f(n * d);
    layer_norm(x, W.g1, W.be1, ln1.data(), n, d, eps);
    attention(ln1.data(), W.wq, W.wk, W.wv, W.wo, att.data(), b, s, d, heads, hdim, 1);
    add(x, att.data(), hh.data(), n * d);
    layer_norm(hh.data(), W.g2, W.be2, ln2.data(), n, d, eps);
    linear(ln2.data(), W.f1, W.c1, u.data(), n, d, ff, 1);
    gelu(u.data(), gl.data(), n * ff);
    linear(gl.data(), W.f2, W.c2, f.data(), n, ff, d, 1);
    add(hh.data(), f.data(), y, n * d);
    if (!dy) return;
    std::vector<T> dgl(n * ff), du(n * ff), dln2(n * d), dh(n * d), dln1(n * d), dxa(n * d);
    linear_backward(gl.data(), W.f2, dy, dgl.data(), G.f2, G.c2, n, ff, d);
    gelu_backward(u.data(), dgl.data(), du.data(), n * ff);
    linear_backward(ln2.data(), W.f1, du.data(), dln2.data(), G.f1, G.c1, n, d, ff);
    layer_norm_backward(hh.data(), W.g2, dln2.data(), dh.data(), G.g2, G.be2, n, d, eps);
    add(dh.data(), dy, dh.data(), n * d);
    attention_backward(ln1.data(), W.wq, W.wk, W.wv, W.wo, dh.data(), dln1.data(), G.wq, G.wk, G.wv,
                       G.wo, b, s, d, heads, hdim, 1);
    layer_norm_backward(x, W.g1, dln1.data(), dxa.data(), G.g1, G.be1, n, d, eps);
    add(dxa.data(), dh.data(), dx, n * d);
}

}  // namespace orc
