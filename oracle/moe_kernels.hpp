// ORACLE — test infrastructure only (see cpu_kernels.hpp header).
//
// Restatement of crates/catnn-compile/src/kernel/moe.rs (RMSNorm, embedding,
// RoPE, GQA with optional sliding window, SwiGLU, router, MoE, LM head) and
// crates/catnn-core/src/lens/moe.rs:175-187 (topk_softmax).
#pragma once
#include "cpu_kernels.hpp"

namespace orc {

// moe.rs:12-14
template <typename T> inline T silu(T x) { return x / ((T)1.0 + std::exp(-x)); }

// moe.rs:17-32 — y = x * (1/sqrt(mean(x^2)+eps)) * w, mean by sequential sum.
template <typename T> void rmsnorm(const T* x, const T* w, T* y, i64 rows, i64 last, T eps) {
    for (i64 r = 0; r < rows; ++r) {
        const T* row = x + r * last;
        T* out = y + r * last;
        T ss = 0;
        for (i64 i = 0; i < last; ++i) ss += row[i] * row[i];
        T mean_sq = ss / (T)last;
        T inv = (T)1.0 / std::sqrt(mean_sq + eps);
        for (i64 i = 0; i < last; ++i) out[i] = row[i] * inv * w[i];
    }
}

// moe.rs:34-45 — gather rows of table [vocab, hidden]. Returns -1 (the
// reference's ShapeMismatch "token {id} >= vocab") on an out-of-range id.
template <typename T>
int embedding(const uint32_t* ids, i64 n_ids, const T* table, i64 vocab, i64 hidden, T* y) {
    for (i64 t = 0; t < n_ids; ++t) {
        if ((i64)ids[t] >= vocab) return -1;
        std::memcpy(y + t * hidden, table + (i64)ids[t] * hidden, sizeof(T) * hidden);
    }
    return 0;
}

// moe.rs:47-59 and adjoint.rs:454-466 — rotate interleaved pairs (2i, 2i+1)
// by pos * theta^(-2i/hd). The frequency and angle are f64; sin and cos are
// rounded to T. A negative theta is the adjoint: |theta| with sin negated.
template <typename T> void apply_rope(T* q, i64 head_dim, i64 pos, double theta) {
    for (i64 i = 0; i < head_dim / 2; ++i) {
        double freq = 1.0 / std::pow(std::fabs(theta), 2.0 * (double)i / (double)head_dim);
        double ang = (double)pos * freq;
        double sd = std::sin(ang), cd = std::cos(ang);
        T s = theta < 0.0 ? (T)(-sd) : (T)sd;
        T c = (T)cd;
        T a = q[2 * i], b = q[2 * i + 1];
        q[2 * i] = a * c - b * s;
        q[2 * i + 1] = a * s + b * c;
    }
}

// Apply RoPE to every head of a [B,S,heads,hd] tensor (moe.rs:88-99).
template <typename T>
void rope_all(T* q, i64 b, i64 s, i64 heads, i64 hd, double theta) {
    for (i64 bi = 0; bi < b; ++bi)
        for (i64 t = 0; t < s; ++t)
            for (i64 h = 0; h < heads; ++h) apply_rope(q + ((bi * s + t) * heads + h) * hd, hd, t, theta);
}

// Window start (moe.rs:105): i.saturating_sub(w - 1), or 0 without a window.
inline i64 win_start(i64 i, i64 window) {
    if (window <= 0) return 0;
    i64 st = i - (window - 1);
    return st < 0 ? 0 : st;
}

// The attention core of moe.rs:100-133 on already-projected, already-rotated
// q [B,S,H,hd], k/v [B,S,Hkv,hd]. ctx [B,S,H*hd] is accumulated from zero.
// When probs != nullptr the normalized probabilities are stored
// ([B,H,S,S], adjoint.rs:324-350) — the multiply by inv happens in place
// there, which rounds the same as `score * inv` in the forward.
template <typename T>
void gqa_core(const T* q, const T* k, const T* v, T* ctx, T* probs, i64 b, i64 s, i64 n_heads,
              i64 n_kv, i64 hd, i64 window) {
    i64 repeats = n_heads / (n_kv > 1 ? n_kv : 1);
    if (repeats < 1) repeats = 1;
    const T scale = (T)1.0 / std::sqrt((T)hd);
    std::fill(ctx, ctx + b * s * n_heads * hd, (T)0);
    // (batch, head) pairs write disjoint ctx / probs slices: one per thread
    split_rows(b * n_heads, [&](i64 bh) {
        const i64 bi = bh / n_heads, h = bh % n_heads;
        std::vector<T> scores(s);
        {
            i64 kv_h = h / repeats;
            for (i64 i = 0; i < s; ++i) {
                i64 start = win_start(i, window);
                i64 q_off = ((bi * s + i) * n_heads + h) * hd;
                for (i64 j = start; j <= i; ++j) {
                    i64 k_off = ((bi * s + j) * n_kv + kv_h) * hd;
                    T dot = 0;
                    for (i64 t = 0; t < hd; ++t) dot += q[q_off + t] * k[k_off + t];
                    scores[j] = dot * scale;
                }
                T mx = -INFINITY;
                for (i64 j = start; j <= i; ++j) mx = tmax(mx, scores[j]);
                T sum = 0;
                for (i64 j = start; j <= i; ++j) {
                    scores[j] = std::exp(scores[j] - mx);
                    sum += scores[j];
                }
                T inv = (T)1.0 / tmax(sum, (T)1e-30);
                for (i64 j = start; j <= i; ++j) {
                    T wgt = scores[j] * inv;
                    if (probs) probs[((bi * n_heads + h) * s + i) * s + j] = wgt;
                    i64 v_off = ((bi * s + j) * n_kv + kv_h) * hd;
                    for (i64 t = 0; t < hd; ++t) ctx[q_off + t] += wgt * v[v_off + t];
                }
            }
        }
    });
}

// moe.rs:64-136 — GQA + RoPE + optional window on x [B,S,d] (RMS-normed).
// All projections are linear_seq (sequential p order). window <= 0 is None.
template <typename T>
void gqa(const T* x, const T* wq, const T* wk, const T* wv, const T* wo, T* y, i64 b, i64 s,
         i64 d, i64 n_heads, i64 n_kv, i64 hd, double theta, i64 window) {
    i64 qd = n_heads * hd, kd = n_kv * hd;
    std::vector<T> q(b * s * qd), k(b * s * kd), v(b * s * kd), ctx(b * s * qd);
    matmul_seq(x, wq, q.data(), b * s, d, qd);
    matmul_seq(x, wk, k.data(), b * s, d, kd);
    matmul_seq(x, wv, v.data(), b * s, d, kd);
    rope_all(q.data(), b, s, n_heads, hd, theta);
    rope_all(k.data(), b, s, n_kv, hd, theta);
    gqa_core(q.data(), k.data(), v.data(), ctx.data(), (T*)nullptr, b, s, n_heads, n_kv, hd, window);
    matmul_seq(ctx.data(), wo, y, b * s, qd, d);
}

// moe.rs:159-174 — w2(silu(x w1) * (x w3)), all through linear_seq.
template <typename T>
void swiglu(const T* x, const T* w1, const T* w3, const T* w2, T* y, i64 tokens, i64 hidden,
            i64 mid) {
    std::vector<T> a(tokens * mid), c(tokens * mid);
    matmul_seq(x, w1, a.data(), tokens, hidden, mid);
    matmul_seq(x, w3, c.data(), tokens, hidden, mid);
    for (i64 i = 0; i < tokens * mid; ++i) a[i] = silu(a[i]) * c[i];
    matmul_seq(a.data(), w2, y, tokens, mid, hidden);
}

// lens/moe.rs:175-187 — indices sorted by descending logit with a stable
// sort (ties keep the lower index first), truncated to k; weights are the
// softmax over the k selected logits only. NaN logits compare Equal in the
// reference's comparator, which is not a strict weak order; the GPU router
// and this restatement are specified for NaN-free rows only.
template <typename T> void topk_softmax(const T* logits, i64 n, i64 k, int64_t* idx, T* w) {
    std::vector<int64_t> order(n);
    for (i64 i = 0; i < n; ++i) order[i] = i;
    std::stable_sort(order.begin(), order.end(),
                     [&](int64_t a, int64_t b) { return logits[a] > logits[b]; });
    i64 kk = k < n ? k : n;
    T mx = -INFINITY;
    for (i64 i = 0; i < kk; ++i) mx = tmax(mx, logits[order[i]]);
    T sum = 0;
    for (i64 i = 0; i < kk; ++i) {
        idx[i] = order[i];
        w[i] = std::exp(logits[order[i]] - mx);
        sum += w[i];
    }
    T inv = (T)1.0 / tmax(sum, (T)1e-30);
    for (i64 i = 0; i < kk; ++i) w[i] *= inv;
}

// Frozen routing (the held-fixed indices of fd64.rs:550-600, topk_fixed /
// route_idx): the k experts are given, the weights are the softmax over
// their logits exactly as topk_softmax computes it.
template <typename T> void softmax_selected(const T* logits, i64 k, const int64_t* idx, T* w) {
    T mx = -INFINITY;
    for (i64 i = 0; i < k; ++i) mx = tmax(mx, logits[idx[i]]);
    T sum = 0;
    for (i64 i = 0; i < k; ++i) {
        w[i] = std::exp(logits[idx[i]] - mx);
        sum += w[i];
    }
    T inv = (T)1.0 / tmax(sum, (T)1e-30);
    for (i64 i = 0; i < k; ++i) w[i] *= inv;
}

// moe.rs:177-195 — logits = x·gate (linear_seq), then topk_softmax per row.
// forced (optional, [tokens, k]) replaces the top-k selection.
template <typename T>
void route(const T* x, const T* gate, i64 tokens, i64 hidden, i64 n_exp, i64 k, int64_t* idx,
           T* w, T* logits, const int64_t* forced = nullptr) {
    matmul_seq(x, gate, logits, tokens, hidden, n_exp);
    for (i64 t = 0; t < tokens; ++t) {
        if (forced) {
            for (i64 i = 0; i < k; ++i) idx[t * k + i] = forced[t * k + i];
            softmax_selected(logits + t * n_exp, k, idx + t * k, w + t * k);
        } else {
            topk_softmax(logits + t * n_exp, n_exp, k, idx + t * k, w + t * k);
        }
    }
}

// moe.rs:197-223 — per token, per slot: out += w_tk * swiglu_e(x_t).
// Expert weights are packed: w1s [E, hidden, mid], w3s [E, hidden, mid],
// w2s [E, mid, hidden].
template <typename T>
void moe(const T* x, const T* gate, const T* w1s, const T* w3s, const T* w2s, T* y, i64 tokens,
         i64 hidden, i64 mid, i64 n_exp, i64 k, const int64_t* forced = nullptr) {
    std::vector<int64_t> idx(tokens * k);
    std::vector<T> wts(tokens * k), logits(tokens * n_exp);
    route(x, gate, tokens, hidden, n_exp, k, idx.data(), wts.data(), logits.data(), forced);
    std::fill(y, y + tokens * hidden, (T)0);
    // tokens are independent (each writes its own output row): one per thread
    split_rows(tokens, [&](i64 t) {
        std::vector<T> ye(hidden);
        for (i64 kk = 0; kk < k; ++kk) {
            i64 e = idx[t * k + kk];
            T wt = wts[t * k + kk];
            swiglu(x + t * hidden, w1s + e * hidden * mid, w3s + e * hidden * mid,
                   w2s + e * mid * hidden, ye.data(), 1, hidden, mid);
            for (i64 i = 0; i < hidden; ++i) y[t * hidden + i] += wt * ye[i];
        }
    });
}

// moe.rs:325-333 — logits = x · w^T with w stored [vocab, hidden]; the
// reference transposes then runs linear_seq, i.e. a sequential p-order dot.
template <typename T> void lm_head(const T* x, const T* w, T* y, i64 rows, i64 hidden, i64 vocab) {
    split_rows(rows, [=](i64 i) {
        for (i64 j = 0; j < vocab; ++j) {
            T s = 0;
            for (i64 p = 0; p < hidden; ++p) s += x[i * hidden + p] * w[j * hidden + p];
            y[i * vocab + j] = s;
        }
    });
}

}  // namespace orc
