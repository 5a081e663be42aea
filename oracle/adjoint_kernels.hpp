// ORACLE — test infrastructure only (see cpu_kernels.hpp header).
//
// Restatement of crates/catnn-compile/src/kernel/adjoint.rs: the reverse
// rules the reference's `adjoint_of` dispatches to.
#pragma once
#include "moe_kernels.hpp"

namespace orc {

// adjoint.rs:35-61 — one sequential i-j-p nest:
// db[j] += g; dw[p][j] += x[i][p]*g; dx[i][p] += g*w[p][j].
// Outputs are overwritten (zeroed first). db may be null.
// Every element's accumulation order is the nest's: dx[i][p] sums over j
// ascending, dw[p][j] and db[j] over i ascending. The three outputs are
// written by separate loops (dx split by rows i, dw by rows p over threads),
// which keeps each of those sums, and so every value, as the single nest
// produces it.
template <typename T>
void linear_backward(const T* x, const T* w, const T* dy, T* dx, T* dw, T* db, i64 m, i64 k, i64 n) {
    std::fill(dx, dx + m * k, (T)0);
    std::fill(dw, dw + k * n, (T)0);
    if (db) {
        std::fill(db, db + n, (T)0);
        for (i64 i = 0; i < m; ++i)
            for (i64 j = 0; j < n; ++j) db[j] += dy[i * n + j];
    }
    split_rows(m, [=](i64 i) {
        T* dxi = dx + i * k;
        for (i64 j = 0; j < n; ++j) {
            T g = dy[i * n + j];
            for (i64 p = 0; p < k; ++p) dxi[p] += g * w[p * n + j];
        }
    });
    split_rows(k, [=](i64 p) {
        T* dwp = dw + p * n;
        for (i64 i = 0; i < m; ++i) {
            T xp = x[i * k + p];
            for (i64 j = 0; j < n; ++j) dwp[j] += xp * dy[i * n + j];
        }
    });
}

// adjoint.rs:63-74
template <typename T> void relu_backward(const T* x, const T* dy, T* dx, i64 n) {
    for (i64 i = 0; i < n; ++i) dx[i] = x[i] <= (T)0 ? (T)0 : dy[i];
}

// adjoint.rs:76-90
template <typename T> void gelu_backward(const T* x, const T* dy, T* dx, i64 n) {
    const T C = (T)0.044715;
    const T k = gelu_k<T>();
    for (i64 i = 0; i < n; ++i) {
        T z = x[i];
        T u = k * (z + C * z * z * z);
        T t = std::tanh(u);
        T sech2 = (T)1.0 - t * t;
        T du = k * ((T)1.0 + (T)3.0 * C * z * z);
        T dgelu = (T)0.5 * ((T)1.0 + t) + (T)0.5 * z * sech2 * du;
        dx[i] = dy[i] * dgelu;
    }
}

// adjoint.rs:92-104 — dx = y * (dy - <y, dy>) per row.
template <typename T> void softmax_backward(const T* y, const T* dy, T* dx, i64 rows, i64 last) {
    for (i64 r = 0; r < rows; ++r) {
        const T* yr = y + r * last;
        const T* gr = dy + r * last;
        T dot = 0;
        for (i64 i = 0; i < last; ++i) dot += yr[i] * gr[i];
        for (i64 i = 0; i < last; ++i) dx[r * last + i] = yr[i] * (gr[i] - dot);
    }
}

// adjoint.rs:106-119 — returns the loss; d = 2e/n.
template <typename T> T mse_loss(const T* pred, const T* target, T* d, i64 n) {
    T nn = (T)n, loss = 0;
    for (i64 i = 0; i < n; ++i) {
        T e = pred[i] - target[i];
        loss += e * e;
        d[i] = (T)2.0 * e / nn;
    }
    return loss / nn;
}

// adjoint.rs:123-145 — mean softmax CE. d = probs / rows, minus 1/rows at
// the target. Returns 0 and writes *loss; -1 when a target >= last.
template <typename T>
int cross_entropy(const T* logits, const uint32_t* targets, T* d, i64 rows, i64 last, T* loss_out) {
    softmax_last(logits, d, rows, last);
    T loss = 0;
    T fr = (T)rows;
    for (i64 r = 0; r < rows; ++r) {
        i64 t = targets[r];
        if (t >= last) return -1;
        T p = tmax(d[r * last + t], (T)1e-30);
        loss -= std::log(p);
        for (i64 j = 0; j < last; ++j) d[r * last + j] /= fr;
        d[r * last + t] -= (T)1.0 / fr;
    }
    *loss_out = loss / fr;
    return 0;
}

// adjoint.rs:148-193
template <typename T>
void rmsnorm_backward(const T* x, const T* w, const T* dy, T* dx, T* dw, i64 rows, i64 last, T eps) {
    const T n = (T)last;
    std::fill(dw, dw + last, (T)0);
    for (i64 r = 0; r < rows; ++r) {
        const T* row = x + r * last;
        const T* yrow = dy + r * last;
        T ss = 0;
        for (i64 i = 0; i < last; ++i) ss += row[i] * row[i];
        T ms = ss / n;
        T inv = (T)1.0 / std::sqrt(ms + eps);
        T dinv = 0;
        for (i64 i = 0; i < last; ++i) {
            dw[i] += yrow[i] * row[i] * inv;
            dinv += yrow[i] * row[i] * w[i];
        }
        T dms = dinv * (T)(-0.5) * std::pow(ms + eps, (T)(-1.5));
        for (i64 i = 0; i < last; ++i)
            dx[r * last + i] = yrow[i] * inv * w[i] + dms * ((T)2.0 * row[i] / n);
    }
}

// adjoint.rs:195-206 — scatter-add rows of dy into a zeroed [vocab, hidden].
template <typename T>
void embedding_backward(const uint32_t* ids, i64 n_ids, const T* dy, T* dw, i64 vocab, i64 hidden) {
    std::fill(dw, dw + vocab * hidden, (T)0);
    for (i64 t = 0; t < n_ids; ++t) {
        i64 off = (i64)ids[t] * hidden;
        for (i64 i = 0; i < hidden; ++i) dw[off + i] += dy[t * hidden + i];
    }
}

// adjoint.rs:212-215
template <typename T> inline T silu_grad(T x) {
    T s = (T)1.0 / ((T)1.0 + std::exp(-x));
    return s + x * s * ((T)1.0 - s);
}

// adjoint.rs:217-251
template <typename T>
void swiglu_backward(const T* x, const T* w1, const T* w3, const T* w2, const T* dy, T* dx, T* dw1,
                     T* dw3, T* dw2, i64 tokens, i64 hidden, i64 mid) {
    std::vector<T> a(tokens * mid), c(tokens * mid), h(tokens * mid), dh(tokens * mid);
    std::vector<T> da(tokens * mid), dc(tokens * mid), dx3(tokens * hidden);
    matmul_seq(x, w1, a.data(), tokens, hidden, mid);
    matmul_seq(x, w3, c.data(), tokens, hidden, mid);
    for (i64 i = 0; i < tokens * mid; ++i) h[i] = silu(a[i]) * c[i];
    linear_backward(h.data(), w2, dy, dh.data(), dw2, (T*)nullptr, tokens, mid, hidden);
    for (i64 i = 0; i < tokens * mid; ++i) {
        da[i] = dh[i] * c[i] * silu_grad(a[i]);
        dc[i] = dh[i] * silu(a[i]);
    }
    linear_backward(x, w1, da.data(), dx, dw1, (T*)nullptr, tokens, hidden, mid);
    linear_backward(x, w3, dc.data(), dx3.data(), dw3, (T*)nullptr, tokens, hidden, mid);
    for (i64 i = 0; i < tokens * hidden; ++i) dx[i] += dx3[i];
}

// adjoint.rs:255-284 — straight-through router adjoint: on the selected
// subset dlogits = w * (g - <w, g>); dx, dgate from linear_backward.
template <typename T>
void router_backward_ste(const T* x, const T* gate, const T* d_weights, T* dx, T* dgate,
                         i64 tokens, i64 hidden, i64 n_exp, i64 k, const int64_t* forced = nullptr) {
    std::vector<T> logits(tokens * n_exp), dlog(tokens * n_exp, (T)0), w(k);
    std::vector<int64_t> idx(k);
    matmul_seq(x, gate, logits.data(), tokens, hidden, n_exp);
    for (i64 t = 0; t < tokens; ++t) {
        if (forced) {
            for (i64 i = 0; i < k; ++i) idx[i] = forced[t * k + i];
            softmax_selected(logits.data() + t * n_exp, k, idx.data(), w.data());
        } else {
            topk_softmax(logits.data() + t * n_exp, n_exp, k, idx.data(), w.data());
        }
        T dot = 0;
        for (i64 kk = 0; kk < k; ++kk) dot += w[kk] * d_weights[t * k + kk];
        for (i64 kk = 0; kk < k; ++kk)
            dlog[t * n_exp + idx[kk]] += w[kk] * (d_weights[t * k + kk] - dot);
    }
    linear_backward(x, gate, dlog.data(), dx, dgate, (T*)nullptr, tokens, hidden, n_exp);
}

// adjoint.rs:471-526 — per token t and slot k (in that order): recompute the
// expert output, d_w = <y_e, dy_t>, backprop w*dy through the SwiGLU, and
// add the single-token expert gradients into the expert's accumulators.
// Then the router STE adjoint adds into dx.
//
// Two phases with the reference's arithmetic per element:
//  1. per (t, k) pair (tokens split over threads; each pair writes only its
//     own rows): the forward recompute, d_w, dh = w2·(w·dy), da, dc and the
//     token's dx contribution — the single-token swiglu_backward, whose weight
//     gradients are the outer products x_t[p]·da[j], x_t[p]·dc[j] and
//     h[p]·(w·dy)[j] (one rounding each: 0 + a·b);
//  2. each expert's gradient rows (split over threads) add those products
//     over the expert's pairs in (t, k) order — the order the sequential loop
//     adds the per-token gradients in.
template <typename T>
void moe_backward(const T* x, const T* gate, const T* w1s, const T* w3s, const T* w2s, const T* dy,
                  T* dx, T* dgate, T* dw1s, T* dw3s, T* dw2s, i64 tokens, i64 hidden, i64 mid,
                  i64 n_exp, i64 k, const int64_t* forced = nullptr) {
    std::vector<int64_t> idx(tokens * k);
    std::vector<T> wts(tokens * k), logits(tokens * n_exp), dwts(tokens * k);
    route(x, gate, tokens, hidden, n_exp, k, idx.data(), wts.data(), logits.data(), forced);
    std::fill(dx, dx + tokens * hidden, (T)0);
    std::fill(dw1s, dw1s + n_exp * hidden * mid, (T)0);
    std::fill(dw3s, dw3s + n_exp * hidden * mid, (T)0);
    std::fill(dw2s, dw2s + n_exp * mid * hidden, (T)0);
    const i64 pairs = tokens * k;
    std::vector<T> H(pairs * mid), DA(pairs * mid), DC(pairs * mid), DYE(pairs * hidden);
    split_rows(tokens, [&](i64 t) {
        const T* xt = x + t * hidden;
        const T* dyt = dy + t * hidden;
        std::vector<T> a(mid), c(mid), ye(hidden), dh(mid), dxe(hidden), dx3(hidden);
        for (i64 kk = 0; kk < k; ++kk) {
            const i64 pr = t * k + kk;
            i64 e = idx[pr];
            T wt = wts[pr];
            const T* w1 = w1s + e * hidden * mid;
            const T* w3 = w3s + e * hidden * mid;
            const T* w2 = w2s + e * mid * hidden;
            T* h = H.data() + pr * mid;
            T* da = DA.data() + pr * mid;
            T* dc = DC.data() + pr * mid;
            T* dye = DYE.data() + pr * hidden;
            // swiglu (moe.rs:159-174) for one token
            matmul_seq(xt, w1, a.data(), 1, hidden, mid);
            matmul_seq(xt, w3, c.data(), 1, hidden, mid);
            for (i64 i = 0; i < mid; ++i) h[i] = silu(a[i]) * c[i];
            matmul_seq(h, w2, ye.data(), 1, mid, hidden);
            T s = 0;
            for (i64 i = 0; i < hidden; ++i) s += ye[i] * dyt[i];
            dwts[pr] = s;
            for (i64 i = 0; i < hidden; ++i) dye[i] = dyt[i] * wt;
            // swiglu_backward (adjoint.rs:217-251) for one token: dh, da, dc, dx
            std::fill(dh.begin(), dh.end(), (T)0);
            for (i64 j = 0; j < hidden; ++j) {
                T g = dye[j];
                for (i64 q = 0; q < mid; ++q) dh[q] += g * w2[q * hidden + j];
            }
            for (i64 i = 0; i < mid; ++i) {
                da[i] = dh[i] * c[i] * silu_grad(a[i]);
                dc[i] = dh[i] * silu(a[i]);
            }
            std::fill(dxe.begin(), dxe.end(), (T)0);
            std::fill(dx3.begin(), dx3.end(), (T)0);
            for (i64 j = 0; j < mid; ++j) {
                T g1 = da[j], g3 = dc[j];
                for (i64 q = 0; q < hidden; ++q) {
                    dxe[q] += g1 * w1[q * mid + j];
                    dx3[q] += g3 * w3[q * mid + j];
                }
            }
            for (i64 i = 0; i < hidden; ++i) dxe[i] += dx3[i];
            for (i64 i = 0; i < hidden; ++i) dx[t * hidden + i] += dxe[i];
        }
    });
    std::vector<std::vector<i64>> of_expert(n_exp);
    for (i64 pr = 0; pr < pairs; ++pr) of_expert[idx[pr]].push_back(pr);
    const i64 rows_e = hidden + mid;  // w1/w3 rows, then w2 rows, per expert
    split_rows(n_exp * rows_e, [&](i64 task) {
        const i64 e = task / rows_e, r = task % rows_e;
        if (r < hidden) {
            T* a1 = dw1s + e * hidden * mid + r * mid;
            T* a3 = dw3s + e * hidden * mid + r * mid;
            for (i64 pr : of_expert[e]) {
                const T xp = x[(pr / k) * hidden + r];
                const T* da = DA.data() + pr * mid;
                const T* dc = DC.data() + pr * mid;
                for (i64 j = 0; j < mid; ++j) {
                    a1[j] += xp * da[j];
                    a3[j] += xp * dc[j];
                }
            }
        } else {
            const i64 q = r - hidden;
            T* a2 = dw2s + e * mid * hidden + q * hidden;
            for (i64 pr : of_expert[e]) {
                const T hq = H[pr * mid + q];
                const T* dye = DYE.data() + pr * hidden;
                for (i64 j = 0; j < hidden; ++j) a2[j] += hq * dye[j];
            }
        }
    });
    std::vector<T> dxg(tokens * hidden);
    router_backward_ste(x, gate, dwts.data(), dxg.data(), dgate, tokens, hidden, n_exp, k, forced);
    for (i64 i = 0; i < tokens * hidden; ++i) dx[i] += dxg[i];
}

// adjoint.rs:530-577
template <typename T>
void layer_norm_backward(const T* x, const T* gamma, const T* dy, T* dx, T* dgamma, T* dbeta,
                         i64 rows, i64 last, T eps) {
    const T n = (T)last;
    std::fill(dgamma, dgamma + last, (T)0);
    std::fill(dbeta, dbeta + last, (T)0);
    std::vector<T> xhat(last), dxhat(last);
    for (i64 r = 0; r < rows; ++r) {
        const T* row = x + r * last;
        const T* yrow = dy + r * last;
        T s = 0;
        for (i64 i = 0; i < last; ++i) s += row[i];
        T mean = s / n;
        T v = 0;
        for (i64 i = 0; i < last; ++i) {
            T d = row[i] - mean;
            v += d * d;
        }
        T var = v / n;
        T inv = (T)1.0 / std::sqrt(var + eps);
        for (i64 i = 0; i < last; ++i) {
            xhat[i] = (row[i] - mean) * inv;
            dbeta[i] += yrow[i];
            dgamma[i] += yrow[i] * xhat[i];
            dxhat[i] = yrow[i] * gamma[i];
        }
        T sd = 0, sdx = 0;
        for (i64 i = 0; i < last; ++i) sd += dxhat[i];
        for (i64 i = 0; i < last; ++i) sdx += dxhat[i] * xhat[i];
        for (i64 i = 0; i < last; ++i)
            dx[r * last + i] = (inv / n) * (n * dxhat[i] - sd - xhat[i] * sdx);
    }
}

// adjoint.rs:287-439 — GQA adjoint: recompute q, k, v (linear_seq) and the
// rotations, store the probabilities, then dctx/dwo by linear_backward,
// the windowed softmax adjoint, dq/dk/dv, RoPE^-1 on dq and dk, and the
// three projection adjoints summed into dx (q, then k, then v).
template <typename T>
void gqa_backward(const T* x, const T* wq, const T* wk, const T* wv, const T* wo, const T* dy,
                  T* dx, T* dwq, T* dwk, T* dwv, T* dwo, i64 b, i64 s, i64 d, i64 n_heads,
                  i64 n_kv, i64 hd, double theta, i64 window) {
    i64 qd = n_heads * hd, kd = n_kv * hd, bs = b * s;
    std::vector<T> q(bs * qd), k(bs * kd), v(bs * kd), ctx(bs * qd), probs(b * n_heads * s * s, (T)0);
    matmul_seq(x, wq, q.data(), bs, d, qd);
    matmul_seq(x, wk, k.data(), bs, d, kd);
    matmul_seq(x, wv, v.data(), bs, d, kd);
    rope_all(q.data(), b, s, n_heads, hd, theta);
    rope_all(k.data(), b, s, n_kv, hd, theta);
    gqa_core(q.data(), k.data(), v.data(), ctx.data(), probs.data(), b, s, n_heads, n_kv, hd, window);
    std::vector<T> dctx(bs * qd);
    linear_backward(ctx.data(), wo, dy, dctx.data(), dwo, (T*)nullptr, bs, qd, d);
    i64 repeats = n_heads / (n_kv > 1 ? n_kv : 1);
    if (repeats < 1) repeats = 1;
    const T scale = (T)1.0 / std::sqrt((T)hd);
    std::vector<T> dq(bs * qd, (T)0), dk(bs * kd, (T)0), dv(bs * kd, (T)0);
    // One thread per (batch, kv head): it runs the query heads that share the
    // kv head in ascending order, so every dk/dv element accumulates over
    // (h, i, j) in the sequential nest's order and dq rows are disjoint.
    const i64 n_groups = n_heads / repeats;
    split_rows(b * n_groups, [&](i64 bg) {
        const i64 bi = bg / n_groups, kv_h = bg % n_groups;
        std::vector<T> dsc(s);
        for (i64 h = kv_h * repeats; h < (kv_h + 1) * repeats; ++h) {
            for (i64 i = 0; i < s; ++i) {
                i64 start = win_start(i, window);
                i64 o_off = ((bi * s + i) * n_heads + h) * hd;
                const T* arow = probs.data() + ((bi * n_heads + h) * s + i) * s;
                for (i64 j = start; j <= i; ++j) {
                    i64 v_off = ((bi * s + j) * n_kv + kv_h) * hd;
                    T dot = 0;
                    for (i64 t = 0; t < hd; ++t) dot += dctx[o_off + t] * v[v_off + t];
                    dsc[j] = dot;
                }
                T dot = 0;
                for (i64 j = start; j <= i; ++j) dot += arow[j] * dsc[j];
                for (i64 j = start; j <= i; ++j) dsc[j] = arow[j] * (dsc[j] - dot);
                for (i64 j = start; j <= i; ++j) {
                    i64 kv_off = ((bi * s + j) * n_kv + kv_h) * hd;
                    T a = arow[j];
                    for (i64 t = 0; t < hd; ++t) {
                        dv[kv_off + t] += a * dctx[o_off + t];
                        dq[o_off + t] += dsc[j] * scale * k[kv_off + t];
                        dk[kv_off + t] += dsc[j] * scale * q[o_off + t];
                    }
                }
            }
        }
    });
    rope_all(dq.data(), b, s, n_heads, hd, -theta);
    rope_all(dk.data(), b, s, n_kv, hd, -theta);
    std::vector<T> dxk(bs * d), dxv(bs * d);
    linear_backward(x, wq, dq.data(), dx, dwq, (T*)nullptr, bs, d, qd);
    linear_backward(x, wk, dk.data(), dxk.data(), dwk, (T*)nullptr, bs, d, kd);
    linear_backward(x, wv, dv.data(), dxv.data(), dwv, (T*)nullptr, bs, d, kd);
    for (i64 i = 0; i < bs * d; ++i) dx[i] += dxk[i];
    for (i64 i = 0; i < bs * d; ++i) dx[i] += dxv[i];
}

// adjoint.rs:582-722 — adjoint of the MHA in cpu.rs:235 (projections via
// cpu::linear, 8-lane order). causal=1 restricts rows to j <= i like the
// forward restatement in cpu_kernels.hpp.
template <typename T>
void attention_backward(const T* x, const T* wq, const T* wk, const T* wv, const T* wo,
                        const T* dy, T* dx, T* dwq, T* dwk, T* dwv, T* dwo, i64 b, i64 s, i64 d,
                        i64 n_heads, i64 d_head, int causal) {
    i64 bs = b * s;
    std::vector<T> q(bs * d), k(bs * d), v(bs * d), ctx(bs * d), attn(b * n_heads * s * s);
    linear<T>(x, wq, nullptr, q.data(), bs, d, d, 1);
    linear<T>(x, wk, nullptr, k.data(), bs, d, d, 1);
    linear<T>(x, wv, nullptr, v.data(), bs, d, d, 1);
    const T scale = (T)1.0 / std::sqrt((T)d_head);
    // The (batch, head) pairs below touch disjoint slices of every buffer:
    // one pair per thread, each element accumulated in the nest's order.
    split_rows(b * n_heads, [&](i64 bh) {
        const i64 bi = bh / n_heads, h = bh % n_heads;
        {
            T* sc = attn.data() + (bi * n_heads + h) * s * s;
            for (i64 i = 0; i < s; ++i)
                for (i64 j = 0; j < s; ++j) {
                    if (causal && j > i) {
                        sc[i * s + j] = -INFINITY;
                        continue;
                    }
                    T dot = 0;
                    for (i64 t = 0; t < d_head; ++t)
                        dot += q[bi * s * d + i * d + h * d_head + t] * k[bi * s * d + j * d + h * d_head + t];
                    sc[i * s + j] = dot * scale;
                }
            softmax_last<T>(sc, sc, s, s);
            for (i64 i = 0; i < s; ++i)
                for (i64 t = 0; t < d_head; ++t) {
                    T acc = 0;
                    for (i64 j = 0; j < s; ++j) acc += sc[i * s + j] * v[bi * s * d + j * d + h * d_head + t];
                    ctx[bi * s * d + i * d + h * d_head + t] = acc;
                }
        }
    });
    std::vector<T> dctx(bs * d);
    linear_backward(ctx.data(), wo, dy, dctx.data(), dwo, (T*)nullptr, bs, d, d);
    std::vector<T> dattn(attn.size()), dv(bs * d, (T)0);
    split_rows(b * n_heads, [&](i64 bh) {
        const i64 bi = bh / n_heads, h = bh % n_heads;
        {
            i64 base = (bi * n_heads + h) * s * s;
            for (i64 i = 0; i < s; ++i)
                for (i64 j = 0; j < s; ++j) {
                    T g = 0;
                    for (i64 t = 0; t < d_head; ++t) {
                        T dc = dctx[bi * s * d + i * d + h * d_head + t];
                        T vv = v[bi * s * d + j * d + h * d_head + t];
                        g += dc * vv;
                        dv[bi * s * d + j * d + h * d_head + t] += attn[base + i * s + j] * dc;
                    }
                    dattn[base + i * s + j] = g;
                }
        }
    });
    std::vector<T> dsc(attn.size());
    split_rows(b * n_heads * s, [&](i64 r) {
        const T* a = attn.data() + r * s;
        const T* g = dattn.data() + r * s;
        T dot = 0;
        for (i64 j = 0; j < s; ++j) dot += a[j] * g[j];
        for (i64 j = 0; j < s; ++j) dsc[r * s + j] = a[j] * (g[j] - dot);
    });
    std::vector<T> dq(bs * d, (T)0), dk(bs * d, (T)0);
    split_rows(b * n_heads, [&](i64 bh) {
        const i64 bi = bh / n_heads, h = bh % n_heads;
        {
            i64 base = (bi * n_heads + h) * s * s;
            for (i64 i = 0; i < s; ++i)
                for (i64 j = 0; j < s; ++j) {
                    T g = dsc[base + i * s + j] * scale;
                    for (i64 t = 0; t < d_head; ++t) {
                        T qi = q[bi * s * d + i * d + h * d_head + t];
                        T kj = k[bi * s * d + j * d + h * d_head + t];
                        dq[bi * s * d + i * d + h * d_head + t] += g * kj;
                        dk[bi * s * d + j * d + h * d_head + t] += g * qi;
                    }
                }
        }
    });
    std::vector<T> dxk(bs * d), dxv(bs * d);
    linear_backward(x, wq, dq.data(), dx, dwq, (T*)nullptr, bs, d, d);
    linear_backward(x, wk, dk.data(), dxk.data(), dwk, (T*)nullptr, bs, d, d);
    linear_backward(x, wv, dv.data(), dxv.data(), dwv, (T*)nullptr, bs, d, d);
    for (i64 i = 0; i < bs * d; ++i) dx[i] += dxk[i];
    for (i64 i = 0; i < bs * d; ++i) dx[i] += dxv[i];
}

// adjoint.rs:903-913 — LM head adjoint: linear_backward against the
// transposed table, then transpose dW back to [vocab, hidden].
template <typename T>
void lm_head_backward(const T* x, const T* w, const T* dy, T* dx, T* dw, i64 rows, i64 hidden, i64 vocab) {
    std::vector<T> wt(hidden * vocab), dwt(hidden * vocab);
    for (i64 v = 0; v < vocab; ++v)
        for (i64 p = 0; p < hidden; ++p) wt[p * vocab + v] = w[v * hidden + p];
    linear_backward(x, wt.data(), dy, dx, dwt.data(), (T*)nullptr, rows, hidden, vocab);
    for (i64 p = 0; p < hidden; ++p)
        for (i64 v = 0; v < vocab; ++v) dw[v * hidden + p] = dwt[p * vocab + v];
}

}  // namespace orc
