// ORACLE — test infrastructure only. Nothing in the product path includes,
// links or calls this file; only tests/, __graft_entry__.smoke() and
// bench.py's CPU-baseline leg use it, and only as the checker.
//
// CPU restatement of the reference's fp32 CPU kernels, templated on the
// scalar type so the same loop nests give the f32 oracle (T = float) and an
// f64 shadow for finite-difference gradient checks (T = double, the role of
// crates/catnn-compile/src/kernel/fd64.rs in the reference).
//
// Compiled with -ffp-contract=off: Rust never contracts a*b+c into an FMA,
// so every product and sum here rounds separately, in the reference's order.
//
// This file: crates/catnn-core/src/tensor.rs (LCG fill, FNV checksum) and
// crates/catnn-compile/src/kernel/cpu.rs + kernel/reference.rs.
#pragma once
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

namespace orc {

typedef int64_t i64;

template <typename T> inline T tmax(T a, T b) { return std::fmax(a, b); }

// Row partitioning across host threads, the role Rayon's par_chunks_mut plays
// in the reference (cpu.rs:39,61,188). Each output row is produced by one
// thread, so the partition never changes a value. ORACLE_THREADS caps the
// count (default: all hardware threads).
//
// The same helper also splits loops the reference runs sequentially, but
// only loops whose iterations write disjoint outputs and where each output
// element is still accumulated by one thread in the reference's order (rows
// of a GEMM, heads of attention, tokens of the MoE forward, rows of a
// weight gradient). Values are then bit-identical to the sequential loop;
// only the wall time changes. A call made from inside a parallel region
// runs sequentially (no nested thread spawning).
inline int oracle_threads() {
    const char* e = std::getenv("ORACLE_THREADS");
    int n = e ? std::atoi(e) : (int)std::thread::hardware_concurrency();
    return n < 1 ? 1 : n;
}
inline bool& in_parallel_region() {
    static thread_local bool flag = false;
    return flag;
}
template <typename F> void parallel_rows(i64 rows, F f) {
    int nt = oracle_threads();
    if (nt <= 1 || rows < 2 || in_parallel_region()) {
        for (i64 r = 0; r < rows; ++r) f(r);
        return;
    }
    if ((i64)nt > rows) nt = (int)rows;
    std::vector<std::thread> pool;
    for (int t = 0; t < nt; ++t)
        pool.emplace_back([=]() {
            in_parallel_region() = true;
            for (i64 r = t; r < rows; r += nt) f(r);
        });
    for (auto& th : pool) th.join();
}
// The oracle-only splits (loops the reference runs on one thread). With
// ORACLE_SPLIT=0 they run sequentially, so a timing run reproduces the
// reference's own threading: threads only where Rayon splits rows.
inline bool oracle_split() {
    const char* e = std::getenv("ORACLE_SPLIT");
    return !e || std::atoi(e) != 0;
}
template <typename F> void split_rows(i64 rows, F f) {
    if (!oracle_split()) {
        for (i64 r = 0; r < rows; ++r) f(r);
        return;
    }
    parallel_rows(rows, f);
}

// tensor.rs:259-268 — Tensor::lcg. state = max(seed,1); per element
// state = state*6364136223846793005 + 1 (wrapping);
// unit = (u32)(state >> 33) as f32 / u32::MAX as f32; value = unit*2 - 1.
inline void lcg_fill(float* out, i64 n, uint64_t seed) {
    uint64_t state = seed < 1 ? 1 : seed;
    const float umax = (float)4294967295u;  // u32::MAX as f32 rounds to 2^32
    for (i64 i = 0; i < n; ++i) {
        state = state * 6364136223846793005ull + 1ull;
        float unit = (float)(uint32_t)(state >> 33) / umax;
        out[i] = unit * 2.0f - 1.0f;
    }
}

// tensor.rs:279-288 — FNV-1a style mix over the f32 bit patterns.
inline uint64_t checksum(const float* x, i64 n) {
    uint64_t h = 0xcbf29ce484222325ull;
    for (i64 i = 0; i < n; ++i) {
        uint32_t bits;
        std::memcpy(&bits, &x[i], 4);
        h ^= (uint64_t)bits;
        h *= 0x100000001b3ull;
    }
    return h;
}

// cpu.rs:14-18
template <typename T> void relu(const T* x, T* y, i64 n) {
    for (i64 i = 0; i < n; ++i) y[i] = tmax(x[i], (T)0);
}

// The constant sqrt(2/pi) as the reference computes it: (2.0f32 / PI).sqrt()
template <typename T> inline T gelu_k() {
    return std::sqrt((T)2.0 / (T)3.14159265358979323846);
}

// cpu.rs:20-29 — tanh GELU, evaluation order kept:
// inner = k * (z + ((0.044715*z)*z)*z); y = (0.5*z) * (1 + tanh(inner)).
template <typename T> void gelu(const T* x, T* y, i64 n) {
    const T k = gelu_k<T>();
    for (i64 i = 0; i < n; ++i) {
        T z = x[i];
        T inner = k * (z + (T)0.044715 * z * z * z);
        y[i] = (T)0.5 * z * ((T)1.0 + std::tanh(inner));
    }
}

// cpu.rs:31-52 (and reference.rs:26-42, same arithmetic): row max by
// NaN-ignoring fold from -inf, e = exp(x - max) summed left to right,
// then multiplied by inv = 1 / max(sum, 1e-30).
template <typename T> void softmax_last(const T* x, T* y, i64 rows, i64 last) {
    parallel_rows(rows, [=](i64 r) {
        const T* in = x + r * last;
        T* out = y + r * last;
        T mx = -INFINITY;
        for (i64 i = 0; i < last; ++i) mx = tmax(mx, in[i]);
        T sum = 0;
        for (i64 i = 0; i < last; ++i) {
            out[i] = std::exp(in[i] - mx);
            sum += out[i];
        }
        T inv = (T)1.0 / tmax(sum, (T)1e-30);
        for (i64 i = 0; i < last; ++i) out[i] *= inv;
    });
}

// cpu.rs:54-78 — two-pass population variance.
template <typename T>
void layer_norm(const T* x, const T* gamma, const T* beta, T* y, i64 rows, i64 last, T eps) {
    const T n = (T)last;
    parallel_rows(rows, [=](i64 r) {
        const T* in = x + r * last;
        T* out = y + r * last;
        T s = 0;
        for (i64 i = 0; i < last; ++i) s += in[i];
        T mean = s / n;
        T v = 0;
        for (i64 i = 0; i < last; ++i) {
            T d = in[i] - mean;
            v += d * d;
        }
        T var = v / n;
        T inv = (T)1.0 / std::sqrt(var + eps);
        for (i64 i = 0; i < last; ++i) out[i] = (in[i] - mean) * inv * gamma[i] + beta[i];
    });
}

// cpu.rs:80-98 — same-length add, or b broadcast over the last dim.
template <typename T> void add(const T* a, const T* b, T* y, i64 n) {
    for (i64 i = 0; i < n; ++i) y[i] = a[i] + b[i];
}
template <typename T> void add_bias(const T* a, const T* b, T* y, i64 rows, i64 last) {
    for (i64 r = 0; r < rows; ++r)
        for (i64 j = 0; j < last; ++j) y[r * last + j] = a[r * last + j] + b[j];
}
// cpu.rs:100-109
template <typename T> void mul(const T* a, const T* b, T* y, i64 n) {
    for (i64 i = 0; i < n; ++i) y[i] = a[i] * b[i];
}

// cpu.rs:115-126 — sequential GEMM, s += a*b in p order (rows split over
// threads; each element's sum is unchanged).
template <typename T> void matmul_seq(const T* a, const T* b, T* c, i64 m, i64 k, i64 n) {
    split_rows(m, [=](i64 i) {
        const T* ai = a + i * k;
        for (i64 j = 0; j < n; ++j) {
            T s = 0;
            for (i64 p = 0; p < k; ++p) s += ai[p] * b[p * n + j];
            c[i * n + j] = s;
        }
    });
}

// cpu.rs:186-232 — the row-parallel GEMM with 8-lane accumulators.
// Lane l accumulates a[p]*b[p][j] for p = l (mod 8) over the full 8-blocks
// (a separate multiply, then add: the `wide` crate's SSE path does not fuse).
// reduce_add order: the crate's f32x8 horizontal sum is not pinned by any
// reference test (only abs-tolerance vs the sequential loop, lib.rs:99);
// this restatement sums the two 4-lane halves lane-wise, then pairs (0+2),
// (1+3), then adds those two. The scalar tail p >= 8*floor(k/8) follows.
template <typename T> T dot_row8(const T* a, const T* b, i64 k, i64 n, i64 j) {
    T acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    i64 p = 0;
    while (p + 8 <= k) {
        for (int l = 0; l < 8; ++l) {
            T prod = a[p + l] * b[(p + l) * n + j];
            acc[l] = acc[l] + prod;
        }
        p += 8;
    }
    T h0 = acc[0] + acc[4], h1 = acc[1] + acc[5], h2 = acc[2] + acc[6], h3 = acc[3] + acc[7];
    T s = (h0 + h2) + (h1 + h3);
    while (p < k) {
        s += a[p] * b[p * n + j];
        ++p;
    }
    return s;
}
template <typename T> void matmul_par(const T* a, const T* b, T* c, i64 m, i64 k, i64 n) {
    parallel_rows(m, [=](i64 i) {
        for (i64 j = 0; j < n; ++j) c[i * n + j] = dot_row8(a + i * k, b, k, n, j);
    });
}

// cpu.rs:128-184 — y = x @ w (+ bias added afterwards, row by row).
// parallel=1 is cpu::linear (8-lane), parallel=0 is cpu::linear_seq.
template <typename T>
void linear(const T* x, const T* w, const T* bias, T* y, i64 m, i64 k, i64 n, int parallel) {
    if (parallel) matmul_par(x, w, y, m, k, n);
    else matmul_seq(x, w, y, m, k, n);
    if (bias)
        for (i64 r = 0; r < m; ++r)
            for (i64 j = 0; j < n; ++j) y[r * n + j] += bias[j];
}

// reference.rs:63-85 — naive loop with the bias added to the finished sum.
template <typename T>
void ref_linear(const T* x, const T* w, const T* bias, T* y, i64 m, i64 k, i64 n) {
    for (i64 i = 0; i < m; ++i)
        for (i64 j = 0; j < n; ++j) {
            T s = 0;
            for (i64 p = 0; p < k; ++p) s += x[i * k + p] * w[p * n + j];
            if (bias) s += bias[j];
            y[i * n + j] = s;
        }
}

// cpu.rs:235-298 — MHA over x [B,S,D], projections through cpu::linear
// (8-lane order), scale 1/sqrt(d_head), softmax rows, ctx = P·V summed over
// j in order, output projection through cpu::linear.
// causal=1 is the derived restatement for the causal transformer block:
// the score row is restricted to j <= i exactly as moe.rs:105-121 does for
// GQA (masked entries get probability 0); causal=0 is the reference as-is.
template <typename T>
void attention(const T* x, const T* wq, const T* wk, const T* wv, const T* wo, T* y, i64 b,
               i64 s, i64 d, i64 n_heads, i64 d_head, int causal) {
    std::vector<T> q(b * s * d), k(b * s * d), v(b * s * d), ctx(b * s * d, (T)0);
    linear<T>(x, wq, nullptr, q.data(), b * s, d, d, 1);
    linear<T>(x, wk, nullptr, k.data(), b * s, d, d, 1);
    linear<T>(x, wv, nullptr, v.data(), b * s, d, d, 1);
    const T scale = (T)1.0 / std::sqrt((T)d_head);
    // (batch, head) pairs are independent: one per thread, own score buffer
    split_rows(b * n_heads, [&](i64 bh) {
        const i64 bi = bh / n_heads, h = bh % n_heads;
        std::vector<T> scores(s * s);
        {
            for (i64 i = 0; i < s; ++i)
                for (i64 j = 0; j < s; ++j) {
                    if (causal && j > i) {
                        scores[i * s + j] = -INFINITY;
                        continue;
                    }
                    T dot = 0;
                    for (i64 t = 0; t < d_head; ++t)
                        dot += q[bi * s * d + i * d + h * d_head + t] *
                               k[bi * s * d + j * d + h * d_head + t];
                    scores[i * s + j] = dot * scale;
                }
            softmax_last<T>(scores.data(), scores.data(), s, s);
            for (i64 i = 0; i < s; ++i)
                for (i64 t = 0; t < d_head; ++t) {
                    T acc = 0;
                    for (i64 j = 0; j < s; ++j)
                        acc += scores[i * s + j] * v[bi * s * d + j * d + h * d_head + t];
                    ctx[bi * s * d + i * d + h * d_head + t] = acc;
                }
        }
    });
    linear<T>(ctx.data(), wo, nullptr, y, b * s, d, d, 1);
}

}  // namespace orc
