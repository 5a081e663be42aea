// Row kernels: softmax and its adjoint, fused softmax cross-entropy
// (forward + backward in one pass pair), MSE, LayerNorm and RMSNorm with
// their adjoints. One CTA per row; reductions are block-wide with a fixed
// order (deterministic run to run). Weight-vector gradients (dgamma,
// dbeta, dw) are column reductions done in row chunks, then chunk order:
// no atomics, so every run gives the same bits.
#include <mutex>
#include <type_traits>

#include "ops.cuh"

namespace catnn {

static int row_threads(i64 last) {
    if (last <= 64) return 32;
    if (last <= 256) return 64;
    if (last <= 1024) return 128;
    return 256;
}

// ---------------------------------------------------------------- softmax
// cpu.rs:31-52: y = exp(x - max) * (1 / max(sum, 1e-30)).
template <typename T>
__global__ void k_softmax(const T* __restrict__ x, T* __restrict__ y, i64 last) {
    __shared__ float red[32];
    const T* in = x + blockIdx.x * last;
    T* out = y + blockIdx.x * last;
    float mx = -INFINITY;
    for (i64 i = threadIdx.x; i < last; i += blockDim.x) mx = fmaxf(mx, ld(in + i));
    mx = block_max(mx, red);
    float s = 0.f;
    for (i64 i = threadIdx.x; i < last; i += blockDim.x) s += expf(ld(in + i) - mx);
    s = block_sum(s, red);
    float inv = 1.0f / fmaxf(s, 1e-30f);
    for (i64 i = threadIdx.x; i < last; i += blockDim.x) st(out + i, expf(ld(in + i) - mx) * inv);
}

// adjoint.rs:92-104: dx = y * (dy - <y, dy>).
template <typename T>
__global__ void k_softmax_bwd(const T* __restrict__ y, const T* __restrict__ dy, T* __restrict__ dx, i64 last) {
    __shared__ float red[32];
    i64 o = blockIdx.x * last;
    float d = 0.f;
    for (i64 i = threadIdx.x; i < last; i += blockDim.x) d += ld(y + o + i) * ld(dy + o + i);
    d = block_sum(d, red);
    for (i64 i = threadIdx.x; i < last; i += blockDim.x) st(dx + o + i, ld(y + o + i) * (ld(dy + o + i) - d));
}

void softmax_fwd(Context* c, const void* x, void* y, i64 rows, i64 last, int dtype) {
    if (rows <= 0 || last <= 0) return;
    int t = row_threads(last);
    if (dtype == CATNN_BF16) k_softmax<<<rows, t, 0, c->stream>>>((const bf16*)x, (bf16*)y, last);
    else k_softmax<<<rows, t, 0, c->stream>>>((const float*)x, (float*)y, last);
    launched(c);
}
void softmax_bwd(Context* c, const void* y, const void* dy, void* dx, i64 rows, i64 last, int dtype) {
    if (rows <= 0 || last <= 0) return;
    int t = row_threads(last);
    if (dtype == CATNN_BF16) k_softmax_bwd<<<rows, t, 0, c->stream>>>((const bf16*)y, (const bf16*)dy, (bf16*)dx, last);
    else k_softmax_bwd<<<rows, t, 0, c->stream>>>((const float*)y, (const float*)dy, (float*)dx, last);
    launched(c);
}

// ---------------------------------------------------------- cross-entropy
// adjoint.rs:123-145, fused. Pass 1 (online max/sum, one read of the row),
// then dlogits = p / rows with 1/rows taken off at the target, and the row
// loss -ln(max(p_t, 1e-30)) into a per-row buffer that a single CTA sums in
// row order.
// e^x for the row kernels: on bf16 logits 2^(x·log2 e) with the MUFU
// ex2.approx instruction (relative error ~1e-7, far below bf16's 4e-3);
// fp32 logits keep expf (the fp32 path is held to the reference at 1e-5).
template <typename T>
__device__ __forceinline__ float row_exp(float x) {
    if constexpr (sizeof(T) == 2) {
        float y;
        asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x * 1.4426950408889634f));
        return y;
    } else {
        return expf(x);
    }
}

// V-wide accesses along the row (16 bytes when aligned); the running
// (max, sum) pair is rescaled once per vector.
template <typename T, int V>
__global__ void k_xent_rows(const T* __restrict__ logits, const uint32_t* __restrict__ tg, i64 vocab, i64 denom,
                            T* __restrict__ dlog, float* __restrict__ row_loss, int* __restrict__ err) {
    __shared__ float red[32];
    __shared__ float sh_m, sh_s;
    i64 r = blockIdx.x;
    const T* in = logits + r * vocab;
    T* out = dlog + r * vocab;
    // online max/sum per thread, then merge
    float m = -INFINITY, s = 0.f;
    for (i64 i = (i64)threadIdx.x * V; i < vocab; i += (i64)blockDim.x * V) {
        float x[V];
        ldv<T, V>(in + i, x);
        float lm = x[0];
#pragma unroll
        for (int j = 1; j < V; ++j) lm = fmaxf(lm, x[j]);
        if (lm > m) {
            s = s * row_exp<T>(m - lm);
            m = lm;
        }
#pragma unroll
        for (int j = 0; j < V; ++j) s += row_exp<T>(x[j] - m);
    }
    float gm = block_max(m, red);
    float sc = (m == -INFINITY) ? 0.f : s * row_exp<T>(m - gm);
    float gs = block_sum(sc, red);
    if (threadIdx.x == 0) {
        sh_m = gm;
        sh_s = gs;
    }
    __syncthreads();
    const float inv = 1.0f / fmaxf(sh_s, 1e-30f);
    const float rinv = 1.0f / (float)denom;
    const uint32_t t = tg[r];
    const bool bad = (i64)t >= vocab;
    if (bad && threadIdx.x == 0 && err) atomicExch(err, 1);
    for (i64 i = (i64)threadIdx.x * V; i < vocab; i += (i64)blockDim.x * V) {
        float x[V], o[V];
        ldv<T, V>(in + i, x);
#pragma unroll
        for (int j = 0; j < V; ++j) {
            float p = row_exp<T>(x[j] - sh_m) * inv;
            float d = p * rinv;
            if (i + j == (i64)t) {
                d = d - rinv;
                row_loss[r] = -logf(fmaxf(p, 1e-30f));
            }
            o[j] = d;
        }
        stv<T, V>(out + i, o);
    }
    if (bad && threadIdx.x == 0) row_loss[r] = 0.f;
}

// One CTA per row; vector width by dtype and alignment of both row tensors.
static void launch_xent_rows(Context* c, const void* logits, const uint32_t* targets, i64 rows, i64 vocab,
                             void* dlogits, int dtype, float* rl, int* err, i64 denom) {
    int t = row_threads(vocab);
    int v = dtype == CATNN_BF16 ? 8 : 4;
    if (vocab % v || !aligned_to(logits, 16) || !aligned_to(dlogits, 16)) v = 1;
    if (dtype == CATNN_BF16) {
        auto x = (const bf16*)logits;
        auto d = (bf16*)dlogits;
        if (v == 8) k_xent_rows<bf16, 8><<<rows, t, 0, c->stream>>>(x, targets, vocab, denom, d, rl, err);
        else k_xent_rows<bf16, 1><<<rows, t, 0, c->stream>>>(x, targets, vocab, denom, d, rl, err);
    } else {
        auto x = (const float*)logits;
        auto d = (float*)dlogits;
        if (v == 4) k_xent_rows<float, 4><<<rows, t, 0, c->stream>>>(x, targets, vocab, denom, d, rl, err);
        else k_xent_rows<float, 1><<<rows, t, 0, c->stream>>>(x, targets, vocab, denom, d, rl, err);
    }
}

__global__ void k_sum_rows_mean(const float* __restrict__ v, i64 n, float* __restrict__ out, i64 denom) {
    __shared__ float red[32];
    float s = 0.f;
    // fixed assignment: thread t sums elements t, t+B, ... in order
    for (i64 i = threadIdx.x; i < n; i += blockDim.x) s += v[i];
    s = block_sum(s, red);
    if (threadIdx.x == 0) *out = s / (float)denom;
}

void xent_fwdbwd(Context* c, const void* logits, const uint32_t* targets, i64 rows, i64 vocab, float* loss,
                 void* dlogits, int dtype, int* err, i64 denom) {
    if (rows <= 0 || vocab <= 0) return;
    if (denom <= 0) denom = rows;
    float* rl = (float*)c->scratch_for(rows * 4);
    launch_xent_rows(c, logits, targets, rows, vocab, dlogits, dtype, rl, err, denom);
    k_sum_rows_mean<<<1, 1024, 0, c->stream>>>(rl, rows, loss, denom);
    launched(c, 2);
}

// adjoint.rs:106-119: loss = Σ e² / n, d = 2e/n.
__global__ void k_mse(const float* __restrict__ p, const float* __restrict__ t, i64 n, float* __restrict__ loss,
                      float* __restrict__ d) {
    __shared__ float red[32];
    float s = 0.f, fn = (float)n;
    for (i64 i = threadIdx.x; i < n; i += blockDim.x) {
        float e = p[i] - t[i];
        s += e * e;
        d[i] = 2.0f * e / fn;
    }
    s = block_sum(s, red);
    if (threadIdx.x == 0) *loss = s / fn;
}
void mse_fwdbwd(Context* c, const float* pred, const float* target, i64 n, float* loss, float* d) {
    if (n <= 0) return;
    k_mse<<<1, 1024, 0, c->stream>>>(pred, target, n, loss, d);
    launched(c);
}

// ---------------------------------------------------------------- LayerNorm
// cpu.rs:54-78: two-pass population variance; y = (x-mean)*inv*g + b.
template <typename T>
__global__ void k_ln_fwd(const T* __restrict__ x, const float* __restrict__ g, const float* __restrict__ b,
                         T* __restrict__ y, i64 last, float eps) {
    __shared__ float red[32];
    const T* in = x + blockIdx.x * last;
    float s = 0.f;
    for (i64 i = threadIdx.x; i < last; i += blockDim.x) s += ld(in + i);
    float mean = block_sum(s, red) / (float)last;
    float v = 0.f;
    for (i64 i = threadIdx.x; i < last; i += blockDim.x) {
        float d = ld(in + i) - mean;
        v += d * d;
    }
    float var = block_sum(v, red) / (float)last;
    float inv = 1.0f / sqrtf(var + eps);
    for (i64 i = threadIdx.x; i < last; i += blockDim.x)
        st(y + blockIdx.x * last + i, (ld(in + i) - mean) * inv * g[i] + b[i]);
}

// adjoint.rs:530-577, row part: dx = (inv/n)(n·dxhat - Σdxhat - xhat·Σ(dxhat·xhat)),
// dxhat = dy·γ. Saves mean/inv per row for the column pass.
template <typename T>
__global__ void k_ln_bwd_rows(const T* __restrict__ x, const float* __restrict__ g, const T* __restrict__ dy,
                              T* __restrict__ dx, float* __restrict__ stats, i64 last, float eps) {
    __shared__ float red[32];
    i64 o = blockIdx.x * last;
    float s = 0.f;
    for (i64 i = threadIdx.x; i < last; i += blockDim.x) s += ld(x + o + i);
    float n = (float)last;
    float mean = block_sum(s, red) / n;
    float v = 0.f;
    for (i64 i = threadIdx.x; i < last; i += blockDim.x) {
        float d = ld(x + o + i) - mean;
        v += d * d;
    }
    float inv = 1.0f / sqrtf(block_sum(v, red) / n + eps);
    float sd = 0.f, sdx = 0.f;
    for (i64 i = threadIdx.x; i < last; i += blockDim.x) {
        float xh = (ld(x + o + i) - mean) * inv;
        float dxh = ld(dy + o + i) * g[i];
        sd += dxh;
        sdx += dxh * xh;
    }
    sd = block_sum(sd, red);
    sdx = block_sum(sdx, red);
    for (i64 i = threadIdx.x; i < last; i += blockDim.x) {
        float xh = (ld(x + o + i) - mean) * inv;
        float dxh = ld(dy + o + i) * g[i];
        st(dx + o + i, (inv / n) * (n * dxh - sd - xh * sdx));
    }
    if (threadIdx.x == 0) {
        stats[2 * blockIdx.x] = mean;
        stats[2 * blockIdx.x + 1] = inv;
    }
}

// Rows per column-partial chunk: 128, or fewer when the rows are few, so
// that the chunk grid still puts about four CTAs on every SM.
static int col_chunk_rows(const Context* c, i64 rows, i64 last) {
    const i64 gx = cdiv(last, 128);
    const i64 want = cdiv((i64)c->sm_count * 4, gx);
    i64 cr = cdiv(rows, want);
    if (cr < 16) cr = 16;
    if (cr > 128) cr = 128;
    return (int)cr;
}
// Column partials for dgamma (Σ dy·xhat) and dbeta (Σ dy) over a chunk of rows.
template <typename T>
__global__ void k_ln_cols(const T* __restrict__ x, const T* __restrict__ dy, const float* __restrict__ stats,
                          i64 rows, i64 last, float* __restrict__ pg, float* __restrict__ pb, int crows) {
    i64 j = blockIdx.x * (i64)blockDim.x + threadIdx.x;
    if (j >= last) return;
    i64 r0 = (i64)blockIdx.y * crows, r1 = min(rows, r0 + crows);
    float sg = 0.f, sb = 0.f;
#pragma unroll 8
    for (i64 r = r0; r < r1; ++r) {
        float d = ld(dy + r * last + j);
        float xh = (ld(x + r * last + j) - stats[2 * r]) * stats[2 * r + 1];
        sg += d * xh;
        sb += d;
    }
    pg[(i64)blockIdx.y * last + j] = sg;
    if (pb) pb[(i64)blockIdx.y * last + j] = sb;
}
__global__ void k_cols_final(const float* __restrict__ p, int chunks, i64 last, float* __restrict__ out, int acc) {
    i64 j = blockIdx.x * (i64)blockDim.x + threadIdx.x;
    if (j >= last) return;
    float s = 0.f;
#pragma unroll 8
    for (int ch = 0; ch < chunks; ++ch) s += p[(i64)ch * last + j];
    out[j] = acc ? out[j] + s : s;
}

void layernorm_fwd(Context* c, const void* x, const float* g, const float* b, void* y, i64 rows, i64 last,
                   float eps, int dtype) {
    if (rows <= 0 || last <= 0) return;
    int t = row_threads(last);
    if (dtype == CATNN_BF16) k_ln_fwd<<<rows, t, 0, c->stream>>>((const bf16*)x, g, b, (bf16*)y, last, eps);
    else k_ln_fwd<<<rows, t, 0, c->stream>>>((const float*)x, g, b, (float*)y, last, eps);
    launched(c);
}

void layernorm_bwd(Context* c, const void* x, const float* g, const void* dy, void* dx, float* dg, float* db,
                   i64 rows, i64 last, float eps, int dtype) {
    if (last <= 0) return;
    if (rows <= 0) {
        if (dg) CUDA_OK(cudaMemsetAsync(dg, 0, last * 4, c->stream));
        if (db) CUDA_OK(cudaMemsetAsync(db, 0, last * 4, c->stream));
        return;
    }
    const int crows = col_chunk_rows(c, rows, last);
    int chunks = cdiv(rows, crows);
    size_t need = (size_t)rows * 2 * 4 + (size_t)chunks * last * 4 * 2;
    float* stats = (float*)c->scratch_for(need);
    float* pg = stats + rows * 2;
    float* pb = pg + (i64)chunks * last;
    int t = row_threads(last);
    dim3 gc(cdiv(last, 128), chunks);
    if (dtype == CATNN_BF16) {
        k_ln_bwd_rows<<<rows, t, 0, c->stream>>>((const bf16*)x, g, (const bf16*)dy, (bf16*)dx, stats, last, eps);
        k_ln_cols<<<gc, 128, 0, c->stream>>>((const bf16*)x, (const bf16*)dy, stats, rows, last, pg, pb, crows);
    } else {
        k_ln_bwd_rows<<<rows, t, 0, c->stream>>>((const float*)x, g, (const float*)dy, (float*)dx, stats, last, eps);
        k_ln_cols<<<gc, 128, 0, c->stream>>>((const float*)x, (const float*)dy, stats, rows, last, pg, pb, crows);
    }
    if (dg) k_cols_final<<<cdiv(last, 128), 128, 0, c->stream>>>(pg, chunks, last, dg, 0);
    if (db) k_cols_final<<<cdiv(last, 128), 128, 0, c->stream>>>(pb, chunks, last, db, 0);
    launched(c, 2 + (dg ? 1 : 0) + (db ? 1 : 0));
}

// ---------------------------------------------------------------- RMSNorm
// moe.rs:17-32: y = x * (1/sqrt(mean(x²)+eps)) * w.
template <typename T>
__global__ void k_rms_fwd(const T* __restrict__ x, const float* __restrict__ w, T* __restrict__ y, i64 last, float eps) {
    __shared__ float red[32];
    const T* in = x + blockIdx.x * last;
    float s = 0.f;
    for (i64 i = threadIdx.x; i < last; i += blockDim.x) {
        float v = ld(in + i);
        s += v * v;
    }
    float inv = 1.0f / sqrtf(block_sum(s, red) / (float)last + eps);
    for (i64 i = threadIdx.x; i < last; i += blockDim.x) st(y + blockIdx.x * last + i, ld(in + i) * inv * w[i]);
}

// adjoint.rs:148-193, row part: dx = dy·inv·w + dms·(2x/n) with
// dms = Σ(dy·x·w) · (-0.5) · (ms+eps)^-1.5; optional + dres (residual).
template <typename T>
__global__ void k_rms_bwd_rows(const T* __restrict__ x, const float* __restrict__ w, const T* __restrict__ dy,
                               const T* __restrict__ dres, T* __restrict__ dx, float* __restrict__ invs, i64 last,
                               float eps) {
    __shared__ float red[32];
    i64 o = blockIdx.x * last;
    float n = (float)last;
    float s = 0.f, di = 0.f;
    for (i64 i = threadIdx.x; i < last; i += blockDim.x) {
        float v = ld(x + o + i);
        s += v * v;
        di += ld(dy + o + i) * v * w[i];
    }
    float ms = block_sum(s, red) / n;
    di = block_sum(di, red);
    float inv = 1.0f / sqrtf(ms + eps);
    float dms = di * -0.5f * powf(ms + eps, -1.5f);
    for (i64 i = threadIdx.x; i < last; i += blockDim.x) {
        float v = ld(x + o + i);
        float r = ld(dy + o + i) * inv * w[i] + dms * (2.0f * v / n);
        if (dres) r += ld(dres + o + i);
        st(dx + o + i, r);
    }
    if (threadIdx.x == 0) invs[blockIdx.x] = inv;
}

template <typename T>
__global__ void k_rms_cols(const T* __restrict__ x, const T* __restrict__ dy, const float* __restrict__ invs, i64 rows,
                           i64 last, float* __restrict__ pw, int crows) {
    i64 j = blockIdx.x * (i64)blockDim.x + threadIdx.x;
    if (j >= last) return;
    i64 r0 = (i64)blockIdx.y * crows, r1 = min(rows, r0 + crows);
    float sw = 0.f;
#pragma unroll 8
    for (i64 r = r0; r < r1; ++r) sw += ld(dy + r * last + j) * ld(x + r * last + j) * invs[r];
    pw[(i64)blockIdx.y * last + j] = sw;
}

void rmsnorm_fwd(Context* c, const void* x, const float* w, void* y, i64 rows, i64 last, float eps, int dtype) {
    if (rows <= 0 || last <= 0) return;
    int t = row_threads(last);
    if (dtype == CATNN_BF16) k_rms_fwd<<<rows, t, 0, c->stream>>>((const bf16*)x, w, (bf16*)y, last, eps);
    else k_rms_fwd<<<rows, t, 0, c->stream>>>((const float*)x, w, (float*)y, last, eps);
    launched(c);
}

void rmsnorm_bwd(Context* c, const void* x, const float* w, const void* dy, void* dx, float* dw, i64 rows, i64 last,
                 float eps, int dtype, bool dw_accumulate, const void* dres) {
    if (last <= 0) return;
    if (rows <= 0) {
        if (dw && !dw_accumulate) CUDA_OK(cudaMemsetAsync(dw, 0, last * 4, c->stream));
        return;
    }
    const int crows = col_chunk_rows(c, rows, last);
    int chunks = cdiv(rows, crows);
    float* invs = (float*)c->scratch_for((size_t)rows * 4 + (size_t)chunks * last * 4);
    float* pw = invs + rows;
    int t = row_threads(last);
    dim3 gc(cdiv(last, 128), chunks);
    if (dtype == CATNN_BF16) {
        k_rms_bwd_rows<<<rows, t, 0, c->stream>>>((const bf16*)x, w, (const bf16*)dy, (const bf16*)dres, (bf16*)dx, invs, last, eps);
        if (dw) k_rms_cols<<<gc, 128, 0, c->stream>>>((const bf16*)x, (const bf16*)dy, invs, rows, last, pw, crows);
    } else {
        k_rms_bwd_rows<<<rows, t, 0, c->stream>>>((const float*)x, w, (const float*)dy, (const float*)dres, (float*)dx, invs, last, eps);
        if (dw) k_rms_cols<<<gc, 128, 0, c->stream>>>((const float*)x, (const float*)dy, invs, rows, last, pw, crows);
    }
    if (dw) k_cols_final<<<cdiv(last, 128), 128, 0, c->stream>>>(pw, chunks, last, dw, dw_accumulate ? 1 : 0);
    launched(c, dw ? 3 : 1);
}

}  // namespace catnn

// ------------------------------------------------ mixed-storage RMSNorm
// The training step keeps the residual stream in fp32 and feeds the
// GEMMs bf16: the forward reads fp32 x and writes bf16 xn; the backward
// reads fp32 x, a gradient in either storage, adds the residual gradient
// and writes the fp32 stream plus (optionally) a bf16 copy for the next GEMM.
namespace catnn {

template <typename TX, typename TY>
__global__ void k_rms_fwd_mx(const TX* __restrict__ x, const float* __restrict__ w, TY* __restrict__ y, i64 last,
                             float eps) {
    __shared__ float red[32];
    const TX* in = x + blockIdx.x * last;
    float s = 0.f;
    for (i64 i = threadIdx.x; i < last; i += blockDim.x) {
        float v = ld(in + i);
        s += v * v;
    }
    float inv = 1.0f / sqrtf(block_sum(s, red) / (float)last + eps);
    for (i64 i = threadIdx.x; i < last; i += blockDim.x) st(y + blockIdx.x * last + i, ld(in + i) * inv * w[i]);
}

template <typename TX, typename TG, typename TC>
__global__ void k_rms_bwd_mx(const TX* __restrict__ x, const float* __restrict__ w, const TG* __restrict__ dy,
                             const float* __restrict__ dres, float* __restrict__ dx, TC* __restrict__ copy,
                             float* __restrict__ invs, i64 last, float eps) {
    __shared__ float red[32];
    i64 o = blockIdx.x * last;
    float n = (float)last;
    float s = 0.f, di = 0.f;
    for (i64 i = threadIdx.x; i < last; i += blockDim.x) {
        float v = ld(x + o + i);
        s += v * v;
        di += ld(dy + o + i) * v * w[i];
    }
    float ms = block_sum(s, red) / n;
    di = block_sum(di, red);
    float inv = 1.0f / sqrtf(ms + eps);
    float dms = di * -0.5f * powf(ms + eps, -1.5f);
    for (i64 i = threadIdx.x; i < last; i += blockDim.x) {
        float v = ld(x + o + i);
        float r = ld(dy + o + i) * inv * w[i] + dms * (2.0f * v / n);
        if (dres) r += dres[o + i];
        dx[o + i] = r;
        if (copy) st(copy + o + i, r);
    }
    if (threadIdx.x == 0) invs[blockIdx.x] = inv;
}

template <typename TX, typename TG>
__global__ void k_rms_cols_mx(const TX* __restrict__ x, const TG* __restrict__ dy, const float* __restrict__ invs, i64 rows,
                              i64 last, float* __restrict__ pw, int crows) {
    i64 j = blockIdx.x * (i64)blockDim.x + threadIdx.x;
    if (j >= last) return;
    i64 r0 = (i64)blockIdx.y * crows, r1 = min(rows, r0 + crows);
    float sw = 0.f;
#pragma unroll 8
    for (i64 r = r0; r < r1; ++r) sw += ld(dy + r * last + j) * ld(x + r * last + j) * invs[r];
    pw[(i64)blockIdx.y * last + j] = sw;
}

// MoE input of a layer in one pass over x (fp32 [rows, NC*1024]): the RMSNorm
// y = x·inv·w (moe.rs:317; k_rms_fwd_mx's expression), stored as bf16 for the
// expert GEMMs and as fp32 for the router, and the router logits y·gate
// (gate fp32 [last, E], E <= 32) from registers: each of the 256 threads
// holds 4·NC columns and their gate rows for every row the CTA visits.
template <int NC, int EB>
__global__ void __launch_bounds__(256) k_rms_router(const float* __restrict__ x, const float* __restrict__ w,
                                                    const float* __restrict__ gate, int E, i64 rows, float eps,
                                                    bf16* __restrict__ y16, float* __restrict__ y32,
                                                    float* __restrict__ logits) {
    constexpr int last = NC * 1024;
    __shared__ float red[8];
    __shared__ float lred[8][EB];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float wv[NC][4], gv[NC][4][EB];
#pragma unroll
    for (int g = 0; g < NC; ++g) {
        const int c = g * 1024 + threadIdx.x * 4;
        ldv<float, 4>(w + c, wv[g]);
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int e = 0; e < EB; ++e) gv[g][u][e] = e < E ? gate[(i64)(c + u) * E + e] : 0.f;
    }
    // two rows per pass (r and r + gridDim.x): their loads are in flight
    // together and they share the block's barriers; each row's arithmetic
    // (and reduction order) is the one-row computation's
    __shared__ float red2[8];
    __shared__ float lred2[8][EB];
    for (i64 r = blockIdx.x; r < rows; r += 2 * (i64)gridDim.x) {
        const i64 r2 = r + gridDim.x;
        const bool two = r2 < rows;
        float xv[NC][4], xw[NC][4];
        float ss = 0.f, ss2 = 0.f;
#pragma unroll
        for (int g = 0; g < NC; ++g) {
            ldv<float, 4>(x + r * last + g * 1024 + threadIdx.x * 4, xv[g]);
            if (two) ldv<float, 4>(x + r2 * last + g * 1024 + threadIdx.x * 4, xw[g]);
            else
#pragma unroll
                for (int u = 0; u < 4; ++u) xw[g][u] = 0.f;
        }
#pragma unroll
        for (int g = 0; g < NC; ++g)
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                ss += xv[g][u] * xv[g][u];
                ss2 += xw[g][u] * xw[g][u];
            }
        ss = warp_sum(ss);
        ss2 = warp_sum(ss2);
        if (lane == 0) {
            red[warp] = ss;
            red2[warp] = ss2;
        }
        __syncthreads();
        float tot = 0.f, tot2 = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            tot += red[k];
            tot2 += red2[k];
        }
        const float inv = 1.0f / sqrtf(tot / (float)last + eps);
        const float inv2 = 1.0f / sqrtf(tot2 / (float)last + eps);
        float lg[EB], lg2[EB];
#pragma unroll
        for (int e = 0; e < EB; ++e) lg[e] = lg2[e] = 0.f;
#pragma unroll
        for (int g = 0; g < NC; ++g) {
            float yv[4], yw[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                yv[u] = xv[g][u] * inv * wv[g][u];
                yw[u] = xw[g][u] * inv2 * wv[g][u];
#pragma unroll
                for (int e = 0; e < EB; ++e) {
                    lg[e] = fmaf(yv[u], gv[g][u][e], lg[e]);
                    lg2[e] = fmaf(yw[u], gv[g][u][e], lg2[e]);
                }
            }
            const i64 o = r * last + g * 1024 + threadIdx.x * 4;
            stv<float, 4>(y32 + o, yv);
            stv<bf16, 4>(y16 + o, yv);
            if (two) {
                const i64 o2 = r2 * last + g * 1024 + threadIdx.x * 4;
                stv<float, 4>(y32 + o2, yw);
                stv<bf16, 4>(y16 + o2, yw);
            }
        }
#pragma unroll
        for (int e = 0; e < EB; ++e) {
            lg[e] = warp_sum(lg[e]);
            lg2[e] = warp_sum(lg2[e]);
        }
        if (lane == 0)
#pragma unroll
            for (int e = 0; e < EB; ++e) {
                lred[warp][e] = lg[e];
                lred2[warp][e] = lg2[e];
            }
        __syncthreads();
        if (threadIdx.x < E) {
            float t = 0.f;
#pragma unroll
            for (int k = 0; k < 8; ++k) t += lred[k][threadIdx.x];
            logits[r * E + threadIdx.x] = t;
        } else if (two && threadIdx.x >= 32 && threadIdx.x < 32 + E) {
            const int e = threadIdx.x - 32;
            float t = 0.f;
#pragma unroll
            for (int k = 0; k < 8; ++k) t += lred2[k][e];
            logits[r2 * E + e] = t;
        }
        __syncthreads();  // red / lred are rewritten by the next pass
    }
}

// Warp-level halving exchange: lanes whose bit `off` is set keep the upper N
// of their 2N partial sums and send the lower N (the others the reverse), so
// each step halves the values a lane holds with N shuffles.
template <int N>
__device__ __forceinline__ void xchg_half(float* v, int lane, int off) {
    const bool up = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const float send = up ? v[i] : v[i + N];
        const float keep = up ? v[i + N] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
}

// The same outputs as k_rms_router<1, 8> (width 1024, E <= 8) with one warp
// per row: each lane holds 32 values of the row (8 float4 chunks 128 columns
// apart), the row sum is a warp reduction, and the gate sits expert-major in
// shared memory (a warp's float4 reads of one expert's row are consecutive).
// The 8 logit partials are summed over the warp by three halving exchanges
// and two shuffles (9 shuffles instead of 8 x 5). Persistent CTAs of 8 warps.
__global__ void __launch_bounds__(256) k_rms_router_warp(const float* __restrict__ x, const float* __restrict__ w,
                                                         const float* __restrict__ gate, int E, i64 rows, float eps,
                                                         bf16* __restrict__ y16, float* __restrict__ y32,
                                                         float* __restrict__ logits) {
    __shared__ __align__(16) float gs[8][1024];
    __shared__ __align__(16) float ws[1024];
    for (int i = threadIdx.x; i < 8 * 1024; i += 256) {
        const int e = i >> 10, c = i & 1023;
        gs[e][c] = e < E ? gate[(i64)c * E + e] : 0.f;
    }
    for (int i = threadIdx.x; i < 1024; i += 256) ws[i] = w[i];
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int my_e = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
    for (i64 r = (i64)blockIdx.x * 8 + warp; r < rows; r += (i64)gridDim.x * 8) {
        const float* xr = x + r * 1024;
        float v[8][4];
#pragma unroll
        for (int k = 0; k < 8; ++k) ldv<float, 4>(xr + k * 128 + lane * 4, v[k]);
        float ss = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k)
#pragma unroll
            for (int u = 0; u < 4; ++u) ss += v[k][u] * v[k][u];
        const float inv = 1.0f / sqrtf(warp_sum(ss) / 1024.f + eps);
        float lg[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) lg[e] = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int c = k * 128 + lane * 4;
            const float4 wq = *(const float4*)&ws[c];
            float yv[4] = {v[k][0] * inv * wq.x, v[k][1] * inv * wq.y, v[k][2] * inv * wq.z, v[k][3] * inv * wq.w};
            stv<float, 4>(y32 + r * 1024 + c, yv);
            stv<bf16, 4>(y16 + r * 1024 + c, yv);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float4 g = *(const float4*)&gs[e][c];
                lg[e] = fmaf(yv[0], g.x, lg[e]);
                lg[e] = fmaf(yv[1], g.y, lg[e]);
                lg[e] = fmaf(yv[2], g.z, lg[e]);
                lg[e] = fmaf(yv[3], g.w, lg[e]);
            }
        }
        xchg_half<4>(lg, lane, 16);
        xchg_half<2>(lg, lane, 8);
        xchg_half<1>(lg, lane, 4);
        float t = lg[0];
        t += __shfl_xor_sync(0xffffffffu, t, 2);
        t += __shfl_xor_sync(0xffffffffu, t, 1);
        if ((lane & 3) == 0 && my_e < E) logits[r * E + my_e] = t;
    }
}

bool rms_router_fused(Context* c, const float* x, const float* w, const float* gate, i64 E, i64 rows, i64 last,
                      float eps, bf16* y16, float* y32, float* logits) {
    const int nc = (int)(last / 1024);
    if (rows <= 0 || last % 1024 != 0 || nc < 1 || nc > 2 || E < 1 || E > 16) return false;
    if (!aligned_to(x, 16) || !aligned_to(w, 16) || !aligned_to(y16, 8) || !aligned_to(y32, 16)) return false;
    if (nc == 1 && E <= 8) {
        const int g8 = (int)std::min<i64>(cdiv(rows, 8), (i64)c->sm_count * 3);  // 3 CTAs fit an SM (80 registers)
        k_rms_router_warp<<<g8, 256, 0, c->stream>>>(x, w, gate, (int)E, rows, eps, y16, y32, logits);
        launched(c);
        return true;
    }
    const int grid = (int)std::min<i64>(rows, (i64)c->sm_count * 8);
    if (nc == 1 && E <= 8) k_rms_router<1, 8><<<grid, 256, 0, c->stream>>>(x, w, gate, (int)E, rows, eps, y16, y32, logits);
    else if (nc == 1) k_rms_router<1, 16><<<grid, 256, 0, c->stream>>>(x, w, gate, (int)E, rows, eps, y16, y32, logits);
    else if (E <= 8) k_rms_router<2, 8><<<grid, 256, 0, c->stream>>>(x, w, gate, (int)E, rows, eps, y16, y32, logits);
    else k_rms_router<2, 16><<<grid, 256, 0, c->stream>>>(x, w, gate, (int)E, rows, eps, y16, y32, logits);
    launched(c);
    return true;
}

// fp32 x -> bf16 y at widths NV·128 (k_rms_fwd_mx's expression): one warp
// per row, each lane holding NV float4 chunks 128 columns apart, so x is read
// once and the row sum needs only warp shuffles; 8 rows per CTA.
template <int NV>
__global__ void __launch_bounds__(256) k_rms_fwd_warp(const float* __restrict__ x, const float* __restrict__ w,
                                                      bf16* __restrict__ y, i64 rows, float eps) {
    constexpr int last = NV * 128;
    const int lane = threadIdx.x & 31;
    const i64 r = (i64)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (r >= rows) return;  // warp-uniform; no block barrier below
    const float* in = x + r * last;
    float v[NV][4];
#pragma unroll
    for (int k = 0; k < NV; ++k) ldv<float, 4>(in + k * 128 + lane * 4, v[k]);
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k)
#pragma unroll
        for (int u = 0; u < 4; ++u) s += v[k][u] * v[k][u];
    const float inv = 1.0f / sqrtf(warp_sum(s) / (float)last + eps);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        float wv[4], o[4];
        ldv<float, 4>(w + k * 128 + lane * 4, wv);
#pragma unroll
        for (int u = 0; u < 4; ++u) o[u] = v[k][u] * inv * wv[u];
        stv<bf16, 4>(y + r * last + k * 128 + lane * 4, o);
    }
}

void rmsnorm_fwd_mixed(Context* c, const void* x, int x_dtype, const float* w, void* y, int y_dtype, i64 rows, i64 last,
                       float eps) {
    if (rows <= 0 || last <= 0) return;
    int t = row_threads(last);
    if (x_dtype == CATNN_F32 && y_dtype == CATNN_BF16 && (last == 512 || last == 1024 || last == 2048) &&
        aligned_to(x, 16) && aligned_to(w, 16) && aligned_to(y, 8)) {
        const int grid = (int)cdiv(rows, 8);
        if (last == 512) k_rms_fwd_warp<4><<<grid, 256, 0, c->stream>>>((const float*)x, w, (bf16*)y, rows, eps);
        else if (last == 1024) k_rms_fwd_warp<8><<<grid, 256, 0, c->stream>>>((const float*)x, w, (bf16*)y, rows, eps);
        else k_rms_fwd_warp<16><<<grid, 256, 0, c->stream>>>((const float*)x, w, (bf16*)y, rows, eps);
    } else if (x_dtype == CATNN_F32 && y_dtype == CATNN_BF16)
        k_rms_fwd_mx<<<rows, t, 0, c->stream>>>((const float*)x, w, (bf16*)y, last, eps);
    else if (x_dtype == CATNN_F32 && y_dtype == CATNN_F32)
        k_rms_fwd_mx<<<rows, t, 0, c->stream>>>((const float*)x, w, (float*)y, last, eps);
    else if (x_dtype == CATNN_BF16 && y_dtype == CATNN_BF16)
        k_rms_fwd_mx<<<rows, t, 0, c->stream>>>((const bf16*)x, w, (bf16*)y, last, eps);
    else throw Error(CATNN_ERR_UNSUPPORTED, "rmsnorm_fwd_mixed: dtype pair");
    launched(c);
}

// Fused RMSNorm backward for widths that are multiples of 1024 (<= 4096):
// a CTA of 256 threads owns a chunk of rows, each thread 4 columns per
// 1024; rows go 4 at a time (their loads in flight together, one block
// reduction for the 8 row sums). x and dy stay in registers between the row
// statistics and dx, and the weight-gradient partial Σ dy·x·inv of the
// chunk accumulates in registers: no second pass over x and dy.
constexpr int RB_ROWS = 4;
template <typename TG, typename TC, int NC>
__global__ void __launch_bounds__(256) k_rms_bwd_fused(const float* __restrict__ x, const float* __restrict__ w,
                                                       const TG* __restrict__ dy, const float* __restrict__ dres,
                                                       float* __restrict__ dx, TC* __restrict__ copy, i64 rows,
                                                       int crows, float* __restrict__ pw, float eps) {
    constexpr int last = NC * 1024;
    __shared__ float red[8][2 * RB_ROWS];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float n = (float)last;
    float wv[NC][4], sw[NC][4];
#pragma unroll
    for (int g = 0; g < NC; ++g) {
        ldv<float, 4>(w + g * 1024 + threadIdx.x * 4, wv[g]);
#pragma unroll
        for (int u = 0; u < 4; ++u) sw[g][u] = 0.f;
    }
    const i64 r0 = (i64)blockIdx.x * crows, r1 = min(rows, r0 + crows);
    for (i64 rb = r0; rb < r1; rb += RB_ROWS) {
        float xv[RB_ROWS][NC][4], gv[RB_ROWS][NC][4], part[2 * RB_ROWS];
#pragma unroll
        for (int q = 0; q < RB_ROWS; ++q) {
            part[2 * q] = part[2 * q + 1] = 0.f;
            const i64 r = rb + q;
            if (r < r1) {
#pragma unroll
                for (int g = 0; g < NC; ++g) {
                    const i64 o = r * last + g * 1024 + threadIdx.x * 4;
                    ldv<float, 4>(x + o, xv[q][g]);
                    ldv<TG, 4>(dy + o, gv[q][g]);
                }
            } else {
#pragma unroll
                for (int g = 0; g < NC; ++g)
#pragma unroll
                    for (int u = 0; u < 4; ++u) xv[q][g][u] = gv[q][g][u] = 0.f;
            }
#pragma unroll
            for (int g = 0; g < NC; ++g)
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    part[2 * q] += xv[q][g][u] * xv[q][g][u];
                    part[2 * q + 1] += gv[q][g][u] * xv[q][g][u] * wv[g][u];
                }
        }
#pragma unroll
        for (int i = 0; i < 2 * RB_ROWS; ++i) part[i] = warp_sum(part[i]);
        __syncthreads();  // the previous rows' reads of red are done
        if (lane == 0)
#pragma unroll
            for (int i = 0; i < 2 * RB_ROWS; ++i) red[warp][i] = part[i];
        __syncthreads();
#pragma unroll
        for (int q = 0; q < RB_ROWS; ++q) {
            const i64 r = rb + q;
            if (r >= r1) break;
            float ssum = 0.f, di = 0.f;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                ssum += red[k][2 * q];
                di += red[k][2 * q + 1];
            }
            const float ms = ssum / n;
            const float inv = 1.0f / sqrtf(ms + eps);
            const float dms = di * -0.5f * powf(ms + eps, -1.5f);
#pragma unroll
            for (int g = 0; g < NC; ++g) {
                const i64 o = r * last + g * 1024 + threadIdx.x * 4;
                float out[4], dr[4];
                if (dres) ldv<float, 4>(dres + o, dr);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float v = xv[q][g][u];
                    float rr = gv[q][g][u] * inv * wv[g][u] + dms * (2.0f * v / n);
                    if (dres) rr += dr[u];
                    out[u] = rr;
                    sw[g][u] += gv[q][g][u] * v * inv;
                }
                stv<float, 4>(dx + o, out);
                if (copy) stv<TC, 4>(copy + o, out);
            }
        }
    }
    if (pw) {
#pragma unroll
        for (int g = 0; g < NC; ++g) stv<float, 4>(pw + (i64)blockIdx.x * last + g * 1024 + threadIdx.x * 4, sw[g]);
    }
}

// Sums the chunk partials of k_rms_bwd_fused: 32 columns x 8 slices per CTA,
// slice j adds chunks j, j+8, ... in order, slices are added 0..7.
__global__ void __launch_bounds__(256) k_cols_final8(const float* __restrict__ p, int chunks, i64 last,
                                                     float* __restrict__ out, int acc) {
    __shared__ float red[8][33];
    const int col = threadIdx.x & 31, slice = threadIdx.x >> 5;
    const i64 j = (i64)blockIdx.x * 32 + col;
    float s = 0.f;
    if (j < last) {
#pragma unroll 4
        for (int ch = slice; ch < chunks; ch += 8) s += p[(i64)ch * last + j];
    }
    red[slice][col] = s;
    __syncthreads();
    if (slice == 0 && j < last) {
        float t = red[0][col];
#pragma unroll
        for (int k = 1; k < 8; ++k) t += red[k][col];
        out[j] = acc ? out[j] + t : t;
    }
}

// k_rms_bwd_fused's arithmetic at width 1024 with one warp per row: each
// lane holds 32 values of x and dy (8 float4 chunks 128 columns apart) and
// the two row sums are warp reductions (no block barrier per row). Each warp
// accumulates the weight-gradient partial Σ dy·x·inv of its rows in its own
// shared-memory row (a lane owns its 32 columns there, which keeps the
// registers at two CTAs per SM); at the end the CTA's 8 warps are added in
// warp order into the CTA's partial row pw[blockIdx.x]. Used on the bf16
// trainer's calls (bf16 dy or a bf16 copy of dx).
template <typename TG, typename TC>
__global__ void __launch_bounds__(256, 2) k_rms_bwd_warp(const float* __restrict__ x, const float* __restrict__ w,
                                                         const TG* __restrict__ dy, const float* __restrict__ dres,
                                                         float* __restrict__ dx, TC* __restrict__ copy, i64 rows,
                                                         float* __restrict__ pw, float eps) {
    __shared__ __align__(16) float ws[1024];
    __shared__ __align__(16) float red[8][1024];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < 1024; i += 256) ws[i] = w[i];
#pragma unroll
    for (int k = 0; k < 8; ++k) *(float4*)&red[warp][k * 128 + lane * 4] = make_float4(0.f, 0.f, 0.f, 0.f);
    __syncthreads();
    const float n = 1024.f;
    for (i64 r = (i64)blockIdx.x * 8 + warp; r < rows; r += (i64)gridDim.x * 8) {
        const i64 o = r * 1024 + lane * 4;
        float xv[8][4], gv[8][4];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            ldv<float, 4>(x + o + k * 128, xv[k]);
            ldv<TG, 4>(dy + o + k * 128, gv[k]);
        }
        float ss = 0.f, di = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float4 wq = *(const float4*)&ws[k * 128 + lane * 4];
            const float wv[4] = {wq.x, wq.y, wq.z, wq.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                ss += xv[k][u] * xv[k][u];
                di += gv[k][u] * xv[k][u] * wv[u];
            }
        }
        const float ms = warp_sum(ss) / n;
        di = warp_sum(di);
        const float inv = 1.0f / sqrtf(ms + eps);
        const float dms = di * -0.5f * powf(ms + eps, -1.5f);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int c = k * 128 + lane * 4;
            const float4 wq = *(const float4*)&ws[c];
            const float wv[4] = {wq.x, wq.y, wq.z, wq.w};
            float out[4], dr[4];
            if (dres) ldv<float, 4>(dres + o + k * 128, dr);
            float4 a = *(float4*)&red[warp][c];
            float acc[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float v = xv[k][u];
                float rr = gv[k][u] * inv * wv[u] + dms * (2.0f * v / n);
                if (dres) rr += dr[u];
                out[u] = rr;
                acc[u] += gv[k][u] * v * inv;
            }
            *(float4*)&red[warp][c] = make_float4(acc[0], acc[1], acc[2], acc[3]);
            stv<float, 4>(dx + o + k * 128, out);
            if (copy) stv<TC, 4>(copy + o + k * 128, out);
        }
    }
    if (pw) {
        __syncthreads();
        for (int col = threadIdx.x; col < 1024; col += 256) {
            float t = red[0][col];
#pragma unroll
            for (int k = 1; k < 8; ++k) t += red[k][col];
            pw[(i64)blockIdx.x * 1024 + col] = t;
        }
    }
}

// Sums the partial rows of k_rms_bwd_warp: 8 columns x 32 slices per CTA
// (four times the CTAs of k_cols_final8, a quarter of the dependent loads per
// thread); slice j adds chunks j, j+32, ... in order, slices are added 0..31.
__global__ void __launch_bounds__(256) k_cols_final32(const float* __restrict__ p, int chunks, i64 last,
                                                      float* __restrict__ out, int acc) {
    __shared__ float red[32][9];
    const int col = threadIdx.x & 7, slice = threadIdx.x >> 3;
    const i64 j = (i64)blockIdx.x * 8 + col;
    float s = 0.f;
    if (j < last) {
#pragma unroll 4
        for (int ch = slice; ch < chunks; ch += 32) s += p[(i64)ch * last + j];
    }
    red[slice][col] = s;
    __syncthreads();
    if (slice == 0 && j < last) {
        float t = red[0][col];
#pragma unroll
        for (int k = 1; k < 32; ++k) t += red[k][col];
        out[j] = acc ? out[j] + t : t;
    }
}

template <typename TG, typename TC>
static bool rms_bwd_fused(Context* c, const float* x, const float* w, const TG* dy, const float* dres, float* dx, TC* copy,
                          float* dw, bool dw_acc, i64 rows, i64 last, float eps) {
    const int nc = (int)(last / 1024);
    if (last % 1024 != 0 || nc < 1 || nc > 4) return false;
    if (!aligned_to(x, 16) || !aligned_to(w, 16) || !aligned_to(dy, 16) || !aligned_to(dres, 16) ||
        !aligned_to(dx, 16) || !aligned_to(copy, 16))
        return false;
    constexpr bool bf16_step = std::is_same<TG, bf16>::value || std::is_same<TC, bf16>::value;
    if (bf16_step && last == 1024 && (std::is_same<TG, bf16>::value || copy)) {
        // persistent CTAs, 2 per SM (registers); one partial row of dw each
        const int chunks = (int)std::min<i64>(cdiv(rows, 8), (i64)c->sm_count * 2);
        float* pw = dw ? (float*)c->scratch_for((size_t)chunks * last * 4) : nullptr;
        k_rms_bwd_warp<TG, TC><<<chunks, 256, 0, c->stream>>>(x, w, dy, dres, dx, copy, rows, pw, eps);
        if (dw) k_cols_final32<<<(unsigned)cdiv(last, 8), 256, 0, c->stream>>>(pw, chunks, last, dw, dw_acc ? 1 : 0);
        launched(c, dw ? 2 : 1);
        return true;
    }
    // chunks: enough CTAs to fill the GPU, a multiple of RB_ROWS rows each
    i64 crows = cdiv(rows, (i64)c->sm_count * 4);
    crows = std::max<i64>(RB_ROWS, cdiv(crows, RB_ROWS) * RB_ROWS);
    const int chunks = (int)cdiv(rows, crows);
    float* pw = dw ? (float*)c->scratch_for((size_t)chunks * last * 4) : nullptr;
#define RBF(NCV) \
    k_rms_bwd_fused<TG, TC, NCV><<<chunks, 256, 0, c->stream>>>(x, w, dy, dres, dx, copy, rows, (int)crows, pw, eps)
    if (nc == 1) RBF(1);
    else if (nc == 2) RBF(2);
    else if (nc == 3) RBF(3);
    else RBF(4);
#undef RBF
    if (dw) k_cols_final8<<<(unsigned)cdiv(last, 32), 256, 0, c->stream>>>(pw, chunks, last, dw, dw_acc ? 1 : 0);
    launched(c, dw ? 2 : 1);
    return true;
}

void rmsnorm_bwd_mixed(Context* c, const float* x, const float* w, const void* dy, int g_dtype, const float* dres, float* dx,
                       void* copy, int copy_dtype, float* dw, bool dw_acc, i64 rows, i64 last, float eps) {
    if (rows <= 0 || last <= 0) return;
    {
        bool done;
        if (g_dtype == CATNN_BF16)
            done = (copy_dtype == CATNN_BF16 || !copy)
                       ? rms_bwd_fused(c, x, w, (const bf16*)dy, dres, dx, (bf16*)copy, dw, dw_acc, rows, last, eps)
                       : rms_bwd_fused(c, x, w, (const bf16*)dy, dres, dx, (float*)copy, dw, dw_acc, rows, last, eps);
        else
            done = (copy_dtype == CATNN_BF16 || !copy)
                       ? rms_bwd_fused(c, x, w, (const float*)dy, dres, dx, (bf16*)copy, dw, dw_acc, rows, last, eps)
                       : rms_bwd_fused(c, x, w, (const float*)dy, dres, dx, (float*)copy, dw, dw_acc, rows, last, eps);
        if (done) return;
    }
    const int crows = col_chunk_rows(c, rows, last);
    int chunks = cdiv(rows, crows);
    float* invs = (float*)c->scratch_for((size_t)rows * 4 + (size_t)chunks * last * 4);
    float* pw = invs + rows;
    int t = row_threads(last);
    dim3 gc(cdiv(last, 128), chunks);
    if (g_dtype == CATNN_BF16) {
        if (copy_dtype == CATNN_BF16 || !copy)
            k_rms_bwd_mx<<<rows, t, 0, c->stream>>>(x, w, (const bf16*)dy, dres, dx, (bf16*)copy, invs, last, eps);
        else k_rms_bwd_mx<<<rows, t, 0, c->stream>>>(x, w, (const bf16*)dy, dres, dx, (float*)copy, invs, last, eps);
        if (dw) k_rms_cols_mx<<<gc, 128, 0, c->stream>>>(x, (const bf16*)dy, invs, rows, last, pw, crows);
    } else {
        if (copy_dtype == CATNN_BF16 || !copy)
            k_rms_bwd_mx<<<rows, t, 0, c->stream>>>(x, w, (const float*)dy, dres, dx, (bf16*)copy, invs, last, eps);
        else k_rms_bwd_mx<<<rows, t, 0, c->stream>>>(x, w, (const float*)dy, dres, dx, (float*)copy, invs, last, eps);
        if (dw) k_rms_cols_mx<<<gc, 128, 0, c->stream>>>(x, (const float*)dy, invs, rows, last, pw, crows);
    }
    if (dw) k_cols_final<<<cdiv(last, 128), 128, 0, c->stream>>>(pw, chunks, last, dw, dw_acc ? 1 : 0);
    launched(c, dw ? 3 : 1);
}

}  // namespace catnn

// ------------------------------------------- cross-entropy without allocation
// Some callers cannot allocate device memory while they run a step: a
// runtime that has planned every byte of a device's memory ahead of time
// (catnn's fixed code/buffer/scratch budgets), or a host thread that must
// not synchronize the device, which a cudaMalloc may do. For them, this
// variant of catnn_xent_fwdbwd keeps its per-row loss scratch in a
// fixed-size array compiled into the library instead of the context's
// grow-on-demand scratch buffer. Every device that loads the library holds
// the array (256 KB) until the process exits.
namespace catnn {

static __device__ __align__(256) float g_xent_row_loss[CATNN_XENT_NOALLOC_MAX_ROWS];

// Device address of g_xent_row_loss for each device, resolved once with
// that device current (the host-side symbol is only a stand-in).
static float* g_xent_row_loss_ptr[64] = {nullptr};
static std::mutex g_xent_row_loss_mu;

float* xent_row_loss_buffer(int device) {
    CATNN_CHECK(device >= 0 && device < 64, CATNN_ERR_INVALID, "device index out of range");
    std::lock_guard<std::mutex> lock(g_xent_row_loss_mu);
    if (!g_xent_row_loss_ptr[device]) {
        int cur = -1;
        CUDA_OK(cudaGetDevice(&cur));
        CATNN_CHECK(cur == device, CATNN_ERR_INVALID, "xent_row_loss_buffer: the device must be current");
        void* p = nullptr;
        CUDA_OK(cudaGetSymbolAddress(&p, g_xent_row_loss));
        g_xent_row_loss_ptr[device] = (float*)p;
    }
    return g_xent_row_loss_ptr[device];
}

void xent_noalloc_forget(int device) {
    if (device < 0 || device >= 64) return;
    std::lock_guard<std::mutex> lock(g_xent_row_loss_mu);
    g_xent_row_loss_ptr[device] = nullptr;
}

// rms_norm, layer_norm, softmax and the cross-entropy loss: one CTA per row.
KernelInfo norms_info(Context* c, const std::string& op, int dtype, const KShape& s) {
    KernelInfo k;
    const bool b = dtype == CATNN_BF16;
    if (op == "rms_norm") k.fn = b ? (const void*)k_rms_fwd<bf16> : (const void*)k_rms_fwd<float>;
    else if (op == "layer_norm") k.fn = b ? (const void*)k_ln_fwd<bf16> : (const void*)k_ln_fwd<float>;
    else if (op == "softmax") k.fn = b ? (const void*)k_softmax<bf16> : (const void*)k_softmax<float>;
    else if (op == "cross_entropy") {
        const int v = b ? 8 : 4;
        if (s.width % v == 0) k.fn = b ? (const void*)k_xent_rows<bf16, 8> : (const void*)k_xent_rows<float, 4>;
        else k.fn = b ? (const void*)k_xent_rows<bf16, 1> : (const void*)k_xent_rows<float, 1>;
    } else return k;
    k.file = "norms.cu";
    k.grid[0] = (unsigned)std::max<i64>(1, s.rows);
    k.block[0] = row_threads(s.width);
    return k;
}

}  // namespace catnn

extern "C" int catnn_xent_fwdbwd_noalloc(catnn_ctx* h, const void* logits, const uint32_t* targets, int64_t rows,
                                         int64_t vocab, float* loss, void* dlogits, int dtype, int check) {
    ABI_BEGIN
    using namespace catnn;
    Context* c = unwrap(h);  // makes the context's device current
    check_dtype(dtype);
    CATNN_CHECK(rows >= 1 && vocab >= 1, CATNN_ERR_SHAPE, "cross_entropy: empty logits");
    CATNN_CHECK(rows <= CATNN_XENT_NOALLOC_MAX_ROWS, CATNN_ERR_SHAPE,
                "catnn_xent_fwdbwd_noalloc: " + std::to_string(rows) + " rows exceed its fixed limit of " +
                    std::to_string(CATNN_XENT_NOALLOC_MAX_ROWS) + " (use catnn_xent_fwdbwd)");
    CATNN_CHECK(logits && targets && loss && dlogits, CATNN_ERR_INVALID, "null argument");
    float* rl = xent_row_loss_buffer(c->device);
    int* err = c->status + 9;
    // every row r < rows writes rl[r] before the reduction reads it, so the
    // array needs no clearing between calls
    launch_xent_rows(c, logits, targets, rows, vocab, dlogits, dtype, rl, err, rows);
    k_sum_rows_mean<<<1, 1024, 0, c->stream>>>(rl, rows, loss, rows);
    launched(c, 2);
    if (check && take_status(c, 9)) throw Error(CATNN_ERR_SHAPE, "ce targets: a target is >= the number of classes");
    ABI_END
}
