// MoE routing and data movement: top-k router (bit-exact indices), the
// stable counting-sort permutation, permute / weighted unpermute and their
// adjoints, the router straight-through adjoint, and the SwiGLU gate.
//
// The reference runs the experts token by token (moe.rs:207-221); here the
// (token, slot) pairs are sorted by expert once so every expert becomes one
// dense GEMM over its rows. Rows of an expert are in token order and each
// expert's row block is padded to `align` rows (zeros) so tensor-core tiles
// never straddle two experts.
#include <initializer_list>
#include <utility>

#include "ops.cuh"

namespace catnn {

// lens/moe.rs:175-187 — k selections of the largest remaining logit, ties
// to the lower index (a stable descending sort), then softmax over the k
// selected: w = exp(l - max) / max(Σ, 1e-30), summed in selection order.
__global__ void k_router_topk(const float* __restrict__ logits, i64 T, int E, int k, int32_t* __restrict__ idx,
                              float* __restrict__ w) {
    i64 t = blockIdx.x * (i64)blockDim.x + threadIdx.x;
    if (t >= T) return;
    const float* row = logits + t * E;
    unsigned long long taken = 0ull;
    float sel[64];
    int kk = k < E ? k : E;
    for (int j = 0; j < kk; ++j) {
        int best = -1;
        float bv = 0.f;
        for (int e = 0; e < E; ++e) {
            if (taken >> e & 1ull) continue;
            float v = row[e];
            if (best < 0 || v > bv) {
                best = e;
                bv = v;
            }
        }
        taken |= 1ull << best;
        idx[t * k + j] = best;
        sel[j] = bv;
    }
    float mx = -INFINITY;
    for (int j = 0; j < kk; ++j) mx = fmaxf(mx, sel[j]);
    float s = 0.f;
    for (int j = 0; j < kk; ++j) {
        sel[j] = expf(sel[j] - mx);
        s = __fadd_rn(s, sel[j]);
    }
    float inv = 1.0f / fmaxf(s, 1e-30f);
    for (int j = 0; j < kk; ++j) w[t * k + j] = __fmul_rn(sel[j], inv);
}

void router_topk(Context* c, const float* logits, i64 T, i64 E, i64 k, int32_t* idx, float* w) {
    if (T <= 0) return;
    CATNN_CHECK(E >= 1 && E <= 64 && k >= 1 && k <= E, CATNN_ERR_SHAPE, "router: need 1 <= k <= E <= 64");
    k_router_topk<<<cdiv(T, 128), 128, 0, c->stream>>>(logits, T, (int)E, (int)k, idx, w);
    launched(c);
}

// Single CTA, 1024 threads. Thread i owns pairs [i*chunk, (i+1)*chunk) in
// order; per-thread expert counts go to shared memory, are scanned down the
// threads per expert, and each thread then places its pairs stably.
// offsets[e] is padded to `align`; src_of[r] is the pair index t*k+j of
// sorted row r, or -1 on padding rows; row_of[pair] is the pair's row.
__global__ void __launch_bounds__(1024) k_permute_map(const int32_t* __restrict__ idx, i64 P, int E, int align,
                                                      int32_t* __restrict__ counts, int32_t* __restrict__ offsets,
                                                      int32_t* __restrict__ row_of, int32_t* __restrict__ src_of,
                                                      i64 rows_cap, int* __restrict__ err) {
    extern __shared__ int32_t cnt[];  // [1024][E] then [E+1] offsets
    int tid = threadIdx.x, nt = blockDim.x;
    i64 chunk = (P + nt - 1) / nt;
    i64 p0 = tid * chunk, p1 = p0 + chunk < P ? p0 + chunk : P;
    for (int e = 0; e < E; ++e) cnt[tid * E + e] = 0;
    for (i64 p = p0; p < p1; ++p) {
        int e = idx[p];
        if (e < 0 || e >= E) {
            atomicExch(err, 1);
            continue;
        }
        cnt[tid * E + e] += 1;
    }
    __syncthreads();
    int32_t* off = cnt + nt * E;
    if (tid < E) {
        int run = 0;
        for (int i = 0; i < nt; ++i) {
            int v = cnt[i * E + tid];
            cnt[i * E + tid] = run;
            run += v;
        }
        counts[tid] = run;
        off[tid] = run;  // temporarily the count
    }
    __syncthreads();
    if (tid == 0) {
        int o = 0;
        for (int e = 0; e < E; ++e) {
            int n = off[e];
            offsets[e] = o;
            off[e] = o;
            o += (n + align - 1) / align * align;
        }
        offsets[E] = o;
        off[E] = o;
        if ((i64)o > rows_cap) atomicExch(err, 2);
    }
    __syncthreads();
    if ((i64)off[E] > rows_cap) return;
    for (i64 p = p0; p < p1; ++p) {
        int e = idx[p];
        if (e < 0 || e >= E) continue;
        int r = off[e] + cnt[tid * E + e];
        cnt[tid * E + e] += 1;
        row_of[p] = r;
        src_of[r] = (int32_t)p;
    }
    __syncthreads();
    // padding rows, then every row past the last expert up to the capacity
    for (int e = 0; e < E; ++e) {
        int n = counts[e];
        for (int r = off[e] + n + tid; r < off[e + 1]; r += nt) src_of[r] = -1;
    }
    for (i64 r = off[E] + tid; r < rows_cap; r += nt) src_of[r] = -1;
}

// ---- the same stable counting sort across many CTAs (large pair counts)
// Chunk g of PM_CHUNK pairs: per-expert histogram -> hist[g][E].
constexpr int PM_CHUNK = 1024, PM_THREADS = 256;
__global__ void __launch_bounds__(PM_THREADS) k_pm_hist(const int32_t* __restrict__ idx, i64 P, int E,
                                                        int32_t* __restrict__ hist, int* __restrict__ err) {
    __shared__ int h[32];
    if (threadIdx.x < 32) h[threadIdx.x] = 0;
    __syncthreads();
    const i64 p0 = (i64)blockIdx.x * PM_CHUNK, p1 = min(P, p0 + PM_CHUNK);
    for (i64 p = p0 + threadIdx.x; p < p1; p += PM_THREADS) {
        int e = idx[p];
        if (e < 0 || e >= E) {
            atomicExch(err, 1);
            continue;
        }
        atomicAdd(&h[e], 1);
    }
    __syncthreads();
    if (threadIdx.x < E) hist[(i64)blockIdx.x * E + threadIdx.x] = h[threadIdx.x];
}

// One CTA: per expert, chunk bases in chunk order (hist becomes the base of
// each chunk's first pair of that expert), counts, padded offsets.
__global__ void k_pm_scan(int32_t* __restrict__ hist, int G, int E, int align, int32_t* __restrict__ counts,
                          int32_t* __restrict__ offsets, i64 rows_cap, int* __restrict__ err) {
    __shared__ int tot[33], off[33];
    const int e = threadIdx.x;
    if (e < E) {
        int run = 0;
        for (int g = 0; g < G; ++g) {
            int v = hist[(i64)g * E + e];
            hist[(i64)g * E + e] = run;
            run += v;
        }
        tot[e] = run;
        counts[e] = run;
    }
    __syncthreads();
    if (e == 0) {
        int o = 0;
        for (int x = 0; x < E; ++x) {
            off[x] = o;
            offsets[x] = o;
            o += (tot[x] + align - 1) / align * align;
        }
        off[E] = o;
        offsets[E] = o;
        if ((i64)o > rows_cap) atomicExch(err, 2);
    }
    __syncthreads();
    if (e < E)
        for (int g = 0; g < G; ++g) hist[(i64)g * E + e] += off[e];
}

// Chunk g places its pairs in pair order: rounds of PM_THREADS pairs, the
// rank among equal experts inside a warp from __match_any_sync, warps in
// order through a shared-memory prefix, chunk base from k_pm_scan.
__global__ void __launch_bounds__(PM_THREADS) k_pm_place(const int32_t* __restrict__ idx, i64 P, int E,
                                                         const int32_t* __restrict__ base, const int32_t* __restrict__ offsets,
                                                         i64 rows_cap, int32_t* __restrict__ row_of,
                                                         int32_t* __restrict__ src_of) {
    __shared__ int run[32], wcnt[PM_THREADS / 32][32], wpre[PM_THREADS / 32][32];
    if ((i64)offsets[E] > rows_cap) return;  // flagged by k_pm_scan; nothing is placed
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x < E) run[threadIdx.x] = base[(i64)blockIdx.x * E + threadIdx.x];
    const i64 p0 = (i64)blockIdx.x * PM_CHUNK, p1 = min(P, p0 + PM_CHUNK);
    for (i64 rb = p0; rb < p1; rb += PM_THREADS) {
        for (int i = threadIdx.x; i < (PM_THREADS / 32) * 32; i += PM_THREADS) (&wcnt[0][0])[i] = 0;
        __syncthreads();
        const i64 p = rb + threadIdx.x;
        int e = p < p1 ? idx[p] : -1;
        if (e >= E) e = -1;
        const unsigned same = __match_any_sync(0xffffffffu, e);
        const int rank = __popc(same & ((1u << lane) - 1u));
        if (e >= 0 && rank == 0) wcnt[warp][e] = __popc(same);
        __syncthreads();
        if (threadIdx.x < E) {
            int r = run[threadIdx.x];
            for (int w = 0; w < PM_THREADS / 32; ++w) {
                wpre[w][threadIdx.x] = r;
                r += wcnt[w][threadIdx.x];
            }
            run[threadIdx.x] = r;
        }
        __syncthreads();
        if (e >= 0) {
            const int row = wpre[warp][e] + rank;
            row_of[p] = row;
            src_of[row] = (int32_t)p;
        }
        __syncthreads();
    }
}

// src_of = -1 on every padding row and on the rows past the last expert.
__global__ void k_pm_pad(const int32_t* __restrict__ counts, const int32_t* __restrict__ offsets, int E, i64 rows_cap,
                         int32_t* __restrict__ src_of) {
    __shared__ int off[33], cnt[32];
    if (threadIdx.x <= E) off[threadIdx.x] = offsets[threadIdx.x];
    if (threadIdx.x < E) cnt[threadIdx.x] = counts[threadIdx.x];
    __syncthreads();
    if ((i64)off[E] > rows_cap) return;
    for (i64 r = blockIdx.x * (i64)blockDim.x + threadIdx.x; r < rows_cap; r += (i64)gridDim.x * blockDim.x) {
        bool pad = r >= off[E];
        if (!pad) {
            int e = 0;
            while (e + 1 < E && r >= off[e + 1]) ++e;
            pad = r >= off[e] + cnt[e];
        }
        if (pad) src_of[r] = -1;
    }
}

void permute_map(Context* c, const int32_t* idx, i64 T, i64 E, i64 k, int align, i64 rows_cap, int32_t* counts,
                 int32_t* offsets, int32_t* row_of, int32_t* src_of) {
    if (T <= 0) {
        CUDA_OK(cudaMemsetAsync(counts, 0, E * 4, c->stream));
        CUDA_OK(cudaMemsetAsync(offsets, 0, (E + 1) * 4, c->stream));
        return;
    }
    CATNN_CHECK(E >= 1 && E <= 32, CATNN_ERR_SHAPE, "permute_map: 1 <= E <= 32");
    CATNN_CHECK(align >= 1, CATNN_ERR_INVALID, "permute_map: align >= 1");
    i64 P = T * k;
    CATNN_CHECK(P < (1ll << 31), CATNN_ERR_SHAPE, "permute_map: too many pairs");
    if (P > 4 * PM_CHUNK) {
        const i64 G = cdiv(P, PM_CHUNK);
        int32_t* hist = (int32_t*)c->scratch_for((size_t)G * E * 4);
        k_pm_hist<<<(unsigned)G, PM_THREADS, 0, c->stream>>>(idx, P, (int)E, hist, c->status + 8);
        k_pm_scan<<<1, 32, 0, c->stream>>>(hist, (int)G, (int)E, align, counts, offsets, rows_cap, c->status + 8);
        k_pm_place<<<(unsigned)G, PM_THREADS, 0, c->stream>>>(idx, P, (int)E, hist, offsets, rows_cap, row_of, src_of);
        k_pm_pad<<<(unsigned)std::min<i64>(cdiv(rows_cap, 256), (i64)c->sm_count * 8), 256, 0, c->stream>>>(
            counts, offsets, (int)E, rows_cap, src_of);
        launched(c, 4);
        return;
    }
    size_t smem = (size_t)(1024 * E + E + 1) * 4;
    static bool attr[64] = {false};
    if (!attr[c->device]) {
        CUDA_OK(cudaFuncSetAttribute(k_permute_map, cudaFuncAttributeMaxDynamicSharedMemorySize, (1024 * 32 + 33) * 4));
        attr[c->device] = true;
    }
    k_permute_map<<<1, 1024, smem, c->stream>>>(idx, P, (int)E, align, counts, offsets, row_of, src_of, rows_cap,
                                                c->status + 8);
    launched(c);
}

// xp[r] = x[src_of[r] / k] (zeros on padding rows). One warp per row, 16-byte vectors.
template <typename T>
__global__ void k_permute(const T* __restrict__ x, const int32_t* __restrict__ src_of, i64 rows, i64 hidden, int k,
                          T* __restrict__ xp) {
    i64 r = blockIdx.x * 4 + (threadIdx.x >> 5);
    int lane = threadIdx.x & 31;
    if (r >= rows) return;
    int p = src_of[r];
    T* dst = xp + r * hidden;
    if ((hidden * sizeof(T)) % 16 == 0) {
        i64 nv = hidden * sizeof(T) / 16;
        uint4* d = (uint4*)dst;
        if (p < 0) {
            for (i64 i = lane; i < nv; i += 32) d[i] = make_uint4(0, 0, 0, 0);
        } else {
            const uint4* s = (const uint4*)(x + (i64)(p / k) * hidden);
            for (i64 i = lane; i < nv; i += 32) d[i] = s[i];
        }
    } else {
        for (i64 i = lane; i < hidden; i += 32) dst[i] = p < 0 ? T(0.f) : x[(i64)(p / k) * hidden + i];
    }
}

void permute_rows(Context* c, const void* x, const int32_t* src_of, i64 rows, i64 hidden, i64 k, void* xp, int dtype) {
    if (rows <= 0) return;
    if (dtype == CATNN_BF16)
        k_permute<<<cdiv(rows, 4), 128, 0, c->stream>>>((const bf16*)x, src_of, rows, hidden, (int)k, (bf16*)xp);
    else k_permute<<<cdiv(rows, 4), 128, 0, c->stream>>>((const float*)x, src_of, rows, hidden, (int)k, (float*)xp);
    launched(c);
}

// y[t] (+)= Σ_j w[t,j] · yp[row_of[t,j]], slots in order (moe.rs:212-219:
// out starts at 0 and adds w·y per slot; with accumulate the finished sum
// is then added to y, as x + moe(x) does).
template <typename TI, typename T>
__global__ void k_unpermute(const TI* __restrict__ yp, const int32_t* __restrict__ row_of, const float* __restrict__ w,
                            i64 Tn, int k, i64 hidden, T* __restrict__ y, int acc, const T* __restrict__ resid) {
    i64 t = blockIdx.y;
    for (i64 i = blockIdx.x * (i64)blockDim.x + threadIdx.x; i < hidden; i += (i64)gridDim.x * blockDim.x) {
        float s = 0.f;
        for (int j = 0; j < k; ++j) {
            int r = row_of[t * k + j];
            s = __fadd_rn(s, __fmul_rn(w[t * k + j], ld(yp + (i64)r * hidden + i)));
        }
        if (acc) s = __fadd_rn(ld(y + t * hidden + i), s);
        if (resid) s = __fadd_rn(ld(resid + t * hidden + i), s);
        st(y + t * hidden + i, s);
    }
}

// Vector form of k_unpermute (same arithmetic per element): CTAs stride over
// tokens, threads over V-wide column groups with 16-byte accesses.
template <typename TI, typename T, int V>
__global__ void __launch_bounds__(128) k_unpermute_v(const TI* __restrict__ yp, const int32_t* __restrict__ row_of,
                                                     const float* __restrict__ w, i64 Tn, int k, i64 hidden,
                                                     T* __restrict__ y, int acc, const T* __restrict__ resid) {
    for (i64 t = blockIdx.x; t < Tn; t += gridDim.x) {
        for (i64 c = (i64)threadIdx.x * V; c < hidden; c += (i64)blockDim.x * V) {
            float s[V];
#pragma unroll
            for (int u = 0; u < V; ++u) s[u] = 0.f;
            for (int j = 0; j < k; ++j) {
                const i64 r = row_of[t * k + j];
                const float wt = w[t * k + j];
                float v[V];
                ldv<TI, V>(yp + r * hidden + c, v);
#pragma unroll
                for (int u = 0; u < V; ++u) s[u] = __fadd_rn(s[u], __fmul_rn(wt, v[u]));
            }
            if (acc) {
                float o[V];
                ldv<T, V>(y + t * hidden + c, o);
#pragma unroll
                for (int u = 0; u < V; ++u) s[u] = __fadd_rn(o[u], s[u]);
            }
            if (resid) {
                float o[V];
                ldv<T, V>(resid + t * hidden + c, o);
#pragma unroll
                for (int u = 0; u < V; ++u) s[u] = __fadd_rn(o[u], s[u]);
            }
            stv<T, V>(y + t * hidden + c, s);
        }
    }
}

// Vector form of k_permute_bwd (same arithmetic per element).
template <typename TI, typename T, int V>
__global__ void __launch_bounds__(128) k_permute_bwd_v(const TI* __restrict__ dxp, const int32_t* __restrict__ row_of,
                                                       i64 Tn, int k, i64 hidden, T* __restrict__ dx, int acc) {
    for (i64 t = blockIdx.x; t < Tn; t += gridDim.x) {
        for (i64 c = (i64)threadIdx.x * V; c < hidden; c += (i64)blockDim.x * V) {
            float s[V];
#pragma unroll
            for (int u = 0; u < V; ++u) s[u] = 0.f;
            for (int j = 0; j < k; ++j) {
                float v[V];
                ldv<TI, V>(dxp + (i64)row_of[t * k + j] * hidden + c, v);
#pragma unroll
                for (int u = 0; u < V; ++u) s[u] = __fadd_rn(s[u], v[u]);
            }
            if (acc) {
                float o[V];
                ldv<T, V>(dx + t * hidden + c, o);
#pragma unroll
                for (int u = 0; u < V; ++u) s[u] = __fadd_rn(o[u], s[u]);
            }
            stv<T, V>(dx + t * hidden + c, s);
        }
    }
}

void unpermute_rows(Context* c, const void* yp, const int32_t* row_of, const float* w, i64 T, i64 k, i64 hidden, void* y,
                    int dtype, bool accumulate, int yp_dtype, const void* resid) {
    if (T <= 0 || hidden <= 0) return;
    if (yp_dtype < 0) yp_dtype = dtype;
    if (yp_dtype == CATNN_BF16 && dtype == CATNN_F32 && hidden % 8 == 0 && aligned_to(yp, 16) && aligned_to(y, 16) &&
        aligned_to(resid, 16)) {
        // the trainer's combine: bf16 expert rows into the fp32 residual stream
        const int grid = (int)std::min<i64>(T, (i64)c->sm_count * 16);
        k_unpermute_v<bf16, float, 8><<<grid, 128, 0, c->stream>>>((const bf16*)yp, row_of, w, T, (int)k, hidden,
                                                                   (float*)y, accumulate ? 1 : 0, (const float*)resid);
        launched(c);
        return;
    }
    CATNN_CHECK(T <= 2147483647ll, CATNN_ERR_SHAPE, "unpermute: too many tokens");
    dim3 grid(cdiv(hidden, 256), (unsigned)T);
    int acc = accumulate ? 1 : 0;
    if (dtype == CATNN_BF16 && yp_dtype == CATNN_BF16)
        k_unpermute<<<grid, 256, 0, c->stream>>>((const bf16*)yp, row_of, w, T, (int)k, hidden, (bf16*)y, acc,
                                                 (const bf16*)resid);
    else if (dtype == CATNN_BF16)
        k_unpermute<<<grid, 256, 0, c->stream>>>((const float*)yp, row_of, w, T, (int)k, hidden, (bf16*)y, acc,
                                                 (const bf16*)resid);
    else if (yp_dtype == CATNN_BF16)
        k_unpermute<<<grid, 256, 0, c->stream>>>((const bf16*)yp, row_of, w, T, (int)k, hidden, (float*)y, acc,
                                                 (const float*)resid);
    else
        k_unpermute<<<grid, 256, 0, c->stream>>>((const float*)yp, row_of, w, T, (int)k, hidden, (float*)y, acc,
                                                 (const float*)resid);
    launched(c);
}

// Per sorted row r (pair p = src_of[r], token t = p/k):
// dw[p] = <yp[r], dy[t]> (adjoint.rs:504), dyp[r] = w[p]·dy[t]; zeros on padding rows.
template <typename TY, typename TG, typename T>
__global__ void k_unpermute_bwd(const TY* __restrict__ yp, const int32_t* __restrict__ src_of, const float* __restrict__ w,
                                const TG* __restrict__ dy, i64 rows, int k, i64 hidden, float* __restrict__ dw,
                                T* __restrict__ dyp) {
    i64 r = blockIdx.x * 4 + (threadIdx.x >> 5);
    int lane = threadIdx.x & 31;
    if (r >= rows) return;
    int p = src_of[r];
    if (p < 0) {
        for (i64 i = lane; i < hidden; i += 32) dyp[r * hidden + i] = T(0.f);
        return;
    }
    i64 t = p / k;
    float wt = w[p], dot = 0.f;
    for (i64 i = lane; i < hidden; i += 32) {
        float g = ld(dy + t * hidden + i);
        dot += ld(yp + r * hidden + i) * g;
        st(dyp + r * hidden + i, __fmul_rn(g, wt));
    }
    dot = warp_sum(dot);
    if (lane == 0) dw[p] = dot;
}

// k_unpermute_bwd for a bf16 dyp at hidden % 256 == 0: a lane takes 8
// consecutive columns per step (16-byte loads of yp and stores of dyp, 8-wide
// loads of dy), hidden/256 steps per row with their loads in flight
// together. The lane's part of the dot product adds its 8 products per step
// in column order, then the warp sums the lanes.
template <typename TY, typename TG>
__global__ void __launch_bounds__(128) k_unpermute_bwd_v(const TY* __restrict__ yp, const int32_t* __restrict__ src_of,
                                                         const float* __restrict__ w, const TG* __restrict__ dy,
                                                         i64 rows, int k, i64 hidden, float* __restrict__ dw,
                                                         bf16* __restrict__ dyp) {
    const i64 r = blockIdx.x * 4 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    const int p = src_of[r];
    bf16* out = dyp + r * hidden;
    if (p < 0) {
        for (i64 i = lane * 8; i < hidden; i += 256) *(uint4*)(out + i) = make_uint4(0, 0, 0, 0);
        return;
    }
    const i64 t = p / k;
    const float wt = w[p];
    const TY* yr = yp + r * hidden;
    const TG* gr = dy + t * hidden;
    float dot = 0.f;
#pragma unroll 4
    for (i64 i = lane * 8; i < hidden; i += 256) {
        float g[8], yv[8], o[8];
        ldv<TG, 8>(gr + i, g);
        ldv<TY, 8>(yr + i, yv);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            dot += yv[j] * g[j];
            o[j] = __fmul_rn(g[j], wt);
        }
        stv<bf16, 8>(out + i, o);
    }
    dot = warp_sum(dot);
    if (lane == 0) dw[p] = dot;
}

// dx[t] (+)= Σ_j dxp[row_of[t,j]] in slot order.
template <typename TI, typename T>
__global__ void k_permute_bwd(const TI* __restrict__ dxp, const int32_t* __restrict__ row_of, i64 Tn, int k, i64 hidden,
                              T* __restrict__ dx, int acc) {
    i64 t = blockIdx.y;
    for (i64 i = blockIdx.x * (i64)blockDim.x + threadIdx.x; i < hidden; i += (i64)gridDim.x * blockDim.x) {
        float s = 0.f;
        for (int j = 0; j < k; ++j) s = __fadd_rn(s, ld(dxp + (i64)row_of[t * k + j] * hidden + i));
        if (acc) s = __fadd_rn(ld(dx + t * hidden + i), s);
        st(dx + t * hidden + i, s);
    }
}

void unpermute_bwd(Context* c, const void* yp, const int32_t* src_of, i64 rows, const float* w, const void* dy, i64 k,
                   i64 hidden, float* dw, void* dyp, int dtype, int yp_dtype, int dy_dtype) {
    if (rows <= 0) return;
    if (yp_dtype < 0) yp_dtype = dtype;
    if (dy_dtype < 0) dy_dtype = dtype;
    dim3 g(cdiv(rows, 4));
#define UPB(TY, TG, T) \
    k_unpermute_bwd<<<g, 128, 0, c->stream>>>((const TY*)yp, src_of, w, (const TG*)dy, rows, (int)k, hidden, dw, (T*)dyp)
#define UPBV(TY, TG) \
    k_unpermute_bwd_v<<<g, 128, 0, c->stream>>>((const TY*)yp, src_of, w, (const TG*)dy, rows, (int)k, hidden, dw, (bf16*)dyp)
    if (dtype == CATNN_BF16 && hidden % 256 == 0 && aligned_to(yp, 16) && aligned_to(dy, 16) && aligned_to(dyp, 16)) {
        if (yp_dtype == CATNN_F32 && dy_dtype == CATNN_F32) UPBV(float, float);
        else if (yp_dtype == CATNN_F32) UPBV(float, bf16);
        else if (dy_dtype == CATNN_F32) UPBV(bf16, float);
        else UPBV(bf16, bf16);
    } else if (dtype == CATNN_BF16) {
        if (yp_dtype == CATNN_F32 && dy_dtype == CATNN_F32) UPB(float, float, bf16);
        else if (yp_dtype == CATNN_F32) UPB(float, bf16, bf16);
        else if (dy_dtype == CATNN_F32) UPB(bf16, float, bf16);
        else UPB(bf16, bf16, bf16);
    } else {
        CATNN_CHECK(yp_dtype == CATNN_F32 && dy_dtype == CATNN_F32, CATNN_ERR_DTYPE, "unpermute_bwd: fp32 path");
        UPB(float, float, float);
    }
#undef UPB
#undef UPBV
    launched(c);
}

void permute_bwd(Context* c, const void* dxp, const int32_t* row_of, i64 T, i64 k, i64 hidden, void* dx, int dtype,
                 bool accumulate, int out_dtype) {
    if (T <= 0 || hidden <= 0) return;
    if (out_dtype < 0) out_dtype = dtype;
    if (dtype == CATNN_BF16 && out_dtype == CATNN_F32 && hidden % 8 == 0 && aligned_to(dxp, 16) && aligned_to(dx, 16)) {
        const int grid = (int)std::min<i64>(T, (i64)c->sm_count * 16);
        k_permute_bwd_v<bf16, float, 8><<<grid, 128, 0, c->stream>>>((const bf16*)dxp, row_of, T, (int)k, hidden,
                                                                     (float*)dx, accumulate ? 1 : 0);
        launched(c);
        return;
    }
    dim3 grid(cdiv(hidden, 256), (unsigned)T);
    if (dtype == CATNN_BF16 && out_dtype == CATNN_F32)
        k_permute_bwd<<<grid, 256, 0, c->stream>>>((const bf16*)dxp, row_of, T, (int)k, hidden, (float*)dx, accumulate);
    else if (dtype == CATNN_BF16)
        k_permute_bwd<<<grid, 256, 0, c->stream>>>((const bf16*)dxp, row_of, T, (int)k, hidden, (bf16*)dx, accumulate);
    else k_permute_bwd<<<grid, 256, 0, c->stream>>>((const float*)dxp, row_of, T, (int)k, hidden, (float*)dx, accumulate);
    launched(c);
}

// adjoint.rs:267-279 — on the selected experts dlogits = w·(g - <w,g>).
__global__ void k_router_ste(const int32_t* __restrict__ idx, const float* __restrict__ w, const float* __restrict__ dw,
                             i64 T, int E, int k, float* __restrict__ dlog) {
    i64 t = blockIdx.x * (i64)blockDim.x + threadIdx.x;
    if (t >= T) return;
    float dot = 0.f;
    for (int j = 0; j < k; ++j) dot = __fadd_rn(dot, __fmul_rn(w[t * k + j], dw[t * k + j]));
    for (int e = 0; e < E; ++e) dlog[t * E + e] = 0.f;
    for (int j = 0; j < k; ++j) dlog[t * E + idx[t * k + j]] = __fmul_rn(w[t * k + j], __fsub_rn(dw[t * k + j], dot));
}

void router_ste(Context* c, const int32_t* idx, const float* w, const float* dw, i64 T, i64 E, i64 k, float* dlogits) {
    if (T <= 0) return;
    k_router_ste<<<cdiv(T, 128), 128, 0, c->stream>>>(idx, w, dw, T, (int)E, (int)k, dlogits);
    launched(c);
}

// moe.rs:12-14 / adjoint.rs:208-215
__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float silu_grad_f(float x) {
    float s = 1.0f / (1.0f + expf(-x));
    return s + x * s * (1.0f - s);
}

// h = silu(a) ⊙ c. a, c: [rows, F] views with leading dimension lda
// (a fused [a | c] buffer passes cc = a + F and lda = 2F). CTAs stride over
// rows, threads over V-wide column vectors (16-byte accesses when aligned).
// One flat index over (row, vector) so every thread has work; 32-bit index
// math (the host guarantees rows * F / V < 2^31).
template <typename TI, typename T, int V>
__global__ void __launch_bounds__(256) k_swiglu(const TI* __restrict__ a, const TI* __restrict__ cc, T* __restrict__ h,
                                                i64 rows, i64 F, i64 lda, i64 ldh, const int32_t* __restrict__ rows_dev) {
    if (rows_dev && *rows_dev < rows) rows = *rows_dev;
    const uint32_t vpr = (uint32_t)(F / V);
    const uint32_t total = (uint32_t)rows * vpr;
    for (uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += gridDim.x * blockDim.x) {
        const uint32_t r = idx / vpr;
        const i64 f = (i64)(idx - r * vpr) * V;
        float av[V], cv[V], o[V];
        ldv<TI, V>(a + r * lda + f, av);
        ldv<TI, V>(cc + r * lda + f, cv);
#pragma unroll
        for (int j = 0; j < V; ++j) o[j] = silu_f(av[j]) * cv[j];
        stv<T, V>(h + r * ldh + f, o);
    }
}

// adjoint.rs:239-242: da = dh·c·silu'(a), dc = dh·silu(a).
template <typename TI, typename TG, typename T, int V>
__global__ void __launch_bounds__(256) k_swiglu_bwd(const TI* __restrict__ a, const TI* __restrict__ cc,
                                                    const TG* __restrict__ dh, T* __restrict__ da, T* __restrict__ dc,
                                                    i64 rows, i64 F, i64 lda, i64 ldd,
                                                    const int32_t* __restrict__ rows_dev) {
    if (rows_dev && *rows_dev < rows) rows = *rows_dev;
    const uint32_t vpr = (uint32_t)(F / V);
    const uint32_t total = (uint32_t)rows * vpr;
    for (uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += gridDim.x * blockDim.x) {
        const uint32_t r = idx / vpr;
        const i64 f = (i64)(idx - r * vpr) * V;
        float av[V], cv[V], g[V], oa[V], oc[V];
        ldv<TI, V>(a + r * lda + f, av);
        ldv<TI, V>(cc + r * lda + f, cv);
        ldv<TG, V>(dh + r * F + f, g);
#pragma unroll
        for (int j = 0; j < V; ++j) {
            oa[j] = g[j] * cv[j] * silu_grad_f(av[j]);
            oc[j] = g[j] * silu_f(av[j]);
        }
        stv<T, V>(da + r * ldd + f, oa);
        stv<T, V>(dc + r * ldd + f, oc);
    }
}

// Vector width for a row-strided stream: 8 when every tensor is bf16, 4
// otherwise, 1 when a pitch, width or base pointer breaks the alignment.
static int swiglu_vec(bool all_bf16, i64 F, std::initializer_list<i64> pitches,
                      std::initializer_list<std::pair<const void*, int>> ptrs) {
    int v = all_bf16 ? 8 : 4;
    if (F % v) return 1;
    for (i64 p : pitches)
        if (p % v) return 1;
    for (auto& q : ptrs)
        if (!aligned_to(q.first, (size_t)v * q.second)) return 1;
    return v;
}

// Grid of the flat (row, vector) loops; the index space must fit 32 bits.
static int row_grid(Context* c, i64 rows, i64 F = 0, int v = 1) {
    const i64 total = F > 0 ? rows * (F / v) : rows * 256;
    CATNN_CHECK(total < (1ll << 31), CATNN_ERR_SHAPE, "swiglu: too many elements for one launch");
    return (int)std::max<i64>(1, std::min<i64>(cdiv(total, 256), (i64)c->sm_count * 16));
}

template <typename TI, typename T>
static void launch_swiglu(Context* c, const void* a, const void* cc, void* h, i64 rows, i64 F, i64 lda, i64 ldh,
                          int v, const int32_t* rows_dev) {
    int g = row_grid(c, rows, F, v);
    auto A = (const TI*)a;
    auto Cc = (const TI*)cc;
    auto H = (T*)h;
    if (v == 8) k_swiglu<TI, T, 8><<<g, 256, 0, c->stream>>>(A, Cc, H, rows, F, lda, ldh, rows_dev);
    else if (v == 4) k_swiglu<TI, T, 4><<<g, 256, 0, c->stream>>>(A, Cc, H, rows, F, lda, ldh, rows_dev);
    else k_swiglu<TI, T, 1><<<g, 256, 0, c->stream>>>(A, Cc, H, rows, F, lda, ldh, rows_dev);
}

void swiglu_act(Context* c, const void* a, const void* cc, void* h, i64 rows, i64 F, i64 lda, i64 ldh, int dtype,
                int in_dtype, const int32_t* rows_dev) {
    if (rows * F <= 0) return;
    if (in_dtype < 0) in_dtype = dtype;
    int is = in_dtype == CATNN_BF16 ? 2 : 4, os = dtype == CATNN_BF16 ? 2 : 4;
    int v = swiglu_vec(is == 2 && os == 2, F, {lda, ldh}, {{a, is}, {cc, is}, {h, os}});
    if (dtype == CATNN_BF16 && in_dtype == CATNN_F32) launch_swiglu<float, bf16>(c, a, cc, h, rows, F, lda, ldh, v, rows_dev);
    else if (dtype == CATNN_BF16) launch_swiglu<bf16, bf16>(c, a, cc, h, rows, F, lda, ldh, v, rows_dev);
    else launch_swiglu<float, float>(c, a, cc, h, rows, F, lda, ldh, v, rows_dev);
    launched(c);
}

template <typename TI, typename TG, typename T>
static void launch_swiglu_bwd(Context* c, const void* a, const void* cc, const void* dh, void* da, void* dc, i64 rows,
                              i64 F, i64 lda, i64 ldd, int v, const int32_t* rows_dev) {
    int g = row_grid(c, rows, F, v);
    auto A = (const TI*)a;
    auto Cc = (const TI*)cc;
    auto G = (const TG*)dh;
    auto DA = (T*)da;
    auto DC = (T*)dc;
    if (v == 8) k_swiglu_bwd<TI, TG, T, 8><<<g, 256, 0, c->stream>>>(A, Cc, G, DA, DC, rows, F, lda, ldd, rows_dev);
    else if (v == 4) k_swiglu_bwd<TI, TG, T, 4><<<g, 256, 0, c->stream>>>(A, Cc, G, DA, DC, rows, F, lda, ldd, rows_dev);
    else k_swiglu_bwd<TI, TG, T, 1><<<g, 256, 0, c->stream>>>(A, Cc, G, DA, DC, rows, F, lda, ldd, rows_dev);
}

void swiglu_act_bwd(Context* c, const void* a, const void* cc, const void* dh, void* da, void* dc, i64 rows, i64 F,
                    i64 lda, i64 ldd, int dtype, int in_dtype, const int32_t* rows_dev) {
    if (rows * F <= 0) return;
    if (in_dtype < 0) in_dtype = dtype;
    int is = in_dtype == CATNN_BF16 ? 2 : 4, os = dtype == CATNN_BF16 ? 2 : 4;
    // dh has the input's type (fp32 intermediates with fp32 inputs)
    int v = swiglu_vec(is == 2 && os == 2, F, {lda, ldd}, {{a, is}, {cc, is}, {dh, is}, {da, os}, {dc, os}});
    if (dtype == CATNN_BF16 && in_dtype == CATNN_F32)
        launch_swiglu_bwd<float, float, bf16>(c, a, cc, dh, da, dc, rows, F, lda, ldd, v, rows_dev);
    else if (dtype == CATNN_BF16) launch_swiglu_bwd<bf16, bf16, bf16>(c, a, cc, dh, da, dc, rows, F, lda, ldd, v, rows_dev);
    else launch_swiglu_bwd<float, float, float>(c, a, cc, dh, da, dc, rows, F, lda, ldd, v, rows_dev);
    launched(c);
}

// The router's top-k (128 tokens per CTA) and the SwiGLU activation
// (grid-stride, 256 threads).
KernelInfo moe_info(Context* c, const std::string& op, int dtype, const KShape& s) {
    KernelInfo k;
    const bool b = dtype == CATNN_BF16;
    if (op == "router") {
        k.fn = (const void*)k_router_topk;
        k.file = "moe.cu";
        k.grid[0] = (unsigned)cdiv(s.rows, 128);
        k.block[0] = 128;
    } else if (op == "swiglu") {
        k.fn = b ? (const void*)k_swiglu<bf16, bf16, 8> : (const void*)k_swiglu<float, float, 4>;
        k.file = "moe.cu";
        k.grid[0] = (unsigned)row_grid(c, std::max<i64>(1, s.rows), s.width, b ? 8 : 4);
        k.block[0] = 256;
    }
    return k;
}

}  // namespace catnn
