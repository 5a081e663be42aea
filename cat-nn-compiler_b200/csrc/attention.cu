// Embedding gather / deterministic scatter-add, RoPE, and the attention
// core (forward with log-sum-exp, backward in two passes: dQ per query
// block; dK/dV per key block). These CUDA-core kernels serve the fp32
// parity path and any head size up to 128; the bf16 tensor-core attention
// lives in attention_tc.cu.
#include "ops.cuh"

namespace catnn {

// ------------------------------------------------------------ embedding
// moe.rs:34-45. Out-of-range ids set *err and write zeros.
template <typename T>
__global__ void k_embed(const uint32_t* __restrict__ ids, i64 n, const T* __restrict__ table, i64 vocab, i64 hidden,
                        T* __restrict__ y, int* err) {
    i64 t = blockIdx.x;
    uint32_t id = ids[t];
    bool bad = (i64)id >= vocab;
    if (bad && threadIdx.x == 0 && err) atomicExch(err, 1);
    for (i64 i = threadIdx.x; i < hidden; i += blockDim.x) y[t * hidden + i] = bad ? T(0.f) : table[(i64)id * hidden + i];
}

void embedding_fwd(Context* c, const uint32_t* ids, i64 n, const void* table, i64 vocab, i64 hidden, void* y, int dtype,
                   int* err) {
    if (n <= 0 || hidden <= 0) return;
    int th = hidden >= 256 ? 256 : 64;
    if (dtype == CATNN_BF16) k_embed<<<n, th, 0, c->stream>>>(ids, n, (const bf16*)table, vocab, hidden, (bf16*)y, err);
    else k_embed<<<n, th, 0, c->stream>>>(ids, n, (const float*)table, vocab, hidden, (float*)y, err);
    launched(c);
}

// Single-CTA bitonic sort of 32-bit keys in shared memory (n <= 32768,
// padded to a power of two with 0xFFFFFFFF). Keys are unique by
// construction (id * n + t), so the order is total and deterministic.
__global__ void k_bitonic_keys(const uint32_t* __restrict__ ids, i64 n, uint32_t* __restrict__ out, int npow) {
    extern __shared__ uint32_t sk[];
    for (int i = threadIdx.x; i < npow; i += blockDim.x)
        sk[i] = i < n ? ids[i] * (uint32_t)n + (uint32_t)i : 0xFFFFFFFFu;
    __syncthreads();
    for (int k = 2; k <= npow; k <<= 1)
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < npow; i += blockDim.x) {
                int p = i ^ j;
                if (p > i) {
                    uint32_t a = sk[i], b = sk[p];
                    bool up = (i & k) == 0;
                    if ((a > b) == up) {
                        sk[i] = b;
                        sk[p] = a;
                    }
                }
            }
            __syncthreads();
        }
    for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = sk[i];
}

// One CTA per sorted position; a CTA that starts a run of equal ids sums
// that run's dy rows in token order into dw[id] (adjoint.rs:195-206 adds
// rows in t order onto zeros, so the fp32 result is bit-identical).
template <typename T>
__global__ void k_embed_bwd_runs(const uint32_t* __restrict__ keys, i64 n, const T* __restrict__ dy, float* __restrict__ dw,
                                 i64 hidden) {
    i64 i = blockIdx.x;
    uint32_t id = keys[i] / (uint32_t)n;
    if (i > 0 && keys[i - 1] / (uint32_t)n == id) return;
    i64 end = i + 1;
    while (end < n && keys[end] / (uint32_t)n == id) ++end;
    for (i64 col = threadIdx.x; col < hidden; col += blockDim.x) {
        float s = 0.f;
        for (i64 r = i; r < end; ++r) {
            i64 t = keys[r] % (uint32_t)n;
            s = __fadd_rn(s, ld(dy + t * hidden + col));
        }
        dw[(i64)id * hidden + col] = s;
    }
}

// k_embed_bwd_runs with 4 consecutive columns per thread (16-byte loads of
// fp32 dy rows and stores of dw, 8-byte loads of bf16 rows); each column is
// still summed in token order onto zero, so the result is the same bits.
template <typename T>
__global__ void __launch_bounds__(256) k_embed_bwd_runs4(const uint32_t* __restrict__ keys, i64 n,
                                                         const T* __restrict__ dy, float* __restrict__ dw, i64 hidden) {
    const i64 i = blockIdx.x;
    const uint32_t id = keys[i] / (uint32_t)n;
    if (i > 0 && keys[i - 1] / (uint32_t)n == id) return;
    i64 end = i + 1;
    while (end < n && keys[end] / (uint32_t)n == id) ++end;
    for (i64 col = (i64)threadIdx.x * 4; col < hidden; col += (i64)blockDim.x * 4) {
        float s[4] = {0.f, 0.f, 0.f, 0.f};
        for (i64 r = i; r < end; ++r) {
            const i64 t = keys[r] % (uint32_t)n;
            float v[4];
            ldv<T, 4>(dy + t * hidden + col, v);
#pragma unroll
            for (int u = 0; u < 4; ++u) s[u] = __fadd_rn(s[u], v[u]);
        }
        stv<float, 4>(dw + (i64)id * hidden + col, s);
    }
}

static void embed_bwd_check(i64 n, i64 vocab) {
    CATNN_CHECK(n <= 32768, CATNN_ERR_UNSUPPORTED, "embedding_bwd: at most 32768 tokens per call");
    CATNN_CHECK((unsigned long long)vocab * (unsigned long long)n < 0xFFFFFFFFull, CATNN_ERR_UNSUPPORTED,
                "embedding_bwd: vocab * tokens must fit in 32 bits");
}

void embedding_bwd_keys(Context* c, const uint32_t* ids, i64 n, i64 vocab, uint32_t* keys) {
    if (n <= 0) return;
    embed_bwd_check(n, vocab);
    int npow = 1;
    while (npow < n) npow <<= 1;
    static bool attr[64] = {false};
    if (!attr[c->device]) {
        CUDA_OK(cudaFuncSetAttribute(k_bitonic_keys, cudaFuncAttributeMaxDynamicSharedMemorySize, 32768 * 4));
        attr[c->device] = true;
    }
    k_bitonic_keys<<<1, 1024, (size_t)npow * 4, c->stream>>>(ids, n, keys, npow);
    launched(c);
}

void embedding_bwd_runs(Context* c, const uint32_t* keys, i64 n, const void* dy, float* dw, i64 vocab, i64 hidden,
                        int dtype) {
    if (vocab <= 0 || hidden <= 0) return;
    CUDA_OK(cudaMemsetAsync(dw, 0, (size_t)vocab * hidden * 4, c->stream));
    if (n <= 0) return;
    int th = hidden >= 256 ? 256 : 64;
    if (hidden % 4 == 0 && aligned_to(dw, 16) && aligned_to(dy, dtype == CATNN_BF16 ? 8 : 16)) {
        const int t4 = (int)std::min<i64>(256, std::max<i64>(32, cdiv(hidden / 4, 32) * 32));
        if (dtype == CATNN_BF16) k_embed_bwd_runs4<<<n, t4, 0, c->stream>>>(keys, n, (const bf16*)dy, dw, hidden);
        else k_embed_bwd_runs4<<<n, t4, 0, c->stream>>>(keys, n, (const float*)dy, dw, hidden);
    } else if (dtype == CATNN_BF16) k_embed_bwd_runs<<<n, th, 0, c->stream>>>(keys, n, (const bf16*)dy, dw, hidden);
    else k_embed_bwd_runs<<<n, th, 0, c->stream>>>(keys, n, (const float*)dy, dw, hidden);
    launched(c);
}

void embedding_bwd(Context* c, const uint32_t* ids, i64 n, const void* dy, float* dw, i64 vocab, i64 hidden, int dtype) {
    if (vocab <= 0 || hidden <= 0) return;
    if (n > 0) embed_bwd_check(n, vocab);
    uint32_t* keys = n > 0 ? (uint32_t*)c->scratch_for((size_t)n * 4) : nullptr;
    embedding_bwd_keys(c, ids, n, vocab, keys);
    embedding_bwd_runs(c, keys, n, dy, dw, vocab, hidden, dtype);
}

// ------------------------------------------------------------ RoPE
// moe.rs:47-59 / adjoint.rs:454-466: angle pos·θ^(-2i/hd) in f64, sin/cos
// rounded to f32, pair (2i, 2i+1) rotated (inverse: sin negated).
// The (cos, sin) pairs depend only on (θ, S, hd): they are computed once in
// f64 into a cached [S, hd/2] table, so the rotation itself is a pure
// bandwidth pass.
__global__ void k_rope_table(float2* __restrict__ tab, i64 s, i64 hd, double theta) {
    i64 half = hd / 2;
    for (i64 idx = blockIdx.x * (i64)blockDim.x + threadIdx.x; idx < s * half; idx += (i64)gridDim.x * blockDim.x) {
        i64 i = idx % half, pos = idx / half;
        double freq = 1.0 / pow(theta, 2.0 * (double)i / (double)hd);
        double sd, cd;
        sincos((double)pos * freq, &sd, &cd);
        tab[idx] = make_float2((float)cd, (float)sd);
    }
}

// Element pair (2i, 2i+1) of one head as one 4-byte (bf16) or 8-byte (fp32) access.
template <typename T> struct Pair;
template <> struct Pair<float> {
    static __device__ __forceinline__ float2 get(const float* p) { return *(const float2*)p; }
    static __device__ __forceinline__ void put(float* p, float a, float b) { *(float2*)p = make_float2(a, b); }
};
template <> struct Pair<bf16> {
    static __device__ __forceinline__ float2 get(const bf16* p) { return __bfloat1622float2(*(const __nv_bfloat162*)p); }
    static __device__ __forceinline__ void put(bf16* p, float a, float b) {
        *(__nv_bfloat162*)p = __floats2bfloat162_rn(a, b);
    }
};

// bf16 form: a thread rotates 4 consecutive pairs (one 16-byte load and
// store); same arithmetic per pair as k_rope.
__global__ void __launch_bounds__(256) k_rope8(bf16* __restrict__ x, const float2* __restrict__ tab, i64 b, i64 s,
                                               int heads, int hd, int inverse, i64 row_stride, i64 col_off) {
    const int half = hd / 2, groups = heads * half / 4;  // 4 pairs per group (half % 4 == 0)
    for (i64 tok = blockIdx.x; tok < b * s; tok += gridDim.x) {
        const float2* trow = tab + (tok % s) * half;
        bf16* xr = x + tok * row_stride + col_off;
        for (int g = threadIdx.x; g < groups; g += blockDim.x) {
            const int j0 = g * 4, h = j0 / half, i0 = j0 - h * half;
            bf16* p = xr + h * hd + 2 * i0;
            float v[8];
            ldv<bf16, 8>(p, v);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                float2 cs_sn = trow[i0 + u];
                float cs = cs_sn.x, sn = inverse ? -cs_sn.y : cs_sn.y;
                float a0 = v[2 * u], b0 = v[2 * u + 1];
                v[2 * u] = __fsub_rn(__fmul_rn(a0, cs), __fmul_rn(b0, sn));
                v[2 * u + 1] = __fadd_rn(__fmul_rn(a0, sn), __fmul_rn(b0, cs));
            }
            stv<bf16, 8>(p, v);
        }
    }
}

// CTAs stride over token rows, threads over the (head, pair) slots of a row.
template <typename T>
__global__ void __launch_bounds__(256) k_rope(T* __restrict__ x, const float2* __restrict__ tab, i64 b, i64 s, int heads,
                                              int hd, int inverse, i64 row_stride, i64 col_off) {
    const int half = hd / 2, slots = heads * half;
    for (i64 tok = blockIdx.x; tok < b * s; tok += gridDim.x) {
        const float2* trow = tab + (tok % s) * half;
        T* xr = x + tok * row_stride + col_off;
        for (int j = threadIdx.x; j < slots; j += blockDim.x) {
            int h = j / half, i = j - h * half;
            float2 cs_sn = trow[i];
            float cs = cs_sn.x, sn = inverse ? -cs_sn.y : cs_sn.y;
            T* p = xr + h * hd + 2 * i;
            float2 v = Pair<T>::get(p);
            Pair<T>::put(p, __fsub_rn(__fmul_rn(v.x, cs), __fmul_rn(v.y, sn)),
                         __fadd_rn(__fmul_rn(v.x, sn), __fmul_rn(v.y, cs)));
        }
    }
}

const float2* rope_table(Context* c, i64 s, i64 hd, double theta) {
    if (c->rope_tab && c->rope_s == s && c->rope_hd == hd && c->rope_theta == theta) return (const float2*)c->rope_tab;
    if (c->rope_tab) {
        CUDA_OK(cudaStreamSynchronize(c->stream));
        CUDA_OK(cudaFree(c->rope_tab));
        c->rope_tab = nullptr;
    }
    i64 n = s * (hd / 2);
    CUDA_OK(cudaMalloc(&c->rope_tab, (size_t)(n > 0 ? n : 1) * sizeof(float2)));
    int grid = (int)((n + 255) / 256);
    if (grid > c->sm_count * 8) grid = c->sm_count * 8;
    if (grid < 1) grid = 1;
    k_rope_table<<<grid, 256, 0, c->stream>>>((float2*)c->rope_tab, s, hd, theta);
    launched(c);
    c->rope_s = s;
    c->rope_hd = hd;
    c->rope_theta = theta;
    return (const float2*)c->rope_tab;
}

void rope(Context* c, void* x, i64 b, i64 s, i64 heads, i64 hd, double theta, bool inverse, int dtype, i64 row_stride,
          i64 col_off) {
    if (b * s * heads * (hd / 2) <= 0) return;
    if (row_stride == 0) row_stride = heads * hd;
    const float2* tab = rope_table(c, s, hd, theta);
    CATNN_CHECK(hd % 2 == 0 && row_stride % 2 == 0 && col_off % 2 == 0 && heads * hd <= (1 << 30), CATNN_ERR_SHAPE,
                "rope: head dim, row stride and column offset must be even");
    CATNN_CHECK(aligned_to(x, dtype == CATNN_BF16 ? 4 : 8), CATNN_ERR_INVALID, "rope: misaligned tensor");
    int grid = (int)std::min<i64>(b * s, (i64)c->sm_count * 16);
    if (dtype == CATNN_BF16 && (hd / 2) % 4 == 0 && row_stride % 8 == 0 && col_off % 8 == 0 && aligned_to(x, 16))
        k_rope8<<<grid, 256, 0, c->stream>>>((bf16*)x, tab, b, s, (int)heads, (int)hd, inverse ? 1 : 0, row_stride,
                                             col_off);
    else if (dtype == CATNN_BF16)
        k_rope<<<grid, 256, 0, c->stream>>>((bf16*)x, tab, b, s, (int)heads, (int)hd, inverse ? 1 : 0, row_stride,
                                            col_off);
    else
        k_rope<<<grid, 256, 0, c->stream>>>((float*)x, tab, b, s, (int)heads, (int)hd, inverse ? 1 : 0, row_stride,
                                            col_off);
    launched(c);
}

// ------------------------------------------------------------ attention
// Key range of query i: [lo, hi]. causal: hi = i (and window: lo = i-w+1);
// non-causal: all keys.
__device__ __forceinline__ void key_range(i64 i, i64 s, int causal, i64 window, i64& lo, i64& hi) {
    if (causal) {
        hi = i;
        lo = window > 0 ? (i - window + 1 > 0 ? i - window + 1 : 0) : 0;
    } else {
        lo = 0;
        hi = s - 1;
    }
}

static const int AQ = 16;   // query rows per CTA (4 warps x 4 rows)
static const int AK = 64;   // keys per shared-memory tile
static const int HDMAX = 128;

// Row-major [rows][P] view of a shared-memory tile (P = hd + 1 pads the
// rows so lanes reading one column of consecutive rows hit distinct banks).
struct SmemMat {
    float* p;
    int P;
    __device__ __forceinline__ float* operator[](int r) const { return p + r * P; }
};

static size_t attn_smem_bytes(int kind, i64 hd) {
    // 0: fwd (K,V: AK rows; Q: AQ), 1: dq (+dO: AQ), 2: dkv (Q,dO: AK; K,V: AQ; lse, D)
    i64 P = hd + 1;
    if (kind == 0) return (size_t)(2 * AK + AQ) * P * 4;
    if (kind == 1) return (size_t)(2 * AK + 2 * AQ) * P * 4;
    return (size_t)(2 * AK + 2 * AQ) * P * 4 + 2 * AK * 4;
}

template <typename Kern>
static void attn_smem_attr(Kern k, size_t bytes) {
    CUDA_OK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
}

struct AttnArgs {
    const void *q, *k, *v, *o, *dout;
    void *out, *dq, *dk, *dv;
    float* lse;
    const float* dsum;  // D_i = <dO_i, O_i>, [B,H,S]
    i64 b, s, h, hkv, hd, q_stride, kv_stride;
    int causal;
    i64 window;
    float scale;
};

// Forward: CTA = (query block, head, batch). Online softmax per row; lane l
// owns output dims {l, l+32, l+64, l+96} < hd.
template <typename T>
__global__ void __launch_bounds__(128) k_attn_fwd(AttnArgs a) {
    extern __shared__ float attn_smem[];
    const int P = (int)a.hd + 1;
    SmemMat Ks{attn_smem, P}, Vs{attn_smem + AK * P, P}, Qs{attn_smem + 2 * AK * P, P};
    const T* Q = (const T*)a.q;
    const T* K = (const T*)a.k;
    const T* V = (const T*)a.v;
    T* O = (T*)a.out;
    i64 bi = blockIdx.z, h = blockIdx.y, q0 = (i64)blockIdx.x * AQ;
    i64 kvh = h / (a.h / a.hkv);
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int idx = threadIdx.x; idx < AQ * a.hd; idx += blockDim.x) {
        int r = idx / (int)a.hd, d = idx % (int)a.hd;
        i64 qi = q0 + r;
        Qs[r][d] = qi < a.s ? ld(Q + (bi * a.s + qi) * a.q_stride + h * a.hd + d) : 0.f;
    }
    float m[4], l[4], acc[4][4];
    for (int r = 0; r < 4; ++r) {
        m[r] = -INFINITY;
        l[r] = 0.f;
        for (int d = 0; d < 4; ++d) acc[r][d] = 0.f;
    }
    // union of the key ranges of this block's queries
    i64 qlast = min(q0 + AQ - 1, a.s - 1);
    i64 lo0, hi0, lo1, hi1;
    key_range(q0, a.s, a.causal, a.window, lo0, hi0);
    key_range(qlast, a.s, a.causal, a.window, lo1, hi1);
    i64 klo = lo0, khi = hi1;
    for (i64 k0 = (klo / AK) * AK; k0 <= khi; k0 += AK) {
        __syncthreads();
        for (int idx = threadIdx.x; idx < AK * a.hd; idx += blockDim.x) {
            int r = idx / (int)a.hd, d = idx % (int)a.hd;
            i64 kj = k0 + r;
            bool ok = kj < a.s;
            Ks[r][d] = ok ? ld(K + (bi * a.s + kj) * a.kv_stride + kvh * a.hd + d) : 0.f;
            Vs[r][d] = ok ? ld(V + (bi * a.s + kj) * a.kv_stride + kvh * a.hd + d) : 0.f;
        }
        __syncthreads();
        for (int r = 0; r < 4; ++r) {
            int qr = warp * 4 + r;
            i64 qi = q0 + qr;
            if (qi >= a.s) continue;
            i64 lo, hi;
            key_range(qi, a.s, a.causal, a.window, lo, hi);
            float sc[2];
            for (int u = 0; u < 2; ++u) {
                i64 kj = k0 + lane + 32 * u;
                float d = -INFINITY;
                if (kj >= lo && kj <= hi && kj < a.s) {
                    float dot = 0.f;
                    for (int t = 0; t < a.hd; ++t) dot += Qs[qr][t] * Ks[lane + 32 * u][t];
                    d = dot * a.scale;
                }
                sc[u] = d;
            }
            float tmax = warp_max(fmaxf(sc[0], sc[1]));
            if (tmax == -INFINITY) continue;
            float mn = fmaxf(m[r], tmax);
            float alpha = expf(m[r] - mn);  // m = -inf -> 0
            float p0 = expf(sc[0] - mn), p1 = expf(sc[1] - mn);
            l[r] = l[r] * alpha + warp_sum(p0 + p1);
            for (int d = 0; d < 4; ++d) acc[r][d] *= alpha;
            for (int j = 0; j < AK; ++j) {
                float pj = __shfl_sync(0xffffffffu, j < 32 ? p0 : p1, j & 31);
                if (pj == 0.f) continue;
                for (int d = 0; d < 4; ++d) {
                    int dd = lane + 32 * d;
                    if (dd < a.hd) acc[r][d] += pj * Vs[j][dd];
                }
            }
            m[r] = mn;
        }
    }
    for (int r = 0; r < 4; ++r) {
        i64 qi = q0 + warp * 4 + r;
        if (qi >= a.s) continue;
        float inv = l[r] > 0.f ? 1.0f / fmaxf(l[r], 1e-30f) : 0.f;
        for (int d = 0; d < 4; ++d) {
            int dd = lane + 32 * d;
            if (dd < a.hd) st(O + (bi * a.s + qi) * (a.h * a.hd) + h * a.hd + dd, acc[r][d] * inv);
        }
        if (lane == 0) a.lse[(bi * a.h + h) * a.s + qi] = l[r] > 0.f ? m[r] + logf(l[r]) : -INFINITY;
    }
}

bool attention_tc_ok(i64 hd, i64 q_stride, i64 kv_stride, const void* q, const void* k, const void* v);
bool attention_fwd_tc5_ok(i64 hd, i64 q_stride, i64 kv_stride, const void* q, const void* k, const void* v);
void attention_fwd_tc5(Context* c, const void* q, const void* k, const void* v, void* o, float* lse, i64 b, i64 s,
                       i64 h, i64 hkv, bool causal, i64 window, i64 q_stride, i64 kv_stride);
void attention_fwd_tc(Context* c, const void* q, const void* k, const void* v, void* o, float* lse, i64 b, i64 s, i64 h,
                      i64 hkv, i64 hd, bool causal, i64 window, i64 q_stride, i64 kv_stride);
void attention_bwd_tc(Context* c, const void* q, const void* k, const void* v, const void* o, const float* lse,
                      const void* dout, void* dq, void* dk, void* dv, i64 b, i64 s, i64 h, i64 hkv, i64 hd, bool causal,
                      i64 window, i64 q_stride, i64 kv_stride);

void attention_fwd(Context* c, const void* q, const void* k, const void* v, void* o, float* lse, i64 b, i64 s, i64 h,
                   i64 hkv, i64 hd, bool causal, i64 window, int dtype, i64 q_stride, i64 kv_stride) {
    if (b <= 0 || s <= 0 || h <= 0) return;
    CATNN_CHECK(hd > 0 && hd <= HDMAX, CATNN_ERR_UNSUPPORTED, "attention: head_dim must be in [1, 128]");
    CATNN_CHECK(hkv > 0 && h % hkv == 0, CATNN_ERR_SHAPE, "attention: n_heads must be a multiple of n_kv_heads");
    const i64 qs = q_stride ? q_stride : h * hd, ks = kv_stride ? kv_stride : hkv * hd;
    if (dtype == CATNN_BF16 && attention_fwd_tc5_ok(hd, qs, ks, q, k, v)) {
        // tcgen05 + TMEM (head_dim 64)
        attention_fwd_tc5(c, q, k, v, o, lse, b, s, h, hkv, causal, window, qs, ks);
        return;
    }
    if (dtype == CATNN_BF16 && attention_tc_ok(hd, qs, ks, q, k, v)) {
        attention_fwd_tc(c, q, k, v, o, lse, b, s, h, hkv, hd, causal, window, qs, ks);
        return;
    }
    AttnArgs a{};
    a.q = q; a.k = k; a.v = v; a.out = o; a.lse = lse;
    a.b = b; a.s = s; a.h = h; a.hkv = hkv; a.hd = hd;
    a.q_stride = q_stride ? q_stride : h * hd;
    a.kv_stride = kv_stride ? kv_stride : hkv * hd;
    a.causal = causal ? 1 : 0;
    a.window = window;
    a.scale = 1.0f / sqrtf((float)hd);
    dim3 grid(cdiv(s, AQ), h, b);
    CATNN_CHECK(grid.y <= 65535 && grid.z <= 65535, CATNN_ERR_SHAPE, "attention: too many heads/batches");
    size_t sm = attn_smem_bytes(0, hd);
    if (dtype == CATNN_BF16) {
        attn_smem_attr(k_attn_fwd<bf16>, sm);
        k_attn_fwd<bf16><<<grid, 128, sm, c->stream>>>(a);
    } else {
        attn_smem_attr(k_attn_fwd<float>, sm);
        k_attn_fwd<float><<<grid, 128, sm, c->stream>>>(a);
    }
    launched(c);
}

// D_i = <dO_i, O_i> per (b, h, i): the softmax-adjoint row term.
template <typename T>
__global__ void k_attn_dsum(const T* __restrict__ o, const T* __restrict__ dout, float* __restrict__ dsum, i64 b, i64 s,
                            i64 h, i64 hd) {
    i64 row = blockIdx.x * 4 + (threadIdx.x >> 5);  // row over (b, s, h)
    int lane = threadIdx.x & 31;
    if (row >= b * s * h) return;
    i64 hh = row % h, tok = row / h;
    float acc = 0.f;
    for (i64 d = lane; d < hd; d += 32) acc += ld(o + tok * h * hd + hh * hd + d) * ld(dout + tok * h * hd + hh * hd + d);
    acc = warp_sum(acc);
    i64 bi = tok / s, i = tok % s;
    if (lane == 0) dsum[(bi * h + hh) * s + i] = acc;
}

// dQ: CTA = (query block, head, batch). dq_i = scale Σ_j p_ij (dp_ij - D_i) k_j.
template <typename T>
__global__ void __launch_bounds__(128) k_attn_dq(AttnArgs a) {
    extern __shared__ float attn_smem[];
    const int P = (int)a.hd + 1;
    SmemMat Ks{attn_smem, P}, Vs{attn_smem + AK * P, P}, Qs{attn_smem + 2 * AK * P, P},
        Gs{attn_smem + (2 * AK + AQ) * P, P};
    const T* Q = (const T*)a.q;
    const T* K = (const T*)a.k;
    const T* V = (const T*)a.v;
    const T* dO = (const T*)a.dout;
    T* dQ = (T*)a.dq;
    i64 bi = blockIdx.z, h = blockIdx.y, q0 = (i64)blockIdx.x * AQ;
    i64 kvh = h / (a.h / a.hkv);
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int idx = threadIdx.x; idx < AQ * a.hd; idx += blockDim.x) {
        int r = idx / (int)a.hd, d = idx % (int)a.hd;
        i64 qi = q0 + r;
        bool ok = qi < a.s;
        Qs[r][d] = ok ? ld(Q + (bi * a.s + qi) * a.q_stride + h * a.hd + d) : 0.f;
        Gs[r][d] = ok ? ld(dO + (bi * a.s + qi) * (a.h * a.hd) + h * a.hd + d) : 0.f;
    }
    float acc[4][4];
    for (int r = 0; r < 4; ++r)
        for (int d = 0; d < 4; ++d) acc[r][d] = 0.f;
    i64 qlast = min(q0 + AQ - 1, a.s - 1);
    i64 lo0, hi0, lo1, hi1;
    key_range(q0, a.s, a.causal, a.window, lo0, hi0);
    key_range(qlast, a.s, a.causal, a.window, lo1, hi1);
    for (i64 k0 = (lo0 / AK) * AK; k0 <= hi1; k0 += AK) {
        __syncthreads();
        for (int idx = threadIdx.x; idx < AK * a.hd; idx += blockDim.x) {
            int r = idx / (int)a.hd, d = idx % (int)a.hd;
            i64 kj = k0 + r;
            bool ok = kj < a.s;
            Ks[r][d] = ok ? ld(K + (bi * a.s + kj) * a.kv_stride + kvh * a.hd + d) : 0.f;
            Vs[r][d] = ok ? ld(V + (bi * a.s + kj) * a.kv_stride + kvh * a.hd + d) : 0.f;
        }
        __syncthreads();
        for (int r = 0; r < 4; ++r) {
            int qr = warp * 4 + r;
            i64 qi = q0 + qr;
            if (qi >= a.s) continue;
            i64 lo, hi;
            key_range(qi, a.s, a.causal, a.window, lo, hi);
            float L = a.lse[(bi * a.h + h) * a.s + qi];
            float Dd = a.dsum[(bi * a.h + h) * a.s + qi];
            float ds[2];
            for (int u = 0; u < 2; ++u) {
                int jj = lane + 32 * u;
                i64 kj = k0 + jj;
                float val = 0.f;
                if (kj >= lo && kj <= hi && kj < a.s) {
                    float dot = 0.f, dp = 0.f;
                    for (int t = 0; t < a.hd; ++t) {
                        dot += Qs[qr][t] * Ks[jj][t];
                        dp += Gs[qr][t] * Vs[jj][t];
                    }
                    float p = expf(dot * a.scale - L);
                    val = p * (dp - Dd) * a.scale;
                }
                ds[u] = val;
            }
            for (int j = 0; j < AK; ++j) {
                float dj = __shfl_sync(0xffffffffu, j < 32 ? ds[0] : ds[1], j & 31);
                if (dj == 0.f) continue;
                for (int d = 0; d < 4; ++d) {
                    int dd = lane + 32 * d;
                    if (dd < a.hd) acc[r][d] += dj * Ks[j][dd];
                }
            }
        }
    }
    for (int r = 0; r < 4; ++r) {
        i64 qi = q0 + warp * 4 + r;
        if (qi >= a.s) continue;
        for (int d = 0; d < 4; ++d) {
            int dd = lane + 32 * d;
            if (dd < a.hd) st(dQ + (bi * a.s + qi) * a.q_stride + h * a.hd + dd, acc[r][d]);
        }
    }
}

// dK, dV: CTA = (key block of 16, kv head, batch); loops over the query
// heads that share the kv head and over the queries that see each key.
template <typename T>
__global__ void __launch_bounds__(128) k_attn_dkv(AttnArgs a) {
    extern __shared__ float attn_smem[];
    const int P = (int)a.hd + 1;
    SmemMat Qs{attn_smem, P}, Gs{attn_smem + AK * P, P}, Ks{attn_smem + 2 * AK * P, P},
        Vs{attn_smem + (2 * AK + AQ) * P, P};
    float* Ls = attn_smem + (2 * AK + 2 * AQ) * P;
    float* Ds = Ls + AK;
    const T* Q = (const T*)a.q;
    const T* K = (const T*)a.k;
    const T* V = (const T*)a.v;
    const T* dO = (const T*)a.dout;
    T* dK = (T*)a.dk;
    T* dV = (T*)a.dv;
    i64 bi = blockIdx.z, kvh = blockIdx.y, j0 = (i64)blockIdx.x * AQ;
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    i64 rep = a.h / a.hkv;
    for (int idx = threadIdx.x; idx < AQ * a.hd; idx += blockDim.x) {
        int r = idx / (int)a.hd, d = idx % (int)a.hd;
        i64 kj = j0 + r;
        bool ok = kj < a.s;
        Ks[r][d] = ok ? ld(K + (bi * a.s + kj) * a.kv_stride + kvh * a.hd + d) : 0.f;
        Vs[r][d] = ok ? ld(V + (bi * a.s + kj) * a.kv_stride + kvh * a.hd + d) : 0.f;
    }
    float dk[4][4], dv[4][4];
    for (int r = 0; r < 4; ++r)
        for (int d = 0; d < 4; ++d) dk[r][d] = dv[r][d] = 0.f;
    // queries that can see keys [j0, j0+AQ): causal -> i >= j0 (and i < j_last + window)
    i64 jlast = min(j0 + AQ - 1, a.s - 1);
    i64 qlo = a.causal ? j0 : 0;
    i64 qhi = a.s - 1;
    if (a.causal && a.window > 0) qhi = min(qhi, jlast + a.window - 1);
    for (i64 hq = kvh * rep; hq < (kvh + 1) * rep; ++hq) {
        for (i64 i0 = (qlo / AK) * AK; i0 <= qhi; i0 += AK) {
            __syncthreads();
            for (int idx = threadIdx.x; idx < AK * a.hd; idx += blockDim.x) {
                int r = idx / (int)a.hd, d = idx % (int)a.hd;
                i64 qi = i0 + r;
                bool ok = qi < a.s;
                Qs[r][d] = ok ? ld(Q + (bi * a.s + qi) * a.q_stride + hq * a.hd + d) : 0.f;
                Gs[r][d] = ok ? ld(dO + (bi * a.s + qi) * (a.h * a.hd) + hq * a.hd + d) : 0.f;
            }
            for (int r = threadIdx.x; r < AK; r += blockDim.x) {
                i64 qi = i0 + r;
                Ls[r] = qi < a.s ? a.lse[(bi * a.h + hq) * a.s + qi] : 0.f;
                Ds[r] = qi < a.s ? a.dsum[(bi * a.h + hq) * a.s + qi] : 0.f;
            }
            __syncthreads();
            for (int r = 0; r < 4; ++r) {
                int kr = warp * 4 + r;
                i64 kj = j0 + kr;
                if (kj >= a.s) continue;
                float pp[2], dss[2];
                for (int u = 0; u < 2; ++u) {
                    int ii = lane + 32 * u;
                    i64 qi = i0 + ii;
                    float p = 0.f, dsv = 0.f;
                    i64 lo, hi;
                    key_range(qi, a.s, a.causal, a.window, lo, hi);
                    if (qi < a.s && kj >= lo && kj <= hi) {
                        float dot = 0.f, dp = 0.f;
                        for (int t = 0; t < a.hd; ++t) {
                            dot += Qs[ii][t] * Ks[kr][t];
                            dp += Gs[ii][t] * Vs[kr][t];
                        }
                        p = expf(dot * a.scale - Ls[ii]);
                        dsv = p * (dp - Ds[ii]) * a.scale;
                    }
                    pp[u] = p;
                    dss[u] = dsv;
                }
                for (int i = 0; i < AK; ++i) {
                    float pi = __shfl_sync(0xffffffffu, i < 32 ? pp[0] : pp[1], i & 31);
                    float di = __shfl_sync(0xffffffffu, i < 32 ? dss[0] : dss[1], i & 31);
                    if (pi == 0.f && di == 0.f) continue;
                    for (int d = 0; d < 4; ++d) {
                        int dd = lane + 32 * d;
                        if (dd < a.hd) {
                            dv[r][d] += pi * Gs[i][dd];
                            dk[r][d] += di * Qs[i][dd];
                        }
                    }
                }
            }
        }
    }
    for (int r = 0; r < 4; ++r) {
        i64 kj = j0 + warp * 4 + r;
        if (kj >= a.s) continue;
        for (int d = 0; d < 4; ++d) {
            int dd = lane + 32 * d;
            if (dd < a.hd) {
                st(dK + (bi * a.s + kj) * a.kv_stride + kvh * a.hd + dd, dk[r][d]);
                st(dV + (bi * a.s + kj) * a.kv_stride + kvh * a.hd + dd, dv[r][d]);
            }
        }
    }
}

void attention_bwd(Context* c, const void* q, const void* k, const void* v, const void* o, const float* lse,
                   const void* dout, void* dq, void* dk, void* dv, i64 b, i64 s, i64 h, i64 hkv, i64 hd, bool causal,
                   i64 window, int dtype, i64 q_stride, i64 kv_stride) {
    if (b <= 0 || s <= 0 || h <= 0) return;
    CATNN_CHECK(hd > 0 && hd <= HDMAX, CATNN_ERR_UNSUPPORTED, "attention: head_dim must be in [1, 128]");
    CATNN_CHECK(hkv > 0 && h % hkv == 0, CATNN_ERR_SHAPE, "attention: n_heads must be a multiple of n_kv_heads");
    if (dtype == CATNN_BF16 && attention_tc_ok(hd, q_stride ? q_stride : h * hd, kv_stride ? kv_stride : hkv * hd, q, k, v)) {
        attention_bwd_tc(c, q, k, v, o, lse, dout, dq, dk, dv, b, s, h, hkv, hd, causal, window,
                         q_stride ? q_stride : h * hd, kv_stride ? kv_stride : hkv * hd);
        return;
    }
    float* dsum = (float*)c->scratch_for((size_t)b * h * s * 4);
    AttnArgs a{};
    a.q = q; a.k = k; a.v = v; a.o = o; a.dout = dout; a.dq = dq; a.dk = dk; a.dv = dv;
    a.lse = const_cast<float*>(lse);
    a.dsum = dsum;
    a.b = b; a.s = s; a.h = h; a.hkv = hkv; a.hd = hd;
    a.q_stride = q_stride ? q_stride : h * hd;
    a.kv_stride = kv_stride ? kv_stride : hkv * hd;
    a.causal = causal ? 1 : 0;
    a.window = window;
    a.scale = 1.0f / sqrtf((float)hd);
    i64 rows = b * s * h;
    size_t s1 = attn_smem_bytes(1, hd), s2 = attn_smem_bytes(2, hd);
    if (dtype == CATNN_BF16) {
        attn_smem_attr(k_attn_dq<bf16>, s1);
        attn_smem_attr(k_attn_dkv<bf16>, s2);
        k_attn_dsum<<<cdiv(rows, 4), 128, 0, c->stream>>>((const bf16*)o, (const bf16*)dout, dsum, b, s, h, hd);
        k_attn_dq<bf16><<<dim3(cdiv(s, AQ), h, b), 128, s1, c->stream>>>(a);
        k_attn_dkv<bf16><<<dim3(cdiv(s, AQ), hkv, b), 128, s2, c->stream>>>(a);
    } else {
        attn_smem_attr(k_attn_dq<float>, s1);
        attn_smem_attr(k_attn_dkv<float>, s2);
        k_attn_dsum<<<cdiv(rows, 4), 128, 0, c->stream>>>((const float*)o, (const float*)dout, dsum, b, s, h, hd);
        k_attn_dq<float><<<dim3(cdiv(s, AQ), h, b), 128, s1, c->stream>>>(a);
        k_attn_dkv<float><<<dim3(cdiv(s, AQ), hkv, b), 128, s2, c->stream>>>(a);
    }
    launched(c, 3);
}

// attention / gqa_attention on the fp32 path (k_attn_fwd, 16 queries per
// CTA) and the embedding gather (one CTA per token).
KernelInfo attention_info(Context* c, const std::string& op, int dtype, const KShape& s) {
    KernelInfo k;
    if (op == "attention" || op == "gqa_attention") {
        k.fn = dtype == CATNN_BF16 ? (const void*)k_attn_fwd<bf16> : (const void*)k_attn_fwd<float>;
        k.file = "attention.cu";
        k.grid[0] = (unsigned)cdiv(s.seq, AQ);
        k.grid[1] = (unsigned)s.heads;
        k.grid[2] = (unsigned)s.batch;
        k.block[0] = 128;
        k.dyn_smem = attn_smem_bytes(0, s.head_dim);
    } else if (op == "embedding") {
        k.fn = dtype == CATNN_BF16 ? (const void*)k_embed<bf16> : (const void*)k_embed<float>;
        k.file = "attention.cu";
        k.grid[0] = (unsigned)std::max<i64>(1, s.rows);
        k.block[0] = s.width >= 256 ? 256 : 64;
    }
    return k;
}

}  // namespace catnn
