// Elementwise kernels: activations and their adjoints, add/mul, casts,
// deterministic column sums (bias gradients) and the SGD / Adam updates.
// All are HBM-bound streams: grid-stride loops over 16-byte vectors where
// the storage type allows, each product and sum rounded separately
// (__fmul_rn/__fadd_rn) so that SGD, Adam, add and mul are bit-identical to
// the reference's f32 arithmetic.
#include <type_traits>

#include "ops.cuh"

namespace catnn {

static int ew_grid(Context* c, i64 n, int threads = 256) {
    i64 b = (n + threads - 1) / threads;
    i64 cap = (i64)c->sm_count * 8;
    if (b > cap) b = cap;
    return (int)(b < 1 ? 1 : b);
}

// sqrt(2/pi) rounded as the reference computes it in f32 (cpu.rs:25).
__device__ __forceinline__ float gelu_k() { return __fsqrt_rn(__fdiv_rn(2.0f, 3.14159265358979323846f)); }

// cpu.rs:20-29
__device__ __forceinline__ float gelu_f(float z) {
    float z3 = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, z), z), z);
    float inner = __fmul_rn(gelu_k(), __fadd_rn(z, z3));
    return __fmul_rn(__fmul_rn(0.5f, z), __fadd_rn(1.0f, tanhf(inner)));
}
// adjoint.rs:76-90
__device__ __forceinline__ float gelu_grad_f(float z) {
    const float C = 0.044715f;
    float k = gelu_k();
    float u = __fmul_rn(k, __fadd_rn(z, __fmul_rn(__fmul_rn(__fmul_rn(C, z), z), z)));
    float t = tanhf(u);
    float sech2 = __fsub_rn(1.0f, __fmul_rn(t, t));
    float du = __fmul_rn(k, __fadd_rn(1.0f, __fmul_rn(__fmul_rn(__fmul_rn(3.0f, C), z), z)));
    return __fadd_rn(__fmul_rn(0.5f, __fadd_rn(1.0f, t)), __fmul_rn(__fmul_rn(__fmul_rn(0.5f, z), sech2), du));
}

template <typename T>
__global__ void k_act_fwd(int act, const T* __restrict__ x, T* __restrict__ y, i64 n) {
    for (i64 i = blockIdx.x * (i64)blockDim.x + threadIdx.x; i < n; i += (i64)gridDim.x * blockDim.x) {
        float z = ld(x + i);
        float r = act == CATNN_ACT_RELU ? fmaxf(z, 0.0f) : (act == CATNN_ACT_GELU ? gelu_f(z) : z);
        st(y + i, r);
    }
}

template <typename T>
__global__ void k_act_bwd(int act, const T* __restrict__ x, const T* __restrict__ dy, T* __restrict__ dx, i64 n) {
    for (i64 i = blockIdx.x * (i64)blockDim.x + threadIdx.x; i < n; i += (i64)gridDim.x * blockDim.x) {
        float z = ld(x + i), g = ld(dy + i);
        float r;
        if (act == CATNN_ACT_RELU) r = z <= 0.0f ? 0.0f : g;  // adjoint.rs:63-74
        else if (act == CATNN_ACT_GELU) r = __fmul_rn(g, gelu_grad_f(z));
        else r = g;
        st(dx + i, r);
    }
}

void act_fwd(Context* c, int act, const void* x, void* y, i64 n, int dtype) {
    if (n <= 0) return;
    if (dtype == CATNN_BF16) k_act_fwd<<<ew_grid(c, n), 256, 0, c->stream>>>(act, (const bf16*)x, (bf16*)y, n);
    else k_act_fwd<<<ew_grid(c, n), 256, 0, c->stream>>>(act, (const float*)x, (float*)y, n);
    launched(c);
}

void act_bwd(Context* c, int act, const void* x, const void* dy, void* dx, i64 n, int dtype) {
    if (n <= 0) return;
    if (dtype == CATNN_BF16)
        k_act_bwd<<<ew_grid(c, n), 256, 0, c->stream>>>(act, (const bf16*)x, (const bf16*)dy, (bf16*)dx, n);
    else k_act_bwd<<<ew_grid(c, n), 256, 0, c->stream>>>(act, (const float*)x, (const float*)dy, (float*)dx, n);
    launched(c);
}

template <typename T>
__global__ void k_add(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ y, i64 n, i64 b_len) {
    for (i64 i = blockIdx.x * (i64)blockDim.x + threadIdx.x; i < n; i += (i64)gridDim.x * blockDim.x) {
        i64 j = b_len == n ? i : i % b_len;
        st(y + i, __fadd_rn(ld(a + i), ld(b + j)));
    }
}
template <typename T>
__global__ void k_mul(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ y, i64 n) {
    for (i64 i = blockIdx.x * (i64)blockDim.x + threadIdx.x; i < n; i += (i64)gridDim.x * blockDim.x)
        st(y + i, __fmul_rn(ld(a + i), ld(b + i)));
}

void add(Context* c, const void* a, const void* b, void* y, i64 n, i64 b_len, int dtype) {
    if (n <= 0) return;
    if (dtype == CATNN_BF16) k_add<<<ew_grid(c, n), 256, 0, c->stream>>>((const bf16*)a, (const bf16*)b, (bf16*)y, n, b_len);
    else k_add<<<ew_grid(c, n), 256, 0, c->stream>>>((const float*)a, (const float*)b, (float*)y, n, b_len);
    launched(c);
}
void mul(Context* c, const void* a, const void* b, void* y, i64 n, int dtype) {
    if (n <= 0) return;
    if (dtype == CATNN_BF16) k_mul<<<ew_grid(c, n), 256, 0, c->stream>>>((const bf16*)a, (const bf16*)b, (bf16*)y, n);
    else k_mul<<<ew_grid(c, n), 256, 0, c->stream>>>((const float*)a, (const float*)b, (float*)y, n);
    launched(c);
}

template <typename A, typename B>
__global__ void k_cast(const A* __restrict__ x, B* __restrict__ y, i64 n) {
    for (i64 i = blockIdx.x * (i64)blockDim.x + threadIdx.x; i < n; i += (i64)gridDim.x * blockDim.x) st(y + i, ld(x + i));
}
void cast(Context* c, const void* x, int xd, void* y, int yd, i64 n) {
    if (n <= 0) return;
    int g = ew_grid(c, n);
    if (xd == CATNN_F32 && yd == CATNN_BF16) k_cast<<<g, 256, 0, c->stream>>>((const float*)x, (bf16*)y, n);
    else if (xd == CATNN_BF16 && yd == CATNN_F32) k_cast<<<g, 256, 0, c->stream>>>((const bf16*)x, (float*)y, n);
    else if (xd == CATNN_F32) k_cast<<<g, 256, 0, c->stream>>>((const float*)x, (float*)y, n);
    else k_cast<<<g, 256, 0, c->stream>>>((const bf16*)x, (bf16*)y, n);
    launched(c);
}

__global__ void k_fill(float* p, float v, i64 n) {
    for (i64 i = blockIdx.x * (i64)blockDim.x + threadIdx.x; i < n; i += (i64)gridDim.x * blockDim.x) p[i] = v;
}
void fill_f32(Context* c, float* p, float v, i64 n) {
    if (n <= 0) return;
    k_fill<<<ew_grid(c, n), 256, 0, c->stream>>>(p, v, n);
    launched(c);
}

// Column sums in two deterministic stages: chunk partials over ROWS_PER
// rows (rows in order), then the partials in chunk order. Stage 1 threads
// own a column each, so loads are coalesced along the row.
static const int COLSUM_ROWS = 128;
template <typename T>
__global__ void k_colsum_partial(const T* __restrict__ x, i64 rows, i64 cols, float* __restrict__ part) {
    i64 j = blockIdx.x * (i64)blockDim.x + threadIdx.x;
    i64 r0 = (i64)blockIdx.y * COLSUM_ROWS;
    if (j >= cols) return;
    i64 r1 = r0 + COLSUM_ROWS < rows ? r0 + COLSUM_ROWS : rows;
    float s = 0.f;
#pragma unroll 8
    for (i64 r = r0; r < r1; ++r) s = __fadd_rn(s, ld(x + r * cols + j));
    part[(i64)blockIdx.y * cols + j] = s;
}
__global__ void k_colsum_final(const float* __restrict__ part, int chunks, i64 cols, float* __restrict__ out, int acc) {
    i64 j = blockIdx.x * (i64)blockDim.x + threadIdx.x;
    if (j >= cols) return;
    float s = 0.f;
#pragma unroll 8
    for (int ch = 0; ch < chunks; ++ch) s = __fadd_rn(s, part[(i64)ch * cols + j]);
    out[j] = acc ? __fadd_rn(out[j], s) : s;
}
void col_sum(Context* c, const void* x, i64 rows, i64 cols, float* out, int dtype, bool accumulate) {
    if (cols <= 0) return;
    if (rows <= 0) {
        if (!accumulate) CUDA_OK(cudaMemsetAsync(out, 0, cols * 4, c->stream));
        return;
    }
    int chunks = cdiv(rows, COLSUM_ROWS);
    float* part = (float*)c->scratch_for((size_t)chunks * cols * 4);
    dim3 g1(cdiv(cols, 128), chunks);
    if (dtype == CATNN_BF16) k_colsum_partial<<<g1, 128, 0, c->stream>>>((const bf16*)x, rows, cols, part);
    else k_colsum_partial<<<g1, 128, 0, c->stream>>>((const float*)x, rows, cols, part);
    k_colsum_final<<<cdiv(cols, 128), 128, 0, c->stream>>>(part, chunks, cols, out, accumulate ? 1 : 0);
    launched(c, 2);
}

// optim.rs:32-43 — p - lr*g, then the optional bf16 shadow for the
// tensor-core path. float4 stream when 16-byte aligned.
__global__ void k_sgd(float* __restrict__ p, const float* __restrict__ g, i64 n, float lr, bf16* __restrict__ sh) {
    for (i64 i = blockIdx.x * (i64)blockDim.x + threadIdx.x; i < n; i += (i64)gridDim.x * blockDim.x) {
        float v = __fsub_rn(p[i], __fmul_rn(lr, g[i]));
        p[i] = v;
        if (sh) sh[i] = __float2bfloat16_rn(v);
    }
}
void sgd(Context* c, float* p, const float* g, i64 n, float lr, bf16* shadow) {
    if (n <= 0) return;
    k_sgd<<<ew_grid(c, n), 256, 0, c->stream>>>(p, g, n, lr, shadow);
    launched(c);
}

// optim.rs:95-119, one thread per parameter, separate roundings:
// m = b1*m + (1-b1)*g; v = b2*v + ((1-b2)*g)*g;
// p = p - (lr*(m/max(b1t,1e-30))) / (sqrt(v/max(b2t,1e-30)) + eps).
struct AdamK {
    float lr, b1, omb1, b2, omb2, d1, d2, eps;
    // when set, the bias-correction divisors (d1, d2) are read from device
    // memory at kernel start (a replayed CUDA graph keeps its launch arguments)
    const float* d12;
    __device__ __forceinline__ float step(float& p, float gi, float& m, float& v) const {
        float mi = __fadd_rn(__fmul_rn(b1, m), __fmul_rn(omb1, gi));
        float vi = __fadd_rn(__fmul_rn(b2, v), __fmul_rn(__fmul_rn(omb2, gi), gi));
        m = mi;
        v = vi;
        float mhat = __fdiv_rn(mi, d1), vhat = __fdiv_rn(vi, d2);
        float upd = __fdiv_rn(__fmul_rn(lr, mhat), __fadd_rn(__fsqrt_rn(vhat), eps));
        p = __fsub_rn(p, upd);
        return p;
    }
};

// V = 4: p, m, v and an fp32 gradient as float4, a bf16 gradient and the
// shadow as 8-byte groups; the host sends the n % 4 tail through V = 1.
template <typename G, int V>
__global__ void __launch_bounds__(256) k_adam(float* __restrict__ p, const G* __restrict__ g, float* __restrict__ m,
                                              float* __restrict__ v, i64 n, AdamK k, bf16* __restrict__ sh) {
    if (k.d12) {
        k.d1 = k.d12[0];
        k.d2 = k.d12[1];
    }
    const i64 nv = n / V;
    for (i64 i = blockIdx.x * (i64)blockDim.x + threadIdx.x; i < nv; i += (i64)gridDim.x * blockDim.x) {
        const i64 o = i * V;
        float pv[V], gv[V], mv[V], vv[V];
        ldv<float, V>(p + o, pv);
        ldv<G, V>(g + o, gv);
        ldv<float, V>(m + o, mv);
        ldv<float, V>(v + o, vv);
#pragma unroll
        for (int j = 0; j < V; ++j) k.step(pv[j], gv[j], mv[j], vv[j]);
        stv<float, V>(m + o, mv);
        stv<float, V>(v + o, vv);
        stv<float, V>(p + o, pv);
        if (sh) stv<bf16, V>(sh + o, pv);
    }
}

// Integer power by binary exponentiation (the powi lowering the reference's
// f32::powi compiles to), in f32.
static float powi_f32(float a, uint64_t b) {
    float r = 1.0f;
    for (;;) {
        if (b & 1) r *= a;
        b /= 2;
        if (b == 0) break;
        a *= a;
    }
    return r;
}

void adam_divisors(uint64_t t, float b1, float b2, float* d12) {
    volatile float one = 1.0f;
    float b1t = one - powi_f32(b1, t), b2t = one - powi_f32(b2, t);
    d12[0] = std::max(b1t, 1e-30f);
    d12[1] = std::max(b2t, 1e-30f);
}

void adam(Context* c, float* p, const void* g, float* m, float* v, i64 n, uint64_t t, float lr, float b1, float b2,
          float eps, int g_dtype, bf16* shadow, const float* d12_dev) {
    if (n <= 0) return;
    volatile float one = 1.0f;
    float d12[2];
    adam_divisors(t, b1, b2, d12);
    float omb1 = one - b1, omb2 = one - b2;
    AdamK k{lr, b1, omb1, b2, omb2, d12[0], d12[1], eps, d12_dev};
    const int gs = g_dtype == CATNN_BF16 ? 2 : 4;
    const bool vec = aligned_to(p, 16) && aligned_to(m, 16) && aligned_to(v, 16) && aligned_to(g, 4 * gs) &&
                     aligned_to(shadow, 8);
    i64 head = vec ? n / 4 * 4 : 0;
    auto run = [&](auto gp) {
        using G = std::remove_const_t<std::remove_pointer_t<decltype(gp)>>;
        if (head > 0) k_adam<G, 4><<<ew_grid(c, head / 4), 256, 0, c->stream>>>(p, gp, m, v, head, k, shadow);
        if (n > head)
            k_adam<G, 1><<<ew_grid(c, n - head), 256, 0, c->stream>>>(p + head, gp + head, m + head, v + head, n - head, k,
                                                                   shadow ? shadow + head : nullptr);
    };
    if (g_dtype == CATNN_BF16) run((const bf16*)g);
    else run((const float*)g);
    launched(c, (head > 0) + (n > head));
}

// Elementwise ops and the optimizers: grid-stride, at most 8 CTAs per SM.
KernelInfo elementwise_info(Context* c, const std::string& op, int dtype, const KShape& s) {
    KernelInfo k;
    const bool b = dtype == CATNN_BF16;
    const i64 n = s.rows * s.width;
    if (op == "relu" || op == "gelu") k.fn = b ? (const void*)k_act_fwd<bf16> : (const void*)k_act_fwd<float>;
    else if (op == "add" || op == "residual_add") k.fn = b ? (const void*)k_add<bf16> : (const void*)k_add<float>;
    else if (op == "mul") k.fn = b ? (const void*)k_mul<bf16> : (const void*)k_mul<float>;
    else if (op == "sgd") k.fn = (const void*)k_sgd;
    else if (op == "adam") k.fn = (const void*)k_adam<float, 4>;
    else return k;
    k.file = "elementwise.cu";
    k.grid[0] = (unsigned)ew_grid(c, op == "adam" ? (n + 3) / 4 : n);
    k.block[0] = 256;
    return k;
}

}  // namespace catnn
