// bf16 flash attention on the tensor cores (mma.sync m16n8k16, fp32
// accumulation), forward and backward, for head_dim 64 or 128.
//
// Forward: CTA = 64 queries x one (head, batch); 4 warps x 16 query rows.
// K/V tiles of 64 keys stream through shared memory (cp.async double
// buffer, XOR-swizzled 16-byte chunks so ldmatrix is conflict-free); the
// scores stay in registers, the softmax is online (log2 domain), P feeds the
// PV product straight from registers. Writes O and the row log-sum-exp.
// Backward (deterministic, no atomics):
//  - dK/dV: CTA = 64 keys x one kv head; loops over the query heads that
//    share the kv head and over the query blocks that see the keys;
//    recomputes P^T = exp(K Q^T - lse) and accumulates dV += P^T dO,
//    dK += dS^T Q with dS^T = P^T (V dO^T - D).
//  - dQ: CTA = 64 queries; loops over key blocks; dQ += dS K.
// Masks: causal (key <= query), optional sliding window (key > query -
// window), sequence end.
#include "ops.cuh"

namespace catnn {
namespace fa {

constexpr int BM = 64, BN = 64, NT = 128;
constexpr float LOG2E = 1.4426950408889634f;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mma(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm4(uint32_t* r, uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm4t(uint32_t* r, uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
// 16-byte async copy; src_bytes = 0 fills the chunk with zeros.
__device__ __forceinline__ void cp16(uint32_t saddr, const void* g, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(saddr), "l"(g), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

// Byte offset of (row, 16-byte chunk) in a [rows][HD] bf16 tile whose chunks
// are XOR-swizzled by the row's low 3 bits.
template <int HD> __device__ __forceinline__ uint32_t toff(int row, int chunk) {
    return (uint32_t)(row * HD * 2 + ((chunk ^ (row & 7)) << 4));
}

// Copy ROWS rows of HD bf16 (row r at base + (row0 + r) * stride) into a tile;
// rows >= limit read as zeros.
template <int HD, int ROWS>
__device__ __forceinline__ void load_tile(uint32_t sbase, const bf16* base, i64 row0, i64 stride, i64 limit) {
    constexpr int CH = HD / 8;
    for (int i = threadIdx.x; i < ROWS * CH; i += NT) {
        int r = i / CH, c = i % CH;
        i64 gr = row0 + r;
        bool ok = gr < limit && gr >= 0;
        const bf16* src = base + (ok ? gr : 0) * stride + c * 8;
        cp16(sbase + toff<HD>(r, c), src, ok ? 16 : 0);
    }
}

struct Args {
    const bf16 *q, *k, *v, *o, *dout;
    bf16 *out, *dq, *dk, *dv;
    float* lse;
    const float* dsum;
    int b, s, h, hkv, q_stride, kv_stride;
    int causal, window;
    float scale;
};

// Key range of query i (inclusive); the window limits how far back it sees.
__device__ __forceinline__ int klo(const Args& a, int i) {
    if (!a.causal || a.window <= 0) return 0;
    int l = i - a.window + 1;
    return l > 0 ? l : 0;
}
__device__ __forceinline__ int khi(const Args& a, int i) { return a.causal ? i : a.s - 1; }

template <int HD>
__global__ void __launch_bounds__(NT) k_fwd(Args a) {
    constexpr int KS = HD / 16;  // k-steps over head_dim
    constexpr int DT = HD / 8;   // n8 tiles over head_dim
    extern __shared__ __align__(128) uint8_t sm[];
    const uint32_t sQ = smem_u32(sm);
    const uint32_t sK = sQ + BM * HD * 2;
    const uint32_t sV = sK + 2 * BN * HD * 2;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
    const int q0 = blockIdx.x * BM, h = blockIdx.y, bi = blockIdx.z;
    const int kvh = h / (a.h / a.hkv);
    const bf16* Qb = a.q + (i64)bi * a.s * a.q_stride + h * HD;
    const bf16* Kb = a.k + (i64)bi * a.s * a.kv_stride + kvh * HD;
    const bf16* Vb = a.v + (i64)bi * a.s * a.kv_stride + kvh * HD;
    const int qlast = min(q0 + BM - 1, a.s - 1);
    const int kb0 = klo(a, q0) / BN, kb1 = khi(a, qlast) / BN;

    load_tile<HD, BM>(sQ, Qb, q0, a.q_stride, a.s);
    load_tile<HD, BN>(sK, Kb, (i64)kb0 * BN, a.kv_stride, a.s);
    load_tile<HD, BN>(sV, Vb, (i64)kb0 * BN, a.kv_stride, a.s);
    cp_commit();
    cp_wait<0>();
    __syncthreads();

    uint32_t qf[KS][4];
    {
        const int m = lane >> 3, rr = lane & 7;
        for (int ks = 0; ks < KS; ++ks) ldsm4(qf[ks], sQ + toff<HD>(warp * 16 + (m & 1) * 8 + rr, 2 * ks + (m >> 1)));
    }
    float o[DT][4];
    for (int t = 0; t < DT; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
    const float sc = a.scale * LOG2E;
    const int row0 = q0 + warp * 16 + g, row1 = row0 + 8;

    for (int kb = kb0; kb <= kb1; ++kb) {
        const int buf = (kb - kb0) & 1;
        if (kb < kb1) {  // prefetch the next tile into the other buffer
            load_tile<HD, BN>(sK + (buf ^ 1) * BN * HD * 2, Kb, (i64)(kb + 1) * BN, a.kv_stride, a.s);
            load_tile<HD, BN>(sV + (buf ^ 1) * BN * HD * 2, Vb, (i64)(kb + 1) * BN, a.kv_stride, a.s);
        }
        cp_commit();
        const uint32_t cK = sK + buf * BN * HD * 2, cV = sV + buf * BN * HD * 2;
        float s[8][4];
        for (int t = 0; t < 8; ++t) s[t][0] = s[t][1] = s[t][2] = s[t][3] = 0.f;
        {
            const int m = lane >> 3, rr = lane & 7;
            for (int np = 0; np < 4; ++np)
                for (int ks = 0; ks < KS; ++ks) {
                    uint32_t bfr[4];
                    ldsm4(bfr, cK + toff<HD>(np * 16 + (m >> 1) * 8 + rr, 2 * ks + (m & 1)));
                    mma(s[2 * np], qf[ks], bfr[0], bfr[1]);
                    mma(s[2 * np + 1], qf[ks], bfr[2], bfr[3]);
                }
        }
        // scale to log2 units and mask
        const int k0 = kb * BN;
        const int lo0 = klo(a, row0), hi0 = min(khi(a, row0), a.s - 1);
        const int lo1 = klo(a, row1), hi1 = min(khi(a, row1), a.s - 1);
        float mx[2] = {-INFINITY, -INFINITY};
        for (int t = 0; t < 8; ++t)
            for (int j = 0; j < 2; ++j) {
                int key = k0 + t * 8 + tig * 2 + j;
                float v0 = (key >= lo0 && key <= hi0) ? s[t][j] * sc : -INFINITY;
                float v1 = (key >= lo1 && key <= hi1) ? s[t][2 + j] * sc : -INFINITY;
                s[t][j] = v0;
                s[t][2 + j] = v1;
                mx[0] = fmaxf(mx[0], v0);
                mx[1] = fmaxf(mx[1], v1);
            }
        float alpha[2];
        for (int r = 0; r < 2; ++r) {
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
            float mn = fmaxf(mrow[r], mx[r]);
            float base = mn == -INFINITY ? 0.f : mn;
            alpha[r] = exp2f(mrow[r] - base);
            mrow[r] = mn;
            mx[r] = base;
        }
        float ls[2] = {0.f, 0.f};
        for (int t = 0; t < 8; ++t) {
            s[t][0] = exp2f(s[t][0] - mx[0]);
            s[t][1] = exp2f(s[t][1] - mx[0]);
            s[t][2] = exp2f(s[t][2] - mx[1]);
            s[t][3] = exp2f(s[t][3] - mx[1]);
            ls[0] += s[t][0] + s[t][1];
            ls[1] += s[t][2] + s[t][3];
        }
        lrow[0] = lrow[0] * alpha[0] + ls[0];
        lrow[1] = lrow[1] * alpha[1] + ls[1];
        for (int t = 0; t < DT; ++t) {
            o[t][0] *= alpha[0];
            o[t][1] *= alpha[0];
            o[t][2] *= alpha[1];
            o[t][3] *= alpha[1];
        }
        {
            const int m = lane >> 3, rr = lane & 7;
            for (int kk = 0; kk < 4; ++kk) {
                uint32_t pa[4] = {pack(s[2 * kk][0], s[2 * kk][1]), pack(s[2 * kk][2], s[2 * kk][3]),
                                  pack(s[2 * kk + 1][0], s[2 * kk + 1][1]), pack(s[2 * kk + 1][2], s[2 * kk + 1][3])};
                for (int dp = 0; dp < DT / 2; ++dp) {
                    uint32_t bfr[4];
                    ldsm4t(bfr, cV + toff<HD>(kk * 16 + (m & 1) * 8 + rr, 2 * dp + (m >> 1)));
                    mma(o[2 * dp], pa, bfr[0], bfr[1]);
                    mma(o[2 * dp + 1], pa, bfr[2], bfr[3]);
                }
            }
        }
        cp_wait<0>();
        __syncthreads();
    }
    for (int r = 0; r < 2; ++r) {
        lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
        lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
    }
    const int rows[2] = {row0, row1};
    for (int r = 0; r < 2; ++r) {
        if (rows[r] >= a.s) continue;
        float inv = lrow[r] > 0.f ? 1.f / lrow[r] : 0.f;
        bf16* op = a.out + ((i64)bi * a.s + rows[r]) * (a.h * HD) + h * HD;
        for (int t = 0; t < DT; ++t)
            *reinterpret_cast<__nv_bfloat162*>(op + t * 8 + tig * 2) =
                __floats2bfloat162_rn(o[t][2 * r] * inv, o[t][2 * r + 1] * inv);
        if (tig == 0)
            a.lse[((i64)bi * a.h + h) * a.s + rows[r]] =
                lrow[r] > 0.f ? (mrow[r] + log2f(lrow[r])) / LOG2E : -INFINITY;
    }
}

// dK, dV for 64 keys of one kv head. Warp w owns keys j0 + 16w .. +15 and
// works in the transposed frame (rows = keys, columns = queries).
template <int HD>
__global__ void __launch_bounds__(NT) k_bwd_dkdv(Args a) {
    constexpr int KS = HD / 16, DT = HD / 8;
    extern __shared__ __align__(128) uint8_t sm[];
    const uint32_t sKt = smem_u32(sm);           // K tile [64][HD]
    const uint32_t sVt = sKt + BN * HD * 2;      // V tile
    const uint32_t sQ = sVt + BN * HD * 2;       // Q tile [64][HD]
    const uint32_t sG = sQ + BM * HD * 2;        // dO tile
    float* sL = reinterpret_cast<float*>(sm + 2 * BN * HD * 2 + 2 * BM * HD * 2);  // lse * log2e
    float* sD = sL + BM;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
    const int j0 = blockIdx.x * BN, kvh = blockIdx.y, bi = blockIdx.z;
    const int rep = a.h / a.hkv;
    const bf16* Kb = a.k + (i64)bi * a.s * a.kv_stride + kvh * HD;
    const bf16* Vb = a.v + (i64)bi * a.s * a.kv_stride + kvh * HD;
    load_tile<HD, BN>(sKt, Kb, j0, a.kv_stride, a.s);
    load_tile<HD, BN>(sVt, Vb, j0, a.kv_stride, a.s);
    cp_commit();
    cp_wait<0>();
    __syncthreads();
    uint32_t kf[KS][4], vf[KS][4];
    {
        const int m = lane >> 3, rr = lane & 7;
        for (int ks = 0; ks < KS; ++ks) {
            ldsm4(kf[ks], sKt + toff<HD>(warp * 16 + (m & 1) * 8 + rr, 2 * ks + (m >> 1)));
            ldsm4(vf[ks], sVt + toff<HD>(warp * 16 + (m & 1) * 8 + rr, 2 * ks + (m >> 1)));
        }
    }
    float dk[DT][4], dv[DT][4];
    for (int t = 0; t < DT; ++t)
        for (int j = 0; j < 4; ++j) dk[t][j] = dv[t][j] = 0.f;
    const int key0 = j0 + warp * 16 + g, key1 = key0 + 8;
    const int jl = min(j0 + BN - 1, a.s - 1);
    int qb0 = a.causal ? j0 / BM : 0;
    int qb1 = (a.s - 1) / BM;
    if (a.causal && a.window > 0) qb1 = min(qb1, (jl + a.window - 1) / BM);
    const float sc = a.scale * LOG2E;
    for (int hq = kvh * rep; hq < (kvh + 1) * rep; ++hq) {
        const bf16* Qb = a.q + (i64)bi * a.s * a.q_stride + hq * HD;
        const bf16* Gb = a.dout + (i64)bi * a.s * (a.h * HD) + hq * HD;
        const float* Lb = a.lse + ((i64)bi * a.h + hq) * a.s;
        const float* Db = a.dsum + ((i64)bi * a.h + hq) * a.s;
        for (int qb = qb0; qb <= qb1; ++qb) {
            const int i0 = qb * BM;
            __syncthreads();
            load_tile<HD, BM>(sQ, Qb, i0, a.q_stride, a.s);
            load_tile<HD, BM>(sG, Gb, i0, a.h * HD, a.s);
            cp_commit();
            for (int r = threadIdx.x; r < BM; r += NT) {
                int qi = i0 + r;
                sL[r] = qi < a.s ? a.lse[((i64)bi * a.h + hq) * a.s + qi] * LOG2E : 0.f;
                sD[r] = qi < a.s ? Db[qi] : 0.f;
            }
            (void)Lb;
            cp_wait<0>();
            __syncthreads();
            // S^T = K Q^T ; dP^T = V dO^T   (16 keys x 64 queries per warp)
            float st[8][4], dpt[8][4];
            for (int t = 0; t < 8; ++t)
                for (int j = 0; j < 4; ++j) st[t][j] = dpt[t][j] = 0.f;
            {
                const int m = lane >> 3, rr = lane & 7;
                for (int np = 0; np < 4; ++np)
                    for (int ks = 0; ks < KS; ++ks) {
                        uint32_t bq[4], bg[4];
                        ldsm4(bq, sQ + toff<HD>(np * 16 + (m >> 1) * 8 + rr, 2 * ks + (m & 1)));
                        ldsm4(bg, sG + toff<HD>(np * 16 + (m >> 1) * 8 + rr, 2 * ks + (m & 1)));
                        mma(st[2 * np], kf[ks], bq[0], bq[1]);
                        mma(st[2 * np + 1], kf[ks], bq[2], bq[3]);
                        mma(dpt[2 * np], vf[ks], bg[0], bg[1]);
                        mma(dpt[2 * np + 1], vf[ks], bg[2], bg[3]);
                    }
            }
            // P^T and dS^T (columns = queries)
            for (int t = 0; t < 8; ++t)
                for (int j = 0; j < 2; ++j) {
                    int qc = t * 8 + tig * 2 + j;
                    int qi = i0 + qc;
                    bool in0 = qi < a.s && key0 < a.s && key0 >= klo(a, qi) && key0 <= khi(a, qi);
                    bool in1 = qi < a.s && key1 < a.s && key1 >= klo(a, qi) && key1 <= khi(a, qi);
                    float p0 = in0 ? exp2f(st[t][j] * sc - sL[qc]) : 0.f;
                    float p1 = in1 ? exp2f(st[t][2 + j] * sc - sL[qc]) : 0.f;
                    st[t][j] = p0;
                    st[t][2 + j] = p1;
                    dpt[t][j] = p0 * (dpt[t][j] - sD[qc]);
                    dpt[t][2 + j] = p1 * (dpt[t][2 + j] - sD[qc]);
                }
            // dV += P^T dO ; dK += dS^T Q    (k = queries)
            {
                const int m = lane >> 3, rr = lane & 7;
                for (int kk = 0; kk < 4; ++kk) {
                    uint32_t pa[4] = {pack(st[2 * kk][0], st[2 * kk][1]), pack(st[2 * kk][2], st[2 * kk][3]),
                                      pack(st[2 * kk + 1][0], st[2 * kk + 1][1]),
                                      pack(st[2 * kk + 1][2], st[2 * kk + 1][3])};
                    uint32_t da[4] = {pack(dpt[2 * kk][0], dpt[2 * kk][1]), pack(dpt[2 * kk][2], dpt[2 * kk][3]),
                                      pack(dpt[2 * kk + 1][0], dpt[2 * kk + 1][1]),
                                      pack(dpt[2 * kk + 1][2], dpt[2 * kk + 1][3])};
                    for (int dp = 0; dp < DT / 2; ++dp) {
                        uint32_t bg[4], bq[4];
                        ldsm4t(bg, sG + toff<HD>(kk * 16 + (m & 1) * 8 + rr, 2 * dp + (m >> 1)));
                        ldsm4t(bq, sQ + toff<HD>(kk * 16 + (m & 1) * 8 + rr, 2 * dp + (m >> 1)));
                        mma(dv[2 * dp], pa, bg[0], bg[1]);
                        mma(dv[2 * dp + 1], pa, bg[2], bg[3]);
                        mma(dk[2 * dp], da, bq[0], bq[1]);
                        mma(dk[2 * dp + 1], da, bq[2], bq[3]);
                    }
                }
            }
        }
    }
    const int keys[2] = {key0, key1};
    for (int r = 0; r < 2; ++r) {
        if (keys[r] >= a.s) continue;
        i64 off = ((i64)bi * a.s + keys[r]) * a.kv_stride + kvh * HD;
        for (int t = 0; t < DT; ++t) {
            *reinterpret_cast<__nv_bfloat162*>(a.dk + off + t * 8 + tig * 2) =
                __floats2bfloat162_rn(dk[t][2 * r] * a.scale, dk[t][2 * r + 1] * a.scale);
            *reinterpret_cast<__nv_bfloat162*>(a.dv + off + t * 8 + tig * 2) =
                __floats2bfloat162_rn(dv[t][2 * r], dv[t][2 * r + 1]);
        }
    }
}

// dQ for 64 queries of one head: dQ = scale * Σ_j dS_ij K_j.
template <int HD>
__global__ void __launch_bounds__(NT) k_bwd_dq(Args a) {
    constexpr int KS = HD / 16, DT = HD / 8;
    extern __shared__ __align__(128) uint8_t sm[];
    const uint32_t sQ = smem_u32(sm);
    const uint32_t sG = sQ + BM * HD * 2;
    const uint32_t sK = sG + BM * HD * 2;  // 2 buffers
    const uint32_t sV = sK + 2 * BN * HD * 2;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
    const int q0 = blockIdx.x * BM, h = blockIdx.y, bi = blockIdx.z;
    const int kvh = h / (a.h / a.hkv);
    const bf16* Qb = a.q + (i64)bi * a.s * a.q_stride + h * HD;
    const bf16* Gb = a.dout + (i64)bi * a.s * (a.h * HD) + h * HD;
    const bf16* Kb = a.k + (i64)bi * a.s * a.kv_stride + kvh * HD;
    const bf16* Vb = a.v + (i64)bi * a.s * a.kv_stride + kvh * HD;
    const int qlast = min(q0 + BM - 1, a.s - 1);
    const int kb0 = klo(a, q0) / BN, kb1 = khi(a, qlast) / BN;
    load_tile<HD, BM>(sQ, Qb, q0, a.q_stride, a.s);
    load_tile<HD, BM>(sG, Gb, q0, a.h * HD, a.s);
    load_tile<HD, BN>(sK, Kb, (i64)kb0 * BN, a.kv_stride, a.s);
    load_tile<HD, BN>(sV, Vb, (i64)kb0 * BN, a.kv_stride, a.s);
    cp_commit();
    cp_wait<0>();
    __syncthreads();
    uint32_t qf[KS][4], gf[KS][4];
    {
        const int m = lane >> 3, rr = lane & 7;
        for (int ks = 0; ks < KS; ++ks) {
            ldsm4(qf[ks], sQ + toff<HD>(warp * 16 + (m & 1) * 8 + rr, 2 * ks + (m >> 1)));
            ldsm4(gf[ks], sG + toff<HD>(warp * 16 + (m & 1) * 8 + rr, 2 * ks + (m >> 1)));
        }
    }
    const int row0 = q0 + warp * 16 + g, row1 = row0 + 8;
    const float sc = a.scale * LOG2E;
    float L[2], D[2];
    L[0] = row0 < a.s ? a.lse[((i64)bi * a.h + h) * a.s + row0] * LOG2E : 0.f;
    L[1] = row1 < a.s ? a.lse[((i64)bi * a.h + h) * a.s + row1] * LOG2E : 0.f;
    D[0] = row0 < a.s ? a.dsum[((i64)bi * a.h + h) * a.s + row0] : 0.f;
    D[1] = row1 < a.s ? a.dsum[((i64)bi * a.h + h) * a.s + row1] : 0.f;
    float dq[DT][4];
    for (int t = 0; t < DT; ++t) dq[t][0] = dq[t][1] = dq[t][2] = dq[t][3] = 0.f;
    const int lo0 = klo(a, row0), hi0 = min(khi(a, row0), a.s - 1);
    const int lo1 = klo(a, row1), hi1 = min(khi(a, row1), a.s - 1);
    for (int kb = kb0; kb <= kb1; ++kb) {
        const int buf = (kb - kb0) & 1;
        if (kb < kb1) {
            load_tile<HD, BN>(sK + (buf ^ 1) * BN * HD * 2, Kb, (i64)(kb + 1) * BN, a.kv_stride, a.s);
            load_tile<HD, BN>(sV + (buf ^ 1) * BN * HD * 2, Vb, (i64)(kb + 1) * BN, a.kv_stride, a.s);
        }
        cp_commit();
        const uint32_t cK = sK + buf * BN * HD * 2, cV = sV + buf * BN * HD * 2;
        float s[8][4], dp[8][4];
        for (int t = 0; t < 8; ++t)
            for (int j = 0; j < 4; ++j) s[t][j] = dp[t][j] = 0.f;
        {
            const int m = lane >> 3, rr = lane & 7;
            for (int np = 0; np < 4; ++np)
                for (int ks = 0; ks < KS; ++ks) {
                    uint32_t bk[4], bv[4];
                    ldsm4(bk, cK + toff<HD>(np * 16 + (m >> 1) * 8 + rr, 2 * ks + (m & 1)));
                    ldsm4(bv, cV + toff<HD>(np * 16 + (m >> 1) * 8 + rr, 2 * ks + (m & 1)));
                    mma(s[2 * np], qf[ks], bk[0], bk[1]);
                    mma(s[2 * np + 1], qf[ks], bk[2], bk[3]);
                    mma(dp[2 * np], gf[ks], bv[0], bv[1]);
                    mma(dp[2 * np + 1], gf[ks], bv[2], bv[3]);
                }
        }
        const int k0 = kb * BN;
        for (int t = 0; t < 8; ++t)
            for (int j = 0; j < 2; ++j) {
                int key = k0 + t * 8 + tig * 2 + j;
                float p0 = (key >= lo0 && key <= hi0) ? exp2f(s[t][j] * sc - L[0]) : 0.f;
                float p1 = (key >= lo1 && key <= hi1) ? exp2f(s[t][2 + j] * sc - L[1]) : 0.f;
                s[t][j] = p0 * (dp[t][j] - D[0]);
                s[t][2 + j] = p1 * (dp[t][2 + j] - D[1]);
            }
        {
            const int m = lane >> 3, rr = lane & 7;
            for (int kk = 0; kk < 4; ++kk) {
                uint32_t da[4] = {pack(s[2 * kk][0], s[2 * kk][1]), pack(s[2 * kk][2], s[2 * kk][3]),
                                  pack(s[2 * kk + 1][0], s[2 * kk + 1][1]), pack(s[2 * kk + 1][2], s[2 * kk + 1][3])};
                for (int d2 = 0; d2 < DT / 2; ++d2) {
                    uint32_t bk[4];
                    ldsm4t(bk, cK + toff<HD>(kk * 16 + (m & 1) * 8 + rr, 2 * d2 + (m >> 1)));
                    mma(dq[2 * d2], da, bk[0], bk[1]);
                    mma(dq[2 * d2 + 1], da, bk[2], bk[3]);
                }
            }
        }
        cp_wait<0>();
        __syncthreads();
    }
    const int rows[2] = {row0, row1};
    for (int r = 0; r < 2; ++r) {
        if (rows[r] >= a.s) continue;
        bf16* p = a.dq + ((i64)bi * a.s + rows[r]) * a.q_stride + h * HD;
        for (int t = 0; t < DT; ++t)
            *reinterpret_cast<__nv_bfloat162*>(p + t * 8 + tig * 2) =
                __floats2bfloat162_rn(dq[t][2 * r] * a.scale, dq[t][2 * r + 1] * a.scale);
    }
}

template <typename K> static void set_smem(K k, size_t bytes) {
    CUDA_OK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
}

}  // namespace fa

// Tensor-core path applies to bf16 with head_dim 64 or 128 and 16-byte
// aligned rows; anything else goes to the CUDA-core kernels.
bool attention_tc_ok(i64 hd, i64 q_stride, i64 kv_stride, const void* q, const void* k, const void* v) {
    auto al = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
    return (hd == 64 || hd == 128) && q_stride % 8 == 0 && kv_stride % 8 == 0 && al(q) && al(k) && al(v);
}

static fa::Args fa_args(const void* q, const void* k, const void* v, i64 b, i64 s, i64 h, i64 hkv, i64 hd, bool causal,
                        i64 window, i64 q_stride, i64 kv_stride) {
    fa::Args a{};
    a.q = (const bf16*)q;
    a.k = (const bf16*)k;
    a.v = (const bf16*)v;
    a.b = (int)b;
    a.s = (int)s;
    a.h = (int)h;
    a.hkv = (int)hkv;
    a.q_stride = (int)q_stride;
    a.kv_stride = (int)kv_stride;
    a.causal = causal ? 1 : 0;
    a.window = (int)window;
    a.scale = 1.0f / sqrtf((float)hd);
    return a;
}

void attention_fwd_tc(Context* c, const void* q, const void* k, const void* v, void* o, float* lse, i64 b, i64 s, i64 h,
                      i64 hkv, i64 hd, bool causal, i64 window, i64 q_stride, i64 kv_stride) {
    fa::Args a = fa_args(q, k, v, b, s, h, hkv, hd, causal, window, q_stride, kv_stride);
    a.out = (bf16*)o;
    a.lse = lse;
    dim3 grid(cdiv(s, fa::BM), h, b);
    if (hd == 64) {
        size_t sm = (size_t)(fa::BM + 4 * fa::BN) * 64 * 2;
        fa::set_smem(fa::k_fwd<64>, sm);
        fa::k_fwd<64><<<grid, fa::NT, sm, c->stream>>>(a);
    } else {
        size_t sm = (size_t)(fa::BM + 4 * fa::BN) * 128 * 2;
        fa::set_smem(fa::k_fwd<128>, sm);
        fa::k_fwd<128><<<grid, fa::NT, sm, c->stream>>>(a);
    }
    launched(c);
}

template <typename T>
__global__ void k_attn_dsum_tc(const T* __restrict__ o, const T* __restrict__ dout, float* __restrict__ dsum, i64 b,
                               i64 s, i64 h, i64 hd) {
    i64 row = blockIdx.x * 4 + (threadIdx.x >> 5);
    int lane = threadIdx.x & 31;
    if (row >= b * s * h) return;
    i64 hh = row % h, tok = row / h;
    float acc = 0.f;
    for (i64 d = lane; d < hd; d += 32) acc += ld(o + tok * h * hd + hh * hd + d) * ld(dout + tok * h * hd + hh * hd + d);
    acc = warp_sum(acc);
    if (lane == 0) dsum[((tok / s) * h + hh) * s + tok % s] = acc;
}

void attention_bwd_tc5(Context* c, const void* q, const void* k, const void* v, const void* dout, const float* lse,
                       const float* dsum, void* dq, void* dk, void* dv, i64 b, i64 s, i64 h, i64 hkv, bool causal,
                       i64 window, i64 q_stride, i64 kv_stride);

// D = rowsum(O ⊙ dO) for head_dim 64: 8 threads per (token, head) row, one
// 16-byte load of each operand per thread, a 3-step shuffle sum.
__global__ void k_attn_dsum64(const bf16* __restrict__ o, const bf16* __restrict__ dout, float* __restrict__ dsum,
                              i64 rows, i64 s, i64 h) {
    const i64 row = (blockIdx.x * (i64)blockDim.x + threadIdx.x) >> 3;
    const int part = threadIdx.x & 7;
    float acc = 0.f;
    if (row < rows) {
        float x[8], y[8];
        ldv<bf16, 8>(o + row * 64 + part * 8, x);
        ldv<bf16, 8>(dout + row * 64 + part * 8, y);
#pragma unroll
        for (int t = 0; t < 8; ++t) acc = fmaf(x[t], y[t], acc);
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    acc += __shfl_xor_sync(0xffffffffu, acc, 4);
    if (row < rows && part == 0) {
        const i64 hh = row % h, tok = row / h;
        dsum[((tok / s) * h + hh) * s + tok % s] = acc;
    }
}

void attention_bwd_tc(Context* c, const void* q, const void* k, const void* v, const void* o, const float* lse,
                      const void* dout, void* dq, void* dk, void* dv, i64 b, i64 s, i64 h, i64 hkv, i64 hd, bool causal,
                      i64 window, i64 q_stride, i64 kv_stride) {
    float* dsum = (float*)c->scratch_for((size_t)b * h * s * 4);
    auto al = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
    if (hd == 64 && al(o) && al(dout))
        k_attn_dsum64<<<cdiv(b * s * h * 8, 256), 256, 0, c->stream>>>((const bf16*)o, (const bf16*)dout, dsum, b * s * h, s,
                                                                       h);
    else
        k_attn_dsum_tc<<<cdiv(b * s * h, 4), 128, 0, c->stream>>>((const bf16*)o, (const bf16*)dout, dsum, b, s, h, hd);
    if (hd == 64 && al(dout) && al(dq) && al(dk) && al(dv)) {
        // tcgen05 + TMEM kernels (q, k, v alignment and pitches were checked by attention_tc_ok)
        attention_bwd_tc5(c, q, k, v, dout, lse, dsum, dq, dk, dv, b, s, h, hkv, causal, window, q_stride, kv_stride);
        launched(c);
        return;
    }
    fa::Args a = fa_args(q, k, v, b, s, h, hkv, hd, causal, window, q_stride, kv_stride);
    a.o = (const bf16*)o;
    a.dout = (const bf16*)dout;
    a.dq = (bf16*)dq;
    a.dk = (bf16*)dk;
    a.dv = (bf16*)dv;
    a.lse = const_cast<float*>(lse);
    a.dsum = dsum;
    dim3 gkv(cdiv(s, fa::BN), hkv, b), gq(cdiv(s, fa::BM), h, b);
    if (hd == 64) {
        size_t s1 = (size_t)(2 * fa::BN + 2 * fa::BM) * 64 * 2 + 2 * fa::BM * 4;
        size_t s2 = (size_t)(2 * fa::BM + 4 * fa::BN) * 64 * 2;
        fa::set_smem(fa::k_bwd_dkdv<64>, s1);
        fa::set_smem(fa::k_bwd_dq<64>, s2);
        fa::k_bwd_dkdv<64><<<gkv, fa::NT, s1, c->stream>>>(a);
        fa::k_bwd_dq<64><<<gq, fa::NT, s2, c->stream>>>(a);
    } else {
        size_t s1 = (size_t)(2 * fa::BN + 2 * fa::BM) * 128 * 2 + 2 * fa::BM * 4;
        size_t s2 = (size_t)(2 * fa::BM + 4 * fa::BN) * 128 * 2;
        fa::set_smem(fa::k_bwd_dkdv<128>, s1);
        fa::set_smem(fa::k_bwd_dq<128>, s2);
        fa::k_bwd_dkdv<128><<<gkv, fa::NT, s1, c->stream>>>(a);
        fa::k_bwd_dq<128><<<gq, fa::NT, s2, c->stream>>>(a);
    }
    launched(c, 3);
}

}  // namespace catnn
