// fp32 parity-path GEMM (FFMA on the CUDA cores) and the dtype dispatcher.
//
// The fp32 path exists to reproduce the reference's f32 results within
// rtol 1e-5 (its linear is plain f32 multiply-add, cpu.rs:186-232); the
// bf16 tensor-core kernels in gemm_tc.cu carry the throughput.
// 128x128 CTA tile, BK=8, 256 threads, 8x8 outputs per thread, all four
// operand layouts (A [M,K] or [K,M]; B [K,N] or [N,K]) and ragged edges.
// Grouped launches (blockIdx.z = group) serve the MoE expert GEMMs.
#include "ops.cuh"

namespace catnn {

struct SgemmArgs {
    i64 M, N, K;
    const void* A;
    i64 lda;
    const void* B;
    i64 ldb;
    void* C;
    i64 ldc;
    int c_bf16;
    const float* bias;
    int act;
    int accumulate;
    const float* resid;  // fp32 [M, ldc] added before the activation
    // grouping (offsets == nullptr: single GEMM)
    const int32_t* offsets;
    int group_mode;  // 0: rows of A/C split by group, B_g = B + g*strideB; 1: K split (wgrad), C_g = C + g*strideC
    i64 strideB, strideC;
};

__device__ __forceinline__ float gelu_dev(float z) {
    const float k = 0.7978845608028654f;
    float inner = k * (z + 0.044715f * z * z * z);
    return 0.5f * z * (1.0f + tanhf(inner));
}

template <typename T, bool TA, bool TB>
__global__ void __launch_bounds__(256) k_sgemm(SgemmArgs a) {
    __shared__ float As[8][128 + 4];
    __shared__ float Bs[8][128 + 4];
    i64 M = a.M, N = a.N, K = a.K;
    const T* A = (const T*)a.A;
    const T* B = (const T*)a.B;
    char* Cb = (char*)a.C;
    if (a.offsets) {
        int g = blockIdx.z;
        i64 o0 = a.offsets[g], o1 = a.offsets[g + 1];
        if (a.group_mode == 0) {
            M = o1 - o0;
            A += o0 * a.lda;
            Cb += o0 * a.ldc * (a.c_bf16 ? 2 : 4);
            B += g * a.strideB;
        } else {
            K = o1 - o0;
            A += o0 * a.lda;
            B += o0 * a.ldb;
            Cb += g * a.strideC * (a.c_bf16 ? 2 : 4);
        }
    }
    i64 m0 = (i64)blockIdx.y * 128, n0 = (i64)blockIdx.x * 128;
    if (m0 >= M || n0 >= N) return;
    int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
    for (i64 k0 = 0; k0 < K; k0 += 8) {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            int l = tid + 256 * r;
            int mm, kk;
            if (TA) { kk = l >> 7; mm = l & 127; } else { mm = l >> 3; kk = l & 7; }
            i64 gm = m0 + mm, gk = k0 + kk;
            float v = 0.f;
            if (gm < M && gk < K) v = TA ? ld(A + gk * a.lda + gm) : ld(A + gm * a.lda + gk);
            As[kk][mm] = v;
            int nn;
            if (TB) { nn = l >> 3; kk = l & 7; } else { kk = l >> 7; nn = l & 127; }
            i64 gn = n0 + nn;
            gk = k0 + kk;
            float w = 0.f;
            if (gn < N && gk < K) w = TB ? ld(B + gn * a.ldb + gk) : ld(B + gk * a.ldb + gn);
            Bs[kk][nn] = w;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            float ra[8], rb[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) ra[i] = As[kk][ty * 8 + i];
#pragma unroll
            for (int j = 0; j < 8; ++j) rb[j] = Bs[kk][tx * 8 + j];
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(ra[i], rb[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        i64 gm = m0 + ty * 8 + i;
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            i64 gn = n0 + tx * 8 + j;
            if (gn >= N) continue;
            float v = acc[i][j];
            if (a.bias) v += a.bias[gn];
            if (a.resid) v += a.resid[gm * a.ldc + gn];
            if (a.act == CATNN_ACT_RELU) v = fmaxf(v, 0.f);
            else if (a.act == CATNN_ACT_GELU) v = gelu_dev(v);
            if (a.c_bf16) {
                bf16* p = (bf16*)Cb + gm * a.ldc + gn;
                if (a.accumulate) v += __bfloat162float(*p);
                *p = __float2bfloat16_rn(v);
            } else {
                float* p = (float*)Cb + gm * a.ldc + gn;
                if (a.accumulate) v += *p;
                *p = v;
            }
        }
    }
}

template <typename T>
static void launch_sgemm(Context* c, bool ta, bool tb, const SgemmArgs& a, i64 maxM, i64 maxN, int groups) {
    dim3 grid(cdiv(maxN, 128), cdiv(maxM, 128), groups);
    if (grid.x == 0 || grid.y == 0) return;
    CATNN_CHECK(grid.y <= 65535, CATNN_ERR_SHAPE, "simt gemm: M too large for one launch");
    if (!ta && !tb) k_sgemm<T, false, false><<<grid, 256, 0, c->stream>>>(a);
    else if (!ta && tb) k_sgemm<T, false, true><<<grid, 256, 0, c->stream>>>(a);
    else if (ta && !tb) k_sgemm<T, true, false><<<grid, 256, 0, c->stream>>>(a);
    else k_sgemm<T, true, true><<<grid, 256, 0, c->stream>>>(a);
    launched(c);
}

void gemm_f32(Context* c, bool ta, bool tb, i64 M, i64 N, i64 K, const float* A, i64 lda, const float* B, i64 ldb,
              void* C, i64 ldc, int c_dtype, const float* bias, int act, bool accumulate, const float* resid) {
    if (M <= 0 || N <= 0) return;
    SgemmArgs a{M, N, K, A, lda, B, ldb, C, ldc, c_dtype == CATNN_BF16, bias, act, accumulate ? 1 : 0, resid,
                nullptr, 0, 0, 0};
    launch_sgemm<float>(c, ta, tb, a, M, N, 1);
}

// CUDA-core bf16 GEMM for shapes the TMA path does not take (tiny N such
// as the router's E, or unaligned pitches).
void gemm_bf16_simt(Context* c, bool ta, bool tb, i64 M, i64 N, i64 K, const bf16* A, i64 lda, const bf16* B, i64 ldb,
                    void* C, i64 ldc, int c_dtype, const float* bias, int act, bool accumulate, const float* resid) {
    if (M <= 0 || N <= 0) return;
    SgemmArgs a{M, N, K, A, lda, B, ldb, C, ldc, c_dtype == CATNN_BF16, bias, act, accumulate ? 1 : 0, resid,
                nullptr, 0, 0, 0};
    launch_sgemm<bf16>(c, ta, tb, a, M, N, 1);
}

void gemm_grouped_f32(Context* c, bool ta_rows, bool tb, i64 total_rows, i64 N, i64 K, int groups,
                      const int32_t* offsets, const float* A, i64 lda, const float* B, i64 strideB, i64 ldb, float* C,
                      i64 ldc, i64 strideC, bool accumulate) {
    if (groups <= 0 || N <= 0) return;
    if (!ta_rows) {
        SgemmArgs a{0, N, K, A, lda, B, ldb, C, ldc, 0, nullptr, 0, accumulate ? 1 : 0, nullptr, offsets, 0, strideB, 0};
        launch_sgemm<float>(c, false, tb, a, total_rows, N, groups);
    } else {
        // C_g[K, N] = A_gᵀ · B_g over the group's rows; here K is A's width.
        SgemmArgs a{K, N, 0, A, lda, B, ldb, C, ldc, 0, nullptr, 0, accumulate ? 1 : 0, nullptr, offsets, 1, 0, strideC};
        launch_sgemm<float>(c, true, false, a, K, N, groups);
    }
}

void gemm(Context* c, bool ta, bool tb, i64 M, i64 N, i64 K, const void* A, i64 lda, const void* B, i64 ldb,
          void* C, i64 ldc, int dtype, int c_dtype, const float* bias, int act, bool accumulate, const float* resid) {
    check_dtype(dtype);
    check_dtype(c_dtype);
    CATNN_CHECK(M >= 0 && N >= 0 && K >= 0, CATNN_ERR_SHAPE, "gemm: negative size");
    CATNN_CHECK(!(accumulate && act != CATNN_ACT_NONE), CATNN_ERR_INVALID, "gemm: accumulate with an activation");
    CATNN_CHECK(!resid || c_dtype == CATNN_F32, CATNN_ERR_DTYPE, "gemm: a residual input needs an fp32 output");
    if (M == 0 || N == 0) return;
    if (dtype == CATNN_F32)
        gemm_f32(c, ta, tb, M, N, K, (const float*)A, lda, (const float*)B, ldb, C, ldc, c_dtype, bias, act, accumulate,
                 resid);
    else
        gemm_bf16_tc(c, ta, tb, M, N, K, (const bf16*)A, lda, (const bf16*)B, ldb, C, ldc, c_dtype, bias, act, accumulate,
                     resid);
}

}  // namespace catnn
