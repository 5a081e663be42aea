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

// Shared epilogue: bias, residual, activation, then store or accumulate.
__device__ __forceinline__ void store_out(const SgemmArgs& a, char* Cb, i64 gm, i64 gn, float v) {
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
            store_out(a, Cb, gm, gn, acc[i][j]);
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

// ---- router-shaped fp32 GEMMs (one side is the expert count, <= 32)
//
// The 128x128 tile above runs the MoE gate's three GEMMs (moe.rs:263 logits,
// adjoint.rs:255-284 input and weight gradients) on a handful of CTAs; these
// kernels give them the whole GPU and keep them at HBM speed.

// C[M, N] = A[M, K] · B with N <= NB: one warp per row of A reads the row
// coalesced (float4 when aligned); B sits in shared memory as [NB][K] so the
// lanes of a warp read consecutive words. Each lane keeps NB partial sums;
// a butterfly reduction gives every lane the totals and lane n stores C[row, n].
template <int NB>
__global__ void __launch_bounds__(256) k_narrow_rows(SgemmArgs a, int tb, int vec) {
    extern __shared__ float Bsh[];  // [NB][K]
    const i64 M = a.M, K = a.K;
    const int N = (int)a.N;
    const float* A = (const float*)a.A;
    const float* B = (const float*)a.B;
    for (i64 i = threadIdx.x; i < (i64)NB * K; i += blockDim.x) {
        int n = (int)(i / K);
        i64 k = i - (i64)n * K;
        float v = 0.f;
        if (n < N) v = tb ? B[(i64)n * a.ldb + k] : B[k * a.ldb + n];
        Bsh[i] = v;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const i64 wstride = (i64)gridDim.x * 16;
    // each warp takes two rows at a time: every B word read from shared
    // memory feeds two FMAs
    for (i64 row = (i64)blockIdx.x * 16 + 2 * warp; row < M; row += wstride) {
        const bool two = row + 1 < M;
        float acc0[NB], acc1[NB];
#pragma unroll
        for (int n = 0; n < NB; ++n) acc0[n] = acc1[n] = 0.f;
        const float* a0 = A + row * a.lda;
        const float* a1 = two ? a0 + a.lda : a0;
        if (vec) {
#pragma unroll 2
            for (i64 k = 4 * lane; k < K; k += 128) {
                float4 x0 = *(const float4*)(a0 + k);
                float4 x1 = *(const float4*)(a1 + k);
#pragma unroll
                for (int n = 0; n < NB; ++n) {
                    float4 b = *(const float4*)(Bsh + (i64)n * K + k);
                    acc0[n] = fmaf(x0.x, b.x, acc0[n]);
                    acc0[n] = fmaf(x0.y, b.y, acc0[n]);
                    acc0[n] = fmaf(x0.z, b.z, acc0[n]);
                    acc0[n] = fmaf(x0.w, b.w, acc0[n]);
                    acc1[n] = fmaf(x1.x, b.x, acc1[n]);
                    acc1[n] = fmaf(x1.y, b.y, acc1[n]);
                    acc1[n] = fmaf(x1.z, b.z, acc1[n]);
                    acc1[n] = fmaf(x1.w, b.w, acc1[n]);
                }
            }
        } else {
            for (i64 k = lane; k < K; k += 32) {
                float x0 = a0[k], x1 = a1[k];
#pragma unroll
                for (int n = 0; n < NB; ++n) {
                    float b = Bsh[(i64)n * K + k];
                    acc0[n] = fmaf(x0, b, acc0[n]);
                    acc1[n] = fmaf(x1, b, acc1[n]);
                }
            }
        }
        float v0 = 0.f, v1 = 0.f;
#pragma unroll
        for (int n = 0; n < NB; ++n) {
            float t0 = warp_sum(acc0[n]), t1 = warp_sum(acc1[n]);
            if (lane == n) {
                v0 = t0;
                v1 = t1;
            }
        }
        if (lane < N) {
            store_out(a, (char*)a.C, row, lane, v0);
            if (two) store_out(a, (char*)a.C, row + 1, lane, v1);
        }
    }
}

// Split-K partial sums of C[M, N] = Aᵀ · B with A [K, M] and B [K, N], N <= NB,
// K long (the gate's weight gradient: K = tokens). CTA (x, y) owns 256
// columns of A and rows [y*kc, (y+1)*kc); B's rows are staged 256 at a time
// and read as broadcasts. part is [chunks][M][NB].
template <int NB>
__global__ void __launch_bounds__(256) k_narrow_wgrad_part(SgemmArgs a, i64 kc, float* __restrict__ part) {
    __shared__ __align__(16) float Bs[256][NB];
    const i64 M = a.M, K = a.K;
    const int N = (int)a.N;
    const float* A = (const float*)a.A;
    const float* B = (const float*)a.B;
    const i64 m = (i64)blockIdx.x * 256 + threadIdx.x;
    const i64 k0 = (i64)blockIdx.y * kc, k1 = min(K, k0 + kc);
    float acc[NB];
#pragma unroll
    for (int n = 0; n < NB; ++n) acc[n] = 0.f;
    for (i64 s = k0; s < k1; s += 256) {
        const int rows = (int)min((i64)256, k1 - s);
        __syncthreads();
        for (int i = threadIdx.x; i < 256 * NB; i += 256) {
            int r = i / NB, n = i - r * NB;
            Bs[r][n] = (r < rows && n < N) ? B[(s + r) * a.ldb + n] : 0.f;
        }
        __syncthreads();
        if (m < M) {
            const float* ap = A + s * a.lda + m;
#pragma unroll 8
            for (int r = 0; r < rows; ++r) {
                float x = ap[(i64)r * a.lda];
#pragma unroll
                for (int n = 0; n < NB; n += 4) {
                    float4 b = *(const float4*)&Bs[r][n];
                    acc[n] = fmaf(x, b.x, acc[n]);
                    acc[n + 1] = fmaf(x, b.y, acc[n + 1]);
                    acc[n + 2] = fmaf(x, b.z, acc[n + 2]);
                    acc[n + 3] = fmaf(x, b.w, acc[n + 3]);
                }
            }
        }
    }
    if (m < M) {
        float4* o = (float4*)(part + ((i64)blockIdx.y * M + m) * NB);
#pragma unroll
        for (int n = 0; n < NB; n += 4) o[n / 4] = make_float4(acc[n], acc[n + 1], acc[n + 2], acc[n + 3]);
    }
}

// Sums the chunk partials and applies the epilogue. A CTA covers 32
// outputs with 8 threads each: thread slice j sums chunks j, j+8, ... in
// order, then slice sums are added 0..7 — a fixed order, so run to run the
// bits are the same.
__global__ void __launch_bounds__(256) k_narrow_wgrad_final(SgemmArgs a, const float* __restrict__ part, int chunks,
                                                            int nb) {
    __shared__ float red[8][33];
    const int col = threadIdx.x & 31, slice = threadIdx.x >> 5;
    const i64 i = (i64)blockIdx.x * 32 + col;
    const i64 MN = a.M * a.N;
    i64 m = 0;
    int n = 0;
    float s = 0.f;
    if (i < MN) {
        m = i / a.N;
        n = (int)(i - m * a.N);
#pragma unroll 4
        for (int ch = slice; ch < chunks; ch += 8) s += part[((i64)ch * a.M + m) * nb + n];
    }
    red[slice][col] = s;
    __syncthreads();
    if (slice == 0 && i < MN) {
        float t = red[0][col];
#pragma unroll
        for (int j = 1; j < 8; ++j) t += red[j][col];
        store_out(a, (char*)a.C, m, n, t);
    }
}

// C[M, N] = A[M, K] · B with K <= KB (the gate's input gradient: K = experts):
// B staged as [K][N] in shared memory, one CTA per row at a time, threads
// across N. Sums run k = 0..K-1 with fmaf, the same order as the tiled kernel.
template <int KB>
__global__ void __launch_bounds__(256) k_short_k(SgemmArgs a, int tb) {
    extern __shared__ float Bsh[];  // [K][N]
    const i64 M = a.M, N = a.N;
    const int K = (int)a.K;
    const float* A = (const float*)a.A;
    const float* B = (const float*)a.B;
    for (i64 i = threadIdx.x; i < (i64)K * N; i += blockDim.x) {
        int k = (int)(i / N);
        i64 n = i - (i64)k * N;
        Bsh[i] = tb ? B[n * a.ldb + k] : B[(i64)k * a.ldb + n];
    }
    __syncthreads();
    for (i64 row = blockIdx.x; row < M; row += gridDim.x) {
        float x[KB];
        const float* ar = A + row * a.lda;
#pragma unroll
        for (int k = 0; k < KB; ++k) x[k] = k < K ? ar[k] : 0.f;
        for (i64 n = threadIdx.x; n < N; n += blockDim.x) {
            float acc = 0.f;
#pragma unroll
            for (int k = 0; k < KB; ++k)
                if (k < K) acc = fmaf(x[k], Bsh[(i64)k * N + n], acc);
            store_out(a, (char*)a.C, row, n, acc);
        }
    }
}

// Fast form of k_short_k for a plain fp32 output (no bias, residual or
// activation; N % 4 == 0, 16-byte aligned rows): each thread owns a float4
// column group and R rows at a time, so R loads of C are in flight per
// thread. Same k order and the same final "+ C" as k_short_k.
template <int KB, int R>
__global__ void __launch_bounds__(256) k_short_k_vec(SgemmArgs a, int tb) {
    extern __shared__ __align__(16) float Bsh4[];  // [K][N]
    const i64 M = a.M, N = a.N;
    const int K = (int)a.K;
    const float* A = (const float*)a.A;
    const float* B = (const float*)a.B;
    float* C = (float*)a.C;
    for (i64 i = threadIdx.x; i < (i64)K * N; i += blockDim.x) {
        int k = (int)(i / N);
        i64 n = i - (i64)k * N;
        Bsh4[i] = tb ? B[n * a.ldb + k] : B[(i64)k * a.ldb + n];
    }
    __syncthreads();
    const i64 N4 = N / 4;
    for (i64 row0 = (i64)blockIdx.x * R; row0 < M; row0 += (i64)gridDim.x * R) {
        for (i64 n4 = threadIdx.x; n4 < N4; n4 += blockDim.x) {
            float4 cin[R];
            if (a.accumulate) {
#pragma unroll
                for (int r = 0; r < R; ++r)
                    if (row0 + r < M) cin[r] = *(const float4*)(C + (row0 + r) * a.ldc + 4 * n4);
            }
            float4 b[KB];
#pragma unroll
            for (int k = 0; k < KB; ++k)
                if (k < K) b[k] = *(const float4*)(Bsh4 + (i64)k * N + 4 * n4);
#pragma unroll
            for (int r = 0; r < R; ++r) {
                if (row0 + r >= M) break;
                const float* ar = A + (row0 + r) * a.lda;
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int k = 0; k < KB; ++k) {
                    if (k < K) {
                        float x = ar[k];
                        acc.x = fmaf(x, b[k].x, acc.x);
                        acc.y = fmaf(x, b[k].y, acc.y);
                        acc.z = fmaf(x, b[k].z, acc.z);
                        acc.w = fmaf(x, b[k].w, acc.w);
                    }
                }
                if (a.accumulate) {
                    acc.x += cin[r].x;
                    acc.y += cin[r].y;
                    acc.z += cin[r].z;
                    acc.w += cin[r].w;
                }
                *(float4*)(C + (row0 + r) * a.ldc + 4 * n4) = acc;
            }
        }
    }
}

template <typename F>
static void allow_smem(F* f, size_t bytes) {
    if (bytes > 48 * 1024) CUDA_OK(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
}

static constexpr size_t NARROW_SMEM_MAX = 96 * 1024;

// Returns true when one of the router-shaped kernels took the GEMM.
static bool gemm_f32_narrow(Context* c, bool ta, bool tb, const SgemmArgs& a) {
    const i64 M = a.M, N = a.N, K = a.K;
    if (!ta && N <= 32 && K >= 32) {
        int nb = N <= 8 ? 8 : N <= 16 ? 16 : 32;
        size_t smem = (size_t)nb * K * 4;
        if (smem > NARROW_SMEM_MAX) return false;
        int vec = (K % 4 == 0 && a.lda % 4 == 0 && ((uintptr_t)a.A & 15) == 0) ? 1 : 0;
        int grid = (int)std::min<i64>(cdiv(M, 16), (i64)c->sm_count * 4);
        if (nb == 8) { allow_smem(k_narrow_rows<8>, smem); k_narrow_rows<8><<<grid, 256, smem, c->stream>>>(a, tb, vec); }
        else if (nb == 16) { allow_smem(k_narrow_rows<16>, smem); k_narrow_rows<16><<<grid, 256, smem, c->stream>>>(a, tb, vec); }
        else { allow_smem(k_narrow_rows<32>, smem); k_narrow_rows<32><<<grid, 256, smem, c->stream>>>(a, tb, vec); }
        launched(c);
        return true;
    }
    if (ta && !tb && N <= 32 && K >= 1024) {
        int nb = N <= 8 ? 8 : N <= 16 ? 16 : 32;
        i64 gx = cdiv(M, 256);
        i64 chunks = std::max<i64>(1, std::min<i64>(cdiv((i64)c->sm_count * 4, gx), cdiv(K, 64)));
        i64 kc = cdiv(K, chunks);
        chunks = cdiv(K, kc);
        CATNN_CHECK(chunks <= 65535, CATNN_ERR_SHAPE, "narrow wgrad: too many chunks");
        float* part = (float*)c->scratch_for((size_t)chunks * M * nb * 4);
        dim3 g(gx, chunks);
        if (nb == 8) k_narrow_wgrad_part<8><<<g, 256, 0, c->stream>>>(a, kc, part);
        else if (nb == 16) k_narrow_wgrad_part<16><<<g, 256, 0, c->stream>>>(a, kc, part);
        else k_narrow_wgrad_part<32><<<g, 256, 0, c->stream>>>(a, kc, part);
        k_narrow_wgrad_final<<<cdiv(M * N, 32), 256, 0, c->stream>>>(a, part, (int)chunks, nb);
        launched(c, 2);
        return true;
    }
    if (!ta && K <= 32 && K >= 1 && N >= 64) {
        int kb = K <= 8 ? 8 : K <= 16 ? 16 : 32;
        size_t smem = (size_t)K * N * 4;
        if (smem > NARROW_SMEM_MAX) return false;
        const bool plain = !a.c_bf16 && !a.bias && !a.resid && a.act == CATNN_ACT_NONE && N % 4 == 0 &&
                           a.ldc % 4 == 0 && aligned_to(a.C, 16);
        if (plain) {
            constexpr int R = 4;
            int grid = (int)std::min<i64>(cdiv(M, R), (i64)c->sm_count * 6);
            if (kb == 8) { allow_smem(k_short_k_vec<8, R>, smem); k_short_k_vec<8, R><<<grid, 256, smem, c->stream>>>(a, tb); }
            else if (kb == 16) { allow_smem(k_short_k_vec<16, R>, smem); k_short_k_vec<16, R><<<grid, 256, smem, c->stream>>>(a, tb); }
            else { allow_smem(k_short_k_vec<32, R>, smem); k_short_k_vec<32, R><<<grid, 256, smem, c->stream>>>(a, tb); }
            launched(c);
            return true;
        }
        int grid = (int)std::min<i64>(M, (i64)c->sm_count * 2);
        if (kb == 8) { allow_smem(k_short_k<8>, smem); k_short_k<8><<<grid, 256, smem, c->stream>>>(a, tb); }
        else if (kb == 16) { allow_smem(k_short_k<16>, smem); k_short_k<16><<<grid, 256, smem, c->stream>>>(a, tb); }
        else { allow_smem(k_short_k<32>, smem); k_short_k<32><<<grid, 256, smem, c->stream>>>(a, tb); }
        launched(c);
        return true;
    }
    return false;
}

void gemm_f32(Context* c, bool ta, bool tb, i64 M, i64 N, i64 K, const float* A, i64 lda, const float* B, i64 ldb,
              void* C, i64 ldc, int c_dtype, const float* bias, int act, bool accumulate, const float* resid) {
    if (M <= 0 || N <= 0) return;
    SgemmArgs a{M, N, K, A, lda, B, ldb, C, ldc, c_dtype == CATNN_BF16, bias, act, accumulate ? 1 : 0, resid,
                nullptr, 0, 0, 0};
    if (gemm_f32_narrow(c, ta, tb, a)) return;
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
    if (dtype == CATNN_TF32) {
        // fp32 operands, multiplied on the tensor cores as TF32
        check_dtype(c_dtype);
        CATNN_CHECK(M >= 0 && N >= 0 && K >= 0, CATNN_ERR_SHAPE, "gemm: negative size");
        CATNN_CHECK(!(accumulate && act != CATNN_ACT_NONE), CATNN_ERR_INVALID, "gemm: accumulate with an activation");
        CATNN_CHECK(!resid, CATNN_ERR_UNSUPPORTED, "tf32 gemm: no residual input");
        gemm_tf32_tc(c, ta, tb, M, N, K, (const float*)A, lda, (const float*)B, ldb, C, ldc, c_dtype, bias, act,
                     accumulate);
        return;
    }
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

// fp32 GEMMs of linear / matmul / lm_head / the MoE experts: 128 x 128
// output tiles, 256 threads.
KernelInfo sgemm_info(Context* c, const std::string& op, const KShape& s) {
    KernelInfo k;
    if (!(op == "linear" || op == "matmul" || op == "lm_head" || op == "moe")) return k;
    k.fn = op == "lm_head" ? (const void*)k_sgemm<float, false, true> : (const void*)k_sgemm<float, false, false>;
    k.file = "gemm.cu";
    k.grid[0] = (unsigned)cdiv(s.width, 128);
    k.grid[1] = (unsigned)cdiv(s.rows, 128);
    k.block[0] = 256;
    return k;
}

}  // namespace catnn
