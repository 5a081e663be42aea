// bf16 GEMM on the 5th-generation tensor cores (tcgen05) with TMEM
// accumulators, fed by TMA. Persistent, warp-specialized:
//   warp 0      TMA producer (one elected thread) over a STAGES-deep ring
//   warp 1      TMEM owner + MMA issuer (one thread), 128 x BN x 16 MMAs
//   warps 2..9  epilogue: TMEM -> registers -> bias/activation -> HBM; two
//               warps per TMEM lane quadrant (warp % 4), each taking half of
//               the tile's columns, so one warp's latency hides behind the
//               other's work on the same sub-partition
// Two TMEM accumulators (2*BN columns) let the epilogue of tile i overlap
// the MMAs of tile i+1. Every mbarrier wait is bounded (see tc::mbar_wait).
//
// One kernel covers the three shapes the hot path needs:
//   mode 0  plain C = op(A)·op(B)       (linear fwd, dgrad, wgrad, LM head)
//   mode 1  M-grouped: rows [off[g], off[g+1]) of A and C use B_g
//           (MoE expert GEMMs over the expert-sorted token rows)
//   mode 2  K-grouped: C_g = A_gᵀ·B_g over the rows of group g
//           (MoE expert weight gradients)
// Operands are K-major or MN-major (instruction-descriptor transpose bits),
// so no transposed copies of weights or activations are ever made.
#include <cudaTypedefs.h>

#include <cstring>

#include "ops.cuh"
#include "tc_prims.cuh"

namespace catnn {

struct TcArgs {
    int mode, groups;
    const int32_t* offsets;
    int M, N, K;
    int b_group_rows;
    void* C;
    long long ldc, c_group_stride;
    int c_bf16, vec_ok;
    const float* bias;
    const float* resid;  // fp32 [M, ldc] added before the activation (C must be fp32)
    int act, accumulate;
    int* status;
    // split-K: ksplit > 1 cuts each tile's K range into ksplit slices whose
    // fp32 partial sums go to part[slice] (no epilogue); k_splitk_reduce
    // then adds the slices in order and applies the epilogue.
    int ksplit, kchunk;
    float* part;
    long long c_group_stride_part;  // elements between two slices of part
    // tma_c: full 32-row blocks of C (no accumulate) are staged in shared memory and
    // written by TMA bulk stores of mapC
    int tma_c;
    // SwiGLU epilogues of the MoE expert GEMMs (mode 1, bf16). The [a | c]
    // columns are interleaved in blocks of 128: block j holds a's columns
    // [128j, 128j + 128) and then the same columns of c, so one 256-wide
    // output tile holds both halves of 128 SwiGLU columns.
    //  epi 1 (x·W13): C = [a | c] in that layout (bf16, what the backward reads)
    //         and aux = h = silu(a)·c ([rows, F], ld ldaux) from the rounded a, c;
    //  epi 2 (dyp·W2ᵀ = dh, never stored): reads a, c from aux ([rows, 2F],
    //         ld ldaux), writes C = [da | dc] (same layout, ld ldc) with
    //         da = dh·c·silu'(a), dc = dh·silu(a) from dh rounded to bf16.
    int epi;
    void* aux;
    long long ldaux;
};

static constexpr int BM = 128, BK = 64;
static constexpr int EPI_WARPS = 8;
static constexpr int GEMM_THREADS = 32 * (2 + EPI_WARPS);
static constexpr uint32_t EPI_STAGE_BYTES = EPI_WARPS * 2 * 2048;  // two 2 KB buffers per epilogue warp

struct TileInfo {
    int g, m0, n0, kstart, klen, mlimit, arow0, ks;
};

// Total tiles and the t-th tile of the static schedule. Groups are few
// (experts), so a linear scan is cheaper than a device-side prefix sum.
template <int BN>
__device__ __forceinline__ int base_tiles(const TcArgs& a) {
    int nt = (a.N + BN - 1) / BN;
    if (a.mode == 0) return ((a.M + BM - 1) / BM) * nt;
    if (a.mode == 2) return a.groups * ((a.M + BM - 1) / BM) * nt;
    int tot = 0;
    for (int g = 0; g < a.groups; ++g) tot += ((a.offsets[g + 1] - a.offsets[g] + BM - 1) / BM) * nt;
    return tot;
}
template <int BN>
__device__ __forceinline__ int total_tiles(const TcArgs& a) {
    return base_tiles<BN>(a) * a.ksplit;
}

template <int BN>
__device__ __forceinline__ TileInfo tile_at_base(const TcArgs& a, int t);

// Tile t of the schedule: the K slice is the slowest index, so the tiles
// running at the same time share their operands' K slice in L2.
template <int BN>
__device__ __forceinline__ TileInfo tile_at(const TcArgs& a, int t) {
    if (a.ksplit <= 1) return tile_at_base<BN>(a, t);
    int nb = base_tiles<BN>(a);
    int ks = t / nb;
    TileInfo ti = tile_at_base<BN>(a, t - ks * nb);
    // mode 2 cuts each group's own row range; modes 0 and 1 share one chunk
    int chunk = a.mode == 2 ? ((ti.klen + a.ksplit - 1) / a.ksplit + BK - 1) / BK * BK : a.kchunk;
    int k0 = ks * chunk;
    int len = ti.klen - k0;
    ti.kstart += k0;
    ti.klen = len < 0 ? 0 : (len < chunk ? len : chunk);
    ti.ks = ks;
    return ti;
}

template <int BN>
__device__ __forceinline__ TileInfo tile_at_base(const TcArgs& a, int t) {
    TileInfo ti;
    ti.ks = 0;
    int nt = (a.N + BN - 1) / BN;
    if (a.mode == 0) {
        ti.g = 0;
        ti.m0 = (t / nt) * BM;
        ti.n0 = (t % nt) * BN;
        ti.kstart = 0;
        ti.klen = a.K;
        ti.mlimit = a.M;
        ti.arow0 = 0;
    } else if (a.mode == 2) {
        int mt = (a.M + BM - 1) / BM;
        int per = mt * nt;
        ti.g = t / per;
        int r = t % per;
        ti.m0 = (r / nt) * BM;
        ti.n0 = (r % nt) * BN;
        ti.kstart = a.offsets[ti.g];
        ti.klen = a.offsets[ti.g + 1] - ti.kstart;
        ti.mlimit = a.M;
        ti.arow0 = 0;
    } else {
        int g = 0;
        for (; g < a.groups; ++g) {
            int cnt = ((a.offsets[g + 1] - a.offsets[g] + BM - 1) / BM) * nt;
            if (t < cnt) break;
            t -= cnt;
        }
        ti.g = g;
        ti.m0 = (t / nt) * BM;
        ti.n0 = (t % nt) * BN;
        ti.kstart = 0;
        ti.klen = a.K;
        ti.arow0 = a.offsets[g];
        ti.mlimit = a.offsets[g + 1] - a.offsets[g];
    }
    return ti;
}

// moe.rs:12-14 / adjoint.rs:208-215 for the bf16 epilogues: σ(x) = 1/(1+e^-x)
// with the hardware exponential and reciprocal (a few ulp of fp32; the
// results are rounded to bf16, whose unit is 2^-8). One epilogue warp per
// sub-partition runs these serially, so short dependency chains matter more
// than the last fp32 bit: the IEEE exp and division cost ~35 instructions
// with branches, these ~4. The reciprocal is the single MUFU instruction
// (rcp.approx.ftz: relative error under 2^-22); for x below about -88 the
// exponential overflows to +inf and its reciprocal is 0, so σ = 0.
__device__ __forceinline__ float tc_rcp(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float tc_sigmoid(float x) { return tc_rcp(1.0f + __expf(-x)); }
__device__ __forceinline__ float tc_silu(float x) { return x * tc_sigmoid(x); }
// silu(x) and silu'(x) = σ + x·σ·(1-σ) from one σ
__device__ __forceinline__ float2 tc_silu_and_grad(float x) {
    const float s = tc_sigmoid(x);
    return make_float2(x * s, s + x * s * (1.0f - s));
}

// 32 bf16 values (packed in pairs) of one row of a warp's 32-row block:
// staged in the warp's shared-memory ring with the store map's 64-byte
// swizzle and written by one TMA store at (x, y) when the block's 32 rows are
// all valid (tma), else stored directly by the lanes with valid rows.
struct Stage32 {
    uint8_t* stage;  // this warp's four 2 KB buffers
    uint32_t* nst;   // stores issued by the warp (picks the buffer)
    int lane;
    __device__ __forceinline__ void put(const uint32_t (&pk)[16], const CUtensorMap* map, bool tma, int x, int y,
                                        bf16* direct, bool row_ok) {
        if (tma) {
            const int b = (int)(*nst & 1u);
            const uint32_t sb = tc::smem_u32(stage + b * 2048);
            if (lane == 0) tc::bulk_wait_read<1>();
            __syncwarp();
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4)
                tc::st_shared_v4(sb + lane * 64 + ((c4 ^ ((lane >> 1) & 3)) << 4),
                                 make_uint4(pk[c4 * 4], pk[c4 * 4 + 1], pk[c4 * 4 + 2], pk[c4 * 4 + 3]));
            tc::fence_proxy_async();
            __syncwarp();
            if (lane == 0) {
                tc::tma_store_2d(map, stage + b * 2048, x, y);
                tc::bulk_commit();
            }
            ++*nst;
        } else if (row_ok) {
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4)
                *(uint4*)(direct + c4 * 8) = make_uint4(pk[c4 * 4], pk[c4 * 4 + 1], pk[c4 * 4 + 2], pk[c4 * 4 + 3]);
        }
    }
};

__device__ __forceinline__ uint32_t pack_bf16x2(float x, float y) {
    __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
    return *(uint32_t*)&h;
}
__device__ __forceinline__ float2 unpack_bf16x2(uint32_t v) { return __bfloat1622float2(*(__nv_bfloat162*)&v); }

__device__ __forceinline__ float act_apply(float v, int act) {
    if (act == CATNN_ACT_RELU) return fmaxf(v, 0.f);
    if (act == CATNN_ACT_GELU) {
        const float k = 0.7978845608028654f;
        return 0.5f * v * (1.0f + tanhf(k * (v + 0.044715f * v * v * v)));
    }
    return v;
}

template <bool A_MN, bool B_MN, int BN, int STAGES, bool TF32 = false>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
              const __grid_constant__ CUtensorMap mapC, const __grid_constant__ CUtensorMap mapD, TcArgs a) {
    constexpr uint32_t A_BYTES = BM * BK * 2;
    constexpr uint32_t B_BYTES = BN * BK * 2;
    constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
    static_assert(!TF32 || (!A_MN && !B_MN), "TF32 operands are K-major");
    constexpr uint32_t IDESC = TF32 ? tc::idesc_tf32(BM, BN) : tc::idesc_bf16(BM, BN, A_MN, B_MN);
    // K elements per stage: one 128-byte swizzle row (64 bf16 or 32 fp32)
    constexpr int KB = TF32 ? BK / 2 : BK;
    constexpr uint32_t TMEM_COLS = 2 * BN;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    // epilogue staging for TMA stores: per epilogue warp four 2 KB blocks
    // of 32 rows x 64 bytes
    uint8_t* stage_c = smem + STAGES * STAGE_BYTES;
    uint64_t* full = (uint64_t*)(stage_c + EPI_STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = (uint32_t*)(drain + 1);

    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&tfull[i], 1);
            tc::mbar_init(&tempty[i], EPI_WARPS);
        }
        tc::mbar_init(drain, 1);
        tc::fence_mbar_init();
        tc::prefetch_tmap(&mapA);
        tc::prefetch_tmap(&mapB);
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, TMEM_COLS);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int ntiles = total_tiles<BN>(a);

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer
        int s = 0;
        uint32_t ph = 0;
        // per stage: was it ever filled (bit in used), and the parity of its last fill
        uint32_t used = 0, last_par = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
            TileInfo ti = tile_at<BN>(a, t);
            int nkb = (ti.klen + KB - 1) / KB;
            for (int kb = 0; kb < nkb; ++kb) {
                if (!tc::mbar_wait(&empty[s], ph ^ 1, a.status, 1)) {
                    ok = false;
                    break;
                }
                uint8_t* sA = smem + s * STAGE_BYTES;
                uint8_t* sB = sA + A_BYTES;
                tc::mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
                int k = ti.kstart + kb * KB;
                if (!A_MN) {
                    tc::tma_load_2d(sA, &mapA, k, ti.arow0 + ti.m0, &full[s]);
                } else {
#pragma unroll
                    for (int j = 0; j < BM / 64; ++j) tc::tma_load_2d(sA + j * 8192, &mapA, ti.m0 + 64 * j, k, &full[s]);
                }
                if (!B_MN) {
                    int brow = (a.mode == 1 ? ti.g * a.b_group_rows : 0) + ti.n0;
                    tc::tma_load_2d(sB, &mapB, k, brow, &full[s]);
                } else {
                    int brow = (a.mode == 1 ? ti.g * a.b_group_rows : 0) + k;
#pragma unroll
                    for (int j = 0; j < BN / 64; ++j) tc::tma_load_2d(sB + j * 8192, &mapB, ti.n0 + 64 * j, brow, &full[s]);
                }
                used |= 1u << s;
                last_par = (last_par & ~(1u << s)) | (ph << s);
                if (++s == STAGES) {
                    s = 0;
                    ph ^= 1;
                }
            }
        }
        if (!ok) {
            // Abort: let the copies already in flight land before the CTA exits.
            for (int i = 0; i < STAGES; ++i)
                if ((used >> i) & 1u) tc::mbar_wait(&full[i], (last_par >> i) & 1u, a.status, 1, 400000000ll, false);
        }
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer
        int s = 0;
        uint32_t ph = 0;
        int it = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++it) {
            TileInfo ti = tile_at<BN>(a, t);
            int acc = it & 1;
            if (!tc::mbar_wait(&tempty[acc], ((it >> 1) & 1) ^ 1, a.status, 2)) break;
            tc::tc_fence_after();
            uint32_t d = tmem_base + acc * BN;
            int nkb = (ti.klen + KB - 1) / KB;
            for (int kb = 0; kb < nkb; ++kb) {
                if (!tc::mbar_wait(&full[s], ph, a.status, 2)) {
                    ok = false;
                    break;
                }
                tc::tc_fence_after();
                uint32_t sA = tc::smem_u32(smem + s * STAGE_BYTES);
                uint32_t sB = sA + A_BYTES;
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk) {
                    uint64_t ad = A_MN ? tc::sdesc(sA + kk * 2048, 8192, 1024) : tc::sdesc(sA + kk * 32, 16, 1024);
                    uint64_t bd = B_MN ? tc::sdesc(sB + kk * 2048, 8192, 1024) : tc::sdesc(sB + kk * 32, 16, 1024);
                    if constexpr (TF32) tc::mma_tf32(d, ad, bd, IDESC, (kb | kk) != 0);
                    else tc::mma_bf16(d, ad, bd, IDESC, (kb | kk) != 0);
                }
                tc::mma_commit(&empty[s]);
                if (++s == STAGES) {
                    s = 0;
                    ph ^= 1;
                }
            }
            if (ok) tc::mma_commit(&tfull[acc]);
        }
        // Drain: no MMA may still write TMEM when it is freed.
        tc::mma_commit(drain);
        tc::mbar_wait(drain, 0, a.status, 2, 400000000ll, false);
    } else if (warp >= 2) {
        // ---------------- epilogue
        const int ew = warp - 2;     // epilogue warp 0..7
        const int q = warp & 3;      // TMEM lane quadrant this warp may read
        const int half = ew >> 2;    // which half of the tile's columns
        const bool plain = !a.bias && !a.resid && a.act == CATNN_ACT_NONE && !a.accumulate;
        int it = 0;
        uint32_t nst = 0;  // TMA stores issued by this warp (picks the staging buffer)
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
            TileInfo ti = tile_at<BN>(a, t);
            int acc = it & 1;
            if (!tc::mbar_wait(&tfull[acc], (it >> 1) & 1, a.status, 3)) break;
            tc::tc_fence_after();
            int row = ti.m0 + q * 32 + lane;
            bool rv = row < ti.mlimit;
            long long crow;
            if (a.mode == 0) crow = (long long)row * a.ldc;
            else if (a.mode == 1) crow = (long long)(ti.arow0 + row) * a.ldc;
            else crow = (long long)ti.g * a.c_group_stride + (long long)row * a.ldc;
            // TMA stores for this warp's 32 rows when they are all valid rows of
            // the output map (warp-uniform; split-K partials keep the direct path)
            const int row0 = ti.m0 + q * 32;
            const bool use_tma = a.tma_c && a.ksplit <= 1 && row0 + 32 <= ti.mlimit;
            const long long ybase =
                a.mode == 0 ? row0 : (a.mode == 1 ? (long long)ti.arow0 + row0 : (long long)ti.g * a.M + row0);
            if (a.epi != 0) {
                // SwiGLU epilogues (mode 1, bf16, no split-K; see TcArgs::epi)
                Stage32 st{stage_c + ew * 4096, &nst, lane};
                const bool tma = a.tma_c && row0 + 32 <= ti.mlimit;
                const long long grow = (long long)ti.arow0 + row;
                if (a.epi == 1) {
                    bf16* acp = (bf16*)a.C + grow * a.ldc;
                    bf16* hp = (bf16*)a.aux + grow * a.ldaux;
                    const int hcol0 = (ti.n0 >> 8) << 7;
#pragma unroll 1
                    for (int cc = half * 2; cc < half * 2 + 2; ++cc) {
                        uint32_t ra[32], rc[32];
                        tc::tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN + cc * 32, ra);
                        tc::tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN + 128 + cc * 32, rc);
                        tc::tmem_ld_wait();
                        uint32_t pa[16], pc[16], ph[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            pa[j] = pack_bf16x2(__uint_as_float(ra[2 * j]), __uint_as_float(ra[2 * j + 1]));
                            pc[j] = pack_bf16x2(__uint_as_float(rc[2 * j]), __uint_as_float(rc[2 * j + 1]));
                            const float2 av = unpack_bf16x2(pa[j]), cv = unpack_bf16x2(pc[j]);
                            ph[j] = pack_bf16x2(tc_silu(av.x) * cv.x, tc_silu(av.y) * cv.y);
                        }
                        const int ca = ti.n0 + cc * 32, ch = hcol0 + cc * 32;
                        st.put(pa, &mapC, tma, ca, (int)ybase, acp + ca, rv);
                        st.put(pc, &mapC, tma, ca + 128, (int)ybase, acp + ca + 128, rv);
                        st.put(ph, &mapD, tma, ch, (int)ybase, hp + ch, rv);
                    }
                } else {
                    const bf16* acin = (const bf16*)a.aux + grow * a.ldaux;
                    bf16* dacp = (bf16*)a.C + grow * a.ldc;
                    // a and c of 32 SwiGLU columns (interleaved layout) for chunk cc,
                    // loaded one chunk ahead so their latency overlaps the math
                    auto load_ac = [&](int cc, uint4 (&va)[4], uint4 (&vc)[4]) {
                        const int f0 = ti.n0 + cc * 32;
                        const int col = ((f0 >> 7) << 8) + (f0 & 127);
                        if (rv && f0 < a.N) {
#pragma unroll
                            for (int c4 = 0; c4 < 4; ++c4) {
                                va[c4] = *(const uint4*)(acin + col + c4 * 8);
                                vc[c4] = *(const uint4*)(acin + col + 128 + c4 * 8);
                            }
                        } else {
#pragma unroll
                            for (int c4 = 0; c4 < 4; ++c4) va[c4] = vc[c4] = make_uint4(0, 0, 0, 0);
                        }
                    };
                    uint4 na[4], nc[4];
                    const int c_beg = half * (BN / 64), c_end = c_beg + BN / 64;
                    load_ac(c_beg, na, nc);
#pragma unroll 1
                    for (int cc = c_beg; cc < c_end; ++cc) {
                        const int f0 = ti.n0 + cc * 32;
                        if (f0 >= a.N) break;  // warp-uniform
                        uint32_t r[32];
                        tc::tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN + cc * 32, r);
                        const int col = ((f0 >> 7) << 8) + (f0 & 127);
                        uint4 va[4], vc[4];
#pragma unroll
                        for (int c4 = 0; c4 < 4; ++c4) {
                            va[c4] = na[c4];
                            vc[c4] = nc[c4];
                        }
                        if (cc + 1 < c_end) load_ac(cc + 1, na, nc);
                        tc::tmem_ld_wait();
                        const uint32_t* ua = (const uint32_t*)va;
                        const uint32_t* uc = (const uint32_t*)vc;
                        uint32_t pda[16], pdc[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const float2 av = unpack_bf16x2(ua[j]), cv = unpack_bf16x2(uc[j]);
                            const float2 g = unpack_bf16x2(pack_bf16x2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1])));
                            const float2 sx = tc_silu_and_grad(av.x), sy = tc_silu_and_grad(av.y);
                            pda[j] = pack_bf16x2(g.x * cv.x * sx.y, g.y * cv.y * sy.y);
                            pdc[j] = pack_bf16x2(g.x * sx.x, g.y * sy.x);
                        }
                        st.put(pda, &mapC, tma, col, (int)ybase, dacp + col, rv);
                        st.put(pdc, &mapC, tma, col + 128, (int)ybase, dacp + col + 128, rv);
                    }
                }
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&tempty[acc]);
                continue;
            }
#pragma unroll 1
            for (int cc = half * (BN / 64); cc < (half + 1) * (BN / 64); ++cc) {
                int col0 = ti.n0 + cc * 32;
                if (col0 >= a.N) break;  // warp-uniform
                uint32_t r[32];
                tc::tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN + cc * 32, r);
                tc::tmem_ld_wait();
                if (!rv) continue;
                if (a.ksplit > 1) {
                    // raw fp32 partial of this K slice: part[ks] is [rows, N] with
                    // rows = M (mode 0), total rows (mode 1), groups·M (mode 2)
                    long long prow = a.mode == 0 ? row : (a.mode == 1 ? ti.arow0 + row : (long long)ti.g * a.M + row);
                    float* p = a.part + (long long)ti.ks * a.c_group_stride_part + prow * a.N + col0;
                    bool vec = (a.N % 4 == 0) && (col0 + 32 <= a.N);
                    if (vec) {
#pragma unroll
                        for (int i4 = 0; i4 < 8; ++i4) {
                            float4 w;
                            w.x = ti.klen > 0 ? __uint_as_float(r[i4 * 4 + 0]) : 0.f;
                            w.y = ti.klen > 0 ? __uint_as_float(r[i4 * 4 + 1]) : 0.f;
                            w.z = ti.klen > 0 ? __uint_as_float(r[i4 * 4 + 2]) : 0.f;
                            w.w = ti.klen > 0 ? __uint_as_float(r[i4 * 4 + 3]) : 0.f;
                            *(float4*)(p + i4 * 4) = w;
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (col0 + i < a.N) p[i] = ti.klen > 0 ? __uint_as_float(r[i]) : 0.f;
                    }
                    continue;
                }
                bool full_chunk = a.vec_ok && (col0 + 32 <= a.N);
                if (use_tma) {
                    // Stage the warp's 32 x 32 block with the store map's swizzle
                    // (16-byte chunk c of row l at chunk c ^ f(l): conflict-free
                    // st.shared), then one lane issues an async TMA store: whole
                    // 64/128-byte row segments, fewer L2 transactions than per-row
                    // 16-byte stores, no stall of the warp. Bias, residual (16-byte
                    // loads) and activation are applied first, one uniform branch
                    // per option.
                    const bool z = ti.klen <= 0;
                    if (!plain) {
                        float v[32];
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = z ? 0.f : __uint_as_float(r[i]);
                        if (a.bias) {
#pragma unroll
                            for (int i = 0; i < 32; ++i)
                                if (col0 + i < a.N) v[i] += a.bias[col0 + i];
                        }
                        if (a.resid) {
                            const float* rs = a.resid + crow + col0;
                            if (col0 + 32 <= a.N) {
#pragma unroll
                                for (int i4 = 0; i4 < 8; ++i4) {
                                    const float4 q4 = *(const float4*)(rs + i4 * 4);
                                    v[i4 * 4] += q4.x;
                                    v[i4 * 4 + 1] += q4.y;
                                    v[i4 * 4 + 2] += q4.z;
                                    v[i4 * 4 + 3] += q4.w;
                                }
                            } else {
#pragma unroll
                                for (int i = 0; i < 32; ++i)
                                    if (col0 + i < a.N) v[i] += rs[i];
                            }
                        }
                        if (a.act == CATNN_ACT_RELU) {
#pragma unroll
                            for (int i = 0; i < 32; ++i) v[i] = act_apply(v[i], CATNN_ACT_RELU);
                        } else if (a.act == CATNN_ACT_GELU) {
#pragma unroll
                            for (int i = 0; i < 32; ++i) v[i] = act_apply(v[i], CATNN_ACT_GELU);
                        }
#pragma unroll
                        for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(v[i]);
                    }
                    const bool zz = plain && z;  // r now holds the final values unless plain
                    // four 2 KB buffers per warp: a bf16 chunk is one 32 x 32 box,
                    // an fp32 chunk two 32 x 16 boxes (64-byte rows either way)
                    const int b = (int)(nst & 1u);
                    const uint32_t sb = tc::smem_u32(stage_c + ew * 4096 + b * 2048);
                    if (lane == 0) tc::bulk_wait_read<1>();  // this buffer's previous store has read it
                    __syncwarp();
                    if (a.c_bf16) {
#pragma unroll
                        for (int c4 = 0; c4 < 4; ++c4) {
                            uint4 pk;
                            __nv_bfloat162* pp = (__nv_bfloat162*)&pk;
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                pp[j] = zz ? __floats2bfloat162_rn(0.f, 0.f)
                                           : __floats2bfloat162_rn(__uint_as_float(r[c4 * 8 + 2 * j]),
                                                                   __uint_as_float(r[c4 * 8 + 2 * j + 1]));
                            tc::st_shared_v4(sb + lane * 64 + ((c4 ^ ((lane >> 1) & 3)) << 4), pk);
                        }
                        tc::fence_proxy_async();
                        __syncwarp();
                        if (lane == 0) {
                            tc::tma_store_2d(&mapC, stage_c + ew * 4096 + b * 2048, col0, (int)ybase);
                            tc::bulk_commit();
                        }
                        ++nst;
                        continue;
                    }
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
                        const int bh = (int)(nst & 1u);
                        const uint32_t sbh = tc::smem_u32(stage_c + ew * 4096 + bh * 2048);
                        if (hh == 1) {
                            if (lane == 0) tc::bulk_wait_read<1>();
                            __syncwarp();
                        }
#pragma unroll
                        for (int c4 = 0; c4 < 4; ++c4) {
                            const int e0 = hh * 16 + c4 * 4;
                            uint4 pk = zz ? make_uint4(0, 0, 0, 0) : make_uint4(r[e0], r[e0 + 1], r[e0 + 2], r[e0 + 3]);
                            tc::st_shared_v4(sbh + lane * 64 + ((c4 ^ ((lane >> 1) & 3)) << 4), pk);
                        }
                        tc::fence_proxy_async();
                        __syncwarp();
                        if (lane == 0) {
                            tc::tma_store_2d(&mapC, stage_c + ew * 4096 + bh * 2048, col0 + hh * 16, (int)ybase);
                            tc::bulk_commit();
                        }
                        ++nst;
                    }
                    continue;
                }
                if (plain && full_chunk) {
                    // the common case (no bias, residual, activation or
                    // accumulate): convert and store, nothing per element else
                    const bool z = ti.klen <= 0;
                    if (a.c_bf16) {
                        bf16* p = (bf16*)a.C + crow + col0;
#pragma unroll
                        for (int i4 = 0; i4 < 4; ++i4) {
                            uint4 pk;
                            __nv_bfloat162* pp = (__nv_bfloat162*)&pk;
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                pp[j] = z ? __floats2bfloat162_rn(0.f, 0.f)
                                          : __floats2bfloat162_rn(__uint_as_float(r[i4 * 8 + 2 * j]),
                                                                  __uint_as_float(r[i4 * 8 + 2 * j + 1]));
                            *(uint4*)(p + i4 * 8) = pk;
                        }
                    } else {
                        float* p = (float*)a.C + crow + col0;
#pragma unroll
                        for (int i4 = 0; i4 < 8; ++i4) {
                            uint4 pk = z ? make_uint4(0, 0, 0, 0)
                                         : make_uint4(r[i4 * 4], r[i4 * 4 + 1], r[i4 * 4 + 2], r[i4 * 4 + 3]);
                            *(uint4*)(p + i4 * 4) = pk;
                        }
                    }
                    continue;
                }
                // General path. Each option is one uniform branch around its
                // own loop, so a disabled option costs nothing per element.
                float v[32];
                const bool z = ti.klen <= 0;
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = z ? 0.f : __uint_as_float(r[i]);
                if (a.bias) {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (full_chunk || col0 + i < a.N) v[i] += a.bias[col0 + i];
                }
                if (a.resid) {
                    const float* rs = a.resid + crow + col0;
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (full_chunk || col0 + i < a.N) v[i] += rs[i];
                }
                if (a.c_bf16) {
                    bf16* p = (bf16*)a.C + crow + col0;
                    if (a.accumulate) {
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (full_chunk || col0 + i < a.N) v[i] += __bfloat162float(p[i]);
                    }
                    if (a.act == CATNN_ACT_RELU) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = act_apply(v[i], CATNN_ACT_RELU);
                    } else if (a.act == CATNN_ACT_GELU) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = act_apply(v[i], CATNN_ACT_GELU);
                    }
                    if (full_chunk) {
#pragma unroll
                        for (int i4 = 0; i4 < 4; ++i4) {
                            uint4 pk;
                            __nv_bfloat162* pp = (__nv_bfloat162*)&pk;
#pragma unroll
                            for (int j = 0; j < 4; ++j) pp[j] = __floats2bfloat162_rn(v[i4 * 8 + 2 * j], v[i4 * 8 + 2 * j + 1]);
                            *(uint4*)(p + i4 * 8) = pk;
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (col0 + i < a.N) p[i] = __float2bfloat16_rn(v[i]);
                    }
                } else {
                    float* p = (float*)a.C + crow + col0;
                    if (a.accumulate) {
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (full_chunk || col0 + i < a.N) v[i] += p[i];
                    }
                    if (a.act == CATNN_ACT_RELU) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = act_apply(v[i], CATNN_ACT_RELU);
                    } else if (a.act == CATNN_ACT_GELU) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = act_apply(v[i], CATNN_ACT_GELU);
                    }
                    if (full_chunk) {
#pragma unroll
                        for (int i4 = 0; i4 < 8; ++i4)
                            *(float4*)(p + i4 * 4) = make_float4(v[i4 * 4], v[i4 * 4 + 1], v[i4 * 4 + 2], v[i4 * 4 + 3]);
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (col0 + i < a.N) p[i] = v[i];
                    }
                }
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&tempty[acc]);
        }
        // the stores must have left shared memory (and landed) before the CTA exits
        if (lane == 0) tc::bulk_wait_all();
        __syncwarp();
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// Split-K epilogue: C = epilogue(Σ_slices part[slice]) with the slices added
// in order (deterministic), then bias, residual, accumulate and activation
// as in k_gemm_tc. CTAs stride over partial rows, threads over columns.
__global__ void __launch_bounds__(256) k_splitk_reduce(TcArgs a, long long prows) {
    int lo = 0, hi = 0x7fffffff;
    if (a.mode == 1) {
        lo = a.offsets[0];
        hi = a.offsets[a.groups];
    }
    const bool vec = (a.N % 4) == 0;
    for (long long prow = blockIdx.x; prow < prows; prow += gridDim.x) {
        if (prow < lo || prow >= hi) continue;
        long long obase;
        if (a.mode == 2) {
            long long g = prow / a.M, row = prow - g * a.M;
            obase = g * a.c_group_stride + row * a.ldc;
        } else {
            obase = prow * a.ldc;
        }
        const float* src = a.part + prow * a.N;
        const int step = vec ? 4 : 1;
        for (int col = threadIdx.x * step; col < a.N; col += blockDim.x * step) {
            float v[4];
            int nv = vec ? 4 : 1;
            if (vec) {
                float4 t = *(const float4*)(src + col);
                v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
                for (int k = 1; k < a.ksplit; ++k) {
                    float4 u = *(const float4*)(src + (long long)k * a.c_group_stride_part + col);
                    v[0] += u.x; v[1] += u.y; v[2] += u.z; v[3] += u.w;
                }
            } else {
                v[0] = src[col];
                for (int k = 1; k < a.ksplit; ++k) v[0] += src[(long long)k * a.c_group_stride_part + col];
            }
            for (int j = 0; j < nv; ++j) {
                float x = v[j];
                long long off = obase + col + j;
                if (a.bias) x += a.bias[col + j];
                if (a.resid) x += a.resid[off];
                if (a.c_bf16) {
                    bf16* p = (bf16*)a.C + off;
                    if (a.accumulate) x += __bfloat162float(*p);
                    *p = __float2bfloat16_rn(act_apply(x, a.act));
                } else {
                    float* p = (float*)a.C + off;
                    if (a.accumulate) x += *p;
                    *p = act_apply(x, a.act);
                }
            }
        }
    }
}

// ------------------------------------------------------------------ host

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        CUDA_OK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
        CATNN_CHECK(p && q == cudaDriverEntryPointSuccess, CATNN_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
        fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    }
    return fn;
}

// 2-D bf16 map over a row-major [rows, cols] matrix with leading dimension
// ld (elements), box [box_cols (inner, 64 = 128 B), box_rows], 128B swizzle.
static CUtensorMap make_map(const void* base, i64 rows, i64 cols, i64 ld, int box_cols, int box_rows, bool f32 = false) {
    CUtensorMap m;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * (f32 ? 4 : 2))};
    cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn()(&m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                             const_cast<void*>(base), dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    CATNN_CHECK(r == CUDA_SUCCESS, CATNN_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    return m;
}

// Store map of the epilogue: [rows, cols] with leading dimension ld, boxes
// of 32 rows x 64 bytes (32 bf16 or 16 fp32 columns), 64-byte swizzle — the
// layout the epilogue's staging writes follow.
static CUtensorMap make_store_map(const void* base, i64 rows, i64 cols, i64 ld, bool fp32) {
    CUtensorMap m;
    const int es = fp32 ? 4 : 2;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * es)};
    cuuint32_t box[2] = {fp32 ? 16u : 32u, 32u};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn()(&m, fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                             const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             CU_TENSOR_MAP_SWIZZLE_64B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    CATNN_CHECK(r == CUDA_SUCCESS, CATNN_ERR_CUDA, "cuTensorMapEncodeTiled (store) failed (" + std::to_string((int)r) + ")");
    return m;
}

// Shared with the tensor-core attention kernels: a 2-D bf16 load map with
// 128-byte swizzle over a row-major [rows, cols] matrix (leading dimension ld).
CUtensorMap tma_map_bf16(const void* base, i64 rows, i64 cols, i64 ld, int box_cols, int box_rows) {
    return make_map(base, rows, cols, ld, box_cols, box_rows);
}

template <bool A_MN, bool B_MN, int BN, int STAGES, bool TF32 = false>
static void launch_tc(Context* c, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc,
                      const CUtensorMap& md, const TcArgs& a, int grid) {
    constexpr size_t smem = (size_t)STAGES * (BM * BK * 2 + BN * BK * 2) + EPI_STAGE_BYTES + 1024 + 256;
    static_assert(smem <= 232448, "shared memory per CTA");
    static bool attr_set[64] = {false};
    int dev = c->device;
    if (!attr_set[dev]) {
        CUDA_OK(cudaFuncSetAttribute(k_gemm_tc<A_MN, B_MN, BN, STAGES, TF32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem));
        attr_set[dev] = true;
    }
    k_gemm_tc<A_MN, B_MN, BN, STAGES, TF32><<<grid, GEMM_THREADS, smem, c->stream>>>(ma, mb, mc, md, a);
    launched(c);
}

template <int BN, int STAGES>
static void dispatch_tc(Context* c, bool a_mn, bool b_mn, const CUtensorMap& ma, const CUtensorMap& mb,
                        const CUtensorMap& mc, const CUtensorMap& md, const TcArgs& a, int grid) {
    if (!a_mn && !b_mn) launch_tc<false, false, BN, STAGES>(c, ma, mb, mc, md, a, grid);
    else if (!a_mn && b_mn) launch_tc<false, true, BN, STAGES>(c, ma, mb, mc, md, a, grid);
    else if (a_mn && !b_mn) launch_tc<true, false, BN, STAGES>(c, ma, mb, mc, md, a, grid);
    else launch_tc<true, true, BN, STAGES>(c, ma, mb, mc, md, a, grid);
}

static bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

// K slices for a launch of `tiles` BM x BN output tiles over a K range of
// klen, writing part_elems outputs: only when the tiles leave SMs idle. The
// count minimises an estimate of the time — tile waves x (tile FLOPs / s) at
// a per-SM rate of 4 TFLOP/s, plus for s > 1 the fp32 partials' round trip
// through HBM (5 TB/s) and the reduction launch. Slices are multiples of BK.
static int pick_ksplit(Context* c, i64 tiles, i64 klen, i64 part_elems, int BN, int* kchunk) {
    *kchunk = 0;
    if (tiles <= 0 || tiles >= c->sm_count || klen < 4 * BK) return 1;
    const double sm_rate = 4e12, hbm = 5e12, launch = 3e-6;
    auto cost = [&](int s) {
        double t = (double)cdiv(tiles * s, c->sm_count) * (2.0 * BM * BN * (double)klen / s) / sm_rate;
        if (s > 1) t += ((double)s * part_elems * 8 + (double)part_elems * 4) / hbm + launch;
        return t;
    };
    int best = 1;
    double best_cost = cost(1);
    for (int s = 2; s <= 16 && (i64)s * 2 * BK <= klen; ++s) {
        double t = cost(s);
        if (t < best_cost * 0.97) {
            best_cost = t;
            best = s;
        }
    }
    if (best > 1) {
        i64 ch = cdiv(cdiv(klen, best), BK) * BK;
        *kchunk = (int)ch;
        best = (int)cdiv(klen, ch);
    }
    return best;
}

// Builds both maps for op(A) [M(or rows), K] and op(B) [K, N] and launches.
// part_rows: rows of one split-K partial slice (0: no split-K).
// Output tile width of a plain GEMM: 256 columns, unless even one wave of
// 128 x 256 tiles leaves SMs idle and the 128 x 128 tiles still fit in one
// wave (then twice as many SMs work; split-K, pick_ksplit, is chosen on top
// for that width). Measured at 2048 rows on B200: x·W_o (2048 x 1024 x 1024)
// 10.8 -> 9.8 us, the QKV dgrad (2048 x 1024 x 3072) 22.9 -> 19.4 us; with
// more tiles than SMs the 128-column tiles lost (QKV forward, 192 tiles:
// 16.5 -> 19.7 us), so the rule stops there.
static int pick_bn(Context* c, i64 M, i64 N) {
    if (N <= 128) return 128;
    const i64 sms = c->sm_count;
    const i64 t256 = cdiv(M, BM) * cdiv(N, 256), t128 = cdiv(M, BM) * cdiv(N, 128);
    return t256 < sms && t128 <= sms ? 128 : 256;
}

static void run_tc(Context* c, TcArgs a, bool a_mn, bool b_mn, const void* A, i64 a_rows, i64 a_cols, i64 lda,
                   const void* B, i64 b_rows, i64 b_cols, i64 ldb, int grid_bound, i64 base_tiles = 0,
                   i64 klen = 0, i64 part_rows = 0, bool tf32 = false, int bn = 0) {
    const int BN = bn ? bn : (a.N <= 128 ? 128 : 256);
    // a box row is one 128-byte swizzle row: 64 bf16 or 32 fp32 elements of K
    const int kbox = tf32 ? 32 : 64;
    CUtensorMap ma = make_map(A, a_rows, a_cols, lda, kbox, a_mn ? 64 : BM, tf32);
    CUtensorMap mb = make_map(B, b_rows, b_cols, ldb, kbox, b_mn ? 64 : BN, tf32);
    a.status = c->status;
    a.ksplit = 1;
    if (part_rows > 0) {
        int kchunk = 0;
        int ks = pick_ksplit(c, base_tiles, klen, part_rows * a.N, BN, &kchunk);
        if (ks > 1) {
            a.ksplit = ks;
            a.kchunk = kchunk;
            a.c_group_stride_part = part_rows * a.N;
            a.part = (float*)c->scratch_for((size_t)ks * part_rows * a.N * 4);
            grid_bound = (int)std::min<i64>((i64)grid_bound * ks, (i64)c->sm_count);
        }
    }
    // output map for the plain epilogue's TMA stores (C as one 2-D [rows, N] matrix)
    CUtensorMap mc, md;
    std::memset(&mc, 0, sizeof(mc));
    std::memset(&md, 0, sizeof(md));
    a.tma_c = 0;
    if (a.epi != 0) {
        // SwiGLU epilogues: C is [rows, 2F] (epi 1: [a | c]; epi 2: [da | dc]),
        // and epi 1 also stores h [rows, F] through md
        const i64 F = a.epi == 1 ? a.N / 2 : a.N;
        if (aligned16(a.C) && (a.ldc * 2) % 16 == 0 && a.M < (1 << 30) &&
            (a.epi == 2 || (aligned16(a.aux) && (a.ldaux * 2) % 16 == 0))) {
            mc = make_store_map(a.C, a.M, 2 * F, a.ldc, false);
            if (a.epi == 1) md = make_store_map(a.aux, a.M, F, a.ldaux, false);
            a.tma_c = 1;
        }
    } else {
        const int es = a.c_bf16 ? 2 : 4;
        const i64 crows = a.mode == 2 ? (i64)a.groups * a.M : (i64)a.M;
        // residual rows are read with 16-byte loads in the staged epilogue
        if (!a.accumulate && aligned16(a.resid) && a.ksplit <= 1 && aligned16(a.C) && (a.ldc * es) % 16 == 0 && a.N >= 32 &&
            (a.mode != 2 || a.c_group_stride == (long long)a.M * a.ldc) && crows < (1ll << 31)) {
            mc = make_store_map(a.C, crows, a.N, a.ldc, !a.c_bf16);
            a.tma_c = 1;
        }
    }
    int grid = grid_bound < c->sm_count ? grid_bound : c->sm_count;
    if (grid < 1) grid = 1;
    if (tf32) {
        CATNN_CHECK(!a_mn && !b_mn, CATNN_ERR_UNSUPPORTED, "tf32 gemm: operands must be K-major");
        if (BN == 128) launch_tc<false, false, 128, 6, true>(c, ma, mb, mc, md, a, grid);
        else launch_tc<false, false, 256, 4, true>(c, ma, mb, mc, md, a, grid);
    } else if (BN == 128) {
        dispatch_tc<128, 6>(c, a_mn, b_mn, ma, mb, mc, md, a, grid);
    } else {
        dispatch_tc<256, 4>(c, a_mn, b_mn, ma, mb, mc, md, a, grid);
    }
    if (a.ksplit > 1) {
        int g = (int)std::min<i64>(part_rows, (i64)c->sm_count * 16);
        k_splitk_reduce<<<g, 256, 0, c->stream>>>(a, part_rows);
        launched(c);
    }
}

// Shapes the TMA path accepts: 16-byte aligned bases and row pitches.
static bool tc_ok(const void* A, i64 lda, const void* B, i64 ldb) {
    return aligned16(A) && aligned16(B) && (lda % 8) == 0 && (ldb % 8) == 0;
}

void gemm_bf16_simt(Context* c, bool ta, bool tb, i64 M, i64 N, i64 K, const bf16* A, i64 lda, const bf16* B, i64 ldb,
                    void* C, i64 ldc, int c_dtype, const float* bias, int act, bool accumulate, const float* resid);

// out[c][r] = in[r][c] for an fp32 [rows, cols] matrix with leading dimension
// ld (out is [cols, rows], dense): 32 x 32 tiles through shared memory.
__global__ void __launch_bounds__(256) k_transpose_f32(const float* __restrict__ in, i64 rows, i64 cols, i64 ld,
                                                       float* __restrict__ out) {
    __shared__ float t[32][33];
    const i64 r0 = (i64)blockIdx.y * 32, c0 = (i64)blockIdx.x * 32;
    for (int i = threadIdx.y; i < 32; i += 8) {
        const i64 r = r0 + i, cc = c0 + threadIdx.x;
        t[i][threadIdx.x] = r < rows && cc < cols ? in[r * ld + cc] : 0.f;
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += 8) {
        const i64 cc = c0 + i, r = r0 + threadIdx.x;
        if (cc < cols && r < rows) out[cc * rows + r] = t[threadIdx.x][i];
    }
}

static void transpose_f32(Context* c, const float* in, i64 rows, i64 cols, i64 ld, float* out) {
    CATNN_CHECK(cdiv(rows, 32) <= 65535, CATNN_ERR_SHAPE, "transpose: too many rows");
    k_transpose_f32<<<dim3((unsigned)cdiv(cols, 32), (unsigned)cdiv(rows, 32)), dim3(32, 8), 0, c->stream>>>(in, rows, cols,
                                                                                                          ld, out);
    launched(c);
}

// C = op(A)·op(B) with fp32 operands multiplied on the tensor cores as TF32
// (kind::tf32: 10-bit mantissas, fp32 accumulation). The MMA reads both
// operands K-major, so a transposed-layout operand (A stored [K, M] or B
// stored [K, N]) is first copied K-major into the context's work arena.
// Shapes the TMA path cannot take (pitches not a multiple of 4 elements,
// N or K under 16, tiny products) run the fp32 CUDA-core GEMM instead.
void gemm_tf32_tc(Context* c, bool ta, bool tb, i64 M, i64 N, i64 K, const float* A, i64 lda, const float* B, i64 ldb,
                  void* C, i64 ldc, int c_dtype, const float* bias, int act, bool accumulate) {
    if (M <= 0 || N <= 0) return;
    CATNN_CHECK(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), CATNN_ERR_SHAPE, "gemm: dimension too large");
    const bool copy = ta || !tb;  // an operand stored MN-major is first copied K-major (pitch K)
    if (N < 16 || K < 16 || M * N < 128 * 64 || (lda % 4) || (ldb % 4) || (copy && K % 4) || !aligned16(A) ||
        !aligned16(B)) {
        gemm_f32(c, ta, tb, M, N, K, A, lda, B, ldb, C, ldc, c_dtype, bias, act, accumulate);
        return;
    }
    const float* Ak = A;
    const float* Bk = B;
    i64 lak = lda, lbk = ldb;
    if (copy) {
        const size_t na = ta ? (size_t)M * K : 0, nb = !tb ? (size_t)N * K : 0;
        Carver cv(c->work_for(Carver::need({na * 4, nb * 4})));
        if (ta) {
            float* t = cv.take<float>(na);
            transpose_f32(c, A, K, M, lda, t);  // A [K, M] -> [M, K]
            Ak = t;
            lak = K;
        }
        if (!tb) {
            float* t = cv.take<float>(nb);
            transpose_f32(c, B, K, N, ldb, t);  // B [K, N] -> [N, K]
            Bk = t;
            lbk = K;
        }
    }
    TcArgs a{};
    a.mode = 0;
    a.groups = 1;
    a.M = (int)M;
    a.N = (int)N;
    a.K = (int)K;
    a.C = C;
    a.ldc = ldc;
    a.c_bf16 = c_dtype == CATNN_BF16;
    a.vec_ok = aligned16(C) && ((ldc * (a.c_bf16 ? 2 : 4)) % 16 == 0);
    a.bias = bias;
    a.act = act;
    a.accumulate = accumulate ? 1 : 0;
    const int BN = pick_bn(c, M, N);
    int tiles = cdiv(M, BM) * cdiv(N, BN);
    run_tc(c, a, false, false, Ak, M, K, lak, Bk, N, K, lbk, tiles, tiles, K, M, true, BN);
}

void gemm_bf16_tc(Context* c, bool ta, bool tb, i64 M, i64 N, i64 K, const bf16* A, i64 lda, const bf16* B, i64 ldb,
                  void* C, i64 ldc, int c_dtype, const float* bias, int act, bool accumulate, const float* resid) {
    if (M <= 0 || N <= 0) return;
    // Tiny or unaligned problems (e.g. the router's N = E) use the CUDA-core kernel.
    if (N < 16 || K < 16 || !tc_ok(A, lda, B, ldb) || M * N < 128 * 64) {
        gemm_bf16_simt(c, ta, tb, M, N, K, A, lda, B, ldb, C, ldc, c_dtype, bias, act, accumulate, resid);
        return;
    }
    CATNN_CHECK(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), CATNN_ERR_SHAPE, "gemm: dimension too large");
    TcArgs a{};
    a.mode = 0;
    a.groups = 1;
    a.M = (int)M;
    a.N = (int)N;
    a.K = (int)K;
    a.C = C;
    a.ldc = ldc;
    a.c_bf16 = c_dtype == CATNN_BF16;
    a.vec_ok = aligned16(C) && ((ldc * (a.c_bf16 ? 2 : 4)) % 16 == 0);
    a.bias = bias;
    a.resid = resid;
    a.act = act;
    a.accumulate = accumulate ? 1 : 0;
    const int BN = pick_bn(c, M, N);
    int tiles = cdiv(M, BM) * cdiv(N, BN);
    // op(A): ta=0 -> A [M,K] K-major; ta=1 -> A [K,M] MN-major.
    // op(B): tb=1 -> B [N,K] K-major; tb=0 -> B [K,N] MN-major.
    run_tc(c, a, ta, !tb, A, ta ? K : M, ta ? M : K, lda, B, tb ? N : K, tb ? K : N, ldb, tiles, tiles, K, M, false,
           BN);
}

void gemm_grouped_bf16_tc(Context* c, bool tb, i64 total_rows, i64 N, i64 K, int groups, const int32_t* offsets,
                          const bf16* A, i64 lda, const bf16* B, i64 strideB, i64 ldb, void* C, i64 ldc, int c_dtype,
                          int act, bool accumulate) {
    if (total_rows <= 0 || N <= 0 || groups <= 0) return;
    CATNN_CHECK(tc_ok(A, lda, B, ldb) && N >= 16 && K >= 16, CATNN_ERR_UNSUPPORTED,
                "grouped gemm: operands must be 16-byte aligned with N, K >= 16");
    // Expert matrices must be stacked contiguously: one 2-D map spans them.
    CATNN_CHECK(strideB == (tb ? N : K) * ldb, CATNN_ERR_SHAPE, "grouped gemm: B groups must be contiguous");
    TcArgs a{};
    a.mode = 1;
    a.groups = groups;
    a.offsets = offsets;
    a.M = (int)total_rows;
    a.N = (int)N;
    a.K = (int)K;
    a.b_group_rows = (int)(tb ? N : K);
    a.C = C;
    a.ldc = ldc;
    a.c_bf16 = c_dtype == CATNN_BF16;
    a.vec_ok = aligned16(C) && ((ldc * (a.c_bf16 ? 2 : 4)) % 16 == 0);
    a.act = act;
    a.accumulate = accumulate ? 1 : 0;
    const int BN = N <= 128 ? 128 : 256;
    int bound = (cdiv(total_rows, BM) + groups) * cdiv(N, BN);
    // the tile count depends on the device offsets: the split is sized for
    // the host-side bound of the rows
    run_tc(c, a, false, !tb, A, total_rows, K, lda, B, (i64)groups * (tb ? N : K), tb ? K : N, ldb, bound,
           cdiv(total_rows, BM) * cdiv(N, BN), K, total_rows);
}

void gemm_grouped_wgrad_bf16_tc(Context* c, i64 total_rows, i64 N, i64 K, int groups, const int32_t* offsets,
                                const bf16* A, i64 lda, const bf16* D, i64 ldd, void* dB, i64 strideB, int c_dtype,
                                bool accumulate) {
    if (N <= 0 || K <= 0 || groups <= 0) return;
    CATNN_CHECK(tc_ok(A, lda, D, ldd) && N >= 16 && K >= 16, CATNN_ERR_UNSUPPORTED,
                "grouped wgrad: operands must be 16-byte aligned with N, K >= 16");
    TcArgs a{};
    a.mode = 2;
    a.groups = groups;
    a.offsets = offsets;
    a.M = (int)K;  // output rows = A's width
    a.N = (int)N;
    a.K = 0;
    a.C = dB;
    a.ldc = N;
    a.c_group_stride = strideB;
    a.c_bf16 = c_dtype == CATNN_BF16;
    a.vec_ok = aligned16(dB) && ((N * (a.c_bf16 ? 2 : 4)) % 16 == 0);
    a.accumulate = accumulate ? 1 : 0;
    const int BN = N <= 128 ? 128 : 256;
    int tiles = groups * cdiv(K, BM) * cdiv(N, BN);
    // A_g: rows of X [rows, K] read MN-major (M = K); D_g: rows of [rows, N] read MN-major.
    // Split-K slices each group's rows; the chunk is sized for the mean group.
    run_tc(c, a, true, true, A, total_rows, K, lda, D, total_rows, N, ldd, tiles, tiles, cdiv(total_rows, groups),
           (i64)groups * K);
}

// MoE expert forward with the SwiGLU fused into the epilogue: per expert g,
// AC[rows_g] = X[rows_g]·W13_g with W13_g [K, 2F] in the 128-column
// interleaved [a | c] layout (TcArgs::epi), and H[rows_g] = silu(a)·c.
void gemm_grouped_swiglu_fwd_tc(Context* c, i64 total_rows, i64 F, i64 K, int groups, const int32_t* offsets,
                                const bf16* X, i64 ldx, const bf16* W13, bf16* AC, bf16* H) {
    if (total_rows <= 0 || groups <= 0) return;
    CATNN_CHECK(F % 128 == 0 && K >= 16 && tc_ok(X, ldx, W13, 2 * F), CATNN_ERR_UNSUPPORTED,
                "swiglu gemm: F must be a multiple of 128, K >= 16, operands 16-byte aligned");
    TcArgs a{};
    a.mode = 1;
    a.groups = groups;
    a.offsets = offsets;
    a.M = (int)total_rows;
    a.N = (int)(2 * F);
    a.K = (int)K;
    a.b_group_rows = (int)K;
    a.C = AC;
    a.ldc = 2 * F;
    a.c_bf16 = 1;
    a.vec_ok = 1;
    a.epi = 1;
    a.aux = H;
    a.ldaux = F;
    int bound = (cdiv(total_rows, BM) + groups) * cdiv(2 * F, 256);
    run_tc(c, a, false, true, X, total_rows, K, ldx, W13, (i64)groups * K, 2 * F, 2 * F, bound);
}

// MoE expert backward through the SwiGLU: per expert g, dh = dY[rows_g]·W2_gᵀ
// (W2_g [F, K] row-major, read K-major) is never stored; the epilogue reads a,
// c from AC (interleaved layout) and writes DAC = [da | dc] in that layout.
void gemm_grouped_swiglu_bwd_tc(Context* c, i64 total_rows, i64 F, i64 K, int groups, const int32_t* offsets,
                                const bf16* DY, i64 lddy, const bf16* W2, const bf16* AC, bf16* DAC) {
    if (total_rows <= 0 || groups <= 0) return;
    CATNN_CHECK(F % 128 == 0 && K >= 16 && tc_ok(DY, lddy, W2, K) && aligned16(AC), CATNN_ERR_UNSUPPORTED,
                "swiglu gemm: F must be a multiple of 128, K >= 16, operands 16-byte aligned");
    TcArgs a{};
    a.mode = 1;
    a.groups = groups;
    a.offsets = offsets;
    a.M = (int)total_rows;
    a.N = (int)F;
    a.K = (int)K;
    a.b_group_rows = (int)F;
    a.C = DAC;
    a.ldc = 2 * F;
    a.c_bf16 = 1;
    a.vec_ok = 1;
    a.epi = 2;
    a.aux = const_cast<bf16*>(AC);
    a.ldaux = 2 * F;
    const int BN = F <= 128 ? 128 : 256;
    int bound = (cdiv(total_rows, BM) + groups) * cdiv(F, BN);
    run_tc(c, a, false, false, DY, total_rows, K, lddy, W2, (i64)groups * F, K, K, bound);
}

// linear / matmul / moe: A K-major, weights [in, out] (MN-major); lm_head:
// table [vocab, hidden] (K-major). Persistent grid: one CTA per SM at most.
KernelInfo gemm_tc_info(Context* c, const std::string& op, const KShape& s) {
    KernelInfo k;
    const bool lm = op == "lm_head";
    if (!(lm || op == "linear" || op == "matmul" || op == "moe")) return k;
    const bool big = s.width > 128;
    if (big) k.fn = lm ? (const void*)k_gemm_tc<false, false, 256, 4> : (const void*)k_gemm_tc<false, true, 256, 4>;
    else k.fn = lm ? (const void*)k_gemm_tc<false, false, 128, 6> : (const void*)k_gemm_tc<false, true, 128, 6>;
    const int BN = big ? 256 : 128, ST = big ? 4 : 6;
    k.file = "gemm_tc.cu";
    const i64 tiles = (i64)cdiv(s.rows, BM) * cdiv(s.width, BN);
    k.grid[0] = (unsigned)std::max<i64>(1, std::min<i64>(tiles, c->sm_count));
    k.block[0] = GEMM_THREADS;
    k.dyn_smem = (size_t)ST * (BM * BK * 2 + BN * BK * 2) + EPI_STAGE_BYTES + 1024 + 256;
    return k;
}

}  // namespace catnn
