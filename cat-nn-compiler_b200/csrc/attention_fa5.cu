// Causal / windowed GQA attention forward on the 5th-generation tensor
// cores (tcgen05 + TMEM, TMA-fed), head_dim 64, bf16 in, fp32 softmax.
//
// One CTA = 128 queries of one (sequence, head); 192 threads:
//   warp 0      TMA producer: the Q tile once, then K and V blocks of 64
//               keys into a 3-deep ring (64-key blocks: two CTAs fit an SM)
//   warp 1      TMEM owner + MMA issuer (one thread):
//                 S_j = Q·K_jᵀ      128 x 64, fp32 in TMEM (2 buffers)
//                 O_j = P_j·V_j     128 x 64,  fp32 in TMEM (2 buffers)
//   warps 2..5  softmax: thread = query row; reads S_j from TMEM, masks,
//               updates the running max / sum (log2 domain, the reference's
//               max-subtracted softmax, moe.rs:105-121 via cpu.rs:31-52),
//               writes P_j (bf16) to shared memory in the MMA's A-operand
//               layout, and folds O_{j-1} into its fp32 row accumulator one
//               block late so that the P·V MMA of block j overlaps the
//               softmax of block j+1.
// The output and the log-sum-exp (natural log, per row) follow the
// convention of the mma.sync kernels in attention_tc.cu, whose backward
// consumes them. Every wait is bounded (tc::mbar_wait).
#include "ops.cuh"
#include "tc_prims.cuh"

namespace catnn {
namespace fa5 {

constexpr int BQ = 128, BKV = 64, HD = 64, ST = 3, NT = 192;
constexpr float LOG2E = 1.4426950408889634f;
constexpr uint32_t Q_BYTES = BQ * HD * 2;        // 16 KB
constexpr uint32_t KV_BYTES = BKV * HD * 2;      // 8 KB each for K and V
constexpr uint32_t STAGE_BYTES = 2 * KV_BYTES;   // K then V
constexpr uint32_t P_BYTES = BQ * BKV * 2;       // 16 KB (one 64-key atom)
constexpr uint32_t TMEM_COLS = 256;              // S: 2 x 64, O: 64 (two CTAs per SM)
constexpr uint32_t S_COL = 0, O_COL = 128;
constexpr size_t SMEM = Q_BYTES + ST * STAGE_BYTES + 2 * P_BYTES + 1024 + 512;

struct Args {
    int b, s, h, hkv;
    int causal, window;
    float scale;
    bf16* out;     // [B*S, H*64]
    float* lse;    // [B, H, S]
    int* status;
};

// 2^x with the MUFU instruction (ex2.approx.ftz: relative error ~2^-22,
// far below the bf16 rounding of P); 2^-inf = 0.
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ int klo(const Args& a, int i) {
    if (!a.causal || a.window <= 0) return 0;
    int l = i - a.window + 1;
    return l > 0 ? l : 0;
}
__device__ __forceinline__ int khi(const Args& a, int i) { return a.causal ? i : a.s - 1; }

// Packed fp32 pairs (sm_100 f32x2 instructions: two lanes of work per issue slot).
__device__ __forceinline__ unsigned long long pk2(float a, float b) {
    return ((unsigned long long)__float_as_uint(b) << 32) | __float_as_uint(a);
}
__device__ __forceinline__ unsigned long long fma2(unsigned long long a, unsigned long long b, unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ unsigned long long add2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ float lo2(unsigned long long v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float hi2(unsigned long long v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ float max3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// 2^x on the FMA pipe, for a share of the exponentials so that the MUFU unit
// (16 results per clock per SM, the forward's bound at head_dim 64) does
// not carry all of them. Round-to-nearest split x = n + f (adding 1.5·2^23
// leaves n in the low mantissa bits), f in [-0.5, 0.5], 2^f by a degree-3
// polynomial fitted here to minimise the relative error on that interval
// (at most 7.5e-5, against bf16's 2^-9 rounding of P), and 2^n added into
// the exponent field. x is clamped at -126 (the result is then at most
// 2^-126: subnormal or the least normal, i.e. zero to every later use).
__device__ __forceinline__ float ex2_fma(float x) {
    constexpr float C0 = 0.99992806f, C1 = 0.69326097f, C2 = 0.24261113f, C3 = 0.055171665f;
    x = fmaxf(x, -126.f);
    const float t = x + 12582912.f;
    const float f = x - (t - 12582912.f);
    const float p = fmaf(fmaf(fmaf(C3, f, C2), f, C1), f, C0);
    return __int_as_float(__float_as_int(p) + ((__float_as_int(t) - 0x4B400000) << 23));
}

// The running max a row's exponentials are taken against is only moved up
// (and O, l rescaled) when a block's max exceeds it by more than this (log2
// units): P then stays below 2^8, and the rescale — a TMEM read-modify-write
// of the row's O — is rare after the first blocks.
constexpr float RESCALE_LOG2 = 8.f;

__global__ void __launch_bounds__(NT, 2)
    k_fwd(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
          const __grid_constant__ CUtensorMap mv, Args a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sQ = smem;
    uint8_t* sKV = sQ + Q_BYTES;
    uint8_t* sP = sKV + ST * STAGE_BYTES;
    uint64_t* bars = (uint64_t*)(sP + 2 * P_BYTES);
    uint64_t* q_full = bars;
    uint64_t* kv_full = q_full + 1;
    uint64_t* kv_empty = kv_full + ST;
    uint64_t* s_full = kv_empty + ST;
    uint64_t* s_free = s_full + 2;
    uint64_t* p_full = s_free + 2;
    uint64_t* o_done = p_full + 2;  // P_j·V_j accumulated into O (and P buffer j&1 read)
    uint64_t* drain = o_done + 2;
    uint32_t* tmem_slot = (uint32_t*)(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // heaviest (latest) query tiles first
    // the block's weight is the slowest grid index, heaviest (latest) query
    // tiles first over every head and sequence: the longest CTAs start in
    // the first wave
    const int qt = gridDim.z - 1 - blockIdx.z;
    const int q0 = qt * BQ, h = blockIdx.x, bi = blockIdx.y;
    const int kvh = h / (a.h / a.hkv);
    const int qlast = min(q0 + BQ - 1, a.s - 1);
    const int j0 = klo(a, q0) / BKV, j1 = min(khi(a, qlast), a.s - 1) / BKV;
    const int nblk = j1 - j0 + 1;

    if (threadIdx.x == 0) {
        tc::mbar_init(q_full, 1);
        for (int i = 0; i < ST; ++i) {
            tc::mbar_init(&kv_full[i], 1);
            tc::mbar_init(&kv_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&s_full[i], 1);
            tc::mbar_init(&s_free[i], 4);
            tc::mbar_init(&p_full[i], 4);
            tc::mbar_init(&o_done[i], 1);
        }
        tc::mbar_init(drain, 1);
        tc::fence_mbar_init();
        tc::prefetch_tmap(&mq);
        tc::prefetch_tmap(&mk);
        tc::prefetch_tmap(&mv);
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, TMEM_COLS);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const long long seq_row = (long long)bi * a.s;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer
            tc::mbar_arrive_expect_tx(q_full, Q_BYTES);
            tc::tma_load_2d(sQ, &mq, h * HD, (int)(seq_row + q0), q_full);
            int last_ph[ST];
            for (int i = 0; i < ST; ++i) last_ph[i] = -1;
            bool ok = true;
            for (int j = 0; j < nblk && ok; ++j) {
                const int st = j % ST;
                const uint32_t ph = (j / ST) & 1;
                if (!tc::mbar_wait(&kv_empty[st], ph ^ 1, a.status, 4)) {
                    ok = false;
                    break;
                }
                uint8_t* sK = sKV + st * STAGE_BYTES;
                tc::mbar_arrive_expect_tx(&kv_full[st], STAGE_BYTES);
                const int krow = (int)(seq_row + (long long)(j0 + j) * BKV);
                tc::tma_load_2d(sK, &mk, kvh * HD, krow, &kv_full[st]);
                tc::tma_load_2d(sK + KV_BYTES, &mv, kvh * HD, krow, &kv_full[st]);
                last_ph[st] = (int)ph;
            }
            if (!ok) {
                // let the copies in flight land before the CTA exits
                tc::mbar_wait(q_full, 0, a.status, 4, 400000000ll, false);
                for (int i = 0; i < ST; ++i)
                    if (last_ph[i] >= 0) tc::mbar_wait(&kv_full[i], (uint32_t)last_ph[i], a.status, 4, 400000000ll, false);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer
            constexpr uint32_t IDS = tc::idesc_bf16(BQ, BKV, false, false);  // S = Q·Kᵀ (K-major both)
            constexpr uint32_t IDO = tc::idesc_bf16(BQ, HD, false, true);    // O += P·V (V MN-major)
            bool ok = tc::mbar_wait(q_full, 0, a.status, 4);
            const uint32_t aq = tc::smem_u32(sQ);
            auto issue_s = [&](int j) -> bool {
                const int st = j % ST, sb = j & 1;
                if (!tc::mbar_wait(&kv_full[st], (j / ST) & 1, a.status, 4)) return false;
                if (!tc::mbar_wait(&s_free[sb], ((j >> 1) & 1) ^ 1, a.status, 4)) return false;
                tc::tc_fence_after();
                const uint32_t bk = tc::smem_u32(sKV + st * STAGE_BYTES);
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk)
                    tc::mma_bf16(tmem + S_COL + sb * BKV, tc::sdesc(aq + kk * 32, 16, 1024),
                                 tc::sdesc(bk + kk * 32, 16, 1024), IDS, kk != 0);
                tc::mma_commit(&s_full[sb]);
                return true;
            };
            if (ok && nblk > 0) ok = issue_s(0);
            for (int j = 0; j < nblk && ok; ++j) {
                if (j + 1 < nblk && !issue_s(j + 1)) {
                    ok = false;
                    break;
                }
                const int st = j % ST, pb = j & 1;
                // P_j is in shared memory and O holds the (rescaled) blocks before j
                if (!tc::mbar_wait(&p_full[pb], (j >> 1) & 1, a.status, 4)) {
                    ok = false;
                    break;
                }
                tc::tc_fence_after();
                const uint32_t ap = tc::smem_u32(sP + pb * P_BYTES);
                const uint32_t bv = tc::smem_u32(sKV + st * STAGE_BYTES + KV_BYTES);
#pragma unroll
                for (int kk = 0; kk < BKV / 16; ++kk)
                    tc::mma_bf16(tmem + O_COL, tc::sdesc(ap + kk * 32, 16, 1024), tc::sdesc(bv + kk * 2048, 8192, 1024),
                                 IDO, (j | kk) != 0);
                tc::mma_commit(&o_done[pb]);
                tc::mma_commit(&kv_empty[st]);
            }
            tc::mma_commit(drain);
            tc::mbar_wait(drain, 0, a.status, 4, 400000000ll, false);
        }
    } else {
        // ---------------- softmax / output
        const int qd = warp & 3;  // TMEM lane quadrant this warp may read
        const int r = qd * 32 + lane;
        const int row = q0 + r;
        const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
        const uint32_t oa = tmem + lane_off + O_COL;
        const float sc = a.scale * LOG2E;
        const unsigned long long sc2 = pk2(sc, sc);
        const int lo = klo(a, row), hi = min(khi(a, row), a.s - 1);
        // m: the max the exponentials use (log2 units, scale folded in), l: Σ P
        float m = -INFINITY, l = 0.f;
        bool ok = nblk > 0;
        for (int j = 0; j < nblk && ok; ++j) {
            const int sb = j & 1;
            if (!tc::mbar_wait(&s_full[sb], (j >> 1) & 1, a.status, 4)) {
                ok = false;
                break;
            }
            tc::tc_fence_after();
            const int k0 = (j0 + j) * BKV;
            // masking only where some key of the block is outside [lo, hi] for some row
            const bool full = k0 >= klo(a, min(q0 + BQ - 1, a.s - 1)) && k0 + BKV - 1 <= min(khi(a, q0), a.s - 1);
            const uint32_t sa = tmem + lane_off + S_COL + sb * BKV;
            uint32_t v[64];
            {
                uint32_t (&v0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&v[0]);
                uint32_t (&v1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&v[32]);
                tc::tmem_ld32(sa, v0);
                tc::tmem_ld32(sa + 32, v1);
                tc::tmem_ld_wait();
            }
            // S_j is in registers: the MMA may overwrite its buffer
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&s_free[sb]);
            if (!full) {
#pragma unroll
                for (int i = 0; i < 64; ++i)
                    if (k0 + i < lo || k0 + i > hi) v[i] = __float_as_uint(-INFINITY);
            }
            // block max: four chains of three-input maxima
            float mxa[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int i = 0; i < 64; i += 8)
#pragma unroll
                for (int u = 0; u < 4; ++u) mxa[u] = max3(mxa[u], __uint_as_float(v[i + 2 * u]), __uint_as_float(v[i + 2 * u + 1]));
            // scale > 0: the max of the scaled scores is the scaled max
            const float mx = fmaxf(fmaxf(mxa[0], mxa[1]), fmaxf(mxa[2], mxa[3])) * sc;
            const bool grow = m != -INFINITY && mx > m + RESCALE_LOG2;
            if (m == -INFINITY) m = mx;  // nothing accumulated yet (O's rows, l are zero)
            if (__any_sync(0xffffffffu, grow)) {
                // O holds blocks < j (m != -inf implies j > 0): wait for P_{j-1}·V_{j-1}
                // to land, then scale the row by 2^(m_old - m_new)
                if (!tc::mbar_wait(&o_done[(j - 1) & 1], ((j - 1) >> 1) & 1, a.status, 4)) {
                    ok = false;
                    break;
                }
                tc::tc_fence_after();
                const float alpha = grow ? ex2(m - mx) : 1.f;
                if (grow) {
                    l *= alpha;
                    m = mx;
                }
#pragma unroll
                for (int c = 0; c < HD / 32; ++c) {
                    uint32_t o[32];
                    tc::tmem_ld32(oa + c * 32, o);
                    tc::tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tc::tmem_st32(oa + c * 32, o);
                }
                tc::tmem_st_wait();
            }
            // P buffer sb was last read by P_{j-2}·V_{j-2}
            if (j >= 2 && !tc::mbar_wait(&o_done[sb], ((j - 2) >> 1) & 1, a.status, 4)) {
                ok = false;
                break;
            }
            const float base = m == -INFINITY ? 0.f : m;
            const unsigned long long nb2 = pk2(-base, -base);
            unsigned long long ls2[4] = {0ull, 0ull, 0ull, 0ull};
            const uint32_t prow = tc::smem_u32(sP + sb * P_BYTES + r * 128);
            // P = 2^(s·scale - m) (masked scores are -inf: P = 0), row sums,
            // bf16 P to shared memory in 16-byte chunks
#pragma unroll
            for (int chunk = 0; chunk < BKV / 8; ++chunk) {
                float p[8];
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const unsigned long long x =
                        fma2(pk2(__uint_as_float(v[chunk * 8 + 2 * t]), __uint_as_float(v[chunk * 8 + 2 * t + 1])), sc2, nb2);
                    p[2 * t] = ex2(lo2(x));
                    // one exponential in four on the FMA pipe
                    p[2 * t + 1] = (t & 1) ? ex2_fma(hi2(x)) : ex2(hi2(x));
                    ls2[t] = add2(ls2[t], pk2(p[2 * t], p[2 * t + 1]));
                }
                uint4 pk;
                __nv_bfloat162* pp = (__nv_bfloat162*)&pk;
#pragma unroll
                for (int t = 0; t < 4; ++t) pp[t] = __floats2bfloat162_rn(p[2 * t], p[2 * t + 1]);
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(prow + ((chunk ^ (r & 7)) << 4)), "r"(pk.x),
                             "r"(pk.y), "r"(pk.z), "r"(pk.w)
                             : "memory");
            }
            const unsigned long long s01 = add2(ls2[0], ls2[1]), s23 = add2(ls2[2], ls2[3]), s4 = add2(s01, s23);
            l += lo2(s4) + hi2(s4);
            // P_j in shared memory (generic proxy) and any O rescale (tcgen05.st) before the MMA reads them
            tc::fence_proxy_async();
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&p_full[sb]);
        }
        // the last P·V has landed: O / l to global, and the natural-log lse
        if (ok && !tc::mbar_wait(&o_done[(nblk - 1) & 1], ((nblk - 1) >> 1) & 1, a.status, 4)) ok = false;
        if (ok) {
            tc::tc_fence_after();
            uint32_t o[64];
            {
                uint32_t (&o0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&o[0]);
                uint32_t (&o1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&o[32]);
                tc::tmem_ld32(oa, o0);
                tc::tmem_ld32(oa + 32, o1);
                tc::tmem_ld_wait();
            }
            if (row < a.s) {
                const float inv = l > 0.f ? 1.f / l : 0.f;
                bf16* op = a.out + (seq_row + row) * (long long)(a.h * HD) + h * HD;
#pragma unroll
                for (int c = 0; c < HD / 8; ++c) {
                    uint4 pk;
                    __nv_bfloat162* pp = (__nv_bfloat162*)&pk;
#pragma unroll
                    for (int t = 0; t < 4; ++t)
                        pp[t] = __floats2bfloat162_rn(__uint_as_float(o[c * 8 + 2 * t]) * inv,
                                                      __uint_as_float(o[c * 8 + 2 * t + 1]) * inv);
                    *(uint4*)(op + c * 8) = pk;
                }
                a.lse[((long long)bi * a.h + h) * a.s + row] = l > 0.f ? (m + log2f(l)) / LOG2E : -INFINITY;
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, TMEM_COLS);
    }
}

// ------------------------------------------------------------------ backward
// dS = P ⊙ (dP - D), D = rowsum(dO ⊙ O), P = 2^(S·scale·log2e - lse·log2e)
// (the adjoint of the max-subtracted softmax, adjoint.rs:92-104, inside the
// attention adjoint adjoint.rs:287-439). Two kernels, each deterministic:
//   k_dkdv  one CTA per 128 keys of a kv head; loops over the query blocks
//           of every head of its group: Sᵀ = K·Qᵀ, dPᵀ = V·dOᵀ (TMEM),
//           then dV += Pᵀ·dO and dK += dSᵀ·Q accumulate in TMEM.
//   k_dq    one CTA per 128 queries; loops over key blocks:
//           S = Q·Kᵀ, dP = dO·Vᵀ, dQ += dS·K in TMEM.
// The same shared-memory tile serves as a K-major B operand (for Qᵀ, dOᵀ,
// Kᵀ, Vᵀ) and as an MN-major B operand (for Q, dO, K): only the descriptor
// changes. P and dS are written by the compute threads in the A-operand
// layout (128-byte rows, 16-byte chunks XOR-swizzled by row).

constexpr int BB = 128;                          // the looped block (queries in k_dkdv, keys in k_dq)
// 8 compute warps: two per TMEM lane quadrant, each takes 64 of the block's
// 128 columns of its rows (the backward has no row reductions to combine)
constexpr int NTB = 320, NCW = 8, HALF = BB / 2;
constexpr uint32_t T128 = 128 * HD * 2;          // 16 KB: a 128-row tile of 64 bf16 (one 128-byte swizzle atom)
constexpr uint32_t TPD = 2 * T128;               // 32 KB: a 128 x 128 bf16 P / dS tile, two atoms of 64 columns
constexpr uint32_t QD_STAGE = 2 * T128 + 1024;   // Q, dO and the block's L[128], D[128]
constexpr int QS = 3;                            // Q/dO stages of k_dkdv
constexpr int KS = 3;                            // K/V stages of k_dq
constexpr size_t SMEM_DKDV = 2 * T128 + QS * QD_STAGE + 2 * TPD + 1024 + 512;
constexpr size_t SMEM_DQ = 2 * T128 + KS * 2 * T128 + 2 * TPD + 1024 + 512;

struct BwdArgs {
    int b, s, h, hkv;
    int causal, window;
    float scale;
    const float* lse;   // [B, H, S], natural log
    const float* dsum;  // [B, H, S]
    bf16 *dq, *dk, *dv;
    int q_stride, kv_stride;
    int* status;
};

__device__ __forceinline__ int bklo(const BwdArgs& a, int i) {
    if (!a.causal || a.window <= 0) return 0;
    int l = i - a.window + 1;
    return l > 0 ? l : 0;
}
__device__ __forceinline__ int bkhi(const BwdArgs& a, int i) { return a.causal ? i : a.s - 1; }
// queries that see key k: [qlo, qhi]
__device__ __forceinline__ int bqlo(const BwdArgs& a, int k) { return a.causal ? k : 0; }
__device__ __forceinline__ int bqhi(const BwdArgs& a, int k) {
    if (!a.causal) return a.s - 1;
    if (a.window <= 0) return a.s - 1;
    return min(a.s - 1, k + a.window - 1);
}

// 16-byte chunk `chunk` (8 bf16, columns 8·chunk..) of row r of a 128 x 128
// tile stored as two 128-byte-row swizzled atoms (columns 0-63, 64-127)
__device__ __forceinline__ void st_chunk8(uint32_t tile, int r, int chunk, const float (&x)[8]) {
    uint4 pk;
    __nv_bfloat162* pp = (__nv_bfloat162*)&pk;
#pragma unroll
    for (int t = 0; t < 4; ++t) pp[t] = __floats2bfloat162_rn(x[2 * t], x[2 * t + 1]);
    const uint32_t addr = tile + (chunk >> 3) * T128 + r * 128 + (((chunk & 7) ^ (r & 7)) << 4);
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(pk.x), "r"(pk.y), "r"(pk.z), "r"(pk.w)
                 : "memory");
}

// A operand descriptor for K-step kk of a 128 x 128 two-atom tile
__device__ __forceinline__ uint64_t a2desc(uint32_t tile, int kk) {
    return tc::sdesc(tile + (kk >> 2) * T128 + (kk & 3) * 32, 16, 1024);
}

// dK/dV: one CTA per 128 keys of a kv head; loops over the 128-query blocks
// of every head of its group. Per block: Sᵀ = K·Qᵀ and dPᵀ = V·dOᵀ (M 128
// keys, N 128 queries) into TMEM; the compute warps turn them into Pᵀ and
// dSᵀ (bf16, shared memory); dV += Pᵀ·dO and dK += dSᵀ·Q (K = 128 queries)
// accumulate in TMEM. Sᵀ/dPᵀ are single-buffered: the next block's products
// are issued as soon as the compute warps hold the current ones in registers.
__global__ void __launch_bounds__(NTB, 1)
    k_dkdv(const __grid_constant__ CUtensorMap mk, const __grid_constant__ CUtensorMap mv,
           const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mdo, BwdArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sK = smem;
    uint8_t* sV = sK + T128;
    uint8_t* sQD = sV + T128;           // QS stages: Q | dO | L[128] D[128]
    uint8_t* sP = sQD + QS * QD_STAGE;  // Pᵀ tile
    uint8_t* sDS = sP + TPD;            // dSᵀ tile
    uint64_t* bars = (uint64_t*)(sDS + TPD);
    uint64_t* kv_full = bars;
    uint64_t* qd_full = kv_full + 1;
    uint64_t* qd_empty = qd_full + QS;
    uint64_t* st_full = qd_empty + QS;
    uint64_t* st_free = st_full + 1;
    uint64_t* pd_full = st_free + 1;
    uint64_t* pd_free = pd_full + 1;
    uint64_t* acc_full = pd_free + 1;
    uint64_t* drain = acc_full + 1;
    uint32_t* tmem_slot = (uint32_t*)(drain + 1);
    // TMEM columns: Sᵀ 0..127, dPᵀ 128..255, dV 256..319, dK 320..383
    constexpr uint32_t C_S = 0, C_DP = 128, C_DV = 256, C_DK = 320;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // early keys see the most queries: the key block is the slowest grid
    // index, first key blocks first over every head and sequence
    const int kb = blockIdx.z;
    const int k0 = kb * 128, kvh = blockIdx.x, bi = blockIdx.y;
    const int grp = a.h / a.hkv;
    const int klast = min(k0 + 127, a.s - 1);
    const int qb0 = bqlo(a, k0) / BB, qb1 = bqhi(a, klast) / BB;
    const int nq = qb1 - qb0 + 1, n = grp * nq;
    const long long seq_row = (long long)bi * a.s;

    if (threadIdx.x == 0) {
        tc::mbar_init(kv_full, 1);
        for (int i = 0; i < QS; ++i) {
            tc::mbar_init(&qd_full[i], 1);
            tc::mbar_init(&qd_empty[i], 1);
        }
        tc::mbar_init(st_full, 1);
        tc::mbar_init(st_free, NCW);
        tc::mbar_init(pd_full, NCW);
        tc::mbar_init(pd_free, 1);
        tc::mbar_init(acc_full, 1);
        tc::mbar_init(drain, 1);
        tc::fence_mbar_init();
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, 512);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- producer (whole warp: lane 0 issues TMA, all lanes fill L and D)
        if (lane == 0) {
            tc::mbar_arrive_expect_tx(kv_full, 2 * T128);
            tc::tma_load_2d(sK, &mk, kvh * HD, (int)(seq_row + k0), kv_full);
            tc::tma_load_2d(sV, &mv, kvh * HD, (int)(seq_row + k0), kv_full);
        }
        uint32_t used = 0, last_par = 0;
        int ok = 1;
        for (int it = 0; it < n; ++it) {
            const int st = it % QS;
            const uint32_t ph = (it / QS) & 1;
            if (lane == 0) ok = tc::mbar_wait(&qd_empty[st], ph ^ 1, a.status, 4);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            const int h = kvh * grp + it / nq;
            const int q0 = (qb0 + it % nq) * BB;
            uint8_t* stg = sQD + st * QD_STAGE;
            float* sL = (float*)(stg + 2 * T128);
            float* sD = sL + 128;
            const long long lrow = ((long long)bi * a.h + h) * a.s;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int c = lane * 4 + u, q = q0 + c;
                sL[c] = q < a.s ? a.lse[lrow + q] * LOG2E : INFINITY;
                sD[c] = q < a.s ? a.dsum[lrow + q] : 0.f;
            }
            __syncwarp();
            if (lane == 0) {
                used |= 1u << st;
                last_par = (last_par & ~(1u << st)) | (ph << st);
                tc::mbar_arrive_expect_tx(&qd_full[st], 2 * T128);
                tc::tma_load_2d(stg, &mq, h * HD, (int)(seq_row + q0), &qd_full[st]);
                tc::tma_load_2d(stg + T128, &mdo, h * HD, (int)(seq_row + q0), &qd_full[st]);
            }
        }
        if (!ok && lane == 0) {
            // let the copies in flight land before the CTA exits
            tc::mbar_wait(kv_full, 0, a.status, 4, 400000000ll, false);
            for (int i = 0; i < QS; ++i)
                if ((used >> i) & 1u) tc::mbar_wait(&qd_full[i], (last_par >> i) & 1u, a.status, 4, 400000000ll, false);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer
            constexpr uint32_t ID_T = tc::idesc_bf16(128, BB, false, false);  // Sᵀ, dPᵀ
            constexpr uint32_t ID_A = tc::idesc_bf16(128, HD, false, true);   // dV, dK
            bool ok = tc::mbar_wait(kv_full, 0, a.status, 4);
            const uint32_t aK = tc::smem_u32(sK), aV = tc::smem_u32(sV);
            const uint32_t aP = tc::smem_u32(sP), aDS = tc::smem_u32(sDS);
            // Sᵀ, dPᵀ of block it, once the compute warps hold block it-1's in registers
            auto issue_st = [&](int it) -> bool {
                const int st = it % QS;
                if (!tc::mbar_wait(&qd_full[st], (it / QS) & 1, a.status, 4) ||
                    !tc::mbar_wait(st_free, (it & 1) ^ 1, a.status, 4))
                    return false;
                tc::tc_fence_after();
                const uint32_t bQ = tc::smem_u32(sQD + st * QD_STAGE), bO = bQ + T128;
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk)
                    tc::mma_bf16(tmem + C_S, tc::sdesc(aK + kk * 32, 16, 1024), tc::sdesc(bQ + kk * 32, 16, 1024), ID_T,
                                 kk != 0);
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk)
                    tc::mma_bf16(tmem + C_DP, tc::sdesc(aV + kk * 32, 16, 1024), tc::sdesc(bO + kk * 32, 16, 1024), ID_T,
                                 kk != 0);
                tc::mma_commit(st_full);
                return true;
            };
            if (ok && n > 0) ok = issue_st(0);
            for (int it = 0; it < n && ok; ++it) {
                const int st = it % QS;
                const uint32_t bQ = tc::smem_u32(sQD + st * QD_STAGE), bO = bQ + T128;
                if (it + 1 < n && !issue_st(it + 1)) {
                    ok = false;
                    break;
                }
                if (!tc::mbar_wait(pd_full, it & 1, a.status, 4)) {
                    ok = false;
                    break;
                }
                tc::tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < BB / 16; ++kk)
                    tc::mma_bf16(tmem + C_DV, a2desc(aP, kk), tc::sdesc(bO + kk * 2048, 8192, 1024), ID_A,
                                 (it | kk) != 0);
#pragma unroll
                for (int kk = 0; kk < BB / 16; ++kk)
                    tc::mma_bf16(tmem + C_DK, a2desc(aDS, kk), tc::sdesc(bQ + kk * 2048, 8192, 1024), ID_A,
                                 (it | kk) != 0);
                tc::mma_commit(pd_free);
                tc::mma_commit(&qd_empty[st]);
            }
            if (ok) tc::mma_commit(acc_full);
            tc::mma_commit(drain);
            tc::mbar_wait(drain, 0, a.status, 4, 400000000ll, false);
        }
    } else {
        // ---------------- compute: thread = key row, 64 of the block's 128 query columns
        const int qd = warp & 3, half = (warp - 2) >> 2, c0 = half * HALF;
        const int r = qd * 32 + lane;
        const int key = k0 + r;
        const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
        const float sc = a.scale * LOG2E;
        const int qlo = bqlo(a, key), qhi = bqhi(a, key);
        const uint32_t prow = tc::smem_u32(sP), dsrow = tc::smem_u32(sDS);
        bool ok = true;
        for (int it = 0; it < n && ok; ++it) {
            const int st = it % QS;
            const int q0 = (qb0 + it % nq) * BB;
            if (!tc::mbar_wait(st_full, it & 1, a.status, 4)) {
                ok = false;
                break;
            }
            tc::tc_fence_after();
            uint32_t s[HALF], dp[HALF];
            {
                uint32_t (&s0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[0]);
                uint32_t (&s1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[32]);
                uint32_t (&d0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&dp[0]);
                uint32_t (&d1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&dp[32]);
                tc::tmem_ld32(tmem + lane_off + C_S + c0, s0);
                tc::tmem_ld32(tmem + lane_off + C_S + c0 + 32, s1);
                tc::tmem_ld32(tmem + lane_off + C_DP + c0, d0);
                tc::tmem_ld32(tmem + lane_off + C_DP + c0 + 32, d1);
                tc::tmem_ld_wait();
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(st_free);
            // no masking when every (query, key) pair of the block is visible
            const bool full = q0 >= bqlo(a, klast) && q0 + BB - 1 <= bqhi(a, k0) && q0 + BB - 1 < a.s;
            const float* sL = (const float*)(sQD + st * QD_STAGE + 2 * T128);
            const float* sD = sL + 128;
            // the MMAs of the previous block have read the Pᵀ / dSᵀ tiles
            if (!tc::mbar_wait(pd_free, (it & 1) ^ 1, a.status, 4)) {
                ok = false;
                break;
            }
#pragma unroll
            for (int ch = 0; ch < HALF / 8; ++ch) {
                float p[8], ds[8];
                const float4 l0 = *(const float4*)(sL + c0 + ch * 8), l1 = *(const float4*)(sL + c0 + ch * 8 + 4);
                const float4 d0 = *(const float4*)(sD + c0 + ch * 8), d1 = *(const float4*)(sD + c0 + ch * 8 + 4);
                const float lv[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
                const float dv8[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
#pragma unroll
                for (int t = 0; t < 8; ++t) {
                    const int c = ch * 8 + t, q = q0 + c0 + c;
                    float pv = ex2(fmaf(__uint_as_float(s[c]), sc, -lv[t]));
                    if (!full && (q < qlo || q > qhi)) pv = 0.f;
                    p[t] = pv;
                    ds[t] = pv * (__uint_as_float(dp[c]) - dv8[t]);
                }
                st_chunk8(prow, r, c0 / 8 + ch, p);
                st_chunk8(dsrow, r, c0 / 8 + ch, ds);
            }
            tc::fence_proxy_async();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(pd_full);
        }
        if (ok && n > 0 && tc::mbar_wait(acc_full, 0, a.status, 4)) {
            tc::tc_fence_after();
            // each warp of a quadrant writes 32 of the 64 head columns
            const int hc = half * 32;
            uint32_t dv[32], dk[32];
            tc::tmem_ld32(tmem + lane_off + C_DV + hc, dv);
            tc::tmem_ld32(tmem + lane_off + C_DK + hc, dk);
            tc::tmem_ld_wait();
            if (key < a.s) {
                const long long off = (seq_row + key) * a.kv_stride + kvh * HD + hc;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint4 pv, pk;
                    __nv_bfloat162* a2 = (__nv_bfloat162*)&pv;
                    __nv_bfloat162* b2 = (__nv_bfloat162*)&pk;
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        a2[t] = __floats2bfloat162_rn(__uint_as_float(dv[c * 8 + 2 * t]), __uint_as_float(dv[c * 8 + 2 * t + 1]));
                        b2[t] = __floats2bfloat162_rn(__uint_as_float(dk[c * 8 + 2 * t]) * a.scale,
                                                      __uint_as_float(dk[c * 8 + 2 * t + 1]) * a.scale);
                    }
                    *(uint4*)(a.dv + off + c * 8) = pv;
                    *(uint4*)(a.dk + off + c * 8) = pk;
                }
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 512);
    }
}

// dQ: one CTA per 128 queries of a head; loops over its 128-key blocks:
// S = Q·Kᵀ and dP = dO·Vᵀ (N = 128 keys) into TMEM, dS (bf16) to shared
// memory (double-buffered), dQ += dS·K (K = 128 keys) in TMEM.
__global__ void __launch_bounds__(NTB, 1)
    k_dq(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mdo,
         const __grid_constant__ CUtensorMap mk, const __grid_constant__ CUtensorMap mv, BwdArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sQ = smem;
    uint8_t* sO = sQ + T128;
    uint8_t* sKV = sO + T128;  // KS stages: K | V (128 keys each)
    uint8_t* sDS = sKV + KS * 2 * T128;  // [2] dS tiles
    uint64_t* bars = (uint64_t*)(sDS + 2 * TPD);
    uint64_t* q_full = bars;
    uint64_t* kv_full = q_full + 1;
    uint64_t* kv_empty = kv_full + KS;
    uint64_t* st_full = kv_empty + KS;
    uint64_t* st_free = st_full + 1;
    uint64_t* ds_full = st_free + 1;
    uint64_t* ds_free = ds_full + 2;
    uint64_t* acc_full = ds_free + 2;
    uint64_t* drain = acc_full + 1;
    uint32_t* tmem_slot = (uint32_t*)(drain + 1);
    // TMEM columns: S 0..127, dP 128..255, dQ 256..319
    constexpr uint32_t C_S = 0, C_DP = 128, C_DQ = 256;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // late queries see the most keys: heaviest query blocks first (slowest grid index)
    const int qt = gridDim.z - 1 - blockIdx.z;
    const int q0 = qt * 128, h = blockIdx.x, bi = blockIdx.y;
    const int kvh = h / (a.h / a.hkv);
    const int qlast = min(q0 + 127, a.s - 1);
    const int j0 = bklo(a, q0) / BB, j1 = min(bkhi(a, qlast), a.s - 1) / BB;
    const int n = j1 - j0 + 1;
    const long long seq_row = (long long)bi * a.s;

    if (threadIdx.x == 0) {
        tc::mbar_init(q_full, 1);
        for (int i = 0; i < KS; ++i) {
            tc::mbar_init(&kv_full[i], 1);
            tc::mbar_init(&kv_empty[i], 1);
        }
        tc::mbar_init(st_full, 1);
        tc::mbar_init(st_free, NCW);
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&ds_full[i], NCW);
            tc::mbar_init(&ds_free[i], 1);
        }
        tc::mbar_init(acc_full, 1);
        tc::mbar_init(drain, 1);
        tc::fence_mbar_init();
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, 512);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            tc::mbar_arrive_expect_tx(q_full, 2 * T128);
            tc::tma_load_2d(sQ, &mq, h * HD, (int)(seq_row + q0), q_full);
            tc::tma_load_2d(sO, &mdo, h * HD, (int)(seq_row + q0), q_full);
            uint32_t used = 0, last_par = 0;
            bool ok = true;
            for (int j = 0; j < n; ++j) {
                const int st = j % KS;
                const uint32_t ph = (j / KS) & 1;
                if (!tc::mbar_wait(&kv_empty[st], ph ^ 1, a.status, 4)) {
                    ok = false;
                    break;
                }
                uint8_t* stg = sKV + st * 2 * T128;
                tc::mbar_arrive_expect_tx(&kv_full[st], 2 * T128);
                const int krow = (int)(seq_row + (long long)(j0 + j) * BB);
                tc::tma_load_2d(stg, &mk, kvh * HD, krow, &kv_full[st]);
                tc::tma_load_2d(stg + T128, &mv, kvh * HD, krow, &kv_full[st]);
                used |= 1u << st;
                last_par = (last_par & ~(1u << st)) | (ph << st);
            }
            if (!ok) {
                tc::mbar_wait(q_full, 0, a.status, 4, 400000000ll, false);
                for (int i = 0; i < KS; ++i)
                    if ((used >> i) & 1u) tc::mbar_wait(&kv_full[i], (last_par >> i) & 1u, a.status, 4, 400000000ll, false);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t ID_S = tc::idesc_bf16(128, BB, false, false);  // S, dP
            constexpr uint32_t ID_Q = tc::idesc_bf16(128, HD, false, true);   // dQ (K MN-major)
            bool ok = tc::mbar_wait(q_full, 0, a.status, 4);
            const uint32_t aQ = tc::smem_u32(sQ), aO = tc::smem_u32(sO), aDS = tc::smem_u32(sDS);
            // S, dP of block j: issued once the compute warps hold block j-1's
            auto issue_st = [&](int j) -> bool {
                const int st = j % KS;
                if (!tc::mbar_wait(&kv_full[st], (j / KS) & 1, a.status, 4) ||
                    !tc::mbar_wait(st_free, (j & 1) ^ 1, a.status, 4))
                    return false;
                tc::tc_fence_after();
                const uint32_t bK = tc::smem_u32(sKV + st * 2 * T128), bV = bK + T128;
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk)
                    tc::mma_bf16(tmem + C_S, tc::sdesc(aQ + kk * 32, 16, 1024), tc::sdesc(bK + kk * 32, 16, 1024), ID_S,
                                 kk != 0);
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk)
                    tc::mma_bf16(tmem + C_DP, tc::sdesc(aO + kk * 32, 16, 1024), tc::sdesc(bV + kk * 32, 16, 1024), ID_S,
                                 kk != 0);
                tc::mma_commit(st_full);
                return true;
            };
            if (ok && n > 0) ok = issue_st(0);
            for (int j = 0; j < n && ok; ++j) {
                const int st = j % KS, db = j & 1;
                const uint32_t bK = tc::smem_u32(sKV + st * 2 * T128);
                if (j + 1 < n && !issue_st(j + 1)) {
                    ok = false;
                    break;
                }
                if (!tc::mbar_wait(&ds_full[db], (j >> 1) & 1, a.status, 4)) {
                    ok = false;
                    break;
                }
                tc::tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < BB / 16; ++kk)
                    tc::mma_bf16(tmem + C_DQ, a2desc(aDS + db * TPD, kk), tc::sdesc(bK + kk * 2048, 8192, 1024), ID_Q,
                                 (j | kk) != 0);
                tc::mma_commit(&ds_free[db]);
                tc::mma_commit(&kv_empty[st]);
            }
            if (ok) tc::mma_commit(acc_full);
            tc::mma_commit(drain);
            tc::mbar_wait(drain, 0, a.status, 4, 400000000ll, false);
        }
    } else {
        // ---------------- compute: thread = query row, 64 of the block's 128 key columns
        const int qd = warp & 3, half = (warp - 2) >> 2, c0 = half * HALF;
        const int r = qd * 32 + lane;
        const int row = q0 + r;
        const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
        const float sc = a.scale * LOG2E;
        const long long lrow = ((long long)bi * a.h + h) * a.s;
        const float L = row < a.s ? a.lse[lrow + row] * LOG2E : INFINITY;
        const float D = row < a.s ? a.dsum[lrow + row] : 0.f;
        const int lo = bklo(a, row), hi = min(bkhi(a, row), a.s - 1);
        bool ok = true;
        for (int j = 0; j < n && ok; ++j) {
            const int kb0 = (j0 + j) * BB, db = j & 1;
            if (!tc::mbar_wait(st_full, j & 1, a.status, 4)) {
                ok = false;
                break;
            }
            tc::tc_fence_after();
            uint32_t s[HALF], dp[HALF];
            {
                uint32_t (&s0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[0]);
                uint32_t (&s1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[32]);
                uint32_t (&d0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&dp[0]);
                uint32_t (&d1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&dp[32]);
                tc::tmem_ld32(tmem + lane_off + C_S + c0, s0);
                tc::tmem_ld32(tmem + lane_off + C_S + c0 + 32, s1);
                tc::tmem_ld32(tmem + lane_off + C_DP + c0, d0);
                tc::tmem_ld32(tmem + lane_off + C_DP + c0 + 32, d1);
                tc::tmem_ld_wait();
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(st_free);
            const bool full = kb0 >= bklo(a, qlast) && kb0 + BB - 1 <= min(bkhi(a, q0), a.s - 1);
            // the dQ MMA of block j - 2 has read this dS buffer
            if (!tc::mbar_wait(&ds_free[db], ((j >> 1) & 1) ^ 1, a.status, 4)) {
                ok = false;
                break;
            }
            const uint32_t dsrow = tc::smem_u32(sDS + db * TPD);
#pragma unroll
            for (int ch = 0; ch < HALF / 8; ++ch) {
                float ds[8];
#pragma unroll
                for (int t = 0; t < 8; ++t) {
                    const int c = ch * 8 + t, key = kb0 + c0 + c;
                    float pv = ex2(fmaf(__uint_as_float(s[c]), sc, -L));
                    if (!full && (key < lo || key > hi)) pv = 0.f;
                    ds[t] = pv * (__uint_as_float(dp[c]) - D);
                }
                st_chunk8(dsrow, r, c0 / 8 + ch, ds);
            }
            tc::fence_proxy_async();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&ds_full[db]);
        }
        if (ok && n > 0 && tc::mbar_wait(acc_full, 0, a.status, 4)) {
            tc::tc_fence_after();
            const int hc = half * 32;
            uint32_t dq[32];
            tc::tmem_ld32(tmem + lane_off + C_DQ + hc, dq);
            tc::tmem_ld_wait();
            if (row < a.s) {
                bf16* out = a.dq + (seq_row + row) * a.q_stride + h * HD + hc;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint4 pk;
                    __nv_bfloat162* b2 = (__nv_bfloat162*)&pk;
#pragma unroll
                    for (int t = 0; t < 4; ++t)
                        b2[t] = __floats2bfloat162_rn(__uint_as_float(dq[c * 8 + 2 * t]) * a.scale,
                                                      __uint_as_float(dq[c * 8 + 2 * t + 1]) * a.scale);
                    *(uint4*)(out + c * 8) = pk;
                }
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 512);
    }
}

}  // namespace fa5

// The tcgen05 forward applies to head_dim 64 with 16-byte aligned bases and
// row pitches (the TMA maps' requirements).
bool attention_fwd_tc5_ok(i64 hd, i64 q_stride, i64 kv_stride, const void* q, const void* k, const void* v) {
    auto al = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
    return hd == 64 && q_stride % 8 == 0 && kv_stride % 8 == 0 && al(q) && al(k) && al(v);
}

void attention_fwd_tc5(Context* c, const void* q, const void* k, const void* v, void* o, float* lse, i64 b, i64 s,
                       i64 h, i64 hkv, bool causal, i64 window, i64 q_stride, i64 kv_stride) {
    using namespace fa5;
    if (b <= 0 || s <= 0 || h <= 0) return;
    CATNN_CHECK(b * s < (1ll << 31) && h % hkv == 0, CATNN_ERR_SHAPE, "attention: sizes");
    CATNN_CHECK(b <= 65535 && cdiv(s, 128) <= 65535, CATNN_ERR_SHAPE, "attention: grid limits (batch, seq / 128)");
    // maps over all B*S rows; a box that runs past the last row reads zeros,
    // rows of the next sequence inside a box are masked (key >= S) or not stored
    CUtensorMap mq = tma_map_bf16(q, b * s, h * HD, q_stride, HD, BQ);
    CUtensorMap mk = tma_map_bf16(k, b * s, hkv * HD, kv_stride, HD, BKV);
    CUtensorMap mv = tma_map_bf16(v, b * s, hkv * HD, kv_stride, HD, BKV);
    Args a{};
    a.b = (int)b;
    a.s = (int)s;
    a.h = (int)h;
    a.hkv = (int)hkv;
    a.causal = causal ? 1 : 0;
    a.window = (int)window;
    a.scale = 1.0f / sqrtf((float)HD);
    a.out = (bf16*)o;
    a.lse = lse;
    a.status = c->status;
    static bool attr[64] = {false};
    if (!attr[c->device]) {
        CUDA_OK(cudaFuncSetAttribute(k_fwd, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM));
        attr[c->device] = true;
    }
    dim3 grid((unsigned)h, (unsigned)b, (unsigned)cdiv(s, BQ));
    k_fwd<<<grid, NT, SMEM, c->stream>>>(mq, mk, mv, a);
    launched(c);
}

}  // namespace catnn

namespace catnn {

void attention_bwd_tc5(Context* c, const void* q, const void* k, const void* v, const void* dout, const float* lse,
                       const float* dsum, void* dq, void* dk, void* dv, i64 b, i64 s, i64 h, i64 hkv, bool causal,
                       i64 window, i64 q_stride, i64 kv_stride) {
    using namespace fa5;
    if (b <= 0 || s <= 0 || h <= 0) return;
    CATNN_CHECK(b * s < (1ll << 31) && h % hkv == 0, CATNN_ERR_SHAPE, "attention: sizes");
    CATNN_CHECK(b <= 65535 && cdiv(s, 128) <= 65535, CATNN_ERR_SHAPE, "attention: grid limits (batch, seq / 128)");
    CUtensorMap mq128 = tma_map_bf16(q, b * s, h * HD, q_stride, HD, 128);
    CUtensorMap mdo128 = tma_map_bf16(dout, b * s, h * HD, h * HD, HD, 128);
    CUtensorMap mk128 = tma_map_bf16(k, b * s, hkv * HD, kv_stride, HD, 128);
    CUtensorMap mv128 = tma_map_bf16(v, b * s, hkv * HD, kv_stride, HD, 128);
    BwdArgs a{};
    a.b = (int)b;
    a.s = (int)s;
    a.h = (int)h;
    a.hkv = (int)hkv;
    a.causal = causal ? 1 : 0;
    a.window = (int)window;
    a.scale = 1.0f / sqrtf((float)HD);
    a.lse = lse;
    a.dsum = dsum;
    a.dq = (bf16*)dq;
    a.dk = (bf16*)dk;
    a.dv = (bf16*)dv;
    a.q_stride = (int)q_stride;
    a.kv_stride = (int)kv_stride;
    a.status = c->status;
    static bool attr[64] = {false};
    if (!attr[c->device]) {
        CUDA_OK(cudaFuncSetAttribute(k_dkdv, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_DKDV));
        CUDA_OK(cudaFuncSetAttribute(k_dq, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_DQ));
        attr[c->device] = true;
    }
    k_dkdv<<<dim3((unsigned)hkv, (unsigned)b, (unsigned)cdiv(s, 128)), NTB, SMEM_DKDV, c->stream>>>(mk128, mv128, mq128,
                                                                                                    mdo128, a);
    k_dq<<<dim3((unsigned)h, (unsigned)b, (unsigned)cdiv(s, 128)), NTB, SMEM_DQ, c->stream>>>(mq128, mdo128, mk128,
                                                                                              mv128, a);
    launched(c, 2);
}

// attention / gqa_attention on the bf16 path (head_dim 64): the forward
// kernel, one CTA per 128 queries of a (batch, head).
KernelInfo fa5_info(Context* c, const std::string& op, const KShape& s) {
    KernelInfo k;
    if (!(op == "attention" || op == "gqa_attention") || s.head_dim != fa5::HD) return k;
    k.fn = (const void*)fa5::k_fwd;
    k.file = "attention_fa5.cu";
    k.grid[0] = (unsigned)s.heads;
    k.grid[1] = (unsigned)s.batch;
    k.grid[2] = (unsigned)cdiv(s.seq, fa5::BQ);
    k.block[0] = fa5::NT;
    k.dyn_smem = fa5::SMEM;
    return k;
}

}  // namespace catnn
