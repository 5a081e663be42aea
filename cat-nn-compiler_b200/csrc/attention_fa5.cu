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
constexpr uint32_t TMEM_COLS = 256;              // S: 2 x 64, O: 2 x 64 (two CTAs per SM)
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
    uint64_t* o_full = p_full + 2;
    uint64_t* o_free = o_full + 2;
    uint64_t* drain = o_free + 2;
    uint32_t* tmem_slot = (uint32_t*)(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // heaviest (latest) query tiles first
    const int qt = gridDim.x - 1 - blockIdx.x;
    const int q0 = qt * BQ, h = blockIdx.y, bi = blockIdx.z;
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
            tc::mbar_init(&o_full[i], 1);
            tc::mbar_init(&o_free[i], 4);
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
            constexpr uint32_t IDO = tc::idesc_bf16(BQ, HD, false, true);    // O = P·V (V MN-major)
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
                if (!tc::mbar_wait(&p_full[pb], (j >> 1) & 1, a.status, 4)) {
                    ok = false;
                    break;
                }
                if (!tc::mbar_wait(&o_free[pb], ((j >> 1) & 1) ^ 1, a.status, 4)) {
                    ok = false;
                    break;
                }
                tc::tc_fence_after();
                const uint32_t ap = tc::smem_u32(sP + pb * P_BYTES);
                const uint32_t bv = tc::smem_u32(sKV + st * STAGE_BYTES + KV_BYTES);
#pragma unroll
                for (int kk = 0; kk < BKV / 16; ++kk)
                    tc::mma_bf16(tmem + O_COL + pb * HD, tc::sdesc(ap + kk * 32, 16, 1024),
                                 tc::sdesc(bv + kk * 2048, 8192, 1024), IDO, kk != 0);
                tc::mma_commit(&o_full[pb]);
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
        const float sc = a.scale * LOG2E;
        const int lo = klo(a, row), hi = min(khi(a, row), a.s - 1);
        float o[HD];
#pragma unroll
        for (int i = 0; i < HD; ++i) o[i] = 0.f;
        float m = -INFINITY, l = 0.f, alpha_prev = 1.f;
        bool ok = true;
        for (int j = 0; j <= nblk && ok; ++j) {
            float alpha = 1.f;
            if (j < nblk) {
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
                // One TMEM read of the block's 64 scores per row (two loads in
                // flight), kept in registers for both passes. Pass 1: block
                // max in eight independent chains.
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
                float mxa[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) mxa[u] = -INFINITY;
#pragma unroll
                for (int i = 0; i < 64; ++i) mxa[i & 7] = fmaxf(mxa[i & 7], __uint_as_float(v[i]));
                float mx = fmaxf(fmaxf(fmaxf(mxa[0], mxa[1]), fmaxf(mxa[2], mxa[3])),
                                 fmaxf(fmaxf(mxa[4], mxa[5]), fmaxf(mxa[6], mxa[7])));
                // scale > 0: the max of the scaled scores is the scaled max
                const float mn = fmaxf(m, mx * sc);
                const float base = mn == -INFINITY ? 0.f : mn;
                alpha = ex2(m - base);
                m = mn;
                float lsa[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) lsa[u] = 0.f;
                const uint32_t prow = tc::smem_u32(sP + sb * P_BYTES + r * 128);
                // Pass 2: P = 2^(s·scale - max) (masked scores are -inf: P = 0),
                // row sums, bf16 P to shared memory in 16-byte chunks
#pragma unroll
                for (int chunk = 0; chunk < BKV / 8; ++chunk) {
                    float p[8];
#pragma unroll
                    for (int t = 0; t < 8; ++t) {
                        p[t] = ex2(fmaf(__uint_as_float(v[chunk * 8 + t]), sc, -base));
                        lsa[t] += p[t];
                    }
                    uint4 pk;
                    __nv_bfloat162* pp = (__nv_bfloat162*)&pk;
#pragma unroll
                    for (int t = 0; t < 4; ++t) pp[t] = __floats2bfloat162_rn(p[2 * t], p[2 * t + 1]);
                    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(prow + ((chunk ^ (r & 7)) << 4)),
                                 "r"(pk.x), "r"(pk.y), "r"(pk.z), "r"(pk.w)
                                 : "memory");
                }
                const float ls = ((lsa[0] + lsa[1]) + (lsa[2] + lsa[3])) + ((lsa[4] + lsa[5]) + (lsa[6] + lsa[7]));
                l = l * alpha + ls;
                // P_j is in shared memory: hand it to the async proxy (the MMA)
                tc::fence_proxy_async();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&p_full[sb]);
            }
            // fold in O_{j-1} = P_{j-1}·V_{j-1} (it used max m_{j-1}, so the
            // accumulator is rescaled by alpha_{j-1} first)
            if (j > 0) {
                const int ob = (j - 1) & 1;
                if (!tc::mbar_wait(&o_full[ob], ((j - 1) >> 1) & 1, a.status, 4)) {
                    ok = false;
                    break;
                }
                tc::tc_fence_after();
                const uint32_t oa = tmem + lane_off + O_COL + ob * HD;
#pragma unroll
                for (int c = 0; c < HD / 32; ++c) {
                    uint32_t v[32];
                    tc::tmem_ld32(oa + c * 32, v);
                    tc::tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[c * 32 + i] = o[c * 32 + i] * alpha_prev + __uint_as_float(v[i]);
                }
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&o_free[ob]);
            }
            alpha_prev = alpha;
        }
        if (ok && row < a.s) {
            const float inv = l > 0.f ? 1.f / l : 0.f;
            bf16* op = a.out + (seq_row + row) * (long long)(a.h * HD) + h * HD;
#pragma unroll
            for (int c = 0; c < HD / 8; ++c) {
                uint4 pk;
                __nv_bfloat162* pp = (__nv_bfloat162*)&pk;
#pragma unroll
                for (int t = 0; t < 4; ++t) pp[t] = __floats2bfloat162_rn(o[c * 8 + 2 * t] * inv, o[c * 8 + 2 * t + 1] * inv);
                *(uint4*)(op + c * 8) = pk;
            }
            a.lse[((long long)bi * a.h + h) * a.s + row] = l > 0.f ? (m + log2f(l)) / LOG2E : -INFINITY;
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, TMEM_COLS);
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
    dim3 grid((unsigned)cdiv(s, BQ), (unsigned)h, (unsigned)b);
    k_fwd<<<grid, NT, SMEM, c->stream>>>(mq, mk, mv, a);
    launched(c);
}

}  // namespace catnn
