// The MoE decoder training step on one GPU: forward with saved
// activations, fused cross-entropy, backward, optimizer — all device
// kernels of this library launched on the context stream, no host sync
// inside a step. Layout choices:
//  - residual stream fp32 (x_in, x_mid per layer); every tensor that feeds a
//    GEMM is stored in the shadow dtype (bf16 on the tensor-core path);
//  - fused QKV weight [d, (H+2Hkv)·hd] and fused expert weight
//    W13_e = [w1_e | w3_e] ([d, 2F]) so one GEMM produces both SwiGLU inputs;
//  - expert rows padded to 128 so every expert GEMM tile is single-expert;
//  - weight gradients land in fp32 directly from the GEMM epilogue.
#include <cstring>
#include <utility>
#include <string>

#include "moe_ep.cuh"
#include "trainer.cuh"

namespace catnn {

namespace {
// Enqueue the launchers' work on another stream for the scope's lifetime.
struct OnStream {
    Context* c;
    cudaStream_t saved;
    OnStream(Context* ctx, cudaStream_t s) : c(ctx), saved(ctx->stream) { c->stream = s; }
    ~OnStream() { c->stream = saved; }
};
}  // namespace

static i64 al128(i64 n) { return (n + 127) / 128 * 128; }

void MoeTrainer::plan_params() {
    i64 o = 0;
    auto take = [&](i64 n) {
        i64 r = o;
        o += al128(n);
        return r;
    };
    // a sharded range starts and ends on a multiple of world*128 elements:
    // its chunks are equal and 512-byte aligned
    const i64 W = world;
    auto pad = [&]() { o = (o + W * 128 - 1) / (W * 128) * (W * 128); };
    Vs = (V + W - 1) / W;
    v0 = std::min<i64>(V, rank * Vs);
    v1 = std::min<i64>(V, v0 + Vs);
    o_embed = take(W * Vs * d);
    lo.resize(L);
    lb.resize(L);
    for (i64 l = 0; l < L; ++l) {
        lb[l].s_off = o;
        lo[l].rms_attn = take(d);
        lo[l].rms_moe = take(d);
        lo[l].gate = take(d * E);
        lb[l].s_len = o - lb[l].s_off;
        pad();
        lb[l].b_off = o;
        lo[l].wqkv = take(d * qkvd);
        lo[l].wo = take(qd * d);
        pad();
        lb[l].b_len = o - lb[l].b_off;
    }
    fin.s_off = o;
    o_final = take(d);
    o_loss = take(1);
    fin.s_len = o - fin.s_off;
    pad();
    fin.b_off = o;
    o_lm = take(V * d);
    pad();
    fin.b_len = o - fin.b_off;
    n_rep = o;
    for (i64 l = 0; l < L; ++l) {
        lo[l].w13 = take(El * d * 2 * F);
        lo[l].w2 = take(El * F * d);
    }
    n_params = o;
}

i64 MoeTrainer::packed_count() const {
    i64 layer = d + d * qd + 2 * d * kd + qd * d + d + d * E + 2 * E * d * F + E * F * d;
    return V * d + L * layer + d + V * d;
}

// Packed (reference) order, per layer: rms_attn, wq, wk, wv, wo, rms_moe,
// gate, w1[E], w3[E], w2[E] — the oracle's MixLayout.
void MoeTrainer::import_packed(const float* pk, float* dst) {
    cudaStream_t s = c->stream;
    auto cp = [&](float* to, const float* from, i64 n) {
        CUDA_OK(cudaMemcpyAsync(to, from, n * 4, cudaMemcpyDeviceToDevice, s));
    };
    auto cp2 = [&](float* to, i64 to_ld, const float* from, i64 from_ld, i64 cols, i64 rows) {
        CUDA_OK(cudaMemcpy2DAsync(to, to_ld * 4, from, from_ld * 4, cols * 4, rows, cudaMemcpyDeviceToDevice, s));
    };
    const float* p = pk;
    cp(dst + o_embed, p, V * d);
    p += V * d;
    for (i64 l = 0; l < L; ++l) {
        const LayerOff& q = lo[l];
        cp(dst + q.rms_attn, p, d); p += d;
        cp2(dst + q.wqkv, qkvd, p, qd, qd, d); p += d * qd;
        cp2(dst + q.wqkv + qd, qkvd, p, kd, kd, d); p += d * kd;
        cp2(dst + q.wqkv + qd + kd, qkvd, p, kd, kd, d); p += d * kd;
        cp(dst + q.wo, p, qd * d); p += qd * d;
        cp(dst + q.rms_moe, p, d); p += d;
        cp(dst + q.gate, p, d * E); p += d * E;
        // this rank's experts [e0, e0 + El) of w1[E], w3[E], w2[E]
        if (ilv) {
            for (i64 j = 0; j < F / 128; ++j) {
                cp2(dst + q.w13 + 256 * j, 2 * F, p + e0 * d * F + 128 * j, F, 128, El * d);
                cp2(dst + q.w13 + 256 * j + 128, 2 * F, p + E * d * F + e0 * d * F + 128 * j, F, 128, El * d);
            }
            p += 2 * E * d * F;
        } else {
            cp2(dst + q.w13, 2 * F, p + e0 * d * F, F, F, El * d); p += E * d * F;
            cp2(dst + q.w13 + F, 2 * F, p + e0 * d * F, F, F, El * d); p += E * d * F;
        }
        cp(dst + q.w2, p + e0 * F * d, El * F * d); p += E * F * d;
    }
    cp(dst + o_final, p, d); p += d;
    cp(dst + o_lm, p, V * d);
}

void MoeTrainer::export_packed(const float* src, float* pk) {
    cudaStream_t s = c->stream;
    auto cp = [&](float* to, const float* from, i64 n) {
        CUDA_OK(cudaMemcpyAsync(to, from, n * 4, cudaMemcpyDeviceToDevice, s));
    };
    auto cp2 = [&](float* to, i64 to_ld, const float* from, i64 from_ld, i64 cols, i64 rows) {
        CUDA_OK(cudaMemcpy2DAsync(to, to_ld * 4, from, from_ld * 4, cols * 4, rows, cudaMemcpyDeviceToDevice, s));
    };
    float* p = pk;
    cp(p, src + o_embed, V * d);
    p += V * d;
    for (i64 l = 0; l < L; ++l) {
        const LayerOff& q = lo[l];
        cp(p, src + q.rms_attn, d); p += d;
        cp2(p, qd, src + q.wqkv, qkvd, qd, d); p += d * qd;
        cp2(p, kd, src + q.wqkv + qd, qkvd, kd, d); p += d * kd;
        cp2(p, kd, src + q.wqkv + qd + kd, qkvd, kd, d); p += d * kd;
        cp(p, src + q.wo, qd * d); p += qd * d;
        cp(p, src + q.rms_moe, d); p += d;
        cp(p, src + q.gate, d * E); p += d * E;
        if (ilv) {
            for (i64 j = 0; j < F / 128; ++j) {
                cp2(p + e0 * d * F + 128 * j, F, src + q.w13 + 256 * j, 2 * F, 128, El * d);
                cp2(p + E * d * F + e0 * d * F + 128 * j, F, src + q.w13 + 256 * j + 128, 2 * F, 128, El * d);
            }
            p += 2 * E * d * F;
        } else {
            cp2(p + e0 * d * F, F, src + q.w13, 2 * F, F, El * d); p += E * d * F;
            cp2(p + e0 * d * F, F, src + q.w13 + F, 2 * F, F, El * d); p += E * d * F;
        }
        cp(p + e0 * F * d, src + q.w2, El * F * d); p += E * F * d;
    }
    cp(p, src + o_final, d); p += d;
    cp(p, src + o_lm, V * d);
}

void MoeTrainer::alloc() {
    size_t e = dsize(dt);
    // parameters: P, G (+ Mo, Vo for Adam) fp32, shadow in dt
    size_t pb = (size_t)n_params * 4;
    size_t ptot = pb * (opt == 1 ? 4 : 2) + (dt == CATNN_BF16 ? (size_t)n_params * e : 0) + 4096;
    CUDA_OK(cudaMalloc(&param_block, ptot));
    CUDA_OK(cudaMemsetAsync(param_block, 0, ptot, c->stream));
    Carver pc(param_block);
    P = pc.take<float>(n_params);
    G = pc.take<float>(n_params);
    if (opt == 1) {
        Mo = pc.take<float>(n_params);
        Vo = pc.take<float>(n_params);
    }
    Sh = dt == CATNN_BF16 ? (void*)pc.take<char>(n_params * e) : (void*)P;

    // activations + scratch
    std::vector<size_t> sz;
    auto add = [&](size_t b) { sz.push_back(b); };
    for (i64 l = 0; l < L; ++l) {
        add(T * d * 4); add(T * d * 4); add(B * H * S * 4); add(T * E * 4); add(T * K * 4);
        add(T * d * e); add(T * qkvd * e); add(T * qd * e); add(T * d * e); add(cap * d * e);
        add(cap * 2 * F * e); add(cap * F * e); add(cap * d * e);
        add(T * K * 4); add(E * 4); add((E + 1) * 4); add(T * K * 4); add(cap * 4);
        if (dt == CATNN_BF16) add(T * d * 4);
        if (ep) { add(world * E * 4); add(ep_plan_len(E, El) * 4); add(T * K * 4); }
    }
    if (ep) add(T * K * 4);
    add(Tg * 4); add(64);
    add(T * d * 4); add(T * d * e); add((size_t)T * V * e); add(Tg * 4); add(T * 4); add(64);
    add(T * d * 4); add(T * d * 4); add(T * d * 4); add(T * E * 4); add(T * K * 4);
    add(T * d * e); add(cap * d * e); add(cap * F * e); add(cap * 2 * F * e); add(cap * d * e); add(T * qkvd * e);
    add(T * qd * e); add(T * d * e); add(T * E * e); add(T * d * e);
    size_t tot = 0;
    for (size_t b : sz) tot += (b + 255) / 256 * 256;
    tot += 4096;
    CUDA_OK(cudaMalloc(&act_block, tot));
    Carver ac(act_block);
    acts.resize(L);
    for (i64 l = 0; l < L; ++l) {
        Act& a = acts[l];
        a.x_in = ac.take<float>(T * d);
        a.x_mid = ac.take<float>(T * d);
        a.lse = ac.take<float>(B * H * S);
        a.logits = ac.take<float>(T * E);
        a.w = ac.take<float>(T * K);
        a.xn = ac.take<char>(T * d * e);
        a.qkv = ac.take<char>(T * qkvd * e);
        a.ctx = ac.take<char>(T * qd * e);
        a.xm = ac.take<char>(T * d * e);
        a.xp = ac.take<char>(cap * d * e);
        a.ac = ac.take<char>(cap * 2 * F * e);
        a.h = ac.take<char>(cap * F * e);
        a.yp = ac.take<char>(cap * d * e);
        a.idx = ac.take<int32_t>(T * K);
        a.counts = ac.take<int32_t>(E);
        a.off = ac.take<int32_t>(E + 1);
        a.row_of = ac.take<int32_t>(T * K);
        a.src_of = ac.take<int32_t>(cap);
        a.xm32 = dt == CATNN_BF16 ? ac.take<float>(T * d) : (float*)a.xm;
        if (ep) {
            a.cnt_all = ac.take<int32_t>(world * E);
            a.plan = ac.take<int32_t>(ep_plan_len(E, El));
            a.dest = ac.take<int32_t>(T * K);
        }
    }
    if (ep) src1 = ac.take<int32_t>(T * K);
    emb_keys = ac.take<uint32_t>(Tg);
    emb_m = ac.take<int>(16);
    x_last = ac.take<float>(T * d);
    xf = ac.take<char>(T * d * e);
    lg = ac.take<char>((size_t)T * V * e);
    tokens = ac.take<uint32_t>(Tg);
    targets = ac.take<uint32_t>(T);
    loss = ac.take<float>(16);
    dx = ac.take<float>(T * d);
    dxmid = ac.take<float>(T * d);
    dxm = ac.take<float>(T * d);
    dlog = ac.take<float>(T * E);
    dwts = ac.take<float>(T * K);
    dxmid_lp = ac.take<char>(T * d * e);
    dyp = ac.take<char>(cap * d * e);
    dh = ac.take<char>(cap * F * e);
    dac = ac.take<char>(cap * 2 * F * e);
    dxp = ac.take<char>(cap * d * e);
    dqkv = ac.take<char>(T * qkvd * e);
    dctx = ac.take<char>(T * qd * e);
    dxn = ac.take<char>(T * d * e);
    dlog_lp = ac.take<char>(T * E * e);
    dxf = ac.take<char>(T * d * e);
    CUDA_OK(cudaMallocHost(&h_tokens, Tg * 4));
    CUDA_OK(cudaMallocHost(&h_loss, 64));
    CUDA_OK(cudaMalloc(&d12, 2 * sizeof(float)));
    act_bytes = tot;
    if (ep) {
        // peers read the embedding rows this rank owns: map the parameter block
        CUDA_OK(cudaStreamSynchronize(c->stream));
        comm->map(param_block, ptot);
        map_pid = (int)comm->maps.size() - 1;
        ev_g.assign(L + 1, nullptr);
        for (auto& ev : ev_g) CUDA_OK(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
        // every activation buffer a peer reads or writes lives in act_block: map it once
        CUDA_OK(cudaMemsetAsync(act_block, 0, tot, c->stream));
        CUDA_OK(cudaStreamSynchronize(c->stream));
        comm->map(act_block, tot);
        map_id = (int)comm->maps.size() - 1;
    }
}

template <typename Q>
PeerTab MoeTrainer::tab(Q* local) const {
    PeerTab t{};
    for (int p = 0; p < world; ++p) t.p[p] = (void*)comm->at(comm->maps[map_id], p, (char*)local);
    return t;
}

template <typename Q>
PeerTab MoeTrainer::ptab(Q* local) const {
    PeerTab t{};
    for (int p = 0; p < world; ++p) t.p[p] = (void*)comm->at(comm->maps[map_pid], p, (char*)local);
    return t;
}

void MoeTrainer::release() {
    if (ep && (map_id >= 0 || map_pid >= 0) && comm) {
        // close this rank's mappings of the peers' arenas; only when every
        // rank has done so may any rank free its own (collective)
        cudaStreamSynchronize(c->stream);
        for (int id : {map_id, map_pid}) {
            if (id < 0) continue;
            Comm::Mapped& m = comm->maps[id];
            for (int p = 0; p < world; ++p)
                if (p != rank && m.base[p]) {
                    cudaIpcCloseMemHandle(m.base[p]);
                    m.base[p] = nullptr;
                }
        }
        try {
            comm->barrier();
        } catch (...) {
        }
        cudaStreamSynchronize(c->stream);
        map_id = map_pid = -1;
    }
    for (auto& ev : ev_g)
        if (ev) cudaEventDestroy(ev);
    ev_g.clear();
    drop_graphs();
    if (gs) {
        cudaStreamSynchronize(gs);
        cudaEventDestroy(ev_in);
        cudaEventDestroy(ev_out);
        cudaStreamDestroy(gs);
        gs = nullptr;
    }
    if (d12) cudaFree(d12);
    d12 = nullptr;
    if (stamps) cudaFree(stamps);
    stamps = nullptr;
    if (ws) {
        cudaStreamSynchronize(ws);
        cudaEventDestroy(ev_w);
        cudaEventDestroy(ev_wd);
        cudaStreamDestroy(ws);
        ws = nullptr;
    }
    if (wscratch) cudaFree(wscratch);
    wscratch = nullptr;
    wscratch_bytes = 0;
    if (ev_k) {
        cudaEventDestroy(ev_k);
        cudaEventDestroy(ev_kd);
        ev_k = ev_kd = nullptr;
    }
    if (us) {
        cudaStreamSynchronize(us);
        cudaEventDestroy(ev_u);
        cudaEventDestroy(ev_u_done);
        cudaStreamDestroy(us);
        us = nullptr;
    }
    if (param_block) cudaFree(param_block);
    if (act_block) cudaFree(act_block);
    if (h_tokens) cudaFreeHost(h_tokens);
    if (h_loss) cudaFreeHost(h_loss);
    param_block = act_block = nullptr;
    h_tokens = nullptr;
    h_loss = nullptr;
}

// train.rs:274-275: targets[i] = tokens[(i+1) % n] % vocab over the global
// token array (n tokens); this rank's targets are those of tokens off .. off+m-1.
__global__ void k_next_token(const uint32_t* __restrict__ tok, uint32_t* __restrict__ tg, i64 off, i64 m, i64 n,
                             i64 vocab) {
    i64 i = blockIdx.x * (i64)blockDim.x + threadIdx.x;
    if (i < m) tg[i] = tok[(off + i + 1) % n] % (uint32_t)vocab;
}

// The device clock (ns) at this point of the stream.
__global__ void k_stamp(unsigned long long* out) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    *out = t;
}

void MoeTrainer::stamp(const char* name) {
    if (!prof || (int)stamp_names.size() >= MAX_STAMPS) return;
    k_stamp<<<1, 1, 0, c->stream>>>(stamps + stamp_names.size());
    launched(c);
    stamp_names.push_back(name);
}

// Expert GEMM over the sorted rows (bf16: tcgen05 grouped; fp32: CUDA cores).
static void expert_gemm(Context* c, int dt, bool tb, i64 rows, i64 N, i64 Kd, int E, const int32_t* off, const void* A,
                        i64 lda, const void* B, void* C, i64 ldc, int c_dtype) {
    i64 strideB = N * Kd;
    if (dt == CATNN_BF16)
        gemm_grouped_bf16_tc(c, tb, rows, N, Kd, E, off, (const bf16*)A, lda, (const bf16*)B, strideB, tb ? Kd : N, C, ldc,
                             c_dtype, CATNN_ACT_NONE, false);
    else
        gemm_grouped_f32(c, false, tb, rows, N, Kd, E, off, (const float*)A, lda, (const float*)B, strideB, tb ? Kd : N,
                         (float*)C, ldc, 0, false);
}

static void expert_wgrad(Context* c, int dt, i64 rows, i64 N, i64 Kd, int E, const int32_t* off, const void* A, i64 lda,
                         const void* D, i64 ldd, float* dB) {
    if (dt == CATNN_BF16)
        gemm_grouped_wgrad_bf16_tc(c, rows, N, Kd, E, off, (const bf16*)A, lda, (const bf16*)D, ldd, dB, Kd * N, CATNN_F32,
                                   false);
    else
        gemm_grouped_f32(c, true, false, rows, N, Kd, E, off, (const float*)A, lda, (const float*)D, 0, ldd, dB, N, Kd * N,
                         false);
}

void MoeTrainer::forward() {
    int* err = c->status + 10;
    k_next_token<<<cdiv(T, 256), 256, 0, c->stream>>>(tokens, targets, tok_off, T, Tg, V);
    launched(c);
    if (ep) ep_embedding_fwd(c, tokens + tok_off, T, ptab(P + o_embed), V, Vs, d, acts[0].x_in, err);
    else embedding_fwd(c, tokens + tok_off, T, P + o_embed, V, d, acts[0].x_in, CATNN_F32, err);
    stamp("embedding");
    const int align = dt == CATNN_BF16 ? 128 : 1;
    for (i64 l = 0; l < L; ++l) {
        Act& a = acts[l];
        const LayerOff& q = lo[l];
        float* x_out = l + 1 < L ? acts[l + 1].x_in : x_last;
        char* qkv = (char*)a.qkv;
        size_t e = dsize(dt);
        // attention half: x_mid = x_in + attn(rmsnorm(x_in))   (moe.rs:303-316)
        rmsnorm_fwd_mixed(c, a.x_in, CATNN_F32, P + q.rms_attn, a.xn, dt, T, d, eps);
        gemm(c, false, false, T, qkvd, d, a.xn, d, W(q.wqkv), qkvd, a.qkv, qkvd, dt, dt, nullptr, 0, false);
        // q and k heads sit side by side at the front of each qkv row: one pass rotates both
        rope(c, qkv, B, S, H + Hkv, hd, theta, false, dt, qkvd, 0);
        attention_fwd(c, qkv, qkv + qd * e, qkv + (qd + kd) * e, a.ctx, a.lse, B, S, H, Hkv, hd, true, window, dt, qkvd,
                      qkvd);
        gemm(c, false, false, T, d, qd, a.ctx, qd, W(q.wo), d, a.x_mid, d, dt, CATNN_F32, nullptr, 0, false, a.x_in);
        stamp("fwd attention");
        // MoE half: x_out = x_mid + moe(rmsnorm(x_mid))   (moe.rs:317-319)
        // The router runs in fp32 on every path (fp32 normalized input, fp32
        // master gate): top-k decisions then match the reference's f32 logits
        // instead of flipping near ties on bf16-rounded inputs.
        if (dt != CATNN_BF16 || !rms_router_fused(c, a.x_mid, P + q.rms_moe, P + q.gate, E, T, d, eps, (bf16*)a.xm,
                                                  a.xm32, a.logits)) {
            rmsnorm_fwd_mixed(c, a.x_mid, CATNN_F32, P + q.rms_moe, a.xm, dt, T, d, eps);
            if (dt == CATNN_BF16) rmsnorm_fwd_mixed(c, a.x_mid, CATNN_F32, P + q.rms_moe, a.xm32, CATNN_F32, T, d, eps);
            gemm(c, false, false, T, E, d, a.xm32, d, P + q.gate, E, a.logits, E, CATNN_F32, CATNN_F32, nullptr, 0,
                 false);
        }
        router_topk(c, a.logits, T, E, K, a.idx, a.w);
        if (!ep) {
            permute_map(c, a.idx, T, E, K, align, cap, a.counts, a.off, a.row_of, a.src_of);
            permute_rows(c, a.xm, a.src_of, cap, d, K, a.xp, dt);
            if (ilv) {
                gemm_grouped_swiglu_fwd_tc(c, cap, F, d, (int)E, a.off, (const bf16*)a.xp, d, (const bf16*)W(q.w13),
                                           (bf16*)a.ac, (bf16*)a.h);
            } else {
                expert_gemm(c, dt, false, cap, 2 * F, d, (int)E, a.off, a.xp, d, W(q.w13), a.ac, 2 * F, dt);
                swiglu_act(c, a.ac, (char*)a.ac + F * e, a.h, cap, F, 2 * F, F, dt);
            }
            expert_gemm(c, dt, false, cap, d, F, (int)E, a.off, a.h, F, W(q.w2), a.yp, d, dt);
            unpermute_rows(c, a.yp, a.row_of, a.w, T, K, d, x_out, CATNN_F32, false, dt, a.x_mid);
        } else {
            // local counts and within-expert ranks (align 1), published to every rank
            permute_map(c, a.idx, T, E, K, 1, T * K, a.counts, a.off, a.row_of, src1);
            ep_publish_counts(c, a.counts, tab(a.cnt_all), rank, world, (int)E);
            comm->barrier();
            ep_plan(c, a.cnt_all, rank, world, (int)E, (int)El, align, a.plan, cap);
            stamp("moe route + counts");
            // rows straight into the owners' receive buffers
            ep_dispatch(c, a.xm, a.idx, a.row_of, a.off, a.plan, tab(a.xp), tab(a.src_of), a.dest, T, (int)K, d,
                        (int)El, align, rank, world, cap, dt);
            comm->barrier();
            stamp("moe dispatch");
            if (ilv) {
                gemm_grouped_swiglu_fwd_tc(c, cap, F, d, (int)El, a.plan, (const bf16*)a.xp, d, (const bf16*)W(q.w13),
                                           (bf16*)a.ac, (bf16*)a.h);
            } else {
                expert_gemm(c, dt, false, cap, 2 * F, d, (int)El, a.plan, a.xp, d, W(q.w13), a.ac, 2 * F, dt);
                swiglu_act(c, a.ac, (char*)a.ac + F * e, a.h, cap, F, 2 * F, F, dt, -1, a.plan + El);
            }
            expert_gemm(c, dt, false, cap, d, F, (int)El, a.plan, a.h, F, W(q.w2), a.yp, d, dt);
            stamp("moe experts");
            comm->barrier();
            // weighted sum read from the owners' expert outputs
            ep_combine(c, tab(a.yp), a.idx, a.dest, a.w, T, (int)K, d, (int)El, world, cap, x_out, a.x_mid, dt);
        }
        stamp("fwd moe");
    }
    // final norm, LM head, fused cross-entropy (dlogits overwrite logits)
    rmsnorm_fwd_mixed(c, x_last, CATNN_F32, P + o_final, xf, dt, T, d, eps);
    gemm(c, false, true, T, V, d, xf, d, W(o_lm), d, lg, V, dt, dt, nullptr, 0, false);
    // mean over the GLOBAL token count: the ranks' gradients then sum to the
    // one-GPU gradient, and so do their losses
    xent_fwdbwd(c, lg, targets, T, V, loss, lg, dt, c->status + 9, Tg);
    stamp("lm head + loss");
}

void MoeTrainer::backward() {
    size_t e = dsize(dt);
    // LM head adjoint (adjoint.rs:903-913) and the final norm
    gemm(c, false, false, T, d, V, lg, V, W(o_lm), d, dxf, d, dt, dt, nullptr, 0, false);
    gemm(c, true, false, V, d, T, lg, V, xf, d, G + o_lm, d, dt, CATNN_F32, nullptr, 0, false);
    rmsnorm_bwd_mixed(c, x_last, P + o_final, dxf, dt, nullptr, dx, nullptr, dt, G + o_final, false, T, d, eps);
    stamp("bwd lm head");
    // the loss rides in the gradient slot o_loss (summed over ranks with the
    // final norm's gradient while the layers' adjoints run)
    if (ep) CUDA_OK(cudaMemcpyAsync(G + o_loss, loss, 4, cudaMemcpyDeviceToDevice, c->stream));
    post_bucket(fin, (int)L);
    for (i64 l = L - 1; l >= 0; --l) {
        Act& a = acts[l];
        const LayerOff& q = lo[l];
        char* qkv = (char*)a.qkv;
        char* dq = (char*)dqkv;
        // MoE adjoint (adjoint.rs:471-526), batched by expert
        const int ng = ep ? (int)El : (int)E;
        const int32_t* goff = ep ? a.plan : a.off;
        const bool defer = ep && ilv;  // weight gradients on ws (see MoeTrainer::ws)
        if (!ep) {
            unpermute_bwd(c, a.yp, a.src_of, cap, a.w, dx, K, d, dwts, dyp, dt, dt, CATNN_F32);
        } else {
            join_wgrads();    // the previous layer's weight gradients have read dyp / dac
            comm->barrier();  // every rank's dx for this layer is final
            ep_unpermute_bwd(c, a.yp, a.src_of, a.plan, tab(a.w), tab(dx), tab(dwts), cap, T * K, (int)K, d, (int)El,
                             world, dyp, dt);
            stamp("moe bwd unpermute");
        }
        if (ilv) {
            gemm_grouped_swiglu_bwd_tc(c, cap, F, d, ng, goff, (const bf16*)dyp, d, (const bf16*)W(q.w2),
                                       (const bf16*)a.ac, (bf16*)dac);
            if (!defer) expert_wgrad(c, dt, cap, d, F, ng, goff, a.h, F, dyp, d, G + q.w2);
        } else {
            expert_gemm(c, dt, true, cap, F, d, ng, goff, dyp, d, W(q.w2), dh, F, dt);
            expert_wgrad(c, dt, cap, d, F, ng, goff, a.h, F, dyp, d, G + q.w2);
            swiglu_act_bwd(c, a.ac, (char*)a.ac + F * e, dh, dac, (char*)dac + F * e, cap, F, 2 * F, 2 * F, dt, -1,
                           ep ? a.plan + El : nullptr);
        }
        expert_gemm(c, dt, true, cap, d, 2 * F, ng, goff, dac, 2 * F, W(q.w13), dxp, d, dt);
        if (defer) {
            if (!ws) {
                CUDA_OK(cudaStreamCreateWithFlags(&ws, cudaStreamNonBlocking));
                CUDA_OK(cudaEventCreateWithFlags(&ev_w, cudaEventDisableTiming));
                CUDA_OK(cudaEventCreateWithFlags(&ev_wd, cudaEventDisableTiming));
            }
            CUDA_OK(cudaEventRecord(ev_w, c->stream));
            CUDA_OK(cudaStreamWaitEvent(ws, ev_w, 0));
            {
                // the split-K partials of these GEMMs must not share the
                // context's scratch with the GEMMs running on the step's stream
                std::swap(c->scratch, wscratch);
                std::swap(c->scratch_bytes, wscratch_bytes);
                OnStream on(c, ws);
                try {
                    expert_wgrad(c, dt, cap, d, F, ng, goff, a.h, F, dyp, d, G + q.w2);
                    expert_wgrad(c, dt, cap, 2 * F, d, ng, goff, a.xp, d, dac, 2 * F, G + q.w13);
                } catch (...) {
                    std::swap(c->scratch, wscratch);
                    std::swap(c->scratch_bytes, wscratch_bytes);
                    throw;
                }
                std::swap(c->scratch, wscratch);
                std::swap(c->scratch_bytes, wscratch_bytes);
            }
            CUDA_OK(cudaEventRecord(ev_wd, ws));
            w_forked = true;
        } else {
            expert_wgrad(c, dt, cap, 2 * F, d, ng, goff, a.xp, d, dac, 2 * F, G + q.w13);
        }
        if (ep) stamp("moe bwd experts");
        if (!ep) {
            permute_bwd(c, dxp, a.row_of, T, K, d, dxm, dt, false, CATNN_F32);
        } else {
            comm->barrier();  // owners' dxp rows and the dwts they wrote are final
            ep_permute_bwd(c, tab(dxp), a.idx, a.dest, T, (int)K, d, (int)El, world, cap, dxm, dt);
            stamp("moe bwd permute");
        }
        // router straight-through adjoint (adjoint.rs:255-284)
        router_ste(c, a.idx, a.w, dwts, T, E, K, dlog);
        gemm(c, false, true, T, d, E, dlog, E, P + q.gate, E, dxm, d, CATNN_F32, CATNN_F32, nullptr, 0, true);
        gemm(c, true, false, d, E, T, a.xm32, d, dlog, E, G + q.gate, E, CATNN_F32, CATNN_F32, nullptr, 0, false);
        // residual around the MoE: dx_mid = dx + rmsnorm'(dxm)   (train.rs:327-330)
        rmsnorm_bwd_mixed(c, a.x_mid, P + q.rms_moe, dxm, CATNN_F32, dx, dxmid, dxmid_lp, dt, G + q.rms_moe, false, T, d,
                          eps);
        stamp("bwd moe");
        // attention adjoint (adjoint.rs:287-439)
        gemm(c, false, true, T, qd, d, dxmid_lp, d, W(q.wo), d, dctx, qd, dt, dt, nullptr, 0, false);
        gemm(c, true, false, qd, d, T, a.ctx, qd, dxmid_lp, d, G + q.wo, d, dt, CATNN_F32, nullptr, 0, false);
        attention_bwd(c, qkv, qkv + qd * e, qkv + (qd + kd) * e, a.ctx, a.lse, dctx, dq, dq + qd * e, dq + (qd + kd) * e,
                      B, S, H, Hkv, hd, true, window, dt, qkvd, qkvd);
        rope(c, dq, B, S, H + Hkv, hd, theta, true, dt, qkvd, 0);
        gemm(c, false, true, T, d, qkvd, dqkv, qkvd, W(q.wqkv), qkvd, dxn, d, dt, dt, nullptr, 0, false);
        gemm(c, true, false, d, qkvd, T, a.xn, d, dqkv, qkvd, G + q.wqkv, qkvd, dt, CATNN_F32, nullptr, 0, false);
        // residual around attention: dx_in = dx_mid + rmsnorm'(dxn)   (train.rs:348-351)
        rmsnorm_bwd_mixed(c, a.x_in, P + q.rms_attn, dxn, dt, dxmid, dx, nullptr, dt, G + q.rms_attn, false, T, d, eps);
        stamp("bwd attention");
        // this layer's replicated gradients and its experts are final
        post_bucket(lb[l], (int)l);
        if (defer) update_after_event(ev_wd, q.w13, q.w2 + El * F * d - q.w13);
        else update_after_main(q.w13, q.w2 + El * F * d - q.w13);
    }
    join_wgrads();
    CUDA_OK(cudaStreamWaitEvent(c->stream, ev_kd, 0));  // the keys formed during the forward
    if (ep) {
        comm->barrier();  // every rank's token rows of dx are final
        ep_embedding_runs(c, emb_keys, emb_m, Tg, T, tab(dx), v0, v1, d, G + o_embed);
        stamp("bwd embedding");
        update_after_main(o_embed + v0 * d, (v1 - v0) * d);
        // the last all-gather also waits for the embedding update: once it
        // completes on any rank, every owner's rows are final for the next
        // step's gather
        if (upd_pending && !pend.empty()) CUDA_OK(cudaEventRecord(ev_g[pend.back()], us));
        flush_gathers();
    } else {
        embedding_bwd_runs(c, emb_keys, T, dx, G + o_embed, V, d, CATNN_F32);
        stamp("bwd embedding");
        update_after_main(o_embed, V * d);
    }
}

void MoeTrainer::post_bucket(const Bucket& b, int id) {
    if (!ep) {
        update_after_main(b.s_off, b.b_off + b.b_len - b.s_off);
        return;
    }
    comm->allreduce_overlapped(G + b.s_off, b.s_len);
    update_after_comm(b.s_off, b.s_len);
    comm->reduce_scatter_overlapped(G + b.b_off, b.b_len);
    const i64 chunk = b.b_len / world;
    update_after_comm(b.b_off + rank * chunk, chunk);
    // the previous bucket's all-gather queues behind this reduce-scatter:
    // its chunk's update has had the time in between
    flush_gathers();
    if (upd_pending) {
        CUDA_OK(cudaEventRecord(ev_g[id], us));
        pend.push_back(id);
    }
}

void MoeTrainer::flush_gathers() {
    for (int id : pend) {
        const Bucket& b = id == (int)L ? fin : lb[id];
        comm->allgather_after((char*)Sh + b.b_off * dsize(dt), b.b_len, dt, ev_g[id]);
    }
    pend.clear();
}

void MoeTrainer::gather_shards(float* base) {
    if (!ep) return;
    comm->allgather(base + o_embed, world * Vs * d, CATNN_F32);
    for (i64 l = 0; l < L; ++l) comm->allgather(base + lb[l].b_off, lb[l].b_len, CATNN_F32);
    comm->allgather(base + fin.b_off, fin.b_len, CATNN_F32);
}

// optim.rs:32-43 (SGD) / :95-119 (Adam) on parameters [off, off + n).
void MoeTrainer::update_range(i64 off, i64 n) {
    if (n <= 0) return;
    bf16* sh = dt == CATNN_BF16 ? (bf16*)Sh + off : nullptr;
    if (opt == 0) sgd(c, P + off, G + off, n, lr, sh);
    else adam(c, P + off, G + off, Mo + off, Vo + off, n, t_step, lr, b1, b2, aeps, CATNN_F32, sh, d12);
}


static void make_update_stream(cudaStream_t* us, cudaEvent_t* a, cudaEvent_t* b) {
    if (*us) return;
    int lo = 0, hi = 0;
    CUDA_OK(cudaDeviceGetStreamPriorityRange(&lo, &hi));
    CUDA_OK(cudaStreamCreateWithPriority(us, cudaStreamNonBlocking, lo));  // lowest: the backward pass goes first
    CUDA_OK(cudaEventCreateWithFlags(a, cudaEventDisableTiming));
    CUDA_OK(cudaEventCreateWithFlags(b, cudaEventDisableTiming));
}

void MoeTrainer::update_after_main(i64 off, i64 n) {
    if (!upd_pending || n <= 0) return;
    make_update_stream(&us, &ev_u, &ev_u_done);
    CUDA_OK(cudaEventRecord(ev_u, c->stream));
    CUDA_OK(cudaStreamWaitEvent(us, ev_u, 0));
    upd_forked = true;
    OnStream on(c, us);
    update_range(off, n);
}

void MoeTrainer::update_after_comm(i64 off, i64 n) {
    if (!upd_pending || n <= 0) return;
    make_update_stream(&us, &ev_u, &ev_u_done);
    CUDA_OK(cudaEventRecord(ev_u, comm->side));
    CUDA_OK(cudaStreamWaitEvent(us, ev_u, 0));
    upd_forked = true;
    OnStream on(c, us);
    update_range(off, n);
}

void MoeTrainer::update_after_event(cudaEvent_t ev, i64 off, i64 n) {
    if (!upd_pending || n <= 0) return;
    make_update_stream(&us, &ev_u, &ev_u_done);
    CUDA_OK(cudaStreamWaitEvent(us, ev, 0));
    upd_forked = true;
    OnStream on(c, us);
    update_range(off, n);
}

void MoeTrainer::join_wgrads() {
    if (!w_forked) return;
    w_forked = false;
    CUDA_OK(cudaStreamWaitEvent(c->stream, ev_wd, 0));
}

void MoeTrainer::join_updates() {
    // only a step that forked updates onto us joins it (inside a graph capture
    // a wait on work the capture never forked is an error)
    if (!us || !upd_forked) return;
    upd_forked = false;
    CUDA_OK(cudaEventRecord(ev_u_done, us));
    CUDA_OK(cudaStreamWaitEvent(c->stream, ev_u_done, 0));
}

void MoeTrainer::run_body() {
    stamp_names.clear();
    stamp("start");
    // the embedding backward's key sort needs only the token ids: it runs on
    // the update stream (idle until the first bucket's update) during the forward
    make_update_stream(&us, &ev_u, &ev_u_done);
    if (!ev_k) {
        CUDA_OK(cudaEventCreateWithFlags(&ev_k, cudaEventDisableTiming));
        CUDA_OK(cudaEventCreateWithFlags(&ev_kd, cudaEventDisableTiming));
    }
    CUDA_OK(cudaEventRecord(ev_k, c->stream));
    CUDA_OK(cudaStreamWaitEvent(us, ev_k, 0));
    {
        OnStream on(c, us);
        if (ep) ep_embedding_keys(c, tokens, Tg, v0, v1, emb_keys, emb_m);
        else embedding_bwd_keys(c, tokens + tok_off, T, V, emb_keys);
    }
    CUDA_OK(cudaEventRecord(ev_kd, us));
    forward();
    backward();  // enqueues the gradient allreduces and the updates bucket by bucket
    if (ep) {
        // The last allreduce completes only once every rank has finished its
        // backward pass, so no rank's next dispatch can overwrite a buffer a
        // peer still reads.
        comm->join_overlapped();
        CUDA_OK(cudaMemcpyAsync(loss, G + o_loss, 4, cudaMemcpyDeviceToDevice, c->stream));
        stamp("gradient all-reduce joined");
    }
    join_updates();
    stamp("updates joined");
}

void MoeTrainer::drop_graphs() {
    for (int k = 0; k < 2; ++k) {
        if (gexec[k]) cudaGraphExecDestroy(gexec[k]);
        gexec[k] = nullptr;
        warmed[k] = false;
    }
}

void MoeTrainer::step(const uint32_t* tokens_dev, float* loss_dev, bool upd) {
    if (tokens_dev != tokens) CUDA_OK(cudaMemcpyAsync(tokens, tokens_dev, Tg * 4, cudaMemcpyDeviceToDevice, c->stream));
    upd_pending = upd;
    if (upd && opt == 1) {
        ++t_step;
        // the divisors travel through device memory, so a replayed graph sees this step's
        float h12[2];
        adam_divisors(t_step, b1, b2, h12);
        CUDA_OK(cudaMemcpyAsync(d12, h12, sizeof(h12), cudaMemcpyHostToDevice, c->stream));
    }
    if (graphs) {
        const int key = upd ? 1 : 0;
        CUDA_OK(cudaEventRecord(ev_in, c->stream));
        CUDA_OK(cudaStreamWaitEvent(gs, ev_in, 0));
        {
            OnStream on(c, gs);
            if (gexec[key]) {
                CUDA_OK(cudaGraphLaunch(gexec[key], gs));
                c->launches += glaunch[key];
            } else if (!warmed[key]) {
                run_body();  // eager: every workspace reaches its size before a capture
                warmed[key] = true;
            } else {
                const uint64_t l0 = c->launches;
                CUDA_OK(cudaStreamBeginCapture(gs, cudaStreamCaptureModeThreadLocal));
                cudaGraph_t g = nullptr;
                try {
                    run_body();
                } catch (...) {
                    cudaStreamEndCapture(gs, &g);
                    if (g) cudaGraphDestroy(g);
                    throw;
                }
                CUDA_OK(cudaStreamEndCapture(gs, &g));
                glaunch[key] = c->launches - l0;
                cudaGraphExec_t ex = nullptr;
                cudaError_t e = cudaGraphInstantiate(&ex, g, 0);
                cudaGraphDestroy(g);
                CUDA_OK(e);
                gexec[key] = ex;
                CUDA_OK(cudaGraphLaunch(ex, gs));  // the captured step has not run yet
            }
        }
        CUDA_OK(cudaEventRecord(ev_out, gs));
        CUDA_OK(cudaStreamWaitEvent(c->stream, ev_out, 0));
    } else {
        run_body();
    }
    upd_pending = false;
    if (loss_dev && loss_dev != loss) CUDA_OK(cudaMemcpyAsync(loss_dev, loss, 4, cudaMemcpyDeviceToDevice, c->stream));
}

}  // namespace catnn

using namespace catnn;

struct catnn_moe_trainer {
    MoeTrainer t;
};

namespace {

MoeTrainer& tr(catnn_moe_trainer* h) {
    CATNN_CHECK(h != nullptr, CATNN_ERR_INVALID, "null catnn_moe_trainer");
    bind(h->t.c);
    return h->t;
}

void configure(MoeTrainer& t, const catnn_moe_config* cf, int rank = 0, int world = 1) {
    CATNN_CHECK(cf != nullptr, CATNN_ERR_INVALID, "null config");
    t.rank = rank;
    t.world = world;
    t.ep = world > 1;
    t.V = cf->vocab;
    t.d = cf->hidden;
    t.F = cf->mid;
    t.L = cf->layers;
    t.H = cf->heads;
    t.Hkv = cf->kv_heads;
    t.E = cf->experts;
    t.K = cf->top_k;
    t.window = cf->window;
    t.B = cf->batch;
    t.S = cf->seq;
    t.eps = cf->rms_eps;
    t.theta = cf->rope_theta;
    t.dt = cf->dtype;
    t.opt = cf->optimizer;
    t.lr = cf->lr;
    t.b1 = cf->beta1;
    t.b2 = cf->beta2;
    t.aeps = cf->adam_eps;
    check_dtype(t.dt);
    CATNN_CHECK(t.V > 0 && t.d > 0 && t.F > 0 && t.L > 0 && t.B > 0 && t.S > 0, CATNN_ERR_SHAPE, "moe config: sizes");
    CATNN_CHECK(t.H > 0 && t.d % t.H == 0, CATNN_ERR_SHAPE, "hidden not divisible by heads");
    CATNN_CHECK(t.Hkv > 0 && t.H % t.Hkv == 0, CATNN_ERR_SHAPE, "heads not divisible by kv heads");
    CATNN_CHECK(t.E >= 1 && t.E <= 32 && t.K >= 1 && t.K <= t.E, CATNN_ERR_SHAPE, "need 1 <= top_k <= experts <= 32");
    CATNN_CHECK(t.opt == 0 || t.opt == 1, CATNN_ERR_INVALID, "optimizer: 0 = SGD, 1 = Adam");
    t.hd = t.d / t.H;
    CATNN_CHECK(t.hd % 2 == 0 && t.hd <= 128, CATNN_ERR_SHAPE, "head_dim must be even and <= 128");
    CATNN_CHECK(t.B % world == 0, CATNN_ERR_SHAPE,
                "expert parallel: batch " + std::to_string(t.B) + " not divisible by " + std::to_string(world) + " ranks");
    CATNN_CHECK(t.E % world == 0, CATNN_ERR_SHAPE,
                "expert parallel: experts " + std::to_string(t.E) + " not divisible by " + std::to_string(world) + " ranks");
    t.Bg = t.B;
    t.Tg = t.B * t.S;
    t.B = t.Bg / world;
    t.T = t.B * t.S;
    t.tok_off = (i64)rank * t.T;
    t.El = t.E / world;
    t.e0 = (i64)rank * t.El;
    t.qd = t.H * t.hd;
    t.kd = t.Hkv * t.hd;
    t.qkvd = t.qd + 2 * t.kd;
    const i64 align = t.dt == CATNN_BF16 ? 128 : 1;
    // worst case: every pair of the global batch that can reach this rank's
    // experts (a token's top-k experts are distinct) does, plus padding
    t.cap = t.Tg * std::min(t.K, t.El) + t.El * (align - 1);
    CATNN_CHECK(t.Tg * t.K < (1ll << 31), CATNN_ERR_SHAPE, "too many (token, slot) pairs");
    if (t.dt == CATNN_BF16)
        CATNN_CHECK(t.d % 64 == 0 && t.F % 64 == 0, CATNN_ERR_SHAPE, "bf16 path: hidden and mid must be multiples of 64");
    t.ilv = t.dt == CATNN_BF16 && t.F % 128 == 0;
}

}  // namespace

extern "C" {

int catnn_moe_trainer_create(catnn_ctx* h, const catnn_moe_config* cf, catnn_moe_trainer** out) {
    ABI_BEGIN
    Context* c = unwrap(h);
    CATNN_CHECK(out != nullptr, CATNN_ERR_INVALID, "null out");
    catnn_moe_trainer* t = new catnn_moe_trainer();
    try {
        t->t.c = c;
        configure(t->t, cf);
        t->t.plan_params();
        t->t.alloc();
    } catch (...) {
        t->t.release();
        delete t;
        throw;
    }
    *out = t;
    ABI_END
}

int catnn_moe_trainer_create_ep(catnn_ctx* h, const catnn_moe_config* cf, catnn_comm* cm, catnn_moe_trainer** out) {
    ABI_BEGIN
    Context* c = unwrap(h);
    CATNN_CHECK(out != nullptr, CATNN_ERR_INVALID, "null out");
    Comm* comm = comm_of(cm);
    CATNN_CHECK(comm->c == c, CATNN_ERR_INVALID, "trainer and communicator must share the context");
    catnn_moe_trainer* t = new catnn_moe_trainer();
    try {
        t->t.c = c;
        t->t.comm = comm;
        configure(t->t, cf, comm->rank, comm->world);
        t->t.plan_params();
        t->t.alloc();
    } catch (...) {
        t->t.release();
        delete t;
        throw;
    }
    *out = t;
    ABI_END
}

int catnn_moe_trainer_set_graphs(catnn_moe_trainer* h, int enable) {
    ABI_BEGIN
    MoeTrainer& t = tr(h);
    if (enable && !t.gs) {
        CUDA_OK(cudaStreamCreateWithFlags(&t.gs, cudaStreamNonBlocking));
        CUDA_OK(cudaEventCreateWithFlags(&t.ev_in, cudaEventDisableTiming));
        CUDA_OK(cudaEventCreateWithFlags(&t.ev_out, cudaEventDisableTiming));
    }
    if (!enable) {
        if (t.gs) CUDA_OK(cudaStreamSynchronize(t.gs));
        t.drop_graphs();
    }
    t.graphs = enable != 0;
    ABI_END
}

int catnn_moe_trainer_set_profile(catnn_moe_trainer* h, int enable) {
    ABI_BEGIN
    MoeTrainer& t = tr(h);
    if (enable && !t.stamps) {
        CUDA_OK(cudaMalloc(&t.stamps, MoeTrainer::MAX_STAMPS * sizeof(unsigned long long)));
        CUDA_OK(cudaMemsetAsync(t.stamps, 0, MoeTrainer::MAX_STAMPS * sizeof(unsigned long long), t.c->stream));
    }
    if ((enable != 0) != t.prof) {
        // the step body changes: captured graphs no longer match it
        if (t.gs) CUDA_OK(cudaStreamSynchronize(t.gs));
        t.drop_graphs();
    }
    t.prof = enable != 0;
    ABI_END
}

int catnn_moe_trainer_timeline(catnn_moe_trainer* h, int64_t* ns, int max, char* names, int64_t names_len, int* count) {
    ABI_BEGIN
    MoeTrainer& t = tr(h);
    CATNN_CHECK(ns && names && count && max >= 0 && names_len > 0, CATNN_ERR_INVALID, "null argument");
    CATNN_CHECK(t.stamps != nullptr, CATNN_ERR_INVALID, "profiling was never enabled on this trainer");
    const int n = std::min<int>((int)t.stamp_names.size(), max);
    std::vector<unsigned long long> host(MoeTrainer::MAX_STAMPS);
    if (t.gs) CUDA_OK(cudaStreamSynchronize(t.gs));
    CUDA_OK(cudaStreamSynchronize(t.c->stream));
    CUDA_OK(cudaMemcpy(host.data(), t.stamps, MoeTrainer::MAX_STAMPS * sizeof(unsigned long long),
                       cudaMemcpyDeviceToHost));
    std::string all;
    for (int i = 0; i < n; ++i) {
        ns[i] = (int64_t)host[i];
        all += t.stamp_names[i];
        all += '\n';
    }
    CATNN_CHECK((int64_t)all.size() < names_len, CATNN_ERR_INVALID, "names buffer too small");
    std::memcpy(names, all.c_str(), all.size() + 1);
    *count = n;
    ABI_END
}

int catnn_moe_trainer_destroy(catnn_moe_trainer* h) {
    ABI_BEGIN
    if (!h) return CATNN_OK;
    bind(h->t.c);
    cudaStreamSynchronize(h->t.c->stream);
    h->t.release();
    delete h;
    ABI_END
}

int catnn_moe_trainer_param_count(const catnn_moe_config* cf, int64_t* out) {
    ABI_BEGIN
    CATNN_CHECK(out != nullptr, CATNN_ERR_INVALID, "null out");
    MoeTrainer t;
    configure(t, cf);
    *out = t.packed_count();
    ABI_END
}

int catnn_moe_trainer_set_params(catnn_moe_trainer* h, const float* packed) {
    ABI_BEGIN
    MoeTrainer& t = tr(h);
    CATNN_CHECK(packed != nullptr, CATNN_ERR_INVALID, "null params");
    t.import_packed(packed, t.P);
    if (t.dt == CATNN_BF16) cast(t.c, t.P, CATNN_F32, t.Sh, CATNN_BF16, t.n_params);
    if (t.opt == 1) {
        CUDA_OK(cudaMemsetAsync(t.Mo, 0, t.n_params * 4, t.c->stream));
        CUDA_OK(cudaMemsetAsync(t.Vo, 0, t.n_params * 4, t.c->stream));
        t.t_step = 0;
    }
    // peers read the embedding rows this rank owns from the next step on
    if (t.ep) t.comm->barrier();
    ABI_END
}

int catnn_moe_trainer_get_params(catnn_moe_trainer* h, float* packed) {
    ABI_BEGIN
    MoeTrainer& t = tr(h);
    CATNN_CHECK(packed != nullptr, CATNN_ERR_INVALID, "null out");
    t.gather_shards(t.P);
    t.export_packed(t.P, packed);
    ABI_END
}

int catnn_moe_trainer_get_grads(catnn_moe_trainer* h, float* packed) {
    ABI_BEGIN
    MoeTrainer& t = tr(h);
    CATNN_CHECK(packed != nullptr, CATNN_ERR_INVALID, "null out");
    t.gather_shards(t.G);
    t.export_packed(t.G, packed);
    ABI_END
}

int catnn_moe_trainer_step(catnn_moe_trainer* h, const uint32_t* tokens, float* loss, int update) {
    ABI_BEGIN
    MoeTrainer& t = tr(h);
    CATNN_CHECK(tokens != nullptr, CATNN_ERR_INVALID, "null tokens");
    t.step(tokens, loss, update != 0);
    ABI_END
}

int catnn_moe_trainer_step_host(catnn_moe_trainer* h, const uint32_t* tokens_host, float* loss_host, int update) {
    ABI_BEGIN
    MoeTrainer& t = tr(h);
    CATNN_CHECK(tokens_host != nullptr && loss_host != nullptr, CATNN_ERR_INVALID, "null tokens/loss");
    // host -> pinned staging -> device, step, loss back to the host
    std::memcpy(t.h_tokens, tokens_host, t.Tg * 4);
    CUDA_OK(cudaMemcpyAsync(t.tokens, t.h_tokens, t.Tg * 4, cudaMemcpyHostToDevice, t.c->stream));
    t.step(t.tokens, nullptr, update != 0);
    CUDA_OK(cudaMemcpyAsync(t.h_loss, t.loss, 4, cudaMemcpyDeviceToHost, t.c->stream));
    CUDA_OK(cudaStreamSynchronize(t.c->stream));
    *loss_host = *t.h_loss;
    ABI_END
}

int catnn_moe_trainer_activation(catnn_moe_trainer* h, int which, int64_t layer, float* out) {
    ABI_BEGIN
    MoeTrainer& t = tr(h);
    CATNN_CHECK(out != nullptr, CATNN_ERR_INVALID, "null out");
    CATNN_CHECK(which == 5 || which == 6 || (layer >= 0 && layer < t.L), CATNN_ERR_INVALID, "layer out of range");
    const MoeTrainer::Act* a = which < 5 ? &t.acts[layer] : nullptr;
    switch (which) {
        case 0: CUDA_OK(cudaMemcpyAsync(out, a->x_in, t.T * t.d * 4, cudaMemcpyDeviceToDevice, t.c->stream)); break;
        case 1: CUDA_OK(cudaMemcpyAsync(out, a->x_mid, t.T * t.d * 4, cudaMemcpyDeviceToDevice, t.c->stream)); break;
        case 2: cast(t.c, a->xm, t.dt, out, CATNN_F32, t.T * t.d); break;
        case 3: cast(t.c, a->ctx, t.dt, out, CATNN_F32, t.T * t.qd); break;
        case 4: CUDA_OK(cudaMemcpyAsync(out, a->logits, t.T * t.E * 4, cudaMemcpyDeviceToDevice, t.c->stream)); break;
        case 5: CUDA_OK(cudaMemcpyAsync(out, t.x_last, t.T * t.d * 4, cudaMemcpyDeviceToDevice, t.c->stream)); break;
        case 6: cast(t.c, t.xf, t.dt, out, CATNN_F32, t.T * t.d); break;
        default: throw Error(CATNN_ERR_INVALID, "activation: which in 0..6");
    }
    ABI_END
}

int catnn_moe_trainer_check(catnn_moe_trainer* h) {
    ABI_BEGIN
    MoeTrainer& t = tr(h);
    int v[16];
    CUDA_OK(cudaMemcpyAsync(v, t.c->status, sizeof(v), cudaMemcpyDeviceToHost, t.c->stream));
    CUDA_OK(cudaStreamSynchronize(t.c->stream));
    if (v[8] || v[9] || v[10]) {
        CUDA_OK(cudaMemsetAsync(t.c->status + 8, 0, 3 * 4, t.c->stream));
        throw Error(CATNN_ERR_SHAPE, v[10] ? "token id >= vocab" : (v[9] ? "ce target out of range"
                                                                         : "router produced an invalid expert"));
    }
    if (v[0] || v[1] || v[2] || v[3]) throw Error(CATNN_ERR_TIMEOUT, "a bounded device wait ran out (GEMM pipeline)");
    if (v[EP_STATUS_SLOT]) throw Error(CATNN_ERR_INVALID, "expert-parallel receive buffer overflow");
    if (v[COMM_STATUS_SLOT]) {
        CUDA_OK(cudaMemsetAsync(t.c->status + COMM_STATUS_SLOT, 0, 8, t.c->stream));
        throw Error(CATNN_ERR_TIMEOUT, "a device wait for another rank ran out (epoch " +
                                           std::to_string(v[COMM_STATUS_SLOT + 1]) + ")");
    }
    ABI_END
}

}  // extern "C"
