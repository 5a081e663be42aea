// Native training step for the Mixtral-style MoE decoder (the reference's
// train::mixtral_step, crates/catnn-compile/src/train.rs:261-356, with
// residual adds, next-token cross-entropy and an SGD or Adam update).
#pragma once
#include <vector>

#include "ops.cuh"

struct catnn_moe_config;

namespace catnn {

struct Comm;     // expert-parallel communicator (comm.cu); null on one GPU
struct PeerTab;  // moe_ep.cuh

struct MoeTrainer {
    Context* c = nullptr;
    Comm* comm = nullptr;
    // group: this rank trains tokens [tok_off, tok_off + T) of the global
    // batch (Tg tokens) and owns experts [e0, e0 + El)
    int rank = 0, world = 1;
    bool ep = false;
    i64 Bg, Tg, tok_off, El, e0;
    // shapes (B, T: this rank's sequences and tokens; cap: expert rows this
    // rank can receive, padding included)
    i64 V, d, F, L, H, Hkv, hd, E, K, window, B, S, T, qd, kd, qkvd, cap;
    float eps;
    double theta;
    int dt;  // activation / weight-shadow storage (CATNN_F32 or CATNN_BF16)
    // bf16 path with F a multiple of 128: the expert GEMMs carry the SwiGLU in
    // their epilogues, and w13 / its gradient / the saved [a | c] rows use the
    // 128-column interleaved layout (blocks [w1 cols 128j.. | w3 cols 128j..])
    bool ilv = false;
    int opt;  // 0 SGD, 1 Adam
    float lr, b1, b2, aeps;
    uint64_t t_step = 0;

    // parameters: fp32 master P, gradients G, Adam moments Mo/Vo, and the
    // storage-dtype shadow S the GEMMs read (S == P on the fp32 path).
    struct LayerOff {
        i64 rms_attn, wqkv, wo, rms_moe, gate, w13, w2;
    };
    std::vector<LayerOff> lo;
    // replicated parameters (and the loss slot) come first, [0, n_rep); this
    // rank's experts follow. Under expert parallelism (world ranks):
    //  - the embedding table is vocab-sharded: rank r owns rows [r*Vs, r*Vs + Vs)
    //    (its gradient, optimizer update and authoritative copy); the forward
    //    gathers token rows from the owners over NVLink;
    //  - every other replicated tensor sits in a bucket (the final norm + loss
    //    slot + LM head, and one per layer). A bucket's small part (norm and
    //    router weights, read in fp32) is allreduced and updated on every rank;
    //    its big part (the GEMM weights, length a multiple of world*128) is
    //    reduce-scattered, each rank updates its chunk, and the updated
    //    storage-dtype copy is all-gathered. The fp32 master of another rank's
    //    chunk is then stale until get_params gathers it.
    struct Bucket {
        i64 s_off, s_len, b_off, b_len;
    };
    Bucket fin{};
    std::vector<Bucket> lb;
    i64 Vs = 0, v0 = 0, v1 = 0;
    i64 o_embed, o_final, o_lm, o_loss, n_rep, n_params;
    float *P = nullptr, *G = nullptr, *Mo = nullptr, *Vo = nullptr;
    void* Sh = nullptr;
    void* param_block = nullptr;

    // saved activations per layer
    struct Act {
        float *x_in, *x_mid, *lse, *logits, *w;
        void *xn, *qkv, *ctx, *xm, *xp, *ac, *h, *yp;
        float* xm32;  // fp32 router input (bf16 path; == xm on the fp32 path)
        int32_t *idx, *counts, *off, *row_of, *src_of;
        // expert parallel: counts of every rank [world][E], the layer plan
        // (moe_ep.cuh) and each local pair's row in its owner's buffer
        int32_t *cnt_all = nullptr, *plan = nullptr, *dest = nullptr;
    };
    std::vector<Act> acts;
    float* x_last = nullptr;
    void *xf = nullptr, *lg = nullptr;
    uint32_t *tokens = nullptr, *targets = nullptr;
    float* loss = nullptr;
    // backward scratch (reused across layers)
    float *dx, *dxmid, *dxm, *dlog, *dwts;
    void *dxmid_lp, *dyp, *dh, *dac, *dxp, *dqkv, *dctx, *dxn, *dlog_lp, *dxf;
    void* act_block = nullptr;
    size_t act_bytes = 0;
    int32_t* src1 = nullptr;  // local align-1 map's row sources (expert parallel)
    // the embedding backward's sorted (id, token) keys: they depend on the
    // token ids only, so they are formed on the update stream during the forward
    uint32_t* emb_keys = nullptr;
    int* emb_m = nullptr;
    cudaEvent_t ev_k = nullptr, ev_kd = nullptr;
    int map_id = -1;          // act_block's entry in comm->maps
    int map_pid = -1;         // param_block's entry in comm->maps
    std::vector<cudaEvent_t> ev_g;  // per bucket (layers, then the final one): its chunk's update is done
    std::vector<int> pend;          // buckets whose all-gather is not yet enqueued
    template <typename Q>
    PeerTab tab(Q* local) const;   // a buffer of act_block on every rank
    template <typename Q>
    PeerTab ptab(Q* local) const;  // a buffer of param_block on every rank
    // host staging for the host-buffer step
    uint32_t* h_tokens = nullptr;
    float* h_loss = nullptr;

    void plan_params();
    void alloc();
    void release();
    const void* W(i64 off) const { return (const char*)Sh + off * dsize(dt); }
    void forward();
    void backward();
    // Optimizer updates run on a low-priority side stream, bucket by bucket,
    // as soon as a bucket's gradients are final (summed over ranks when
    // replicated), overlapping the rest of the backward pass.
    bool upd_pending = false;
    bool upd_forked = false;  // this step enqueued work on us
    cudaStream_t us = nullptr;
    cudaEvent_t ev_u = nullptr, ev_u_done = nullptr;
    // CUDA-graph replay of the single-GPU step (catnn_moe_trainer_set_graphs):
    // the body (forward, backward, updates) runs on the trainer's own stream
    // gs; the first step of each kind (with / without update) runs eagerly
    // and sizes every workspace, the second is captured, later ones replay.
    bool graphs = false;
    cudaStream_t gs = nullptr;
    cudaEvent_t ev_in = nullptr, ev_out = nullptr;
    cudaGraphExec_t gexec[2] = {nullptr, nullptr};
    bool warmed[2] = {false, false};
    uint64_t glaunch[2] = {0, 0};
    float* d12 = nullptr;  // device [2]: Adam bias-correction divisors of the running step
    // phase timeline (catnn_moe_trainer_set_profile): device clock stamps taken
    // on the step's stream at phase boundaries
    static constexpr int MAX_STAMPS = 64;
    bool prof = false;
    unsigned long long* stamps = nullptr;  // device [MAX_STAMPS]
    std::vector<const char*> stamp_names;
    void stamp(const char* name);
    void run_body();
    void drop_graphs();
    void update_range(i64 off, i64 n);          // on the context's current stream
    void update_after_main(i64 off, i64 n);     // on us, after the work enqueued so far
    void update_after_comm(i64 off, i64 n);     // on us, after the last allreduce enqueued
    void join_updates();
    // Expert parallel: the expert weight-gradient GEMMs run on their own
    // stream (ws) with their own split-K scratch, beside the barrier, the
    // permute adjoint and the attention adjoint that follow. No other rank
    // waits for them, so the barrier after the expert GEMMs waits only for
    // the slowest rank's data-gradient GEMMs. The next layer's adjoint (which
    // rewrites dyp / dac) and the experts' update wait for ev_wd.
    cudaStream_t ws = nullptr;
    cudaEvent_t ev_w = nullptr, ev_wd = nullptr;
    bool w_forked = false;
    void* wscratch = nullptr;
    size_t wscratch_bytes = 0;
    void join_wgrads();
    void update_after_event(cudaEvent_t ev, i64 off, i64 n);  // on us, after ev
    // a bucket's gradients are final: sum and update them (see Bucket)
    void post_bucket(const Bucket& b, int id);
    void flush_gathers();
    // expert parallel: make the fp32 master (or the gradients) whole on every
    // rank before an export. Collective.
    void gather_shards(float* base);
    void step(const uint32_t* tokens_dev, float* loss_dev, bool upd);
    void import_packed(const float* packed, float* dst);
    void export_packed(const float* src, float* packed);
    i64 packed_count() const;
};

}  // namespace catnn
