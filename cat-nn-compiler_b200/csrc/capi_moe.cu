// extern "C" entry points for the MoE path (router, permutation, SwiGLU
// experts, the full MoE block and its adjoint), the optimizers and the MLP
// training step.
#include "ops.cuh"

using namespace catnn;

namespace {

void need(bool ok, const char* what) { CATNN_CHECK(ok, CATNN_ERR_INVALID, std::string("null argument: ") + what); }
void shape(bool ok, const std::string& what) { CATNN_CHECK(ok, CATNN_ERR_SHAPE, what); }


// Row alignment of the expert blocks: tensor-core tiles are 128 rows.
int moe_align(int dtype) { return dtype == CATNN_BF16 ? 128 : 1; }

// Expert GEMM over the expert-sorted rows: C[rows_g] = A[rows_g] · op(B_g).
void grouped(Context* c, int dtype, bool tb, i64 rows, i64 N, i64 K, int E, const int32_t* off, const void* A, const void* B,
             void* C, bool accumulate, int c_dtype = -1) {
    i64 strideB = N * K;
    if (c_dtype < 0) c_dtype = dtype;
    if (dtype == CATNN_BF16)
        gemm_grouped_bf16_tc(c, tb, rows, N, K, E, off, (const bf16*)A, K, (const bf16*)B, strideB, tb ? K : N, C, N,
                             c_dtype, CATNN_ACT_NONE, accumulate);
    else
        gemm_grouped_f32(c, false, tb, rows, N, K, E, off, (const float*)A, K, (const float*)B, strideB, tb ? K : N,
                         (float*)C, N, 0, accumulate);
}

// Per-expert weight gradient dB_g [K, N] = A_gᵀ · D_g.
void grouped_wgrad(Context* c, int dtype, i64 rows, i64 N, i64 K, int E, const int32_t* off, const void* A, const void* D,
                   void* dB) {
    if (dtype == CATNN_BF16)
        gemm_grouped_wgrad_bf16_tc(c, rows, N, K, E, off, (const bf16*)A, K, (const bf16*)D, N, dB, K * N, CATNN_BF16, false);
    else
        gemm_grouped_f32(c, true, false, rows, N, K, E, off, (const float*)A, K, (const float*)D, 0, N, (float*)dB, N, K * N,
                         false);
}

struct MoeTemps {
    float *logits, *w, *dwt, *dlog;
    int32_t *idx, *counts, *off, *row_of, *src_of;
    void *xp, *a, *cc, *hh, *yp, *dyp, *dh, *da, *dc, *dxp, *dlog_lp;
    i64 rows_cap;
};

// Pre-activations (a, c), expert outputs (yp) and dh stay fp32 on every
// path: the bf16 path rounds only the tensors that feed a tensor-core GEMM
// (xp, h, dyp, da, dc) and the block output.
MoeTemps moe_temps(Context* c, i64 T, i64 H, i64 F, i64 E, i64 k, int dtype, bool bwd) {
    size_t e = dsize(dtype);
    const size_t f4 = 4;
    i64 P = T * k;
    i64 cap = P + E * (moe_align(dtype) - 1);
    std::initializer_list<size_t> sizes = {
        (size_t)T * E * 4, (size_t)P * 4, (size_t)P * 4, (size_t)T * E * 4, (size_t)P * 4, (size_t)E * 4,
        (size_t)(E + 1) * 4, (size_t)P * 4, (size_t)cap * 4, cap * H * e, cap * F * f4, cap * F * f4, cap * F * e,
        cap * H * f4, cap * H * e, cap * F * f4, cap * F * e, cap * F * e, cap * H * e, (size_t)T * E * e};
    Carver cv(c->work_for(Carver::need(sizes)));
    MoeTemps t{};
    t.rows_cap = cap;
    t.logits = cv.take<float>(T * E);
    t.w = cv.take<float>(P);
    t.dwt = cv.take<float>(P);
    t.dlog = cv.take<float>(T * E);
    t.idx = cv.take<int32_t>(P);
    t.counts = cv.take<int32_t>(E);
    t.off = cv.take<int32_t>(E + 1);
    t.row_of = cv.take<int32_t>(P);
    t.src_of = cv.take<int32_t>(cap);
    t.xp = cv.take<char>(cap * H * e);
    t.a = cv.take<char>(cap * F * f4);
    t.cc = cv.take<char>(cap * F * f4);
    t.hh = cv.take<char>(cap * F * e);
    t.yp = cv.take<char>(cap * H * f4);
    if (bwd) {
        t.dyp = cv.take<char>(cap * H * e);
        t.dh = cv.take<char>(cap * F * f4);
        t.da = cv.take<char>(cap * F * e);
        t.dc = cv.take<char>(cap * F * e);
        t.dxp = cv.take<char>(cap * H * e);
        t.dlog_lp = cv.take<char>(T * E * e);
    }
    return t;
}

// moe.rs:197-223 restructured: route, sort pairs by expert, three grouped
// GEMMs, weighted unpermute. Leaves every intermediate in t for the adjoint.
void moe_forward(Context* c, const void* x, const void* gate, const void* w1s, const void* w3s, const void* w2s, void* y,
                 i64 T, i64 H, i64 F, i64 E, i64 k, int dtype, MoeTemps& t) {
    gemm(c, false, false, T, E, H, x, H, gate, E, t.logits, E, dtype, CATNN_F32, nullptr, 0, false);
    router_topk(c, t.logits, T, E, k, t.idx, t.w);
    permute_map(c, t.idx, T, E, k, moe_align(dtype), t.rows_cap, t.counts, t.off, t.row_of, t.src_of);
    i64 rows = t.rows_cap;  // padded rows beyond off[E] are never touched by the grouped GEMMs
    permute_rows(c, x, t.src_of, rows, H, k, t.xp, dtype);
    grouped(c, dtype, false, rows, F, H, (int)E, t.off, t.xp, w1s, t.a, false, CATNN_F32);
    grouped(c, dtype, false, rows, F, H, (int)E, t.off, t.xp, w3s, t.cc, false, CATNN_F32);
    swiglu_act(c, t.a, t.cc, t.hh, rows, F, F, F, dtype, CATNN_F32);
    grouped(c, dtype, false, rows, H, F, (int)E, t.off, t.hh, w2s, t.yp, false, CATNN_F32);
    if (y) unpermute_rows(c, t.yp, t.row_of, t.w, T, k, H, y, dtype, false, CATNN_F32);
}

}  // namespace

extern "C" {

int catnn_router_topk(catnn_ctx* h, const float* logits, int64_t T, int64_t E, int64_t k, int32_t* idx, float* w) {
    ABI_BEGIN
    Context* c = unwrap(h);
    need(T == 0 || (logits && idx && w), "logits/idx/w");
    router_topk(c, logits, T, E, k, idx, w);
    ABI_END
}

int catnn_moe_permute_map(catnn_ctx* h, const int32_t* idx, int64_t T, int64_t E, int64_t k, int64_t align,
                          int32_t* counts, int32_t* offsets, int32_t* row_of, int32_t* src_of) {
    ABI_BEGIN
    Context* c = unwrap(h);
    need(counts && offsets && (T == 0 || (idx && row_of && src_of)), "permute_map arguments");
    shape(align >= 1 && align <= 1024, "permute_map: align in [1, 1024]");
    i64 cap = T * k + E * (align - 1);
    permute_map(c, idx, T, E, k, (int)align, cap, counts, offsets, row_of, src_of);
    int st = take_status(c, 8);
    if (st == 1) throw Error(CATNN_ERR_SHAPE, "permute_map: expert index out of range");
    if (st) throw Error(CATNN_ERR_SHAPE, "permute_map: padded rows exceed capacity");
    ABI_END
}

int catnn_moe_permute(catnn_ctx* h, const void* x, const int32_t* src_of, int64_t rows, int64_t hidden, int64_t k, void* xp,
                      int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(rows == 0 || (x && src_of && xp), "x/src_of/xp");
    permute_rows(c, x, src_of, rows, hidden, k, xp, dtype);
    ABI_END
}

int catnn_moe_unpermute(catnn_ctx* h, const void* yp, const int32_t* row_of, const float* w, int64_t T, int64_t k,
                        int64_t hidden, void* y, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(T == 0 || (yp && row_of && w && y), "yp/row_of/w/y");
    unpermute_rows(c, yp, row_of, w, T, k, hidden, y, dtype, false);
    ABI_END
}

int catnn_grouped_gemm(catnn_ctx* h, int trans_b, int64_t rows, int64_t N, int64_t K, int64_t groups,
                       const int32_t* offsets, const void* A, const void* B, void* C, int dtype, int c_dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    check_dtype(c_dtype);
    need(offsets && A && B && C, "grouped_gemm arguments");
    shape(rows >= 0 && N > 0 && K > 0 && groups >= 1 && groups <= 1024, "grouped_gemm: sizes");
    CATNN_CHECK(dtype == CATNN_BF16 || c_dtype == CATNN_F32, CATNN_ERR_DTYPE, "fp32 grouped gemm writes fp32");
    grouped(c, dtype, trans_b != 0, rows, N, K, (int)groups, offsets, A, B, C, false, c_dtype);
    ABI_END
}

int catnn_moe_expert_swiglu_fwd(catnn_ctx* h, const void* x, const void* w13, const int32_t* offsets, int64_t rows,
                                int64_t hidden, int64_t mid, int64_t groups, void* ac, void* hh) {
    ABI_BEGIN
    Context* c = unwrap(h);
    need(x && w13 && offsets && ac && hh, "expert swiglu arguments");
    shape(rows >= 0 && hidden >= 16 && mid > 0 && mid % 128 == 0 && groups >= 1 && groups <= 1024,
          "expert swiglu: sizes (mid a multiple of 128)");
    gemm_grouped_swiglu_fwd_tc(c, rows, mid, hidden, (int)groups, offsets, (const bf16*)x, hidden, (const bf16*)w13,
                               (bf16*)ac, (bf16*)hh);
    ABI_END
}

int catnn_moe_expert_swiglu_bwd(catnn_ctx* h, const void* dy, const void* w2, const void* ac, const int32_t* offsets,
                                int64_t rows, int64_t hidden, int64_t mid, int64_t groups, void* dac) {
    ABI_BEGIN
    Context* c = unwrap(h);
    need(dy && w2 && ac && offsets && dac, "expert swiglu backward arguments");
    shape(rows >= 0 && hidden >= 16 && mid > 0 && mid % 128 == 0 && groups >= 1 && groups <= 1024,
          "expert swiglu backward: sizes (mid a multiple of 128)");
    gemm_grouped_swiglu_bwd_tc(c, rows, mid, hidden, (int)groups, offsets, (const bf16*)dy, hidden, (const bf16*)w2,
                               (const bf16*)ac, (bf16*)dac);
    ABI_END
}

int catnn_swiglu_fwd(catnn_ctx* h, const void* x, const void* w1, const void* w3, const void* w2, void* y, int64_t T,
                     int64_t hidden, int64_t mid, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(x && w1 && w3 && w2 && y, "swiglu arguments");
    size_t e = dsize(dtype);
    Carver cv(c->work_for(Carver::need({T * mid * e, T * mid * e, T * mid * e})));
    void* a = cv.take<char>(T * mid * e);
    void* cc = cv.take<char>(T * mid * e);
    void* hh = cv.take<char>(T * mid * e);
    gemm(c, false, false, T, mid, hidden, x, hidden, w1, mid, a, mid, dtype, dtype, nullptr, 0, false);
    gemm(c, false, false, T, mid, hidden, x, hidden, w3, mid, cc, mid, dtype, dtype, nullptr, 0, false);
    swiglu_act(c, a, cc, hh, T, mid, mid, mid, dtype);
    gemm(c, false, false, T, hidden, mid, hh, mid, w2, hidden, y, hidden, dtype, dtype, nullptr, 0, false);
    ABI_END
}

int catnn_swiglu_bwd(catnn_ctx* h, const void* x, const void* w1, const void* w3, const void* w2, const void* dy, void* dx,
                     void* dw1, void* dw3, void* dw2, int64_t T, int64_t hidden, int64_t mid, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(x && w1 && w3 && w2 && dy && dx && dw1 && dw3 && dw2, "swiglu_bwd arguments");
    size_t e = dsize(dtype);
    size_t tm = T * mid * e;
    Carver cv(c->work_for(Carver::need({tm, tm, tm, tm, tm, tm})));
    void* a = cv.take<char>(tm);
    void* cc = cv.take<char>(tm);
    void* hh = cv.take<char>(tm);
    void* dh = cv.take<char>(tm);
    void* da = cv.take<char>(tm);
    void* dc = cv.take<char>(tm);
    gemm(c, false, false, T, mid, hidden, x, hidden, w1, mid, a, mid, dtype, dtype, nullptr, 0, false);
    gemm(c, false, false, T, mid, hidden, x, hidden, w3, mid, cc, mid, dtype, dtype, nullptr, 0, false);
    swiglu_act(c, a, cc, hh, T, mid, mid, mid, dtype);
    // adjoint.rs:236: (dh, dw2) from linear_backward(h, w2, dy)
    gemm(c, false, true, T, mid, hidden, dy, hidden, w2, hidden, dh, mid, dtype, dtype, nullptr, 0, false);
    gemm(c, true, false, mid, hidden, T, hh, mid, dy, hidden, dw2, hidden, dtype, dtype, nullptr, 0, false);
    swiglu_act_bwd(c, a, cc, dh, da, dc, T, mid, mid, mid, dtype);
    gemm(c, false, true, T, hidden, mid, da, mid, w1, mid, dx, hidden, dtype, dtype, nullptr, 0, false);
    gemm(c, false, true, T, hidden, mid, dc, mid, w3, mid, dx, hidden, dtype, dtype, nullptr, 0, true);
    gemm(c, true, false, hidden, mid, T, x, hidden, da, mid, dw1, mid, dtype, dtype, nullptr, 0, false);
    gemm(c, true, false, hidden, mid, T, x, hidden, dc, mid, dw3, mid, dtype, dtype, nullptr, 0, false);
    ABI_END
}

int catnn_moe_fwd(catnn_ctx* h, const void* x, const void* gate, const void* w1s, const void* w3s, const void* w2s, void* y,
                  int64_t T, int64_t hidden, int64_t mid, int64_t E, int64_t k, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(x && gate && w1s && w3s && w2s && y, "moe_fwd arguments");
    shape(E >= 1 && E <= 32 && k >= 1 && k <= E, "moe: need 1 <= k <= E <= 32");
    if (T == 0) return CATNN_OK;
    MoeTemps t = moe_temps(c, T, hidden, mid, E, k, dtype, false);
    moe_forward(c, x, gate, w1s, w3s, w2s, y, T, hidden, mid, E, k, dtype, t);
    ABI_END
}

// adjoint.rs:471-526 batched by expert: d_w from <y_e, dy>, the expert
// adjoints as grouped GEMMs over the same sorted rows, then the router STE
// (adjoint.rs:255-284) into dx and dgate.
int catnn_moe_bwd(catnn_ctx* h, const void* x, const void* gate, const void* w1s, const void* w3s, const void* w2s,
                  const void* dy, void* dx, void* dgate, void* dw1s, void* dw3s, void* dw2s, int64_t T, int64_t hidden,
                  int64_t mid, int64_t E, int64_t k, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(x && gate && w1s && w3s && w2s && dy && dx && dgate && dw1s && dw3s && dw2s, "moe_bwd arguments");
    shape(E >= 1 && E <= 32 && k >= 1 && k <= E, "moe: need 1 <= k <= E <= 32");
    if (T == 0) return CATNN_OK;
    MoeTemps t = moe_temps(c, T, hidden, mid, E, k, dtype, true);
    moe_forward(c, x, gate, w1s, w3s, w2s, nullptr, T, hidden, mid, E, k, dtype, t);
    i64 rows = t.rows_cap, H = hidden, F = mid;
    unpermute_bwd(c, t.yp, t.src_of, rows, t.w, dy, k, H, t.dwt, t.dyp, dtype, CATNN_F32);
    grouped(c, dtype, true, rows, F, H, (int)E, t.off, t.dyp, w2s, t.dh, false, CATNN_F32);  // dh = dyp · w2ᵀ
    grouped_wgrad(c, dtype, rows, H, F, (int)E, t.off, t.hh, t.dyp, dw2s);                   // dw2 = hᵀ · dyp
    swiglu_act_bwd(c, t.a, t.cc, t.dh, t.da, t.dc, rows, F, F, F, dtype, CATNN_F32);
    grouped(c, dtype, true, rows, H, F, (int)E, t.off, t.da, w1s, t.dxp, false);      // dxp = da · w1ᵀ
    grouped(c, dtype, true, rows, H, F, (int)E, t.off, t.dc, w3s, t.dxp, true);       //     + dc · w3ᵀ
    grouped_wgrad(c, dtype, rows, F, H, (int)E, t.off, t.xp, t.da, dw1s);             // dw1 = xpᵀ · da
    grouped_wgrad(c, dtype, rows, F, H, (int)E, t.off, t.xp, t.dc, dw3s);             // dw3 = xpᵀ · dc
    permute_bwd(c, t.dxp, t.row_of, T, k, H, dx, dtype, false);
    router_ste(c, t.idx, t.w, t.dwt, T, E, k, t.dlog);
    const void* dl = t.dlog;
    if (dtype == CATNN_BF16) {
        cast(c, t.dlog, CATNN_F32, t.dlog_lp, CATNN_BF16, T * E);
        dl = t.dlog_lp;
    }
    gemm(c, false, true, T, H, E, dl, E, gate, E, dx, H, dtype, dtype, nullptr, 0, true);       // dx += dlog · gateᵀ
    gemm(c, true, false, H, E, T, x, H, dl, E, dgate, E, dtype, dtype, nullptr, 0, false);      // dgate = xᵀ · dlog
    ABI_END
}

// ------------------------------------------------------------ optimizers
int catnn_sgd(catnn_ctx* h, float* p, const float* g, int64_t n, float lr, void* shadow_bf16) {
    ABI_BEGIN
    Context* c = unwrap(h);
    need(n == 0 || (p && g), "p/g");
    sgd(c, p, g, n, lr, (bf16*)shadow_bf16);
    ABI_END
}

int catnn_adam(catnn_ctx* h, float* p, const void* g, float* m, float* v, int64_t n, uint64_t t, float lr, float beta1,
               float beta2, float eps, int g_dtype, void* shadow_bf16) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(g_dtype);
    need(n == 0 || (p && g && m && v), "p/g/m/v");
    CATNN_CHECK(t >= 1, CATNN_ERR_INVALID, "adam: step count t starts at 1");
    adam(c, p, g, m, v, n, t, lr, beta1, beta2, eps, g_dtype, (bf16*)shadow_bf16);
    ABI_END
}

// ------------------------------------------------------------ MLP step
// train.rs:71-91 on the fp32 path; ce selects cross-entropy (labels) or
// MSE (y_mse). Gradients and the device loss scalar are written.
int catnn_mlp_step(catnn_ctx* h, const float* w1, const float* b1, const float* w2, const float* b2, const float* x,
                   const uint32_t* labels, const float* y_mse, int ce, int64_t batch, int64_t din, int64_t hid,
                   int64_t dout, float* loss, float* dw1, float* db1, float* dw2, float* db2) {
    ABI_BEGIN
    Context* c = unwrap(h);
    need(w1 && b1 && w2 && b2 && x && loss && dw1 && db1 && dw2 && db2, "mlp_step arguments");
    need(ce ? labels != nullptr : y_mse != nullptr, ce ? "labels" : "y_mse");
    shape(batch >= 1 && din >= 1 && hid >= 1 && dout >= 1, "mlp_step: empty shape");
    Carver cv(c->work_for(Carver::need({(size_t)batch * hid * 4 * 4, (size_t)batch * dout * 4 * 2})));
    float* z1 = cv.take<float>(batch * hid);
    float* h1 = cv.take<float>(batch * hid);
    float* dh1 = cv.take<float>(batch * hid);
    float* dz1 = cv.take<float>(batch * hid);
    float* pred = cv.take<float>(batch * dout);
    float* dpred = cv.take<float>(batch * dout);
    gemm(c, false, false, batch, hid, din, x, din, w1, hid, z1, hid, CATNN_F32, CATNN_F32, b1, 0, false);
    act_fwd(c, CATNN_ACT_RELU, z1, h1, batch * hid, CATNN_F32);
    gemm(c, false, false, batch, dout, hid, h1, hid, w2, dout, pred, dout, CATNN_F32, CATNN_F32, b2, 0, false);
    if (ce) xent_fwdbwd(c, pred, labels, batch, dout, loss, dpred, CATNN_F32, c->status + 9);
    else mse_fwdbwd(c, pred, y_mse, batch * dout, loss, dpred);
    gemm(c, false, true, batch, hid, dout, dpred, dout, w2, dout, dh1, hid, CATNN_F32, CATNN_F32, nullptr, 0, false);
    gemm(c, true, false, hid, dout, batch, h1, hid, dpred, dout, dw2, dout, CATNN_F32, CATNN_F32, nullptr, 0, false);
    col_sum(c, dpred, batch, dout, db2, CATNN_F32, false);
    act_bwd(c, CATNN_ACT_RELU, z1, dh1, dz1, batch * hid, CATNN_F32);
    gemm(c, true, false, din, hid, batch, x, din, dz1, hid, dw1, hid, CATNN_F32, CATNN_F32, nullptr, 0, false);
    col_sum(c, dz1, batch, hid, db1, CATNN_F32, false);
    ABI_END
}

}  // extern "C"
