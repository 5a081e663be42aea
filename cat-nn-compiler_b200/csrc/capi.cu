// extern "C" entry points of libcatnn_b200 (declared in include/catnn_b200.h):
// argument validation, then the launchers in ops.cuh. Composite ops (MHA,
// GQA, SwiGLU, MoE, the MLP step) sequence several launchers over
// temporaries carved from the context's work arena.
#include "ops.cuh"

using namespace catnn;

namespace {

void need(bool ok, const char* what) { CATNN_CHECK(ok, CATNN_ERR_INVALID, std::string("null argument: ") + what); }
void shape(bool ok, const std::string& what) { CATNN_CHECK(ok, CATNN_ERR_SHAPE, what); }


void linear_fwd_impl(Context* c, const void* x, const void* w, const float* b, void* y, i64 M, i64 K, i64 N, int act,
                     int dtype) {
    gemm(c, false, false, M, N, K, x, K, w, N, y, N, dtype, dtype, b, act, false);
}

void linear_bwd_impl(Context* c, const void* x, const void* w, const void* dy, void* dx, void* dw, float* db, i64 M,
                     i64 K, i64 N, int dtype, bool acc_dx = false) {
    if (dx) gemm(c, false, true, M, K, N, dy, N, w, N, dx, K, dtype, dtype, nullptr, CATNN_ACT_NONE, acc_dx);
    if (dw) gemm(c, true, false, K, N, M, x, K, dy, N, dw, N, dtype, dtype, nullptr, CATNN_ACT_NONE, false);
    if (db) col_sum(c, dy, M, N, db, dtype, false);
}

}  // namespace

extern "C" {

// ------------------------------------------------------------ dense
int catnn_gemm(catnn_ctx* h, int trans_a, int trans_b, int64_t M, int64_t N, int64_t K, const void* A, int64_t lda,
               const void* B, int64_t ldb, void* C, int64_t ldc, int dtype, int c_dtype, const float* bias, int act,
               int accumulate) {
    ABI_BEGIN
    Context* c = unwrap(h);
    shape(M >= 0 && N >= 0 && K >= 0, "gemm: negative size");
    if (M == 0 || N == 0) return CATNN_OK;
    need(C, "C");
    need(K == 0 || (A && B), "A/B");
    shape(lda >= (trans_a ? M : K) && ldb >= (trans_b ? K : N) && ldc >= N, "gemm: leading dimension too small");
    gemm(c, trans_a != 0, trans_b != 0, M, N, K, A, lda, B, ldb, C, ldc, dtype, c_dtype, bias, act, accumulate != 0);
    ABI_END
}

int catnn_linear_fwd(catnn_ctx* h, const void* x, const void* w, const float* b, void* y, int64_t M, int64_t K,
                     int64_t N, int act, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    shape(M >= 0 && K >= 0 && N >= 0, "linear: negative size");
    if (M == 0 || N == 0) return CATNN_OK;
    need(y && (K == 0 || (x && w)), "x/w/y");
    linear_fwd_impl(c, x, w, b, y, M, K, N, act, dtype);
    ABI_END
}

int catnn_linear_bwd(catnn_ctx* h, const void* x, const void* w, const void* dy, void* dx, void* dw, float* db,
                     int64_t M, int64_t K, int64_t N, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    shape(M >= 0 && K >= 0 && N >= 0, "linear_bwd: negative size");
    need(!dx || (dy && w), "dy/w");
    need(!dw || (dy && x), "dy/x");
    linear_bwd_impl(c, x, w, dy, dx, dw, db, M, K, N, dtype);
    ABI_END
}

int catnn_lm_head_fwd(catnn_ctx* h, const void* x, const void* w, void* y, int64_t rows, int64_t hidden, int64_t vocab,
                      int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(x && w && y, "x/w/y");
    gemm(c, false, true, rows, vocab, hidden, x, hidden, w, hidden, y, vocab, dtype, dtype, nullptr, 0, false);
    ABI_END
}

int catnn_lm_head_bwd(catnn_ctx* h, const void* x, const void* w, const void* dy, void* dx, void* dw, int64_t rows,
                      int64_t hidden, int64_t vocab, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(x && w && dy, "x/w/dy");
    if (dx) gemm(c, false, false, rows, hidden, vocab, dy, vocab, w, hidden, dx, hidden, dtype, dtype, nullptr, 0, false);
    if (dw) gemm(c, true, false, vocab, hidden, rows, dy, vocab, x, hidden, dw, hidden, dtype, dtype, nullptr, 0, false);
    ABI_END
}

// ------------------------------------------------------------ elementwise
int catnn_relu_fwd(catnn_ctx* h, const void* x, void* y, int64_t n, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(n == 0 || (x && y), "x/y");
    act_fwd(c, CATNN_ACT_RELU, x, y, n, dtype);
    ABI_END
}
int catnn_gelu_fwd(catnn_ctx* h, const void* x, void* y, int64_t n, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(n == 0 || (x && y), "x/y");
    act_fwd(c, CATNN_ACT_GELU, x, y, n, dtype);
    ABI_END
}
int catnn_relu_bwd(catnn_ctx* h, const void* x, const void* dy, void* dx, int64_t n, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(n == 0 || (x && dy && dx), "x/dy/dx");
    act_bwd(c, CATNN_ACT_RELU, x, dy, dx, n, dtype);
    ABI_END
}
int catnn_gelu_bwd(catnn_ctx* h, const void* x, const void* dy, void* dx, int64_t n, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(n == 0 || (x && dy && dx), "x/dy/dx");
    act_bwd(c, CATNN_ACT_GELU, x, dy, dx, n, dtype);
    ABI_END
}
int catnn_add(catnn_ctx* h, const void* a, const void* b, void* y, int64_t n, int64_t b_len, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    if (n == 0) return CATNN_OK;
    need(a && b && y, "a/b/y");
    // cpu.rs:80-98: same length, or b broadcast over the last dim.
    shape(b_len == n || (b_len > 0 && n % b_len == 0), "add: b is neither same-length nor a last-dim bias");
    add(c, a, b, y, n, b_len, dtype);
    ABI_END
}
int catnn_mul(catnn_ctx* h, const void* a, const void* b, void* y, int64_t n, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(n == 0 || (a && b && y), "a/b/y");
    mul(c, a, b, y, n, dtype);
    ABI_END
}

// ------------------------------------------------------------ softmax / losses
int catnn_softmax_fwd(catnn_ctx* h, const void* x, void* y, int64_t rows, int64_t last, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(rows * last == 0 || (x && y), "x/y");
    softmax_fwd(c, x, y, rows, last, dtype);
    ABI_END
}
int catnn_softmax_bwd(catnn_ctx* h, const void* y, const void* dy, void* dx, int64_t rows, int64_t last, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(rows * last == 0 || (y && dy && dx), "y/dy/dx");
    softmax_bwd(c, y, dy, dx, rows, last, dtype);
    ABI_END
}
int catnn_xent_fwdbwd(catnn_ctx* h, const void* logits, const uint32_t* targets, int64_t rows, int64_t vocab, float* loss,
                      void* dlogits, int dtype, int check) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    shape(rows >= 1 && vocab >= 1, "cross_entropy: empty logits");
    need(logits && targets && loss && dlogits, "logits/targets/loss/dlogits");
    xent_fwdbwd(c, logits, targets, rows, vocab, loss, dlogits, dtype, c->status + 9);
    if (check && take_status(c, 9)) throw Error(CATNN_ERR_SHAPE, "ce targets: a target is >= the number of classes");
    ABI_END
}
int catnn_mse_fwdbwd(catnn_ctx* h, const float* pred, const float* target, int64_t n, float* loss, float* d) {
    ABI_BEGIN
    Context* c = unwrap(h);
    shape(n >= 1, "mse: empty");
    need(pred && target && loss && d, "pred/target/loss/d");
    mse_fwdbwd(c, pred, target, n, loss, d);
    ABI_END
}

// ------------------------------------------------------------ norms
int catnn_layernorm_fwd(catnn_ctx* h, const void* x, const float* gamma, const float* beta, void* y, int64_t rows,
                        int64_t last, float eps, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(rows * last == 0 || (x && gamma && beta && y), "x/gamma/beta/y");
    layernorm_fwd(c, x, gamma, beta, y, rows, last, eps, dtype);
    ABI_END
}
int catnn_layernorm_bwd(catnn_ctx* h, const void* x, const float* gamma, const void* dy, void* dx, float* dgamma,
                        float* dbeta, int64_t rows, int64_t last, float eps, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(rows * last == 0 || (x && gamma && dy && dx), "x/gamma/dy/dx");
    layernorm_bwd(c, x, gamma, dy, dx, dgamma, dbeta, rows, last, eps, dtype);
    ABI_END
}
int catnn_rmsnorm_fwd(catnn_ctx* h, const void* x, const float* w, void* y, int64_t rows, int64_t last, float eps,
                      int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(rows * last == 0 || (x && w && y), "x/w/y");
    rmsnorm_fwd(c, x, w, y, rows, last, eps, dtype);
    ABI_END
}
int catnn_rmsnorm_bwd(catnn_ctx* h, const void* x, const float* w, const void* dy, void* dx, float* dw, int64_t rows,
                      int64_t last, float eps, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(rows * last == 0 || (x && w && dy && dx), "x/w/dy/dx");
    rmsnorm_bwd(c, x, w, dy, dx, dw, rows, last, eps, dtype, false);
    ABI_END
}

// ------------------------------------------------------------ embedding
int catnn_embedding_fwd(catnn_ctx* h, const uint32_t* ids, int64_t n, const void* table, int64_t vocab, int64_t hidden,
                        void* y, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    if (n == 0) return CATNN_OK;
    need(ids && table && y, "ids/table/y");
    embedding_fwd(c, ids, n, table, vocab, hidden, y, dtype, c->status + 10);
    if (take_status(c, 10)) throw Error(CATNN_ERR_SHAPE, "embedding: token id >= vocab");
    ABI_END
}
int catnn_embedding_bwd(catnn_ctx* h, const uint32_t* ids, int64_t n, const void* dy, float* dw, int64_t vocab,
                        int64_t hidden, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(dw && (n == 0 || (ids && dy)), "ids/dy/dw");
    embedding_bwd(c, ids, n, dy, dw, vocab, hidden, dtype);
    ABI_END
}

// ------------------------------------------------------------ attention
int catnn_rope(catnn_ctx* h, void* x, int64_t b, int64_t s, int64_t heads, int64_t hd, double theta, int inverse,
               int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(b * s * heads * hd == 0 || x, "x");
    shape(hd % 2 == 0, "rope: head_dim must be even");
    rope(c, x, b, s, heads, hd, theta, inverse != 0, dtype);
    ABI_END
}
int catnn_attention_fwd(catnn_ctx* h, const void* q, const void* k, const void* v, void* o, float* lse, int64_t b,
                        int64_t s, int64_t n_heads, int64_t n_kv, int64_t hd, int causal, int64_t window, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(q && k && v && o && lse, "q/k/v/o/lse");
    attention_fwd(c, q, k, v, o, lse, b, s, n_heads, n_kv, hd, causal != 0, window, dtype);
    ABI_END
}
int catnn_attention_bwd(catnn_ctx* h, const void* q, const void* k, const void* v, const void* o, const float* lse,
                        const void* dout, void* dq, void* dk, void* dv, int64_t b, int64_t s, int64_t n_heads,
                        int64_t n_kv, int64_t hd, int causal, int64_t window, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(q && k && v && o && lse && dout && dq && dk && dv, "attention_bwd arguments");
    attention_bwd(c, q, k, v, o, lse, dout, dq, dk, dv, b, s, n_heads, n_kv, hd, causal != 0, window, dtype);
    ABI_END
}

}  // extern "C"

// ---- composite attention ops: projections + core (+ RoPE for GQA)
namespace {

struct AttnTemps {
    void *q, *k, *v, *ctx, *dq, *dk, *dv, *dctx;
    float* lse;
};

AttnTemps attn_temps(Context* c, i64 bs, i64 qd, i64 kd, i64 bh_s, int dtype, bool bwd) {
    size_t e = dsize(dtype);
    size_t tot = Carver::need({bs * qd * e, bs * kd * e, bs * kd * e, bs * qd * e, (size_t)bh_s * 4, bs * qd * e,
                               bs * kd * e, bs * kd * e, bs * qd * e});
    Carver cv(c->work_for(tot));
    AttnTemps t{};
    t.q = cv.take<char>(bs * qd * e);
    t.k = cv.take<char>(bs * kd * e);
    t.v = cv.take<char>(bs * kd * e);
    t.ctx = cv.take<char>(bs * qd * e);
    t.lse = cv.take<float>(bh_s);
    if (bwd) {
        t.dq = cv.take<char>(bs * qd * e);
        t.dk = cv.take<char>(bs * kd * e);
        t.dv = cv.take<char>(bs * kd * e);
        t.dctx = cv.take<char>(bs * qd * e);
    }
    return t;
}

// q,k,v projections (+RoPE) and the attention core; leaves ctx, lse in t.
void attn_forward_core(Context* c, const void* x, const void* wq, const void* wk, const void* wv, AttnTemps& t, i64 b,
                       i64 s, i64 d, i64 H, i64 Hkv, i64 hd, bool causal, bool use_rope, double theta, i64 window,
                       int dtype) {
    i64 bs = b * s, qd = H * hd, kd = Hkv * hd;
    linear_fwd_impl(c, x, wq, nullptr, t.q, bs, d, qd, 0, dtype);
    linear_fwd_impl(c, x, wk, nullptr, t.k, bs, d, kd, 0, dtype);
    linear_fwd_impl(c, x, wv, nullptr, t.v, bs, d, kd, 0, dtype);
    if (use_rope) {
        rope(c, t.q, b, s, H, hd, theta, false, dtype);
        rope(c, t.k, b, s, Hkv, hd, theta, false, dtype);
    }
    attention_fwd(c, t.q, t.k, t.v, t.ctx, t.lse, b, s, H, Hkv, hd, causal, window, dtype);
}

void attn_op_fwd(Context* c, const void* x, const void* wq, const void* wk, const void* wv, const void* wo, void* y,
                 i64 b, i64 s, i64 d, i64 H, i64 Hkv, i64 hd, bool causal, bool use_rope, double theta, i64 window,
                 int dtype) {
    i64 bs = b * s;
    AttnTemps t = attn_temps(c, bs, H * hd, Hkv * hd, b * H * s, dtype, false);
    attn_forward_core(c, x, wq, wk, wv, t, b, s, d, H, Hkv, hd, causal, use_rope, theta, window, dtype);
    linear_fwd_impl(c, t.ctx, wo, nullptr, y, bs, H * hd, d, 0, dtype);
}

// adjoint.rs:287-439 (GQA) and :582-722 (MHA), recompute-then-adjoint.
void attn_op_bwd(Context* c, const void* x, const void* wq, const void* wk, const void* wv, const void* wo,
                 const void* dy, void* dx, void* dwq, void* dwk, void* dwv, void* dwo, i64 b, i64 s, i64 d, i64 H,
                 i64 Hkv, i64 hd, bool causal, bool use_rope, double theta, i64 window, int dtype) {
    i64 bs = b * s, qd = H * hd, kd = Hkv * hd;
    AttnTemps t = attn_temps(c, bs, qd, kd, b * H * s, dtype, true);
    attn_forward_core(c, x, wq, wk, wv, t, b, s, d, H, Hkv, hd, causal, use_rope, theta, window, dtype);
    linear_bwd_impl(c, t.ctx, wo, dy, t.dctx, dwo, nullptr, bs, qd, d, dtype);
    attention_bwd(c, t.q, t.k, t.v, t.ctx, t.lse, t.dctx, t.dq, t.dk, t.dv, b, s, H, Hkv, hd, causal, window, dtype);
    if (use_rope) {
        rope(c, t.dq, b, s, H, hd, theta, true, dtype);
        rope(c, t.dk, b, s, Hkv, hd, theta, true, dtype);
    }
    // dx = dq·wqᵀ + dk·wkᵀ + dv·wvᵀ (q first, as the reference sums).
    linear_bwd_impl(c, x, wq, t.dq, dx, dwq, nullptr, bs, d, qd, dtype, false);
    linear_bwd_impl(c, x, wk, t.dk, dx, dwk, nullptr, bs, d, kd, dtype, true);
    linear_bwd_impl(c, x, wv, t.dv, dx, dwv, nullptr, bs, d, kd, dtype, true);
}

}  // namespace

extern "C" {

int catnn_mha_fwd(catnn_ctx* h, const void* x, const void* wq, const void* wk, const void* wv, const void* wo, void* y,
                  int64_t b, int64_t s, int64_t d, int64_t n_heads, int causal, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(x && wq && wk && wv && wo && y, "mha_fwd arguments");
    shape(n_heads > 0 && d % n_heads == 0, "attention head split");
    attn_op_fwd(c, x, wq, wk, wv, wo, y, b, s, d, n_heads, n_heads, d / n_heads, causal != 0, false, 0.0, 0, dtype);
    ABI_END
}
int catnn_mha_bwd(catnn_ctx* h, const void* x, const void* wq, const void* wk, const void* wv, const void* wo,
                  const void* dy, void* dx, void* dwq, void* dwk, void* dwv, void* dwo, int64_t b, int64_t s, int64_t d,
                  int64_t n_heads, int causal, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(x && wq && wk && wv && wo && dy && dx, "mha_bwd arguments");
    shape(n_heads > 0 && d % n_heads == 0, "attention head split");
    attn_op_bwd(c, x, wq, wk, wv, wo, dy, dx, dwq, dwk, dwv, dwo, b, s, d, n_heads, n_heads, d / n_heads, causal != 0,
                false, 0.0, 0, dtype);
    ABI_END
}
int catnn_gqa_fwd(catnn_ctx* h, const void* x, const void* wq, const void* wk, const void* wv, const void* wo, void* y,
                  int64_t b, int64_t s, int64_t d, int64_t n_heads, int64_t n_kv, int64_t hd, double theta,
                  int64_t window, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(x && wq && wk && wv && wo && y, "gqa_fwd arguments");
    shape(n_kv > 0 && n_heads % n_kv == 0 && hd % 2 == 0, "gqa: heads / kv heads / head_dim");
    attn_op_fwd(c, x, wq, wk, wv, wo, y, b, s, d, n_heads, n_kv, hd, true, true, theta, window, dtype);
    ABI_END
}
int catnn_gqa_bwd(catnn_ctx* h, const void* x, const void* wq, const void* wk, const void* wv, const void* wo,
                  const void* dy, void* dx, void* dwq, void* dwk, void* dwv, void* dwo, int64_t b, int64_t s, int64_t d,
                  int64_t n_heads, int64_t n_kv, int64_t hd, double theta, int64_t window, int dtype) {
    ABI_BEGIN
    Context* c = unwrap(h);
    check_dtype(dtype);
    need(x && wq && wk && wv && wo && dy && dx, "gqa_bwd arguments");
    shape(n_kv > 0 && n_heads % n_kv == 0 && hd % 2 == 0, "gqa: heads / kv heads / head_dim");
    attn_op_bwd(c, x, wq, wk, wv, wo, dy, dx, dwq, dwk, dwv, dwo, b, s, d, n_heads, n_kv, hd, true, true, theta, window,
                dtype);
    ABI_END
}

}  // extern "C"
