// ORACLE — test infrastructure only (see cpu_kernels.hpp header).
//
// extern "C" surface of the oracle for ctypes. Every kernel is exported as
// orc_<name> (T = float, the oracle proper) and, where finite differences
// need it, orc64_<name> (T = double, the f64 shadow of kernel/fd64.rs).
#include "train_kernels.hpp"

using orc::i64;

#define ORC_BOTH(RET, NAME, PARAMS_F, PARAMS_D, ARGS)  \
    extern "C" RET orc_##NAME PARAMS_F { return orc::NAME<float> ARGS; } \
    extern "C" RET orc64_##NAME PARAMS_D { return orc::NAME<double> ARGS; }

extern "C" {

void orc_lcg(float* out, i64 n, uint64_t seed) { orc::lcg_fill(out, n, seed); }
uint64_t orc_checksum(const float* x, i64 n) { return orc::checksum(x, n); }

// ---- cpu.rs / reference.rs
void orc_matmul_seq(const float* a, const float* b, float* c, i64 m, i64 k, i64 n) { orc::matmul_seq(a, b, c, m, k, n); }
void orc_linear(const float* x, const float* w, const float* b, float* y, i64 m, i64 k, i64 n, int par) { orc::linear(x, w, b, y, m, k, n, par); }
void orc64_linear(const double* x, const double* w, const double* b, double* y, i64 m, i64 k, i64 n, int par) { orc::linear(x, w, b, y, m, k, n, par); }
void orc_ref_linear(const float* x, const float* w, const float* b, float* y, i64 m, i64 k, i64 n) { orc::ref_linear(x, w, b, y, m, k, n); }
void orc_relu(const float* x, float* y, i64 n) { orc::relu(x, y, n); }
void orc64_relu(const double* x, double* y, i64 n) { orc::relu(x, y, n); }
void orc_gelu(const float* x, float* y, i64 n) { orc::gelu(x, y, n); }
void orc64_gelu(const double* x, double* y, i64 n) { orc::gelu(x, y, n); }
void orc_softmax_last(const float* x, float* y, i64 rows, i64 last) { orc::softmax_last(x, y, rows, last); }
void orc64_softmax_last(const double* x, double* y, i64 rows, i64 last) { orc::softmax_last(x, y, rows, last); }
void orc_layer_norm(const float* x, const float* g, const float* b, float* y, i64 rows, i64 last, float eps) { orc::layer_norm(x, g, b, y, rows, last, eps); }
void orc64_layer_norm(const double* x, const double* g, const double* b, double* y, i64 rows, i64 last, double eps) { orc::layer_norm(x, g, b, y, rows, last, eps); }
void orc_add(const float* a, const float* b, float* y, i64 n) { orc::add(a, b, y, n); }
void orc_add_bias(const float* a, const float* b, float* y, i64 rows, i64 last) { orc::add_bias(a, b, y, rows, last); }
void orc_mul(const float* a, const float* b, float* y, i64 n) { orc::mul(a, b, y, n); }
void orc_attention(const float* x, const float* wq, const float* wk, const float* wv, const float* wo, float* y,
                   i64 b, i64 s, i64 d, i64 h, i64 dh, int causal) { orc::attention(x, wq, wk, wv, wo, y, b, s, d, h, dh, causal); }
void orc64_attention(const double* x, const double* wq, const double* wk, const double* wv, const double* wo, double* y,
                     i64 b, i64 s, i64 d, i64 h, i64 dh, int causal) { orc::attention(x, wq, wk, wv, wo, y, b, s, d, h, dh, causal); }

// ---- moe.rs / lens/moe.rs
void orc_rmsnorm(const float* x, const float* w, float* y, i64 rows, i64 last, float eps) { orc::rmsnorm(x, w, y, rows, last, eps); }
void orc64_rmsnorm(const double* x, const double* w, double* y, i64 rows, i64 last, double eps) { orc::rmsnorm(x, w, y, rows, last, eps); }
int orc_embedding(const uint32_t* ids, i64 n, const float* table, i64 vocab, i64 hidden, float* y) { return orc::embedding(ids, n, table, vocab, hidden, y); }
int orc64_embedding(const uint32_t* ids, i64 n, const double* table, i64 vocab, i64 hidden, double* y) { return orc::embedding(ids, n, table, vocab, hidden, y); }
void orc_rope(float* q, i64 b, i64 s, i64 heads, i64 hd, double theta) { orc::rope_all(q, b, s, heads, hd, theta); }
void orc_gqa(const float* x, const float* wq, const float* wk, const float* wv, const float* wo, float* y, i64 b, i64 s,
             i64 d, i64 h, i64 kv, i64 hd, double theta, i64 window) { orc::gqa(x, wq, wk, wv, wo, y, b, s, d, h, kv, hd, theta, window); }
void orc64_gqa(const double* x, const double* wq, const double* wk, const double* wv, const double* wo, double* y, i64 b, i64 s,
               i64 d, i64 h, i64 kv, i64 hd, double theta, i64 window) { orc::gqa(x, wq, wk, wv, wo, y, b, s, d, h, kv, hd, theta, window); }
void orc_gqa_core(const float* q, const float* k, const float* v, float* ctx, i64 b, i64 s, i64 h, i64 kv, i64 hd, i64 window) {
    orc::gqa_core(q, k, v, ctx, (float*)nullptr, b, s, h, kv, hd, window);
}
void orc_swiglu(const float* x, const float* w1, const float* w3, const float* w2, float* y, i64 t, i64 h, i64 m) { orc::swiglu(x, w1, w3, w2, y, t, h, m); }
void orc64_swiglu(const double* x, const double* w1, const double* w3, const double* w2, double* y, i64 t, i64 h, i64 m) { orc::swiglu(x, w1, w3, w2, y, t, h, m); }
void orc_topk_softmax(const float* logits, i64 n, i64 k, int64_t* idx, float* w) { orc::topk_softmax(logits, n, k, idx, w); }
void orc_route(const float* x, const float* gate, i64 t, i64 h, i64 e, i64 k, int64_t* idx, float* w, float* logits) { orc::route(x, gate, t, h, e, k, idx, w, logits); }
void orc_moe(const float* x, const float* gate, const float* w1s, const float* w3s, const float* w2s, float* y, i64 t, i64 h,
             i64 m, i64 e, i64 k) { orc::moe(x, gate, w1s, w3s, w2s, y, t, h, m, e, k); }
void orc64_moe(const double* x, const double* gate, const double* w1s, const double* w3s, const double* w2s, double* y, i64 t,
               i64 h, i64 m, i64 e, i64 k) { orc::moe(x, gate, w1s, w3s, w2s, y, t, h, m, e, k); }
void orc_lm_head(const float* x, const float* w, float* y, i64 rows, i64 h, i64 v) { orc::lm_head(x, w, y, rows, h, v); }

// ---- adjoint.rs
void orc_linear_backward(const float* x, const float* w, const float* dy, float* dx, float* dw, float* db, i64 m, i64 k, i64 n) { orc::linear_backward(x, w, dy, dx, dw, db, m, k, n); }
void orc64_linear_backward(const double* x, const double* w, const double* dy, double* dx, double* dw, double* db, i64 m, i64 k, i64 n) { orc::linear_backward(x, w, dy, dx, dw, db, m, k, n); }
void orc_relu_backward(const float* x, const float* dy, float* dx, i64 n) { orc::relu_backward(x, dy, dx, n); }
void orc64_relu_backward(const double* x, const double* dy, double* dx, i64 n) { orc::relu_backward(x, dy, dx, n); }
void orc_gelu_backward(const float* x, const float* dy, float* dx, i64 n) { orc::gelu_backward(x, dy, dx, n); }
void orc64_gelu_backward(const double* x, const double* dy, double* dx, i64 n) { orc::gelu_backward(x, dy, dx, n); }
void orc_softmax_backward(const float* y, const float* dy, float* dx, i64 rows, i64 last) { orc::softmax_backward(y, dy, dx, rows, last); }
void orc64_softmax_backward(const double* y, const double* dy, double* dx, i64 rows, i64 last) { orc::softmax_backward(y, dy, dx, rows, last); }
float orc_mse_loss(const float* p, const float* t, float* d, i64 n) { return orc::mse_loss(p, t, d, n); }
double orc64_mse_loss(const double* p, const double* t, double* d, i64 n) { return orc::mse_loss(p, t, d, n); }
int orc_cross_entropy(const float* logits, const uint32_t* tg, float* d, i64 rows, i64 last, float* loss) { return orc::cross_entropy(logits, tg, d, rows, last, loss); }
int orc64_cross_entropy(const double* logits, const uint32_t* tg, double* d, i64 rows, i64 last, double* loss) { return orc::cross_entropy(logits, tg, d, rows, last, loss); }
void orc_rmsnorm_backward(const float* x, const float* w, const float* dy, float* dx, float* dw, i64 rows, i64 last, float eps) { orc::rmsnorm_backward(x, w, dy, dx, dw, rows, last, eps); }
void orc64_rmsnorm_backward(const double* x, const double* w, const double* dy, double* dx, double* dw, i64 rows, i64 last, double eps) { orc::rmsnorm_backward(x, w, dy, dx, dw, rows, last, eps); }
void orc_embedding_backward(const uint32_t* ids, i64 n, const float* dy, float* dw, i64 vocab, i64 hidden) { orc::embedding_backward(ids, n, dy, dw, vocab, hidden); }
void orc64_embedding_backward(const uint32_t* ids, i64 n, const double* dy, double* dw, i64 vocab, i64 hidden) { orc::embedding_backward(ids, n, dy, dw, vocab, hidden); }
void orc_swiglu_backward(const float* x, const float* w1, const float* w3, const float* w2, const float* dy, float* dx, float* dw1,
                         float* dw3, float* dw2, i64 t, i64 h, i64 m) { orc::swiglu_backward(x, w1, w3, w2, dy, dx, dw1, dw3, dw2, t, h, m); }
void orc64_swiglu_backward(const double* x, const double* w1, const double* w3, const double* w2, const double* dy, double* dx,
                           double* dw1, double* dw3, double* dw2, i64 t, i64 h, i64 m) { orc::swiglu_backward(x, w1, w3, w2, dy, dx, dw1, dw3, dw2, t, h, m); }
void orc_router_backward_ste(const float* x, const float* gate, const float* dwts, float* dx, float* dgate, i64 t, i64 h, i64 e, i64 k) {
    orc::router_backward_ste(x, gate, dwts, dx, dgate, t, h, e, k);
}
void orc_moe_backward(const float* x, const float* gate, const float* w1s, const float* w3s, const float* w2s, const float* dy,
                      float* dx, float* dgate, float* dw1s, float* dw3s, float* dw2s, i64 t, i64 h, i64 m, i64 e, i64 k) {
    orc::moe_backward(x, gate, w1s, w3s, w2s, dy, dx, dgate, dw1s, dw3s, dw2s, t, h, m, e, k);
}
void orc64_moe_backward(const double* x, const double* gate, const double* w1s, const double* w3s, const double* w2s, const double* dy,
                        double* dx, double* dgate, double* dw1s, double* dw3s, double* dw2s, i64 t, i64 h, i64 m, i64 e, i64 k) {
    orc::moe_backward(x, gate, w1s, w3s, w2s, dy, dx, dgate, dw1s, dw3s, dw2s, t, h, m, e, k);
}
void orc_layer_norm_backward(const float* x, const float* g, const float* dy, float* dx, float* dg, float* db, i64 rows, i64 last, float eps) {
    orc::layer_norm_backward(x, g, dy, dx, dg, db, rows, last, eps);
}
void orc64_layer_norm_backward(const double* x, const double* g, const double* dy, double* dx, double* dg, double* db, i64 rows, i64 last, double eps) {
    orc::layer_norm_backward(x, g, dy, dx, dg, db, rows, last, eps);
}
void orc_gqa_backward(const float* x, const float* wq, const float* wk, const float* wv, const float* wo, const float* dy, float* dx,
                      float* dwq, float* dwk, float* dwv, float* dwo, i64 b, i64 s, i64 d, i64 h, i64 kv, i64 hd, double theta, i64 window) {
    orc::gqa_backward(x, wq, wk, wv, wo, dy, dx, dwq, dwk, dwv, dwo, b, s, d, h, kv, hd, theta, window);
}
void orc64_gqa_backward(const double* x, const double* wq, const double* wk, const double* wv, const double* wo, const double* dy, double* dx,
                        double* dwq, double* dwk, double* dwv, double* dwo, i64 b, i64 s, i64 d, i64 h, i64 kv, i64 hd, double theta, i64 window) {
    orc::gqa_backward(x, wq, wk, wv, wo, dy, dx, dwq, dwk, dwv, dwo, b, s, d, h, kv, hd, theta, window);
}
void orc_attention_backward(const float* x, const float* wq, const float* wk, const float* wv, const float* wo, const float* dy,
                            float* dx, float* dwq, float* dwk, float* dwv, float* dwo, i64 b, i64 s, i64 d, i64 h, i64 dh, int causal) {
    orc::attention_backward(x, wq, wk, wv, wo, dy, dx, dwq, dwk, dwv, dwo, b, s, d, h, dh, causal);
}
void orc64_attention_backward(const double* x, const double* wq, const double* wk, const double* wv, const double* wo, const double* dy,
                              double* dx, double* dwq, double* dwk, double* dwv, double* dwo, i64 b, i64 s, i64 d, i64 h, i64 dh, int causal) {
    orc::attention_backward(x, wq, wk, wv, wo, dy, dx, dwq, dwk, dwv, dwo, b, s, d, h, dh, causal);
}
void orc_lm_head_backward(const float* x, const float* w, const float* dy, float* dx, float* dw, i64 rows, i64 h, i64 v) {
    orc::lm_head_backward(x, w, dy, dx, dw, rows, h, v);
}

// ---- optim.rs
void orc_sgd_put(const float* p, const float* g, float* out, i64 n, float lr) { orc::sgd_put(p, g, out, n, lr); }
uint64_t orc_adam_put(float* p, const float* g, float* m, float* v, i64 n, uint64_t t_prev, float lr, float b1, float b2, float eps) {
    return orc::adam_put(p, g, m, v, n, t_prev, lr, b1, b2, eps);
}
float orc_powi(float a, int b) { return orc::powi(a, b); }

// ---- train.rs
// cfg array: vocab, hidden, mid, layers, heads, kv_heads, experts, top_k, window
static orc::MixCfg mkcfg(const i64* c, float eps, double theta) {
    orc::MixCfg m;
    m.vocab = c[0]; m.hidden = c[1]; m.mid = c[2]; m.layers = c[3]; m.heads = c[4];
    m.kv_heads = c[5]; m.experts = c[6]; m.top_k = c[7]; m.window = c[8];
    m.eps = eps; m.theta = theta;
    return m;
}
i64 orc_mixtral_param_count(const i64* c) { return orc::MixLayout(mkcfg(c, 1e-5f, 1e4)).total; }
void orc_mixtral_layout(const i64* c, i64* out) {
    orc::MixLayout L(mkcfg(c, 1e-5f, 1e4));
    i64 v[] = {L.embed, L.final_norm, L.lm_head, L.total, L.layer0, L.layer_stride, L.rms_attn, L.wq,
               L.wk, L.wv, L.wo, L.rms_moe, L.gate, L.w1, L.w3, L.w2};
    for (int i = 0; i < 16; ++i) out[i] = v[i];
}
void orc_mixtral_seeded(const i64* c, uint64_t seed, float* P) { orc::mixtral_seeded(mkcfg(c, 1e-5f, 1e4), seed, P); }
int orc_mixtral_forward(const i64* c, float eps, double theta, const float* P, const uint32_t* tok, i64 b, i64 s, float* logits) {
    return orc::mixtral_forward(mkcfg(c, eps, theta), P, tok, b, s, logits);
}
int orc_mixtral_step(const i64* c, float eps, double theta, const float* P, const uint32_t* tok, i64 b, i64 s, float* loss, float* G) {
    return orc::mixtral_step(mkcfg(c, eps, theta), P, tok, b, s, loss, G);
}
int orc64_mixtral_step(const i64* c, float eps, double theta, const double* P, const uint32_t* tok, i64 b, i64 s, double* loss, double* G) {
    return orc::mixtral_step(mkcfg(c, eps, theta), P, tok, b, s, loss, G);
}
// forced: [layers][b*s][top_k] routing indices held fixed
int orc_mixtral_step_frozen(const i64* c, float eps, double theta, const float* P, const uint32_t* tok, i64 b, i64 s,
                            const int64_t* forced, float* loss, float* G) {
    return orc::mixtral_step(mkcfg(c, eps, theta), P, tok, b, s, loss, G, forced);
}
int orc_mlp_step(const float* w1, const float* b1, const float* w2, const float* b2, const float* x, const float* y_mse,
                 const uint32_t* labels, int ce, i64 batch, i64 din, i64 hid, i64 dout, float* loss, float* dw1, float* db1,
                 float* dw2, float* db2) {
    return orc::mlp_step(w1, b1, w2, b2, x, y_mse, labels, ce, batch, din, hid, dout, loss, dw1, db1, dw2, db2);
}
// W and G: 12 pointers each in the order g1, be1, wq, wk, wv, wo, g2, be2, f1, c1, f2, c2.
void orc_block_fwd_bwd(const float* const* W, float* const* G, const float* x, const float* dy, float* y, float* dx,
                       i64 b, i64 s, i64 d, i64 heads, i64 ff, float eps) {
    orc::BlockW<float> w{W[0], W[1], W[2], W[3], W[4], W[5], W[6], W[7], W[8], W[9], W[10], W[11]};
    orc::BlockG<float> g{G[0], G[1], G[2], G[3], G[4], G[5], G[6], G[7], G[8], G[9], G[10], G[11]};
    orc::block_fwd_bwd(w, x, dy, y, dx, g, b, s, d, heads, ff, eps);
}
void orc64_block_fwd_bwd(const double* const* W, double* const* G, const double* x, const double* dy, double* y,
                         double* dx, i64 b, i64 s, i64 d, i64 heads, i64 ff, double eps) {
    orc::BlockW<double> w{W[0], W[1], W[2], W[3], W[4], W[5], W[6], W[7], W[8], W[9], W[10], W[11]};
    orc::BlockG<double> g{G[0], G[1], G[2], G[3], G[4], G[5], G[6], G[7], G[8], G[9], G[10], G[11]};
    orc::block_fwd_bwd(w, x, dy, y, dx, g, b, s, d, heads, ff, eps);
}

}  // extern "C"
