/*
 * catnn_b200.h — C ABI of libcatnn_b200, the B200 (sm_100a) execution backend
 * for catnn's data-parallel hot path.
 *
 * Conventions
 * - Every entry point returns int status (CATNN_OK = 0). On failure the
 *   text is available from catnn_last_error() (thread-local). No C++
 *   exception crosses this boundary.
 * - Tensors are device pointers, row-major, dense, with explicit sizes.
 *   Shapes follow the reference's layouts: linear weights are [in, out]
 *   (crates/catnn-core/src/category/morphism.rs:249-252), embedding and
 *   LM-head tables are [vocab, hidden], expert weights w1/w3 [hidden, mid],
 *   w2 [mid, hidden], Q [B,S,H,hd], K/V [B,S,Hkv,hd].
 * - `dtype` selects the storage type of the activations/weights of a call:
 *   CATNN_F32 runs the fp32 parity path (FFMA, rtol 1e-5 vs the reference);
 *   CATNN_BF16 runs the tensor-core path (bf16 operands, fp32 accumulation,
 *   rtol 2e-2 / atol 1e-3). Scalars, losses, router weights, norms' weight
 *   vectors and optimizer state are always fp32.
 * - All work is enqueued on the context's stream (catnn_ctx_set_stream);
 *   calls return before the GPU finishes unless documented otherwise.
 * - Every call first makes the context's device current: a context may be
 *   driven from different host threads, one at a time.
 *
 * Each declaration names the reference interface (file:line in
 * dkarapetyan-afk/cat-nn-compiler) whose behaviour it reproduces.
 */
#ifndef CATNN_B200_H
#define CATNN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. The first five mirror CatError variants
 * (crates/catnn-core/src/error.rs:9-54). */
#define CATNN_OK 0
#define CATNN_ERR_SHAPE 1        /* CatError::ShapeMismatch */
#define CATNN_ERR_DTYPE 2        /* CatError::DTypeMismatch */
#define CATNN_ERR_UNKNOWN_PORT 3 /* CatError::UnknownPort */
#define CATNN_ERR_WIRING 4       /* CatError::Wiring */
#define CATNN_ERR_UNLAWFUL 5     /* CatError::Unlawful */
#define CATNN_ERR_CUDA 6         /* a CUDA runtime call failed */
#define CATNN_ERR_INVALID 7      /* null handle / bad argument */
#define CATNN_ERR_TIMEOUT 8      /* a bounded device wait ran out */
#define CATNN_ERR_UNSUPPORTED 9  /* combination not built (e.g. dtype) */
#define CATNN_ERR_COMM 10        /* collective backend failure */

#define CATNN_F32 0
#define CATNN_BF16 1
/* catnn_gemm's `dtype` only: fp32 A/B multiplied on the tensor cores as TF32
 * (10-bit mantissas, fp32 accumulation), for callers that keep fp32
 * storage and accept the bf16 tolerance band. */
#define CATNN_TF32 2

#define CATNN_ACT_NONE 0
#define CATNN_ACT_RELU 1 /* cpu.rs:14 */
#define CATNN_ACT_GELU 2 /* cpu.rs:20, tanh approximation */

typedef struct catnn_ctx catnn_ctx;

/* ------------------------------------------------------------ context */
int catnn_version(void);
/* Text of the last failure on this host thread ("" if none). */
const char* catnn_last_error(void);
/* Per-device context; replaces the CPU DeviceHandler state
 * (crates/catnn-rt/src/handler.rs:14-28). */
int catnn_ctx_create(int device, catnn_ctx** out);
int catnn_ctx_destroy(catnn_ctx* ctx);
/* stream: a cudaStream_t (NULL = legacy default stream). */
int catnn_ctx_set_stream(catnn_ctx* ctx, void* stream);
int catnn_ctx_synchronize(catnn_ctx* ctx);
/* Number of kernels this context has launched (for launch accounting). */
int catnn_ctx_launch_count(catnn_ctx* ctx, uint64_t* out);
/* Device memory owned by the caller, and host<->device copies (synchronous
 * w.r.t. the context stream on return). */
int catnn_malloc(catnn_ctx* ctx, size_t bytes, void** out);
int catnn_free(catnn_ctx* ctx, void* ptr);
int catnn_upload(catnn_ctx* ctx, void* dst_dev, const void* src_host, size_t bytes);
int catnn_download(catnn_ctx* ctx, void* dst_host, const void* src_dev, size_t bytes);
/* FNV-1a checksum over the f32 bit patterns of a device tensor, the value
 * DeviceHandler::run_kernel records per kernel (handler.rs:46-53,
 * tensor.rs:279-288). Synchronous. */
int catnn_checksum_f32(catnn_ctx* ctx, const float* x, int64_t n, uint64_t* out);

/* ------------------------------------------------------------ dense */
/* C[M,N] = act(op(A)·op(B) + bias) (+ C if accumulate).
 * op(A) is [M,K]: trans_a=0 reads A as [M,K] (lda >= K), trans_a=1 as [K,M].
 * op(B) is [K,N]: trans_b=0 reads B as [K,N] (ldb >= N), trans_b=1 as [N,K].
 * A/B in `dtype` (CATNN_TF32: fp32 A/B multiplied as TF32 on the tensor
 * cores); C in c_dtype; bias fp32 [N] or NULL.
 * The contraction behind cpu::matmul_mk_kn (crates/catnn-compile/src/kernel/cpu.rs:186). */
int catnn_gemm(catnn_ctx* ctx, int trans_a, int trans_b, int64_t M, int64_t N, int64_t K,
               const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
               int dtype, int c_dtype, const float* bias, int act, int accumulate);
/* y[M,N] = act(x[M,K]·w[K,N] + b). cpu::linear (cpu.rs:135) and
 * apply_fused_linear_relu (cpu.rs:306). b may be NULL. */
int catnn_linear_fwd(catnn_ctx* ctx, const void* x, const void* w, const float* b, void* y,
                     int64_t M, int64_t K, int64_t N, int act, int dtype);
/* dx = dy·wᵀ, dw = xᵀ·dy, db = Σ_rows dy. adjoint::linear_backward
 * (crates/catnn-compile/src/kernel/adjoint.rs:35). dx/dw/db may each be NULL. */
int catnn_linear_bwd(catnn_ctx* ctx, const void* x, const void* w, const void* dy, void* dx,
                     void* dw, float* db, int64_t M, int64_t K, int64_t N, int dtype);
/* logits = x·wᵀ, w [vocab, hidden]. moe::lm_head (moe.rs:325). */
int catnn_lm_head_fwd(catnn_ctx* ctx, const void* x, const void* w, void* y, int64_t rows,
                      int64_t hidden, int64_t vocab, int dtype);
/* LmHead adjoint (adjoint.rs:903-913). */
int catnn_lm_head_bwd(catnn_ctx* ctx, const void* x, const void* w, const void* dy, void* dx,
                      void* dw, int64_t rows, int64_t hidden, int64_t vocab, int dtype);

/* ------------------------------------------------------------ elementwise */
int catnn_relu_fwd(catnn_ctx* ctx, const void* x, void* y, int64_t n, int dtype);      /* cpu.rs:14 */
int catnn_gelu_fwd(catnn_ctx* ctx, const void* x, void* y, int64_t n, int dtype);      /* cpu.rs:20 */
int catnn_relu_bwd(catnn_ctx* ctx, const void* x, const void* dy, void* dx, int64_t n, int dtype); /* adjoint.rs:63 */
int catnn_gelu_bwd(catnn_ctx* ctx, const void* x, const void* dy, void* dx, int64_t n, int dtype); /* adjoint.rs:76 */
/* y = a + b; b has n elements, or b_len = last-dim elements broadcast
 * over rows (cpu.rs:80-98). */
int catnn_add(catnn_ctx* ctx, const void* a, const void* b, void* y, int64_t n, int64_t b_len, int dtype);
int catnn_mul(catnn_ctx* ctx, const void* a, const void* b, void* y, int64_t n, int dtype); /* cpu.rs:100 */

/* ------------------------------------------------------------ softmax / losses */
int catnn_softmax_fwd(catnn_ctx* ctx, const void* x, void* y, int64_t rows, int64_t last, int dtype); /* cpu.rs:31 */
int catnn_softmax_bwd(catnn_ctx* ctx, const void* y, const void* dy, void* dx, int64_t rows,
                      int64_t last, int dtype); /* adjoint.rs:92 */
/* Mean softmax cross-entropy, fused forward + backward. loss: device fp32
 * scalar; dlogits may alias logits. Targets >= vocab are a ShapeMismatch
 * (detected on device, reported by the call, which synchronizes only when
 * check != 0). adjoint::cross_entropy (adjoint.rs:123). */
int catnn_xent_fwdbwd(catnn_ctx* ctx, const void* logits, const uint32_t* targets, int64_t rows,
                      int64_t vocab, float* loss, void* dlogits, int dtype, int check);
/* catnn_xent_fwdbwd for callers that cannot allocate device memory during
 * a step (a runtime with a fixed memory plan, or a thread that must not
 * block on the allocator). Same arguments, same results; its per-row scratch
 * is a fixed array inside the library (CATNN_XENT_NOALLOC_MAX_ROWS floats per
 * device, held until exit), so rows above that limit are rejected with
 * CATNN_ERR_SHAPE. It calls no allocator: catnn_ctx_create already looked up
 * the array's device address on that device (the lookup can load the
 * library's device code, which allocates), and the address is dropped when
 * the device's last context is destroyed. Calls share the array: two calls
 * whose kernels overlap on the GPU (other streams, other contexts of the
 * device) race. No counterpart in the reference: its CPU kernels allocate on
 * the host per call. */
#define CATNN_XENT_NOALLOC_MAX_ROWS 65536
int catnn_xent_fwdbwd_noalloc(catnn_ctx* ctx, const void* logits, const uint32_t* targets, int64_t rows,
                              int64_t vocab, float* loss, void* dlogits, int dtype, int check);
/* Mean squared error, d = 2(p - t)/n. adjoint::mse_loss (adjoint.rs:106). fp32. */
int catnn_mse_fwdbwd(catnn_ctx* ctx, const float* pred, const float* target, int64_t n, float* loss, float* d);

/* ------------------------------------------------------------ norms */
int catnn_layernorm_fwd(catnn_ctx* ctx, const void* x, const float* gamma, const float* beta, void* y,
                        int64_t rows, int64_t last, float eps, int dtype); /* cpu.rs:54 */
int catnn_layernorm_bwd(catnn_ctx* ctx, const void* x, const float* gamma, const void* dy, void* dx,
                        float* dgamma, float* dbeta, int64_t rows, int64_t last, float eps,
                        int dtype); /* adjoint.rs:530 */
int catnn_rmsnorm_fwd(catnn_ctx* ctx, const void* x, const float* w, void* y, int64_t rows,
                      int64_t last, float eps, int dtype); /* moe.rs:17 */
int catnn_rmsnorm_bwd(catnn_ctx* ctx, const void* x, const float* w, const void* dy, void* dx,
                      float* dw, int64_t rows, int64_t last, float eps, int dtype); /* adjoint.rs:148 */

/* ------------------------------------------------------------ embedding */
/* y[t] = table[ids[t]]. Synchronizes to report an id >= vocab as a
 * ShapeMismatch, as moe::embedding does (moe.rs:34-45). */
int catnn_embedding_fwd(catnn_ctx* ctx, const uint32_t* ids, int64_t n, const void* table,
                        int64_t vocab, int64_t hidden, void* y, int dtype);
/* dw[v] = Σ_{t: ids[t]=v} dy[t], summed in t order (deterministic, no
 * atomics); dw is fp32 [vocab, hidden]. adjoint::embedding_backward
 * (adjoint.rs:195). Uses context scratch. */
int catnn_embedding_bwd(catnn_ctx* ctx, const uint32_t* ids, int64_t n, const void* dy, float* dw,
                        int64_t vocab, int64_t hidden, int dtype);

/* ------------------------------------------------------------ attention */
/* Rotate interleaved pairs of x [B,S,heads,hd] in place by pos·θ^(-2i/hd);
 * inverse=1 applies the adjoint rotation. moe.rs:47 / adjoint.rs:454. */
int catnn_rope(catnn_ctx* ctx, void* x, int64_t b, int64_t s, int64_t heads, int64_t hd,
               double theta, int inverse, int dtype);
/* Attention core on projected (and rotated) q [B,S,H,hd], k/v [B,S,Hkv,hd]:
 * o [B,S,H*hd], lse fp32 [B,H,S] (log-sum-exp of the scaled scores, kept
 * for the backward). causal: j <= i; window > 0 further limits to
 * j > i - window (moe.rs:105). Scale 1/sqrt(hd). Head h reads kv head
 * h / (H/Hkv). The inner loops of moe::gqa (moe.rs:100-133) and
 * cpu::attention (cpu.rs:254-295). */
int catnn_attention_fwd(catnn_ctx* ctx, const void* q, const void* k, const void* v, void* o,
                        float* lse, int64_t b, int64_t s, int64_t n_heads, int64_t n_kv,
                        int64_t hd, int causal, int64_t window, int dtype);
/* Adjoint of catnn_attention_fwd given o, lse and dout. The inner loops of
 * gqa_backward (adjoint.rs:366-407) and attention_backward (adjoint.rs:652-703). */
int catnn_attention_bwd(catnn_ctx* ctx, const void* q, const void* k, const void* v, const void* o,
                        const float* lse, const void* dout, void* dq, void* dk, void* dv,
                        int64_t b, int64_t s, int64_t n_heads, int64_t n_kv, int64_t hd, int causal,
                        int64_t window, int dtype);
/* Full MHA op x [B,S,d] -> y (cpu::attention, cpu.rs:235; causal=0 is the
 * reference as-is). Weights [d,d]. Uses context scratch. */
int catnn_mha_fwd(catnn_ctx* ctx, const void* x, const void* wq, const void* wk, const void* wv,
                  const void* wo, void* y, int64_t b, int64_t s, int64_t d, int64_t n_heads,
                  int causal, int dtype);
/* attention_backward (adjoint.rs:582). */
int catnn_mha_bwd(catnn_ctx* ctx, const void* x, const void* wq, const void* wk, const void* wv,
                  const void* wo, const void* dy, void* dx, void* dwq, void* dwk, void* dwv,
                  void* dwo, int64_t b, int64_t s, int64_t d, int64_t n_heads, int causal, int dtype);
/* GQA + RoPE + optional window (moe::gqa, moe.rs:64). window <= 0: none. */
int catnn_gqa_fwd(catnn_ctx* ctx, const void* x, const void* wq, const void* wk, const void* wv,
                  const void* wo, void* y, int64_t b, int64_t s, int64_t d, int64_t n_heads,
                  int64_t n_kv, int64_t hd, double theta, int64_t window, int dtype);
/* gqa_backward (adjoint.rs:287). */
int catnn_gqa_bwd(catnn_ctx* ctx, const void* x, const void* wq, const void* wk, const void* wv,
                  const void* wo, const void* dy, void* dx, void* dwq, void* dwk, void* dwv,
                  void* dwo, int64_t b, int64_t s, int64_t d, int64_t n_heads, int64_t n_kv,
                  int64_t hd, double theta, int64_t window, int dtype);

/* ------------------------------------------------------------ MoE */
/* Per row of logits [T,E]: the k largest, ties to the lower index, then a
 * softmax over those k. idx int32 [T,k], w fp32 [T,k]. Bit-exact indices.
 * lens::moe::topk_softmax (crates/catnn-core/src/lens/moe.rs:175). */
int catnn_router_topk(catnn_ctx* ctx, const float* logits, int64_t T, int64_t E, int64_t k,
                      int32_t* idx, float* w);
/* Stable counting sort of the T·k (token, slot) pairs by expert (E <= 32).
 * counts int32 [E]; offsets int32 [E+1], each expert's block padded to a
 * multiple of `align` rows; row_of int32 [T·k]: sorted row of pair t·k+j;
 * src_of int32 [T·k + E·(align-1)]: pair index of each sorted row, -1 on
 * padding. Rows of one expert are in token order. Synchronizes to report an
 * out-of-range expert index. The permutation moe::moe performs implicitly
 * (moe.rs:207-221). */
int catnn_moe_permute_map(catnn_ctx* ctx, const int32_t* idx, int64_t T, int64_t E, int64_t k,
                          int64_t align, int32_t* counts, int32_t* offsets, int32_t* row_of,
                          int32_t* src_of);
/* xp[r] = x[src_of[r] / k] for r < rows (zero rows where src_of[r] < 0). */
int catnn_moe_permute(catnn_ctx* ctx, const void* x, const int32_t* src_of, int64_t rows,
                      int64_t hidden, int64_t k, void* xp, int dtype);
/* y[t] = Σ_j w[t,j] · yp[row_of[t·k+j]] in j order (moe.rs:217-219). */
int catnn_moe_unpermute(catnn_ctx* ctx, const void* yp, const int32_t* row_of, const float* w,
                        int64_t T, int64_t k, int64_t hidden, void* y, int dtype);
/* Expert GEMM over expert-sorted rows: for each group g, rows
 * [offsets[g], offsets[g+1]) of A [rows, K] times op(B_g), B_g = B + g·K·N
 * stored [K,N] (trans_b=0) or [N,K] (trans_b=1), into the same rows of
 * C [rows, N]. offsets: device int32 [groups+1]; on the bf16 path each
 * group's row count is a multiple of 128 (catnn_moe_permute_map, align 128).
 * The per-expert products moe::moe computes token by token (moe.rs:207-221). */
int catnn_grouped_gemm(catnn_ctx* ctx, int trans_b, int64_t rows, int64_t N, int64_t K, int64_t groups,
                       const int32_t* offsets, const void* A, const void* B, void* C, int dtype, int c_dtype);
/* The SwiGLU expert GEMMs with the activation in the tensor-core GEMM's
 * epilogue (bf16 only; mid a multiple of 128; each group's rows a multiple
 * of 128 as catnn_moe_permute_map with align 128 gives them). w13 [groups,
 * hidden, 2·mid] holds each expert's w1 and w3 columns interleaved in blocks
 * of 128 (block j: w1 columns 128j..128j+127, then the same w3 columns), and
 * ac / dac use that column layout too.
 * _fwd: per group g, ac = x_g·w13_g ([a | c] rounded to bf16) and
 *       h = silu(a)·c [rows, mid] from the rounded a, c — the first half of
 *       moe::swiglu (moe.rs:159-174).
 * _bwd: per group g, dh = dy_g·w2_gᵀ (w2 [groups, mid, hidden]) rounded to
 *       bf16 and, from the saved ac, dac = [da | dc] with da = dh·c·silu'(a),
 *       dc = dh·silu(a) — swiglu_backward's activation adjoint
 *       (adjoint.rs:239-242); dh itself is never stored. */
int catnn_moe_expert_swiglu_fwd(catnn_ctx* ctx, const void* x, const void* w13, const int32_t* offsets,
                                int64_t rows, int64_t hidden, int64_t mid, int64_t groups, void* ac, void* h);
int catnn_moe_expert_swiglu_bwd(catnn_ctx* ctx, const void* dy, const void* w2, const void* ac,
                                const int32_t* offsets, int64_t rows, int64_t hidden, int64_t mid,
                                int64_t groups, void* dac);
/* SwiGLU expert w2(silu(x·w1) ⊙ (x·w3)) on x [T,hidden]. moe::swiglu (moe.rs:159). */
int catnn_swiglu_fwd(catnn_ctx* ctx, const void* x, const void* w1, const void* w3, const void* w2,
                     void* y, int64_t T, int64_t hidden, int64_t mid, int dtype);
/* swiglu_backward (adjoint.rs:217). */
int catnn_swiglu_bwd(catnn_ctx* ctx, const void* x, const void* w1, const void* w3, const void* w2,
                     const void* dy, void* dx, void* dw1, void* dw3, void* dw2, int64_t T,
                     int64_t hidden, int64_t mid, int dtype);
/* Full MoE block: route, permute, grouped SwiGLU experts, weighted
 * unpermute. w1s/w3s [E,hidden,mid], w2s [E,mid,hidden]. moe::moe (moe.rs:197). */
int catnn_moe_fwd(catnn_ctx* ctx, const void* x, const void* gate, const void* w1s, const void* w3s,
                  const void* w2s, void* y, int64_t T, int64_t hidden, int64_t mid, int64_t E,
                  int64_t k, int dtype);
/* moe_backward (adjoint.rs:471) including the router STE adjoint
 * (adjoint.rs:255). */
int catnn_moe_bwd(catnn_ctx* ctx, const void* x, const void* gate, const void* w1s, const void* w3s,
                  const void* w2s, const void* dy, void* dx, void* dgate, void* dw1s, void* dw3s,
                  void* dw2s, int64_t T, int64_t hidden, int64_t mid, int64_t E, int64_t k, int dtype);

/* ------------------------------------------------------------ optimizers */
/* p -= lr·g (Sgd::put, crates/catnn-core/src/lens/optim.rs:32). fp32
 * master; shadow_bf16 (optional) receives bf16(p). */
int catnn_sgd(catnn_ctx* ctx, float* p, const float* g, int64_t n, float lr, void* shadow_bf16);
/* One Adam step at step count t (t >= 1, already incremented), in place on
 * p, m, v (Adam::put, optim.rs:95-119; bias correction 1-β^t, divisors
 * clamped at 1e-30). g may be fp32 or bf16 (g_dtype). */
int catnn_adam(catnn_ctx* ctx, float* p, const void* g, float* m, float* v, int64_t n, uint64_t t,
               float lr, float beta1, float beta2, float eps, int g_dtype, void* shadow_bf16);

/* ------------------------------------------------------------ training steps */
/* One MLP step: forward, loss, backward (train::mlp_step, train.rs:71).
 * ce=1: softmax cross-entropy on labels (u32 [batch]); ce=0: MSE on
 * y_mse [batch,dout]. Gradients into dw1 [din,hid], db1, dw2 [hid,dout],
 * db2 (fp32). loss: device fp32 scalar. Uses context scratch. */
int catnn_mlp_step(catnn_ctx* ctx, const float* w1, const float* b1, const float* w2, const float* b2,
                   const float* x, const uint32_t* labels, const float* y_mse, int ce, int64_t batch,
                   int64_t din, int64_t hid, int64_t dout, float* loss, float* dw1, float* db1,
                   float* dw2, float* db2);

/* ------------------------------------------------------------ MoE decoder trainer */
/* Shapes and optimizer of a Mixtral-style decoder (the fields of
 * MixtralConfig, crates/catnn-core/src/spec/mixtral.rs:28-51, plus the step's
 * batch/seq and the update rule). window <= 0: no sliding window.
 * optimizer: 0 = SGD (Sgd::put), 1 = Adam (Adam::put). */
typedef struct catnn_moe_config {
    int64_t vocab, hidden, mid, layers, heads, kv_heads, experts, top_k, window, batch, seq;
    float rms_eps;
    double rope_theta;
    int dtype;
    int optimizer;
    float lr, beta1, beta2, adam_eps;
} catnn_moe_config;

typedef struct catnn_moe_trainer catnn_moe_trainer;

/* Allocates parameters (fp32 master + optimizer state + bf16 shadow),
 * activations and scratch on the context's device. */
int catnn_moe_trainer_create(catnn_ctx* ctx, const catnn_moe_config* cfg, catnn_moe_trainer** out);
int catnn_moe_trainer_destroy(catnn_moe_trainer* t);
/* Element count of the packed fp32 parameter vector: embed [V,d]; per layer
 * rms_attn, wq, wk, wv, wo, rms_moe, gate, w1[E], w3[E], w2[E]; final norm;
 * LM head [V,d] — the MixtralWeights fields (moe.rs:227-244) in order. */
int catnn_moe_trainer_param_count(const catnn_moe_config* cfg, int64_t* out);
/* Load parameters from / export parameters or last gradients to a packed
 * fp32 device vector. Loading resets the optimizer state. */
int catnn_moe_trainer_set_params(catnn_moe_trainer* t, const float* packed_dev);
int catnn_moe_trainer_get_params(catnn_moe_trainer* t, float* packed_dev);
int catnn_moe_trainer_get_grads(catnn_moe_trainer* t, float* packed_dev);
/* One training step on device token ids [batch*seq]: forward with residual
 * adds, next-token cross-entropy (targets[i] = tokens[(i+1) % n] % vocab),
 * backward, and the update when update != 0. loss_dev (optional) receives
 * the mean loss. Asynchronous. train::mixtral_step + apply_grads_sgd
 * (crates/catnn-compile/src/train.rs:261-356, :403) / Adam::put. */
int catnn_moe_trainer_step(catnn_moe_trainer* t, const uint32_t* tokens_dev, float* loss_dev, int update);
/* The same step from host token ids to a host loss (copies inside; synchronous). */
int catnn_moe_trainer_step_host(catnn_moe_trainer* t, const uint32_t* tokens_host, float* loss_host, int update);
/* Copies a saved activation of the last step to out (fp32): which = 0 x_in
 * [T,d] (input of `layer`), 1 x_mid [T,d], 2 normalized MoE input [T,d],
 * 3 attention context [T,H·hd], 4 router logits [T,E], 5 final residual
 * [T,d], 6 final normalized [T,d] (layer ignored for 5 and 6). The
 * device-resident counterpart of the activations coord::ensure_act
 * rematerializes (crates/catnn-rt/src/coord.rs:436-473). */
int catnn_moe_trainer_activation(catnn_moe_trainer* t, int which, int64_t layer, float* out);
/* Synchronizes and reports device-side errors of earlier steps (token id or
 * target out of range, a bounded wait that ran out). */
int catnn_moe_trainer_check(catnn_moe_trainer* t);
/* enable != 0: later steps replay a CUDA graph of the step body (forward,
 * backward, updates, and for an expert-parallel trainer its device barriers,
 * peer-memory exchanges and NCCL allreduces) on the trainer's own stream,
 * ordered after the work already on the context stream; the first step with
 * and without update runs eagerly and sizes every workspace, the second is
 * captured. Same results as eager steps. Tensor shapes and buffers are fixed
 * per trainer, so a graph never goes stale; disable to release the graphs.
 * On an expert-parallel trainer every rank must use the same setting. */
int catnn_moe_trainer_set_graphs(catnn_moe_trainer* t, int enable);
/* Phase timeline of a step, for finding where a rank's step time goes
 * (the reference's simulated per-layer timeline, train.rs
 * mixtral_layer_timeline_excerpt, measured instead). With profiling on, the
 * step records the device clock (%globaltimer, ns) on its stream at each
 * phase boundary (the start, after the embedding, after each layer's
 * attention and MoE halves, after the loss, after each layer's MoE and
 * attention adjoints, after the embedding gradient, after the last gradient
 * all-reduce, after the updates). Turning it on or off drops captured step
 * graphs. catnn_moe_trainer_timeline copies the last step's stamps (up to
 * max) into ns and their names, separated by '\n', into names (names_len
 * bytes); *count receives the number of stamps. Synchronizes. */
int catnn_moe_trainer_set_profile(catnn_moe_trainer* t, int enable);
int catnn_moe_trainer_timeline(catnn_moe_trainer* t, int64_t* ns, int max, char* names, int64_t names_len,
                               int* count);

/* ------------------------------------------------------------ multi-GPU (one node) */
/* One rank of a group of 1..8 processes, one GPU each. The reference runs
 * one device handler per device and moves tensors between them on the host
 * (crates/catnn-rt/src/dist.rs:441-517, transfer.rs); it models expert
 * parallelism as E/EP experts per rank with an activation all-to-all
 * (crates/catnn-compile/src/spark_place.rs:119-131,196). Here NCCL carries
 * the bulk collectives and CUDA IPC peer mappings over NVLink carry the
 * fused expert dispatch/combine. Device waits are bounded (default 10 s,
 * catnn_comm_set_timeout_ms); a wait that runs out makes the next
 * catnn_comm_check / catnn_moe_trainer_check return CATNN_ERR_TIMEOUT. */
typedef struct catnn_comm catnn_comm;
#define CATNN_COMM_ID_BYTES 128
/* Rank 0 creates the group id (CATNN_COMM_ID_BYTES bytes) and sends it to
 * every rank over any host channel. */
int catnn_comm_unique_id(void* id_out);
/* Collective over all ranks. world == 1 needs no id (id may be NULL). */
int catnn_comm_create(catnn_ctx* ctx, int rank, int world, const void* id, catnn_comm** out);
int catnn_comm_destroy(catnn_comm* comm);
int catnn_comm_rank(catnn_comm* comm, int* rank, int* world);
int catnn_comm_set_timeout_ms(catnn_comm* comm, int64_t ms);
/* In-place sum over ranks of n elements (CATNN_F32 or CATNN_BF16), on the context stream. */
int catnn_comm_allreduce(catnn_comm* comm, void* buf, int64_t n, int dtype);
/* Bytes send[off_p .. off_p + send_bytes[p]) go to rank p, which receives
 * them at recv + (sum of recv_bytes before this rank); counts are host arrays of world entries. */
int catnn_comm_all_to_all(catnn_comm* comm, const void* send, const int64_t* send_bytes, void* recv,
                          const int64_t* recv_bytes);
/* Device barrier on peer flags (bounded waits). */
int catnn_comm_barrier(catnn_comm* comm);
/* Point-to-point flag primitives under the barrier: signal sets this
 * rank's flag at `peer` to epoch (synchronous); wait enqueues a bounded wait
 * until peer's flag at this rank reaches epoch. For diagnostics and tests. */
int catnn_comm_signal(catnn_comm* comm, int peer, uint64_t epoch);
int catnn_comm_wait(catnn_comm* comm, int peer, uint64_t epoch);
/* Synchronizes; CATNN_ERR_TIMEOUT if a device wait gave up (and clears it). */
int catnn_comm_check(catnn_comm* comm);

/* Data-parallel + expert-parallel trainer over the ranks of comm.
 * cfg->batch is the GLOBAL batch: rank r trains sequences
 * [r*batch/world, (r+1)*batch/world) and owns experts
 * [r*experts/world, (r+1)*experts/world) of every layer. The embedding
 * table is vocab-sharded (rank r owns rows [r*ceil(vocab/world), ...): their
 * gradient, from every rank's token rows read over NVLink, and their update);
 * the other parameters are replicated: norm and router weights are
 * allreduced and updated on every rank, the attention and LM-head weights
 * are reduce-scattered, updated in chunks and their storage-dtype copy
 * all-gathered (NCCL). Needs batch % world == 0 and experts % world == 0.
 * Steps take the GLOBAL token array [batch*seq] on every rank and report the
 * global mean loss; set_params reads the full packed vector; get_params /
 * get_grads are collective (every rank calls them: they first all-gather the
 * sharded fp32 values) and write the replicated parameters and this rank's
 * experts into a full packed vector, leaving the other experts' entries
 * untouched. activation() returns this rank's rows. With world == 1 it is
 * the single-GPU trainer. */
int catnn_moe_trainer_create_ep(catnn_ctx* ctx, const catnn_moe_config* cfg, catnn_comm* comm,
                                catnn_moe_trainer** out);

/* ------------------------------------------------------------ kernel resources */
/* The measured KernelResource of an IR op on this backend — what
 * resource::describe (crates/catnn-compile/src/kernel/resource.rs:159-193)
 * returns for the CudaSm121 backend as estimates, here for the sm_100a
 * kernel the op's launcher actually runs: registers per thread, static and
 * local memory and the kernel-argument bytes from the CUDA runtime; the
 * launch geometry and dynamic shared memory the launcher uses for `shape`;
 * the code size as the cubin of the kernel's source file, measured at build
 * time (code_estimated = 0). op: linear, matmul, lm_head, moe, attention,
 * gqa_attention, embedding, rms_norm, layer_norm, softmax, cross_entropy,
 * relu, gelu, add, residual_add, mul, router, swiglu, sgd, adam; other ops
 * are CATNN_ERR_UNSUPPORTED. shape: GEMMs M = rows, N = width, K = inner;
 * row kernels rows x width; attention batch, seq, heads, head_dim. */
typedef struct catnn_kernel_shape {
    int64_t rows, width, inner;
    int64_t batch, seq, heads, head_dim;
} catnn_kernel_shape;
typedef struct catnn_kernel_resource {
    char kernel[192];  /* the __global__ function (mangled name) */
    char file[32];     /* the source file it is compiled from */
    int32_t registers_per_thread;
    int32_t max_threads_per_block;
    int64_t static_smem_bytes;
    int64_t dynamic_smem_bytes;
    int64_t local_bytes_per_thread;
    uint32_t grid[3];
    uint32_t block[3];
    int64_t launch_arg_bytes;
    int64_t code_bytes;
    int32_t code_estimated;
    int32_t binary_version;
} catnn_kernel_resource;
int catnn_kernel_describe(catnn_ctx* ctx, const char* op, int dtype, const catnn_kernel_shape* shape,
                          catnn_kernel_resource* out);

#ifdef __cplusplus
}
#endif
#endif /* CATNN_B200_H */
