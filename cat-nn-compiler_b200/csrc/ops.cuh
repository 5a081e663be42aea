// Internal launch API of libcatnn_b200. The extern "C" layer (capi.cu) and
// the composite training steps (train.cu) both call these; every launcher
// enqueues on ctx->stream and counts its launches.
#pragma once
#include "common.cuh"

struct catnn_ctx {
    catnn::Context c;
};

#define ABI_BEGIN try {
#define ABI_END                                \
    return CATNN_OK;                           \
    }                                          \
    catch (const ::catnn::Error& e) {          \
        ::catnn::set_last_error(e.what());     \
        return e.code;                         \
    }                                          \
    catch (const std::exception& e) {          \
        ::catnn::set_last_error(e.what());     \
        return CATNN_ERR_INVALID;              \
    }

namespace catnn {

Context* unwrap(catnn_ctx* h);

// One kernel of this library as catnn_kernel_describe reports it: the host
// stub of the __global__ function, the translation unit it is compiled in
// (whose cubin size is the code size), and the launch geometry its launcher
// uses for a problem of the given shape. fn is null when a file has no
// kernel for the op.
struct KShape {
    i64 rows, width, inner;    // GEMM: M, N, K; row kernels: rows x width
    i64 batch, seq, heads, head_dim;
};
struct KernelInfo {
    const void* fn = nullptr;
    const char* file = "";
    unsigned grid[3] = {1, 1, 1};
    unsigned block[3] = {1, 1, 1};
    size_t dyn_smem = 0;
};
// per-file lookups of the kernel that carries an IR op (resource.cu)
KernelInfo gemm_tc_info(Context* c, const std::string& op, const KShape& s);
KernelInfo sgemm_info(Context* c, const std::string& op, const KShape& s);
KernelInfo fa5_info(Context* c, const std::string& op, const KShape& s);
KernelInfo attention_info(Context* c, const std::string& op, int dtype, const KShape& s);
KernelInfo norms_info(Context* c, const std::string& op, int dtype, const KShape& s);
KernelInfo elementwise_info(Context* c, const std::string& op, int dtype, const KShape& s);
KernelInfo moe_info(Context* c, const std::string& op, int dtype, const KShape& s);

// Reads and clears device status slot `slot` of the context; synchronizes
// the stream. Returns the value that was there.
int take_status(Context* c, int slot);

// The allocation-free cross-entropy's row-loss array (norms.cu): its device
// address on `device`, resolved once per device with that device current.
// catnn_ctx_create calls this, so that the lookup (which can load the
// library's code on the device) happens where allocation is allowed;
// xent_noalloc_forget drops the address when the device's last context is
// destroyed (a later cudaDeviceReset invalidates it).
float* xent_row_loss_buffer(int device);
void xent_noalloc_forget(int device);

inline size_t dsize(int dtype) { return dtype == CATNN_BF16 ? 2 : 4; }
inline void check_dtype(int dtype) {
    CATNN_CHECK(dtype == CATNN_F32 || dtype == CATNN_BF16, CATNN_ERR_DTYPE,
                "dtype must be CATNN_F32 or CATNN_BF16");
}

// ---- dense (gemm.cu / gemm_tc.cu)
// C = act(op(A)op(B) + bias) (+C). See catnn_gemm in catnn_b200.h.
// resid (fp32 [M, ldc], optional) is added before the activation; it needs
// an fp32 C (the residual stream: x_out = x_in + A·B in one pass).
void gemm(Context* c, bool ta, bool tb, i64 M, i64 N, i64 K, const void* A, i64 lda, const void* B,
          i64 ldb, void* C, i64 ldc, int dtype, int c_dtype, const float* bias, int act, bool accumulate,
          const float* resid = nullptr);
void gemm_f32(Context* c, bool ta, bool tb, i64 M, i64 N, i64 K, const float* A, i64 lda, const float* B,
              i64 ldb, void* C, i64 ldc, int c_dtype, const float* bias, int act, bool accumulate,
              const float* resid = nullptr);
// bf16 operands on tcgen05 tensor cores, fp32 accumulation in TMEM.
void gemm_bf16_tc(Context* c, bool ta, bool tb, i64 M, i64 N, i64 K, const bf16* A, i64 lda,
                  const bf16* B, i64 ldb, void* C, i64 ldc, int c_dtype, const float* bias, int act,
                  bool accumulate, const float* resid = nullptr);
// Grouped variant: for each group g, rows [off[g], off[g+1]) of A (and C)
// against B_g = B + g*strideB. A is [rows,K] row-major; B_g is [K,N]
// (tb=0) or [N,K] (tb=1). Offsets live on the device.
void gemm_grouped_bf16_tc(Context* c, bool tb, i64 total_rows, i64 N, i64 K, int groups,
                          const int32_t* offsets, const bf16* A, i64 lda, const bf16* B, i64 strideB,
                          i64 ldb, void* C, i64 ldc, int c_dtype, int act, bool accumulate = false);
// Grouped weight-gradient: dB_g[K,N] = A_gᵀ·D_g over the rows of group g.
void gemm_grouped_wgrad_bf16_tc(Context* c, i64 total_rows, i64 N, i64 K, int groups,
                                const int32_t* offsets, const bf16* A, i64 lda, const bf16* D, i64 ldd,
                                void* dB, i64 strideB, int c_dtype, bool accumulate);
// fp32 grouped GEMM for the parity path (same conventions).
// fp32 operands on the tensor cores as TF32 (gemm_tc.cu).
void gemm_tf32_tc(Context* c, bool ta, bool tb, i64 M, i64 N, i64 K, const float* A, i64 lda, const float* B, i64 ldb,
                  void* C, i64 ldc, int c_dtype, const float* bias, int act, bool accumulate);
// The expert GEMMs with the SwiGLU fused into the epilogue (gemm_tc.cu):
// W13 / AC / DAC use the 128-column interleaved [a | c] layout.
void gemm_grouped_swiglu_fwd_tc(Context* c, i64 total_rows, i64 F, i64 K, int groups, const int32_t* offsets,
                                const bf16* X, i64 ldx, const bf16* W13, bf16* AC, bf16* H);
void gemm_grouped_swiglu_bwd_tc(Context* c, i64 total_rows, i64 F, i64 K, int groups, const int32_t* offsets,
                                const bf16* DY, i64 lddy, const bf16* W2, const bf16* AC, bf16* DAC);
void gemm_grouped_f32(Context* c, bool ta_rows, bool tb, i64 total_rows, i64 N, i64 K, int groups,
                      const int32_t* offsets, const float* A, i64 lda, const float* B, i64 strideB,
                      i64 ldb, float* C, i64 ldc, i64 strideC, bool accumulate);

// ---- elementwise (elementwise.cu)
void act_fwd(Context* c, int act, const void* x, void* y, i64 n, int dtype);
void act_bwd(Context* c, int act, const void* x, const void* dy, void* dx, i64 n, int dtype);
void add(Context* c, const void* a, const void* b, void* y, i64 n, i64 b_len, int dtype);
void mul(Context* c, const void* a, const void* b, void* y, i64 n, int dtype);
void cast(Context* c, const void* x, int xd, void* y, int yd, i64 n);
void fill_f32(Context* c, float* p, float v, i64 n);
// out[j] (+)= Σ_rows x[r, j], rows summed in order per column.
void col_sum(Context* c, const void* x, i64 rows, i64 cols, float* out, int dtype, bool accumulate);
void sgd(Context* c, float* p, const float* g, i64 n, float lr, bf16* shadow);
void adam(Context* c, float* p, const void* g, float* m, float* v, i64 n, uint64_t t, float lr, float b1,
          float b2, float eps, int g_dtype, bf16* shadow, const float* d12_dev = nullptr);
// Adam bias-correction divisors max(1 - b^t, 1e-30) for step t (host).
void adam_divisors(uint64_t t, float b1, float b2, float* d12);

// ---- softmax / losses / norms (norms.cu)
void softmax_fwd(Context* c, const void* x, void* y, i64 rows, i64 last, int dtype);
void softmax_bwd(Context* c, const void* y, const void* dy, void* dx, i64 rows, i64 last, int dtype);
// loss: device fp32 scalar (written, not accumulated). err: device int set
// to 1 when a target is out of range (may be null). denom (0: rows) is the
// count the mean divides by — the global token count when the rows are one
// rank's share of a batch.
void xent_fwdbwd(Context* c, const void* logits, const uint32_t* targets, i64 rows, i64 vocab, float* loss,
                 void* dlogits, int dtype, int* err, i64 denom = 0);
void mse_fwdbwd(Context* c, const float* pred, const float* target, i64 n, float* loss, float* d);
void layernorm_fwd(Context* c, const void* x, const float* g, const float* b, void* y, i64 rows, i64 last,
                   float eps, int dtype);
void layernorm_bwd(Context* c, const void* x, const float* g, const void* dy, void* dx, float* dg, float* db,
                   i64 rows, i64 last, float eps, int dtype);
void rmsnorm_fwd(Context* c, const void* x, const float* w, void* y, i64 rows, i64 last, float eps, int dtype);
// dw_accumulate: add into dw instead of overwriting it.
void rmsnorm_bwd(Context* c, const void* x, const float* w, const void* dy, void* dx, float* dw, i64 rows,
                 i64 last, float eps, int dtype, bool dw_accumulate, const void* dres = nullptr);

// Mixed storage: fp32 residual stream in, bf16 (or fp32) normalized out.
// The MoE input in one pass (width a multiple of 1024 up to 2048, E <= 16,
// aligned rows): bf16 and fp32 RMSNorm outputs and the router logits
// y32·gate. Returns false (nothing launched) when the shape does not fit.
bool rms_router_fused(Context* c, const float* x, const float* w, const float* gate, i64 E, i64 rows, i64 last,
                      float eps, bf16* y16, float* y32, float* logits);
void rmsnorm_fwd_mixed(Context* c, const void* x, int x_dtype, const float* w, void* y, int y_dtype, i64 rows, i64 last,
                       float eps);
// dx (fp32) = rmsnorm adjoint of dy (g_dtype) at x (fp32) + dres (fp32, optional);
// copy (optional, copy_dtype) receives dx too; dw (+)= Σ dy·x·inv.
void rmsnorm_bwd_mixed(Context* c, const float* x, const float* w, const void* dy, int g_dtype, const float* dres, float* dx,
                       void* copy, int copy_dtype, float* dw, bool dw_acc, i64 rows, i64 last, float eps);

// ---- embedding / attention (attention.cu)
void embedding_fwd(Context* c, const uint32_t* ids, i64 n, const void* table, i64 vocab, i64 hidden, void* y,
                   int dtype, int* err);
void embedding_bwd(Context* c, const uint32_t* ids, i64 n, const void* dy, float* dw, i64 vocab, i64 hidden,
                   int dtype);
// The two halves of embedding_bwd: the sorted (id, token) keys, which depend
// on the ids only (keys: n uint32), and the run sums from them.
void embedding_bwd_keys(Context* c, const uint32_t* ids, i64 n, i64 vocab, uint32_t* keys);
void embedding_bwd_runs(Context* c, const uint32_t* keys, i64 n, const void* dy, float* dw, i64 vocab, i64 hidden,
                        int dtype);
void rope(Context* c, void* x, i64 b, i64 s, i64 heads, i64 hd, double theta, bool inverse, int dtype,
          i64 row_stride = 0, i64 col_off = 0);
void attention_fwd(Context* c, const void* q, const void* k, const void* v, void* o, float* lse, i64 b, i64 s,
                   i64 h, i64 hkv, i64 hd, bool causal, i64 window, int dtype, i64 q_stride = 0,
                   i64 kv_stride = 0);
void attention_bwd(Context* c, const void* q, const void* k, const void* v, const void* o, const float* lse,
                   const void* dout, void* dq, void* dk, void* dv, i64 b, i64 s, i64 h, i64 hkv, i64 hd,
                   bool causal, i64 window, int dtype, i64 q_stride = 0, i64 kv_stride = 0);

// ---- MoE (moe.cu)
void router_topk(Context* c, const float* logits, i64 T, i64 E, i64 k, int32_t* idx, float* w);
// Stable counting sort of the T*k (token, slot) pairs by expert; each
// expert's rows padded to `align`; fails (status) if rows exceed rows_cap.
// src_of[r] = pair index t*k+j of row r, or -1 on padding rows.
void permute_map(Context* c, const int32_t* idx, i64 T, i64 E, i64 k, int align, i64 rows_cap, int32_t* counts,
                 int32_t* offsets, int32_t* row_of, int32_t* src_of);
void permute_rows(Context* c, const void* x, const int32_t* src_of, i64 rows, i64 hidden, i64 k, void* xp, int dtype);
// yp_dtype (default: dtype) lets an fp32 expert output feed a bf16 result.
// resid (optional, y's storage): y = resid + Σ_j w·yp, the residual add of x + moe(x).
void unpermute_rows(Context* c, const void* yp, const int32_t* row_of, const float* w, i64 T, i64 k, i64 hidden,
                    void* y, int dtype, bool accumulate, int yp_dtype = -1, const void* resid = nullptr);
// Over sorted rows r (pair p = src_of[r], token t = p/k):
// d_w[p] = <yp[r], dy[t]>; dyp[r] = w[p]*dy[t]; zeros on padding rows.
void unpermute_bwd(Context* c, const void* yp, const int32_t* src_of, i64 rows, const float* w, const void* dy, i64 k,
                   i64 hidden, float* dw, void* dyp, int dtype, int yp_dtype = -1, int dy_dtype = -1);
// dx[t] (+)= Σ_j dxp[row_of[t,j]].
void permute_bwd(Context* c, const void* dxp, const int32_t* row_of, i64 T, i64 k, i64 hidden, void* dx,
                 int dtype, bool accumulate, int out_dtype = -1);
// Router STE: dlogits[t, idx[t,j]] = w*(g - <w,g>), zero elsewhere.
void router_ste(Context* c, const int32_t* idx, const float* w, const float* dw, i64 T, i64 E, i64 k,
                float* dlogits);
// h = silu(a) * c with a, c read from one [rows, 2F] buffer ([a | c]) or
// separate buffers; and its adjoint.
// in_dtype (default: dtype) is the storage of a, c (and dh): fp32 pre-activations
// may feed bf16 outputs.
// rows_dev (optional, device int): only the first min(rows, *rows_dev) rows
// are computed (the rows an expert-parallel rank actually received).
void swiglu_act(Context* c, const void* a, const void* cc, void* h, i64 rows, i64 F, i64 lda, i64 ldh,
                int dtype, int in_dtype = -1, const int32_t* rows_dev = nullptr);
void swiglu_act_bwd(Context* c, const void* a, const void* cc, const void* dh, void* da, void* dc, i64 rows,
                    i64 F, i64 lda, i64 ldd, int dtype, int in_dtype = -1, const int32_t* rows_dev = nullptr);

}  // namespace catnn
