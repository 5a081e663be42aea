// Expert-parallel dispatch / combine over peer memory (moe_ep.cu).
#pragma once
#include "comm.cuh"

namespace catnn {

// Set when a layer's plan needs more receive rows than were allocated.
constexpr int EP_STATUS_SLOT = 11;

// The same buffer on every rank, as addressed from this process.
struct PeerTab {
    void* p[COMM_MAX_WORLD];
};

// plan layout (int32): off_own[El + 1], total_own[El], base[E].
inline i64 ep_plan_len(i64 E, i64 El) { return 2 * El + 1 + E; }

void ep_publish_counts(Context* c, const int32_t* counts, const PeerTab& cnt_all, int rank, int world, int E);
void ep_plan(Context* c, const int32_t* counts_all, int rank, int world, int E, int El, int align, int32_t* plan,
             i64 rows_cap);
void ep_dispatch(Context* c, const void* x, const int32_t* idx, const int32_t* row_of1, const int32_t* off1,
                 const int32_t* plan, const PeerTab& xp, const PeerTab& src, int32_t* dest, i64 T, int k, i64 hidden,
                 int El, int align, int rank, int world, i64 rows_cap, int dtype);
void ep_combine(Context* c, const PeerTab& yp, const int32_t* idx, const int32_t* dest, const float* w, i64 T, int k,
                i64 hidden, int El, int world, i64 rows_cap, float* y, const float* resid, int yp_dtype);
void ep_unpermute_bwd(Context* c, const void* yp, const int32_t* src, const int32_t* plan, const PeerTab& w,
                      const PeerTab& dy, const PeerTab& dw, i64 rows_cap, i64 pairs, int k, i64 hidden, int El,
                      int world, void* dyp, int dtype);
void ep_permute_bwd(Context* c, const PeerTab& dxp, const int32_t* idx, const int32_t* dest, i64 T, int k, i64 hidden,
                    int El, int world, i64 rows_cap, float* dx, int dtype);

}  // namespace catnn
