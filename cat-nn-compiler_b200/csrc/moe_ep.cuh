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

// Vocab-sharded embedding: rank r holds the authoritative rows
// [r*rows_per_rank, (r+1)*rows_per_rank) of the table (table.p[r] is its
// copy of the whole table's address range).
//  ep_embedding_fwd: y[t] = table.p[owner(id)][id] for this rank's n tokens,
//    read over NVLink (ids >= vocab set *err and give zeros, as embedding_fwd);
//  ep_embedding_keys + ep_embedding_runs: for this rank's rows [v0, v1), dw[v] = the sum in global
//    token order of dy rows of every token with id v, dy of global token t
//    read from rank t / tokens_per_rank (the order embedding_bwd sums in on
//    one GPU). dw is the whole table's gradient; only rows [v0, v1) are written.
void ep_embedding_fwd(Context* c, const uint32_t* ids, i64 n, const PeerTab& table, i64 vocab, i64 rows_per_rank,
                      i64 hidden, float* y, int* err);
// in two launches: the keys (they depend on the ids only: keys n_global
// uint32, *m their count) and the run sums
void ep_embedding_keys(Context* c, const uint32_t* ids_global, i64 n_global, i64 v0, i64 v1, uint32_t* keys, int* m);
void ep_embedding_runs(Context* c, const uint32_t* keys, const int* m, i64 n_global, i64 tokens_per_rank,
                       const PeerTab& dy, i64 v0, i64 v1, i64 hidden, float* dw);

}  // namespace catnn
