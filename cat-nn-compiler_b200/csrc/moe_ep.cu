// Expert-parallel MoE exchange over NVLink peer memory, fused with the
// permutation it serves: the dispatch kernel writes each routed row straight
// into the expert owner's receive buffer, the combine kernel reads the
// owners' expert outputs while it forms the weighted sum, and the two
// backward kernels mirror them. Rows land in the owner's buffer grouped by
// expert, padded like the one-GPU path, and ordered by global pair index
// (source rank, token, slot) — the order the one-GPU permutation gives
// (moe.rs:186-205 groups pairs by expert in pair order) — so every expert
// GEMM sees the rows it would see on one GPU. The arithmetic of each kernel
// is that of its one-GPU counterpart in moe.cu, element for element.
//
// Synchronisation: kernels only touch peer memory between two device
// barriers (Comm::barrier); the trainer places the barriers.
#include "moe_ep.cuh"

namespace catnn {

// Plan of one layer from counts_all [world][E] (pairs rank s routes to
// expert e). Written by one thread:
//   off_own[0..El]   row offsets of this rank's experts in its receive buffer
//   total_own[El]    rows actually received per own expert (the rest is padding)
//   base[E]          first row, in expert e's owner buffer, of this rank's pairs for e
__global__ void k_ep_plan(const int32_t* __restrict__ counts_all, int rank, int world, int E, int El, int align,
                          int32_t* __restrict__ plan, int64_t rows_cap, int* err) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    int32_t* off_own = plan;
    int32_t* total_own = plan + El + 1;
    int32_t* base = plan + 2 * El + 1;
    int64_t off = 0;  // running offset inside the current owner's buffer
    for (int e = 0; e < E; ++e) {
        if (e % El == 0) off = 0;
        int64_t tot = 0, before = 0;
        for (int s = 0; s < world; ++s) {
            int64_t n = counts_all[s * E + e];
            if (s < rank) before += n;
            tot += n;
        }
        base[e] = (int32_t)(off + before);
        int owner = e / El;
        if (owner == rank) {
            off_own[e - rank * El] = (int32_t)off;
            total_own[e - rank * El] = (int32_t)tot;
        }
        off += (tot + align - 1) / align * align;
        if (off > rows_cap && err) atomicExch(err, 1);
        if (owner == rank && e % El == El - 1) off_own[El] = (int32_t)off;
    }
}

// Pair i = t*k + j of this rank (expert e = idx[i], local rank within e from
// the align-1 local map) goes to row base[e] + (row_of1[i] - off1[e]) of the
// owner's buffer: its x row is copied there, the owner's src tag of that row
// becomes the global pair id rank*T*k + i, and dest[i] remembers the row.
// Slots past the pairs zero this rank's own padding rows (tag -1).
template <typename T, int V>
__global__ void __launch_bounds__(128) k_ep_dispatch(const T* __restrict__ x, const int32_t* __restrict__ idx,
                                                     const int32_t* __restrict__ row_of1,
                                                     const int32_t* __restrict__ off1, const int32_t* __restrict__ plan,
                                                     PeerTab xp_tab, PeerTab src_tab, int32_t* __restrict__ dest,
                                                     i64 Tn, int k, i64 hidden, int El, int align, int rank, int world,
                                                     i64 rows_cap, int* __restrict__ err) {
    const int lane = threadIdx.x & 31;
    const i64 pairs = Tn * k;
    const i64 slot = (i64)blockIdx.x * 4 + (threadIdx.x >> 5);
    const int32_t* off_own = plan;
    const int32_t* total_own = plan + El + 1;
    const int32_t* base = plan + 2 * El + 1;
    if (slot < pairs) {
        const int e = idx[slot];
        const int owner = e / El;
        const i64 row = (e >= 0 && owner < world) ? (i64)base[e] + (row_of1[slot] - off1[e]) : -1;
        if (row < 0 || row >= rows_cap) {  // never for a valid plan; no peer write then
            if (lane == 0) {
                dest[slot] = -1;
                atomicExch(err, 1);
            }
            return;
        }
        if (lane == 0) {
            dest[slot] = (int32_t)row;
            ((int32_t*)src_tab.p[owner])[row] = (int32_t)((i64)rank * pairs + slot);
        }
        const T* s = x + (slot / k) * hidden;
        T* d = (T*)xp_tab.p[owner] + row * hidden;
        for (i64 c = (i64)lane * V; c < hidden; c += 32 * V) {
            float v[V];
            ldv<T, V>(s + c, v);
            stv<T, V>(d + c, v);
        }
        __threadfence_system();
        return;
    }
    // padding rows of this rank's own experts
    const i64 q = slot - pairs;
    const int j = (int)(q / align);
    if (j >= El) return;
    const i64 row = (i64)off_own[j] + total_own[j] + (q - (i64)j * align);
    if (row >= off_own[j + 1] || row >= rows_cap) return;
    if (lane == 0) ((int32_t*)src_tab.p[rank])[row] = -1;
    T* d = (T*)xp_tab.p[rank] + row * hidden;
    float z[V];
#pragma unroll
    for (int u = 0; u < V; ++u) z[u] = 0.f;
    for (i64 c = (i64)lane * V; c < hidden; c += 32 * V) stv<T, V>(d + c, z);
}

// y[t] = resid[t] + Σ_j w[t,j] · yp_owner(j)[dest[t,j]], slots in order
// (k_unpermute's arithmetic with the rows read from the owners' memory).
template <typename TI, int V>
__global__ void __launch_bounds__(128) k_ep_combine(PeerTab yp_tab, const int32_t* __restrict__ idx,
                                                    const int32_t* __restrict__ dest, const float* __restrict__ w,
                                                    i64 Tn, int k, i64 hidden, int El, int world, i64 rows_cap,
                                                    float* __restrict__ y, const float* __restrict__ resid) {
    for (i64 t = blockIdx.x; t < Tn; t += gridDim.x) {
        for (i64 c = (i64)threadIdx.x * V; c < hidden; c += (i64)blockDim.x * V) {
            float s[V];
#pragma unroll
            for (int u = 0; u < V; ++u) s[u] = 0.f;
            for (int j = 0; j < k; ++j) {
                const i64 p = t * k + j;
                const int o = idx[p] / El;
                const i64 r = dest[p];
                if (idx[p] < 0 || o >= world || r < 0 || r >= rows_cap) continue;  // flagged by the dispatch
                float v[V];
                ldv<TI, V>((const TI*)yp_tab.p[o] + r * hidden + c, v);
                const float wt = w[p];
#pragma unroll
                for (int u = 0; u < V; ++u) s[u] = __fadd_rn(s[u], __fmul_rn(wt, v[u]));
            }
            if (resid) {
                float r[V];
                ldv<float, V>(resid + t * hidden + c, r);
#pragma unroll
                for (int u = 0; u < V; ++u) s[u] = __fadd_rn(r[u], s[u]);
            }
            stv<float, V>(y + t * hidden + c, s);
        }
    }
}

// Owner side of the combine's adjoint, per received row r < off_own[El]
// (global pair g = src[r] = s*T*k + i, token t = i / k on rank s):
// dw_s[i] = <yp[r], dy_s[t]> and dyp[r] = w_s[i] · dy_s[t] (k_unpermute_bwd's
// arithmetic); zeros on padding rows.
template <typename TY, typename T>
__global__ void __launch_bounds__(128) k_ep_unpermute_bwd(const TY* __restrict__ yp, const int32_t* __restrict__ src,
                                                          const int32_t* __restrict__ plan, PeerTab w_tab,
                                                          PeerTab dy_tab, PeerTab dw_tab, i64 pairs, int k,
                                                          i64 hidden, int El, int world, T* __restrict__ dyp) {
    const i64 r = (i64)blockIdx.x * 4 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= plan[El]) return;
    const int g = src[r];
    if (g < 0 || g >= (i64)world * pairs) {
        for (i64 i = lane; i < hidden; i += 32) dyp[r * hidden + i] = T(0.f);
        return;
    }
    const int s = (int)(g / pairs);
    const i64 i = g - (i64)s * pairs;
    const i64 t = i / k;
    const float wt = ((const float*)w_tab.p[s])[i];
    const float* __restrict__ dy = (const float*)dy_tab.p[s] + t * hidden;
    float dot = 0.f;
    // eight of the lane's columns per round: the (remote) loads are all issued
    // before the stores, and the sum runs over the columns in the same order
    for (i64 c0 = lane; c0 < hidden; c0 += 32 * 8) {
        float gv[8], yv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const i64 c = c0 + 32 * u;
            gv[u] = c < hidden ? dy[c] : 0.f;
            yv[u] = c < hidden ? ld(yp + r * hidden + c) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const i64 c = c0 + 32 * u;
            if (c < hidden) {
                dot += yv[u] * gv[u];
                st(dyp + r * hidden + c, __fmul_rn(gv[u], wt));
            }
        }
    }
    dot = warp_sum(dot);
    if (lane == 0) ((float*)dw_tab.p[s])[i] = dot;
}

// dx[t] = Σ_j dxp_owner(j)[dest[t,j]] in slot order (k_permute_bwd's arithmetic).
template <typename TI, int V>
__global__ void __launch_bounds__(128) k_ep_permute_bwd(PeerTab dxp_tab, const int32_t* __restrict__ idx,
                                                        const int32_t* __restrict__ dest, i64 Tn, int k, i64 hidden,
                                                        int El, int world, i64 rows_cap, float* __restrict__ dx) {
    for (i64 t = blockIdx.x; t < Tn; t += gridDim.x) {
        for (i64 c = (i64)threadIdx.x * V; c < hidden; c += (i64)blockDim.x * V) {
            float s[V];
#pragma unroll
            for (int u = 0; u < V; ++u) s[u] = 0.f;
            for (int j = 0; j < k; ++j) {
                const i64 p = t * k + j;
                const int o = idx[p] / El;
                const i64 r = dest[p];
                if (idx[p] < 0 || o >= world || r < 0 || r >= rows_cap) continue;
                float v[V];
                ldv<TI, V>((const TI*)dxp_tab.p[o] + r * hidden + c, v);
#pragma unroll
                for (int u = 0; u < V; ++u) s[u] = __fadd_rn(s[u], v[u]);
            }
            stv<float, V>(dx + t * hidden + c, s);
        }
    }
}

// counts_all[rank][e] := counts[e] on every rank (thread e, one store per rank).
__global__ void k_ep_publish(const int32_t* __restrict__ counts, PeerTab cnt_all, int rank, int world, int E) {
    int e = threadIdx.x;
    if (e >= E) return;
    int32_t v = counts[e];
    for (int p = 0; p < world; ++p) ((int32_t*)cnt_all.p[p])[rank * E + e] = v;
    __threadfence_system();
}

// ---------------------------------------------------------------- launchers

void ep_publish_counts(Context* c, const int32_t* counts, const PeerTab& cnt_all, int rank, int world, int E) {
    k_ep_publish<<<1, 32, 0, c->stream>>>(counts, cnt_all, rank, world, E);
    launched(c);
}

static int row_vec(int dtype, i64 hidden) {
    int v = dtype == CATNN_BF16 ? 8 : 4;
    return hidden % v == 0 ? v : 1;
}

void ep_plan(Context* c, const int32_t* counts_all, int rank, int world, int E, int El, int align, int32_t* plan,
             i64 rows_cap) {
    k_ep_plan<<<1, 32, 0, c->stream>>>(counts_all, rank, world, E, El, align, plan, rows_cap, c->status + EP_STATUS_SLOT);
    launched(c);
}

void ep_dispatch(Context* c, const void* x, const int32_t* idx, const int32_t* row_of1, const int32_t* off1,
                 const int32_t* plan, const PeerTab& xp, const PeerTab& src, int32_t* dest, i64 T, int k, i64 hidden,
                 int El, int align, int rank, int world, i64 rows_cap, int dtype) {
    const i64 slots = T * k + (i64)El * align;
    if (slots <= 0) return;
    const int v = row_vec(dtype, hidden);
    dim3 g((unsigned)cdiv(slots, 4));
#define DISP(TT, VV) \
    k_ep_dispatch<TT, VV><<<g, 128, 0, c->stream>>>((const TT*)x, idx, row_of1, off1, plan, xp, src, dest, T, k, hidden, El, align, rank, \
                                                    world, rows_cap, c->status + EP_STATUS_SLOT)
    if (dtype == CATNN_BF16) {
        if (v == 8) DISP(bf16, 8);
        else DISP(bf16, 1);
    } else {
        if (v == 4) DISP(float, 4);
        else DISP(float, 1);
    }
#undef DISP
    launched(c);
}

void ep_combine(Context* c, const PeerTab& yp, const int32_t* idx, const int32_t* dest, const float* w, i64 T, int k,
                i64 hidden, int El, int world, i64 rows_cap, float* y, const float* resid, int yp_dtype) {
    if (T <= 0) return;
    const int v = row_vec(yp_dtype, hidden);
    const int grid = (int)std::min<i64>(T, (i64)c->sm_count * 16);
    if (yp_dtype == CATNN_BF16) {
        if (v == 8) k_ep_combine<bf16, 8><<<grid, 128, 0, c->stream>>>(yp, idx, dest, w, T, k, hidden, El, world, rows_cap, y, resid);
        else k_ep_combine<bf16, 1><<<grid, 128, 0, c->stream>>>(yp, idx, dest, w, T, k, hidden, El, world, rows_cap, y, resid);
    } else {
        if (v == 4) k_ep_combine<float, 4><<<grid, 128, 0, c->stream>>>(yp, idx, dest, w, T, k, hidden, El, world, rows_cap, y, resid);
        else k_ep_combine<float, 1><<<grid, 128, 0, c->stream>>>(yp, idx, dest, w, T, k, hidden, El, world, rows_cap, y, resid);
    }
    launched(c);
}

void ep_unpermute_bwd(Context* c, const void* yp, const int32_t* src, const int32_t* plan, const PeerTab& w,
                      const PeerTab& dy, const PeerTab& dw, i64 rows_cap, i64 pairs, int k, i64 hidden, int El,
                      int world, void* dyp, int dtype) {
    if (rows_cap <= 0) return;
    dim3 g((unsigned)cdiv(rows_cap, 4));
    if (dtype == CATNN_BF16)
        k_ep_unpermute_bwd<bf16, bf16><<<g, 128, 0, c->stream>>>((const bf16*)yp, src, plan, w, dy, dw, pairs, k,
                                                                 hidden, El, world, (bf16*)dyp);
    else
        k_ep_unpermute_bwd<float, float><<<g, 128, 0, c->stream>>>((const float*)yp, src, plan, w, dy, dw, pairs, k,
                                                                   hidden, El, world, (float*)dyp);
    launched(c);
}

void ep_permute_bwd(Context* c, const PeerTab& dxp, const int32_t* idx, const int32_t* dest, i64 T, int k, i64 hidden,
                    int El, int world, i64 rows_cap, float* dx, int dtype) {
    if (T <= 0) return;
    const int v = row_vec(dtype, hidden);
    const int grid = (int)std::min<i64>(T, (i64)c->sm_count * 16);
    if (dtype == CATNN_BF16) {
        if (v == 8) k_ep_permute_bwd<bf16, 8><<<grid, 128, 0, c->stream>>>(dxp, idx, dest, T, k, hidden, El, world, rows_cap, dx);
        else k_ep_permute_bwd<bf16, 1><<<grid, 128, 0, c->stream>>>(dxp, idx, dest, T, k, hidden, El, world, rows_cap, dx);
    } else {
        if (v == 4) k_ep_permute_bwd<float, 4><<<grid, 128, 0, c->stream>>>(dxp, idx, dest, T, k, hidden, El, world, rows_cap, dx);
        else k_ep_permute_bwd<float, 1><<<grid, 128, 0, c->stream>>>(dxp, idx, dest, T, k, hidden, El, world, rows_cap, dx);
    }
    launched(c);
}

// ------------------------------------------------------------ vocab-sharded embedding
// One CTA per token: the row comes from its owner's table over NVLink, 16 bytes per thread.
__global__ void __launch_bounds__(256) k_ep_embed(const uint32_t* __restrict__ ids, PeerTab table, i64 vocab, i64 vs,
                                                  i64 hidden, float* __restrict__ y, int* err) {
    const i64 t = blockIdx.x;
    const uint32_t id = ids[t];
    const bool bad = (i64)id >= vocab;
    if (bad && threadIdx.x == 0 && err) atomicExch(err, 1);
    float* yr = y + t * hidden;
    const float* row = bad ? nullptr : (const float*)table.p[id / vs] + (i64)id * hidden;
    if ((hidden & 3) == 0) {
        for (i64 i = threadIdx.x; i < hidden / 4; i += blockDim.x)
            ((float4*)yr)[i] = bad ? make_float4(0.f, 0.f, 0.f, 0.f) : ((const float4*)row)[i];
    } else {
        for (i64 i = threadIdx.x; i < hidden; i += blockDim.x) yr[i] = bad ? 0.f : row[i];
    }
}

// Keys (id - v0) * n + t of the global tokens t whose id lies in [v0, v1),
// sorted ascending (by id, then token): one CTA compacts them in token
// order (block scan) and bitonic-sorts the compacted list in shared memory.
// Keys are unique, so the order is total. *m = number of keys.
__global__ void __launch_bounds__(1024) k_ep_embed_keys(const uint32_t* __restrict__ ids, i64 n, i64 v0, i64 v1,
                                                        uint32_t* __restrict__ keys, int* __restrict__ m) {
    extern __shared__ uint32_t sk[];
    __shared__ int wsum[32];
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, w = tid >> 5;
    const i64 per = (n + nt - 1) / nt;
    const i64 t0 = (i64)tid * per, t1 = t0 + per < n ? t0 + per : n;
    int cnt = 0;
    for (i64 t = t0; t < t1; ++t) cnt += (i64)ids[t] >= v0 && (i64)ids[t] < v1;
    int x = cnt;
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) wsum[w] = x;
    __syncthreads();
    if (w == 0) {
        int sum = lane < (nt >> 5) ? wsum[lane] : 0;
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, sum, o);
            if (lane >= o) sum += y;
        }
        wsum[lane] = sum;  // inclusive prefix over warps
    }
    __syncthreads();
    const int total = wsum[31];
    int pos = x - cnt + (w > 0 ? wsum[w - 1] : 0);
    for (i64 t = t0; t < t1; ++t) {
        const i64 id = ids[t];
        if (id >= v0 && id < v1) sk[pos++] = (uint32_t)((id - v0) * n + t);
    }
    int npow = 1;
    while (npow < total) npow <<= 1;
    __syncthreads();
    for (int i = total + tid; i < npow; i += nt) sk[i] = 0xFFFFFFFFu;
    __syncthreads();
    for (int k = 2; k <= npow; k <<= 1)
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = tid; i < npow; i += nt) {
                int p = i ^ j;
                if (p > i) {
                    uint32_t a = sk[i], b = sk[p];
                    if ((a > b) == ((i & k) == 0)) {
                        sk[i] = b;
                        sk[p] = a;
                    }
                }
            }
            __syncthreads();
        }
    for (int i = tid; i < total; i += nt) keys[i] = sk[i];
    if (tid == 0) *m = total;
}

// A CTA that starts a run of equal ids sums that run's dy rows in token
// order onto zero (the one-GPU k_embed_bwd_runs arithmetic); token t's row
// is row t % tpr of rank t / tpr's dy.
__global__ void __launch_bounds__(256) k_ep_embed_bwd_runs(const uint32_t* __restrict__ keys, const int* __restrict__ m,
                                                           i64 n, i64 tpr, PeerTab dy, float* __restrict__ dw_own,
                                                           i64 hidden) {
    const i64 cnt = *m;
    for (i64 i = blockIdx.x; i < cnt; i += gridDim.x) {
        const uint32_t id = keys[i] / (uint32_t)n;
        if (i > 0 && keys[i - 1] / (uint32_t)n == id) continue;
        i64 end = i + 1;
        while (end < cnt && keys[end] / (uint32_t)n == id) ++end;
        for (i64 col = threadIdx.x; col < hidden; col += blockDim.x) {
            float s = 0.f;
            for (i64 r = i; r < end; ++r) {
                const i64 t = keys[r] % (uint32_t)n;
                s = __fadd_rn(s, ((const float*)dy.p[t / tpr])[(t % tpr) * hidden + col]);
            }
            dw_own[(i64)id * hidden + col] = s;
        }
    }
}

void ep_embedding_fwd(Context* c, const uint32_t* ids, i64 n, const PeerTab& table, i64 vocab, i64 rows_per_rank,
                      i64 hidden, float* y, int* err) {
    if (n <= 0 || hidden <= 0) return;
    k_ep_embed<<<(unsigned)n, 256, 0, c->stream>>>(ids, table, vocab, rows_per_rank, hidden, y, err);
    launched(c);
}

void ep_embedding_keys(Context* c, const uint32_t* ids_global, i64 n_global, i64 v0, i64 v1, uint32_t* keys, int* m) {
    if (n_global <= 0) return;
    CATNN_CHECK(n_global <= 32768, CATNN_ERR_UNSUPPORTED, "embedding backward: at most 32768 tokens per step");
    CATNN_CHECK((unsigned long long)(v1 - v0 + 1) * (unsigned long long)n_global < 0xFFFFFFFFull, CATNN_ERR_UNSUPPORTED,
                "embedding backward: rows * tokens must fit in 32 bits");
    static bool attr[64] = {false};
    if (!attr[c->device]) {
        CUDA_OK(cudaFuncSetAttribute(k_ep_embed_keys, cudaFuncAttributeMaxDynamicSharedMemorySize, 32768 * 4));
        attr[c->device] = true;
    }
    i64 npow = 1;
    while (npow < n_global) npow <<= 1;
    k_ep_embed_keys<<<1, 1024, (size_t)npow * 4, c->stream>>>(ids_global, n_global, v0, v1, keys, m);
    launched(c);
}

void ep_embedding_runs(Context* c, const uint32_t* keys, const int* m, i64 n_global, i64 tokens_per_rank,
                       const PeerTab& dy, i64 v0, i64 v1, i64 hidden, float* dw) {
    if (v1 <= v0 || hidden <= 0) return;
    float* own = dw + v0 * hidden;
    CUDA_OK(cudaMemsetAsync(own, 0, (size_t)(v1 - v0) * hidden * 4, c->stream));
    if (n_global <= 0) return;
    const int grid = (int)std::min<i64>(n_global, (i64)c->sm_count * 8);
    k_ep_embed_bwd_runs<<<grid, 256, 0, c->stream>>>(keys, m, n_global, tokens_per_rank, dy, own, hidden);
    launched(c);
}

}  // namespace catnn
