// Communicator of one rank in a single-node group: NCCL for the bulk
// collectives (gradient allreduce, generic all-to-all) and peer-mapped
// device memory (CUDA IPC over NVLink) for the fused MoE dispatch/combine
// kernels, which read and write the other ranks' buffers directly and
// synchronise through epoch flags with bounded waits.
//
// The reference models expert parallelism as E/EP experts per rank with an
// activation all-to-all whose remote fraction is (EP-1)/EP
// (crates/catnn-compile/src/spark_place.rs:119-131,196) and runs device
// handlers one worker per device (crates/catnn-rt/src/dist.rs:441-517).
#pragma once
#include <vector>

#include "ops.cuh"

namespace catnn {

// Status slot set by a device wait that ran out of time (and the epoch it waited for).
constexpr int COMM_STATUS_SLOT = 12;
constexpr int COMM_MAX_WORLD = 8;
// word of the (256-byte, zeroed) flag block holding this rank's barrier count
constexpr int EPOCH_SLOT = 31;

struct NcclFns;

struct Comm {
    Context* c = nullptr;
    int rank = 0, world = 1;
    void* nccl = nullptr;  // ncclComm_t
    const NcclFns* fn = nullptr;
    // Peer-mapped allocations: base[p] is rank p's copy as seen from this
    // process (base[rank] is the local pointer).
    struct Mapped {
        void* base[COMM_MAX_WORLD] = {};
        size_t bytes = 0;
    };
    std::vector<Mapped> maps;
    // flags[src] in each rank's flag block: the last epoch rank src signalled.
    uint64_t* flag_block = nullptr;           // local, world x uint64
    uint64_t** flag_ptrs_dev = nullptr;       // device [world] -> each rank's flag block
    uint64_t epoch = 0;
    int64_t timeout_ns = 10ll * 1000 * 1000 * 1000;

    // Exchange an IPC handle of `local` (the base of a cudaMalloc block of
    // `bytes`, same size on every rank) and map the peers' blocks. Collective.
    Mapped map(void* local, size_t bytes);
    // Pointer q inside mapped block m, translated to rank p's copy.
    template <typename T>
    T* at(const Mapped& m, int p, T* q) const {
        return (T*)((char*)m.base[p] + ((char*)q - (char*)m.base[rank]));
    }
    // Device barrier: every rank signals every rank, then waits (bounded)
    // for all signals of this epoch. Enqueued on the context stream.
    void barrier();
    void allreduce_sum(void* buf, i64 n, int dtype);
    // fp32 sum of n elements on the communication stream, after the work
    // enqueued so far on the context stream; join_overlapped makes the
    // context stream wait for every such allreduce.
    void allreduce_overlapped(float* buf, i64 n);
    // Sharded counterparts on the communication stream (n divisible by the
    // ranks, chunk = n / world): reduce_scatter_overlapped leaves the fp32 sum
    // of chunk `rank` of buf in place (after the work enqueued so far on the
    // context stream); allgather_after fills every chunk of buf from its
    // owner's copy once `after` has completed (dtype CATNN_F32 or CATNN_BF16).
    void reduce_scatter_overlapped(float* buf, i64 n);
    void allgather_after(void* buf, i64 n, int dtype, cudaEvent_t after);
    // In-place all-gather on the context stream.
    void allgather(void* buf, i64 n, int dtype);
    void join_overlapped();
    void make_side();
    cudaStream_t side = nullptr;
    cudaEvent_t ev_ready = nullptr, ev_done = nullptr;
    void release();
};

// The communicator behind a catnn_comm handle (binds its context).
Comm* comm_of(catnn_comm* h);

}  // namespace catnn
