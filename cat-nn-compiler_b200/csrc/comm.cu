// Single-node communicator: NCCL (resolved at run time with dlopen, so the
// library loads on hosts without it) for allreduce and the generic
// all-to-all, CUDA IPC peer mappings for the fused expert-parallel kernels,
// and a device barrier on epoch flags whose waits are bounded by a
// timeout: a rank that never arrives turns into CATNN_ERR_TIMEOUT on the
// host, not a hung GPU.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "comm.cuh"

struct catnn_comm {
    catnn::Comm m;
};

namespace catnn {

struct NcclFns {
    ncclResult_t (*getUniqueId)(ncclUniqueId*);
    ncclResult_t (*commInitRank)(ncclComm_t*, int, ncclUniqueId, int);
    ncclResult_t (*commDestroy)(ncclComm_t);
    ncclResult_t (*allReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*allGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*reduceScatter)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*groupStart)();
    ncclResult_t (*groupEnd)();
    const char* (*getErrorString)(ncclResult_t);
};

static const NcclFns* nccl_fns() {
    static std::mutex mu;
    static NcclFns fns;
    static bool done = false;
    static std::string why;
    std::lock_guard<std::mutex> g(mu);
    if (!done) {
        done = true;
        // the NCCL already in the process (e.g. the one torch loaded) wins
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            why = std::string("NCCL not found: ") + dlerror();
        } else {
            bool ok = true;
            auto sym = [&](const char* name) {
                void* p = dlsym(h, name);
                if (!p) ok = false;
                return p;
            };
            fns.getUniqueId = (decltype(fns.getUniqueId))sym("ncclGetUniqueId");
            fns.commInitRank = (decltype(fns.commInitRank))sym("ncclCommInitRank");
            fns.commDestroy = (decltype(fns.commDestroy))sym("ncclCommDestroy");
            fns.allReduce = (decltype(fns.allReduce))sym("ncclAllReduce");
            fns.allGather = (decltype(fns.allGather))sym("ncclAllGather");
            fns.reduceScatter = (decltype(fns.reduceScatter))sym("ncclReduceScatter");
            fns.send = (decltype(fns.send))sym("ncclSend");
            fns.recv = (decltype(fns.recv))sym("ncclRecv");
            fns.groupStart = (decltype(fns.groupStart))sym("ncclGroupStart");
            fns.groupEnd = (decltype(fns.groupEnd))sym("ncclGroupEnd");
            fns.getErrorString = (decltype(fns.getErrorString))sym("ncclGetErrorString");
            if (!ok) why = "NCCL library lacks a required symbol";
        }
    }
    CATNN_CHECK(why.empty(), CATNN_ERR_COMM, why);
    return &fns;
}

#define NCCL_OK(fn, expr)                                                                             \
    do {                                                                                              \
        ncclResult_t r__ = (expr);                                                                    \
        if (r__ != ncclSuccess)                                                                       \
            throw ::catnn::Error(CATNN_ERR_COMM, std::string(#expr) + ": " + (fn)->getErrorString(r__)); \
    } while (0)

static ncclComm_t nc(const Comm& m) { return (ncclComm_t)m.nccl; }

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Thread p < world: wait until flags[p] of this rank reaches `epoch`. The
// wait gives up after timeout_ns, records the epoch in the status slot and
// returns; once any wait has given up, later waits return at once.
__device__ void wait_flags(uint64_t* const* flag_ptrs, int rank, int world, uint64_t epoch, int64_t timeout_ns,
                           int* status) {
    int p = threadIdx.x;
    if (p >= world) return;
    if (*(volatile int*)(status + COMM_STATUS_SLOT)) return;
    const uint64_t* f = flag_ptrs[rank] + p;
    uint64_t t0 = global_ns();
    while (ld_acquire_sys(f) < epoch) {
        if ((int64_t)(global_ns() - t0) > timeout_ns) {
            atomicExch(status + COMM_STATUS_SLOT, 1);
            atomicExch(status + COMM_STATUS_SLOT + 1, (int)epoch);
            return;
        }
        __nanosleep(200);
    }
}

// All ranks: flags[rank] of every rank := epoch (release, system scope),
// then wait for this epoch from every rank. Writes of earlier kernels on
// the stream are complete when this kernel starts, so the release publishes them.
// The epoch is this rank's barrier count, kept on the device (*ctr, touched
// only by this rank's barriers, in stream order): every rank passes the same
// barriers in the same order, so the counts agree, and a barrier replayed in
// a CUDA graph takes the next epoch like an eager one.
__global__ void k_comm_barrier(uint64_t* const* flag_ptrs, int rank, int world, uint64_t* ctr, int64_t timeout_ns,
                               int* status) {
    __shared__ uint64_t e;
    if (threadIdx.x == 0) {
        e = *ctr + 1;
        *ctr = e;
    }
    __syncthreads();
    const uint64_t epoch = e;
    int p = threadIdx.x;
    if (p < world) {
        __threadfence_system();
        st_release_sys(flag_ptrs[p] + rank, epoch);
    }
    wait_flags(flag_ptrs, rank, world, epoch, timeout_ns, status);
}

// One wait on one peer's flag (the primitive under the barrier).
__global__ void k_comm_wait_one(uint64_t* const* flag_ptrs, int rank, int peer, uint64_t epoch, int64_t timeout_ns,
                                int* status) {
    if (threadIdx.x != 0) return;
    if (*(volatile int*)(status + COMM_STATUS_SLOT)) return;
    const uint64_t* f = flag_ptrs[rank] + peer;
    uint64_t t0 = global_ns();
    while (ld_acquire_sys(f) < epoch) {
        if ((int64_t)(global_ns() - t0) > timeout_ns) {
            atomicExch(status + COMM_STATUS_SLOT, 1);
            atomicExch(status + COMM_STATUS_SLOT + 1, (int)epoch);
            return;
        }
        __nanosleep(200);
    }
}

Comm::Mapped Comm::map(void* local, size_t bytes) {
    CATNN_CHECK(local != nullptr && bytes > 0, CATNN_ERR_INVALID, "comm map: empty block");
    Mapped m;
    m.bytes = bytes;
    m.base[rank] = local;
    if (world == 1) {
        maps.push_back(m);
        return m;
    }
    cudaIpcMemHandle_t mine;
    CUDA_OK(cudaIpcGetMemHandle(&mine, local));
    // all-gather the handles (and sizes) through NCCL
    struct Rec {
        cudaIpcMemHandle_t h;
        uint64_t bytes;
    };
    static_assert(sizeof(Rec) % 8 == 0, "record size");
    Rec rec{mine, (uint64_t)bytes};
    Rec* dev = nullptr;
    CUDA_OK(cudaMalloc(&dev, sizeof(Rec) * (world + 1)));
    std::vector<Rec> all(world);
    try {
        CUDA_OK(cudaMemcpyAsync(dev + world, &rec, sizeof(Rec), cudaMemcpyHostToDevice, c->stream));
        NCCL_OK(fn, fn->allGather(dev + world, dev, sizeof(Rec), ncclChar, nc(*this), c->stream));
        CUDA_OK(cudaMemcpyAsync(all.data(), dev, sizeof(Rec) * world, cudaMemcpyDeviceToHost, c->stream));
        CUDA_OK(cudaStreamSynchronize(c->stream));
    } catch (...) {
        cudaFree(dev);
        throw;
    }
    CUDA_OK(cudaFree(dev));
    for (int p = 0; p < world; ++p) {
        CATNN_CHECK(all[p].bytes == bytes, CATNN_ERR_COMM,
                    "comm map: rank " + std::to_string(p) + " maps a block of another size (configs differ?)");
        if (p == rank) continue;
        void* q = nullptr;
        CUDA_OK(cudaIpcOpenMemHandle(&q, all[p].h, cudaIpcMemLazyEnablePeerAccess));
        m.base[p] = q;
    }
    maps.push_back(m);
    return m;
}

void Comm::barrier() {
    ++epoch;  // host mirror of the device count (diagnostics)
    k_comm_barrier<<<1, 32, 0, c->stream>>>(flag_ptrs_dev, rank, world, flag_block + EPOCH_SLOT, timeout_ns,
                                             c->status);
    launched(c);
}

static ncclDataType_t nccl_type(int dtype) { return dtype == CATNN_BF16 ? ncclBfloat16 : ncclFloat32; }

void Comm::allreduce_sum(void* buf, i64 n, int dtype) {
    if (world == 1 || n <= 0) return;
    NCCL_OK(fn, fn->allReduce(buf, buf, (size_t)n, nccl_type(dtype), ncclSum, nc(*this), c->stream));
}

void Comm::allreduce_overlapped(float* buf, i64 n) {
    if (world == 1 || n <= 0) return;
    make_side();
    CUDA_OK(cudaEventRecord(ev_ready, c->stream));
    CUDA_OK(cudaStreamWaitEvent(side, ev_ready, 0));
    NCCL_OK(fn, fn->allReduce(buf, buf, (size_t)n, ncclFloat32, ncclSum, nc(*this), side));
}

void Comm::make_side() {
    if (side) return;
    int lo = 0, hi = 0;
    CUDA_OK(cudaDeviceGetStreamPriorityRange(&lo, &hi));
    CUDA_OK(cudaStreamCreateWithPriority(&side, cudaStreamNonBlocking, hi));
    CUDA_OK(cudaEventCreateWithFlags(&ev_ready, cudaEventDisableTiming));
    CUDA_OK(cudaEventCreateWithFlags(&ev_done, cudaEventDisableTiming));
}

void Comm::reduce_scatter_overlapped(float* buf, i64 n) {
    if (world == 1 || n <= 0) return;
    CATNN_CHECK(n % world == 0, CATNN_ERR_SHAPE, "reduce-scatter: length not divisible by the ranks");
    make_side();
    CUDA_OK(cudaEventRecord(ev_ready, c->stream));
    CUDA_OK(cudaStreamWaitEvent(side, ev_ready, 0));
    const i64 chunk = n / world;
    NCCL_OK(fn, fn->reduceScatter(buf, buf + rank * chunk, (size_t)chunk, ncclFloat32, ncclSum, nc(*this), side));
}

void Comm::allgather_after(void* buf, i64 n, int dtype, cudaEvent_t after) {
    if (world == 1 || n <= 0) return;
    CATNN_CHECK(n % world == 0, CATNN_ERR_SHAPE, "all-gather: length not divisible by the ranks");
    make_side();
    CUDA_OK(cudaStreamWaitEvent(side, after, 0));
    const i64 chunk = n / world;
    const size_t es = dtype == CATNN_BF16 ? 2 : 4;
    NCCL_OK(fn, fn->allGather((char*)buf + rank * chunk * es, buf, (size_t)chunk, nccl_type(dtype), nc(*this), side));
}

void Comm::allgather(void* buf, i64 n, int dtype) {
    if (world == 1 || n <= 0) return;
    CATNN_CHECK(n % world == 0, CATNN_ERR_SHAPE, "all-gather: length not divisible by the ranks");
    const i64 chunk = n / world;
    const size_t es = dtype == CATNN_BF16 ? 2 : 4;
    NCCL_OK(fn, fn->allGather((char*)buf + rank * chunk * es, buf, (size_t)chunk, nccl_type(dtype), nc(*this),
                              c->stream));
}

void Comm::join_overlapped() {
    if (!side) return;
    CUDA_OK(cudaEventRecord(ev_done, side));
    CUDA_OK(cudaStreamWaitEvent(c->stream, ev_done, 0));
}

void Comm::release() {
    if (c) cudaStreamSynchronize(c->stream);
    if (side) {
        cudaStreamSynchronize(side);
        cudaEventDestroy(ev_ready);
        cudaEventDestroy(ev_done);
        cudaStreamDestroy(side);
        side = nullptr;
    }
    for (auto& m : maps)
        for (int p = 0; p < world; ++p)
            if (p != rank && m.base[p]) cudaIpcCloseMemHandle(m.base[p]);
    maps.clear();
    if (flag_block) cudaFree(flag_block);
    if (flag_ptrs_dev) cudaFree(flag_ptrs_dev);
    flag_block = nullptr;
    flag_ptrs_dev = nullptr;
    if (nccl && fn) fn->commDestroy(nc(*this));
    nccl = nullptr;
}

static Comm& cm(catnn_comm* h) {
    CATNN_CHECK(h != nullptr, CATNN_ERR_INVALID, "null catnn_comm");
    bind(h->m.c);
    return h->m;
}

Comm* comm_of(catnn_comm* h) { return &cm(h); }

}  // namespace catnn

using namespace catnn;

extern "C" {

int catnn_comm_unique_id(void* id) {
    ABI_BEGIN
    CATNN_CHECK(id != nullptr, CATNN_ERR_INVALID, "null id buffer");
    static_assert(sizeof(ncclUniqueId) == CATNN_COMM_ID_BYTES, "NCCL unique id size");
    const NcclFns* fn = nccl_fns();
    ncclUniqueId u;
    NCCL_OK(fn, fn->getUniqueId(&u));
    std::memcpy(id, &u, sizeof(u));
    ABI_END
}

int catnn_comm_create(catnn_ctx* h, int rank, int world, const void* id, catnn_comm** out) {
    ABI_BEGIN
    Context* c = unwrap(h);
    CATNN_CHECK(out != nullptr, CATNN_ERR_INVALID, "null out");
    CATNN_CHECK(world >= 1 && world <= COMM_MAX_WORLD && rank >= 0 && rank < world, CATNN_ERR_INVALID,
                "comm: need 0 <= rank < world <= " + std::to_string(COMM_MAX_WORLD));
    catnn_comm* cc = new catnn_comm();
    Comm& m = cc->m;
    m.c = c;
    m.rank = rank;
    m.world = world;
    try {
        if (world > 1) {
            CATNN_CHECK(id != nullptr, CATNN_ERR_INVALID, "comm: null unique id");
            m.fn = nccl_fns();
            ncclUniqueId u;
            std::memcpy(&u, id, sizeof(u));
            ncclComm_t n = nullptr;
            NCCL_OK(m.fn, m.fn->commInitRank(&n, world, u, rank));
            m.nccl = n;
        }
        // flag block: its own allocation so it maps on its own
        CUDA_OK(cudaMalloc(&m.flag_block, 256));
        CUDA_OK(cudaMemsetAsync(m.flag_block, 0, 256, c->stream));
        CUDA_OK(cudaStreamSynchronize(c->stream));
        Comm::Mapped fm = m.map(m.flag_block, 256);
        CUDA_OK(cudaMalloc(&m.flag_ptrs_dev, sizeof(uint64_t*) * COMM_MAX_WORLD));
        uint64_t* ptrs[COMM_MAX_WORLD] = {};
        for (int p = 0; p < world; ++p) ptrs[p] = (uint64_t*)fm.base[p];
        CUDA_OK(cudaMemcpyAsync(m.flag_ptrs_dev, ptrs, sizeof(ptrs), cudaMemcpyHostToDevice, c->stream));
        // every rank has zeroed its flags before anyone signals
        m.barrier();
        CUDA_OK(cudaStreamSynchronize(c->stream));
        int st = 0;
        CUDA_OK(cudaMemcpy(&st, c->status + COMM_STATUS_SLOT, 4, cudaMemcpyDeviceToHost));
        CATNN_CHECK(st == 0, CATNN_ERR_TIMEOUT, "comm: ranks did not meet at creation");
    } catch (...) {
        m.release();
        delete cc;
        throw;
    }
    *out = cc;
    ABI_END
}

int catnn_comm_destroy(catnn_comm* h) {
    ABI_BEGIN
    if (!h) return CATNN_OK;
    bind(h->m.c);
    h->m.release();
    delete h;
    ABI_END
}

int catnn_comm_rank(catnn_comm* h, int* rank, int* world) {
    ABI_BEGIN
    Comm& m = cm(h);
    if (rank) *rank = m.rank;
    if (world) *world = m.world;
    ABI_END
}

int catnn_comm_set_timeout_ms(catnn_comm* h, int64_t ms) {
    ABI_BEGIN
    Comm& m = cm(h);
    CATNN_CHECK(ms > 0, CATNN_ERR_INVALID, "timeout must be positive");
    m.timeout_ns = ms * 1000000ll;
    ABI_END
}

int catnn_comm_allreduce(catnn_comm* h, void* buf, int64_t n, int dtype) {
    ABI_BEGIN
    Comm& m = cm(h);
    check_dtype(dtype);
    CATNN_CHECK(n >= 0 && (buf || n == 0), CATNN_ERR_INVALID, "allreduce: bad buffer");
    m.allreduce_sum(buf, n, dtype);
    ABI_END
}

int catnn_comm_all_to_all(catnn_comm* h, const void* send, const int64_t* send_bytes, void* recv,
                          const int64_t* recv_bytes) {
    ABI_BEGIN
    Comm& m = cm(h);
    CATNN_CHECK(send_bytes && recv_bytes, CATNN_ERR_INVALID, "all_to_all: null counts");
    int64_t so = 0, ro = 0;
    for (int p = 0; p < m.world; ++p) {
        CATNN_CHECK(send_bytes[p] >= 0 && recv_bytes[p] >= 0, CATNN_ERR_INVALID, "all_to_all: negative count");
        so += send_bytes[p];
        ro += recv_bytes[p];
    }
    CATNN_CHECK((send || so == 0) && (recv || ro == 0), CATNN_ERR_INVALID, "all_to_all: null buffer");
    if (m.world == 1) {
        if (so) CUDA_OK(cudaMemcpyAsync(recv, send, so, cudaMemcpyDeviceToDevice, m.c->stream));
        return CATNN_OK;
    }
    const NcclFns* fn = m.fn;
    NCCL_OK(fn, fn->groupStart());
    so = ro = 0;
    for (int p = 0; p < m.world; ++p) {
        if (send_bytes[p])
            NCCL_OK(fn, fn->send((const char*)send + so, send_bytes[p], ncclChar, p, nc(m), m.c->stream));
        if (recv_bytes[p]) NCCL_OK(fn, fn->recv((char*)recv + ro, recv_bytes[p], ncclChar, p, nc(m), m.c->stream));
        so += send_bytes[p];
        ro += recv_bytes[p];
    }
    NCCL_OK(fn, fn->groupEnd());
    ABI_END
}

int catnn_comm_barrier(catnn_comm* h) {
    ABI_BEGIN
    Comm& m = cm(h);
    m.barrier();
    ABI_END
}

int catnn_comm_signal(catnn_comm* h, int peer, uint64_t epoch) {
    ABI_BEGIN
    Comm& m = cm(h);
    CATNN_CHECK(peer >= 0 && peer < m.world, CATNN_ERR_INVALID, "signal: peer out of range");
    uint64_t* dst = m.maps[0].base[peer] ? (uint64_t*)m.maps[0].base[peer] + m.rank : nullptr;
    CATNN_CHECK(dst != nullptr, CATNN_ERR_COMM, "signal: flag block not mapped");
    CUDA_OK(cudaMemcpyAsync(dst, &epoch, 8, cudaMemcpyHostToDevice, m.c->stream));
    CUDA_OK(cudaStreamSynchronize(m.c->stream));
    ABI_END
}

int catnn_comm_wait(catnn_comm* h, int peer, uint64_t epoch) {
    ABI_BEGIN
    Comm& m = cm(h);
    CATNN_CHECK(peer >= 0 && peer < m.world, CATNN_ERR_INVALID, "wait: peer out of range");
    k_comm_wait_one<<<1, 32, 0, m.c->stream>>>(m.flag_ptrs_dev, m.rank, peer, epoch, m.timeout_ns, m.c->status);
    launched(m.c);
    ABI_END
}

int catnn_comm_check(catnn_comm* h) {
    ABI_BEGIN
    Comm& m = cm(h);
    int v[2] = {0, 0};
    CUDA_OK(cudaMemcpyAsync(v, m.c->status + COMM_STATUS_SLOT, 8, cudaMemcpyDeviceToHost, m.c->stream));
    CUDA_OK(cudaStreamSynchronize(m.c->stream));
    if (v[0]) {
        CUDA_OK(cudaMemsetAsync(m.c->status + COMM_STATUS_SLOT, 0, 8, m.c->stream));
        CUDA_OK(cudaStreamSynchronize(m.c->stream));
        throw Error(CATNN_ERR_TIMEOUT, "a device wait for epoch " + std::to_string(v[1]) +
                                           " gave up: a rank did not arrive within the timeout");
    }
    ABI_END
}

}  // extern "C"
