// Context lifecycle, error text, memory helpers and the checksum — the
// device-side state a catnn DeviceHandler (crates/catnn-rt/src/handler.rs)
// needs once its kernels run on a GPU.
#include <mutex>

#include "ops.cuh"

namespace catnn {

static thread_local std::string g_last_error;
void set_last_error(const std::string& msg) { g_last_error = msg; }

int take_status(Context* c, int slot) {
    int v = 0;
    CUDA_OK(cudaMemcpyAsync(&v, c->status + slot, 4, cudaMemcpyDeviceToHost, c->stream));
    CUDA_OK(cudaStreamSynchronize(c->stream));
    if (v) CUDA_OK(cudaMemsetAsync(c->status + slot, 0, 4, c->stream));
    return v;
}

// Live contexts per device (the allocation-free entry point's cached
// address is dropped with the device's last context).
static int g_live_ctx[64] = {0};
static std::mutex g_live_ctx_mu;

void* Context::scratch_for(size_t bytes) {
    if (bytes <= scratch_bytes) return scratch;
    // Grow-only: the stream must not still be reading the old buffer.
    if (scratch) {
        CUDA_OK(cudaStreamSynchronize(stream));
        CUDA_OK(cudaFree(scratch));
        scratch = nullptr;
        scratch_bytes = 0;
    }
    size_t b = bytes < (1u << 20) ? (1u << 20) : bytes;
    b = (b + 255) & ~(size_t)255;
    CUDA_OK(cudaMalloc(&scratch, b));
    scratch_bytes = b;
    return scratch;
}

void* Context::work_for(size_t bytes) {
    if (bytes <= work_bytes) return work;
    if (work) {
        CUDA_OK(cudaStreamSynchronize(stream));
        CUDA_OK(cudaFree(work));
        work = nullptr;
        work_bytes = 0;
    }
    size_t b = (bytes + 255) & ~(size_t)255;
    CUDA_OK(cudaMalloc(&work, b));
    work_bytes = b;
    return work;
}

// FNV-1a over f32 bit patterns is inherently sequential; a single thread
// walks the tensor (it is a debugging/sheaf checksum, not a hot kernel).
__global__ void k_checksum(const float* x, i64 n, unsigned long long* out) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    unsigned long long h = 0xcbf29ce484222325ull;
    const unsigned int* b = reinterpret_cast<const unsigned int*>(x);
    for (i64 i = 0; i < n; ++i) {
        h ^= (unsigned long long)b[i];
        h *= 0x100000001b3ull;
    }
    *out = h;
}

}  // namespace catnn

using namespace catnn;

namespace catnn {
Context* unwrap(catnn_ctx* h) {
    CATNN_CHECK(h != nullptr, CATNN_ERR_INVALID, "null catnn_ctx");
    bind(&h->c);
    return &h->c;
}
}  // namespace catnn

extern "C" {

int catnn_version(void) { return 1; }

const char* catnn_last_error(void) { return g_last_error.c_str(); }

int catnn_ctx_create(int device, catnn_ctx** out) {
    ABI_BEGIN
    CATNN_CHECK(out != nullptr, CATNN_ERR_INVALID, "catnn_ctx_create: out is null");
    int n = 0;
    CUDA_OK(cudaGetDeviceCount(&n));
    CATNN_CHECK(device >= 0 && device < n, CATNN_ERR_INVALID,
                "catnn_ctx_create: device " + std::to_string(device) + " of " + std::to_string(n));
    CUDA_OK(cudaSetDevice(device));
    cudaDeviceProp prop;
    CUDA_OK(cudaGetDeviceProperties(&prop, device));
    CATNN_CHECK(prop.major == 10 && prop.minor == 0, CATNN_ERR_UNSUPPORTED,
                std::string("libcatnn_b200 is built for sm_100a (B200); device is ") + prop.name);
    CATNN_CHECK(device < 64, CATNN_ERR_INVALID, "catnn_ctx_create: device index above 63");
    // resolve the allocation-free entry point's array here, where loading the
    // library's code on the device may allocate
    xent_row_loss_buffer(device);
    catnn_ctx* h = new catnn_ctx();
    h->c.device = device;
    h->c.sm_count = prop.multiProcessorCount;
    CUDA_OK(cudaMalloc(&h->c.status, 64 * sizeof(int)));
    CUDA_OK(cudaMemset(h->c.status, 0, 64 * sizeof(int)));
    {
        std::lock_guard<std::mutex> lock(g_live_ctx_mu);
        ++g_live_ctx[device];
    }
    *out = h;
    ABI_END
}

int catnn_ctx_destroy(catnn_ctx* h) {
    ABI_BEGIN
    if (!h) return CATNN_OK;
    bind(&h->c);
    cudaStreamSynchronize(h->c.stream);
    if (h->c.scratch) cudaFree(h->c.scratch);
    if (h->c.status) cudaFree(h->c.status);
    if (h->c.tc_sched) cudaFree(h->c.tc_sched);
    if (h->c.rope_tab) cudaFree(h->c.rope_tab);
    if (h->c.work) cudaFree(h->c.work);
    {
        std::lock_guard<std::mutex> lock(g_live_ctx_mu);
        if (--g_live_ctx[h->c.device] == 0) xent_noalloc_forget(h->c.device);
    }
    delete h;
    ABI_END
}

int catnn_ctx_set_stream(catnn_ctx* h, void* stream) {
    ABI_BEGIN
    Context* c = unwrap(h);
    c->stream = (cudaStream_t)stream;
    ABI_END
}

int catnn_ctx_synchronize(catnn_ctx* h) {
    ABI_BEGIN
    Context* c = unwrap(h);
    CUDA_OK(cudaStreamSynchronize(c->stream));
    ABI_END
}

int catnn_ctx_launch_count(catnn_ctx* h, uint64_t* out) {
    ABI_BEGIN
    Context* c = unwrap(h);
    CATNN_CHECK(out, CATNN_ERR_INVALID, "null out");
    *out = c->launches;
    ABI_END
}

int catnn_malloc(catnn_ctx* h, size_t bytes, void** out) {
    ABI_BEGIN
    unwrap(h);
    CATNN_CHECK(out, CATNN_ERR_INVALID, "null out");
    *out = nullptr;
    if (bytes) CUDA_OK(cudaMalloc(out, bytes));
    ABI_END
}

int catnn_free(catnn_ctx* h, void* p) {
    ABI_BEGIN
    unwrap(h);
    if (p) CUDA_OK(cudaFree(p));
    ABI_END
}

int catnn_upload(catnn_ctx* h, void* dst, const void* src, size_t bytes) {
    ABI_BEGIN
    Context* c = unwrap(h);
    if (!bytes) return CATNN_OK;
    CATNN_CHECK(dst && src, CATNN_ERR_INVALID, "catnn_upload: null pointer");
    CUDA_OK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, c->stream));
    CUDA_OK(cudaStreamSynchronize(c->stream));
    ABI_END
}

int catnn_download(catnn_ctx* h, void* dst, const void* src, size_t bytes) {
    ABI_BEGIN
    Context* c = unwrap(h);
    if (!bytes) return CATNN_OK;
    CATNN_CHECK(dst && src, CATNN_ERR_INVALID, "catnn_download: null pointer");
    CUDA_OK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, c->stream));
    CUDA_OK(cudaStreamSynchronize(c->stream));
    ABI_END
}

int catnn_checksum_f32(catnn_ctx* h, const float* x, int64_t n, uint64_t* out) {
    ABI_BEGIN
    Context* c = unwrap(h);
    CATNN_CHECK(out && (x || n == 0) && n >= 0, CATNN_ERR_INVALID, "catnn_checksum_f32: bad args");
    unsigned long long* d = (unsigned long long*)c->scratch_for(8);
    k_checksum<<<1, 32, 0, c->stream>>>(x, n, d);
    launched(c);
    unsigned long long hv = 0;
    CUDA_OK(cudaMemcpyAsync(&hv, d, 8, cudaMemcpyDeviceToHost, c->stream));
    CUDA_OK(cudaStreamSynchronize(c->stream));
    *out = hv;
    ABI_END
}

}  // extern "C"
