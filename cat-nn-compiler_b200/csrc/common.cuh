// Shared device/host plumbing for libcatnn_b200: the per-device context,
// error reporting across the C ABI, launch accounting and small device
// helpers (bf16 conversion, warp reductions).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <initializer_list>
#include <string>

#include "../../include/catnn_b200.h"

namespace catnn {

typedef int64_t i64;

// A failed check inside the library. Thrown on the host only and turned
// into a status code + catnn_last_error() text at the ABI boundary.
struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

void set_last_error(const std::string& msg);

#define CATNN_CHECK(cond, code, msg)                                  \
    do {                                                              \
        if (!(cond)) throw ::catnn::Error((code), (msg));             \
    } while (0)
#define CUDA_OK(expr)                                                               \
    do {                                                                            \
        cudaError_t e__ = (expr);                                                   \
        if (e__ != cudaSuccess)                                                     \
            throw ::catnn::Error(CATNN_ERR_CUDA, std::string(#expr) + ": " +        \
                                                     cudaGetErrorString(e__));      \
    } while (0)

// Per-device state. One context per (device, caller thread of control);
// calls on one context are never concurrent (the reference moves each
// device's handler into one worker per wave, catnn-rt/src/dist.rs:441).
struct Context {
    int device = 0;
    cudaStream_t stream = nullptr;  // 0 = legacy default stream
    uint64_t launches = 0;          // kernels launched through this context
    int sm_count = 148;
    // Grow-only scratch arena for kernels that need global temporaries.
    void* scratch = nullptr;
    size_t scratch_bytes = 0;
    // Device status word for bounded waits / guarded kernels.
    int* status = nullptr;
    void* tc_sched = nullptr;  // GEMM tile-scheduler counters
    // Cached RoPE (cos, sin) table for (theta, seq, head_dim).
    void* rope_tab = nullptr;
    i64 rope_s = 0, rope_hd = 0;
    double rope_theta = 0.0;
    // Grow-only arena for composite ops (several temporaries held across
    // the leaf launchers, which use `scratch`).
    void* work = nullptr;
    size_t work_bytes = 0;
    void* scratch_for(size_t bytes);
    void* work_for(size_t bytes);
};

// Carves aligned sub-buffers out of one arena allocation.
struct Carver {
    char* base;
    size_t off = 0;
    explicit Carver(void* b) : base((char*)b) {}
    template <typename T> T* take(size_t n) {
        off = (off + 255) & ~(size_t)255;
        T* p = (T*)(base + off);
        off += n * sizeof(T);
        return p;
    }
    static size_t need(std::initializer_list<size_t> bytes) {
        size_t t = 0;
        for (size_t b : bytes) t += ((b + 255) & ~(size_t)255);
        return t + 256;
    }
};

// Every entry point: select the context's device first (consecutive waves can
// land on different host threads).
inline void bind(Context* c) { CUDA_OK(cudaSetDevice(c->device)); }

// After each launch: count it and surface launch-configuration errors.
inline void launched(Context* c, int n = 1) {
    c->launches += n;
    CUDA_OK(cudaGetLastError());
}

inline int cdiv(i64 a, i64 b) { return (int)((a + b - 1) / b); }

// ---- device helpers
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum over all threads of a 1-D block (blockDim.x multiple of 32,
// at most 1024). `red` is >= 32 floats of shared memory. All threads get it.
__device__ __forceinline__ float block_sum(float v, float* red) {
    int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    float t = lane < nw ? red[lane] : 0.f;
    t = warp_sum(t);
    return t;
}
__device__ __forceinline__ float block_max(float v, float* red) {
    int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    float t = lane < nw ? red[lane] : -INFINITY;
    t = warp_max(t);
    return t;
}

// Load/store one element of a tensor whose storage type is T (float or
// bf16), computing in f32.
template <typename T> __device__ __forceinline__ float ld(const T* p);
template <> __device__ __forceinline__ float ld<float>(const float* p) { return *p; }
template <> __device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <typename T> __device__ __forceinline__ void st(T* p, float v);
template <> __device__ __forceinline__ void st<float>(float* p, float v) { *p = v; }
template <> __device__ __forceinline__ void st<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

typedef __nv_bfloat16 bf16;

// V consecutive elements in one (or two) 16-byte accesses: the streaming
// kernels' loads and stores. The caller guarantees alignment of
// V * sizeof(T) bytes (checked on the host with vec_ok).
template <typename T, int V>
__device__ __forceinline__ void ldv(const T* p, float (&o)[V]) {
    if constexpr (V == 1) {
        o[0] = ld(p);
    } else if constexpr (sizeof(T) == 4) {
        static_assert(V % 4 == 0, "fp32 vectors are multiples of 4");
#pragma unroll
        for (int j = 0; j < V; j += 4) {
            float4 t = *(const float4*)((const float*)p + j);
            o[j] = t.x; o[j + 1] = t.y; o[j + 2] = t.z; o[j + 3] = t.w;
        }
    } else if constexpr (V == 8) {
        uint4 t = *(const uint4*)p;
        const __nv_bfloat162* h = (const __nv_bfloat162*)&t;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float2 f = __bfloat1622float2(h[j]);
            o[2 * j] = f.x; o[2 * j + 1] = f.y;
        }
    } else {
        static_assert(V == 4, "bf16 vectors are 4 or 8 wide");
        uint2 t = *(const uint2*)p;
        const __nv_bfloat162* h = (const __nv_bfloat162*)&t;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            float2 f = __bfloat1622float2(h[j]);
            o[2 * j] = f.x; o[2 * j + 1] = f.y;
        }
    }
}
template <typename T, int V>
__device__ __forceinline__ void stv(T* p, const float (&v)[V]) {
    if constexpr (V == 1) {
        st(p, v[0]);
    } else if constexpr (sizeof(T) == 4) {
#pragma unroll
        for (int j = 0; j < V; j += 4) *(float4*)((float*)p + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    } else if constexpr (V == 8) {
        uint4 t;
        __nv_bfloat162* h = (__nv_bfloat162*)&t;
#pragma unroll
        for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
        *(uint4*)p = t;
    } else {
        uint2 t;
        __nv_bfloat162* h = (__nv_bfloat162*)&t;
#pragma unroll
        for (int j = 0; j < 2; ++j) h[j] = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
        *(uint2*)p = t;
    }
}

// Host check: pointer aligned to `bytes` (nullptr passes).
inline bool aligned_to(const void* p, size_t bytes) { return ((uintptr_t)p % bytes) == 0; }

}  // namespace catnn
