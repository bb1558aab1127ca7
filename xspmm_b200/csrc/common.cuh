// common.cuh -- shared pieces of the xspmm_b200 CUDA library: status handling, the handle,
// launch accounting, device-wide exclusive scan and small device helpers.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <cstdio>
#include <algorithm>
#include <string>
#include <stdexcept>

#include "../../include/xspmm_b200.h"

namespace xspmm_b200 {

// ------------------------------------------------------------------------------------------------
// Errors. Host code throws Error; every C entry point catches it and returns its status, keeping
// the message for xspmm_last_error().
// ------------------------------------------------------------------------------------------------
struct Error : std::runtime_error {
    xspmm_status_t status;
    Error(xspmm_status_t s, const std::string& m) : std::runtime_error(m), status(s) {}
};

void set_last_error(const std::string& msg);

#define XS_CHECK_CUDA(call)                                                                       \
    do {                                                                                          \
        cudaError_t e_ = (call);                                                                  \
        if (e_ != cudaSuccess) {                                                                  \
            throw ::xspmm_b200::Error(e_ == cudaErrorMemoryAllocation                             \
                                          ? XSPMM_STATUS_OUT_OF_MEMORY                            \
                                          : XSPMM_STATUS_CUDA_ERROR,                              \
                                      std::string(#call) + ": " + cudaGetErrorString(e_) +       \
                                          " at " + __FILE__ + ":" + std::to_string(__LINE__));    \
        }                                                                                         \
    } while (0)

#define XS_REQUIRE(cond, status, msg)                                                             \
    do {                                                                                          \
        if (!(cond)) throw ::xspmm_b200::Error((status), (msg));                                  \
    } while (0)

// Device-side error flags (bit set by kernels, read back by the host at sync points).
enum DeviceError : unsigned {
    DERR_COL_OUT_OF_RANGE = 1u << 0,
    DERR_ROW_PTR = 1u << 1,
    DERR_PERM_OUT_OF_RANGE = 1u << 2,
    DERR_INTERNAL = 1u << 3,
    DERR_CAPACITY = 1u << 4,
    DERR_TIMEOUT = 1u << 5,
};

// ------------------------------------------------------------------------------------------------
// The handle: device, stream, a device error word and the launch counter.
// ------------------------------------------------------------------------------------------------
struct Handle {
    int device = 0;
    cudaStream_t stream = nullptr;
    unsigned* d_err = nullptr;       // device error word
    unsigned* h_err = nullptr;       // pinned mirror
    unsigned long long launches = 0;  // kernels this library launched on the handle
    cudaEvent_t ev[8] = {};           // stage timing events
    int tier1_kernel = 0;             // 0 auto, 1 mma.sync, 2 tcgen05 (xspmm_set_tier1_kernel)
};

// RAII: make the handle's device current for the duration of a call.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        XS_CHECK_CUDA(cudaGetDevice(&prev));
        if (prev != dev) XS_CHECK_CUDA(cudaSetDevice(dev));
    }
    ~DeviceGuard() {
        int cur = -1;
        if (cudaGetDevice(&cur) == cudaSuccess && prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

// Checks the launch that was just enqueued and counts it.
inline void after_launch(Handle& h, const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        throw Error(XSPMM_STATUS_CUDA_ERROR, std::string("launch of ") + what + ": " +
                                                 cudaGetErrorString(e));
    ++h.launches;
}

// Reads and clears the device error word (synchronizes the stream).
unsigned read_device_errors(Handle& h);
void throw_on_device_errors(Handle& h, const char* stage);

// Stream-ordered scratch allocation (the device's default memory pool; the handle raises its
// release threshold so freed blocks are reused instead of returned to the driver).
template <typename T>
struct DevBuf {
    T* p = nullptr;
    size_t n = 0;
    cudaStream_t s = nullptr;
    DevBuf() = default;
    DevBuf(size_t count, cudaStream_t stream) : n(count), s(stream) {
        if (count) XS_CHECK_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&p), count * sizeof(T), s));
    }
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    DevBuf(DevBuf&& o) noexcept : p(o.p), n(o.n), s(o.s) { o.p = nullptr; o.n = 0; }
    DevBuf& operator=(DevBuf&& o) noexcept {
        if (this != &o) {
            release();
            p = o.p; n = o.n; s = o.s;
            o.p = nullptr; o.n = 0;
        }
        return *this;
    }
    ~DevBuf() { release(); }
    void release() {
        if (p) cudaFreeAsync(p, s);
        p = nullptr;
        n = 0;
    }
    T* get() const { return p; }
};

// ------------------------------------------------------------------------------------------------
// Device-wide exclusive scan of n values of type T (int32 or int64): out[i] = sum(in[0..i)),
// out[n] = total. in and out may alias. Three-phase reduce / scan-of-partials / downsweep with
// recursion on the partials; every launch counted on the handle.
// ------------------------------------------------------------------------------------------------
template <typename T>
void exclusive_scan(Handle& h, const T* in, T* out, int64_t n);

// Same scan with caller-provided scratch for the tile partials (no allocation). Needs
// scan_scratch_elems(n) elements; throws INVALID_ARGUMENT if scratch_elems is smaller.
int64_t scan_scratch_elems(int64_t n);
template <typename T>
void exclusive_scan_scratch(Handle& h, const T* in, T* out, int64_t n, T* scratch,
                            int64_t scratch_elems);

// Copies the last element of an exclusive scan (the total) to the host.
template <typename T>
T read_scalar(Handle& h, const T* dptr);

// ------------------------------------------------------------------------------------------------
// Small device helpers
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ void flag_error(unsigned* err, unsigned bit) { atomicOr(err, bit); }

// A stored value as float (exact for every value type of the library).
__device__ __forceinline__ float to_float(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_float(float x) { return x; }

// 16-bit value types share every data-movement kernel (the bits are copied, never converted);
// only the arithmetic differs. half_like<VT> selects the 16-bit paths, as_half() views the bits.
template <typename VT> struct half_like { static constexpr bool value = false; };
template <> struct half_like<__half> { static constexpr bool value = true; };
template <> struct half_like<__nv_bfloat16> { static constexpr bool value = true; };
template <typename VT> inline const __half* as_half(const VT* p) {
    static_assert(sizeof(VT) == 2, "16-bit value type");
    return reinterpret_cast<const __half*>(p);
}
template <typename VT> inline __half* as_half(VT* p) {
    static_assert(sizeof(VT) == 2, "16-bit value type");
    return reinterpret_cast<__half*>(p);
}

__device__ __forceinline__ unsigned lane_id() { return threadIdx.x & 31u; }

template <typename T>
__device__ __forceinline__ T warp_inclusive_sum(T v) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        T t = __shfl_up_sync(0xffffffffu, v, o);
        if ((int)lane_id() >= o) v += t;
    }
    return v;
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

int sm_count(int device);

}  // namespace xspmm_b200
