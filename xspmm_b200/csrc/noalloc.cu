// noalloc.cu -- CSR row permutation that allocates no device memory.
//
// Some callers cannot allocate device memory while they run: a serving process whose device
// memory is fully reserved up front by its own pool, or code that must not take the device-wide
// synchronization cudaMalloc/cudaFree can cause. xspmm_permute_rows_noalloc_i32 gives them the
// row permutation (the same kernels and result as xspmm_permute_rows_*_i32) with its scratch in a
// fixed array compiled into this library instead of allocated per call.
//
// The scratch holds the duplicate-entry bitmap of the permutation check and the tile partials of
// the row_ptr scan, sized for at most NOALLOC_MAX_ROWS rows (270,336 bytes). Every GPU that loads
// the library holds one copy of it until the process exits. All calls on a device share it, and it
// keeps the last call's contents: the bitmap is cleared at the start of every call and the
// partials are fully rewritten before they are read. Calls that overlap on the GPU (different
// streams or handles at the same time) race on it and must be serialized by the caller.
#include "ops.cuh"

#include <cuda.h>

#include <mutex>

namespace {

constexpr int64_t NOALLOC_MAX_ROWS = int64_t(1) << 21;        // 2,097,152 rows
constexpr int64_t SEEN_WORDS = NOALLOC_MAX_ROWS / 32;         // duplicate-check bitmap
constexpr int64_t SCAN_ELEMS = 2048;                          // scan partials (int32)
constexpr size_t SCRATCH_BYTES = (size_t)(SEEN_WORDS + SCAN_ELEMS) * sizeof(int32_t);

static __device__ __align__(256) unsigned char g_permute_scratch[SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[MAX_DEVICES] = {};
CUcontext g_scratch_ctx[MAX_DEVICES] = {};

// The context current on the calling thread (driver entry point fetched through the runtime, so
// the library needs no link against libcuda).
CUcontext current_context() {
    using Fn = CUresult (*)(CUcontext*);
    static Fn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<Fn>(p);
    });
    CUcontext c = nullptr;
    if (fn == nullptr || fn(&c) != CUDA_SUCCESS) return nullptr;
    return c;
}

// Device address of the scratch array on the current device. In host code g_permute_scratch names
// a host-side stand-in, not device memory, so the address comes from cudaGetSymbolAddress with the
// device current. It is looked up at a device's first call and again whenever the device's
// context has changed since (after cudaDeviceReset the old address is no longer valid).
void* scratch_on(int device) {
    XS_REQUIRE(device >= 0 && device < MAX_DEVICES, XSPMM_STATUS_UNSUPPORTED,
               "device ordinal above 63");
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    const CUcontext ctx = current_context();
    if (!g_scratch_addr[device] || ctx == nullptr || ctx != g_scratch_ctx[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_permute_scratch);
        if (e != cudaSuccess || p == nullptr)
            throw xspmm_b200::Error(XSPMM_STATUS_CUDA_ERROR,
                                    std::string("cudaGetSymbolAddress(scratch): ") +
                                        cudaGetErrorString(e));
        g_scratch_addr[device] = p;
        g_scratch_ctx[device] = ctx;
    }
    return g_scratch_addr[device];
}

}  // namespace

using namespace xspmm_b200;

XS_API xspmm_status_t xspmm_permute_rows_noalloc_i32(xspmm_handle_t hh, int32_t M, int32_t K,
                                                     int32_t nnz, const int32_t* row_ptr,
                                                     const int32_t* col_ind, const void* values,
                                                     int32_t value_bytes, const int32_t* perm,
                                                     int32_t* out_row_ptr, int32_t* out_col_ind,
                                                     void* out_values) {
    return guarded([&] {
        Handle& h = H(hh);
        need(M >= 0 && K >= 0 && nnz >= 0, "negative dimension");
        XS_REQUIRE(M <= NOALLOC_MAX_ROWS, XSPMM_STATUS_INVALID_ARGUMENT,
                   "M above the no-allocation limit of 2,097,152 rows; use "
                   "xspmm_permute_rows_*_i32");
        need(value_bytes == 2 || value_bytes == 4, "value_bytes must be 2 (fp16) or 4 (fp32)");
        need(out_row_ptr != nullptr, "null out_row_ptr");
        need(M == 0 || (row_ptr && perm), "null row_ptr or perm");
        need(nnz == 0 || (col_ind && out_col_ind), "null col_ind");
        DeviceGuard g(h.device);
        auto* base = static_cast<unsigned char*>(scratch_on(h.device));
        auto* seen = reinterpret_cast<unsigned*>(base);
        auto* scan = reinterpret_cast<int32_t*>(base + SEEN_WORDS * sizeof(int32_t));
        if (value_bytes == 2)
            permute_rows_scratch<__half, int32_t>(h, M, nnz, row_ptr, col_ind,
                                                  static_cast<const __half*>(values), perm,
                                                  out_row_ptr, out_col_ind,
                                                  static_cast<__half*>(out_values), seen, scan,
                                                  SCAN_ELEMS);
        else
            permute_rows_scratch<float, int32_t>(h, M, nnz, row_ptr, col_ind,
                                                 static_cast<const float*>(values), perm,
                                                 out_row_ptr, out_col_ind,
                                                 static_cast<float*>(out_values), seen, scan,
                                                 SCAN_ELEMS);
    });
}
