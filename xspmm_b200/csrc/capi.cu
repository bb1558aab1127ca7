// capi.cu -- the extern "C" boundary (include/xspmm_b200.h). Validates arguments, makes the
// handle's device current, dispatches to the typed host functions and turns exceptions into
// status codes plus a per-thread message.
#include "ops.cuh"

#include <new>

namespace xspmm_b200 {
const char* last_error_cstr();
}

using namespace xspmm_b200;

XS_API const char* xspmm_status_string(xspmm_status_t s) {
    switch (s) {
        case XSPMM_STATUS_OK: return "ok";
        case XSPMM_STATUS_INVALID_ARGUMENT: return "invalid argument";
        case XSPMM_STATUS_UNSUPPORTED: return "unsupported";
        case XSPMM_STATUS_CUDA_ERROR: return "CUDA error";
        case XSPMM_STATUS_OUT_OF_MEMORY: return "out of memory";
        case XSPMM_STATUS_NCCL_ERROR: return "NCCL error";
        case XSPMM_STATUS_TIMEOUT: return "timeout";
        case XSPMM_STATUS_INTERNAL: return "internal error";
    }
    return "unknown status";
}

XS_API const char* xspmm_last_error(void) { return last_error_cstr(); }

XS_API xspmm_status_t xspmm_create(int device, void* stream, xspmm_handle_t* out) {
    return guarded([&] {
        need(out != nullptr, "out is null");
        *out = nullptr;
        int count = 0;
        XS_CHECK_CUDA(cudaGetDeviceCount(&count));
        need(device >= 0 && device < count, "device ordinal out of range");
        DeviceGuard g(device);
        auto* hh = new xspmm_handle_s();
        Handle& h = hh->h;
        h.device = device;
        h.stream = static_cast<cudaStream_t>(stream);
        try {
            XS_CHECK_CUDA(cudaMalloc(reinterpret_cast<void**>(&h.d_err), sizeof(unsigned)));
            XS_CHECK_CUDA(cudaMemset(h.d_err, 0, sizeof(unsigned)));
            XS_CHECK_CUDA(cudaMallocHost(reinterpret_cast<void**>(&h.h_err), sizeof(unsigned)));
            for (auto& e : h.ev) XS_CHECK_CUDA(cudaEventCreate(&e));
            cudaMemPool_t pool;
            XS_CHECK_CUDA(cudaDeviceGetDefaultMemPool(&pool, device));
            uint64_t keep = ~0ull;  // keep freed scratch in the pool between calls
            XS_CHECK_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep));
        } catch (...) {
            if (h.d_err) cudaFree(h.d_err);
            if (h.h_err) cudaFreeHost(h.h_err);
            for (auto& e : h.ev)
                if (e) cudaEventDestroy(e);
            delete hh;
            throw;
        }
        *out = hh;
    });
}

XS_API xspmm_status_t xspmm_destroy(xspmm_handle_t hh) {
    return guarded([&] {
        if (!hh) return;
        Handle& h = H(hh);
        need(hh->live_plans == 0, "the handle still has plans; destroy them first");
        DeviceGuard g(h.device);
        cudaStreamSynchronize(h.stream);
        cudaFree(h.d_err);
        cudaFreeHost(h.h_err);
        for (auto& e : h.ev) cudaEventDestroy(e);
        hh->destroyed = true;
        delete hh;
    });
}

XS_API xspmm_status_t xspmm_set_stream(xspmm_handle_t hh, void* stream) {
    return guarded([&] { H(hh).stream = static_cast<cudaStream_t>(stream); });
}

XS_API xspmm_status_t xspmm_get_device(xspmm_handle_t hh, int* device) {
    return guarded([&] {
        need(device != nullptr, "device is null");
        *device = H(hh).device;
    });
}

XS_API xspmm_status_t xspmm_get_launch_count(xspmm_handle_t hh, uint64_t* count) {
    return guarded([&] {
        need(count != nullptr, "count is null");
        *count = H(hh).launches;
    });
}

XS_API xspmm_status_t xspmm_reset_launch_count(xspmm_handle_t hh) {
    return guarded([&] { H(hh).launches = 0; });
}

XS_API xspmm_status_t xspmm_set_tier1_kernel(xspmm_handle_t hh, int kind) {
    return guarded([&] {
        need(kind >= 0 && kind <= 2, "kind must be 0 (auto), 1 (mma.sync) or 2 (tcgen05)");
        H(hh).tier1_kernel = kind;
    });
}

XS_API xspmm_status_t xspmm_malloc(xspmm_handle_t hh, void** ptr, size_t bytes) {
    return guarded([&] {
        Handle& h = H(hh);
        need(ptr != nullptr, "ptr is null");
        DeviceGuard g(h.device);
        *ptr = nullptr;
        if (bytes) XS_CHECK_CUDA(cudaMalloc(ptr, bytes));
    });
}

XS_API xspmm_status_t xspmm_free(xspmm_handle_t hh, void* ptr) {
    return guarded([&] {
        Handle& h = H(hh);
        DeviceGuard g(h.device);
        if (ptr) XS_CHECK_CUDA(cudaFree(ptr));
    });
}

static xspmm_status_t copy(xspmm_handle_t hh, void* dst, const void* src, size_t bytes,
                           cudaMemcpyKind kind) {
    return guarded([&] {
        Handle& h = H(hh);
        if (!bytes) return;
        need(dst && src, "null copy pointer");
        DeviceGuard g(h.device);
        XS_CHECK_CUDA(cudaMemcpyAsync(dst, src, bytes, kind, h.stream));
        XS_CHECK_CUDA(cudaStreamSynchronize(h.stream));
    });
}

XS_API xspmm_status_t xspmm_memcpy_h2d(xspmm_handle_t h, void* d, const void* s, size_t n) {
    return copy(h, d, s, n, cudaMemcpyHostToDevice);
}
XS_API xspmm_status_t xspmm_memcpy_d2h(xspmm_handle_t h, void* d, const void* s, size_t n) {
    return copy(h, d, s, n, cudaMemcpyDeviceToHost);
}
XS_API xspmm_status_t xspmm_memcpy_d2d(xspmm_handle_t h, void* d, const void* s, size_t n) {
    return copy(h, d, s, n, cudaMemcpyDeviceToDevice);
}

XS_API xspmm_status_t xspmm_synchronize(xspmm_handle_t hh) {
    return guarded([&] {
        Handle& h = H(hh);
        DeviceGuard g(h.device);
        XS_CHECK_CUDA(cudaStreamSynchronize(h.stream));
        throw_on_device_errors(h, "synchronize");
    });
}

// ------------------------------------------------------------------------------------------------
// Typed entry points
// ------------------------------------------------------------------------------------------------
#define XS_SPMM(SUF, VT, IT)                                                                      \
    XS_API xspmm_status_t xspmm_bcsr_spmm_##SUF(                                                  \
        xspmm_handle_t hh, IT nbr, IT nbc, IT nnzb, IT rb, IT cb, const IT* rp, const IT* ci,     \
        const void* vals, const void* B, float* C, IT M, IT K, IT N, const IT* map) {             \
        return guarded([&] {                                                                      \
            Handle& h = H(hh);                                                                    \
            need(rb >= 1 && cb >= 1, "block shape must be at least 1 x 1");                       \
            need(nbr >= 0 && nbc >= 0 && nnzb >= 0 && M >= 0 && K >= 0 && N >= 0,                 \
                 "negative dimension");                                                           \
            need((int64_t)M <= (int64_t)nbr * rb && (int64_t)K <= (int64_t)nbc * cb,              \
                 "M or K larger than the block grid");                                            \
            need((int64_t)M > ((int64_t)nbr - 1) * rb, "M smaller than the block rows cover");    \
            if (nbr == 0 || N == 0) return;                                                       \
            need(rp && C, "null row_ptr or C");                                                   \
            need(nnzb == 0 || (ci && vals && B), "null col_ind, values or B");                    \
            DeviceGuard g(h.device);                                                              \
            if (rb == 16 && cb == 16)                                                             \
                bcsr_spmm<VT, IT>(h, nbr, nbc, nnzb, rp, ci, static_cast<const VT*>(vals),        \
                                  static_cast<const VT*>(B), C, M, K, N, map);                    \
            else                                                                                  \
                bcsr_spmm_blocks<VT, IT>(h, nbr, rb, cb, rp, ci, static_cast<const VT*>(vals),    \
                                         static_cast<const VT*>(B), C, M, K, N, map);             \
        });                                                                                       \
    }
XS_SPMM(f16f32_i32, __half, int32_t)
XS_SPMM(f16f32_i64, __half, int64_t)
XS_SPMM(bf16f32_i32, __nv_bfloat16, int32_t)
XS_SPMM(bf16f32_i64, __nv_bfloat16, int64_t)
XS_SPMM(f32f32_i32, float, int32_t)
XS_SPMM(f32f32_i64, float, int64_t)

#define XS_CLUSTER(SUF, IT)                                                                       \
    XS_API xspmm_status_t xspmm_cluster_jaccard_##SUF(xspmm_handle_t hh, IT M, IT K, IT nnz,      \
                                                      const IT* rp, const IT* ci, float tau,      \
                                                      IT w, IT* perm) {                           \
        return guarded([&] {                                                                      \
            Handle& h = H(hh);                                                                    \
            need(M >= 0 && K >= 0 && nnz >= 0 && w >= 1, "bad dimension or block width");        \
            if (M == 0) return;                                                                   \
            need(rp && perm && (nnz == 0 || ci), "null pointer");                                 \
            DeviceGuard g(h.device);                                                              \
            cluster_jaccard<IT>(h, M, K, nnz, rp, ci, tau, w, perm);                              \
            throw_on_device_errors(h, "compute_1d_jaccard_clustering");                           \
        });                                                                                       \
    }
XS_CLUSTER(i32, int32_t)
XS_CLUSTER(i64, int64_t)

#define XS_PERMUTE(SUF, VT, IT)                                                                   \
    XS_API xspmm_status_t xspmm_permute_rows_##SUF(xspmm_handle_t hh, IT M, IT K, IT nnz,         \
                                                   const IT* rp, const IT* ci, const void* v,     \
                                                   const IT* perm, IT* orp, IT* oci, void* ov) {  \
        return guarded([&] {                                                                      \
            Handle& h = H(hh);                                                                    \
            need(M >= 0 && K >= 0 && nnz >= 0, "negative dimension");                             \
            need(orp != nullptr, "null out_row_ptr");                                             \
            need(M == 0 || (rp && perm), "null row_ptr or perm");                                 \
            need(nnz == 0 || (ci && oci), "null col_ind");                                        \
            DeviceGuard g(h.device);                                                              \
            permute_rows<VT, IT>(h, M, nnz, rp, ci, static_cast<const VT*>(v), perm, orp, oci,    \
                                 static_cast<VT*>(ov), true);                                     \
        });                                                                                       \
    }
XS_PERMUTE(f16_i32, __half, int32_t)
XS_PERMUTE(f16_i64, __half, int64_t)
XS_PERMUTE(bf16_i32, __nv_bfloat16, int32_t)
XS_PERMUTE(bf16_i64, __nv_bfloat16, int64_t)
XS_PERMUTE(f32_i32, float, int32_t)
XS_PERMUTE(f32_i64, float, int64_t)

#define XS_COUNT(SUF, IT)                                                                         \
    XS_API xspmm_status_t xspmm_csr_to_bcsr_count_##SUF(xspmm_handle_t hh, IT M, IT K, IT nnz,    \
                                                        const IT* rp, const IT* ci, IT rb, IT cb, \
                                                        IT* brp, int64_t* nnzb) {                 \
        return guarded([&] {                                                                      \
            Handle& h = H(hh);                                                                    \
            need(M >= 0 && K >= 0 && nnz >= 0 && rb >= 1 && cb >= 1, "bad dimension");           \
            need(brp && nnzb, "null output");                                                     \
            need(M == 0 || rp, "null row_ptr");                                                   \
            DeviceGuard g(h.device);                                                              \
            *nnzb = csr_to_bcsr_count<IT>(h, M, K, nnz, rp, ci, rb, cb, brp);                     \
        });                                                                                       \
    }
XS_COUNT(i32, int32_t)
XS_COUNT(i64, int64_t)

#define XS_FILL(SUF, VT, IT)                                                                      \
    XS_API xspmm_status_t xspmm_csr_to_bcsr_fill_##SUF(                                           \
        xspmm_handle_t hh, IT M, IT K, IT nnz, const IT* rp, const IT* ci, const void* v, IT rb,  \
        IT cb, const IT* brp, IT* bci, void* bv) {                                                \
        return guarded([&] {                                                                      \
            Handle& h = H(hh);                                                                    \
            need(M >= 0 && K >= 0 && nnz >= 0 && rb >= 1 && cb >= 1, "bad dimension");           \
            need(M == 0 || (rp && brp), "null row_ptr");                                          \
            DeviceGuard g(h.device);                                                              \
            csr_to_bcsr_fill<VT, IT>(h, M, K, nnz, rp, ci, static_cast<const VT*>(v), rb, cb,     \
                                     brp, bci, static_cast<VT*>(bv));                             \
        });                                                                                       \
    }
XS_FILL(f16_i32, __half, int32_t)
XS_FILL(f16_i64, __half, int64_t)
XS_FILL(bf16_i32, __nv_bfloat16, int32_t)
XS_FILL(bf16_i64, __nv_bfloat16, int64_t)
XS_FILL(f32_i32, float, int32_t)
XS_FILL(f32_i64, float, int64_t)

#define XS_UNPERM(SUF, VT, IT)                                                                    \
    XS_API xspmm_status_t xspmm_unpermute_dense_##SUF(xspmm_handle_t hh, const void* in,          \
                                                      void* out, const IT* perm, IT M, IT N) {    \
        return guarded([&] {                                                                      \
            Handle& h = H(hh);                                                                    \
            need(M >= 0 && N >= 0, "negative dimension");                                         \
            if (M == 0 || N == 0) return;                                                         \
            need(in && out && perm, "null pointer");                                              \
            DeviceGuard g(h.device);                                                              \
            unpermute_dense<VT, IT>(h, static_cast<const VT*>(in), static_cast<VT*>(out), perm,   \
                                    M, N, true);                                                  \
        });                                                                                       \
    }
XS_UNPERM(f32_i32, float, int32_t)
XS_UNPERM(f32_i64, float, int64_t)
XS_UNPERM(f16_i32, __half, int32_t)
XS_UNPERM(f16_i64, __half, int64_t)
XS_UNPERM(bf16_i32, __nv_bfloat16, int32_t)
XS_UNPERM(bf16_i64, __nv_bfloat16, int64_t)

#define XS_PIPE(SUF, VT, IT)                                                                      \
    XS_API xspmm_status_t xspmm_spmm_csr_##SUF(                                                   \
        xspmm_handle_t hh, IT M, IT K, IT nnz, const IT* rp, const IT* ci, const void* v,         \
        const void* B, float* C, IT N, IT hw, int clustering, xspmm_timings_t* t) {               \
        return guarded([&] {                                                                      \
            Handle& h = H(hh);                                                                    \
            need(M >= 0 && K >= 0 && nnz >= 0 && N >= 0, "negative dimension");                   \
            need(hw >= 1, "hw_block_size must be at least 1");                                    \
            if (t) *t = xspmm_timings_t{0, 0, 0, 0, 0, 0};                                        \
            if (M == 0 || N == 0) return;                                                         \
            need(rp && C && (nnz == 0 || (ci && v && B)), "null pointer");                        \
            DeviceGuard g(h.device);                                                              \
            spmm_csr_pipeline<VT, IT>(h, M, K, nnz, rp, ci, static_cast<const VT*>(v),            \
                                      static_cast<const VT*>(B), C, N, hw, clustering != 0, t);   \
        });                                                                                       \
    }
XS_PIPE(f16f32_i32, __half, int32_t)
XS_PIPE(f16f32_i64, __half, int64_t)
XS_PIPE(bf16f32_i32, __nv_bfloat16, int32_t)
XS_PIPE(bf16f32_i64, __nv_bfloat16, int64_t)
XS_PIPE(f32f32_i32, float, int32_t)
XS_PIPE(f32f32_i64, float, int64_t)
