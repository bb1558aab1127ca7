// permute.cu -- CSR row permutation and dense unpermutation (bandwidth kernels).
//
// permute_rows follows the reference's three steps (src/cuda/mtx_permutation.cu:12-65 with the
// kernels of src/common/permutation.hpp:15-66): new row lengths from perm, an exclusive scan into
// the new row_ptr (the reference uses thrust::exclusive_scan plus a synchronous H2D of nnz for the
// last entry; here the library's own scan writes the total), then a warp-per-row copy of column
// indices and values in their original order. The copy is guarded against a perm that is not a
// permutation (the reference would write out of bounds).
//
// unpermute_dense is out[perm[r]] = in[r] for rows of N elements (permutation.hpp:89-108), one warp
// per row, 16-byte vectors when the rows allow it.
#include "ops.cuh"

namespace xspmm_b200 {
namespace {

template <typename IT>
__global__ void permute_lengths_kernel(const IT* __restrict__ rp, const IT* __restrict__ perm,
                                       IT* __restrict__ len, int64_t M, unsigned* seen,
                                       unsigned* err) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < M;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t p = (int64_t)perm[i];
        if (p < 0 || p >= M) {
            flag_error(err, DERR_PERM_OUT_OF_RANGE);
            len[i] = 0;
            continue;
        }
        if (seen) {
            const unsigned bit = 1u << (p & 31);
            if (atomicOr(&seen[p >> 5], bit) & bit) flag_error(err, DERR_PERM_OUT_OF_RANGE);
        }
        len[i] = rp[p + 1] - rp[p];
    }
}

template <typename VT, typename IT>
__global__ void permute_copy_kernel(const IT* __restrict__ rp, const IT* __restrict__ ci,
                                    const VT* __restrict__ v, const IT* __restrict__ perm,
                                    const IT* __restrict__ nrp, IT* __restrict__ nci,
                                    VT* __restrict__ nv, int64_t M, int64_t nnz, unsigned* err) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < M; i += warps) {
        const int64_t p = (int64_t)perm[i];
        if (p < 0 || p >= M) continue;
        const int64_t os = rp[p], len = (int64_t)rp[p + 1] - os, ns = nrp[i];
        if (ns < 0 || ns + len > nnz) {
            if (lane == 0) flag_error(err, DERR_PERM_OUT_OF_RANGE);
            continue;
        }
        for (int64_t e = lane; e < len; e += 32) {
            nci[ns + e] = ci[os + e];
            if (v) nv[ns + e] = v[os + e];
        }
    }
}

template <typename VT, typename IT, bool VEC>
__global__ void unpermute_kernel(const VT* __restrict__ in, VT* __restrict__ out,
                                 const IT* __restrict__ perm, int64_t M, int64_t N,
                                 unsigned* err) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < M; r += warps) {
        const int64_t o = (int64_t)perm[r];
        if (o < 0 || o >= M) {
            if (lane == 0) flag_error(err, DERR_PERM_OUT_OF_RANGE);
            continue;
        }
        if constexpr (VEC) {
            constexpr int PER = 16 / sizeof(VT);
            const uint4* src = reinterpret_cast<const uint4*>(in + r * N);
            uint4* dst = reinterpret_cast<uint4*>(out + o * N);
            for (int64_t c = lane; c < N / PER; c += 32) dst[c] = src[c];
        } else {
            for (int64_t c = lane; c < N; c += 32) out[o * N + c] = in[r * N + c];
        }
    }
}

unsigned grid_for(Handle& h, int64_t work_items, int threads) {
    const int64_t want = ceil_div(work_items, threads);
    const int64_t cap = (int64_t)sm_count(h.device) * 16;
    return (unsigned)std::max<int64_t>(1, std::min(want, cap));
}

}  // namespace

template <typename VT, typename IT>
void permute_rows(Handle& h, int64_t M, int64_t nnz, const IT* row_ptr, const IT* col_ind,
                  const VT* values, const IT* perm, IT* out_row_ptr, IT* out_col_ind,
                  VT* out_values, bool check) {
    if (M == 0) {
        XS_CHECK_CUDA(cudaMemsetAsync(out_row_ptr, 0, sizeof(IT), h.stream));
        return;
    }
    DevBuf<unsigned> seen(check ? (size_t)ceil_div(M, 32) : 0, h.stream);
    if (check) XS_CHECK_CUDA(cudaMemsetAsync(seen.get(), 0, seen.n * sizeof(unsigned), h.stream));
    permute_lengths_kernel<IT><<<grid_for(h, M, 256), 256, 0, h.stream>>>(
        row_ptr, perm, out_row_ptr, M, seen.get(), h.d_err);
    after_launch(h, "permute_lengths");
    exclusive_scan<IT>(h, out_row_ptr, out_row_ptr, M);
    permute_copy_kernel<VT, IT><<<grid_for(h, M * 32, 256), 256, 0, h.stream>>>(
        row_ptr, col_ind, values, perm, out_row_ptr, out_col_ind, out_values, M, nnz, h.d_err);
    after_launch(h, "permute_copy");
    if (check) throw_on_device_errors(h, "apply_permutation");
}

template <typename VT, typename IT>
void permute_rows_scratch(Handle& h, int64_t M, int64_t nnz, const IT* row_ptr, const IT* col_ind,
                          const VT* values, const IT* perm, IT* out_row_ptr, IT* out_col_ind,
                          VT* out_values, unsigned* seen, IT* scan_scratch,
                          int64_t scan_scratch_elems) {
    if (M == 0) {
        XS_CHECK_CUDA(cudaMemsetAsync(out_row_ptr, 0, sizeof(IT), h.stream));
        return;
    }
    XS_CHECK_CUDA(cudaMemsetAsync(seen, 0, (size_t)ceil_div(M, 32) * sizeof(unsigned), h.stream));
    permute_lengths_kernel<IT><<<grid_for(h, M, 256), 256, 0, h.stream>>>(
        row_ptr, perm, out_row_ptr, M, seen, h.d_err);
    after_launch(h, "permute_lengths");
    exclusive_scan_scratch<IT>(h, out_row_ptr, out_row_ptr, M, scan_scratch, scan_scratch_elems);
    permute_copy_kernel<VT, IT><<<grid_for(h, M * 32, 256), 256, 0, h.stream>>>(
        row_ptr, col_ind, values, perm, out_row_ptr, out_col_ind, out_values, M, nnz, h.d_err);
    after_launch(h, "permute_copy");
    throw_on_device_errors(h, "apply_permutation");
}

template <typename VT, typename IT>
void unpermute_dense(Handle& h, const VT* in, VT* out, const IT* perm, int64_t M, int64_t N,
                     bool check) {
    if (M == 0 || N == 0) return;
    const bool vec = ((N * (int64_t)sizeof(VT)) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(in) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(out) % 16 == 0);
    const unsigned grid = grid_for(h, M * 32, 256);
    if (vec)
        unpermute_kernel<VT, IT, true><<<grid, 256, 0, h.stream>>>(in, out, perm, M, N, h.d_err);
    else
        unpermute_kernel<VT, IT, false><<<grid, 256, 0, h.stream>>>(in, out, perm, M, N, h.d_err);
    after_launch(h, "unpermute_dense");
    if (check) throw_on_device_errors(h, "unpermute_dense_matrix");
}

#define XS_INST_PERM(VT, IT)                                                                      \
    template void permute_rows<VT, IT>(Handle&, int64_t, int64_t, const IT*, const IT*, const VT*, \
                                       const IT*, IT*, IT*, VT*, bool);                           \
    template void unpermute_dense<VT, IT>(Handle&, const VT*, VT*, const IT*, int64_t, int64_t,   \
                                          bool);
template void permute_rows_scratch<__half, int32_t>(Handle&, int64_t, int64_t, const int32_t*,
                                                    const int32_t*, const __half*, const int32_t*,
                                                    int32_t*, int32_t*, __half*, unsigned*,
                                                    int32_t*, int64_t);
template void permute_rows_scratch<float, int32_t>(Handle&, int64_t, int64_t, const int32_t*,
                                                   const int32_t*, const float*, const int32_t*,
                                                   int32_t*, int32_t*, float*, unsigned*, int32_t*,
                                                   int64_t);
XS_INST_PERM(__half, int32_t)
XS_INST_PERM(__half, int64_t)
XS_INST_PERM(float, int32_t)
XS_INST_PERM(float, int64_t)

}  // namespace xspmm_b200
