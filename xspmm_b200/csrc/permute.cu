// permute.cu -- CSR row permutation and dense unpermutation (bandwidth kernels).
//
// permute_rows follows the reference's three steps (src/cuda/mtx_permutation.cu:12-65 with the
// kernels of src/common/permutation.hpp:15-66): new row lengths from perm, an exclusive scan into
// the new row_ptr (the reference uses thrust::exclusive_scan plus a synchronous H2D of nnz for the
// last entry; here the library's own scan writes the total), then a copy of column indices and
// values in their original order (the reference copies a row per warp; here a warp copies the
// entries of 32 rows as one stream, and a CTA each row above PERM_LONG entries). The copy is
// guarded against a perm that is not a permutation (the reference would write out of bounds).
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

// Row-per-warp copy (the reference's scheme), kept for the fixed-scratch entry point, which may
// not allocate the long-row list of the kernels below.
template <typename VT, typename IT>
__global__ void permute_copy_rows_kernel(const IT* __restrict__ rp, const IT* __restrict__ ci,
                                         const VT* __restrict__ v, const IT* __restrict__ perm,
                                         const IT* __restrict__ nrp, IT* __restrict__ nci,
                                         VT* __restrict__ nv, int64_t M, int64_t nnz,
                                         unsigned* err) {
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

// The copy of permute_rows takes 32 consecutive new rows per warp and walks their entries as one
// stream with every lane busy: lane i holds new row i0+i's source and destination offsets and the
// inclusive prefix of the lengths, and the row of stream position k is found by a 5-step search
// over that prefix. Writes are coalesced whatever the row lengths (most rows of graph matrices
// hold a few entries, which a warp per row would copy with most lanes idle); reads are contiguous
// within each source row. Rows longer than PERM_LONG entries (the hub rows of power-law graphs,
// which clustering tends to place next to each other) are left out of the stream and listed, and
// permute_copy_long_kernel copies each of them with a whole CTA.
constexpr int64_t PERM_LONG = 1024;

template <typename VT, typename IT>
__global__ void permute_copy_kernel(const IT* __restrict__ rp, const IT* __restrict__ ci,
                                    const VT* __restrict__ v, const IT* __restrict__ perm,
                                    const IT* __restrict__ nrp, IT* __restrict__ nci,
                                    VT* __restrict__ nv, int64_t M, int64_t nnz,
                                    int64_t* __restrict__ long_rows, unsigned* __restrict__ nlong,
                                    unsigned long_cap, unsigned* err) {
    const unsigned FULL = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t g = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; g * 32 < M;
         g += warps) {
        const int64_t i = g * 32 + lane;
        int64_t os = 0, ns = 0, len = 0;
        if (i < M) {
            const int64_t p = (int64_t)perm[i];
            if (p >= 0 && p < M) {  // else the lengths kernel flagged it and gave it length 0
                os = (int64_t)rp[p];
                len = (int64_t)rp[p + 1] - os;
                ns = (int64_t)nrp[i];
                if (ns < 0 || ns + len > nnz) {  // only with a perm that is not a permutation
                    flag_error(err, DERR_PERM_OUT_OF_RANGE);
                    len = 0;
                }
            }
        }
        int slen = (int)len;  // this row's part of the warp's stream
        if (len > PERM_LONG) {
            const unsigned k = atomicAdd(nlong, 1u);
            if (k < long_cap) long_rows[k] = i;
            else flag_error(err, DERR_INTERNAL);
            slen = 0;
        }
        int incl = slen;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(FULL, incl, o);
            if (lane >= o) incl += t;
        }
        const int total = __shfl_sync(FULL, incl, 31);  // <= 32 * PERM_LONG
        const int64_t dsrc = os - (int64_t)(incl - slen);  // stream position k of this row:
        const int64_t ddst = ns - (int64_t)(incl - slen);  // source k + dsrc, destination k + ddst
        // 8 entries per lane per round: every load of the round is issued before its stores
        constexpr int U = 8;
        for (int k0 = 0; k0 < total; k0 += 32 * U) {
            int64_t dst[U];
            IT cv[U];
            VT vv[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int k = k0 + u * 32 + lane;
                int j = 0;
#pragma unroll
                for (int step = 16; step >= 1; step >>= 1)
                    if (__shfl_sync(FULL, incl, j + step - 1) <= k) j += step;
                const int64_t src = __shfl_sync(FULL, dsrc, j) + k;
                const int64_t d = __shfl_sync(FULL, ddst, j) + k;  // every lane shuffles
                dst[u] = k < total ? d : -1;
                if (dst[u] >= 0) {
                    cv[u] = ci[src];
                    if (v) vv[u] = v[src];
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (dst[u] >= 0) {
                    nci[dst[u]] = cv[u];
                    if (v) nv[dst[u]] = vv[u];
                }
            }
        }
    }
}

// The listed long rows, a CTA each (4 entries in flight per thread).
template <typename VT, typename IT>
__global__ void __launch_bounds__(256)
permute_copy_long_kernel(const IT* __restrict__ rp, const IT* __restrict__ ci,
                         const VT* __restrict__ v, const IT* __restrict__ perm,
                         const IT* __restrict__ nrp, IT* __restrict__ nci, VT* __restrict__ nv,
                         const int64_t* __restrict__ long_rows, const unsigned* __restrict__ nlong,
                         unsigned long_cap) {
    const unsigned n = min(*nlong, long_cap);
    for (unsigned e = blockIdx.x; e < n; e += gridDim.x) {
        const int64_t i = long_rows[e];
        const int64_t p = (int64_t)perm[i];  // checked when the row was listed
        const int64_t os = (int64_t)rp[p], len = (int64_t)rp[p + 1] - os, ns = (int64_t)nrp[i];
        for (int64_t t0 = 0; t0 < len; t0 += 4 * 256) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int64_t t = t0 + u * 256 + threadIdx.x;
                if (t < len) {
                    nci[ns + t] = ci[os + t];
                    if (v) nv[ns + t] = v[os + t];
                }
            }
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
    // rows above PERM_LONG entries: at most nnz / PERM_LONG of them
    const unsigned long_cap = (unsigned)std::min<int64_t>(M, nnz / PERM_LONG + 1);
    DevBuf<int64_t> long_rows(long_cap, h.stream);
    DevBuf<unsigned> nlong(1, h.stream);
    XS_CHECK_CUDA(cudaMemsetAsync(nlong.get(), 0, sizeof(unsigned), h.stream));
    permute_copy_kernel<VT, IT><<<grid_for(h, M, 256), 256, 0, h.stream>>>(
        row_ptr, col_ind, values, perm, out_row_ptr, out_col_ind, out_values, M, nnz,
        long_rows.get(), nlong.get(), long_cap, h.d_err);
    after_launch(h, "permute_copy");
    if (nnz > PERM_LONG) {
        permute_copy_long_kernel<VT, IT><<<(unsigned)sm_count(h.device) * 2, 256, 0, h.stream>>>(
            row_ptr, col_ind, values, perm, out_row_ptr, out_col_ind, out_values, long_rows.get(),
            nlong.get(), long_cap);
        after_launch(h, "permute_copy_long");
    }
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
    permute_copy_rows_kernel<VT, IT><<<grid_for(h, M * 32, 256), 256, 0, h.stream>>>(
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
XS_INST_PERM(__nv_bfloat16, int32_t)
XS_INST_PERM(__nv_bfloat16, int64_t)
XS_INST_PERM(float, int32_t)
XS_INST_PERM(float, int64_t)

}  // namespace xspmm_b200
