// spmm_blocks.cu -- Tier-1 BCSR SpMM for block shapes other than 16x16.
//
// The reference's Tier-1 kernel hard-codes 16x16 tiles (src/cuda/unstructured_mtx_mul.cu:39,
// src/common/spmm_math.hpp:20-146): given a BCSR of r x c blocks it reads each block as 256
// values and so computes a wrong product (or reads past the values) whenever r or c is not 16.
// This library instead computes the product the BCSR describes,
//   C[r br + i, n] = sum over the blocks j of block row br (col_ind order), k < c, of
//                    values[j r c + i c + k] * B[c col_ind[j] + k, n],
// for any r, c >= 1: the row's terms are added in that (column) order in fp64 and rounded once
// to fp32, so the result does not depend on the launch shape. Rows >= M are not written and B
// rows >= K are read as zero, as for the 16x16 kernels.
//
// The 16x16 tensor-core kernels are what the Tier-2 pipeline and the plans use (they build a
// 16x16 BCSR whatever block width clusters the rows); this kernel serves Tier-1 calls given
// another block shape, so it is written for clarity: a CTA per (block row, 128-column tile), a
// thread per column, the block row's rows one after another, each value read once per CTA from L1.
#include "ops.cuh"

namespace xspmm_b200 {
namespace {

constexpr int BS_TN = 128;

template <typename VT, typename IT>
__global__ void __launch_bounds__(BS_TN)
bcsr_spmm_blocks_kernel(const IT* __restrict__ rp, const IT* __restrict__ ci,
                        const VT* __restrict__ v, const VT* __restrict__ B, float* __restrict__ C,
                        const IT* __restrict__ row_map, int64_t nbr, int64_t rb, int64_t cb,
                        int64_t M, int64_t K, int64_t N, unsigned* __restrict__ err) {
    const int64_t n = (int64_t)blockIdx.y * BS_TN + threadIdx.x;
    for (int64_t br = blockIdx.x; br < nbr; br += gridDim.x) {
        const int64_t j0 = (int64_t)rp[br], j1 = (int64_t)rp[br + 1];
        for (int64_t i = 0; i < rb; ++i) {
            const int64_t r = br * rb + i;
            if (r >= M) break;
            double acc = 0.0;
            if (n < N) {
                for (int64_t j = j0; j < j1; ++j) {
                    const int64_t col0 = (int64_t)ci[j] * cb;
                    const VT* a = v + (j * rb + i) * cb;
                    for (int64_t k = 0; k < cb; ++k) {
                        const int64_t col = col0 + k;
                        if (col >= K) break;
                        acc = fma((double)to_float(a[k]), (double)to_float(B[col * N + n]), acc);
                    }
                }
            }
            const int64_t orow = row_map ? (int64_t)row_map[r] : r;
            if (orow < 0 || orow >= M) {
                if (threadIdx.x == 0) flag_error(err, DERR_PERM_OUT_OF_RANGE);
                continue;
            }
            if (n < N) C[orow * N + n] = (float)acc;
        }
    }
}

}  // namespace

template <typename VT, typename IT>
void bcsr_spmm_blocks(Handle& h, int64_t nbr, int64_t rb, int64_t cb, const IT* rp, const IT* ci,
                      const VT* v, const VT* B, float* C, int64_t M, int64_t K, int64_t N,
                      const IT* map) {
    if (nbr == 0 || N == 0 || M == 0) return;
    const int64_t tiles = ceil_div(N, BS_TN);
    XS_REQUIRE(tiles <= 65535, XSPMM_STATUS_UNSUPPORTED, "N too large for the block-shape kernel");
    const unsigned grid_x = (unsigned)std::max<int64_t>(
        1, std::min(nbr, (int64_t)sm_count(h.device) * 32));
    bcsr_spmm_blocks_kernel<VT, IT><<<dim3(grid_x, (unsigned)tiles), BS_TN, 0, h.stream>>>(
        rp, ci, v, B, C, map, nbr, rb, cb, M, K, N, h.d_err);
    after_launch(h, "bcsr_spmm_blocks");
}

#define XS_INST_BS(VT, IT)                                                                        \
    template void bcsr_spmm_blocks<VT, IT>(Handle&, int64_t, int64_t, int64_t, const IT*,        \
                                           const IT*, const VT*, const VT*, float*, int64_t,      \
                                           int64_t, int64_t, const IT*);
XS_INST_BS(__half, int32_t)
XS_INST_BS(__half, int64_t)
XS_INST_BS(__nv_bfloat16, int32_t)
XS_INST_BS(__nv_bfloat16, int64_t)
XS_INST_BS(float, int32_t)
XS_INST_BS(float, int64_t)

}  // namespace xspmm_b200
