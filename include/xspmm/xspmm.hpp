// xspmm/xspmm.hpp -- the public API of the hot path, drop-in for the reference's
// include/xspmm/xspmm.hpp:14-40.
//
//   Tier 1: spmm(const BCSRMatrix<In, Idx>& A, const In* B, Out* C, Idx N)
//   Tier 2: spmm(exec, const CSRMatrix<In, Idx>& A, const In* B, Out* C, Idx N,
//                Idx hw_block_size = 16, bool optimize_pattern = true, SpMMTimings* = nullptr)
//   unpermute_dense_matrix(exec, in, out, perm, M, N)
//
// B is K x N and C is M x N, row-major device arrays (leading dimension N), as in the reference.
// Instantiations: In = __half or float with Out = float, Idx = int32_t or int64_t (the reference's
// CUDA backend names the same four, src/cuda/unstructured_mtx_mul.cu:137-148), and In =
// __nv_bfloat16 (tensor-core bf16, fp32 accumulation) as an addition. Work is enqueued on
// the executor's stream and is asynchronous, like the reference's kernel launches; Tier 2 returns
// after its last launch and, when timings is given, after the stage events have completed.
#pragma once

#include <memory>
#include <type_traits>

#include "clustering.hpp"
#include "core/executor.hpp"
#include "core/timings.hpp"
#include "detail/abi.hpp"
#include "matrix/bcsr.hpp"
#include "matrix/conversion.hpp"
#include "matrix/csr.hpp"
#include "plan.hpp"

namespace xspmm {

// Tier 1: C = A * B for A in BCSR (16x16 blocks on the tensor cores; other block shapes on a SIMT
// kernel that computes the product the BCSR describes). Every row of C is written.
template <typename InputType, typename OutputType, typename IndexType = int64_t>
void spmm(const BCSRMatrix<InputType, IndexType>& A, const InputType* B, OutputType* C,
          IndexType N) {
    static_assert(std::is_same<OutputType, float>::value, "C is float");
    detail::check(detail::Abi<InputType, IndexType>::spmm(
        detail::handle_of(A.get_executor()), A.get_num_block_rows(), A.get_num_block_cols(),
        A.get_num_blocks(), A.get_r_block(), A.get_c_block(), A.get_bcsr_row_ptr(),
        A.get_bcsr_col_ind(), A.get_bcsr_values(), B, C, A.get_num_rows(), A.get_num_cols(), N,
        nullptr));
}

// Tier 2: clustering (optional) -> permutation -> CSR->BCSR -> Tier 1 -> unpermute.
template <typename InputType, typename OutputType, typename IndexType = int64_t>
void spmm(std::shared_ptr<const Executor> exec, const CSRMatrix<InputType, IndexType>& A,
          const InputType* B, OutputType* C, IndexType N, IndexType hw_block_size = 16,
          bool optimize_pattern = true, SpMMTimings* timings = nullptr) {
    static_assert(std::is_same<OutputType, float>::value, "C is float");
    xspmm_timings_t t{};
    detail::check(detail::Abi<InputType, IndexType>::pipeline(
        detail::handle_of(exec), A.get_num_rows(), A.get_num_cols(), A.get_nnz(), A.get_row_ptr(),
        A.get_col_ind(), A.get_values(), B, C, N, hw_block_size, optimize_pattern ? 1 : 0,
        timings ? &t : nullptr));
    if (timings) {
        timings->clustering_ms = t.clustering_ms;
        timings->permutation_ms = t.permutation_ms;
        timings->conversion_ms = t.conversion_ms;
        timings->spmm_ms = t.spmm_ms;
        timings->unpermutation_ms = t.unpermutation_ms;
        timings->total_pipeline_ms = t.total_pipeline_ms;
    }
}

// out[perm[r] * N + c] = in[r * N + c]
template <typename ValueType, typename IndexType>
void unpermute_dense_matrix(std::shared_ptr<const Executor> exec, const ValueType* in_matrix,
                            ValueType* out_matrix, const IndexType* perm, IndexType M,
                            IndexType N) {
    detail::check(detail::Abi<ValueType, IndexType>::unpermute(detail::handle_of(exec), in_matrix,
                                                               out_matrix, perm, M, N));
}

}  // namespace xspmm
