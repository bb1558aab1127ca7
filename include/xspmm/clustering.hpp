// xspmm/clustering.hpp -- row clustering and CSR row permutation.
// Same signatures and results as the reference (include/xspmm/clustering.hpp:19-38):
// compute_1d_jaccard_clustering writes perm_out[M] (perm[new] = old, caller-allocated on exec),
// bit-identical to the reference's greedy Sylos-Labini clustering, computed on the device;
// apply_permutation returns the row-permuted CSR.
#pragma once

#include <memory>

#include "detail/abi.hpp"
#include "matrix/csr.hpp"

namespace xspmm {

template <typename ValueType, typename IndexType = int64_t>
void compute_1d_jaccard_clustering(std::shared_ptr<const Executor> exec,
                                   const CSRMatrix<ValueType, IndexType>& A, float dist_thresh,
                                   IndexType block_width, IndexType* perm_out) {
    detail::check(detail::Abi<ValueType, IndexType>::cluster(
        detail::handle_of(exec), A.get_num_rows(), A.get_num_cols(), A.get_nnz(),
        A.get_row_ptr(), A.get_col_ind(), dist_thresh, block_width, perm_out));
}

template <typename ValueType, typename IndexType = int64_t>
CSRMatrix<ValueType, IndexType> apply_permutation(std::shared_ptr<const Executor> target_exec,
                                                  const CSRMatrix<ValueType, IndexType>& A,
                                                  const IndexType* perm) {
    CSRMatrix<ValueType, IndexType> out(target_exec, A.get_num_rows(), A.get_num_cols(),
                                        A.get_nnz());
    detail::check(detail::Abi<ValueType, IndexType>::permute(
        detail::handle_of(target_exec), A.get_num_rows(), A.get_num_cols(), A.get_nnz(),
        A.get_row_ptr(), A.get_col_ind(), A.get_values(), perm, out.get_row_ptr(),
        out.get_col_ind(), out.get_values()));
    return out;
}

}  // namespace xspmm
