// xspmm/matrix/conversion.hpp -- CSR -> BCSR.
// Same signature and result as the reference's csr_to_bcsr (include/xspmm/matrix/conversion.hpp:
// 19-22, src/core/conversion.cpp:8-100), computed on the device instead of the host. The block
// count is read back to size the result (one synchronization), as the reference's BCSRMatrix
// needs it at construction.
#pragma once

#include <memory>

#include "../detail/abi.hpp"
#include "bcsr.hpp"
#include "csr.hpp"

namespace xspmm {

template <typename ValueType, typename IndexType = int64_t>
BCSRMatrix<ValueType, IndexType> csr_to_bcsr(std::shared_ptr<const Executor> target_exec,
                                             const CSRMatrix<ValueType, IndexType>& csr,
                                             IndexType r_block, IndexType c_block) {
    using A = detail::Abi<ValueType, IndexType>;
    if (r_block < 1 || c_block < 1) throw std::invalid_argument("block sizes must be positive");
    auto h = detail::handle_of(target_exec);
    const IndexType M = csr.get_num_rows(), K = csr.get_num_cols();
    const IndexType nbr = (M + r_block - 1) / r_block, nbc = (K + c_block - 1) / c_block;
    IndexType* brp = nullptr;
    target_exec->allocate(reinterpret_cast<void**>(&brp), static_cast<size_t>(nbr + 1) * sizeof(IndexType));
    int64_t nnzb = 0;
    try {
        detail::check(A::count(h, M, K, csr.get_nnz(), csr.get_row_ptr(), csr.get_col_ind(),
                               r_block, c_block, brp, &nnzb));
    } catch (...) {
        target_exec->free(brp);
        throw;
    }
    BCSRMatrix<ValueType, IndexType> out(target_exec, nbr, nbc, static_cast<IndexType>(nnzb),
                                         r_block, c_block);
    out.set_extent(M, K);
    target_exec->copy_device_to_device(out.get_bcsr_row_ptr(), brp,
                                       static_cast<size_t>(nbr + 1) * sizeof(IndexType));
    target_exec->free(brp);
    detail::check(A::fill(h, M, K, csr.get_nnz(), csr.get_row_ptr(), csr.get_col_ind(),
                          csr.get_values(), r_block, c_block, out.get_bcsr_row_ptr(),
                          out.get_bcsr_col_ind(), out.get_bcsr_values()));
    return out;
}

}  // namespace xspmm
