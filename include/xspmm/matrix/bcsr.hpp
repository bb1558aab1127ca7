// xspmm/matrix/bcsr.hpp -- device-resident BCSR matrix (r_block x c_block blocks, row-major
// inside a block).
//
// Same layout, constructor, move semantics, accessors and copy_from_host as the reference's
// BCSRMatrix (include/xspmm/matrix/bcsr.hpp:15-103): row_ptr[nbr+1], col_ind[nnzb],
// values[nnzb*r*c]. Sizes are computed in size_t (the reference's IndexType product
// num_blocks*r*c overflows int32 past 2^31 values, bcsr.hpp:30). It additionally records the row
// and column counts of the matrix it was built from (get_num_rows/get_num_cols, defaulting to the
// block grid's extent) so the Tier-1 SpMM can guard a ragged last block row or column.
#pragma once

#include <cstdint>
#include <memory>
#include <stdexcept>
#include <utility>

#include "../core/executor.hpp"

namespace xspmm {

template <typename ValueType, typename IndexType = int64_t>
class BCSRMatrix {
public:
    BCSRMatrix(std::shared_ptr<const Executor> exec, IndexType num_block_rows,
               IndexType num_block_cols, IndexType num_blocks, IndexType r_block,
               IndexType c_block)
        : exec_(std::move(exec)), num_block_rows_(num_block_rows), num_block_cols_(num_block_cols),
          num_blocks_(num_blocks), r_block_(r_block), c_block_(c_block),
          num_rows_(num_block_rows * r_block), num_cols_(num_block_cols * c_block) {
        if (num_block_rows < 0 || num_block_cols < 0 || num_blocks < 0)
            throw std::invalid_argument("BCSR dimensions must be non-negative.");
        exec_->allocate(reinterpret_cast<void**>(&row_ptr_),
                        static_cast<size_t>(num_block_rows + 1) * sizeof(IndexType));
        if (num_blocks > 0) {
            exec_->allocate(reinterpret_cast<void**>(&col_ind_),
                            static_cast<size_t>(num_blocks) * sizeof(IndexType));
            exec_->allocate(reinterpret_cast<void**>(&values_), value_count() * sizeof(ValueType));
        }
    }
    ~BCSRMatrix() { release(); }
    BCSRMatrix(const BCSRMatrix&) = delete;
    BCSRMatrix& operator=(const BCSRMatrix&) = delete;
    BCSRMatrix(BCSRMatrix&& o) noexcept { take(o); }
    BCSRMatrix& operator=(BCSRMatrix&& o) noexcept {
        if (this != &o) {
            release();
            take(o);
        }
        return *this;
    }

    IndexType get_num_block_rows() const { return num_block_rows_; }
    IndexType get_num_block_cols() const { return num_block_cols_; }
    IndexType get_num_blocks() const { return num_blocks_; }
    IndexType get_r_block() const { return r_block_; }
    IndexType get_c_block() const { return c_block_; }
    IndexType get_num_rows() const { return num_rows_; }
    IndexType get_num_cols() const { return num_cols_; }
    void set_extent(IndexType num_rows, IndexType num_cols) {
        num_rows_ = num_rows;
        num_cols_ = num_cols;
    }
    IndexType* get_bcsr_row_ptr() const { return row_ptr_; }
    IndexType* get_bcsr_col_ind() const { return col_ind_; }
    ValueType* get_bcsr_values() const { return values_; }
    std::shared_ptr<const Executor> get_executor() const { return exec_; }

    void copy_from_host(const IndexType* host_row_ptr, const IndexType* host_col_ind,
                        const ValueType* host_values) {
        exec_->copy_from_host(row_ptr_, host_row_ptr,
                              static_cast<size_t>(num_block_rows_ + 1) * sizeof(IndexType));
        if (num_blocks_ > 0) {
            exec_->copy_from_host(col_ind_, host_col_ind,
                                  static_cast<size_t>(num_blocks_) * sizeof(IndexType));
            exec_->copy_from_host(values_, host_values, value_count() * sizeof(ValueType));
        }
    }

private:
    size_t value_count() const {
        return static_cast<size_t>(num_blocks_) * static_cast<size_t>(r_block_) *
               static_cast<size_t>(c_block_);
    }
    void take(BCSRMatrix& o) noexcept {
        exec_ = std::move(o.exec_);
        num_block_rows_ = o.num_block_rows_;
        num_block_cols_ = o.num_block_cols_;
        num_blocks_ = o.num_blocks_;
        r_block_ = o.r_block_;
        c_block_ = o.c_block_;
        num_rows_ = o.num_rows_;
        num_cols_ = o.num_cols_;
        row_ptr_ = o.row_ptr_;
        col_ind_ = o.col_ind_;
        values_ = o.values_;
        o.row_ptr_ = nullptr;
        o.col_ind_ = nullptr;
        o.values_ = nullptr;
    }
    void release() noexcept {
        if (!exec_) return;
        try {
            if (row_ptr_) exec_->free(row_ptr_);
            if (col_ind_) exec_->free(col_ind_);
            if (values_) exec_->free(values_);
        } catch (...) {
        }
        row_ptr_ = nullptr;
        col_ind_ = nullptr;
        values_ = nullptr;
    }

    std::shared_ptr<const Executor> exec_;
    IndexType num_block_rows_ = 0, num_block_cols_ = 0, num_blocks_ = 0, r_block_ = 0,
              c_block_ = 0, num_rows_ = 0, num_cols_ = 0;
    IndexType* row_ptr_ = nullptr;
    IndexType* col_ind_ = nullptr;
    ValueType* values_ = nullptr;
};

}  // namespace xspmm
