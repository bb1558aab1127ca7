// xspmm/matrix/csr.hpp -- device-resident CSR matrix.
//
// Same layout, constructor, accessors and copy_from_host as the reference's CSRMatrix
// (include/xspmm/matrix/csr.hpp:15-60): row_ptr[M+1], col_ind[nnz], values[nnz], allocated
// through the executor. Unlike the reference (whose copy constructor is the implicit shallow one,
// csr.hpp:36) it is move-only, so a temporary cannot free buffers another object still uses.
#pragma once

#include <cstdint>
#include <memory>
#include <stdexcept>
#include <utility>

#include "../core/executor.hpp"

namespace xspmm {

template <typename ValueType, typename IndexType = int64_t>
class CSRMatrix {
public:
    CSRMatrix(std::shared_ptr<const Executor> exec, IndexType num_rows, IndexType num_cols,
              IndexType nnz)
        : exec_(std::move(exec)), num_rows_(num_rows), num_cols_(num_cols), nnz_(nnz) {
        if (num_rows < 0 || num_cols < 0 || nnz < 0)
            throw std::invalid_argument("CSR dimensions must be non-negative.");
        exec_->allocate(reinterpret_cast<void**>(&row_ptr_),
                        static_cast<size_t>(num_rows + 1) * sizeof(IndexType));
        if (nnz > 0) {
            exec_->allocate(reinterpret_cast<void**>(&col_ind_), static_cast<size_t>(nnz) * sizeof(IndexType));
            exec_->allocate(reinterpret_cast<void**>(&values_), static_cast<size_t>(nnz) * sizeof(ValueType));
        }
    }
    ~CSRMatrix() { release(); }
    CSRMatrix(const CSRMatrix&) = delete;
    CSRMatrix& operator=(const CSRMatrix&) = delete;
    CSRMatrix(CSRMatrix&& o) noexcept
        : exec_(std::move(o.exec_)), num_rows_(o.num_rows_), num_cols_(o.num_cols_), nnz_(o.nnz_),
          row_ptr_(o.row_ptr_), col_ind_(o.col_ind_), values_(o.values_) {
        o.row_ptr_ = nullptr;
        o.col_ind_ = nullptr;
        o.values_ = nullptr;
    }
    CSRMatrix& operator=(CSRMatrix&& o) noexcept {
        if (this != &o) {
            release();
            exec_ = std::move(o.exec_);
            num_rows_ = o.num_rows_;
            num_cols_ = o.num_cols_;
            nnz_ = o.nnz_;
            row_ptr_ = o.row_ptr_;
            col_ind_ = o.col_ind_;
            values_ = o.values_;
            o.row_ptr_ = nullptr;
            o.col_ind_ = nullptr;
            o.values_ = nullptr;
        }
        return *this;
    }

    IndexType get_num_rows() const { return num_rows_; }
    IndexType get_num_cols() const { return num_cols_; }
    IndexType get_nnz() const { return nnz_; }
    IndexType* get_row_ptr() const { return row_ptr_; }
    IndexType* get_col_ind() const { return col_ind_; }
    ValueType* get_values() const { return values_; }
    std::shared_ptr<const Executor> get_executor() const { return exec_; }

    void copy_from_host(const IndexType* host_row_ptr, const IndexType* host_col_ind,
                        const ValueType* host_values) {
        exec_->copy_from_host(row_ptr_, host_row_ptr, static_cast<size_t>(num_rows_ + 1) * sizeof(IndexType));
        if (nnz_ > 0) {
            exec_->copy_from_host(col_ind_, host_col_ind, static_cast<size_t>(nnz_) * sizeof(IndexType));
            exec_->copy_from_host(values_, host_values, static_cast<size_t>(nnz_) * sizeof(ValueType));
        }
    }

private:
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
    IndexType num_rows_, num_cols_, nnz_;
    IndexType* row_ptr_ = nullptr;
    IndexType* col_ind_ = nullptr;
    ValueType* values_ = nullptr;
};

}  // namespace xspmm
