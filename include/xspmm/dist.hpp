// xspmm/dist.hpp -- one matrix split by block rows over GPUs (xspmm_dist_* in include/xspmm_b200.h).
// The reference runs on one device; its Tier-1 product is independent per block row given B
// (src/common/spmm_math.hpp:68-114), so a caller that wants several GPUs splits the block rows.
// DistPlan does that split inside the library over an NCCL communicator, one process or thread per
// GPU:
//
//   unsigned char id[128];  xspmm::dist_unique_id(id);   // on one rank; hand it to the others
//   xspmm::DistComm comm(exec, nranks, rank, id);          // joins within a time limit
//   xspmm::DistPlan<__half, int32_t> plan(comm, exec, A);  // every rank passes the whole CSR A
//   plan.execute(d_B, d_C_local, N, /*bcast_root=*/0);     // B broadcast from rank 0, then
//                                                          //   this rank's rows of C
//   plan.gather(d_C_local, d_C, N, /*root=*/0);            // C on rank 0, caller's row order
//
// A rank that never joins or stops makes the others' calls throw (TIMEOUT) instead of hanging.
#pragma once

#include <cstdint>
#include <memory>
#include <stdexcept>
#include <type_traits>

#include "core/executor.hpp"
#include "detail/abi.hpp"
#include "matrix/csr.hpp"

namespace xspmm {

inline void dist_unique_id(unsigned char (&id)[128]) {
    detail::check(xspmm_dist_unique_id(id, 128));
}

class DistComm {
public:
    DistComm(std::shared_ptr<const Executor> exec, int nranks, int rank, const unsigned char* id,
             int timeout_ms = 60000)
        : exec_(std::move(exec)) {
        detail::check(xspmm_dist_comm_init(detail::handle_of(exec_), nranks, rank, id, 128,
                                           timeout_ms, &c_));
    }
    DistComm(const DistComm&) = delete;
    DistComm& operator=(const DistComm&) = delete;
    ~DistComm() {
        if (c_) xspmm_dist_comm_destroy(c_);
    }
    xspmm_dist_comm_t get() const { return c_; }

private:
    std::shared_ptr<const Executor> exec_;
    xspmm_dist_comm_t c_ = nullptr;
};

template <typename ValueType, typename IndexType = int64_t>
class DistPlan {
public:
    DistPlan(const DistComm& comm, std::shared_ptr<const Executor> exec,
             const CSRMatrix<ValueType, IndexType>& A, IndexType hw_block_size = 16,
             bool optimize_pattern = true, double row_weight = 0.0)
        : exec_(std::move(exec)) {
        detail::check(detail::Abi<ValueType, IndexType>::dist_plan_csr(
            detail::handle_of(exec_), comm.get(), A.get_num_rows(), A.get_num_cols(),
            A.get_nnz(), A.get_row_ptr(), A.get_col_ind(), A.get_values(), hw_block_size,
            optimize_pattern ? 1 : 0, row_weight, &p_));
    }
    DistPlan(const DistPlan&) = delete;
    DistPlan& operator=(const DistPlan&) = delete;
    ~DistPlan() {
        if (p_) xspmm_dist_plan_destroy(p_);
    }

    xspmm_dist_plan_info_t info() const {
        xspmm_dist_plan_info_t i{};
        detail::check(xspmm_dist_plan_get_info(p_, &i));
        return i;
    }
    // C_local (this rank's rows of the clustered matrix x N, fp32) = those rows of A * B.
    void execute(ValueType* B, float* C_local, IndexType N, int bcast_root = -1,
                 int timeout_ms = 60000) const {
        detail::check(xspmm_dist_plan_execute(p_, B, C_local, (int64_t)N, bcast_root, timeout_ms));
    }
    // C (M x N, fp32, the caller's row order) on `root`; other ranks may pass C = nullptr.
    void gather(const float* C_local, float* C, IndexType N, int root = 0,
                int timeout_ms = 60000) const {
        detail::check(xspmm_dist_gather(p_, C_local, C, (int64_t)N, root, timeout_ms));
    }

private:
    std::shared_ptr<const Executor> exec_;
    xspmm_dist_plan_t p_ = nullptr;
};

}  // namespace xspmm
