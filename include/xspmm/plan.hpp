// xspmm/plan.hpp -- SpMMPlan: the Tier-2 stages (clustering, permutation, CSR->BCSR) done once for
// repeated products with the same A. The reference has no such object: its Tier-2 spmm
// (include/xspmm/xspmm.hpp:24-32) redoes every stage per call, and its README.md:127 points
// callers who multiply one A many times to Tier 1 for "amortizing clustering time over thousands
// of iterations". A plan is that amortization inside the library (xspmm_plan_* in
// include/xspmm_b200.h):
//
//   xspmm::SpMMPlan<__half, int32_t> plan(exec, A, /*hw_block_size=*/16, /*optimize=*/true, &t);
//   for (...) plan.execute(d_B, d_C, N);   // C = A * B, C's rows in A's order
//
// A plan built from a BCSRMatrix reads that matrix's arrays at every product: keep it alive.
// Destroy plans before their executor (the executor's handle refuses to go while plans exist).
#pragma once

#include <memory>
#include <stdexcept>
#include <type_traits>

#include "core/executor.hpp"
#include "core/timings.hpp"
#include "detail/abi.hpp"
#include "matrix/bcsr.hpp"
#include "matrix/csr.hpp"

namespace xspmm {

template <typename ValueType, typename IndexType = int64_t>
class SpMMPlan {
public:
    SpMMPlan(std::shared_ptr<const Executor> exec, const CSRMatrix<ValueType, IndexType>& A,
             IndexType hw_block_size = 16, bool optimize_pattern = true,
             SpMMTimings* build_timings = nullptr)
        : exec_(std::move(exec)) {
        xspmm_timings_t t{};
        detail::check(detail::Abi<ValueType, IndexType>::plan_csr(
            detail::handle_of(exec_), A.get_num_rows(), A.get_num_cols(), A.get_nnz(),
            A.get_row_ptr(), A.get_col_ind(), A.get_values(), hw_block_size,
            optimize_pattern ? 1 : 0, &plan_, build_timings ? &t : nullptr));
        if (build_timings) {
            build_timings->clustering_ms = t.clustering_ms;
            build_timings->permutation_ms = t.permutation_ms;
            build_timings->conversion_ms = t.conversion_ms;
            build_timings->spmm_ms = t.spmm_ms;
            build_timings->unpermutation_ms = t.unpermutation_ms;
            build_timings->total_pipeline_ms = t.total_pipeline_ms;
        }
    }

    explicit SpMMPlan(const BCSRMatrix<ValueType, IndexType>& A) : exec_(A.get_executor()) {
        detail::check(detail::Abi<ValueType, IndexType>::plan_bcsr(
            detail::handle_of(exec_), A.get_num_block_rows(), A.get_num_block_cols(),
            A.get_num_blocks(), A.get_r_block(), A.get_c_block(), A.get_bcsr_row_ptr(),
            A.get_bcsr_col_ind(), A.get_bcsr_values(), A.get_num_rows(), A.get_num_cols(),
            &plan_));
    }

    SpMMPlan(const SpMMPlan&) = delete;
    SpMMPlan& operator=(const SpMMPlan&) = delete;
    SpMMPlan(SpMMPlan&& o) noexcept : exec_(std::move(o.exec_)), plan_(o.plan_) { o.plan_ = nullptr; }
    SpMMPlan& operator=(SpMMPlan&& o) noexcept {
        if (this != &o) {
            reset();
            exec_ = std::move(o.exec_);
            plan_ = o.plan_;
            o.plan_ = nullptr;
        }
        return *this;
    }
    ~SpMMPlan() { reset(); }

    // C (M x N, fp32) = A * B (K x N), rows of C in A's original order. Asynchronous.
    template <typename OutputType>
    void execute(const ValueType* B, OutputType* C, IndexType N) const {
        static_assert(std::is_same<OutputType, float>::value, "C is float");
        detail::check(xspmm_plan_execute(plan_, B, C, (int64_t)N));
    }

    xspmm_plan_info_t info() const {
        xspmm_plan_info_t i{};
        detail::check(xspmm_plan_get_info(plan_, &i));
        return i;
    }

private:
    void reset() noexcept {
        if (plan_) xspmm_plan_destroy(plan_);
        plan_ = nullptr;
    }
    std::shared_ptr<const Executor> exec_;
    xspmm_plan_t plan_ = nullptr;
};

}  // namespace xspmm
