// xspmm/detail/abi.hpp -- compile-time mapping of the reference's (ValueType, IndexType)
// template arguments onto the typed entry points of the C ABI (include/xspmm_b200.h).
#pragma once

#include <cstdint>
#include <type_traits>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "../../xspmm_b200.h"

namespace xspmm {
namespace detail {

template <typename V, typename I>
struct Abi;

#define XSPMM_ABI_ROW(V, I, VS, IS)                                                                \
    template <>                                                                                    \
    struct Abi<V, I> {                                                                             \
        static constexpr auto spmm = xspmm_bcsr_spmm_##VS##f32_##IS;                               \
        static constexpr auto pipeline = xspmm_spmm_csr_##VS##f32_##IS;                            \
        static constexpr auto cluster = xspmm_cluster_jaccard_##IS;                                \
        static constexpr auto permute = xspmm_permute_rows_##VS##_##IS;                            \
        static constexpr auto count = xspmm_csr_to_bcsr_count_##IS;                                \
        static constexpr auto fill = xspmm_csr_to_bcsr_fill_##VS##_##IS;                           \
        static constexpr auto unpermute = xspmm_unpermute_dense_##VS##_##IS;                       \
        static constexpr auto plan_csr = xspmm_plan_csr_##VS##f32_##IS;                            \
        static constexpr auto plan_bcsr = xspmm_plan_bcsr_##VS##f32_##IS;                          \
        static constexpr auto dist_plan_csr = xspmm_dist_plan_csr_##VS##f32_##IS;                  \
    };
XSPMM_ABI_ROW(__half, int32_t, f16, i32)
XSPMM_ABI_ROW(__half, int64_t, f16, i64)
XSPMM_ABI_ROW(__nv_bfloat16, int32_t, bf16, i32)
XSPMM_ABI_ROW(__nv_bfloat16, int64_t, bf16, i64)
XSPMM_ABI_ROW(float, int32_t, f32, i32)
XSPMM_ABI_ROW(float, int64_t, f32, i64)
#undef XSPMM_ABI_ROW

}  // namespace detail
}  // namespace xspmm
