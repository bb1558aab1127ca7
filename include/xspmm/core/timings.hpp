// xspmm/core/timings.hpp -- per-stage times of the Tier-2 pipeline.
// Same fields and meaning as the reference's SpMMTimings (include/xspmm/core/timings.hpp:7-14):
// milliseconds of device time measured with CUDA events. unpermutation_ms is 0 here because the
// unpermute is fused into the SpMM store.
#pragma once

namespace xspmm {

struct SpMMTimings {
    double clustering_ms = 0.0;
    double permutation_ms = 0.0;
    double conversion_ms = 0.0;
    double spmm_ms = 0.0;
    double unpermutation_ms = 0.0;
    double total_pipeline_ms = 0.0;
};

}  // namespace xspmm
