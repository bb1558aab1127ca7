// blockcols.cuh -- warp-level helpers that find the distinct column blocks of a run of CSR/BCSR
// entries with a bitmap window in shared memory (shared by the CSR->BCSR conversion and the
// tensor-core SpMM's group plan).
#pragma once

#include "common.cuh"

namespace xspmm_b200 {

constexpr int WIN_WORDS = 256;                        // bitmap window per warp: 8192 bits
constexpr int64_t WIN_BITS = (int64_t)WIN_WORDS * 32;
constexpr int WORDS_PER_LANE = WIN_WORDS / 32;

// column -> column block, as a shift when the block width is a power of two
struct BlockDiv {
    int shift;    // >= 0 when the block width is a power of two
    int64_t div;  // block width
    __device__ __forceinline__ int64_t operator()(int64_t c) const {
        return shift >= 0 ? (c >> shift) : (c / div);
    }
};

inline BlockDiv make_div(int64_t w) {
    BlockDiv d{-1, w};
    if (w > 0 && (w & (w - 1)) == 0) {
        int s = 0;
        while ((int64_t(1) << s) < w) ++s;
        d.shift = s;
    }
    return d;
}

__device__ __forceinline__ int64_t warp_min64(int64_t v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = min(v, (int64_t)__shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ int64_t warp_max64(int64_t v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = max(v, (int64_t)__shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ int64_t warp_sum64(int64_t v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Column-block range [lo, hi] of entries [e0, e1); flags out-of-range columns. hi < 0 if none.
template <typename IT>
__device__ void block_col_range(const IT* ci, int64_t e0, int64_t e1, int64_t K, BlockDiv bd,
                                int64_t& lo, int64_t& hi, unsigned* err) {
    const int lane = threadIdx.x & 31;
    lo = INT64_MAX;
    hi = -1;
    bool bad = false;
    for (int64_t e = e0 + lane; e < e1; e += 32) {
        const int64_t c = (int64_t)ci[e];
        if (c < 0 || c >= K) {
            bad = true;
            continue;
        }
        const int64_t b = bd(c);
        lo = min(lo, b);
        hi = max(hi, b);
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0 && err) flag_error(err, DERR_COL_OUT_OF_RANGE);
    lo = warp_min64(lo);
    hi = warp_max64(hi);
}

// Marks the column blocks of entries [e0, e1) that fall in [wb, wb + nwords*32) in win.
template <typename IT>
__device__ void mark_window(uint32_t* win, int nwords, const IT* ci, int64_t e0, int64_t e1,
                            int64_t K, BlockDiv bd, int64_t wb) {
    const int lane = threadIdx.x & 31;
    for (int w = lane; w < nwords; w += 32) win[w] = 0u;
    __syncwarp();
    const int64_t span = (int64_t)nwords * 32;
    for (int64_t e = e0 + lane; e < e1; e += 32) {
        const int64_t c = (int64_t)ci[e];
        if (c < 0 || c >= K) continue;
        const int64_t d = bd(c) - wb;
        if (d >= 0 && d < span) atomicOr(&win[d >> 5], 1u << (d & 31));
    }
    __syncwarp();
}

// Exclusive prefix popcount of the window's words (lane owns words [lane*8, lane*8+8)) into pre;
// returns the window's total population (same value in every lane).
__device__ __forceinline__ uint32_t window_prefix(const uint32_t* win, uint32_t* pre, int nwords) {
    const int lane = threadIdx.x & 31;
    uint32_t local[WORDS_PER_LANE];
    uint32_t lsum = 0;
#pragma unroll
    for (int k = 0; k < WORDS_PER_LANE; ++k) {
        const int w = lane * WORDS_PER_LANE + k;
        local[k] = w < nwords ? __popc(win[w]) : 0u;
        lsum += local[k];
    }
    const uint32_t incl = warp_inclusive_sum(lsum);
    uint32_t run = incl - lsum;
#pragma unroll
    for (int k = 0; k < WORDS_PER_LANE; ++k) {
        const int w = lane * WORDS_PER_LANE + k;
        if (w < nwords) pre[w] = run;
        run += local[k];
    }
    __syncwarp();
    return __shfl_sync(0xffffffffu, incl, 31);
}

}  // namespace xspmm_b200
