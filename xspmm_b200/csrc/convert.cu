// convert.cu -- CSR -> BCSR on the device.
//
// Reproduces src/core/conversion.cpp:8-100 bit for bit:
//   * block row br covers rows [br*rb, min(M, br*rb+rb)); its blocks are the distinct column
//     blocks floor(col/cb) of those rows, sorted ascending (conversion.cpp:42-64);
//   * row_ptr is the running count (:66-68);
//   * values are zero-filled, then every CSR entry is stored at
//     (row_ptr[br] + rank(bc))*rb*cb + (r % rb)*cb + col % cb, in CSR order, so a duplicated
//     (row, col) keeps its last value (:75-91). Explicit zeros still create blocks.
//
// Design: one warp per block row. The warp marks the block columns of its rows in a bitmap window
// of 8192 bits held in shared memory (atomicOr), so the sorted distinct list falls out of the bit
// order: count = sum of popc over the window, and an entry's rank = the prefix popcount up to its
// bit. Ranges wider than a window take several passes. The count kernel writes per-block-row
// counts (scanned on the device into row_ptr); the fill kernel rebuilds the bitmap, writes the
// column indices and scatters values. Rows whose columns are strictly increasing (no duplicates)
// scatter in parallel across lanes -- distinct rows never share a destination; any other row is
// written by one lane in CSR order so the last duplicate wins, as in the reference.
#include "ops.cuh"
#include "blockcols.cuh"

#include <algorithm>

namespace xspmm_b200 {
namespace {

constexpr int CV_WARPS = 8;
constexpr int64_t CV_LONG = 4096;  // entries above which a block row gets a CTA of its own

// Validates row_ptr over [r0, r1]; returns false (and flags) when it is malformed.
template <typename IT>
__device__ bool rows_ok(const IT* rp, int64_t r0, int64_t r1, int64_t nnz, unsigned* err) {
    const int lane = threadIdx.x & 31;
    bool bad = false;
    for (int64_t r = r0 + lane; r < r1; r += 32) {
        const int64_t a = (int64_t)rp[r], b = (int64_t)rp[r + 1];
        if (a < 0 || a > b || b > nnz) bad = true;
    }
    if (__any_sync(0xffffffffu, bad)) {
        if (lane == 0 && err) flag_error(err, DERR_ROW_PTR);
        return false;
    }
    return true;
}

template <typename IT>
__global__ void __launch_bounds__(CV_WARPS * 32)
bcsr_count_kernel(const IT* __restrict__ rp, const IT* __restrict__ ci, int64_t M, int64_t K,
                  int64_t nnz, int64_t nbr, int64_t rb, BlockDiv bd, IT* __restrict__ counts,
                  int64_t* __restrict__ long_list, unsigned* __restrict__ long_n,
                  unsigned long_cap, unsigned* err) {
    __shared__ uint32_t win_all[CV_WARPS][WIN_WORDS];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t* win = win_all[warp];
    for (int64_t br = (int64_t)blockIdx.x * CV_WARPS + warp; br < nbr;
         br += (int64_t)gridDim.x * CV_WARPS) {
        const int64_t r0 = br * rb, r1 = min(M, r0 + rb);
        if (!rows_ok(rp, r0, r1, nnz, err)) {
            if (lane == 0) counts[br] = 0;
            continue;
        }
        const int64_t e0 = rp[r0], e1 = rp[r1];
        if (long_list && e1 - e0 > CV_LONG) {  // a CTA of its own counts it (below)
            if (lane == 0) {
                const unsigned k = atomicAdd(long_n, 1u);
                if (k < long_cap) long_list[k] = br;
                else flag_error(err, DERR_INTERNAL);
            }
            continue;
        }
        int64_t lo, hi;
        block_col_range(ci, e0, e1, K, bd, lo, hi, err);
        int64_t count = 0;
        for (int64_t wb = lo; wb <= hi; wb += WIN_BITS) {
            const int nwords = (int)min((int64_t)WIN_WORDS, (hi - wb) / 32 + 1);
            mark_window(win, nwords, ci, e0, e1, K, bd, wb);
            int64_t c = 0;
            for (int w = lane; w < nwords; w += 32) c += __popc(win[w]);
            count += warp_sum64(c);
            __syncwarp();
        }
        if (lane == 0) counts[br] = (IT)count;
    }
}

template <typename VT, typename IT>
__global__ void __launch_bounds__(CV_WARPS * 32)
bcsr_fill_kernel(const IT* __restrict__ rp, const IT* __restrict__ ci, const VT* __restrict__ v,
                 int64_t M, int64_t K, int64_t nbr, int64_t rb, int64_t cb, BlockDiv bd,
                 const IT* __restrict__ brp, IT* __restrict__ bci, VT* __restrict__ bvals,
                 int64_t* __restrict__ long_list, unsigned* __restrict__ long_n,
                 unsigned long_cap) {
    __shared__ uint32_t win_all[CV_WARPS][WIN_WORDS];
    __shared__ uint32_t pre_all[CV_WARPS][WIN_WORDS];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t* win = win_all[warp];
    uint32_t* pre = pre_all[warp];
    const int64_t bsz = rb * cb;
    for (int64_t br = (int64_t)blockIdx.x * CV_WARPS + warp; br < nbr;
         br += (int64_t)gridDim.x * CV_WARPS) {
        const int64_t base = brp[br], nb = (int64_t)brp[br + 1] - base;
        if (nb <= 0) continue;
        const int64_t r0 = br * rb, r1 = min(M, r0 + rb);
        const int64_t e0 = rp[r0], e1 = rp[r1];
        if (long_list && e1 - e0 > CV_LONG) {  // filled by bcsr_fill_long_kernel (below)
            if (lane == 0) {
                const unsigned k = atomicAdd(long_n, 1u);
                if (k < long_cap) long_list[k] = br;
            }
            continue;
        }
        if (bvals) {  // zero the block row's blocks
            VT* z = bvals + base * bsz;
            const int64_t n = nb * bsz;
            const int64_t bytes = n * (int64_t)sizeof(VT);
            if (reinterpret_cast<uintptr_t>(z) % 16 == 0 && bytes % 16 == 0) {
                uint4* z4 = reinterpret_cast<uint4*>(z);
                for (int64_t t = lane; t < bytes / 16; t += 32) z4[t] = make_uint4(0, 0, 0, 0);
            } else {
                for (int64_t t = lane; t < n; t += 32) z[t] = VT(0.0f);
            }
            __syncwarp();
        }
        int64_t lo, hi;
        block_col_range(ci, e0, e1, K, bd, lo, hi, nullptr);
        int64_t rank_base = 0;
        for (int64_t wb = lo; wb <= hi; wb += WIN_BITS) {
            const int nwords = (int)min((int64_t)WIN_WORDS, (hi - wb) / 32 + 1);
            mark_window(win, nwords, ci, e0, e1, K, bd, wb);
            // exclusive prefix popcount per word; lane owns words [lane*8, lane*8+8)
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
                if (w < nwords) {
                    pre[w] = run;
                    // column indices of this word's blocks, ascending
                    uint32_t x = win[w];
                    int64_t o = base + rank_base + run;
                    while (x) {
                        const int b = __ffs(x) - 1;
                        bci[o++] = (IT)(wb + (int64_t)w * 32 + b);
                        x &= x - 1;
                    }
                }
                run += local[k];
            }
            const uint32_t wtotal = __shfl_sync(0xffffffffu, incl, 31);
            __syncwarp();
            if (bvals) {
                for (int64_t r = r0; r < r1; ++r) {
                    const int64_t s = rp[r], t = rp[r + 1];
                    bool unsorted = false;
                    for (int64_t e = s + lane; e + 1 < t; e += 32)
                        if (ci[e] >= ci[e + 1]) unsorted = true;
                    unsorted = __any_sync(0xffffffffu, unsorted);
                    const int64_t roff = (r - r0) * cb;
                    auto put = [&](int64_t e) {
                        const int64_t c = (int64_t)ci[e];
                        if (c < 0 || c >= K) return;
                        const int64_t b = bd(c);
                        const int64_t d = b - wb;
                        if (d < 0 || d >= (int64_t)nwords * 32) return;
                        const uint32_t word = win[d >> 5];
                        const int64_t rank =
                            rank_base + pre[d >> 5] + __popc(word & ((1u << (d & 31)) - 1u));
                        bvals[(base + rank) * bsz + roff + (c - b * cb)] = v[e];
                    };
                    if (!unsorted) {
                        for (int64_t e = s + lane; e < t; e += 32) put(e);
                    } else if (lane == 0) {
                        for (int64_t e = s; e < t; ++e) put(e);
                    }
                }
            }
            rank_base += wtotal;
            __syncwarp();
        }
    }
}

// The same fill with the blocks assembled in shared memory (block rows of at most 32 rows): the
// kernel above zeroes a block row's blocks in global memory and then scatters 2- or 4-byte values
// into them, one row at a time (a chain of dependent loads per row, and partial sector writes
// that reach L2 after the zero fill). Here a warp takes all entries of the block row at once
// (lane-strided over the contiguous range; an entry's row is found by a search over the row ends
// the lanes hold), assembles up to CV_ASM_BYTES of blocks in shared memory (zeroed, values
// scattered, the last duplicate of a row whose columns are not strictly increasing winning as
// in the reference) and writes them once with 16-byte stores.
constexpr int CV_ASM_BYTES = 4096;  // per warp

template <typename VT, typename IT>
__global__ void __launch_bounds__(CV_WARPS * 32)
bcsr_fill_asm_kernel(const IT* __restrict__ rp, const IT* __restrict__ ci, const VT* __restrict__ v,
                     int64_t M, int64_t K, int64_t nbr, int64_t rb, int64_t cb, BlockDiv bd,
                     const IT* __restrict__ brp, IT* __restrict__ bci, VT* __restrict__ bvals,
                     int64_t* __restrict__ long_list, unsigned* __restrict__ long_n,
                     unsigned long_cap) {
    __shared__ uint32_t win_all[CV_WARPS][WIN_WORDS];
    __shared__ uint32_t pre_all[CV_WARPS][WIN_WORDS];
    __shared__ __align__(16) uint8_t asm_all[CV_WARPS][CV_ASM_BYTES];
    const unsigned FULL = 0xffffffffu;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t* win = win_all[warp];
    uint32_t* pre = pre_all[warp];
    VT* sv = reinterpret_cast<VT*>(asm_all[warp]);
    const int64_t bsz = rb * cb;
    const int sb = (int)(CV_ASM_BYTES / (bsz * (int64_t)sizeof(VT)));  // blocks per round (>= 1)
    for (int64_t br = (int64_t)blockIdx.x * CV_WARPS + warp; br < nbr;
         br += (int64_t)gridDim.x * CV_WARPS) {
        const int64_t base = brp[br], nb = (int64_t)brp[br + 1] - base;
        if (nb <= 0) continue;
        const int64_t r0 = br * rb, r1 = min(M, r0 + rb);
        const int nrows = (int)(r1 - r0);  // <= 32
        const int64_t e0 = rp[r0], e1 = rp[r1];
        if (long_list && e1 - e0 > CV_LONG) {  // filled by bcsr_fill_long_kernel
            if (lane == 0) {
                const unsigned k = atomicAdd(long_n, 1u);
                if (k < long_cap) long_list[k] = br;
            }
            continue;
        }
        // lane j holds the end of row r0 + j (past the block row: no end)
        const int64_t rend = lane < nrows ? (int64_t)rp[r0 + lane + 1] : INT64_MAX;
        auto row_of = [&](int64_t e) {  // rows whose end is <= e, i.e. the row holding e
            int j = 0;
#pragma unroll
            for (int step = 16; step >= 1; step >>= 1)
                if (__shfl_sync(FULL, rend, j + step - 1) <= e) j += step;
            return j;
        };
        // rows whose columns are not strictly increasing
        uint32_t unsorted = 0;
        for (int64_t b0 = e0; b0 < e1; b0 += 32) {
            const int64_t e = b0 + lane;
            const int j = row_of(e < e1 ? e : e1 - 1);
            const int64_t end = __shfl_sync(FULL, rend, j);
            if (e < e1 && e + 1 < end && ci[e] >= ci[e + 1]) unsorted |= 1u << j;
        }
        unsorted = __reduce_or_sync(FULL, unsorted);
        int64_t lo, hi;
        block_col_range(ci, e0, e1, K, bd, lo, hi, nullptr);
        int64_t rank_base = 0;
        for (int64_t wb = lo; wb <= hi; wb += WIN_BITS) {
            const int nwords = (int)min((int64_t)WIN_WORDS, (hi - wb) / 32 + 1);
            mark_window(win, nwords, ci, e0, e1, K, bd, wb);
            const uint32_t wtotal = window_prefix(win, pre, nwords);
            for (int w = lane; w < nwords; w += 32) {  // column indices of the window's blocks
                uint32_t x = win[w];
                int64_t o = base + rank_base + pre[w];
                while (x) {
                    const int b = __ffs(x) - 1;
                    bci[o++] = (IT)(wb + (int64_t)w * 32 + b);
                    x &= x - 1;
                }
            }
            // Windows of more than two buffers of blocks (block rows of scattered columns, e.g.
            // R-MAT's) are zero-filled and scattered in global memory in one pass instead of being
            // assembled a buffer at a time (a pass over the entries per buffer).
            const bool direct = (int)wtotal > 2 * sb;
            const int step = direct ? (int)wtotal : sb;
            for (int k0 = 0; k0 < (int)wtotal; k0 += step) {
                const int kn = min(step, (int)wtotal - k0);
                const int64_t bytes = (int64_t)kn * bsz * (int64_t)sizeof(VT);
                VT* gdst = bvals + (base + rank_base + k0) * bsz;
                VT* tgt = direct ? gdst : sv;
                const bool vec = reinterpret_cast<uintptr_t>(gdst) % 16 == 0 && bytes % 16 == 0;
                uint4* s4 = reinterpret_cast<uint4*>(asm_all[warp]);
                if (!direct) {
                    for (int64_t q = lane; q < (bytes + 15) / 16; q += 32) s4[q] = make_uint4(0, 0, 0, 0);
                } else if (vec) {
                    uint4* d4 = reinterpret_cast<uint4*>(gdst);
                    for (int64_t q = lane; q < bytes / 16; q += 32) d4[q] = make_uint4(0, 0, 0, 0);
                } else {
                    for (int64_t q = lane; q < (int64_t)kn * bsz; q += 32) gdst[q] = VT(0.0f);
                }
                __syncwarp();
                auto put = [&](int64_t e, int j) {
                    const int64_t c = (int64_t)ci[e];
                    if (c < 0 || c >= K) return;
                    const int64_t b = bd(c);
                    const int64_t d = b - wb;
                    if (d < 0 || d >= (int64_t)nwords * 32) return;
                    const int rank = (int)(pre[d >> 5] + __popc(win[d >> 5] & ((1u << (d & 31)) - 1u)));
                    if (rank < k0 || rank >= k0 + kn) return;
                    tgt[(int64_t)(rank - k0) * bsz + (int64_t)j * cb + (c - b * cb)] = v[e];
                };
                for (int64_t b0 = e0; b0 < e1; b0 += 32) {
                    const int64_t e = b0 + lane;
                    const int j = row_of(e < e1 ? e : e1 - 1);
                    if (e < e1 && !((unsorted >> j) & 1u)) put(e, j);
                }
                if (unsorted) {  // those rows by one lane, in CSR order: the last duplicate wins
                    for (int j = 0; j < nrows; ++j) {
                        if (!((unsorted >> j) & 1u)) continue;
                        const int64_t prev = __shfl_sync(FULL, rend, j > 0 ? j - 1 : 0);
                        const int64_t s = j == 0 ? e0 : prev;
                        const int64_t t = __shfl_sync(FULL, rend, j);
                        if (lane == 0)
                            for (int64_t e = s; e < t; ++e) put(e, j);
                    }
                }
                __syncwarp();
                if (!direct) {
                    if (vec) {
                        uint4* d4 = reinterpret_cast<uint4*>(gdst);
                        for (int64_t q = lane; q < bytes / 16; q += 32) d4[q] = s4[q];
                    } else {
                        for (int64_t q = lane; q < (int64_t)kn * bsz; q += 32) gdst[q] = sv[q];
                    }
                }
                __syncwarp();
            }
            rank_base += wtotal;
            __syncwarp();
        }
    }
}

// ---- block rows with more than CV_LONG entries: one CTA each ---------------------------------
// A warp walking tens of thousands of entries (a dense row, the hub rows of a power-law graph,
// the 16 x 688-block rows of the pruned-LLM config) would serialize the launch; these rows are
// listed by the count kernel and done by a whole CTA: the window is marked by all threads, its
// prefix popcount is a CTA scan, and the value scatter gives each warp its own rows.
constexpr int CL_T = CV_WARPS * 32;

__device__ __forceinline__ int64_t cta_reduce_min(int64_t v, int64_t* red) {
    v = warp_min64(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    int64_t r = red[0];
    for (int w = 1; w < CV_WARPS; ++w) r = min(r, red[w]);
    __syncthreads();
    return r;
}
__device__ __forceinline__ int64_t cta_reduce_max(int64_t v, int64_t* red) {
    v = warp_max64(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    int64_t r = red[0];
    for (int w = 1; w < CV_WARPS; ++w) r = max(r, red[w]);
    __syncthreads();
    return r;
}

// Column-block range of [e0, e1) over the CTA (hi < 0 if empty).
template <typename IT>
__device__ void cta_col_range(const IT* ci, int64_t e0, int64_t e1, int64_t K, BlockDiv bd,
                              int64_t* red, int64_t& lo, int64_t& hi) {
    int64_t l = INT64_MAX, h = -1;
    for (int64_t e = e0 + threadIdx.x; e < e1; e += CL_T) {
        const int64_t c = (int64_t)ci[e];
        if (c < 0 || c >= K) continue;
        const int64_t b = bd(c);
        l = min(l, b);
        h = max(h, b);
    }
    lo = cta_reduce_min(l, red);
    hi = cta_reduce_max(h, red);
}

// Marks [wb, wb + WIN_BITS) over the CTA; returns this thread's word population (thread t owns
// word t) with the exclusive prefix in *pre_out and the window total in *tot_out.
template <typename IT>
__device__ void cta_mark(uint32_t* win, const IT* ci, int64_t e0, int64_t e1, int64_t K,
                         BlockDiv bd, int64_t wb, uint32_t* s_warp, uint32_t* pre_out,
                         uint32_t* tot_out) {
    static_assert(CL_T == WIN_WORDS, "one window word per thread");
    win[threadIdx.x] = 0u;
    __syncthreads();
    for (int64_t e = e0 + threadIdx.x; e < e1; e += CL_T) {
        const int64_t c = (int64_t)ci[e];
        if (c < 0 || c >= K) continue;
        const int64_t d = bd(c) - wb;
        if (d >= 0 && d < WIN_BITS) atomicOr(&win[d >> 5], 1u << (d & 31));
    }
    __syncthreads();
    const uint32_t pc = __popc(win[threadIdx.x]);
    const uint32_t inc = warp_inclusive_sum(pc);
    if ((threadIdx.x & 31) == 31) s_warp[threadIdx.x >> 5] = inc;
    __syncthreads();
    uint32_t off = 0, tot = 0;
    for (int w = 0; w < CV_WARPS; ++w) {
        if (w < (int)(threadIdx.x >> 5)) off += s_warp[w];
        tot += s_warp[w];
    }
    *pre_out = off + inc - pc;
    *tot_out = tot;
}

template <typename IT>
__global__ void __launch_bounds__(CL_T)
bcsr_count_long_kernel(const IT* __restrict__ rp, const IT* __restrict__ ci, int64_t M, int64_t K,
                       int64_t rb, BlockDiv bd, const int64_t* __restrict__ long_list,
                       const unsigned* __restrict__ long_n, IT* __restrict__ counts) {
    __shared__ uint32_t win[WIN_WORDS];
    __shared__ uint32_t s_warp[CV_WARPS];
    __shared__ int64_t red[CV_WARPS];
    const unsigned n = *long_n;
    for (unsigned i = blockIdx.x; i < n; i += gridDim.x) {
        const int64_t br = long_list[i];
        const int64_t r0 = br * rb, r1 = min(M, r0 + rb);
        const int64_t e0 = rp[r0], e1 = rp[r1];
        int64_t lo, hi;
        cta_col_range(ci, e0, e1, K, bd, red, lo, hi);
        int64_t count = 0;
        for (int64_t wb = lo; wb <= hi; wb += WIN_BITS) {
            uint32_t pre, tot;
            cta_mark(win, ci, e0, e1, K, bd, wb, s_warp, &pre, &tot);
            count += tot;
            __syncthreads();
        }
        if (threadIdx.x == 0) counts[br] = (IT)count;
    }
}

template <typename VT, typename IT>
__global__ void __launch_bounds__(CL_T)
bcsr_fill_long_kernel(const IT* __restrict__ rp, const IT* __restrict__ ci,
                      const VT* __restrict__ v, int64_t M, int64_t K, int64_t rb, int64_t cb,
                      BlockDiv bd, const IT* __restrict__ brp, IT* __restrict__ bci,
                      VT* __restrict__ bvals, const int64_t* __restrict__ long_list,
                      const unsigned* __restrict__ long_n) {
    __shared__ uint32_t win[WIN_WORDS];
    __shared__ uint32_t pre_s[WIN_WORDS];
    __shared__ uint32_t s_warp[CV_WARPS];
    __shared__ int64_t red[CV_WARPS];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t bsz = rb * cb;
    const unsigned n = *long_n;
    for (unsigned i = blockIdx.x; i < n; i += gridDim.x) {
        const int64_t br = long_list[i];
        const int64_t base = brp[br], nb = (int64_t)brp[br + 1] - base;
        const int64_t r0 = br * rb, r1 = min(M, r0 + rb);
        const int64_t e0 = rp[r0], e1 = rp[r1];
        if (bvals && nb > 0) {  // zero the block row's blocks
            VT* z = bvals + base * bsz;
            const int64_t cnt = nb * bsz;
            const int64_t bytes = cnt * (int64_t)sizeof(VT);
            if (reinterpret_cast<uintptr_t>(z) % 16 == 0 && bytes % 16 == 0) {
                uint4* z4 = reinterpret_cast<uint4*>(z);
                for (int64_t t = threadIdx.x; t < bytes / 16; t += CL_T) z4[t] = make_uint4(0, 0, 0, 0);
            } else {
                for (int64_t t = threadIdx.x; t < cnt; t += CL_T) z[t] = VT(0.0f);
            }
        }
        __syncthreads();
        int64_t lo, hi;
        cta_col_range(ci, e0, e1, K, bd, red, lo, hi);
        int64_t rank_base = 0;
        for (int64_t wb = lo; wb <= hi; wb += WIN_BITS) {
            uint32_t pre, tot;
            cta_mark(win, ci, e0, e1, K, bd, wb, s_warp, &pre, &tot);
            pre_s[threadIdx.x] = pre;
            {
                uint32_t x = win[threadIdx.x];
                int64_t o = base + rank_base + pre;
                while (x) {
                    const int b = __ffs(x) - 1;
                    bci[o++] = (IT)(wb + (int64_t)threadIdx.x * 32 + b);
                    x &= x - 1;
                }
            }
            __syncthreads();
            if (bvals) {
                // warp w scatters rows r0 + w, r0 + w + WARPS, ...: distinct rows never share a
                // destination; a row whose columns are not strictly increasing is written by one
                // lane in CSR order, so its last duplicate wins
                for (int64_t r = r0 + warp; r < r1; r += CV_WARPS) {
                    const int64_t s0 = rp[r], t0 = rp[r + 1];
                    bool unsorted = false;
                    for (int64_t e = s0 + lane; e + 1 < t0; e += 32)
                        if (ci[e] >= ci[e + 1]) unsorted = true;
                    unsorted = __any_sync(0xffffffffu, unsorted);
                    const int64_t roff = (r - r0) * cb;
                    auto put = [&](int64_t e) {
                        const int64_t c = (int64_t)ci[e];
                        if (c < 0 || c >= K) return;
                        const int64_t b = bd(c);
                        const int64_t d = b - wb;
                        if (d < 0 || d >= WIN_BITS) return;
                        const uint32_t word = win[d >> 5];
                        const int64_t rank =
                            rank_base + pre_s[d >> 5] + __popc(word & ((1u << (d & 31)) - 1u));
                        bvals[(base + rank) * bsz + roff + (c - b * cb)] = v[e];
                    };
                    if (!unsorted) {
                        for (int64_t e = s0 + lane; e < t0; e += 32) put(e);
                    } else if (lane == 0) {
                        for (int64_t e = s0; e < t0; ++e) put(e);
                    }
                }
            }
            rank_base += tot;
            __syncthreads();
        }
    }
}

unsigned cv_grid(Handle& h, int64_t nbr) {
    const int64_t want = ceil_div(nbr, CV_WARPS);
    const int64_t cap = (int64_t)sm_count(h.device) * 32;
    return (unsigned)std::max<int64_t>(1, std::min(want, cap));
}

// CTAs for the long block rows: at most one per listed row, at most 4 per SM (a grid-stride loop
// over the device-side list, whose length the host does not read)
unsigned cl_grid(Handle& h, int64_t cap) {
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>(cap, (int64_t)sm_count(h.device) * 4));
}

}  // namespace

template <typename IT>
int64_t csr_to_bcsr_count(Handle& h, int64_t M, int64_t K, int64_t nnz, const IT* row_ptr,
                          const IT* col_ind, int64_t rb, int64_t cb, IT* brp) {
    const int64_t nbr = ceil_div(M, rb);
    if (nbr == 0) {
        XS_CHECK_CUDA(cudaMemsetAsync(brp, 0, sizeof(IT), h.stream));
        return 0;
    }
    // block rows above CV_LONG entries are listed by the warp kernel and counted by CTAs
    const bool may_be_long = nnz > CV_LONG;
    const int64_t cap = std::max<int64_t>(1, std::min<int64_t>(nbr, nnz / CV_LONG + 1));
    DevBuf<int64_t> long_list(may_be_long ? cap : 0, h.stream);
    DevBuf<unsigned> long_n(may_be_long ? 1 : 0, h.stream);
    if (may_be_long) XS_CHECK_CUDA(cudaMemsetAsync(long_n.get(), 0, sizeof(unsigned), h.stream));
    bcsr_count_kernel<IT><<<cv_grid(h, nbr), CV_WARPS * 32, 0, h.stream>>>(
        row_ptr, col_ind, M, K, nnz, nbr, rb, make_div(cb), brp, long_list.get(), long_n.get(),
        (unsigned)cap, h.d_err);
    after_launch(h, "bcsr_count");
    if (may_be_long) {
        bcsr_count_long_kernel<IT><<<cl_grid(h, cap), CL_T, 0, h.stream>>>(
            row_ptr, col_ind, M, K, rb, make_div(cb), long_list.get(), long_n.get(), brp);
        after_launch(h, "bcsr_count_long");
    }
    exclusive_scan<IT>(h, brp, brp, nbr);
    throw_on_device_errors(h, "csr_to_bcsr");
    return (int64_t)read_scalar<IT>(h, brp + nbr);
}

template <typename VT, typename IT>
void csr_to_bcsr_fill(Handle& h, int64_t M, int64_t K, int64_t nnz, const IT* row_ptr,
                      const IT* col_ind, const VT* values, int64_t rb, int64_t cb, const IT* brp,
                      IT* bci, VT* bvals) {
    const int64_t nbr = ceil_div(M, rb);
    if (nbr == 0) return;
    // block rows above CV_LONG entries (the same ones the count listed; row_ptr was validated
    // there) are listed by the warp kernel and filled by CTAs
    const bool may_be_long = nnz > CV_LONG;
    const int64_t cap = std::max<int64_t>(1, std::min<int64_t>(nbr, nnz / CV_LONG + 1));
    DevBuf<int64_t> long_list(may_be_long ? cap : 0, h.stream);
    DevBuf<unsigned> long_n(may_be_long ? 1 : 0, h.stream);
    if (may_be_long) XS_CHECK_CUDA(cudaMemsetAsync(long_n.get(), 0, sizeof(unsigned), h.stream));
    // blocks assembled in shared memory when a block row has at most 32 rows and at least four
    // blocks fit a warp's buffer; otherwise zero-fill and scatter in global memory
    if (bvals && rb <= 32 && rb * cb * (int64_t)sizeof(VT) * 4 <= CV_ASM_BYTES) {
        bcsr_fill_asm_kernel<VT, IT><<<cv_grid(h, nbr), CV_WARPS * 32, 0, h.stream>>>(
            row_ptr, col_ind, values, M, K, nbr, rb, cb, make_div(cb), brp, bci, bvals,
            long_list.get(), long_n.get(), (unsigned)cap);
    } else {
        bcsr_fill_kernel<VT, IT><<<cv_grid(h, nbr), CV_WARPS * 32, 0, h.stream>>>(
            row_ptr, col_ind, values, M, K, nbr, rb, cb, make_div(cb), brp, bci, bvals,
            long_list.get(), long_n.get(), (unsigned)cap);
    }
    after_launch(h, "bcsr_fill");
    if (may_be_long) {
        bcsr_fill_long_kernel<VT, IT><<<cl_grid(h, cap), CL_T, 0, h.stream>>>(
            row_ptr, col_ind, values, M, K, rb, cb, make_div(cb), brp, bci, bvals,
            long_list.get(), long_n.get());
        after_launch(h, "bcsr_fill_long");
    }
}

template int64_t csr_to_bcsr_count<int32_t>(Handle&, int64_t, int64_t, int64_t, const int32_t*,
                                            const int32_t*, int64_t, int64_t, int32_t*);
template int64_t csr_to_bcsr_count<int64_t>(Handle&, int64_t, int64_t, int64_t, const int64_t*,
                                            const int64_t*, int64_t, int64_t, int64_t*);
#define XS_INST_FILL(VT, IT)                                                                      \
    template void csr_to_bcsr_fill<VT, IT>(Handle&, int64_t, int64_t, int64_t, const IT*,         \
                                           const IT*, const VT*, int64_t, int64_t, const IT*, IT*, \
                                           VT*);
XS_INST_FILL(__half, int32_t)
XS_INST_FILL(__half, int64_t)
XS_INST_FILL(__nv_bfloat16, int32_t)
XS_INST_FILL(__nv_bfloat16, int64_t)
XS_INST_FILL(float, int32_t)
XS_INST_FILL(float, int64_t)

}  // namespace xspmm_b200
