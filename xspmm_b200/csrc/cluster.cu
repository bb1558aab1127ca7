// cluster.cu -- exact greedy 1-D Jaccard (Sylos-Labini) row clustering on the device.
//
// Output is bit-identical to the reference's compute_1d_jaccard_clustering
// (src/cpu/clustering_sylos_labini.cpp:51-120):
//   q_r = set of floor(col/w) over row r (:13-33); U = [0..M); repeat: seed = U.back(), pop;
//   p = q_seed; c = [seed]; for i = |U|-1 down to 0: d = |p u q|==0 ? 0 : 1 - (float)|p n q|/|p u q|
//   (:35-46); if d <= tau: c += U[i], p |= q_U[i], U[i] = U.back(), pop (:93-105).
//   perm = concatenation of the clusters in creation order (:110-116).
//
// The reference costs O(M * clusters * K/w/64) with dense bitsets. This implementation visits
// only rows that can pass the test, using facts that follow from the loop above:
//  (1) tau >= 1 accepts everything and tau < 0 or NaN accepts nothing; both yield M-1..0.
//  (2) For 0 <= tau < 1 an accepted row shares >= m = max(1, ceil(t|p|)) block columns with p and
//      has m <= |q| <= |p|/t, t = 1 - tau less 2^-22 (a margin above the float rounding of the
//      test). So it meets every subset of p with |p| - m + 1 columns: gathering the rows of any
//      such subset (cheapest inverted lists first), restricted to that size window, finds every
//      row that can be accepted. An empty seed accepts exactly the empty rows.
//  (3) In one pass the scan pointer only moves down and swap-with-back writes only at or above
//      it, so the not-yet-scanned positions are fixed during the pass. Candidates are evaluated in
//      parallel against the current p; the highest-position accepted candidate that adds columns
//      to p ends the round: everything above it is final, p grows, rows below it are
//      re-evaluated next round. Rows are still decided in decreasing position order.
//  (4) The pass's removals (holes h_0 > h_1 > ... > h_{k-1}, U[h] = U.back(); pop) are replayed
//      in parallel: for h_t < n-k, U'[h_t] = U[chase(n-1-t)] with chase(x) = x if x is not a hole
//      of this pass, else chase(n-1-rank(x)). An element can move more than once.
//
// Data: row patterns come from the CSR->BCSR kernels run with r_block = 1, c_block = w (sorted
// distinct block columns per row). The inverted index maps a block column to its rows grouped by
// pattern size in 32 classes (sizes 1..31 exact, 32 = "32 or more"), so a size window is a
// contiguous slice.
//
// Gathering: for a column of p whose inverted list is short ("light") the size window of (2) is
// walked once (and, when p grows, the classes the widened window newly admits), and every
// eligible row on it gets one hit on a per-row counter, so |q n p| over light columns is a
// counter read -- no dependent load of the candidate's pattern. Long lists ("heavy", the hub
// columns of power-law matrices) are walked only when the light columns of p are fewer than
// |p| - m + 1, and then only over the size window of (2); a candidate's hits in heavy columns are
// looked up in its pattern (after a bound check that rejects most candidates without it).
//
// The greedy loop is inherently sequential across clusters and runs in one persistent CTA of 256
// threads; all per-pass work (gather, evaluate, compaction, sorting, replay) is parallel inside
// it, and a pass is a chain of latency, so the code keeps that chain short: every thread reads the
// seed itself, the first walk starts from the seed's pattern entries and their window slices
// (precomputed per pattern entry) with no barrier before it, hit counters are 16-bit shared-memory
// atomics when the row state fits in shared memory, and a pass with at most 256 candidates, no
// heavy column and no accepted row that grows p -- the common case -- is decided in one
// evaluation, ranked by counting and replayed in place (a handful of barriers); every other pass
// takes the general round loop of (3). Every loop is bounded by the data sizes; an internal
// consistency failure sets an error flag and stops instead of spinning.

#include "ops.cuh"

#include <cstdlib>
#include <cstring>

namespace xspmm_b200 {
namespace {

constexpr int CL_THREADS = 256;
constexpr int NCLS = 32;            // size classes per block column in the inverted index
constexpr int SORT_CAP = 1024;      // settled acceptances kept in shared memory (uint64 keys)
constexpr int CAND_CAP = 1024;      // candidates kept in shared memory (the rest in global)
constexpr int HOLE_CAP = 1024;      // holes of a pass kept in shared memory (the rest in global)
constexpr int FAST_PER = 4;         // candidates per thread the fast path evaluates
static_assert(FAST_PER * CL_THREADS <= CAND_CAP && FAST_PER * CL_THREADS <= SORT_CAP,
              "fast-path candidates stay in shared memory");
constexpr int SMEM_ROWS = 20480;    // U and pos live in shared memory up to this many rows
constexpr int64_t HEAVY = 2048;     // inverted lists longer than this are walked by size window
constexpr int LIGHT_MASK = (1 << 30) - 1;
// Expected inverted-list entries per pass above which the cluster sweep (cluster_bits.cu) is
// faster, from measurements on B200 (index kernel ~2 ns per entry, sweep ~10 us per pass).
constexpr int64_t SWEEP_VISITS = 8192;
// Below this many expected entries per pass the index path (with seed sets) is chosen even when
// the bitsets fit: measured on the reference's benchmark patterns at 4096 rows, the index path
// won at up to ~400 (arrowhead, block diagonal, 0.1 % random, power law) and the bitsets from
// ~6,000 (1 % and 10 % random). At 1024 rows the bitset rounds are so cheap that they won on
// nearly every pattern, so below INDEX_MIN_ROWS rows the bitsets are kept whenever they fit.
constexpr int64_t INDEX_VISITS = 1024;
constexpr int64_t INDEX_MIN_ROWS = 4096;
constexpr int HEAVY_MARK = 1 << 30;
// Seed sets (seed_sets_kernel): a record of SS_REC ints per row -- the count (-1: not available)
// and, for sets of up to SS_REC-1 rows, the rows within tau of the row, each with bit 31 set when
// it would add columns to the row's pattern; larger sets, up to SS_CAP rows, sit in a pool and the
// record's first row slot holds their offset there. A row whose walk would exceed SS_WALK_MAX
// list entries, or whose set exceeds SS_CAP rows, gets no record.
constexpr int SS_REC = 64;
constexpr int SS_CAP = 1023;
constexpr int64_t SS_WALK_MAX = int64_t(1) << 24;
constexpr int SS_BM_MAX = 65536;  // block columns up to which seed_sets_kernel uses bitmaps
constexpr int SS_RUN_SET = 8;     // set size up to which a seed is tested for a singleton run
// Rows whose walk exceeds SS_HEAVY list entries get their seed set from seed_sets_heavy_kernel
// (a CTA per row, hit estimates in a count-min sketch of 2 x SSH_SKETCH counters).
constexpr int64_t SS_HEAVY = 4096;
constexpr int SSH_SKETCH_LOG = 13;
constexpr int SSH_SKETCH = 1 << SSH_SKETCH_LOG;
static_assert(SS_CAP <= SORT_CAP, "a pool record is settled in the shared sort buffer");

struct ClusterArgs {
    int32_t M;
    int32_t nbc;
    const int64_t* qptr;    // [M+1] row pattern offsets
    const int32_t* qcol;    // row patterns (block columns, ascending)
    const int64_t* iptr;    // [nbc*NCLS+1] inverted index offsets
    const int2* ient;       // inverted index entries (row, pattern size)
    int32_t* U;             // [M] unclustered rows by position
    int32_t* pos;           // [M] position of a row in U, -1 once clustered
    int32_t* cnt;           // [M] light-column hits this pass (| HEAVY_MARK); 0 between passes
    int32_t* cstamp;        // [nbc] pass in which the column was first walked / joined the
                            //       window-gathered heavy set
    int32_t* cslot;         // [nbc] next size class to walk / gather for that column
    int32_t* hstamp;        // [nbc] pass in which the column was classified heavy
    const longlong2* qslice;  // [pattern entries] slice of the entry's inverted list over the
                              //   size window of a pattern of the row's own size
    uint32_t* pbits;        // [ceil(nbc/32)] pattern of the current cluster
    int32_t* plist;         // [nbc] columns of p, in insertion order
    int32_t* hlist;         // [nbc] heavy columns of p
    int32_t* glist;         // [nbc] window-gathered heavy columns of this pass
    int32_t* crow;          // [2*M] candidates beyond the shared-memory part (two buffers)
    int32_t* clen;          // [2*M]
    int32_t* cpos;          // [2*M]
    uint8_t* cflag;         // [M]
    uint64_t* racc;         // [max(M,nbc)] scratch: settled keys / (cost << 32 | col)
    uint64_t* gsort;        // [pow2 >= M] global sort scratch
    int32_t* holes;         // [M] holes of a pass beyond the shared-memory part
    int32_t* perm;          // [M] output (int32 view)
    float tau;
    double t_lo;
    const int32_t* sets;    // [M*SS_REC] seed sets, or null
    const int32_t* spool;   // rows of the seed sets larger than SS_REC-1, or null
    unsigned* err;
};

__device__ __forceinline__ int slot_of(int64_t len) {
    return (int)(len >= NCLS ? NCLS - 1 : len - 1);
}

__device__ __forceinline__ int64_t min_inter(double t_lo, int64_t psz) {
    const double m = ceil(t_lo * (double)psz);
    return m < 1.0 ? 1 : (int64_t)m;
}
__device__ __forceinline__ int64_t max_len(double t_lo, int64_t psz) {
    if (t_lo <= 0.0) return INT64_MAX / 4;
    return (int64_t)floor((double)psz / t_lo);
}

// Jaccard distance exactly as the reference evaluates it (float division, float subtraction).
__device__ __forceinline__ float jaccard_distance(int64_t inter, int64_t uni) {
    if (uni == 0) return 0.0f;
    const float q = __fdiv_rn((float)inter, (float)uni);
    return __fsub_rn(1.0f, q);
}

// CTA-wide exclusive scans of one value per thread (3 barriers).
__device__ int cta_excl_scan(int v, int* s_warp, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int inc = warp_inclusive_sum(v);
    if (lane == 31) s_warp[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        const int w = lane < CL_THREADS / 32 ? s_warp[lane] : 0;
        const int wi = warp_inclusive_sum(w);
        if (lane < CL_THREADS / 32) s_warp[lane] = wi - w;
        if (lane == CL_THREADS / 32 - 1) *total = wi;
    }
    __syncthreads();
    const int r = s_warp[warp] + inc - v;
    __syncthreads();
    return r;
}

__device__ int64_t cta_excl_scan64(int64_t v, int64_t* s_warp, int64_t* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t inc = warp_inclusive_sum(v);
    if (lane == 31) s_warp[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        const int64_t w = lane < CL_THREADS / 32 ? s_warp[lane] : 0;
        const int64_t wi = warp_inclusive_sum(w);
        if (lane < CL_THREADS / 32) s_warp[lane] = wi - w;
        if (lane == CL_THREADS / 32 - 1) *total = wi;
    }
    __syncthreads();
    const int64_t r = s_warp[warp] + inc - v;
    __syncthreads();
    return r;
}

__device__ int64_t cta_max64_cl(int64_t v, int64_t* s_warp) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) s_warp[warp] = v;
    __syncthreads();
    int64_t r = s_warp[0];
    for (int w = 1; w < CL_THREADS / 32; ++w) r = max(r, s_warp[w]);
    __syncthreads();
    return r;
}

// Bitonic sort of n uint64 keys in `a` (shared or global memory), ascending or descending,
// padded up to cap (a power of two >= n) with sentinels.
__device__ void cta_bitonic_sort(uint64_t* a, int n, int cap, bool desc) {
    const uint64_t pad = desc ? 0ull : ~0ull;
    for (int i = n + threadIdx.x; i < cap; i += CL_THREADS) a[i] = pad;
    __syncthreads();
    for (int size = 2; size <= cap; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < cap / 2; i += CL_THREADS) {
                const int lo = 2 * i - (i & (stride - 1));
                const int hi = lo + stride;
                const bool up = ((lo & size) == 0) != desc;
                const uint64_t x = a[lo], y = a[hi];
                if ((x > y) == up) {
                    a[lo] = y;
                    a[hi] = x;
                }
            }
            __syncthreads();
        }
    }
}

__device__ int pow2_at_least(int n) {
    int c = 1;
    while (c < n) c <<= 1;
    return c;
}

struct Shared {
    int s_warp[32];
    int total;
    int64_t s_warp64[32];
    int64_t total64;
    int64_t col_beg[CL_THREADS];      // flattened walks of heavy windows
    int64_t col_off[CL_THREADS + 1];
    int n, out, k, pass, seed, stop;
    int pcount, nproc, nheavy, hg, ncand, nkeep, nr, smax, limit, grown, need, cur, wshi;
    int64_t m, ub;
    int crow[2][CAND_CAP];            // pending candidates (double-buffered): row,
    int clen[2][CAND_CAP];            //   pattern size,
    int cpos[2][CAND_CAP];            //   position in U (fixed during the pass)
    uint8_t cflag[CAND_CAP];
    uint64_t sortbuf[SORT_CAP];
    int holes[HOLE_CAP];              // first HOLE_CAP holes of the pass
};

// Rows' positions and U live in shared memory when they fit (SU), else in global memory. The
// per-row hit counters live in shared memory too when there is room and a light count fits in 15
// bits (SC): two 16-bit counters per word (bit 15 = found through a heavy column), so a hit is a
// shared-memory atomic instead of an L2 round trip.
template <bool SU, bool SC>
struct RowState {
    int32_t* U;
    int32_t* pos;
    int32_t* gcnt;   // global counters (SC false)
    uint32_t* scnt;  // shared counters (SC true)
    __device__ __forceinline__ int u(int i) const { return U[i]; }
    __device__ __forceinline__ void set_u(int i, int v) const { U[i] = v; }
    __device__ __forceinline__ int p(int r) const { return pos[r]; }
    __device__ __forceinline__ void set_p(int r, int v) const { pos[r] = v; }
    // one light hit; returns the previous value (0: first time the row is touched this pass)
    __device__ __forceinline__ int cnt_add(int r) const {
        if constexpr (SC) {
            const int sft = (r & 1) * 16;
            return (int)((atomicAdd(&scnt[r >> 1], 1u << sft) >> sft) & 0xFFFFu);
        } else {
            return atomicAdd(&gcnt[r], 1);
        }
    }
    // marks a row found through a heavy column; returns the previous value
    __device__ __forceinline__ int cnt_heavy(int r) const {
        if constexpr (SC) {
            const int sft = (r & 1) * 16;
            return (int)((atomicOr(&scnt[r >> 1], 0x8000u << sft) >> sft) & 0xFFFFu);
        } else {
            return atomicOr(&gcnt[r], HEAVY_MARK);
        }
    }
    __device__ __forceinline__ int cnt_light(int r) const {
        if constexpr (SC) return (int)((scnt[r >> 1] >> ((r & 1) * 16)) & 0x7FFFu);
        else return gcnt[r] & LIGHT_MASK;
    }
    __device__ __forceinline__ void cnt_clear(int r) const {
        if constexpr (SC) atomicAnd(&scnt[r >> 1], ~(0xFFFFu << ((r & 1) * 16)));
        else gcnt[r] = 0;
    }
};

__device__ __forceinline__ void cand_get(const Shared& sh, const ClusterArgs& a, int buf, int c,
                                         int& r, int& len, int& pr) {
    if (c < CAND_CAP) {
        r = sh.crow[buf][c];
        len = sh.clen[buf][c];
        pr = sh.cpos[buf][c];
    } else {
        const int64_t g = (int64_t)buf * a.M + c;
        r = a.crow[g];
        len = a.clen[g];
        pr = a.cpos[g];
    }
}
__device__ __forceinline__ void cand_set(Shared& sh, ClusterArgs& a, int buf, int c, int r,
                                         int len, int pr) {
    if (c < CAND_CAP) {
        sh.crow[buf][c] = r;
        sh.clen[buf][c] = len;
        sh.cpos[buf][c] = pr;
    } else {
        const int64_t g = (int64_t)buf * a.M + c;
        a.crow[g] = r;
        a.clen[g] = len;
        a.cpos[g] = pr;
    }
}
__device__ __forceinline__ uint8_t flag_get(const Shared& sh, const ClusterArgs& a, int c) {
    return c < CAND_CAP ? sh.cflag[c] : a.cflag[c];
}
__device__ __forceinline__ void flag_set(Shared& sh, ClusterArgs& a, int c, uint8_t f) {
    if (c < CAND_CAP) sh.cflag[c] = f; else a.cflag[c] = f;
}
__device__ __forceinline__ int hole_get(const Shared& sh, const ClusterArgs& a, int t) {
    return t < HOLE_CAP ? sh.holes[t] : a.holes[t];
}
__device__ __forceinline__ void hole_set(Shared& sh, ClusterArgs& a, int t, int v) {
    if (t < HOLE_CAP) sh.holes[t] = v; else a.holes[t] = v;
}

__device__ __forceinline__ void append_candidate(Shared& sh, ClusterArgs& a, int r, int len,
                                                 int pr) {
    const int slot = atomicAdd(&sh.ncand, 1);
    if (slot < a.M) cand_set(sh, a, sh.cur, slot, r, len, pr);
    else flag_error(a.err, DERR_INTERNAL);
}

// One warp walks the inverted-list entries [e_beg, e_end), four loads in flight per lane (the
// entries are L2 round trips; issuing them one after another would serialize them).
template <typename F>
__device__ __forceinline__ void warp_walk(const int2* ient, int64_t e_beg, int64_t e_end, int lane,
                                          F&& f) {
    for (int64_t e0 = e_beg; e0 < e_end; e0 += 128) {
        int2 en[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t e = e0 + lane + 32 * u;
            if (e < e_end) en[u] = ient[e];
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (e0 + lane + 32 * u < e_end) f(en[u]);
    }
}

// Walks the entries of up to CL_THREADS inverted-list slices (one per thread) spread over the
// whole CTA.
template <typename F>
__device__ void flat_walk(Shared& sh, const int2* ient, int64_t e_beg, int64_t e_cnt, F&& f) {
    const int tid = threadIdx.x;
    const int64_t off = cta_excl_scan64(e_cnt, sh.s_warp64, &sh.total64);
    sh.col_beg[tid] = e_beg;
    sh.col_off[tid] = off;
    if (tid == CL_THREADS - 1) sh.col_off[CL_THREADS] = off + e_cnt;
    __syncthreads();
    const int64_t total = sh.total64;
    for (int64_t f0 = tid; f0 < total; f0 += 4 * CL_THREADS) {
        int2 en[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t fi = f0 + (int64_t)u * CL_THREADS;
            if (fi >= total) break;
            int lo = 0, hi = CL_THREADS - 1;  // last slice with col_off <= fi (a non-empty one)
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (sh.col_off[mid] <= fi) lo = mid; else hi = mid - 1;
            }
            en[u] = ient[sh.col_beg[lo] + (fi - sh.col_off[lo])];
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (f0 + (int64_t)u * CL_THREADS < total) f(en[u]);
    }
    __syncthreads();
}

// Does the sorted pattern [b, e) contain column x?
__device__ __forceinline__ bool pattern_has(const int32_t* qcol, int64_t b, int64_t e, int x) {
    while (b < e) {
        const int64_t mid = b + ((e - b) >> 1);
        const int v = qcol[mid];
        if (v == x) return true;
        if (v < x) b = mid + 1; else e = mid;
    }
    return false;
}

template <bool SU, bool SC>
__global__ void __launch_bounds__(CL_THREADS, 1) cluster_kernel(ClusterArgs a) {
    static_assert(SU || !SC, "shared counters need U/pos in shared memory");
    __shared__ Shared sh;
    extern __shared__ int32_t dyn[];
    RowState<SU, SC> st;
    st.gcnt = a.cnt;
    st.scnt = nullptr;
    if constexpr (SU) {
        st.U = dyn;
        st.pos = dyn + a.M;
        if constexpr (SC) st.scnt = reinterpret_cast<uint32_t*>(dyn + 2 * a.M);
    } else {
        st.U = a.U;
        st.pos = a.pos;
    }
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if constexpr (SU) {
        for (int i = tid; i < a.M; i += CL_THREADS) {
            st.U[i] = i;
            st.pos[i] = i;
        }
        if constexpr (SC)
            for (int i = tid; i < (a.M + 1) / 2; i += CL_THREADS) st.scnt[i] = 0u;
    }
    if (tid == 0) {
        sh.n = a.M;
        sh.out = 0;
        sh.pass = 0;
        sh.stop = 0;
        sh.ncand = 0;  // the first walk of a pass appends to these before its first barrier
        sh.nheavy = 0;
        sh.cur = 0;
        sh.nr = 0;
    }
    __syncthreads();

    while (sh.n > 0 && !sh.stop) {
        // Passes decided from seed sets, by warp 0 alone (no CTA barrier): when no row that is
        // still unclustered in the seed's set would add columns to p, p stays the seed's pattern
        // for the whole pass, so the pass accepts exactly the unclustered rows of the set (the
        // rows within tau of the seed's pattern), in decreasing position order. The record is
        // usually loaded during the previous pass; the acceptances are ranked across the warp
        // and replayed as in fact 4. Any other pass (no record, a growing row, more than 32
        // acceptances) runs the CTA-wide code.
        if (a.sets) {
            if (warp == 0) {
                int n_cur = sh.n, out_cur = sh.out;
                int pf_seed = -1, pf0 = 0;  // first half of the predicted next seed's record
                // A run is looked for at the start and after a pass that accepted nothing, not
                // after one that found none or accepted rows (matrices whose passes mostly
                // accept, like hidden blocks, would pay a record round trip per pass for nothing).
                bool try_run = true;
                while (n_cur > 0) {
                    // Singleton run: lane i looks at the seed s_i = U[n-1-i] of the i-th pass
                    // from now. When the passes before it accepted nothing, s_i's pass accepts
                    // nothing either exactly when no row of its (complete) set is unclustered at
                    // a position below its own -- the seeds s_0..s_{i-1} have left by then. The
                    // leading lanes for which that holds are clustered alone, at once. Sets of
                    // more than SS_RUN_SET rows end the run.
                    if (try_run) {
                        const int pi = n_cur - 1 - lane;
                        int si = -1;
                        bool single = false;
                        if (pi >= 0) {
                            si = st.u(pi);
                            if (si >= 0 && si < a.M) {
                                const int32_t* rc = a.sets + (int64_t)si * SS_REC;
                                const int c = rc[0];
                                if (c >= 0 && c <= SS_RUN_SET) {
                                    int xs[SS_RUN_SET];
#pragma unroll
                                    for (int j = 0; j < SS_RUN_SET; ++j)
                                        xs[j] = j < c ? (rc[1 + j] & 0x7fffffff) : -1;
                                    single = true;
#pragma unroll
                                    for (int j = 0; j < SS_RUN_SET; ++j) {
                                        if (xs[j] < 0 || xs[j] >= a.M) continue;
                                        const int px = st.p(xs[j]);
                                        if (px >= 0 && px < pi) single = false;
                                    }
                                }
                            }
                        }
                        const unsigned sb = __ballot_sync(0xffffffffu, single);
                        const int run = sb == 0xffffffffu ? 32 : __ffs(~sb) - 1;
                        try_run = run == 32;  // the run ended at a seed that accepts something
                        if (run > 0) {
                            if (out_cur + run > a.M) break;
                            if (lane < run) {
                                a.perm[out_cur + lane] = si;
                                st.set_p(si, -1);
                            }
                            __syncwarp();
                            out_cur += run;
                            n_cur -= run;
                            pf_seed = -1;
                            continue;
                        }
                    }
                    const int seed = st.u(n_cur - 1);
                    if (seed < 0 || seed >= a.M) break;  // the CTA-wide code flags it
                    const int32_t* rec = a.sets + (int64_t)seed * SS_REC;
                    const int v0 = seed == pf_seed ? pf0 : rec[lane];
                    const int cnt = __shfl_sync(0xffffffffu, v0, 0);
                    if (cnt < 0 || cnt > SS_REC - 1) break;
                    const int n = n_cur - 1;
                    // Entry j of the set sits at record index 1 + j. Each lane ends up with one
                    // accepted row and its position (key -1 for none): in place when the set fits
                    // the first half of the record, else compacted through shared memory.
                    int key = -1, row = 0, nr;
                    if (cnt <= 31) {  // uniform across the warp
                        const bool e0 = lane >= 1 && lane <= cnt;
                        const int x0 = e0 ? (v0 & 0x7fffffff) : 0;
                        const int p0 = e0 ? st.p(x0) : -1;
                        const bool l0 = p0 >= 0 && p0 < n;
                        if (__any_sync(0xffffffffu, l0 && v0 < 0)) break;
                        nr = __popc(__ballot_sync(0xffffffffu, l0));
                        if (l0) {
                            key = p0;
                            row = x0;
                        }
                    } else {
                        const int v1 = rec[32 + lane];
                        const bool e0 = lane >= 1, e1 = 32 + lane <= cnt;
                        const int x0 = e0 ? (v0 & 0x7fffffff) : 0, x1 = e1 ? (v1 & 0x7fffffff) : 0;
                        const int p0 = e0 ? st.p(x0) : -1, p1 = e1 ? st.p(x1) : -1;
                        const bool l0 = p0 >= 0 && p0 < n, l1 = p1 >= 0 && p1 < n;
                        if (__any_sync(0xffffffffu, (l0 && v0 < 0) || (l1 && v1 < 0))) break;
                        const unsigned b0 = __ballot_sync(0xffffffffu, l0);
                        const unsigned b1 = __ballot_sync(0xffffffffu, l1);
                        nr = __popc(b0) + __popc(b1);
                        if (nr > 32) break;
                        const unsigned lt = (1u << lane) - 1u;
                        if (l0) sh.sortbuf[__popc(b0 & lt)] = ((uint64_t)(uint32_t)p0 << 32) | (uint32_t)x0;
                        if (l1)
                            sh.sortbuf[__popc(b0) + __popc(b1 & lt)] =
                                ((uint64_t)(uint32_t)p1 << 32) | (uint32_t)x1;
                        __syncwarp();
                        if (lane < nr) {
                            const uint64_t kv = sh.sortbuf[lane];
                            key = (int)(kv >> 32);
                            row = (int)(uint32_t)kv;
                        }
                        __syncwarp();
                    }
                    if (out_cur + 1 + nr > a.M) break;
                    // The next seed is U[n-nr-1] unless that position is a hole of this pass:
                    // its record loads while this pass is ranked and replayed.
                    pf_seed = n - nr >= 1 ? st.u(n - nr - 1) : -1;
                    if (pf_seed >= 0 && pf_seed < a.M)
                        pf0 = a.sets[(int64_t)pf_seed * SS_REC + lane];
                    else
                        pf_seed = -1;
                    // Rank of each acceptance by decreasing position (positions are distinct):
                    // independent shuffles of one 32-bit key, so they overlap; only the lanes
                    // that can hold one (1..cnt, or 0..nr-1 after compaction), 8 at a time.
                    const bool acc = key >= 0;
                    const int kmax = cnt <= 31 ? cnt : nr - 1;  // last lane that can hold a key
                    int rank = 0;
#pragma unroll
                    for (int g = 0; g < 32; g += 8) {
                        if (g > kmax) break;  // uniform across the warp
#pragma unroll
                        for (int j = g; j < g + 8; ++j)
                            rank += __shfl_sync(0xffffffffu, key, j) > key;
                    }
                    const int rr = row, pp = key, hbase = n - nr;
                    // Fact 4: hole h_t < n-nr receives U[chase(n-1-t)]. Without a hole at or
                    // above n-nr the chase stops at once.
                    const unsigned hi = __ballot_sync(0xffffffffu, acc && pp >= hbase);
                    int mv = -1;
                    if (hi == 0u) {
                        if (acc) mv = st.u(n - 1 - rank);
                    } else {
                        if (lane < nr) sh.holes[lane] = -1;
                        __syncwarp();
                        if (acc && pp >= hbase) sh.holes[pp - hbase] = rank;
                        __syncwarp();
                        if (acc && pp < hbase) {
                            int x = n - 1 - rank, steps = 0;
                            while (x >= hbase && steps <= nr) {
                                const int hr = sh.holes[x - hbase];
                                if (hr < 0) break;
                                x = n - 1 - hr;
                                ++steps;
                            }
                            if (steps > nr || x >= n) flag_error(a.err, DERR_INTERNAL);
                            else mv = st.u(x);
                        }
                        __syncwarp();
                    }
                    // U is read above at positions >= n-nr only and written below at holes
                    // < n-nr only, so the two never meet.
                    if (acc) {
                        a.perm[out_cur + 1 + rank] = rr;
                        st.set_p(rr, -1);
                        if (pp < hbase && mv >= 0) {
                            st.set_u(pp, mv);
                            st.set_p(mv, pp);
                        }
                    }
                    if (lane == 0) {
                        a.perm[out_cur] = seed;
                        st.set_p(seed, -1);
                    }
                    __syncwarp();
                    out_cur += 1 + nr;
                    n_cur = n - nr;
                    try_run = nr == 0;
                }
                if (lane == 0) {
                    sh.n = n_cur;
                    sh.out = out_cur;
                }
            }
            __syncthreads();
            if (sh.n == 0) break;
        }
        // A pass decided from a pool record (a set of SS_REC..SS_CAP rows), by the whole CTA:
        // when no unclustered row of the set adds columns to p, the pass accepts exactly the
        // unclustered rows of the set. They are sorted by decreasing position (the order the
        // reference appends them in) and their removals replayed as in fact 4, the holes found
        // by bisection in the sorted positions.
        if (a.sets && a.spool) {
            const int n_old = sh.n;
            const int seed = st.u(n_old - 1);
            const int c = (seed >= 0 && seed < a.M) ? a.sets[(int64_t)seed * SS_REC] : -1;
            if (c > SS_REC - 1 && c <= SS_CAP) {  // uniform: every thread read the same record
                const int32_t* mem = a.spool + a.sets[(int64_t)seed * SS_REC + 1];
                const int n = n_old - 1;
                const int out0 = sh.out;
                constexpr int PER = (SS_CAP + CL_THREADS) / CL_THREADS;
                int xr[PER], xp[PER];
                bool grow = false;
#pragma unroll
                for (int q = 0; q < PER; ++q) {
                    const int i = tid + q * CL_THREADS;
                    xr[q] = -1;
                    xp[q] = -1;
                    if (i < c) {
                        const int v = mem[i];
                        const int x = v & 0x7fffffff;
                        const int px = (x >= 0 && x < a.M) ? st.p(x) : -1;
                        if (px >= 0 && px < n) {
                            xr[q] = x;
                            xp[q] = px;
                            grow |= v < 0;
                        }
                    }
                }
                if (tid == 0) sh.nr = 0;
                const int any_grow = __syncthreads_or(grow);
                if (!any_grow) {
#pragma unroll
                    for (int q = 0; q < PER; ++q)
                        if (xr[q] >= 0)
                            sh.sortbuf[atomicAdd(&sh.nr, 1)] =
                                ((uint64_t)(uint32_t)xp[q] << 32) | (uint32_t)xr[q];
                    __syncthreads();
                    const int nr = sh.nr;
                    if (nr > 1) cta_bitonic_sort(sh.sortbuf, nr, pow2_at_least(nr), true);
                    if (out0 + 1 + nr > a.M) {
                        if (tid == 0) { flag_error(a.err, DERR_INTERNAL); sh.stop = 1; }
                        __syncthreads();
                        break;
                    }
                    for (int t = tid; t < nr; t += CL_THREADS) {
                        const int r = (int)(uint32_t)sh.sortbuf[t];
                        a.perm[out0 + 1 + t] = r;
                        st.set_p(r, -1);
                    }
                    // holes sortbuf[t] >> 32, decreasing; those >= n-nr are a prefix
                    int ktop;
                    {
                        int lo = 0, hi = nr;
                        while (lo < hi) {
                            const int mid = (lo + hi) >> 1;
                            if ((int)(sh.sortbuf[mid] >> 32) >= n - nr) lo = mid + 1; else hi = mid;
                        }
                        ktop = lo;
                    }
                    for (int t = ktop + tid; t < nr; t += CL_THREADS) {
                        const int h = (int)(sh.sortbuf[t] >> 32);
                        int x = n - 1 - t, steps = 0;
                        for (;;) {
                            int lo = 0, hi = ktop;
                            while (lo < hi) {
                                const int mid = (lo + hi) >> 1;
                                if ((int)(sh.sortbuf[mid] >> 32) > x) lo = mid + 1; else hi = mid;
                            }
                            if (lo < ktop && (int)(sh.sortbuf[lo] >> 32) == x && steps <= nr) {
                                x = n - 1 - lo;
                                ++steps;
                            } else {
                                break;
                            }
                        }
                        if (steps > nr || x >= n) {
                            flag_error(a.err, DERR_INTERNAL);
                            continue;
                        }
                        const int r = st.u(x);
                        st.set_u(h, r);
                        st.set_p(r, h);
                    }
                    if (tid == 0) {
                        a.perm[out0] = seed;
                        st.set_p(seed, -1);
                        sh.out = out0 + 1 + nr;
                        sh.n = n - nr;
                        sh.pass += 1;
                        sh.nr = 0;
                    }
                    __syncthreads();
                    continue;
                }
                __syncthreads();
                if (tid == 0) sh.nr = 0;
                __syncthreads();
            }
        }
        // Pass start without a barrier: every thread reads the seed (U.back()) and its pattern,
        // and the first walk of p's columns runs straight from the seed's pattern entries and
        // their precomputed window slices, so the chain of dependent loads before the first
        // barrier is seed -> pattern -> inverted-list slice -> counter. The seed is at position
        // n = |U| - 1, outside every candidate test (pos < limit = n).
        const int pass = sh.pass;
        const int n_old = sh.n;
        const int out0 = sh.out;
        const int seed = st.u(n_old - 1);
        if (seed < 0 || seed >= a.M || out0 >= a.M) {  // uniform: all threads read the same state
            if (tid == 0) flag_error(a.err, DERR_INTERNAL);
            break;
        }
        const int n = n_old - 1;
        // read by the fast path until the previous pass's last barrier; first used after B2
        if (tid == 0) sh.nr = 0;
        const int64_t s0 = a.qptr[seed];
        const int64_t slen = a.qptr[seed + 1] - s0;
        if (slen > 0) {
            const int64_t m0 = min_inter(a.t_lo, slen), ub0 = max_len(a.t_lo, slen);
            const int slo0 = slot_of(m0), shi0 = slot_of(ub0 < NCLS ? ub0 : NCLS);
            auto first_hit = [&](int2 en) {
                const int pr = st.p(en.x);
                if (pr < 0 || pr >= n) return;
                if (st.cnt_add(en.x) == 0) append_candidate(sh, a, en.x, en.y, pr);
            };
            // column t of the seed: record it in p, classify it, return its window slice
            auto first_column = [&](int t, bool writer, int64_t& e_beg, int64_t& e_cnt) {
                const int b = a.qcol[s0 + t];
                const longlong2 sl = a.qslice[s0 + t];
                e_beg = sl.x;
                e_cnt = sl.y - sl.x;
                const bool heavy = e_cnt > HEAVY;
                if (writer && heavy) {  // p's bitmap and column list wait for the general path
                    a.hstamp[b] = pass;
                    a.hlist[atomicAdd(&sh.nheavy, 1)] = b;
                }
                if (heavy) e_cnt = 0;
            };
            if (slen <= 2 * (CL_THREADS / 32)) {
                for (int t = warp; t < slen; t += CL_THREADS / 32) {
                    int64_t e_beg, e_cnt;
                    first_column(t, lane == 0, e_beg, e_cnt);
                    warp_walk(a.ient, e_beg, e_beg + e_cnt, lane, first_hit);
                }
            } else {
                for (int64_t c0 = 0; c0 < slen; c0 += CL_THREADS) {
                    const int64_t t = c0 + tid;
                    int64_t e_beg = 0, e_cnt = 0;
                    if (t < slen) first_column((int)t, true, e_beg, e_cnt);
                    flat_walk(sh, a.ient, e_beg, e_cnt, first_hit);
                }
            }
        }
        __syncthreads();

        // Fast path for the common pass: at most FAST_PER*CL_THREADS candidates, no heavy column and no
        // accepted row that adds columns to p. Then every candidate is decided against the seed's
        // pattern alone and nothing depends on the order of the decisions: evaluate, rank the
        // accepted rows by position, done -- a handful of barriers instead of the general round
        // loop. Anything else (growth, heavy columns, many candidates, an empty seed) goes through
        // the general path, which starts from the same state (the evaluation writes nothing).
        bool fast_done = false;
        {
            const int ncand0 = sh.ncand;
            // up to FAST_PER candidates per thread (the candidate buffer holds CAND_CAP)
            const bool fast = slen > 0 && ncand0 <= FAST_PER * CL_THREADS && sh.nheavy == 0;
            int rq[FAST_PER], prq[FAST_PER], accq[FAST_PER];
            int grow = 0;
#pragma unroll
            for (int q = 0; q < FAST_PER; ++q) {
                rq[q] = -1;
                prq[q] = -1;
                accq[q] = 0;
                const int c = tid + q * CL_THREADS;
                if (fast && c < ncand0) {
                    int len = 0;
                    cand_get(sh, a, 0, c, rq[q], len, prq[q]);
                    const int64_t inter = st.cnt_light(rq[q]);
                    accq[q] =
                        jaccard_distance(inter, slen + (int64_t)len - inter) <= a.tau ? 1 : 0;
                    grow |= accq[q] && len > inter;
                }
            }
            const int any_grow = __syncthreads_or(grow);
            if (fast && !any_grow) {
#pragma unroll
                for (int q = 0; q < FAST_PER; ++q) {
                    if (rq[q] < 0) continue;
                    st.cnt_clear(rq[q]);
                    if (accq[q])
                        sh.sortbuf[atomicAdd(&sh.nr, 1)] =
                            ((uint64_t)(uint32_t)prq[q] << 32) | (uint32_t)rq[q];
                }
                __syncthreads();
                const int nr = sh.nr;  // <= ncand0 <= SORT_CAP
                if (nr <= 32) {
                    // The common case, in warp 0 alone: lane j holds acceptance j; its rank (by
                    // decreasing position) comes from 32 shuffles, and the holes at positions
                    // >= n-nr -- the only ones the chase of fact 4 can meet -- are looked up in a
                    // table of their ranks instead of rescanning the acceptances.
                    if (warp == 0) {
                        const uint64_t kv = lane < nr ? sh.sortbuf[lane] : 0ull;
                        int rank = 0;
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const uint64_t kj = __shfl_sync(0xffffffffu, kv, j);
                            rank += (j < nr && kj > kv) ? 1 : 0;
                        }
                        const int rr = (int)(uint32_t)kv, pp = (int)(kv >> 32);
                        const int hbase = n - nr;  // holes at or above it are table entries
                        if (lane < nr) sh.holes[lane] = -1;
                        __syncwarp();
                        if (lane < nr && pp >= hbase) sh.holes[pp - hbase] = rank;
                        __syncwarp();
                        if (lane < nr) {
                            if (out0 + 1 + rank < a.M) {
                                a.perm[out0 + 1 + rank] = rr;
                                st.set_p(rr, -1);
                            } else {
                                flag_error(a.err, DERR_INTERNAL);
                            }
                            if (pp < hbase) {  // hole h_rank receives U[chase(n-1-rank)]
                                int x = n - 1 - rank, steps = 0;
                                while (x >= hbase && steps <= nr) {
                                    const int hr = sh.holes[x - hbase];
                                    if (hr < 0) break;
                                    x = n - 1 - hr;
                                    ++steps;
                                }
                                if (steps > nr || x >= n) {
                                    flag_error(a.err, DERR_INTERNAL);
                                } else {
                                    const int mv = st.u(x);
                                    st.set_u(pp, mv);
                                    st.set_p(mv, pp);
                                }
                            }
                        }
                    }
                } else {  // decreasing position order, ranked by counting
                  for (int kq = tid; kq < nr; kq += CL_THREADS) {
                    const uint64_t kv = sh.sortbuf[kq];
                    int rank = 0;
                    for (int j = 0; j < nr; ++j) rank += sh.sortbuf[j] > kv;
                    const int rr = (int)(uint32_t)kv, pp = (int)(kv >> 32);
                    if (out0 + 1 + rank < a.M) {
                        a.perm[out0 + 1 + rank] = rr;
                        st.set_p(rr, -1);
                    } else {
                        flag_error(a.err, DERR_INTERNAL);
                    }
                    // The removals, replayed here (fact 4): hole h_rank < n-nr receives
                    // U[chase(n-1-rank)]; chase steps to n-1-rank(x) while x is a hole. The reads
                    // (positions >= n-nr) and the writes (holes < n-nr) never meet.
                    if (pp < n - nr) {
                        int x = n - 1 - rank, steps = 0;
                        for (;;) {
                            int hr = -1;  // rank of x among the holes, or -1
                            for (int j = 0; j < nr; ++j)
                                if ((int)(sh.sortbuf[j] >> 32) == x) {
                                    hr = 0;
                                    for (int i = 0; i < nr; ++i) hr += sh.sortbuf[i] > sh.sortbuf[j];
                                    break;
                                }
                            if (hr < 0 || steps > nr) break;
                            x = n - 1 - hr;
                            ++steps;
                        }
                        if (steps > nr || x >= n) {
                            flag_error(a.err, DERR_INTERNAL);
                        } else {
                            const int mv = st.u(x);
                            st.set_u(pp, mv);
                            st.set_p(mv, pp);
                        }
                    }
                  }
                }
                if (tid == 0) {
                    sh.seed = seed;
                    sh.n = n;
                    st.set_p(seed, -1);
                    a.perm[out0] = seed;
                    sh.out = out0 + 1 + nr;
                    sh.k = nr;  // sh.nr is cleared at the end of the pass
                }
                fast_done = true;
            }
        }
        if (!fast_done) {
            if (slen > 0) {
                const int64_t ub0 = max_len(a.t_lo, slen);
                const int shi0 = slot_of(ub0 < NCLS ? ub0 : NCLS);
                for (int64_t t = tid; t < slen; t += CL_THREADS) {  // p = q_seed
                    const int b = a.qcol[s0 + t];
                    atomicOr(&a.pbits[b >> 5], 1u << (b & 31));
                    a.plist[t] = b;
                    if (a.hstamp[b] != pass) {  // light: walked up to shi0 by the first walk
                        a.cstamp[b] = pass;
                        a.cslot[b] = shi0 + 1;
                    }
                }
            }
            if (tid == 0) {
                sh.seed = seed;
                sh.n = n;
                st.set_p(seed, -1);
                a.perm[out0] = seed;
                sh.out = out0 + 1;
                sh.k = 0;
                if (slen > 0) {
                    sh.pcount = (int)slen;
                    sh.nproc = (int)slen;  // walked above
                    sh.wshi = slot_of(max_len(a.t_lo, slen) < NCLS ? max_len(a.t_lo, slen) : NCLS);
                    sh.hg = 0;
                    sh.limit = n;
                    sh.grown = 1;  // the heavy-column step of the first round still has to run
                    sh.m = min_inter(a.t_lo, slen);
                    sh.ub = max_len(a.t_lo, slen);
                    sh.need = (int)(slen - sh.m + 1);
                }
            }
            __syncthreads();

            if (slen == 0) {
                // Empty pattern: accepts exactly the empty rows, in decreasing position order.
                for (int hi = n; hi > 0; hi -= CL_THREADS) {
                    const int i = hi - 1 - tid;
                    int f = 0, r = -1;
                    if (i >= 0) {
                        r = st.u(i);
                        f = (a.qptr[r + 1] == a.qptr[r]) ? 1 : 0;
                    }
                    const int idx = cta_excl_scan(f, sh.s_warp, &sh.total);
                    if (f) {
                        if (sh.out + idx < a.M && sh.k + idx < a.M) {
                            a.perm[sh.out + idx] = r;
                            hole_set(sh, a, sh.k + idx, i);
                            st.set_p(r, -1);
                        } else {
                            flag_error(a.err, DERR_INTERNAL);
                        }
                    }
                    __syncthreads();
                    if (tid == 0) {
                        sh.out += sh.total;
                        sh.k += sh.total;
                    }
                    __syncthreads();
                }
            } else {
                for (int round = 0;; ++round) {
                    if (round > a.M + 1) {  // each round settles >= 1 candidate
                        if (tid == 0) { flag_error(a.err, DERR_INTERNAL); sh.stop = 1; }
                        __syncthreads();
                        break;
                    }
                    if (sh.grown) {
                        const int64_t m = sh.m, ub = sh.ub;
                        const int limit = sh.limit;
                        const int pc = sh.pcount;
                        const int slo = slot_of(m), shi = slot_of(ub < NCLS ? ub : NCLS);
                        // (1) Columns of p with a short ("light") list: one warp walks the size
                        // window [m, ub] of the list and every eligible row on it gets one hit, so
                        // |q n p| over light columns is a counter for every row the window admits
                        // (a row's size class is the same in all of its columns). Each column keeps
                        // the first class it has not walked; when p grows the window only widens
                        // upwards, so old columns walk just the newly admitted classes and no
                        // (column, row) pair is counted twice. Heavy lists are set aside.
                        // A column is heavy when its window slice is long at the time it joins p
                        // (hub columns against small patterns); against a large pattern the window
                        // sits in high size classes and even hub columns are light.
                        const int t_first = shi != sh.wshi ? 0 : sh.nproc;
                        const int nproc0 = sh.nproc;
                        // Column t of p: its slice of the window still to walk ([e_beg, e_beg +
                        // e_cnt)), or none if it is heavy. A column that joined p since the last walk
                        // (t >= nproc0) has not been walked in this pass: its slice starts at slo.
                        struct Col {
                            int b, kind;  // kind: 0 light, 1 heavy (new), 2 heavy (known)
                            int64_t e_beg, e_cnt;
                        };
                        auto column = [&](int t) {
                            Col c{a.plist[t], 0, 0, 0};
                            const int64_t* ib = a.iptr + (int64_t)c.b * NCLS;
                            int from = slo;
                            if (t >= nproc0) {
                                if (ib[shi + 1] - ib[slo] > HEAVY) {
                                    c.kind = 1;
                                    return c;
                                }
                            } else {
                                if (a.hstamp[c.b] == pass) {
                                    c.kind = 2;
                                    return c;
                                }
                                if (a.cstamp[c.b] == pass) from = max(a.cslot[c.b], slo);
                            }
                            if (from <= shi) {
                                c.e_beg = ib[from];
                                c.e_cnt = ib[shi + 1] - c.e_beg;
                            }
                            return c;
                        };
                        auto record = [&](const Col& c) {
                            if (c.kind == 1) {
                                a.hstamp[c.b] = pass;
                                a.hlist[atomicAdd(&sh.nheavy, 1)] = c.b;
                            } else if (c.kind == 0) {
                                a.cstamp[c.b] = pass;
                                a.cslot[c.b] = shi + 1;
                            }
                        };
                        auto hit = [&](int2 en) {
                            const int pr = st.p(en.x);
                            if (pr < 0 || pr >= limit) return;
                            if (st.cnt_add(en.x) == 0) append_candidate(sh, a, en.x, en.y, pr);
                        };
                        if (pc - t_first <= 2 * (CL_THREADS / 32)) {
                            // few columns: one warp per column, no CTA-wide scan
                            for (int t = t_first + warp; t < pc; t += CL_THREADS / 32) {
                                const Col c = column(t);
                                __syncwarp();
                                if (lane == 0) record(c);
                                warp_walk(a.ient, c.e_beg, c.e_beg + c.e_cnt, lane, hit);
                            }
                        } else {
                            // many columns (large patterns): CL_THREADS at a time, one per thread,
                            // their slices walked as one flattened range by the whole CTA
                            for (int c0 = t_first; c0 < pc; c0 += CL_THREADS) {
                                const int t = c0 + tid;
                                int64_t e_beg = 0, e_cnt = 0;
                                if (t < pc) {
                                    const Col c = column(t);
                                    record(c);
                                    e_beg = c.e_beg;
                                    e_cnt = c.e_cnt;
                                }
                                flat_walk(sh, a.ient, e_beg, e_cnt, hit);
                            }
                        }
                        __syncthreads();
                        if (tid == 0) {
                            sh.nproc = pc;
                            sh.wshi = shi;
                        }
                        // (2) Heavy columns are needed only when the light ones are fewer than
                        // |p| - m + 1; then take the cheapest ones over the size window [m, ub].
                        const int nheavy = sh.nheavy;
                        const int want = sh.need - (pc - nheavy) - sh.hg;
                        if (want > 0) {
                            if (tid == 0) sh.nr = 0;
                            __syncthreads();
                            for (int t = tid; t < nheavy; t += CL_THREADS) {
                                const int b = a.hlist[t];
                                if (a.cstamp[b] != pass) {
                                    const int64_t c = a.iptr[(int64_t)b * NCLS + shi + 1] -
                                                      a.iptr[(int64_t)b * NCLS + slo];
                                    const uint64_t cost = c > 0xffffffffll ? 0xffffffffull : (uint64_t)c;
                                    a.racc[atomicAdd(&sh.nr, 1)] = (cost << 32) | (uint32_t)b;
                                }
                            }
                            __syncthreads();
                            const int nu = sh.nr;
                            int take = nu;
                            if (want < nu && nu <= SORT_CAP) {
                                for (int t = tid; t < nu; t += CL_THREADS) sh.sortbuf[t] = a.racc[t];
                                __syncthreads();
                                cta_bitonic_sort(sh.sortbuf, nu, pow2_at_least(nu), false);
                                for (int t = tid; t < want; t += CL_THREADS) a.racc[t] = sh.sortbuf[t];
                                __syncthreads();
                                take = want;
                            }
                            for (int t = tid; t < take; t += CL_THREADS) {
                                const int b = (int)(uint32_t)a.racc[t];
                                a.cstamp[b] = pass;
                                a.cslot[b] = slo;
                                a.glist[sh.hg + t] = b;
                            }
                            __syncthreads();
                            if (tid == 0) sh.hg += take;
                            __syncthreads();
                        }
                        const int hg = sh.hg;
                        for (int c0 = 0; c0 < hg; c0 += CL_THREADS) {
                            const int ci = c0 + tid;
                            int64_t e_beg = 0, e_cnt = 0;
                            if (ci < hg) {
                                const int b = a.glist[ci];
                                const int from = max(a.cslot[b], slo);
                                if (from <= shi) {
                                    e_beg = a.iptr[(int64_t)b * NCLS + from];
                                    e_cnt = a.iptr[(int64_t)b * NCLS + shi + 1] - e_beg;
                                }
                                if (a.cslot[b] < shi + 1) a.cslot[b] = shi + 1;
                            }
                            flat_walk(sh, a.ient, e_beg, e_cnt, [&](int2 en) {
                                if ((int64_t)en.y < m) return;
                                const int pr = st.p(en.x);
                                if (pr < 0 || pr >= limit) return;
                                if (st.cnt_heavy(en.x) == 0)
                                    append_candidate(sh, a, en.x, en.y, pr);
                            });
                        }
                        if (tid == 0) {
                            sh.grown = 0;
                            sh.smax = -1;
                            sh.nr = 0;
                            sh.nkeep = 0;
                        }
                        __syncthreads();
                    }
                    const int ncand = sh.ncand;
                    if (ncand == 0) break;
                    const int buf = sh.cur;

                    // Evaluate every pending candidate against the current p.
                    const int pcount = sh.pcount;
                    const int nheavy = sh.nheavy;
                    for (int c = tid; c < ncand; c += CL_THREADS) {
                        int r, len, pr;
                        cand_get(sh, a, buf, c, r, len, pr);
                        int64_t inter = st.cnt_light(r);
                        // Light hits are exact; each heavy column adds at most one. The distance is
                        // non-increasing in the intersection (fixed |p| + |q|), so a candidate that
                        // fails even with every heavy column counted is rejected without reading its
                        // pattern.
                        bool hopeless = false;
                        if (nheavy > 0) {
                            const int64_t imax = min(inter + (int64_t)nheavy, (int64_t)len);
                            hopeless = jaccard_distance(imax, pcount + (int64_t)len - imax) > a.tau;
                        }
                        if (nheavy > 0 && !hopeless) {
                            const int64_t q0 = a.qptr[r], q1 = a.qptr[r + 1];
                            if ((int64_t)nheavy * 4 >= len) {  // scan q against all of p
                                inter = 0;
                                for (int64_t j = q0; j < q1; ++j) {
                                    const int b = a.qcol[j];
                                    inter += (a.pbits[b >> 5] >> (b & 31)) & 1u;
                                }
                            } else {  // light hits are counted; look the heavy columns up in q
                                for (int h = 0; h < nheavy; ++h)
                                    inter += pattern_has(a.qcol, q0, q1, a.hlist[h]) ? 1 : 0;
                            }
                        }
                        const int64_t uni = pcount + (int64_t)len - inter;
                        const bool acc = !hopeless && jaccard_distance(inter, uni) <= a.tau;
                        const bool grow = acc && len > inter;
                        flag_set(sh, a, c, acc ? (grow ? 2 : 1) : 0);
                        if (grow) atomicMax(&sh.smax, pr);
                    }
                    __syncthreads();
                    const int smax = sh.smax;

                    // Settle every candidate at or above smax (its counter is cleared: it can never
                    // be gathered again in this pass); keep the rest, in any order, in the other
                    // buffer. Settled acceptances are collected with their positions.
                    for (int c = tid; c < ncand; c += CL_THREADS) {
                        int r, len, pr;
                        cand_get(sh, a, buf, c, r, len, pr);
                        if (pr < smax) {
                            cand_set(sh, a, buf ^ 1, atomicAdd(&sh.nkeep, 1), r, len, pr);
                        } else {
                            st.cnt_clear(r);
                            if (flag_get(sh, a, c)) {
                                const int slot = atomicAdd(&sh.nr, 1);
                                const uint64_t kv = ((uint64_t)(uint32_t)pr << 32) | (uint32_t)r;
                                if (slot < SORT_CAP) sh.sortbuf[slot] = kv; else a.racc[slot] = kv;
                            }
                        }
                    }
                    __syncthreads();
                    const int nr = sh.nr;
                    // Append the settled acceptances in decreasing position order.
                    if (nr <= CL_THREADS) {  // rank by counting
                        if (tid < nr) {
                            const uint64_t kv = sh.sortbuf[tid];
                            int rank = 0;
                            for (int j = 0; j < nr; ++j) rank += sh.sortbuf[j] > kv;
                            const int r = (int)(uint32_t)kv, pr = (int)(kv >> 32);
                            if (sh.out + rank < a.M && sh.k + rank < a.M) {
                                a.perm[sh.out + rank] = r;
                                hole_set(sh, a, sh.k + rank, pr);
                                st.set_p(r, -1);
                            } else {
                                flag_error(a.err, DERR_INTERNAL);
                            }
                        }
                    } else {
                        uint64_t* keys = a.gsort;
                        for (int t = tid; t < nr; t += CL_THREADS)
                            keys[t] = t < SORT_CAP ? sh.sortbuf[t] : a.racc[t];
                        __syncthreads();
                        cta_bitonic_sort(keys, nr, pow2_at_least(nr), true);
                        for (int t = tid; t < nr; t += CL_THREADS) {
                            const uint64_t kv = keys[t];
                            const int r = (int)(uint32_t)kv, pr = (int)(kv >> 32);
                            if (sh.out + t < a.M && sh.k + t < a.M) {
                                a.perm[sh.out + t] = r;
                                hole_set(sh, a, sh.k + t, pr);
                                st.set_p(r, -1);
                            } else {
                                flag_error(a.err, DERR_INTERNAL);
                            }
                        }
                    }
                    // The candidate at smax was accepted and adds columns: grow p, in the same
                    // barrier interval as the appends above (they touch neither p nor U, and the
                    // grower's position is settled, so U[smax] is its row).
                    if (smax >= 0) {
                        const int grow_row = st.u(smax);
                        const int64_t g0 = a.qptr[grow_row], g1 = a.qptr[grow_row + 1];
                        for (int64_t j = g0 + tid; j < g1; j += CL_THREADS) {
                            const int b = a.qcol[j];
                            const uint32_t bit = 1u << (b & 31);
                            if (!(atomicOr(&a.pbits[b >> 5], bit) & bit))
                                a.plist[atomicAdd(&sh.pcount, 1)] = b;
                        }
                    }
                    __syncthreads();
                    if (tid == 0) {
                        sh.out += nr;
                        sh.k += nr;
                        sh.ncand = sh.nkeep;
                        sh.cur = buf ^ 1;
                        sh.smax = -1;
                        sh.nr = 0;
                        sh.nkeep = 0;
                        if (smax >= 0) {
                            sh.limit = smax;
                            sh.grown = 1;
                            sh.m = min_inter(a.t_lo, sh.pcount);
                            sh.ub = max_len(a.t_lo, sh.pcount);
                            sh.need = (int)(sh.pcount - sh.m + 1);
                        }
                    }
                    __syncthreads();
                    if (smax < 0) break;  // nothing grew p: every candidate is settled
                }
                for (int t = tid; t < sh.pcount; t += CL_THREADS) a.pbits[a.plist[t] >> 5] = 0u;
            }

            // Replay the pass's removals (U[h] = U.back(); pop, h decreasing): for a hole h_t below
            // n-k the element that lands there is U[chase(n-1-t)], chase(x) = x unless x is itself a
            // hole h_j, then chase(n-1-j). Only holes >= n-k can be chased into; they are a prefix of
            // the decreasing holes list, searched by bisection.
            __syncthreads();
            const int k = sh.k;
            int ktop;
            {
                int lo = 0, hi = k;  // first index with holes[idx] < n-k
                while (lo < hi) {
                    const int mid = (lo + hi) >> 1;
                    if (hole_get(sh, a, mid) >= n - k) lo = mid + 1; else hi = mid;
                }
                ktop = lo;
            }
            for (int t = ktop + tid; t < k; t += CL_THREADS) {
                const int h = hole_get(sh, a, t);
                int x = n - 1 - t;
                int steps = 0;
                for (;;) {
                    int lo = 0, hi = ktop;  // find x in holes[0, ktop) (decreasing)
                    while (lo < hi) {
                        const int mid = (lo + hi) >> 1;
                        if (hole_get(sh, a, mid) > x) lo = mid + 1; else hi = mid;
                    }
                    if (lo < ktop && hole_get(sh, a, lo) == x && steps <= k) {
                        x = n - 1 - lo;
                        ++steps;
                    } else {
                        break;
                    }
                }
                if (steps > k || x >= n) {
                    flag_error(a.err, DERR_INTERNAL);
                    continue;
                }
                const int r = st.u(x);
                st.set_u(h, r);
                st.set_p(r, h);
            }
        }
        // No barrier before this: the replay reads none of these fields, and sh.k was written by
        // thread 0 itself (fast path) or read after a barrier (general path).
        if (tid == 0) {
            sh.n = n - sh.k;
            sh.pass += 1;
            sh.ncand = 0;
            sh.nheavy = 0;
            sh.cur = 0;  // the next first walk appends to candidate buffer 0
            if (sh.out > a.M) { flag_error(a.err, DERR_INTERNAL); sh.stop = 1; }
        }
        __syncthreads();
    }
    if constexpr (SU) {  // leave U/pos in global memory consistent for debugging
        for (int i = tid; i < a.M; i += CL_THREADS) {
            a.U[i] = st.U[i];
            a.pos[i] = st.pos[i];
        }
    }
}

// --- preprocessing kernels -----------------------------------------------------------------------

// For every pattern entry (row r, block column b): the slice of b's inverted list over the size
// window a pattern of |r| columns admits (fact 2) -- where the first walk of a pass seeded by r
// starts and ends, with no lookup of the index at pass time.
__global__ void qslice_kernel(const int64_t* __restrict__ qptr, const int32_t* __restrict__ qcol,
                              int32_t M, const int64_t* __restrict__ iptr, double t_lo,
                              longlong2* __restrict__ qslice) {
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < M;
         r += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j0 = qptr[r], j1 = qptr[r + 1], len = j1 - j0;
        if (len == 0) continue;
        const int64_t m = min_inter(t_lo, len), ub = max_len(t_lo, len);
        const int slo = slot_of(m), shi = slot_of(ub < NCLS ? ub : NCLS);
        for (int64_t j = j0; j < j1; ++j) {
            const int64_t* ib = iptr + (int64_t)qcol[j] * NCLS;
            qslice[j] = make_longlong2(ib[slo], ib[shi + 1]);
        }
    }
}

// Seed set of every row r: the rows x != r with d(q_r, q_x) <= tau, i.e. the rows a pass seeded
// by r accepts while p stays q_r, each flagged when q_x is not a subset of q_r. One warp per row.
// By fact 2 every such x has its size in r's window and meets any |q_r| - m + 1 columns of q_r, so
// the warp walks the window slices of |q_r| - m + 1 columns only (the cheapest ones), skipping
// entries whose size is outside the window; a candidate met in several of them is counted in the
// first (it holds no column walked before). |q_r n q_x| comes from x's pattern, looked up in q_r:
// a shared-memory bitmap of q_r (BM: up to SS_BM_MAX block columns, any pattern size), or a
// binary search in a copy of q_r (patterns up to 32 columns). A candidate is dropped as soon as
// the columns left in its pattern cannot lift the intersection to the test's bound.
//
// Pass 1 (pool == null) handles every row: the record gets the set size (or -1: unavailable --
// empty pattern, a set above SS_CAP rows, a walk above SS_WALK_MAX entries, or a pattern the
// lookup cannot hold) and its first SS_REC-1 rows. Pass 2 (pool != null) walks again the rows
// whose sets have more than SS_REC-1 rows, writes them to the pool at poff[r] (the same walk, so
// the same rows), and stores that offset in the record's first row slot.
template <bool BM>
__global__ void __launch_bounds__(256)
seed_sets_kernel(const int64_t* __restrict__ qptr, const int32_t* __restrict__ qcol,
                 const longlong2* __restrict__ qslice, const int2* __restrict__ ient, int32_t M,
                 float tau, double t_lo, int32_t nbcw, int32_t* __restrict__ sets,
                 int32_t* __restrict__ pool, const int64_t* __restrict__ poff,
                 int32_t* __restrict__ hlist, int32_t* __restrict__ nheavy,
                 uint8_t* __restrict__ hflag) {
    extern __shared__ uint32_t ss_dyn[];
    __shared__ int32_t spat[8][32];   // q_r of each warp's row (without bitmaps)
    __shared__ int32_t srank[8][32];  // walk order of q_r's columns (32: not walked)
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nw = blockDim.x >> 5;
    // BM: q_r as a bitmap, and the columns whose lists were walked already
    uint32_t* pbm = ss_dyn + (size_t)warp * 2 * nbcw;
    uint32_t* ebm = pbm + nbcw;
    if constexpr (BM) {
        for (int i = lane; i < 2 * nbcw; i += 32) pbm[i] = 0u;
        __syncwarp();
    }
    // I >= t_lo * U = t_lo * (|q_r| + |q_x| - I) for an accepted x: the least intersection
    const double ilo_f = t_lo / (1.0 + t_lo);
    const int64_t nwarps = (int64_t)gridDim.x * nw;
    for (int64_t r = (int64_t)blockIdx.x * nw + warp; r < M; r += nwarps) {
        int32_t* out = sets + r * SS_REC;
        int32_t* pout = nullptr;
        int pcap = 0;  // pass 2: the set size found by pass 1 (the pool slots of this row)
        if (pool != nullptr) {  // pass 2: only the rows whose sets overflow the record
            if (hflag != nullptr && hflag[r]) continue;  // seed_sets_heavy_kernel's
            pcap = out[0];
            if (pcap <= SS_REC - 1) continue;
            pout = pool + poff[r];
        }
        const int64_t s0 = qptr[r], slen = qptr[r + 1] - s0;
        if (slen == 0 || (!BM && slen > 32)) {
            // without bitmaps, longer patterns go to seed_sets_heavy_kernel when it runs
            const bool to_heavy = slen > 0 && hlist != nullptr && pool == nullptr;
            if (lane == 0) {
                out[0] = -1;
                if (to_heavy) {
                    hflag[r] = 1;
                    hlist[atomicAdd(nheavy, 1)] = (int32_t)r;
                }
            }
            continue;
        }
        const int64_t m = min_inter(t_lo, slen), ub = max_len(t_lo, slen);
        const int64_t need = slen - m + 1;
        // Which columns to walk: the `need` ones with the shortest window slices. Up to 32
        // columns, by rank (slice length, index); beyond, by a length threshold T found by
        // bisection: every column shorter than T, and the first ones (by index) of length T.
        int64_t T = 0, ties = 0;
        if (slen > 32) {
            int64_t lo = 0, hi = 0;  // hi: the longest slice
            for (int64_t j = lane; j < slen; j += 32) {
                const longlong2 s2 = qslice[s0 + j];
                hi = max(hi, (int64_t)(s2.y - s2.x));
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
            while (lo < hi) {  // smallest T with #(len <= T) >= need
                const int64_t mid = lo + (hi - lo) / 2;
                int64_t c = 0;
                for (int64_t j = lane; j < slen; j += 32) {
                    const longlong2 s2 = qslice[s0 + j];
                    c += (s2.y - s2.x) <= mid ? 1 : 0;
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
                if (c >= need) hi = mid; else lo = mid + 1;
            }
            T = lo;
            int64_t below = 0;
            for (int64_t j = lane; j < slen; j += 32) {
                const longlong2 s2 = qslice[s0 + j];
                below += (s2.y - s2.x) < T ? 1 : 0;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) below += __shfl_xor_sync(0xffffffffu, below, o);
            ties = need - below;  // columns of length exactly T to take, first by index
        }
        const int pl = (int)(slen < 32 ? slen : 32);
        int col = 0x7fffffff, rank = 32;
        longlong2 sl = make_longlong2(0, 0);
        if (slen <= 32) {
            col = lane < pl ? qcol[s0 + lane] : 0x7fffffff;
            sl = lane < pl ? qslice[s0 + lane] : make_longlong2(0, 0);
            const int64_t len = sl.y - sl.x;
            int rk = 0;  // rank of this column by (slice length, index)
            for (int j = 0; j < pl; ++j) {
                const int64_t lj = __shfl_sync(0xffffffffu, len, j);
                rk += (lj < len || (lj == len && j < lane)) ? 1 : 0;
            }
            rank = (lane < pl && rk < need) ? rk : 32;
            if constexpr (!BM) {
                __syncwarp();
                spat[warp][lane] = col;
                srank[warp][lane] = rank;
                __syncwarp();
            }
        }
        // Column j of q_r is walked iff chosen(j); the walk takes them by rank (<= 32 columns)
        // or by index (beyond). Returns the chosen flag of this lane's column j0 + lane, with
        // the running count of ties at T seen before this chunk.
        auto chosen = [&](int64_t j, int64_t len, int64_t& tseen) {
            if (slen <= 32) return j < slen && rank < 32;
            bool w = j < slen && len < T;
            const bool tie = j < slen && len == T;
            const unsigned tb = __ballot_sync(0xffffffffu, tie);
            const int64_t tr = tseen + __popc(tb & ((1u << lane) - 1u));
            if (tie && tr < ties) w = true;
            tseen += __popc(tb);
            return w;
        };
        // total walk (bounded) and, with bitmaps, q_r into the bitmap
        int64_t total = 0;
        {
            int64_t tseen = 0;
            for (int64_t j0 = 0; j0 < slen; j0 += 32) {
                const int64_t j = j0 + lane;
                int64_t len = 0;
                int c = 0;
                if (j < slen) {
                    const longlong2 s2 = slen <= 32 ? sl : qslice[s0 + j];
                    len = s2.y - s2.x;
                    c = slen <= 32 ? col : qcol[s0 + j];
                }
                const bool w = chosen(j, len, tseen);
                total += w ? len : 0;
                if constexpr (BM) {
                    if (j < slen) atomicOr(&pbm[c >> 5], 1u << (c & 31));
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
        }
        __syncwarp();
        int cnt = 0;
        bool over = total > SS_WALK_MAX;
        // a long walk goes to seed_sets_heavy_kernel (pass 1 lists it; pass 2 never sees it)
        const bool defer = !over && hlist != nullptr && total > SS_HEAVY;
        if (defer && lane == 0) {
            hflag[r] = 1;
            hlist[atomicAdd(nheavy, 1)] = (int32_t)r;
        }
        over |= defer;
        // One chosen column's window slice [e_beg, e_end); k: its walk order (without bitmaps).
        auto walk = [&](int c, int64_t e_beg, int64_t e_end, int k) {
            for (int64_t e0 = e_beg; e0 < e_end && !over; e0 += 32) {
                const int64_t e = e0 + lane;
                bool acc = false, grow = false;
                int x = 0;
                if (e < e_end) {
                    const int2 en = ient[e];
                    x = en.x;
                    if (x != (int)r && en.y >= m && en.y <= ub) {
                        const int64_t qlen = en.y;
                        const int64_t b = qptr[x];
                        // floor: never above the least intersection an accepted row has
                        const int64_t inone = (int64_t)floor(ilo_f * (double)(slen + qlen));
                        int64_t inter = 0;
                        bool dup = false, dead = false;
                        for (int64_t j0 = 0; j0 < qlen && !dup && !dead; j0 += 8) {
                            int cb[8];
#pragma unroll
                            for (int j = 0; j < 8; ++j) cb[j] = j0 + j < qlen ? qcol[b + j0 + j] : -1;
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                const int cc = cb[j];
                                if (cc < 0) break;
                                if constexpr (BM) {
                                    const uint32_t bit = 1u << (cc & 31);
                                    if (pbm[cc >> 5] & bit) {
                                        ++inter;
                                        dup |= (ebm[cc >> 5] & bit) != 0u;
                                    }
                                } else {
                                    int lo = 0, hi = pl;
                                    while (lo < hi) {
                                        const int mid = (lo + hi) >> 1;
                                        if (spat[warp][mid] < cc) lo = mid + 1; else hi = mid;
                                    }
                                    if (lo < pl && spat[warp][lo] == cc) {
                                        ++inter;
                                        dup |= srank[warp][lo] < k;
                                    }
                                }
                            }
                            dead = inter + (qlen - min(qlen, j0 + 8)) < inone;
                        }
                        if (!dup && !dead) {
                            acc = jaccard_distance(inter, slen + qlen - inter) <= tau;
                            grow = qlen > inter;
                        }
                    }
                }
                const unsigned ba = __ballot_sync(0xffffffffu, acc);
                if (acc) {
                    const int at = cnt + __popc(ba & ((1u << lane) - 1u));
                    const int v = grow ? (int)((unsigned)x | 0x80000000u) : x;
                    if (pout) {
                        if (at < pcap) pout[at] = v;
                    } else if (at < SS_REC - 1) {
                        out[1 + at] = v;
                    }
                }
                cnt += __popc(ba);
                if (cnt > SS_CAP) over = true;  // uniform across the warp
            }
            if constexpr (BM) {  // c is done: later lists count a candidate holding it as seen
                __syncwarp();
                if (lane == 0) ebm[c >> 5] |= 1u << (c & 31);
                __syncwarp();
            }
        };
        if (slen <= 32) {
            for (int k = 0; k < need && !over; ++k) {
                const int tk = __ffs(__ballot_sync(0xffffffffu, rank == k)) - 1;
                walk(__shfl_sync(0xffffffffu, col, tk), __shfl_sync(0xffffffffu, sl.x, tk),
                     __shfl_sync(0xffffffffu, sl.y, tk), k);
            }
        } else {
            int64_t tseen = 0;
            for (int64_t j0 = 0; j0 < slen && !over; j0 += 32) {
                const int64_t j = j0 + lane;
                longlong2 s2 = make_longlong2(0, 0);
                int c = 0;
                if (j < slen) {
                    s2 = qslice[s0 + j];
                    c = qcol[s0 + j];
                }
                unsigned wb = __ballot_sync(0xffffffffu, chosen(j, s2.y - s2.x, tseen));
                while (wb && !over) {
                    const int t = __ffs(wb) - 1;
                    wb &= wb - 1;
                    walk(__shfl_sync(0xffffffffu, c, t), __shfl_sync(0xffffffffu, s2.x, t),
                         __shfl_sync(0xffffffffu, s2.y, t), 0);
                }
            }
        }
        if (lane == 0) {
            if (pout) out[1] = (int32_t)poff[r];
            else out[0] = over ? -1 : cnt;
        }
        if constexpr (BM) {  // clear this row's bits for the next one
            __syncwarp();
            for (int64_t j = lane; j < slen; j += 32) {
                const int c = qcol[s0 + j];
                pbm[c >> 5] = 0u;
                ebm[c >> 5] = 0u;
            }
            __syncwarp();
        }
    }
}

// Seed sets of the rows whose walk is long (more than SS_HEAVY list entries; hub-like rows of
// hundreds of block columns against other long rows): one CTA per row, every thread on the walk.
// A candidate x met through a walked column can only pass when |q_r n q_x| reaches the bound
// floor(t/(1+t) (|q_r| + |q_x|)), and |q_r n q_x| <= h_x + (m - 1), h_x = the walked columns x
// holds (the other columns of q_r number m - 1). A first walk counts h_x in a count-min sketch
// (two hashed counter arrays in shared memory; the smaller counter can only overestimate h_x), a
// second walk reads the pattern of a candidate only when its estimate passes that bound -- rejected
// candidates cost no pattern read, and the survivors are evaluated exactly. A candidate is counted
// at its smallest walked column (it holds no walked column with a smaller index), so both walks
// run over all walked columns at once. Same record format and passes as seed_sets_kernel.
__global__ void __launch_bounds__(CL_THREADS)
seed_sets_heavy_kernel(const int64_t* __restrict__ qptr, const int32_t* __restrict__ qcol,
                       const longlong2* __restrict__ qslice, const int2* __restrict__ ient,
                       int32_t M, float tau, double t_lo, int32_t nbcw,
                       int32_t* __restrict__ sets, int32_t* __restrict__ pool,
                       const int64_t* __restrict__ poff, const int32_t* __restrict__ hlist,
                       const int32_t* __restrict__ nheavy) {
    extern __shared__ uint32_t hs_dyn[];
    uint32_t* pbm = hs_dyn;                 // q_r
    uint32_t* cbm = pbm + nbcw;             // the walked columns
    uint32_t* sk = cbm + nbcw;              // sketch: 2 x SSH_SKETCH counters
    __shared__ int64_t s_w64[32];
    __shared__ int64_t s_tot64;
    __shared__ int s_w[32];
    __shared__ int s_tot;
    __shared__ int64_t s_off[CL_THREADS + 1];
    __shared__ int64_t s_beg[CL_THREADS];
    __shared__ int s_col[CL_THREADS];
    __shared__ int s_cnt;
    const int tid = threadIdx.x;
    const double ilo_f = t_lo / (1.0 + t_lo);
    const int nh = *nheavy;
    auto h1 = [](uint32_t x) { return (x * 2654435761u) >> (32 - SSH_SKETCH_LOG); };
    auto h2 = [](uint32_t x) { return ((x ^ 0x9e3779b9u) * 2246822519u) >> (32 - SSH_SKETCH_LOG); };
    // Dynamic shared memory starts with whatever the SM's previous kernel left there: the two
    // bitmaps start empty here, and each row clears its own bits when it is done.
    for (int i = tid; i < 2 * nbcw; i += CL_THREADS) hs_dyn[i] = 0u;
    __syncthreads();
    for (int hi = blockIdx.x; hi < nh; hi += gridDim.x) {
        const int r = hlist[hi];
        int32_t* out = sets + (int64_t)r * SS_REC;
        int32_t* pout = nullptr;
        int pcap = 0;
        if (pool != nullptr) {
            pcap = out[0];
            if (pcap <= SS_REC - 1) continue;  // uniform: every thread read the same record
            pout = pool + poff[r];
        }
        const int64_t s0 = qptr[r], slen = qptr[r + 1] - s0;
        const int64_t m = min_inter(t_lo, slen), ub = max_len(t_lo, slen);
        const int64_t need = slen - m + 1;
        // threshold T: the smallest slice length with #(len <= T) >= need (bisection)
        int64_t lo = 0, hi2 = 0;
        for (int64_t j = tid; j < slen; j += CL_THREADS) {
            const longlong2 s2 = qslice[s0 + j];
            hi2 = max(hi2, (int64_t)(s2.y - s2.x));
        }
        hi2 = cta_max64_cl(hi2, s_w64);
        while (lo < hi2) {
            const int64_t mid = lo + (hi2 - lo) / 2;
            int64_t c = 0;
            for (int64_t j = tid; j < slen; j += CL_THREADS) {
                const longlong2 s2 = qslice[s0 + j];
                c += (s2.y - s2.x) <= mid ? 1 : 0;
            }
            int64_t tot;
            cta_excl_scan64(c, s_w64, &s_tot64);
            tot = s_tot64;
            __syncthreads();
            if (tot >= need) hi2 = mid; else lo = mid + 1;
        }
        const int64_t T = lo;
        // q_r and the walked columns into their bitmaps; clear the sketch
        for (int i = tid; i < 2 * SSH_SKETCH; i += CL_THREADS) sk[i] = 0u;
        int64_t below = 0;
        for (int64_t j = tid; j < slen; j += CL_THREADS) {
            const longlong2 s2 = qslice[s0 + j];
            below += (s2.y - s2.x) < T ? 1 : 0;
        }
        cta_excl_scan64(below, s_w64, &s_tot64);
        const int64_t ties = need - s_tot64;
        __syncthreads();
        int64_t tseen = 0;
        for (int64_t c0 = 0; c0 < slen; c0 += CL_THREADS) {
            const int64_t j = c0 + tid;
            int64_t len = -1;
            int col = 0;
            if (j < slen) {
                const longlong2 s2 = qslice[s0 + j];
                len = s2.y - s2.x;
                col = qcol[s0 + j];
                atomicOr(&pbm[col >> 5], 1u << (col & 31));
            }
            const int tie = (len == T) ? 1 : 0;
            const int tr = cta_excl_scan(tie, s_w, &s_tot);
            const bool w = j < slen && (len < T || (tie && tseen + tr < ties));
            tseen += s_tot;
            if (w) atomicOr(&cbm[col >> 5], 1u << (col & 31));
        }
        if (tid == 0) s_cnt = 0;
        __syncthreads();
        // The two walks: over chunks of CL_THREADS pattern entries, each thread holding one
        // (walked) column's window slice, flattened so that the CTA's threads share the entries.
        auto walk = [&](auto&& f) {
            for (int64_t c0 = 0; c0 < slen; c0 += CL_THREADS) {
                const int64_t j = c0 + tid;
                int64_t beg = 0, len = 0;
                int col = 0;
                if (j < slen) {
                    col = qcol[s0 + j];
                    if (cbm[col >> 5] & (1u << (col & 31))) {
                        const longlong2 s2 = qslice[s0 + j];
                        beg = s2.x;
                        len = s2.y - s2.x;
                    }
                }
                const int64_t off = cta_excl_scan64(len, s_w64, &s_tot64);
                s_off[tid] = off;
                s_beg[tid] = beg;
                s_col[tid] = col;
                if (tid == 0) s_off[CL_THREADS] = s_tot64;
                const int64_t tot = s_tot64;
                __syncthreads();
                // entry t of the flattened range belongs to the thread k with off_k <= t < off_{k+1}
                for (int64_t t = tid; t < tot; t += CL_THREADS) {
                    int a = 0, b = CL_THREADS;
                    while (b - a > 1) {
                        const int mid = (a + b) >> 1;
                        if (s_off[mid] <= t) a = mid; else b = mid;
                    }
                    f(ient[s_beg[a] + (t - s_off[a])], s_col[a]);
                }
                __syncthreads();
            }
        };
        // walk 1: h_x estimates
        walk([&](int2 en, int) {
            if (en.x == r || en.y < m || en.y > ub) return;
            atomicAdd(&sk[h1((uint32_t)en.x)], 1u);
            atomicAdd(&sk[SSH_SKETCH + h2((uint32_t)en.x)], 1u);
        });
        // walk 2: candidates whose estimate can pass, evaluated exactly at their smallest walked
        // column
        walk([&](int2 en, int ca) {
            const int x = en.x;
            if (x == r || en.y < m || en.y > ub) return;
            const int64_t qlen = en.y;
            const int64_t inone = (int64_t)floor(ilo_f * (double)(slen + qlen));
            const int64_t est = min(sk[h1((uint32_t)x)], sk[SSH_SKETCH + h2((uint32_t)x)]);
            if (est + (m - 1) < inone) return;
            const int64_t b = qptr[x];
            int64_t inter = 0;
            bool dup = false;
            for (int64_t j = 0; j < qlen; ++j) {
                const int cc = qcol[b + j];
                const uint32_t bit = 1u << (cc & 31);
                if (cc < ca && (cbm[cc >> 5] & bit)) {
                    dup = true;  // counted at a smaller walked column
                    break;
                }
                inter += (pbm[cc >> 5] & bit) ? 1 : 0;
                if (inter + (qlen - j - 1) < inone) break;
            }
            if (dup) return;
            if (jaccard_distance(inter, slen + qlen - inter) <= tau) {
                const int v = qlen > inter ? (int)((unsigned)x | 0x80000000u) : x;
                const int at = atomicAdd(&s_cnt, 1);
                if (pout) {
                    if (at < pcap) pout[at] = v;
                } else if (at < SS_REC - 1) {
                    out[1 + at] = v;
                }
            }
        });
        __syncthreads();
        if (tid == 0) {
            if (pout) out[1] = (int32_t)poff[r];
            else out[0] = s_cnt > SS_CAP ? -1 : s_cnt;
        }
        // clear this row's bits
        for (int64_t j = tid; j < slen; j += CL_THREADS) {
            const int c = qcol[s0 + j];
            pbm[c >> 5] = 0u;
            cbm[c >> 5] = 0u;
        }
        __syncthreads();
    }
}

// Sizes of the sets that overflow their record (more than SS_REC-1 rows), 0 for the others.
__global__ void seed_sets_overflow_kernel(const int32_t* __restrict__ sets, int32_t M,
                                          int64_t* __restrict__ ocnt) {
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < M;
         r += (int64_t)gridDim.x * blockDim.x) {
        const int c = sets[r * SS_REC];
        ocnt[r] = c > SS_REC - 1 ? c : 0;
    }
}

// Records whose overflow could not be kept (the pool would not fit): unavailable.
__global__ void seed_sets_drop_overflow_kernel(int32_t* __restrict__ sets, int32_t M) {
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < M;
         r += (int64_t)gridDim.x * blockDim.x)
        if (sets[r * SS_REC] > SS_REC - 1) sets[r * SS_REC] = -1;
}

__global__ void init_rows_kernel(int32_t* U, int32_t* pos, int32_t* cnt, int32_t M) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < M;
         i += (int64_t)gridDim.x * blockDim.x) {
        U[i] = (int32_t)i;
        pos[i] = (int32_t)i;
        cnt[i] = 0;
    }
}

__global__ void init_cols_kernel(int32_t* cstamp, int32_t* hstamp, uint32_t* pbits, int32_t nbc) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nbc;
         i += (int64_t)gridDim.x * blockDim.x) {
        cstamp[i] = -1;
        hstamp[i] = -1;
        if ((i & 31) == 0) pbits[i >> 5] = 0u;
    }
}

// Histogram of (column, size class) pairs over all row patterns.
__global__ void inv_count_kernel(const int64_t* qptr, const int32_t* qcol, int32_t M,
                                 int64_t* cnt) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < M; r += warps) {
        const int64_t q0 = qptr[r], q1 = qptr[r + 1];
        if (q1 == q0) continue;
        const int s = slot_of(q1 - q0);
        for (int64_t j = q0 + lane; j < q1; j += 32)
            atomicAdd(reinterpret_cast<unsigned long long*>(&cnt[(int64_t)qcol[j] * NCLS + s]), 1ull);
    }
}

__global__ void inv_fill_kernel(const int64_t* qptr, const int32_t* qcol, int32_t M,
                                int64_t* cursor, int2* ient) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < M; r += warps) {
        const int64_t q0 = qptr[r], q1 = qptr[r + 1];
        if (q1 == q0) continue;
        const int64_t len = q1 - q0;
        const int s = slot_of(len);
        for (int64_t j = q0 + lane; j < q1; j += 32) {
            const int64_t at = (int64_t)atomicAdd(
                reinterpret_cast<unsigned long long*>(&cursor[(int64_t)qcol[j] * NCLS + s]), 1ull);
            ient[at] = make_int2((int)r, (int)(len > 0x7fffffff ? 0x7fffffff : len));
        }
    }
}

template <typename IT>
__global__ void widen_index_kernel(const IT* in, int64_t* out, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = (int64_t)in[i];
}

template <typename IT>
__global__ void narrow_cols_kernel(const IT* in, int32_t* out, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = (int32_t)in[i];
}

template <typename IT>
__global__ void store_perm_kernel(const int32_t* in, IT* out, int64_t M) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < M;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = (IT)in[i];
}

template <typename IT>
__global__ void reversed_perm_kernel(IT* perm, int64_t M) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < M;
         i += (int64_t)gridDim.x * blockDim.x)
        perm[i] = (IT)(M - 1 - i);
}

unsigned grid_1d(Handle& h, int64_t n, int threads) {
    const int64_t want = ceil_div(n, threads);
    const int64_t cap = (int64_t)sm_count(h.device) * 16;
    return (unsigned)std::max<int64_t>(1, std::min(want, cap));
}

}  // namespace

template <typename IT>
void cluster_jaccard(Handle& h, int64_t M, int64_t K, int64_t nnz, const IT* row_ptr,
                     const IT* col_ind, float tau, int64_t w, IT* perm) {
    if (M == 0) return;
    XS_REQUIRE(M < (int64_t(1) << 31) - 1, XSPMM_STATUS_UNSUPPORTED,
               "clustering supports at most 2^31-2 rows");
    if (!(tau >= 0.0f) || tau >= 1.0f) {  // fact 1
        reversed_perm_kernel<IT><<<grid_1d(h, M, 256), 256, 0, h.stream>>>(perm, M);
        after_launch(h, "reversed_perm");
        return;
    }
    // Three exact implementations (cluster_bits.cu, this file): row bitsets in one SM's shared
    // memory (when they fit and index passes would be expensive, see INDEX_VISITS); row patterns
    // spread over a cluster's shared memory (when they fit and the inverted lists are long, see
    // SWEEP_VISITS); the inverted index with seed sets otherwise.
    // XSPMM_CLUSTER_KERNEL = bits | sweep | index forces one (bits and sweep fail if the matrix
    // does not fit them).
    const char* ck = std::getenv("XSPMM_CLUSTER_KERNEL");
    const bool want_index = ck && std::strcmp(ck, "index") == 0;
    const bool want_bits = ck && std::strcmp(ck, "bits") == 0;
    const bool want_sweep = ck && std::strcmp(ck, "sweep") == 0;
    if (want_bits) {
        XS_REQUIRE(cluster_jaccard_bits<IT>(h, M, K, row_ptr, col_ind, tau, w, perm),
                   XSPMM_STATUS_UNSUPPORTED,
                   "bitset clustering: the row patterns do not fit in shared memory");
        return;
    }
    const int64_t nbc = ceil_div(K, w);
    XS_REQUIRE(nbc < (int64_t(1) << 31) / NCLS, XSPMM_STATUS_UNSUPPORTED,
               "clustering supports at most 2^26 block columns");
    cudaStream_t s = h.stream;

    // Row patterns: sorted distinct block columns per row (CSR->BCSR with r_block=1, c_block=w).
    DevBuf<IT> qptr_it(M + 1, s);
    const int64_t npat = csr_to_bcsr_count<IT>(h, M, K, nnz, row_ptr, col_ind, 1, w, qptr_it.get());
    DevBuf<IT> qcol_it(std::max<int64_t>(npat, 1), s);
    csr_to_bcsr_fill<__half, IT>(h, M, K, nnz, row_ptr, col_ind, nullptr, 1, w, qptr_it.get(),
                                 qcol_it.get(), nullptr);
    DevBuf<int64_t> qptr(M + 1, s);
    DevBuf<int32_t> qcol(std::max<int64_t>(npat, 1), s);
    widen_index_kernel<IT><<<grid_1d(h, M + 1, 256), 256, 0, s>>>(qptr_it.get(), qptr.get(), M + 1);
    after_launch(h, "widen_index");
    if (npat) {
        narrow_cols_kernel<IT><<<grid_1d(h, npat, 256), 256, 0, s>>>(qcol_it.get(), qcol.get(), npat);
        after_launch(h, "narrow_cols");
    }
    qptr_it.release();
    qcol_it.release();
    // An inverted-index pass visits ~sum_c len_c^2 / M list entries for a random seed (~2 ns
    // each on a B200), at least npat^2 / (nbc M) (equal when the columns are evenly used, as in
    // random structure); the cluster sweep's pass costs ~10 us whatever the structure.
    const double visits_lb = (double)npat * (double)npat / ((double)nbc * (double)M);
    // Where index passes are cheap the index path with seed sets beats the bitset sweep, whose
    // rounds cost the same whatever the structure; elsewhere the bitsets win when they fit.
    if (!want_index && !want_sweep && (visits_lb > (double)INDEX_VISITS || M < INDEX_MIN_ROWS) &&
        cluster_jaccard_bits<IT>(h, M, K, row_ptr, col_ind, tau, w, perm))
        return;
    if (want_sweep || (!want_index && visits_lb > (double)SWEEP_VISITS)) {
        if (cluster_jaccard_sweep<IT>(h, M, nbc, qptr.get(), qcol.get(), tau, perm)) return;
        XS_REQUIRE(!want_sweep, XSPMM_STATUS_UNSUPPORTED,
                   "cluster sweep: the row patterns do not fit a cluster's shared memory");
    }

    // Inverted index by (block column, size class).
    const int64_t nb = std::max<int64_t>(nbc, 1);
    const int64_t nslots = nb * NCLS;
    DevBuf<int64_t> iptr(nslots + 1, s);
    DevBuf<int64_t> cursor(nslots + 1, s);
    DevBuf<int2> ient(std::max<int64_t>(npat, 1), s);
    XS_CHECK_CUDA(cudaMemsetAsync(iptr.get(), 0, (nslots + 1) * sizeof(int64_t), s));
    const unsigned g_rows = grid_1d(h, M * 32, 256);
    inv_count_kernel<<<g_rows, 256, 0, s>>>(qptr.get(), qcol.get(), (int32_t)M, iptr.get());
    after_launch(h, "inv_count");
    exclusive_scan<int64_t>(h, iptr.get(), iptr.get(), nslots);
    XS_CHECK_CUDA(cudaMemcpyAsync(cursor.get(), iptr.get(), (nslots + 1) * sizeof(int64_t),
                                  cudaMemcpyDeviceToDevice, s));
    inv_fill_kernel<<<g_rows, 256, 0, s>>>(qptr.get(), qcol.get(), (int32_t)M, cursor.get(),
                                          ient.get());
    after_launch(h, "inv_fill");
    cursor.release();
    const double t_lo = (1.0 - (double)tau) - 1.0 / (double)(1 << 22);
    DevBuf<longlong2> qslice(std::max<int64_t>(npat, 1), s);
    qslice_kernel<<<grid_1d(h, M, 256), 256, 0, s>>>(qptr.get(), qcol.get(), (int32_t)M,
                                                      iptr.get(), t_lo, qslice.get());
    after_launch(h, "cluster_qslice");

    // Seed sets of every row (one parallel pass over the index), so that most passes of the
    // greedy loop need one record read instead of a walk; XSPMM_CLUSTER_SEED_SETS=0 turns them off.
    const char* ss_env = std::getenv("XSPMM_CLUSTER_SEED_SETS");
    const bool use_sets = !(ss_env && std::strcmp(ss_env, "0") == 0) &&
                          M * SS_REC * (int64_t)sizeof(int32_t) <= (int64_t(1) << 30);
    DevBuf<int32_t> sets(use_sets ? M * SS_REC : 0, s);
    DevBuf<int32_t> spool;
    if (use_sets) {
        // With bitmaps (q_r and the walked columns, 2 bits per block column per warp) as many
        // warps per CTA as fit 96 KB, so two CTAs share an SM; without, eight.
        const bool bm = nbc <= SS_BM_MAX;
        const int64_t nbcw = bm ? ceil_div(nbc, 32) : 0;
        const int warps = bm ? (int)std::max<int64_t>(1, std::min<int64_t>(8, 98304 / (8 * nbcw)))
                             : 8;
        const size_t dsm = bm ? (size_t)warps * 2 * nbcw * sizeof(uint32_t) : 0;
        const unsigned g_ss = (unsigned)std::max<int64_t>(
            1, std::min<int64_t>(ceil_div(M, warps), (int64_t)sm_count(h.device) * 16));
        // Rows with long walks: a CTA each (seed_sets_heavy_kernel), when its bitmaps of q_r and
        // of the walked columns plus the sketch fit shared memory.
        const int64_t hw = ceil_div(nbc, 32);
        const size_t hsm = (size_t)(2 * hw + 2 * SSH_SKETCH) * sizeof(uint32_t);
        const bool heavy = hsm <= 200 * 1024;
        DevBuf<int32_t> hlist(heavy ? M : 0, s), nheavy(heavy ? 1 : 0, s);
        DevBuf<uint8_t> hflag(heavy ? M : 0, s);
        if (heavy) {
            XS_CHECK_CUDA(cudaMemsetAsync(nheavy.get(), 0, sizeof(int32_t), s));
            XS_CHECK_CUDA(cudaMemsetAsync(hflag.get(), 0, (size_t)M, s));
            XS_CHECK_CUDA(cudaFuncSetAttribute(seed_sets_heavy_kernel,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)hsm));
        }
        auto launch = [&](int32_t* pool, const int64_t* poff) {
            if (bm) {
                XS_CHECK_CUDA(cudaFuncSetAttribute(seed_sets_kernel<true>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)dsm));
                seed_sets_kernel<true><<<g_ss, 32 * warps, dsm, s>>>(
                    qptr.get(), qcol.get(), qslice.get(), ient.get(), (int32_t)M, tau, t_lo,
                    (int32_t)nbcw, sets.get(), pool, poff, hlist.get(), nheavy.get(),
                    hflag.get());
            } else {
                seed_sets_kernel<false><<<g_ss, 32 * warps, 0, s>>>(
                    qptr.get(), qcol.get(), qslice.get(), ient.get(), (int32_t)M, tau, t_lo, 0,
                    sets.get(), pool, poff, hlist.get(), nheavy.get(), hflag.get());
            }
            after_launch(h, "cluster_seed_sets");
            if (heavy) {
                seed_sets_heavy_kernel<<<(unsigned)sm_count(h.device) * 2, CL_THREADS, hsm, s>>>(
                    qptr.get(), qcol.get(), qslice.get(), ient.get(), (int32_t)M, tau, t_lo,
                    (int32_t)hw, sets.get(), pool, poff, hlist.get(), nheavy.get());
                after_launch(h, "cluster_seed_sets_heavy");
            }
        };
        launch(nullptr, nullptr);
        // Sets of more than SS_REC-1 rows: into a pool at scanned offsets (second walk of those
        // rows only), or dropped (no record) if the pool would not fit 32-bit offsets.
        DevBuf<int64_t> poff(M + 1, s);
        seed_sets_overflow_kernel<<<grid_1d(h, M, 256), 256, 0, s>>>(sets.get(), (int32_t)M,
                                                                    poff.get());
        after_launch(h, "cluster_seed_sets_overflow");
        exclusive_scan<int64_t>(h, poff.get(), poff.get(), M);
        const int64_t pool_n = read_scalar<int64_t>(h, poff.get() + M);
        if (pool_n > 0 && pool_n < (int64_t(1) << 31)) {
            spool = DevBuf<int32_t>(pool_n, s);
            launch(spool.get(), poff.get());
        } else if (pool_n > 0) {
            seed_sets_drop_overflow_kernel<<<grid_1d(h, M, 256), 256, 0, s>>>(sets.get(),
                                                                            (int32_t)M);
            after_launch(h, "cluster_seed_sets_drop");
        }
    }

    // State of the greedy loop.
    int sort_cap = 1;
    while (sort_cap < M) sort_cap <<= 1;
    DevBuf<int32_t> U(M, s), pos(M, s), cnt(M, s), cstamp(nb, s), cslot(nb, s), hstamp(nb, s),
        plist(nb, s),
        hlist(nb, s), glist(nb, s), crow(2 * M, s), clen(2 * M, s), cpos(2 * M, s), holes(M, s),
        perm32(M, s);
    DevBuf<uint32_t> pbits(ceil_div(nb, 32), s);
    DevBuf<uint8_t> cflag(M, s);
    DevBuf<uint64_t> racc(std::max<int64_t>(M, nb), s), gsort(sort_cap, s);
    init_rows_kernel<<<grid_1d(h, M, 256), 256, 0, s>>>(U.get(), pos.get(), cnt.get(), (int32_t)M);
    after_launch(h, "cluster_init_rows");
    init_cols_kernel<<<grid_1d(h, nb, 256), 256, 0, s>>>(cstamp.get(), hstamp.get(), pbits.get(),
                                                           (int32_t)nb);
    after_launch(h, "cluster_init_cols");

    ClusterArgs a;
    a.M = (int32_t)M;
    a.nbc = (int32_t)nbc;
    a.qptr = qptr.get();
    a.qcol = qcol.get();
    a.iptr = iptr.get();
    a.ient = ient.get();
    a.U = U.get();
    a.pos = pos.get();
    a.cnt = cnt.get();
    a.cstamp = cstamp.get();
    a.cslot = cslot.get();
    a.hstamp = hstamp.get();
    a.pbits = pbits.get();
    a.plist = plist.get();
    a.hlist = hlist.get();
    a.glist = glist.get();
    a.crow = crow.get();
    a.clen = clen.get();
    a.cpos = cpos.get();
    a.cflag = cflag.get();
    a.racc = racc.get();
    a.gsort = gsort.get();
    a.holes = holes.get();
    a.perm = perm32.get();
    a.tau = tau;
    a.t_lo = t_lo;
    a.qslice = qslice.get();
    a.sets = use_sets ? sets.get() : nullptr;
    a.spool = spool.get();
    a.err = h.d_err;
    int smem_optin = 0;
    XS_CHECK_CUDA(cudaDeviceGetAttribute(&smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin,
                                         h.device));
    const size_t dyn_u = (size_t)M * 2 * sizeof(int32_t);
    const size_t dyn_c = dyn_u + (size_t)((M + 1) / 2) * sizeof(uint32_t);
    if (M <= SMEM_ROWS && nbc < 32768 && dyn_c + sizeof(Shared) + 1024 <= (size_t)smem_optin) {
        XS_CHECK_CUDA(cudaFuncSetAttribute(cluster_kernel<true, true>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn_c));
        cluster_kernel<true, true><<<1, CL_THREADS, dyn_c, s>>>(a);
    } else if (M <= SMEM_ROWS) {
        XS_CHECK_CUDA(cudaFuncSetAttribute(cluster_kernel<true, false>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn_u));
        cluster_kernel<true, false><<<1, CL_THREADS, dyn_u, s>>>(a);
    } else {
        cluster_kernel<false, false><<<1, CL_THREADS, 0, s>>>(a);
    }
    after_launch(h, "cluster_greedy");
    store_perm_kernel<IT><<<grid_1d(h, M, 256), 256, 0, s>>>(perm32.get(), perm, M);
    after_launch(h, "cluster_store_perm");
}

template void cluster_jaccard<int32_t>(Handle&, int64_t, int64_t, int64_t, const int32_t*,
                                       const int32_t*, float, int64_t, int32_t*);
template void cluster_jaccard<int64_t>(Handle&, int64_t, int64_t, int64_t, const int64_t*,
                                       const int64_t*, float, int64_t, int64_t*);

}  // namespace xspmm_b200
