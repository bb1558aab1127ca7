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
// contiguous slice. The greedy loop itself is inherently sequential across clusters and runs in
// one persistent CTA of 1024 threads; all per-pass work (gather, evaluate, compaction, sorting,
// replay) is parallel inside it. Every loop is bounded by the data sizes; an internal consistency
// failure sets an error flag and stops instead of spinning.
#include "ops.cuh"

namespace xspmm_b200 {
namespace {

constexpr int CL_THREADS = 1024;
constexpr int NCLS = 32;          // size classes per block column
constexpr int SORT_CAP = 2048;    // in-shared-memory sort capacity (uint64 keys)

struct ClusterArgs {
    int32_t M;
    int32_t nbc;
    const int64_t* qptr;    // [M+1] row pattern offsets
    const int32_t* qcol;    // row patterns (block columns, ascending)
    const int64_t* iptr;    // [nbc*NCLS+1] inverted index offsets
    const int2* ient;       // inverted index entries (row, pattern size)
    int32_t* U;             // [M] unclustered rows by position
    int32_t* pos;           // [M] position of a row in U, -1 once clustered
    int32_t* stamp;         // [M] pass in which a row was gathered
    int32_t* cstamp;        // [nbc] pass in which a column joined the gathered set
    int32_t* cslot;         // [nbc] next size class to gather for that column
    uint32_t* pbits;        // [ceil(nbc/32)] pattern of the current cluster
    int32_t* plist;         // [nbc] columns of p
    int32_t* glist;         // [nbc] gathered columns of this pass
    int32_t* cand;          // [M] pending candidate rows
    int32_t* cand2;         // [M] compaction buffer
    uint8_t* cflag;         // [M] evaluation result per candidate slot
    uint64_t* racc;         // [M] (pos << 32 | row) accepted in the current round
    uint64_t* gsort;        // [M] global sort scratch (pow2-padded sizes up to 2M)
    int32_t* holes;         // [M] accepted positions of this pass, decreasing
    int32_t* hpass;         // [M] by position: pass in which it became a hole
    int32_t* hrank;         // [M] by position: rank among the pass's holes
    int32_t* perm;          // [M] output (int32 view)
    float tau;
    double t_lo;
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

// CTA-wide exclusive scan of one int per thread; returns the prefix, *total gets the sum.
__device__ int cta_excl_scan(int v, int* s_warp, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int inc = warp_inclusive_sum(v);
    if (lane == 31) s_warp[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        const int w = s_warp[lane];
        const int wi = warp_inclusive_sum(w);
        s_warp[lane] = wi - w;
        if (lane == 31) *total = wi;
    }
    __syncthreads();
    const int r = s_warp[warp] + inc - v;
    __syncthreads();
    return r;
}

// CTA-wide exclusive scan of one int64 per thread.
__device__ int64_t cta_excl_scan64(int64_t v, int64_t* s_warp, int64_t* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t inc = warp_inclusive_sum(v);
    if (lane == 31) s_warp[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        const int64_t w = s_warp[lane];
        const int64_t wi = warp_inclusive_sum(w);
        s_warp[lane] = wi - w;
        if (lane == 31) *total = wi;
    }
    __syncthreads();
    const int64_t r = s_warp[warp] + inc - v;
    __syncthreads();
    return r;
}

// Bitonic sort of n uint64 keys (ascending, or descending if desc) held in `a`, which may live in
// shared or global memory; padded to a power of two with +inf/-inf sentinels by the caller's
// capacity. cap must be a power of two >= n.
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
    int64_t col_beg[CL_THREADS];      // gather: first entry of each column's slice
    int64_t col_off[CL_THREADS + 1];  // gather: exclusive offsets of the slices
    int n, out, k, pass, seed;
    int pcount, gcount, ncand, nracc, need;
    int64_t m, ub;
    int limit;
    int smax;
    int grown;
    int stop;
    int new_cols;
    uint64_t sortbuf[SORT_CAP];
};

__global__ void __launch_bounds__(CL_THREADS, 1) cluster_kernel(ClusterArgs a) {
    __shared__ Shared sh;
    const int tid = threadIdx.x;
    if (tid == 0) {
        sh.n = a.M;
        sh.out = 0;
        sh.pass = 0;
        sh.stop = 0;
    }
    __syncthreads();

    while (sh.n > 0 && !sh.stop) {
        if (tid == 0) {
            const int seed = a.U[sh.n - 1];
            if (seed < 0 || seed >= a.M || sh.out >= a.M) {
                flag_error(a.err, DERR_INTERNAL);
                sh.stop = 1;
            } else {
                sh.seed = seed;
                sh.n -= 1;
                a.pos[seed] = -1;
                a.perm[sh.out++] = seed;
                sh.k = 0;
            }
        }
        __syncthreads();
        if (sh.stop) break;
        const int pass = sh.pass;
        const int seed = sh.seed;
        const int n = sh.n;
        const int64_t slen = a.qptr[seed + 1] - a.qptr[seed];

        if (slen == 0) {
            // Empty pattern: accepts exactly the empty rows, in decreasing position order.
            for (int hi = n; hi > 0; hi -= CL_THREADS) {
                const int i = hi - 1 - tid;
                int f = 0, r = -1;
                if (i >= 0) {
                    r = a.U[i];
                    f = (a.qptr[r + 1] == a.qptr[r]) ? 1 : 0;
                }
                const int idx = cta_excl_scan(f, sh.s_warp, &sh.total);
                if (f) {
                    if (sh.out + idx < a.M && sh.k + idx < a.M) {
                        a.perm[sh.out + idx] = r;
                        a.holes[sh.k + idx] = i;
                        a.pos[r] = -1;
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
            // p = q_seed
            const int64_t s0 = a.qptr[seed];
            for (int t = tid; t < slen; t += CL_THREADS) {
                const int b = a.qcol[s0 + t];
                atomicOr(&a.pbits[b >> 5], 1u << (b & 31));
                a.plist[t] = b;
            }
            if (tid == 0) {
                sh.pcount = (int)slen;
                sh.gcount = 0;
                sh.ncand = 0;
                sh.limit = n;
                sh.grown = 1;
            }
            __syncthreads();

            for (int round = 0;; ++round) {
                if (round > a.M + 1) {  // each round settles >= 1 candidate; cannot exceed M
                    if (tid == 0) { flag_error(a.err, DERR_INTERNAL); sh.stop = 1; }
                    __syncthreads();
                    break;
                }
                if (sh.grown) {
                    if (tid == 0) {
                        sh.m = min_inter(a.t_lo, sh.pcount);
                        sh.ub = max_len(a.t_lo, sh.pcount);
                        sh.need = (int)(sh.pcount - sh.m + 1);
                        sh.new_cols = 0;
                    }
                    __syncthreads();
                    const int64_t m = sh.m, ub = sh.ub;
                    const int slo = slot_of(m), shi = slot_of(ub < NCLS ? ub : NCLS);
                    // Columns to add: the cheapest ungathered columns of p.
                    const int want = sh.need - sh.gcount;
                    if (want > 0) {
                        // collect ungathered columns with their window cost
                        if (tid == 0) sh.nracc = 0;
                        __syncthreads();
                        for (int t = tid; t < sh.pcount; t += CL_THREADS) {
                            const int b = a.plist[t];
                            if (a.cstamp[b] != pass) {
                                const int64_t c = a.iptr[(int64_t)b * NCLS + shi + 1] -
                                                  a.iptr[(int64_t)b * NCLS + slo];
                                const uint64_t cost = c > 0xffffffffll ? 0xffffffffull : (uint64_t)c;
                                const int slot = atomicAdd(&sh.nracc, 1);
                                a.racc[slot] = (cost << 32) | (uint32_t)b;
                            }
                        }
                        __syncthreads();
                        const int nu = sh.nracc;
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
                            a.glist[sh.gcount + t] = b;
                        }
                        __syncthreads();
                        if (tid == 0) sh.gcount += take;
                        __syncthreads();
                    }
                    // Gather every gathered column over its not-yet-gathered classes up to shi.
                    // Work is flattened over (column, entry): a scan of the slice lengths of up
                    // to CL_THREADS columns, then threads stride over the entries and find their
                    // column by binary search, so one long column is spread over the CTA.
                    const int limit = sh.limit;
                    for (int c0 = 0; c0 < sh.gcount; c0 += CL_THREADS) {
                        const int ci = c0 + tid;
                        int64_t e_beg = 0, e_cnt = 0;
                        if (ci < sh.gcount) {
                            const int b = a.glist[ci];
                            const int from = max(a.cslot[b], slo);
                            if (from <= shi) {
                                e_beg = a.iptr[(int64_t)b * NCLS + from];
                                e_cnt = a.iptr[(int64_t)b * NCLS + shi + 1] - e_beg;
                            }
                            if (a.cslot[b] < shi + 1) a.cslot[b] = shi + 1;
                        }
                        const int64_t off = cta_excl_scan64(e_cnt, sh.s_warp64, &sh.total64);
                        sh.col_beg[tid] = e_beg;
                        sh.col_off[tid] = off;
                        if (tid == CL_THREADS - 1) sh.col_off[CL_THREADS] = off + e_cnt;
                        __syncthreads();
                        const int64_t total = sh.total64;
                        for (int64_t f = tid; f < total; f += CL_THREADS) {
                            int lo = 0, hi = CL_THREADS - 1;  // last j with col_off[j] <= f
                            while (lo < hi) {
                                const int mid = (lo + hi + 1) >> 1;
                                if (sh.col_off[mid] <= f) lo = mid; else hi = mid - 1;
                            }
                            const int2 en = a.ient[sh.col_beg[lo] + (f - sh.col_off[lo])];
                            if ((int64_t)en.y < m) continue;
                            const int r = en.x;
                            const int pr = a.pos[r];
                            if (pr < 0 || pr >= limit) continue;
                            if (atomicExch(&a.stamp[r], pass) == pass) continue;
                            const int slot = atomicAdd(&sh.ncand, 1);
                            a.cand[slot] = r;
                        }
                        __syncthreads();
                    }
                    __syncthreads();
                    if (tid == 0) sh.grown = 0;
                    __syncthreads();
                }
                const int ncand = sh.ncand;
                if (ncand == 0) break;

                // Evaluate every pending candidate against the current p.
                if (tid == 0) sh.smax = -1;
                __syncthreads();
                const int pcount = sh.pcount;
                for (int c = tid; c < ncand; c += CL_THREADS) {
                    const int r = a.cand[c];
                    const int64_t q0 = a.qptr[r], q1 = a.qptr[r + 1];
                    int64_t inter = 0;
                    for (int64_t j = q0; j < q1; ++j) {
                        const int b = a.qcol[j];
                        inter += (a.pbits[b >> 5] >> (b & 31)) & 1u;
                    }
                    const int64_t len = q1 - q0;
                    const int64_t uni = pcount + len - inter;
                    const bool acc = jaccard_distance(inter, uni) <= a.tau;
                    const bool grow = acc && len > inter;
                    a.cflag[c] = acc ? (grow ? 2 : 1) : 0;
                    if (grow) atomicMax(&sh.smax, a.pos[r]);
                }
                __syncthreads();
                const int smax = sh.smax;

                // Settle every candidate at or above smax; keep the rest pending.
                if (tid == 0) sh.nracc = 0;
                __syncthreads();
                int keep_total = 0;
                for (int c0 = 0; c0 < ncand; c0 += CL_THREADS) {
                    const int c = c0 + tid;
                    int keep = 0;
                    int r = -1, pr = -1;
                    uint8_t f = 0;
                    if (c < ncand) {
                        r = a.cand[c];
                        pr = a.pos[r];
                        f = a.cflag[c];
                        if (pr < smax) keep = 1;
                        else if (f) {
                            const int slot = atomicAdd(&sh.nracc, 1);
                            a.racc[slot] = ((uint64_t)(uint32_t)pr << 32) | (uint32_t)r;
                        }
                    }
                    const int idx = cta_excl_scan(keep, sh.s_warp, &sh.total);
                    if (keep) a.cand2[keep_total + idx] = r;
                    keep_total += sh.total;
                    __syncthreads();
                }
                for (int c = tid; c < keep_total; c += CL_THREADS) a.cand[c] = a.cand2[c];
                __syncthreads();
                const int nr = sh.nracc;
                // order the settled accepted rows by decreasing position
                if (nr > 1) {
                    if (nr <= SORT_CAP) {
                        for (int t = tid; t < nr; t += CL_THREADS) sh.sortbuf[t] = a.racc[t];
                        __syncthreads();
                        cta_bitonic_sort(sh.sortbuf, nr, pow2_at_least(nr), true);
                        for (int t = tid; t < nr; t += CL_THREADS) a.racc[t] = sh.sortbuf[t];
                    } else {
                        for (int t = tid; t < nr; t += CL_THREADS) a.gsort[t] = a.racc[t];
                        __syncthreads();
                        cta_bitonic_sort(a.gsort, nr, pow2_at_least(nr), true);
                        for (int t = tid; t < nr; t += CL_THREADS) a.racc[t] = a.gsort[t];
                    }
                    __syncthreads();
                }
                for (int t = tid; t < nr; t += CL_THREADS) {
                    const uint64_t kv = a.racc[t];
                    const int r = (int)(uint32_t)kv, pr = (int)(kv >> 32);
                    if (sh.out + t < a.M && sh.k + t < a.M) {
                        a.perm[sh.out + t] = r;
                        a.holes[sh.k + t] = pr;
                        a.pos[r] = -1;
                    } else {
                        flag_error(a.err, DERR_INTERNAL);
                    }
                }
                __syncthreads();
                if (tid == 0) {
                    sh.out += nr;
                    sh.k += nr;
                    sh.ncand = keep_total;
                }
                __syncthreads();
                if (smax < 0) break;  // nothing grew p: every candidate is settled

                // The candidate at smax was accepted and adds columns: grow p.
                const int grow_row = a.U[smax];
                const int64_t g0 = a.qptr[grow_row], g1 = a.qptr[grow_row + 1];
                for (int64_t j = g0 + tid; j < g1; j += CL_THREADS) {
                    const int b = a.qcol[j];
                    const uint32_t bit = 1u << (b & 31);
                    if (!(atomicOr(&a.pbits[b >> 5], bit) & bit)) {
                        const int slot = atomicAdd(&sh.pcount, 1);
                        a.plist[slot] = b;
                    }
                }
                __syncthreads();
                if (tid == 0) {
                    sh.limit = smax;
                    sh.grown = 1;
                }
                __syncthreads();
            }
            // clear p
            for (int t = tid; t < sh.pcount; t += CL_THREADS) {
                const int b = a.plist[t];
                a.pbits[b >> 5] = 0u;
            }
            __syncthreads();
        }

        // Replay the pass's removals (fact 4).
        const int k = sh.k;
        for (int t = tid; t < k; t += CL_THREADS) {
            const int h = a.holes[t];
            a.hpass[h] = pass;
            a.hrank[h] = t;
        }
        __syncthreads();
        for (int t = tid; t < k; t += CL_THREADS) {
            const int h = a.holes[t];
            if (h >= n - k) continue;
            int x = n - 1 - t;
            int steps = 0;
            while (x < n && a.hpass[x] == pass && steps <= k) {
                x = n - 1 - a.hrank[x];
                ++steps;
            }
            if (steps > k || x >= n) {
                flag_error(a.err, DERR_INTERNAL);
                continue;
            }
            const int r = a.U[x];
            a.U[h] = r;
            a.pos[r] = h;
        }
        __syncthreads();
        if (tid == 0) {
            sh.n = n - k;
            sh.pass += 1;
            if (sh.out > a.M) { flag_error(a.err, DERR_INTERNAL); sh.stop = 1; }
        }
        __syncthreads();
    }
}

// --- preprocessing kernels -----------------------------------------------------------------------

__global__ void init_rows_kernel(int32_t* U, int32_t* pos, int32_t* stamp, int32_t* hpass,
                                 int32_t M) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < M;
         i += (int64_t)gridDim.x * blockDim.x) {
        U[i] = (int32_t)i;
        pos[i] = (int32_t)i;
        stamp[i] = -1;
        hpass[i] = -1;
    }
}

__global__ void init_cols_kernel(int32_t* cstamp, uint32_t* pbits, int32_t nbc) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nbc;
         i += (int64_t)gridDim.x * blockDim.x) {
        cstamp[i] = -1;
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

    // Inverted index by (block column, size class).
    const int64_t nslots = std::max<int64_t>(nbc, 1) * NCLS;
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

    // State of the greedy loop.
    const int64_t nb = std::max<int64_t>(nbc, 1);
    int sort_cap = 1;
    while (sort_cap < M) sort_cap <<= 1;
    DevBuf<int32_t> U(M, s), pos(M, s), stamp(M, s), cstamp(nb, s), cslot(nb, s), plist(nb, s),
        glist(nb, s), cand(M, s), cand2(M, s), holes(M, s), hpass(M, s), hrank(M, s), perm32(M, s);
    DevBuf<uint32_t> pbits(ceil_div(nb, 32), s);
    DevBuf<uint8_t> cflag(M, s);
    DevBuf<uint64_t> racc(std::max<int64_t>(M, nb), s), gsort(sort_cap, s);
    init_rows_kernel<<<grid_1d(h, M, 256), 256, 0, s>>>(U.get(), pos.get(), stamp.get(),
                                                         hpass.get(), (int32_t)M);
    after_launch(h, "cluster_init_rows");
    init_cols_kernel<<<grid_1d(h, nb, 256), 256, 0, s>>>(cstamp.get(), pbits.get(), (int32_t)nb);
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
    a.stamp = stamp.get();
    a.cstamp = cstamp.get();
    a.cslot = cslot.get();
    a.pbits = pbits.get();
    a.plist = plist.get();
    a.glist = glist.get();
    a.cand = cand.get();
    a.cand2 = cand2.get();
    a.cflag = cflag.get();
    a.racc = racc.get();
    a.gsort = gsort.get();
    a.holes = holes.get();
    a.hpass = hpass.get();
    a.hrank = hrank.get();
    a.perm = perm32.get();
    a.tau = tau;
    a.t_lo = (1.0 - (double)tau) - 1.0 / (double)(1 << 22);
    a.err = h.d_err;
    cluster_kernel<<<1, CL_THREADS, 0, s>>>(a);
    after_launch(h, "cluster_greedy");
    store_perm_kernel<IT><<<grid_1d(h, M, 256), 256, 0, s>>>(perm32.get(), perm, M);
    after_launch(h, "cluster_store_perm");
}

template void cluster_jaccard<int32_t>(Handle&, int64_t, int64_t, int64_t, const int32_t*,
                                       const int32_t*, float, int64_t, int32_t*);
template void cluster_jaccard<int64_t>(Handle&, int64_t, int64_t, int64_t, const int64_t*,
                                       const int64_t*, float, int64_t, int64_t*);

}  // namespace xspmm_b200
