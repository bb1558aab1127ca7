// cluster_bits.cu -- exact greedy 1-D Jaccard clustering for matrices whose row patterns fit in
// shared memory as bitsets.
//
// Same result, bit for bit, as the reference's compute_1d_jaccard_clustering
// (src/cpu/clustering_sylos_labini.cpp:51-120) and as the inverted-index kernel of cluster.cu.
// The reference holds each row's block-column set q_r as a dense bitset (:13-33) and tests every
// remaining row against the cluster pattern p (:86-107). When M x ceil(nbc/32) words fit in one
// SM's shared memory, that is also the fastest layout on the GPU: one CTA keeps all bitsets, the
// pattern sizes |q_r| and the position array U on chip, and a round evaluates every unscanned
// position at once -- |p n q| is a few AND + popc, |p u q| = |p| + |q| - |p n q| -- with one warp
// per 32 consecutive positions, so acceptance and growth come out as ballot words. The inverted
// index pays off when p meets few rows; on patterns where every pass meets a large share of the
// matrix (random structure of a few thousand rows) its walk costs more than this sweep.
//
// Pass structure (facts (3) and (4) of cluster.cu): positions below the scan pointer are fixed
// during a pass, so a round evaluates positions [0, top] against the current p; g = the highest
// accepted position whose row adds block columns to p. Accepted positions in (g, top] and g are
// final in this round: one thread replays them in decreasing order exactly as the reference does
// (perm gets U[j]; U[j] = U.back(); pop), p |= q_{U[g]}, and the next round scans [0, g - 1].
// With no growth the pass ends and the next seed is U.back(). Two CTA barriers per round.
#include "ops.cuh"

#include <vector>

namespace xspmm_b200 {
namespace {

constexpr int CB_THREADS = 512;
constexpr int CB_WARPS = CB_THREADS / 32;

__device__ __forceinline__ bool cb_accept(int inter, int uni, float tau, float t_lo) {
    // 1 - (float)|p n q| / (float)|p u q| <= tau, |p u q| == 0 -> distance 0 (:35-46). A row
    // the test accepts has |p n q| >= t_lo |p u q| with t_lo = 1 - tau - 2^-22 (the margin is
    // above the float rounding of the test, and of the product here for |p u q| < 2^24), so rows
    // below that are rejected without the division.
    if (uni == 0) return 0.0f <= tau;
    if ((float)inter < t_lo * (float)uni) return false;
    return __fsub_rn(1.0f, __fdiv_rn((float)inter, (float)uni)) <= tau;
}

struct CbShared {
    int n;      // rows still unclustered (positions [0, n) of U)
    int top;    // highest position the next round evaluates (-1: none)
    int out;    // next perm slot
    int g;      // highest accepted position whose row grows p (-1: none)
    int prow;   // row whose pattern joins p (pmode 1) or becomes p (pmode 2)
    int pmode;  // 0: p unchanged, 1: p |= q_prow, 2: p = q_prow (new seed)
    int psz;    // |p|
    int kacc;   // acceptances marked this round (an upper bound of the round's final ones)
};

// smem: bits[M * ns] | qsz[M] (uint16) | U[M] | acc[ceil(M/32)] | wpre[ceil(M/32)] | p[nw]. A
// row's bitset takes
// ns = nw | 1 words: with an odd stride the rows that a warp reads at once fall on different
// banks.
template <typename IT>
__global__ void __launch_bounds__(CB_THREADS, 1)
cluster_bits_kernel(const IT* __restrict__ row_ptr, const IT* __restrict__ col_ind, int M,
                    int64_t K, int64_t w, int nw, float tau, float t_lo, IT* __restrict__ perm,
                    unsigned* __restrict__ err) {
    extern __shared__ __align__(16) uint8_t cb_smem[];
    __shared__ CbShared st;
    const int nmw = (M + 31) >> 5;
    const int ns = nw | 1;
    uint32_t* bits = reinterpret_cast<uint32_t*>(cb_smem);
    uint16_t* qsz = reinterpret_cast<uint16_t*>(bits + (size_t)M * ns);
    int32_t* U = reinterpret_cast<int32_t*>(
        cb_smem + (((size_t)M * ns * 4 + (size_t)M * 2 + 15) & ~size_t(15)));
    uint32_t* acc = reinterpret_cast<uint32_t*>(U + M);
    int* wpre = reinterpret_cast<int*>(acc + nmw);  // acceptances above each word, this round
    uint32_t* p = reinterpret_cast<uint32_t*>(wpre + nmw);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    // ---- row bitsets from the CSR (block column = col / w) ----
    for (int64_t i = tid; i < (int64_t)M * ns; i += CB_THREADS) bits[i] = 0u;
    for (int i = tid; i < M; i += CB_THREADS) U[i] = i;  // U = [0, 1, ..., M-1] (:78-82)
    if (tid == 0) {
        st.n = M;
        st.top = -1;  // the first iteration only takes the first seed
        st.out = 0;
        st.g = -1;
        st.prow = -1;
        st.pmode = 0;
        st.psz = 0;
        st.kacc = 0;
    }
    __syncthreads();
    for (int r = warp; r < M; r += CB_WARPS) {
        const int64_t b = (int64_t)row_ptr[r], e = (int64_t)row_ptr[r + 1];
        if (e < b) {
            if (lane == 0) flag_error(err, DERR_ROW_PTR);
            continue;
        }
        for (int64_t j = b + lane; j < e; j += 32) {
            const int64_t c = (int64_t)col_ind[j];
            if (c < 0 || c >= K) {
                flag_error(err, DERR_COL_OUT_OF_RANGE);
                continue;
            }
            const int64_t bc = c / w;
            atomicOr(&bits[(size_t)r * ns + (bc >> 5)], 1u << (bc & 31));
        }
    }
    __syncthreads();
    for (int r = tid; r < M; r += CB_THREADS) {
        int sz = 0;
        for (int k = 0; k < nw; ++k) sz += __popc(bits[(size_t)r * ns + k]);
        qsz[r] = (uint16_t)sz;
    }
    __syncthreads();

    // ---- greedy passes: one iteration per round ----
    // Each iteration either ends a pass (at most M passes) or accepts the row that grows p (at
    // most M such rows), so the loop ends after at most 2M + 1 rounds.
    for (;;) {
        const int top = st.top, n = st.n, psz = st.psz;
        if (top < 0 && n <= 0) break;
        if (top >= 0) {
            // warp w evaluates positions [32c, 32c + 32) for c = w, w + WARPS, ...
            int gmax = -1, kw = 0;
            for (int c = warp; c <= (top >> 5); c += CB_WARPS) {
                const int j = (c << 5) + lane;
                bool a = false, gr = false;
                if (j <= top) {
                    const int r = U[j];
                    const uint32_t* q = bits + (size_t)r * ns;
                    int inter = 0;
                    for (int k = 0; k < nw; ++k) inter += __popc(p[k] & q[k]);
                    const int qs = qsz[r];
                    a = cb_accept(inter, psz + qs - inter, tau, t_lo);
                    gr = a && inter < qs;
                }
                const uint32_t av = __ballot_sync(0xffffffffu, a);
                const uint32_t gv = __ballot_sync(0xffffffffu, gr);
                if (lane == 0) acc[c] = av;
                kw += __popc(av);
                if (gv) gmax = max(gmax, (c << 5) + 31 - __clz(gv));
            }
            if (lane == 0 && gmax >= 0) atomicMax(&st.g, gmax);
            if (lane == 0 && kw) atomicAdd(&st.kacc, kw);
        }
        __syncthreads();
        if (warp == 0) {
            const int g = st.g;
            int nn = n, out = st.out;
            const int kacc = st.kacc;
            if (top >= 0 && kacc > 0 && kacc <= 8) {
                // few acceptances: lane 0 replays them as the reference removes them
                // (perm += U[j]; U[j] = U.back(); pop), in decreasing position
                const int lo = g < 0 ? 0 : g;
                const int chi = top >> 5, clo = lo >> 5;
                for (int base = chi; base >= clo; base -= 32) {
                    const int c = base - lane;
                    uint32_t v = 0u;
                    if (c >= clo) {
                        v = acc[c];
                        const int hi_bit = top - (c << 5);
                        if (hi_bit < 31) v &= (1u << (hi_bit + 1)) - 1u;
                        const int lo_bit = lo - (c << 5);
                        if (lo_bit > 0) v &= ~((1u << lo_bit) - 1u);
                    }
                    uint32_t live = __ballot_sync(0xffffffffu, v != 0u);
                    while (live) {  // lowest lane = highest word first
                        const int l = __ffs(live) - 1;
                        live &= live - 1u;
                        uint32_t vv = __shfl_sync(0xffffffffu, v, l);
                        if (lane == 0) {
                            const int cc = base - l;
                            while (vv) {
                                const int b = 31 - __clz(vv);
                                vv &= ~(1u << b);
                                const int j = (cc << 5) + b;
                                const int row = U[j];
                                if (j == g) st.prow = row;
                                perm[out++] = (IT)row;
                                U[j] = U[nn - 1];
                                --nn;
                            }
                        }
                    }
                }
                nn = __shfl_sync(0xffffffffu, nn, 0);
                out = __shfl_sync(0xffffffffu, out, 0);
                __syncwarp();
            } else if (top >= 0 && kacc > 8) {
                // The round's acceptances, (g, top] then g, in decreasing position, replayed as
                // the reference removes them (perm += U[j]; U[j] = U.back(); pop), in parallel:
                // the t-th acceptance goes to perm[out + t], and a hole h_t below n - k receives
                // U[chase(n - 1 - t)] (fact 4 of cluster.cu), chase stepping from x to
                // n - 1 - rank(x) while x is a hole of this round. rank() comes from per-word
                // prefix counts of the acceptance bitmap; the reads (positions >= n - k) and the
                // writes (holes < n - k) never meet.
                const int lo = g < 0 ? 0 : g;
                const int chi = top >> 5, clo = lo >> 5;
                auto masked = [&](int c) {
                    uint32_t v = acc[c];
                    const int hi_bit = top - (c << 5);  // bits above it are past top
                    if (hi_bit < 31) v &= (1u << (hi_bit + 1)) - 1u;
                    const int lo_bit = lo - (c << 5);   // bits below it wait for next round
                    if (lo_bit > 0) v &= ~((1u << lo_bit) - 1u);
                    return v;
                };
                int run = 0;  // acceptances in the words above the current chunk
                for (int base = chi; base >= clo; base -= 32) {
                    const int c = base - lane;
                    const int pc = c >= clo ? __popc(masked(c)) : 0;
                    int incl = pc;
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        const int t = __shfl_up_sync(0xffffffffu, incl, o);
                        if (lane >= o) incl += t;
                    }
                    if (c >= clo) wpre[c] = run + incl - pc;
                    run += __shfl_sync(0xffffffffu, incl, 31);
                }
                const int k = run;
                __syncwarp();
                auto rank_of = [&](int x) {  // acceptances above position x (x accepted)
                    const int c = x >> 5;
                    return wpre[c] + __popc(masked(c) & ~((2u << (x & 31)) - 1u));
                };
                auto is_hole = [&](int x) {
                    return x >= lo && x <= top && ((masked(x >> 5) >> (x & 31)) & 1u);
                };
                for (int base = chi; base >= clo; base -= 32) {
                    const int c = base - lane;
                    if (c < clo) continue;
                    uint32_t v = masked(c);
                    int t = wpre[c];
                    while (v) {
                        const int b = 31 - __clz(v);
                        v &= ~(1u << b);
                        const int j = (c << 5) + b;
                        const int row = U[j];
                        if (j == g) st.prow = row;  // joins p below
                        perm[out + t] = (IT)row;
                        if (j < n - k) {
                            int x = n - 1 - t, steps = 0;
                            while (is_hole(x) && steps <= k) {
                                x = n - 1 - rank_of(x);
                                ++steps;
                            }
                            if (steps > k) flag_error(err, DERR_INTERNAL);
                            else U[j] = U[x];
                        }
                        ++t;
                    }
                }
                nn = n - k;
                out += k;
                __syncwarp();
            }
            const int grow_row = (top >= 0 && g >= 0) ? st.prow : -1;
            if (lane == 0) {
                st.g = -1;
                st.kacc = 0;
                if (grow_row >= 0) {  // p grows; rows below g are evaluated again
                    st.top = g - 1;
                    st.prow = grow_row;
                    st.pmode = 1;
                } else if (nn > 0) {  // pass over: next seed = U.back()
                    const int seed = U[nn - 1];
                    perm[out++] = (IT)seed;
                    --nn;
                    st.top = nn - 1;
                    st.prow = seed;
                    st.pmode = 2;
                } else {
                    st.top = -1;
                    st.pmode = 0;
                }
                st.n = nn;
                st.out = out;
            }
            __syncwarp();
            const int mode = st.pmode, row = st.prow;
            if (mode != 0) {
                int sz = 0;
                for (int k = lane; k < nw; k += 32) {
                    const uint32_t q = bits[(size_t)row * ns + k];
                    const uint32_t v = mode == 2 ? q : (p[k] | q);
                    p[k] = v;
                    sz += __popc(v);
                }
                for (int o = 16; o; o >>= 1) sz += __shfl_xor_sync(0xffffffffu, sz, o);
                if (lane == 0) st.psz = sz;
            }
        }
        __syncthreads();
    }
}

// ---- the same sweep over a thread-block cluster ----------------------------------------------
// For matrices whose bitsets exceed one SM but whose row patterns (sorted distinct block
// columns, 2 bytes each) fit the distributed shared memory of a cluster of up to 8 CTAs (the
// hidden-block config: 16384 rows, ~84K pattern entries). CTA k owns rows [kR, (k+1)R): their
// pattern lists, |q| and positions pos[r] live in its shared memory, and it evaluates its own rows
// whose position is in [0, top] against a copy of p held as a bitmap (|p n q| = bits of p at the
// row's columns). Acceptances are marked in CTA 0's acceptance bitmap and the highest growing
// position in CTA 0's state, through distributed shared memory. After a cluster barrier CTA 0
// (which holds U) replays the round exactly as above, writes the new positions of the rows it
// moves into their owners' shared memory, updates p from the owner's pattern, and a second
// cluster barrier publishes it. No global memory is read after the set-up.
constexpr int CS_THREADS = 512;
constexpr int CS_WARPS = CS_THREADS / 32;

__device__ __forceinline__ uint32_t cs_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint32_t cs_mapa(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(cs_u32(p)), "r"(rank));
    return r;
}
__device__ __forceinline__ uint32_t cs_ld32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t cs_ld16(uint32_t a) {
    unsigned short v;
    asm volatile("ld.shared::cluster.u16 %0, [%1];" : "=h"(v) : "r"(a) : "memory");
    return v;
}
__device__ __forceinline__ void cs_st32(uint32_t a, uint32_t v) {
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ void cs_red_or(uint32_t a, uint32_t v) {
    asm volatile("red.shared::cluster.or.b32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ void cs_red_max(uint32_t a, int v) {
    asm volatile("red.shared::cluster.max.s32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ void cs_cluster_sync() {
    __syncwarp();
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                     : "memory");
}
__device__ __forceinline__ uint32_t cs_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

struct CsShared {
    int n, top, out, g, psz, prow, pmode, pad;
};

// Shared-memory layout (identical in every CTA, so mapa finds a peer's copy at the same offset):
// pos[R] int32 | loff[R + 1] uint32 | acc[nmw] uint32 | pl[nw] uint32 | qsz[R] uint16 |
// lq[emax] uint16 | (16-byte aligned) U[M] int32 (used by CTA 0 only)
struct CsLayout {
    size_t pos, loff, acc, pl, qsz, lq, U, total;
};
__host__ __device__ inline CsLayout cs_layout(int64_t M, int64_t R, int64_t nw, int64_t emax) {
    CsLayout L;
    const int64_t nmw = (M + 31) / 32;
    L.pos = 0;
    L.loff = L.pos + 4 * (size_t)R;
    L.acc = L.loff + 4 * (size_t)(R + 1);
    L.pl = L.acc + 4 * (size_t)nmw;
    L.qsz = L.pl + 4 * (size_t)nw;
    L.lq = L.qsz + 2 * (size_t)R;
    L.U = (L.lq + 2 * (size_t)emax + 15) & ~size_t(15);
    L.total = L.U + 4 * (size_t)M;
    return L;
}

template <typename IT>
__global__ void __launch_bounds__(CS_THREADS, 1)
cluster_sweep_kernel(const int64_t* __restrict__ qptr, const int32_t* __restrict__ qcol, int M,
                     int R, int nw, int emax, float tau, float t_lo, IT* __restrict__ perm,
                     unsigned* __restrict__ err) {
    extern __shared__ __align__(16) uint8_t cs_smem[];
    __shared__ CsShared st;
    const CsLayout L = cs_layout(M, R, nw, emax);
    int32_t* pos = reinterpret_cast<int32_t*>(cs_smem + L.pos);
    uint32_t* loff = reinterpret_cast<uint32_t*>(cs_smem + L.loff);
    uint32_t* acc = reinterpret_cast<uint32_t*>(cs_smem + L.acc);
    uint32_t* pl = reinterpret_cast<uint32_t*>(cs_smem + L.pl);
    uint16_t* qsz = reinterpret_cast<uint16_t*>(cs_smem + L.qsz);
    uint16_t* lq = reinterpret_cast<uint16_t*>(cs_smem + L.lq);
    int32_t* U = reinterpret_cast<int32_t*>(cs_smem + L.U);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t rank = cs_rank();
    const int nmw = (M + 31) >> 5;
    const int r0 = (int)min((int64_t)rank * R, (int64_t)M), r1 = (int)min((int64_t)r0 + R, (int64_t)M);
    const int nr = r1 - r0;

    // ---- set-up: this CTA's rows ----
    const int64_t base = qptr[r0];
    const int64_t ne = qptr[r1] - base;
    if (ne > emax) {  // the host sized emax from the same offsets
        if (tid == 0) flag_error(err, DERR_INTERNAL);
    }
    for (int i = tid; i < nr; i += CS_THREADS) {
        const int64_t a = qptr[r0 + i], b = qptr[r0 + i + 1];
        loff[i] = (uint32_t)(a - base);
        qsz[i] = (uint16_t)(b - a);
        pos[i] = r0 + i;  // U starts as [0, 1, ..., M-1]
    }
    if (tid == 0) loff[nr] = (uint32_t)ne;
    for (int64_t e = tid; e < min(ne, (int64_t)emax); e += CS_THREADS) lq[e] = (uint16_t)qcol[base + e];
    for (int i = tid; i < nmw; i += CS_THREADS) acc[i] = 0u;
    if (rank == 0) {
        for (int j = tid; j < M; j += CS_THREADS) U[j] = j;
        if (tid == 0) {
            st.n = M;
            st.top = -1;  // the first iteration only takes the first seed
            st.out = 0;
            st.g = -1;
            st.psz = 0;
            st.prow = -1;
            st.pmode = 0;
        }
        for (int k = tid; k < nw; k += CS_THREADS) pl[k] = 0u;
    }
    __syncthreads();
    cs_cluster_sync();

    const uint32_t st_g_remote = cs_mapa(&st.g, 0);
    // Each iteration either ends a pass (at most M) or accepts the row that grows p (at most M):
    // at most 2M + 1 iterations, the same number in every CTA (all read CTA 0's state).
    for (;;) {
        if (rank != 0) {
            if (tid == 0) {
                st.n = (int)cs_ld32(cs_mapa(&st.n, 0));
                st.top = (int)cs_ld32(cs_mapa(&st.top, 0));
                st.psz = (int)cs_ld32(cs_mapa(&st.psz, 0));
            }
            for (int k = tid; k < nw; k += CS_THREADS) pl[k] = cs_ld32(cs_mapa(&pl[k], 0));
        }
        __syncthreads();
        const int top = st.top, n = st.n, psz = st.psz;
        if (top < 0 && n <= 0) break;
        if (top >= 0) {
            for (int i = tid; i < nr; i += CS_THREADS) {
                const int j = pos[i];
                if (j < 0 || j > top) continue;
                int inter = 0;
                for (uint32_t e = loff[i], e1 = loff[i + 1]; e < e1; ++e) {
                    const uint32_t c = lq[e];
                    inter += (pl[c >> 5] >> (c & 31)) & 1u;
                }
                const int qs = qsz[i];
                if (cb_accept(inter, psz + qs - inter, tau, t_lo)) {
                    cs_red_or(cs_mapa(&acc[j >> 5], 0), 1u << (j & 31));
                    if (inter < qs) cs_red_max(st_g_remote, j);
                }
            }
        }
        cs_cluster_sync();  // acceptances are in CTA 0
        if (rank == 0) {
            const int g = st.g;
            const int lo = g < 0 ? 0 : g;
            if (warp == 0) {
                int nn = n, out = st.out, grow_row = -1;
                if (top >= 0) {
                    const int chi = top >> 5, clo = lo >> 5;
                    for (int bw = chi; bw >= clo; bw -= 32) {
                        const int c = bw - lane;
                        uint32_t v = 0u;
                        if (c >= clo) {
                            v = acc[c];
                            acc[c] = 0u;  // consumed (bits below lo are re-marked next round)
                            const int hi_bit = top - (c << 5);
                            if (hi_bit < 31) v &= (1u << (hi_bit + 1)) - 1u;
                            const int lo_bit = lo - (c << 5);
                            if (lo_bit > 0) v &= ~((1u << lo_bit) - 1u);
                        }
                        uint32_t live = __ballot_sync(0xffffffffu, v != 0u);
                        while (live) {
                            const int l = __ffs(live) - 1;
                            live &= live - 1u;
                            uint32_t vv = __shfl_sync(0xffffffffu, v, l);
                            if (lane == 0) {
                                const int cc = bw - l;
                                while (vv) {
                                    const int b = 31 - __clz(vv);
                                    vv &= ~(1u << b);
                                    const int j = (cc << 5) + b;
                                    const int row = U[j];
                                    if (j == g) grow_row = row;
                                    perm[out++] = (IT)row;
                                    const int moved = U[nn - 1];
                                    U[j] = moved;
                                    --nn;
                                    cs_st32(cs_mapa(&pos[row % R], row / R), (uint32_t)-1);
                                    if (moved != row)
                                        cs_st32(cs_mapa(&pos[moved % R], moved / R), (uint32_t)j);
                                }
                            }
                        }
                    }
                }
                if (lane == 0) {
                    st.g = -1;
                    if (grow_row >= 0) {
                        st.top = g - 1;
                        st.prow = grow_row;
                        st.pmode = 1;
                    } else if (nn > 0) {
                        const int seed = U[nn - 1];
                        perm[out++] = (IT)seed;
                        --nn;
                        cs_st32(cs_mapa(&pos[seed % R], seed / R), (uint32_t)-1);
                        st.top = nn - 1;
                        st.prow = seed;
                        st.pmode = 2;
                    } else {
                        st.top = -1;
                        st.pmode = 0;
                    }
                    st.n = nn;
                    st.out = out;
                }
                __syncwarp();
                const int mode = st.pmode, prow = st.prow;
                if (mode != 0) {
                    if (mode == 2)
                        for (int k = lane; k < nw; k += 32) pl[k] = 0u;
                    __syncwarp();
                    const uint32_t owner = (uint32_t)(prow / R);
                    const int li = prow % R;
                    const uint32_t e0 = cs_ld32(cs_mapa(&loff[li], owner));
                    const uint32_t e1 = cs_ld32(cs_mapa(&loff[li + 1], owner));
                    for (uint32_t e = e0 + lane; e < e1; e += 32) {
                        const uint32_t c = cs_ld16(cs_mapa(&lq[e], owner));
                        atomicOr(&pl[c >> 5], 1u << (c & 31));
                    }
                    __syncwarp();
                    int sz = 0;
                    for (int k = lane; k < nw; k += 32) sz += __popc(pl[k]);
                    for (int o = 16; o; o >>= 1) sz += __shfl_xor_sync(0xffffffffu, sz, o);
                    if (lane == 0) st.psz = sz;
                }
            } else if (top >= 0) {
                // acceptance words below lo>>5 were marked for rows that are evaluated again
                for (int c = tid - 32; c < (lo >> 5); c += CS_THREADS - 32) acc[c] = 0u;
            }
        }
        cs_cluster_sync();  // CTA 0's state, p and the moved rows' positions are published
    }
    cs_cluster_sync();  // no CTA leaves while a peer may still read its shared memory
}

}  // namespace

// Shared memory the bitset kernel needs for M rows of nbc block columns (0 if it cannot run).
size_t cluster_bits_smem(int64_t M, int64_t nbc) {
    if (M <= 0 || M >= (int64_t(1) << 24) || nbc <= 0 || nbc >= 65536) return 0;
    const int64_t nw = (nbc + 31) / 32, ns = nw | 1;
    const int64_t nmw = (M + 31) / 32;
    const size_t head = (((size_t)M * ns * 4 + (size_t)M * 2 + 15) & ~size_t(15));
    return head + (size_t)M * 4 + (size_t)nmw * 8 + (size_t)nw * 4;
}

template <typename IT>
bool cluster_jaccard_bits(Handle& h, int64_t M, int64_t K, const IT* row_ptr, const IT* col_ind,
                          float tau, int64_t w, IT* perm) {
    const int64_t nbc = ceil_div(K, w);
    const size_t smem = cluster_bits_smem(M, nbc);
    int optin = 0;
    XS_CHECK_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, h.device));
    if (smem == 0 || smem + sizeof(CbShared) + 1024 > (size_t)optin) return false;
    auto kern = cluster_bits_kernel<IT>;
    XS_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const float t_lo = (float)((1.0 - (double)tau) - 1.0 / (double)(1 << 22));
    kern<<<1, CB_THREADS, smem, h.stream>>>(row_ptr, col_ind, (int)M, K, w, (int)((nbc + 31) / 32),
                                           tau, t_lo, perm, h.d_err);
    after_launch(h, "cluster_bits");
    return true;
}

// Cluster size and shared memory of the cluster sweep for M rows with the given pattern offsets
// (qptr on the device); 0 CTAs if it does not fit 8 CTAs.
template <typename IT>
bool cluster_jaccard_sweep(Handle& h, int64_t M, int64_t nbc, const int64_t* qptr,
                           const int32_t* qcol, float tau, IT* perm) {
    if (M <= 0 || M >= (int64_t(1) << 24) || nbc <= 0 || nbc >= 65536) return false;
    int optin = 0;
    XS_CHECK_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, h.device));
    const int64_t nw = (nbc + 31) / 32;
    for (int C = 4; C <= 8; C *= 2) {
        const int64_t R = ceil_div(M, C);  // the last CTAs may own no row
        std::vector<int64_t> off(C + 1);
        for (int k = 0; k <= C; ++k) {
            const int64_t r = std::min<int64_t>((int64_t)k * R, M);
            XS_CHECK_CUDA(cudaMemcpyAsync(&off[k], qptr + r, sizeof(int64_t),
                                          cudaMemcpyDeviceToHost, h.stream));
        }
        XS_CHECK_CUDA(cudaStreamSynchronize(h.stream));
        int64_t emax = 1;
        for (int k = 0; k < C; ++k) emax = std::max<int64_t>(emax, off[k + 1] - off[k]);
        if (emax >= (int64_t(1) << 31)) return false;
        const CsLayout L = cs_layout(M, R, nw, emax);
        if (L.total + sizeof(CsShared) + 1024 > (size_t)optin) continue;
        auto kern = cluster_sweep_kernel<IT>;
        XS_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)L.total));
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)C);
        cfg.blockDim = dim3(CS_THREADS);
        cfg.dynamicSmemBytes = L.total;
        cfg.stream = h.stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = (unsigned)C;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int nclusters = 0;
        if (cudaOccupancyMaxActiveClusters(&nclusters, kern, &cfg) != cudaSuccess || nclusters < 1) {
            cudaGetLastError();
            continue;
        }
        const float t_lo = (float)((1.0 - (double)tau) - 1.0 / (double)(1 << 22));
        XS_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, qptr, qcol, (int)M, (int)R, (int)nw,
                                         (int)emax, tau, t_lo, perm, h.d_err));
        after_launch(h, "cluster_sweep");
        return true;
    }
    return false;
}

template bool cluster_jaccard_sweep<int32_t>(Handle&, int64_t, int64_t, const int64_t*,
                                             const int32_t*, float, int32_t*);
template bool cluster_jaccard_sweep<int64_t>(Handle&, int64_t, int64_t, const int64_t*,
                                             const int32_t*, float, int64_t*);
template bool cluster_jaccard_bits<int32_t>(Handle&, int64_t, int64_t, const int32_t*,
                                            const int32_t*, float, int64_t, int32_t*);
template bool cluster_jaccard_bits<int64_t>(Handle&, int64_t, int64_t, const int64_t*,
                                            const int64_t*, float, int64_t, int64_t*);

}  // namespace xspmm_b200
