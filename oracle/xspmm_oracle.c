/*
 * xspmm_oracle.c -- CPU restatement of the xSpMM hot path, used ONLY as a checker.
 *
 * TEST INFRASTRUCTURE. Nothing in the xspmm_b200 product links, loads or calls this file.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it, and always as
 * the thing results are checked against (or the CPU time reported beside the GPU), never as
 * the thing measured or shipped.
 *
 * Pinning: the structural functions (clustering, row permutation, CSR->BCSR, unpermute) are
 * checked bit-for-bit against the reference's own host code compiled from its sources
 * (oracle/Makefile -> oracle/_ref/) and against the golden fixtures that code produced
 * (tests/golden/). The SpMM restatement has no runnable reference (the reference's CUDA path
 * does not compile and it has no CPU SpMM), so C is pinned by this fp64 restatement of the
 * kernel's block loop plus an independent dense cross-check in the tests.
 *
 * All index arrays are int64; callers widen int32 inputs. Values are passed as opaque bytes
 * (esize = 2 for fp16, 4 for fp32) wherever the reference only copies them.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>

typedef int64_t idx_t;

/* ------------------------------------------------------------------------------------------ */
/* Jaccard distance exactly as the reference evaluates it:                                     */
/*   union == 0 ? 0 : 1 - (float)inter / union     (clustering_sylos_labini.cpp:35-46)        */
/* The int union is converted to float before the division, both operands are float.          */
/* ------------------------------------------------------------------------------------------ */
static float jaccard_distance(idx_t inter, idx_t uni) {
    if (uni == 0) return 0.0f;
    volatile float q = (float)inter / (float)uni; /* volatile: keep the IEEE float division */
    volatile float d = 1.0f - q;
    return d;
}

static int popcount64(uint64_t x) { return __builtin_popcountll(x); }

/* ------------------------------------------------------------------------------------------ */
/* Literal clustering: the reference algorithm with dense per-row bitsets.                    */
/* Follows clustering_sylos_labini.cpp:13-33 (quotient rows), :35-46 (distance), :51-120      */
/* (greedy loop: seed = back, scan i = size-1..0, swap-with-back removal, flatten clusters).  */
/* Memory is M * ceil(ceil(K/w)/64) words, so it is for small and medium inputs only.         */
/* Returns 0 on success, -1 on bad arguments, -2 on allocation failure.                       */
/* ------------------------------------------------------------------------------------------ */
int orc_cluster_literal(idx_t M, idx_t K, const idx_t* rp, const idx_t* ci,
                        float tau, idx_t w, idx_t* perm) {
    if (M < 0 || K < 0 || w <= 0) return -1;
    if (M == 0) return 0;
    idx_t nblk = (K + w - 1) / w;
    idx_t words = (nblk + 63) / 64;
    uint64_t* q = (uint64_t*)calloc((size_t)(M * (words ? words : 1)), sizeof(uint64_t));
    idx_t* U = (idx_t*)malloc(sizeof(idx_t) * (size_t)M);
    uint64_t* p = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)(words ? words : 1));
    if (!q || !U || !p) { free(q); free(U); free(p); return -2; }
    for (idx_t i = 0; i < M; ++i)
        for (idx_t j = rp[i]; j < rp[i + 1]; ++j) {
            idx_t b = ci[j] / w;
            q[i * words + b / 64] |= 1ULL << (b % 64);
        }
    for (idx_t i = 0; i < M; ++i) U[i] = i;
    idx_t n = M, out = 0;
    while (n > 0) {
        idx_t seed = U[--n];
        perm[out++] = seed;
        memcpy(p, q + seed * words, sizeof(uint64_t) * (size_t)words);
        for (idx_t i = n - 1; i >= 0; --i) {
            idx_t cand = U[i];
            const uint64_t* qc = q + cand * words;
            idx_t inter = 0, uni = 0;
            for (idx_t k = 0; k < words; ++k) {
                inter += popcount64(p[k] & qc[k]);
                uni += popcount64(p[k] | qc[k]);
            }
            if (jaccard_distance(inter, uni) <= tau) {
                perm[out++] = cand;
                for (idx_t k = 0; k < words; ++k) p[k] |= qc[k];
                U[i] = U[n - 1];
                --n;
            }
        }
    }
    free(q); free(U); free(p);
    return 0;
}

/* ------------------------------------------------------------------------------------------ */
/* Fast exact clustering: same output as orc_cluster_literal, in time proportional to the     */
/* candidates that share a block column with the growing cluster pattern.                      */
/*                                                                                            */
/* Facts it relies on (all follow from the reference loop at clustering_sylos_labini.cpp:86-107):
 *  1. For 0 <= tau < 1 a candidate with no block column in common with p is rejected (d = 1),
 *     unless p and q are both empty (d = 0). So only rows reachable through an inverted index
 *     block-col -> rows of p need evaluating; an empty seed collects exactly the empty rows.
 *  2. For tau >= 1 every candidate is accepted and for tau < 0 or NaN none is; both give the
 *     reversed order M-1..0, which is what the reference loop produces in those cases.
 *  3. During one pass the scan pointer only moves down, and swap-with-back only writes to
 *     positions at or above it, so the positions of the not-yet-scanned rows are fixed for the
 *     whole pass. Candidates can therefore be visited with a max-heap on position.
 *  4. Because of 3, the removals of one pass (U[s] = U.back(); pop, at each accepted position
 *     s in decreasing order) can be replayed after the pass has decided all its members.     */
/* ------------------------------------------------------------------------------------------ */
typedef struct { idx_t pos, row; } heap_ent;

static void heap_push(heap_ent* h, idx_t* hn, heap_ent e) {
    idx_t i = (*hn)++;
    h[i] = e;
    while (i > 0) {
        idx_t par = (i - 1) / 2;
        if (h[par].pos >= h[i].pos) break;
        heap_ent t = h[par]; h[par] = h[i]; h[i] = t; i = par;
    }
}

static heap_ent heap_pop(heap_ent* h, idx_t* hn) {
    heap_ent top = h[0];
    h[0] = h[--(*hn)];
    idx_t i = 0, n = *hn;
    for (;;) {
        idx_t l = 2 * i + 1, r = l + 1, m = i;
        if (l < n && h[l].pos > h[m].pos) m = l;
        if (r < n && h[r].pos > h[m].pos) m = r;
        if (m == i) break;
        heap_ent t = h[m]; h[m] = h[i]; h[i] = t; i = m;
    }
    return top;
}

static int cmp_idx(const void* a, const void* b) {
    idx_t x = *(const idx_t*)a, y = *(const idx_t*)b;
    return (x > y) - (x < y);
}

/* Smallest integer I the Jaccard test can accept for a pattern of size psz: an accepted pair
 * has inter/union >= 1 - tau - 2^-23 (float rounding of the division and the subtraction, each
 * within 2^-24), union >= psz, and inter >= 1 whenever tau < 1 and the pattern is not empty. */
static idx_t min_inter(double t_lo, idx_t psz) {
    double m = ceil(t_lo * (double)psz);
    return m < 1.0 ? 1 : (idx_t)m;
}

typedef struct { idx_t len, col, lo, hi; } col_len;

/* Largest pattern size an accepted row can have against a pattern of size psz. */
static idx_t max_len(double t_lo, idx_t psz) {
    if (t_lo <= 0.0) return INT64_MAX / 4;
    return (idx_t)floor((double)psz / t_lo);
}

/* First index in irow[b0, b1) (sorted by increasing pattern size) whose row has size >= len. */
static idx_t size_bound(const idx_t* irow, const idx_t* qptr, idx_t b0, idx_t b1, idx_t len) {
    while (b0 < b1) {
        idx_t mid = b0 + (b1 - b0) / 2;
        idx_t r = irow[mid];
        if (qptr[r + 1] - qptr[r] < len) b0 = mid + 1; else b1 = mid;
    }
    return b0;
}
static int cmp_col_len(const void* a, const void* b) {
    const col_len* x = (const col_len*)a;
    const col_len* y = (const col_len*)b;
    if (x->len != y->len) return (x->len > y->len) - (x->len < y->len);
    return (x->col > y->col) - (x->col < y->col);
}

int orc_cluster_fast(idx_t M, idx_t K, const idx_t* rp, const idx_t* ci,
                     float tau, idx_t w, idx_t* perm) {
    if (M < 0 || K < 0 || w <= 0) return -1;
    if (M == 0) return 0;
    if (!(tau >= 0.0f) || tau >= 1.0f) { /* fact 2 */
        for (idx_t i = 0; i < M; ++i) perm[i] = M - 1 - i;
        return 0;
    }
    const double t_lo = (1.0 - (double)tau) - 1.0 / (double)(1 << 22);
    idx_t nblk = (K + w - 1) / w;
    idx_t nnz = rp[M] - rp[0];
    idx_t* qptr = (idx_t*)malloc(sizeof(idx_t) * (size_t)(M + 1));
    idx_t* qcol = (idx_t*)malloc(sizeof(idx_t) * (size_t)(nnz > 0 ? nnz : 1));
    idx_t* iptr = (idx_t*)calloc((size_t)(nblk + 2), sizeof(idx_t));
    idx_t* U = (idx_t*)malloc(sizeof(idx_t) * (size_t)M);
    idx_t* pos = (idx_t*)malloc(sizeof(idx_t) * (size_t)M);
    idx_t* stamp = (idx_t*)malloc(sizeof(idx_t) * (size_t)M);
    idx_t* cstamp = (idx_t*)malloc(sizeof(idx_t) * (size_t)(nblk > 0 ? nblk : 1));
    idx_t* ghi = (idx_t*)malloc(sizeof(idx_t) * (size_t)(nblk > 0 ? nblk : 1));
    uint8_t* inP = (uint8_t*)calloc((size_t)(nblk > 0 ? nblk : 1), 1);
    col_len* plist = (col_len*)malloc(sizeof(col_len) * (size_t)(nblk > 0 ? nblk : 1));
    heap_ent* heap = (heap_ent*)malloc(sizeof(heap_ent) * (size_t)M);
    idx_t* holes = (idx_t*)malloc(sizeof(idx_t) * (size_t)M);
    idx_t* irow = NULL;
    idx_t* fill = NULL;
    int rc = -2;
    if (!qptr || !qcol || !iptr || !U || !pos || !stamp || !cstamp || !ghi || !inP || !plist ||
        !heap || !holes)
        goto done;
    /* per-row sorted distinct block columns (the reference's quotient row, as a list) */
    idx_t qn = 0;
    qptr[0] = 0;
    for (idx_t r = 0; r < M; ++r) {
        idx_t s0 = qn;
        for (idx_t j = rp[r]; j < rp[r + 1]; ++j) qcol[qn++] = ci[j] / w;
        qsort(qcol + s0, (size_t)(qn - s0), sizeof(idx_t), cmp_idx);
        idx_t u = s0;
        for (idx_t j = s0; j < qn; ++j)
            if (j == s0 || qcol[j] != qcol[u - 1]) qcol[u++] = qcol[j];
        qn = u;
        qptr[r + 1] = qn;
    }
    /* inverted index block column -> rows, each list ordered by increasing row pattern size so
     * the rows a size window admits form one contiguous slice */
    for (idx_t j = 0; j < qn; ++j) iptr[qcol[j] + 1]++;
    for (idx_t b = 0; b < nblk; ++b) iptr[b + 1] += iptr[b];
    irow = (idx_t*)malloc(sizeof(idx_t) * (size_t)(qn > 0 ? qn : 1));
    fill = (idx_t*)malloc(sizeof(idx_t) * (size_t)(nblk > 0 ? nblk : 1));
    if (!irow || !fill) goto done;
    {
        /* counting sort of rows by increasing pattern size, then bucket by column */
        idx_t maxlen = 0;
        for (idx_t r = 0; r < M; ++r)
            if (qptr[r + 1] - qptr[r] > maxlen) maxlen = qptr[r + 1] - qptr[r];
        idx_t* cnt = (idx_t*)calloc((size_t)(maxlen + 2), sizeof(idx_t));
        idx_t* order = (idx_t*)malloc(sizeof(idx_t) * (size_t)M);
        if (!cnt || !order) { free(cnt); free(order); goto done; }
        for (idx_t r = 0; r < M; ++r) cnt[qptr[r + 1] - qptr[r] + 1]++;
        for (idx_t l = 0; l <= maxlen; ++l) cnt[l + 1] += cnt[l];
        for (idx_t r = 0; r < M; ++r) order[cnt[qptr[r + 1] - qptr[r]]++] = r;
        memcpy(fill, iptr, sizeof(idx_t) * (size_t)nblk);
        for (idx_t t = 0; t < M; ++t) {
            idx_t r = order[t];
            for (idx_t j = qptr[r]; j < qptr[r + 1]; ++j) irow[fill[qcol[j]]++] = r;
        }
        free(cnt); free(order);
    }

    for (idx_t i = 0; i < M; ++i) { U[i] = i; pos[i] = i; stamp[i] = -1; }
    for (idx_t b = 0; b < nblk; ++b) cstamp[b] = -1;
    idx_t n = M, out = 0, cid = 0;
    while (n > 0) {
        idx_t seed = U[--n];
        pos[seed] = -1;
        perm[out++] = seed;
        idx_t k = 0; /* number of accepted rows (holes) this pass */
        if (qptr[seed + 1] == qptr[seed]) {
            /* fact 1: an empty pattern accepts exactly the empty rows, in scan order */
            for (idx_t i = n - 1; i >= 0; --i) {
                idx_t r = U[i];
                if (qptr[r + 1] == qptr[r]) { holes[k++] = i; perm[out++] = r; }
            }
        } else {
            idx_t pcount = 0, hn = 0, limit = n;
            for (idx_t j = qptr[seed]; j < qptr[seed + 1]; ++j) {
                idx_t b = qcol[j];
                inP[b] = 1;
                plist[pcount++].col = b;
            }
            int grown = 1;
            for (;;) {
                if (grown) {
                    /* An accepted row q shares >= m columns with p and has m <= |q| <= ub
                     * (inter >= t|p| and |q| <= union <= inter/t). So it meets every subset of
                     * p with pcount - m + 1 columns: gather through the columns whose size
                     * window holds the fewest rows. Both bounds only widen upwards as p grows,
                     * so each column keeps the end of the slice it has gathered so far. */
                    idx_t m = min_inter(t_lo, pcount);
                    idx_t ub = max_len(t_lo, pcount);
                    for (idx_t t = 0; t < pcount; ++t) {
                        idx_t b = plist[t].col;
                        idx_t lo = size_bound(irow, qptr, iptr[b], iptr[b + 1], m);
                        idx_t hi = size_bound(irow, qptr, iptr[b], iptr[b + 1], ub + 1);
                        plist[t].len = hi - lo;
                        plist[t].lo = lo;
                        plist[t].hi = hi;
                    }
                    qsort(plist, (size_t)pcount, sizeof(col_len), cmp_col_len);
                    idx_t pre = pcount - m + 1;
                    for (idx_t t = 0; t < pre; ++t) {
                        idx_t b = plist[t].col;
                        if (cstamp[b] != cid) { cstamp[b] = cid; ghi[b] = plist[t].lo; }
                        idx_t e0 = ghi[b] > plist[t].lo ? ghi[b] : plist[t].lo;
                        for (idx_t e = e0; e < plist[t].hi; ++e) {
                            idx_t r = irow[e];
                            if (pos[r] >= 0 && pos[r] < limit && stamp[r] != cid) {
                                stamp[r] = cid;
                                heap_ent he = {pos[r], r};
                                heap_push(heap, &hn, he);
                            }
                        }
                        if (plist[t].hi > ghi[b]) ghi[b] = plist[t].hi;
                    }
                    grown = 0;
                }
                if (hn == 0) break;
                heap_ent he = heap_pop(heap, &hn);
                idx_t r = he.row, s = he.pos;
                idx_t inter = 0, len = qptr[r + 1] - qptr[r];
                for (idx_t j = qptr[r]; j < qptr[r + 1]; ++j) inter += inP[qcol[j]];
                idx_t uni = pcount + len - inter;
                if (jaccard_distance(inter, uni) <= tau) {
                    holes[k++] = s;
                    perm[out++] = r;
                    pos[r] = -1; /* accepted: never a candidate again */
                    limit = s;
                    for (idx_t j = qptr[r]; j < qptr[r + 1]; ++j) {
                        idx_t b = qcol[j];
                        if (!inP[b]) {
                            inP[b] = 1;
                            plist[pcount++].col = b;
                            grown = 1;
                        }
                    }
                }
            }
            for (idx_t t = 0; t < pcount; ++t) inP[plist[t].col] = 0;
        }
        /* Removal of this pass's rows, replayed in decreasing position order exactly as the
         * reference does it (U[s] = U.back(); pop). holes[] is already in that order; an
         * element can move more than once (back -> hole -> back again -> lower hole). */
        idx_t cur = n;
        for (idx_t t = 0; t < k; ++t) {
            idx_t s = holes[t], r = U[cur - 1];
            U[s] = r;
            pos[r] = s;
            --cur;
        }
        for (idx_t t = out - k; t < out; ++t) pos[perm[t]] = -1; /* accepted rows left U */
        n = cur;
        ++cid;
    }
    rc = 0;
done:
    free(qptr); free(qcol); free(iptr); free(U); free(pos); free(stamp); free(cstamp); free(ghi);
    free(inP); free(plist); free(heap); free(holes); free(irow); free(fill);
    return rc;
}

/* ------------------------------------------------------------------------------------------ */
/* Row permutation: new row i = old row perm[i], entries in their original order.            */
/* Follows clustering_sylos_labini.cpp:125-178 (CPU) and permutation.hpp:15-66 +              */
/* mtx_permutation.cu:12-65 (GPU: lengths, exclusive scan, last = nnz, copy).                 */
/* ------------------------------------------------------------------------------------------ */
int orc_permute_rows(idx_t M, const idx_t* rp, const idx_t* ci, const void* vals, int esize,
                     const idx_t* perm, idx_t* out_rp, idx_t* out_ci, void* out_vals) {
    if (M < 0 || esize <= 0) return -1;
    idx_t o = 0;
    out_rp[0] = 0;
    for (idx_t i = 0; i < M; ++i) {
        idx_t r = perm[i];
        if (r < 0 || r >= M) return -1;
        idx_t len = rp[r + 1] - rp[r];
        memcpy(out_ci + o, ci + rp[r], sizeof(idx_t) * (size_t)len);
        memcpy((char*)out_vals + (size_t)o * esize, (const char*)vals + (size_t)rp[r] * esize,
               (size_t)len * esize);
        o += len;
        out_rp[i + 1] = o;
    }
    return 0;
}

/* ------------------------------------------------------------------------------------------ */
/* CSR -> BCSR, split in two calls so the caller can size the outputs.                        */
/* Follows conversion.cpp:8-100: per block row the distinct block columns of its rows, sorted */
/* ascending (:42-64); cumulative row_ptr (:66-68); values zero-filled, then every CSR entry  */
/* written in CSR order to (row_ptr[br] + rank(bc)) * rb*cb + (r % rb) * cb + c % cb, so a    */
/* duplicate (row, col) keeps its last value (:75-91).                                        */
/* ------------------------------------------------------------------------------------------ */
static idx_t distinct_block_cols(idx_t M, const idx_t* rp, const idx_t* ci, idx_t rb, idx_t cb,
                                 idx_t br, idx_t* mark, idx_t* list) {
    idx_t r0 = br * rb, r1 = r0 + rb < M ? r0 + rb : M, n = 0;
    for (idx_t r = r0; r < r1; ++r)
        for (idx_t j = rp[r]; j < rp[r + 1]; ++j) {
            idx_t b = ci[j] / cb;
            if (mark[b] != br) { mark[b] = br; list[n++] = b; }
        }
    qsort(list, (size_t)n, sizeof(idx_t), cmp_idx);
    return n;
}

/* Writes bcsr_row_ptr[nbr+1]; returns nnzb (>= 0) or a negative error. */
idx_t orc_csr_to_bcsr_count(idx_t M, idx_t K, const idx_t* rp, const idx_t* ci,
                            idx_t rb, idx_t cb, idx_t* brp) {
    if (M < 0 || K < 0 || rb <= 0 || cb <= 0) return -1;
    idx_t nbr = (M + rb - 1) / rb, nbc = (K + cb - 1) / cb;
    idx_t* mark = (idx_t*)malloc(sizeof(idx_t) * (size_t)(nbc > 0 ? nbc : 1));
    idx_t* list = (idx_t*)malloc(sizeof(idx_t) * (size_t)(nbc > 0 ? nbc : 1));
    if (!mark || !list) { free(mark); free(list); return -2; }
    for (idx_t b = 0; b < nbc; ++b) mark[b] = -1;
    brp[0] = 0;
    for (idx_t br = 0; br < nbr; ++br)
        brp[br + 1] = brp[br] + distinct_block_cols(M, rp, ci, rb, cb, br, mark, list);
    free(mark); free(list);
    return brp[nbr];
}

int orc_csr_to_bcsr_fill(idx_t M, idx_t K, const idx_t* rp, const idx_t* ci, const void* vals,
                         int esize, idx_t rb, idx_t cb, const idx_t* brp, idx_t* bci,
                         void* bvals) {
    if (M < 0 || K < 0 || rb <= 0 || cb <= 0 || esize <= 0) return -1;
    idx_t nbr = (M + rb - 1) / rb, nbc = (K + cb - 1) / cb;
    idx_t* mark = (idx_t*)malloc(sizeof(idx_t) * (size_t)(nbc > 0 ? nbc : 1));
    idx_t* list = (idx_t*)malloc(sizeof(idx_t) * (size_t)(nbc > 0 ? nbc : 1));
    idx_t* rank = (idx_t*)malloc(sizeof(idx_t) * (size_t)(nbc > 0 ? nbc : 1));
    if (!mark || !list || !rank) { free(mark); free(list); free(rank); return -2; }
    for (idx_t b = 0; b < nbc; ++b) mark[b] = -1;
    idx_t bs = rb * cb;
    memset(bvals, 0, (size_t)(brp[nbr] * bs) * (size_t)esize);
    for (idx_t br = 0; br < nbr; ++br) {
        idx_t n = distinct_block_cols(M, rp, ci, rb, cb, br, mark, list);
        for (idx_t t = 0; t < n; ++t) { bci[brp[br] + t] = list[t]; rank[list[t]] = t; }
        idx_t r0 = br * rb, r1 = r0 + rb < M ? r0 + rb : M;
        for (idx_t r = r0; r < r1; ++r)
            for (idx_t j = rp[r]; j < rp[r + 1]; ++j) {
                idx_t c = ci[j];
                idx_t flat = (brp[br] + rank[c / cb]) * bs + (r % rb) * cb + c % cb;
                memcpy((char*)bvals + (size_t)flat * esize, (const char*)vals + (size_t)j * esize,
                       (size_t)esize);
            }
    }
    free(mark); free(list); free(rank);
    return 0;
}

/* ------------------------------------------------------------------------------------------ */
/* Tier-1 BCSR SpMM, restated from the kernel's block loop (spmm_math.hpp:59-122):            */
/*   C[rb*br + i, n] = sum over blocks j of row br (in col_ind order), k in [0, cb):           */
/*                     A_j[i, k] * B[cb*col_j + k, n]                                          */
/* every row of C is written (block rows without blocks give zeros, spmm_math.hpp:55-57 and   */
/* :116-122). fp16 inputs are widened exactly by the caller; accumulation here is fp64.       */
/* B rows at or beyond K and C rows at or beyond M are not touched (the reference kernel has  */
/* no guards there; this restatement defines the zero-padded meaning).                        */
/* ------------------------------------------------------------------------------------------ */
int orc_bcsr_spmm_f64(idx_t M, idx_t K, idx_t N, idx_t rb, idx_t cb, const idx_t* brp,
                      const idx_t* bci, const float* bvals, const float* B, double* C) {
    if (M < 0 || K < 0 || N < 0 || rb <= 0 || cb <= 0) return -1;
    idx_t nbr = (M + rb - 1) / rb, bs = rb * cb;
#pragma omp parallel for schedule(dynamic, 4)
    for (idx_t br = 0; br < nbr; ++br) {
        idx_t r0 = br * rb;
        double* acc = (double*)calloc((size_t)(rb * N > 0 ? rb * N : 1), sizeof(double));
        for (idx_t j = brp[br]; j < brp[br + 1]; ++j) {
            const float* a = bvals + j * bs;
            idx_t k0 = bci[j] * cb;
            for (idx_t i = 0; i < rb; ++i)
                for (idx_t k = 0; k < cb; ++k) {
                    double av = (double)a[i * cb + k];
                    if (k0 + k >= K) continue;
                    const float* brow = B + (k0 + k) * N;
                    double* crow = acc + i * N;
                    for (idx_t n = 0; n < N; ++n) crow[n] += av * (double)brow[n];
                }
        }
        for (idx_t i = 0; i < rb && r0 + i < M; ++i)
            memcpy(C + (r0 + i) * N, acc + i * N, sizeof(double) * (size_t)N);
        free(acc);
    }
    return 0;
}

/* ------------------------------------------------------------------------------------------ */
/* Dense unpermute: out[perm[r] * N + c] = in[r * N + c]  (permutation.hpp:89-108).            */
/* ------------------------------------------------------------------------------------------ */
int orc_unpermute_dense(idx_t M, idx_t N, const idx_t* perm, const void* in, void* out, int esize) {
    if (M < 0 || N < 0 || esize <= 0) return -1;
    for (idx_t r = 0; r < M; ++r) {
        idx_t o = perm[r];
        if (o < 0 || o >= M) return -1;
        memcpy((char*)out + (size_t)(o * N) * esize, (const char*)in + (size_t)(r * N) * esize,
               (size_t)(N * esize));
    }
    return 0;
}

/* Number of OpenMP threads the SpMM restatement uses (1 when built without OpenMP). */
int orc_num_threads(void) {
#ifdef _OPENMP
    extern int omp_get_max_threads(void);
    return omp_get_max_threads();
#else
    return 1;
#endif
}
