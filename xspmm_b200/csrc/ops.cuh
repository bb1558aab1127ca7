// ops.cuh -- internal host entry points of the library, one per hot-path operation. The C ABI in
// capi.cu validates arguments, picks the instantiation and calls these; the Tier-2 pipeline
// composes them.
#pragma once

#include "common.cuh"

#include <new>
#include <vector>

namespace xspmm_b200 {

// Tier-1 BCSR SpMM (16x16 blocks). VT = __half or float; C is fp32. row_map may be null.
template <typename VT, typename IT>
void bcsr_spmm(Handle& h, int64_t nbr, int64_t nbc, int64_t nnzb, const IT* row_ptr,
               const IT* col_ind, const VT* values, const VT* B, float* C, int64_t M, int64_t K,
               int64_t N, const IT* row_map);

// Tier-1 on tcgen05 (block rows stacked to M=128, TMA-fed); tc_supported says whether the
// shapes and alignments allow it.
bool tc_supported(int64_t nbr, int64_t nbc, int64_t nnzb, const void* vals, const void* B,
                  const void* C, int64_t N);
// Tier-1 for BCSR block shapes other than 16x16 (spmm_blocks.cu): rb x cb blocks.
template <typename VT, typename IT>
void bcsr_spmm_blocks(Handle& h, int64_t nbr, int64_t rb, int64_t cb, const IT* rp, const IT* ci,
                      const VT* v, const VT* B, float* C, int64_t M, int64_t K, int64_t N,
                      const IT* map);
// 16-bit values: fp16, or bf16 when bf16 is set (the bits are read through __half pointers).
template <typename IT>
void bcsr_spmm_tc(Handle& h, int64_t nbr, int64_t nbc, int64_t nnzb, const IT* rp, const IT* ci,
                  const __half* vals, const __half* B, float* C, int64_t M, int64_t K, int64_t N,
                  const IT* map, bool bf16);

// What the tcgen05 kernel derives from A once: per group of 8 block rows the union of block
// columns (gptr/gcol) and the stacked A tiles packed 128 x 16 per union entry, with their TMA map.
struct TcPrep {
    int64_t ngroups = 0, bound = 0;
    DevBuf<int64_t> gptr;
    DevBuf<int32_t> gcol;
    DevBuf<__half> apk;  // 4 KB per union entry, laid out as the MMA reads it from shared memory
};
template <typename IT>
void tc_prepare(Handle& h, int64_t nbr, int64_t nbc, int64_t nnzb, const IT* rp, const IT* ci,
                const __half* vals, TcPrep& out);
template <typename IT>
void tc_execute(Handle& h, const TcPrep& p, const __half* B, float* C, int64_t M, int64_t K,
                int64_t N, const IT* map, bool bf16);
bool tc_preferred(int64_t nbr, int64_t nbc, int64_t nnzb);

// The mma.sync Tier-1 kernel, without the automatic choice of tcgen05.
// Work list of the mma.sync kernel built once by a plan: block rows in execution order, long
// block rows cut into slices whose partial sums are reduced in a fixed order afterwards.
struct MmaItem {
    int64_t jb;    // first block
    int32_t br;    // block row
    int32_t nblk;  // blocks in this item
    int32_t slot;  // workspace slot of a slice of a split row, -1 for a whole row
    int32_t pad;
};
struct MmaWork {
    DevBuf<MmaItem> items;
    DevBuf<int32_t> long_rows, first_slot;
    int64_t nitems = 0, nlong = 0, nslots = 0;
    bool empty = false;  // every block row was left to another kernel: nothing to launch
};
// keep (optional, host): block rows to include (1) or leave to another kernel (0).
template <typename IT>
void mma_work_build(Handle& h, int64_t nbr, int64_t nbc, int64_t nnzb, const IT* rp,
                    const IT* ci, bool by_first_col, MmaWork& out,
                    const std::vector<uint8_t>* keep = nullptr);
template <typename IT>
void bcsr_spmm_mma_f16(Handle& h, int64_t nbr, const IT* rp, const IT* ci, const __half* v,
                       const __half* B, float* C, int64_t M, int64_t K, int64_t N, const IT* map,
                       const MmaWork* work, bool bf16);
// Execution order of block rows for the mma.sync kernel: sorted by first block column.
template <typename IT>
void block_row_order(Handle& h, int64_t nbr, int64_t nbc, const IT* rp, const IT* ci,
                     DevBuf<int32_t>& order);

// Block rows whose blocks are nearly empty, taken off the block kernels by a plan: their
// nonzeros extracted per row in column order (spmm_sparse.cu) and multiplied by gathering one B
// row per nonzero. dense_br (host) marks the block rows that stay on the block kernels.
// Nonzeros per block (of 256) above which a block row stays on the block kernels: the fp16
// tensor-core kernels cost little per block; the fp32 SIMT kernel pays 16 fp64 FMAs per nonzero
// column of a block, which a gather beats until blocks are about a quarter full.
constexpr int64_t SP_DENSE_NNZ_F16 = 12;
constexpr int64_t SP_DENSE_NNZ_F32 = 64;
struct SparseChunk {
    int64_t e0, e1;  // nonzeros [e0, e1) of row `row`, partial sum into workspace slot `slot`
    int32_t row, slot;
};
struct SpRow {  // a row of the gather kernels with at most SP_LONG nonzeros
    int64_t e0;   // its first nonzero
    int32_t row, cnt;
};
struct SpTask {  // consecutive short rows [first, first + nrows) taken by one warp (nrows <= 32)
    int32_t first, nrows;
};
// Tensor-core gather (16-bit values): the nonzeros of a task as k-steps of 16 stream positions.
// col[i] is the B row of position i (-1: padding). Positions 2p and 2p+1 share two words:
// pair[2p] = value(2p) | value(2p+1) << 16 (their 16 bits), pair[2p+1] = onehot(2p) |
// onehot(2p+1) << 16 with onehot = 1 << (row offset in the task's block row, 0..15), 0 for padding.
struct SpKStep {
    int32_t col[16];
    uint32_t pair[16];
};
struct SpMmaTask {
    int64_t ks0;    // first k-step record
    int64_t e0;     // chunk tasks: first nonzero of the chunk
    int32_t nks;    // k-steps
    int32_t out;    // >= 0: block row, rows 16*out + i for the bits i of mask; < 0: chunk of a long
                    // row whose fp64 partial goes to workspace slot -(out + 1)
    uint32_t mask;  // block-row tasks: the rows the task owns (and writes, zeros included)
    int32_t nnz;    // chunk tasks: nonzeros in the chunk
};
struct SparseRows {
    std::vector<uint8_t> dense_br;
    std::vector<int64_t> host_rp;  // the block row pointers, read back once at build
    DevBuf<int64_t> rptr;  // [M+1]: row r's nonzeros are [rptr[r], rptr[r+1]) (empty if dense)
    DevBuf<int32_t> col;
    DevBuf<uint8_t> val;   // nnz values of the matrix's value type
    DevBuf<int32_t> brs, long_rows;
    DevBuf<SpRow> short_rows;
    DevBuf<SpTask> tasks;          // short rows packed into warp tasks
    DevBuf<SparseChunk> chunks;    // long rows cut into chunks
    DevBuf<int32_t> long_first;    // [nlong+1] first chunk of each long row
    int64_t nbrs = 0, nnz = 0, nshort = 0, ntasks = 0, nlong = 0, nchunks = 0;
    int64_t nplain_tasks = 0;      // tasks [0, nplain_tasks) hold rows of <= SP_PLAIN nonzeros
    // tensor-core gather (16-bit values only)
    DevBuf<SpKStep> ksteps;
    DevBuf<SpMmaTask> mtasks;      // chunk tasks of the long rows first, then block-row tasks
    DevBuf<int32_t> mlong_rows;    // its rows cut into chunks (more than SPM_ROW_MAX nonzeros)
    DevBuf<int32_t> mlong_first;   // [nmlong+1] first workspace slot of each of them
    DevBuf<int32_t> mranges;       // [nmranges+1]: warp ranges of consecutive tasks
    int64_t nksteps = 0, nmtasks = 0, nmslots = 0, nmlong = 0, nmranges = 0;
    bool mma_built = false;
};
template <typename VT, typename IT>
void sparse_rows_build(Handle& h, int64_t nbr, int64_t M, const IT* rp, const IT* ci,
                       const VT* v, int64_t dense_nnz, SparseRows& out);
template <typename VT, typename IT>
void sparse_rows_execute(Handle& h, const SparseRows& sp, const VT* B, float* C, int64_t M,
                         int64_t K, int64_t N, const IT* map);
// Work list of the fp32 block kernel inside a plan (spmm_f32.cu): the block rows to compute
// (those a SparseRows split leaves), each a piece of blocks [j0, j1); block rows far above the
// average length are cut into several pieces whose fp64 partials (workspace slots) are added in
// piece order afterwards.
struct F32Piece {
    int64_t j0, j1;
    int32_t br, slot;  // slot -1: the piece is the whole block row and writes C itself
};
struct F32Work {
    DevBuf<F32Piece> pieces;
    DevBuf<int32_t> long_br, long_first;  // cut block rows, [nlong+1] first slot of each
    int64_t npieces = 0, nlong = 0, nslots = 0;
    bool built = false;
};
// hrp: the block row pointers on the host (nbr+1); keep: block rows to include (all if null).
void f32_work_build(Handle& h, int64_t nbr, const std::vector<int64_t>& hrp,
                    const std::vector<uint8_t>* keep, F32Work& out);
template <typename IT>
void bcsr_spmm_f32_work(Handle& h, const F32Work& w, const IT* rp, const IT* ci, const float* v,
                        const float* B, float* C, int64_t M, int64_t K, int64_t N, const IT* map);

// Which Tier-1 fp16 kernel runs: the handle's setting (xspmm_set_tier1_kernel) if not auto, else
// the environment XSPMM_TIER1_KERNEL = mma | tc | auto (default auto).
enum class Tier1Kernel { Auto, Mma, Tc };
Tier1Kernel tier1_kernel_choice(const Handle& h);

// The same clustering with every row's block-column bitset in one CTA's shared memory; returns
// false (and does nothing) when they do not fit.
template <typename IT>
bool cluster_jaccard_bits(Handle& h, int64_t M, int64_t K, const IT* row_ptr, const IT* col_ind,
                          float tau, int64_t w, IT* perm);
size_t cluster_bits_smem(int64_t M, int64_t nbc);
// The same clustering with the row patterns (qptr/qcol: sorted distinct block columns per row)
// spread over the shared memory of a thread-block cluster of 4 or 8 CTAs; false if they do not fit.
template <typename IT>
bool cluster_jaccard_sweep(Handle& h, int64_t M, int64_t nbc, const int64_t* qptr,
                           const int32_t* qcol, float tau, IT* perm);

// Exact greedy Jaccard clustering (writes perm[M]).
template <typename IT>
void cluster_jaccard(Handle& h, int64_t M, int64_t K, int64_t nnz, const IT* row_ptr,
                     const IT* col_ind, float tau, int64_t w, IT* perm);

// CSR row permutation into caller-provided arrays. check = validate perm and synchronize.
template <typename VT, typename IT>
void permute_rows(Handle& h, int64_t M, int64_t nnz, const IT* row_ptr, const IT* col_ind,
                  const VT* values, const IT* perm, IT* out_row_ptr, IT* out_col_ind,
                  VT* out_values, bool check);

// permute_rows with caller-provided scratch instead of allocations: seen = ceil(M/32) words
// (cleared here), scan scratch of scan_scratch_elems(M) elements. Validates and synchronizes.
template <typename VT, typename IT>
void permute_rows_scratch(Handle& h, int64_t M, int64_t nnz, const IT* row_ptr, const IT* col_ind,
                          const VT* values, const IT* perm, IT* out_row_ptr, IT* out_col_ind,
                          VT* out_values, unsigned* seen, IT* scan_scratch,
                          int64_t scan_scratch_elems);

// CSR -> BCSR: count (writes brp[nbr+1], returns nnzb, synchronizes) and fill.
template <typename IT>
int64_t csr_to_bcsr_count(Handle& h, int64_t M, int64_t K, int64_t nnz, const IT* row_ptr,
                          const IT* col_ind, int64_t rb, int64_t cb, IT* brp);
template <typename VT, typename IT>
void csr_to_bcsr_fill(Handle& h, int64_t M, int64_t K, int64_t nnz, const IT* row_ptr,
                      const IT* col_ind, const VT* values, int64_t rb, int64_t cb, const IT* brp,
                      IT* bci, VT* bvals);

// Dense unpermute out[perm[r]] = in[r] (rows of N elements).
template <typename VT, typename IT>
void unpermute_dense(Handle& h, const VT* in, VT* out, const IT* perm, int64_t M, int64_t N,
                     bool check);

// Tier-2 pipeline.
template <typename VT, typename IT>
void spmm_csr_pipeline(Handle& h, int64_t M, int64_t K, int64_t nnz, const IT* row_ptr,
                       const IT* col_ind, const VT* values, const VT* B, float* C, int64_t N,
                       int64_t hw, bool clustering, xspmm_timings_t* timings);

}  // namespace xspmm_b200

// ------------------------------------------------------------------------------------------------
// Pieces shared by the files that define extern "C" entry points.
// ------------------------------------------------------------------------------------------------
#define XS_API extern "C" __attribute__((visibility("default")))

struct xspmm_handle_s {
    xspmm_b200::Handle h;
    bool destroyed = false;
    int live_plans = 0;  // plans built on this handle and not yet destroyed
};

namespace xspmm_b200 {

// Runs f, turning exceptions into a status code and the calling thread's last-error message.
template <typename F>
xspmm_status_t guarded(F&& f) {
    try {
        f();
        return XSPMM_STATUS_OK;
    } catch (const Error& e) {
        set_last_error(e.what());
        return e.status;
    } catch (const std::bad_alloc&) {
        set_last_error("host allocation failed");
        return XSPMM_STATUS_OUT_OF_MEMORY;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return XSPMM_STATUS_INTERNAL;
    } catch (...) {
        set_last_error("unknown exception");
        return XSPMM_STATUS_INTERNAL;
    }
}

inline Handle& H(xspmm_handle_t h) {
    XS_REQUIRE(h != nullptr && !h->destroyed, XSPMM_STATUS_INVALID_ARGUMENT, "null handle");
    return h->h;
}

inline void need(bool ok, const char* what) {
    XS_REQUIRE(ok, XSPMM_STATUS_INVALID_ARGUMENT, what);
}

}  // namespace xspmm_b200
