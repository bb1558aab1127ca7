// plan.cuh -- what the SpMM derives from A once, kept on the device for repeated products.
//
// The reference recomputes clustering, permutation and CSR->BCSR on every Tier-2 call
// (src/cuda/unstructured_mtx_mul.cu:56-130) and leaves reuse to callers of Tier 1 (README.md:127,
// "amortizing clustering time over thousands of iterations"). A plan holds the result of those
// stages -- the clustering permutation, the permuted BCSR matrix and, for the tcgen05 kernel, the
// stacked 128 x 16 A tiles -- so that each product afterwards is the Tier-1 kernel alone.
// The Tier-2 entry point builds a plan, executes it once and drops it.
#pragma once
#include <memory>
#include <type_traits>
#include <vector>

#include "ops.cuh"

struct xspmm_dist_comm_s;

namespace xspmm_b200 {

struct PlanBase {
    int64_t M = 0, K = 0, nbr = 0, nbc = 0, nnzb = 0;
    bool clustered = false;
    int value_bytes = 0;
    virtual ~PlanBase() = default;
    // C (M x N, fp32, row-major) = A * B (K x N, row-major, the plan's value type), rows of C in
    // the caller's order.
    virtual void execute(Handle& h, const void* B, float* C, int64_t N) = 0;
    // Builds what the tcgen05 kernel needs now instead of at the first product that takes it.
    virtual void prepare_tc(Handle& h) = 0;
    virtual bool tc_ready() const = 0;
    virtual int64_t tc_tiles() const = 0;
    virtual int64_t device_bytes() const = 0;
    virtual void rebind_stream(cudaStream_t s) = 0;
};

template <typename VT, typename IT>
struct Plan final : PlanBase {
    DevBuf<IT> perm, brp, bci;  // owned when built from CSR
    DevBuf<VT> bv;
    const IT* rp = nullptr;     // the BCSR arrays the product reads (owned or the caller's)
    const IT* ci = nullptr;
    const VT* v = nullptr;
    TcPrep tc;
    bool tc_built = false;
    MmaWork work;  // work list of the mma.sync kernel (order, split long rows)
    bool work_built = false;
    SparseRows sparse;  // block rows of nearly empty blocks, on the gather kernels
    bool sparse_built = false;
    F32Work f32work;  // fp32: the block rows left to the SIMT block kernel, long ones cut
    bool work_sorted = false;
    bool one_shot = false;  // built for a single product (the Tier-2 call)

    void execute(Handle& h, const void* B, float* C, int64_t N) override;
    void prepare_tc(Handle& h) override;
    bool tc_ready() const override { return tc_built; }
    int64_t tc_tiles() const override { return tc_built ? tc.bound : 0; }
    int64_t device_bytes() const override {
        return (int64_t)(perm.n + brp.n + bci.n) * (int64_t)sizeof(IT) +
               (int64_t)work.items.n * (int64_t)sizeof(MmaItem) +
               (int64_t)(work.long_rows.n + work.first_slot.n) * (int64_t)sizeof(int32_t) +
               (int64_t)bv.n * (int64_t)sizeof(VT) +
               (int64_t)(sparse.rptr.n * sizeof(int64_t) + sparse.col.n * sizeof(int32_t) +
                         sparse.val.n +
                         (sparse.brs.n + sparse.long_rows.n + sparse.long_first.n) *
                             sizeof(int32_t) +
                         sparse.short_rows.n * sizeof(SpRow) +
                         sparse.tasks.n * sizeof(SpTask) +
                         sparse.chunks.n * sizeof(SparseChunk) +
                         sparse.ksteps.n * sizeof(SpKStep) + sparse.mtasks.n * sizeof(SpMmaTask) +
                         (sparse.mlong_first.n + sparse.mlong_rows.n + sparse.mranges.n) * sizeof(int32_t)) +
               (int64_t)(f32work.pieces.n * sizeof(F32Piece) +
                         (f32work.long_br.n + f32work.long_first.n) * sizeof(int32_t)) +
               (int64_t)(tc.gptr.n * sizeof(int64_t) + tc.gcol.n * sizeof(int32_t) +
                         tc.apk.n * sizeof(__half));
    }
    void rebind_stream(cudaStream_t s) override {
        perm.s = brp.s = bci.s = s;
        work.items.s = s;
        work.long_rows.s = s;
        work.first_slot.s = s;
        bv.s = s;
        sparse.rptr.s = sparse.col.s = sparse.val.s = s;
        sparse.brs.s = sparse.short_rows.s = sparse.long_rows.s = sparse.long_first.s = s;
        sparse.chunks.s = sparse.tasks.s = s;
        sparse.ksteps.s = s;
        sparse.mtasks.s = s;
        sparse.mlong_first.s = s;
        sparse.mlong_rows.s = s;
        sparse.mranges.s = s;
        f32work.pieces.s = f32work.long_br.s = f32work.long_first.s = s;
        tc.gptr.s = s;
        tc.gcol.s = s;
        tc.apk.s = s;
    }
};

// Stage events: ev[first] before clustering, ev[first+1] after it, ev[first+2] after the
// permutation, ev[first+3] after the conversion (recorded only when mark is true).
template <typename VT, typename IT>
void plan_from_csr(Handle& h, int64_t M, int64_t K, int64_t nnz, const IT* row_ptr,
                   const IT* col_ind, const VT* values, int64_t hw, bool clustering, bool mark,
                   Plan<VT, IT>& out);

template <typename VT, typename IT>
void plan_from_bcsr(Handle& h, int64_t nbr, int64_t nbc, int64_t nnzb, const IT* row_ptr,
                    const IT* col_ind, const VT* values, int64_t M, int64_t K, Plan<VT, IT>& out);

// Whether the automatic Tier-1 choice (or the handle's forced kernel) would take tcgen05 for
// this matrix at some N.
bool plan_wants_tc(const Handle& h, int64_t nbr, int64_t nbc, int64_t nnzb);

// A rank's share of a matrix split by block rows over an NCCL communicator (dist.cu).
struct DistPlanBase {
    int64_t M = 0, K = 0, nbc = 0;
    int64_t row_begin = 0, row_end = 0;      // this rank's rows of the clustered matrix
    int64_t block_begin = 0, block_end = 0;  // and block rows
    int64_t nnzb = 0, nnzb_total = 0;        // this rank's blocks, and all ranks'
    bool clustered = false;
    int value_bytes = 0;
    std::vector<int64_t> rank_rows;          // rows of rank r: [rank_rows[r], rank_rows[r+1])
    virtual ~DistPlanBase() = default;
    virtual void execute(Handle& h, xspmm_dist_comm_s* c, void* B, float* C_local, int64_t N,
                         int root, int timeout_ms) = 0;
    virtual void gather(Handle& h, xspmm_dist_comm_s* c, const float* C_local, float* C,
                        int64_t N, int root, int timeout_ms) = 0;
    virtual int64_t device_bytes() const = 0;
    virtual void rebind_stream(cudaStream_t s) = 0;
};

}  // namespace xspmm_b200

struct xspmm_plan_s {
    xspmm_handle_s* owner = nullptr;
    std::unique_ptr<xspmm_b200::PlanBase> p;
};
