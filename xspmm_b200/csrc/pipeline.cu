// pipeline.cu -- Tier-2: C = A * B for a CSR matrix A, with optional row clustering, and the
// plan that keeps the stages' results for repeated products.
//
// Same stages as the reference pipeline (src/cuda/unstructured_mtx_mul.cu:56-130):
//   clustering (tau = 0.5, block width = hw_block_size, :83) -> row permutation (:88) ->
//   CSR->BCSR (:102) -> Tier-1 SpMM (:113) -> unpermute (:122),
// with three differences that change no result:
//   * the unpermute is fused into the SpMM store (row i of the product is written to C[perm[i]]),
//     so there is no M x N temporary and unpermutation_ms is 0;
//   * no cudaMemset of C before the SpMM -- the kernel writes every row (the reference's memset,
//     :111, is redundant and counted in its spmm_ms);
//   * every stage runs on the device (the reference pulls A to the host for clustering and
//     conversion, clustering_sylos_labini.cpp:70-73, conversion.cpp:22-26).
// Timings are CUDA events on the handle's stream, read once at the end when requested.
#include "plan.cuh"

namespace xspmm_b200 {

bool plan_wants_tc(const Handle& h, int64_t nbr, int64_t nbc, int64_t nnzb) {
    const Tier1Kernel choice = tier1_kernel_choice(h);
    if (choice == Tier1Kernel::Mma || nbr == 0 || nbc == 0 || nnzb == 0) return false;
    return choice == Tier1Kernel::Tc || tc_preferred(nbr, nbc, nnzb);
}

template <typename VT, typename IT>
void plan_from_csr(Handle& h, int64_t M, int64_t K, int64_t nnz, const IT* row_ptr,
                   const IT* col_ind, const VT* values, int64_t hw, bool clustering, bool mark,
                   Plan<VT, IT>& out) {
    // hw_block_size is the clustering's column block width, as in the reference (:83). The
    // product always runs on 16 x 16 blocks: the reference converts to hw x hw blocks (:102) but
    // its kernel reads them as 16 x 16 (:39), so for hw != 16 its C is wrong; C here is A * B.
    XS_REQUIRE(hw >= 1, XSPMM_STATUS_INVALID_ARGUMENT, "hw_block_size must be at least 1");
    cudaStream_t s = h.stream;
    auto ev = [&](int i) {
        if (mark) XS_CHECK_CUDA(cudaEventRecord(h.ev[i], s));
    };
    out.M = M;
    out.K = K;
    out.value_bytes = (int)sizeof(VT);
    ev(0);
    const IT* arp = row_ptr;
    const IT* aci = col_ind;
    const VT* av = values;
    DevBuf<IT> prp, pci;
    DevBuf<VT> pv;
    if (clustering && M > 0) {
        out.perm = DevBuf<IT>(M, s);
        cluster_jaccard<IT>(h, M, K, nnz, row_ptr, col_ind, 0.5f, hw, out.perm.get());
        ev(1);
        prp = DevBuf<IT>(M + 1, s);
        pci = DevBuf<IT>(std::max<int64_t>(nnz, 1), s);
        pv = DevBuf<VT>(std::max<int64_t>(nnz, 1), s);
        permute_rows<VT, IT>(h, M, nnz, row_ptr, col_ind, values, out.perm.get(), prp.get(),
                             pci.get(), pv.get(), false);
        ev(2);
        arp = prp.get();
        aci = pci.get();
        av = pv.get();
        out.clustered = true;
    } else {
        ev(1);
        ev(2);
    }
    out.nbr = ceil_div(M, 16);
    out.nbc = ceil_div(K, 16);
    out.brp = DevBuf<IT>(out.nbr + 1, s);
    out.nnzb = csr_to_bcsr_count<IT>(h, M, K, nnz, arp, aci, 16, 16, out.brp.get());
    out.bci = DevBuf<IT>(std::max<int64_t>(out.nnzb, 1), s);
    out.bv = DevBuf<VT>(std::max<int64_t>(out.nnzb, 1) * 256, s);
    csr_to_bcsr_fill<VT, IT>(h, M, K, nnz, arp, aci, av, 16, 16, out.brp.get(), out.bci.get(),
                             out.bv.get());
    ev(3);
    out.rp = out.brp.get();
    out.ci = out.bci.get();
    out.v = out.bv.get();
}

template <typename VT, typename IT>
void plan_from_bcsr(Handle& h, int64_t nbr, int64_t nbc, int64_t nnzb, const IT* row_ptr,
                    const IT* col_ind, const VT* values, int64_t M, int64_t K,
                    Plan<VT, IT>& out) {
    (void)h;
    out.M = M;
    out.K = K;
    out.nbr = nbr;
    out.nbc = nbc;
    out.nnzb = nnzb;
    out.value_bytes = (int)sizeof(VT);
    out.rp = row_ptr;
    out.ci = col_ind;
    out.v = values;
}

template <typename VT, typename IT>
void Plan<VT, IT>::prepare_tc(Handle& h) {
    if constexpr (half_like<VT>::value) {
        if (tc_built || nbr == 0 || nbc == 0 || nnzb == 0) return;
        XS_REQUIRE(nnzb * 16 < (int64_t(1) << 31) && nbc * 16 < (int64_t(1) << 31) &&
                       reinterpret_cast<uintptr_t>(v) % 16 == 0,
                   XSPMM_STATUS_UNSUPPORTED, "matrix not supported by the tcgen05 kernel");
        tc_prepare<IT>(h, nbr, nbc, nnzb, rp, ci, as_half(v), tc);
        tc_built = true;
    } else {
        (void)h;
    }
}

template <typename VT, typename IT>
void Plan<VT, IT>::execute(Handle& h, const void* Bv, float* C, int64_t N) {
    if (M == 0 || N == 0) return;
    const VT* B = static_cast<const VT*>(Bv);
    const IT* map = clustered ? perm.get() : nullptr;
    if constexpr (half_like<VT>::value) {
        constexpr bool bf16 = std::is_same<VT, __nv_bfloat16>::value;
        if (plan_wants_tc(h, nbr, nbc, nnzb) && tc_supported(nbr, nbc, nnzb, v, B, C, N)) {
            prepare_tc(h);
            tc_execute<IT>(h, tc, as_half(B), C, M, K, N, map, bf16);
            return;
        }
        // When B is well beyond what L2 holds, run the block rows in order of their first
        // block column so that CTAs in flight together gather nearby rows of B.
        const bool big_b = (double)K * (double)N * sizeof(VT) > 48.0 * (1 << 20);
        // A single product of a small matrix does not repay building the list (one host
        // round trip); a large one does (long rows would serialize on one CTA).
        const bool want_work = !one_shot || nnzb >= (int64_t(1) << 18);
        // Block rows of nearly empty blocks go to the gather kernels (spmm_sparse.cu); the
        // split is decided once per plan from the block values.
        if (want_work && nbr > 0 && !sparse_built && tier1_kernel_choice(h) == Tier1Kernel::Auto &&
            reinterpret_cast<uintptr_t>(v) % 16 == 0) {
            sparse_rows_build<VT, IT>(h, nbr, M, rp, ci, v, SP_DENSE_NNZ_F16, sparse);
            sparse_built = true;
            work_built = false;  // the work list must leave those rows out
        }
        const bool split = sparse_built && sparse.nbrs > 0;
        if (want_work && nbr > 0 && (!work_built || (big_b && !work_sorted))) {
            work = MmaWork();
            mma_work_build<IT>(h, nbr, nbc, nnzb, rp, ci, big_b, work,
                               split ? &sparse.dense_br : nullptr);
            work_built = true;
            work_sorted = big_b;
        }
        if (!(split && work.empty))
            bcsr_spmm_mma_f16<IT>(h, nbr, rp, ci, as_half(v), as_half(B), C, M, K, N, map,
                                  work_built ? &work : nullptr, bf16);
        if (split) sparse_rows_execute<VT, IT>(h, sparse, B, C, M, K, N, map);
    } else {
        // fp32: the same split, at a higher fill (the SIMT block kernel pays per nonzero column
        // of a block, a gather per nonzero). A single product splits only when the block kernel
        // would take long against the split's one host round trip.
        // The block rows left to the block kernel run from a work list that cuts rows far
        // above the average length.
        const bool want_split = !one_shot || (double)nnzb * (double)N >= (double)(1 << 21);
        if (want_split && nbr > 0 && !sparse_built &&
            tier1_kernel_choice(h) == Tier1Kernel::Auto && reinterpret_cast<uintptr_t>(v) % 16 == 0) {
            sparse_rows_build<VT, IT>(h, nbr, M, rp, ci, v, SP_DENSE_NNZ_F32, sparse);
            sparse_built = true;
            f32_work_build(h, nbr, sparse.host_rp, sparse.nbrs > 0 ? &sparse.dense_br : nullptr,
                           f32work);
        }
        if (sparse_built) {
            bcsr_spmm_f32_work<IT>(h, f32work, rp, ci, v, B, C, M, K, N, map);
            if (sparse.nbrs > 0) sparse_rows_execute<VT, IT>(h, sparse, B, C, M, K, N, map);
        } else {
            bcsr_spmm<VT, IT>(h, nbr, nbc, nnzb, rp, ci, v, B, C, M, K, N, map);
        }
    }
}

template <typename VT, typename IT>
void spmm_csr_pipeline(Handle& h, int64_t M, int64_t K, int64_t nnz, const IT* row_ptr,
                       const IT* col_ind, const VT* values, const VT* B, float* C, int64_t N,
                       int64_t hw, bool clustering, xspmm_timings_t* timings) {
    Plan<VT, IT> plan;
    plan.one_shot = true;
    plan_from_csr<VT, IT>(h, M, K, nnz, row_ptr, col_ind, values, hw, clustering,
                          timings != nullptr, plan);
    plan.execute(h, B, C, N);
    if (timings) {
        cudaEvent_t* ev = h.ev;
        XS_CHECK_CUDA(cudaEventRecord(ev[4], h.stream));
        XS_CHECK_CUDA(cudaEventSynchronize(ev[4]));
        float t[4];
        for (int i = 0; i < 4; ++i) XS_CHECK_CUDA(cudaEventElapsedTime(&t[i], ev[i], ev[i + 1]));
        float tot = 0.f;
        XS_CHECK_CUDA(cudaEventElapsedTime(&tot, ev[0], ev[4]));
        timings->clustering_ms = t[0];
        timings->permutation_ms = t[1];
        timings->conversion_ms = t[2];
        timings->spmm_ms = t[3];
        timings->unpermutation_ms = 0.0;
        timings->total_pipeline_ms = tot;
    }
}

#define XS_INST_PIPE(VT, IT)                                                                      \
    template struct Plan<VT, IT>;                                                                 \
    template void plan_from_csr<VT, IT>(Handle&, int64_t, int64_t, int64_t, const IT*, const IT*, \
                                        const VT*, int64_t, bool, bool, Plan<VT, IT>&);           \
    template void plan_from_bcsr<VT, IT>(Handle&, int64_t, int64_t, int64_t, const IT*,           \
                                         const IT*, const VT*, int64_t, int64_t, Plan<VT, IT>&);  \
    template void spmm_csr_pipeline<VT, IT>(Handle&, int64_t, int64_t, int64_t, const IT*,        \
                                            const IT*, const VT*, const VT*, float*, int64_t,     \
                                            int64_t, bool, xspmm_timings_t*);
XS_INST_PIPE(__half, int32_t)
XS_INST_PIPE(__half, int64_t)
XS_INST_PIPE(__nv_bfloat16, int32_t)
XS_INST_PIPE(__nv_bfloat16, int64_t)
XS_INST_PIPE(float, int32_t)
XS_INST_PIPE(float, int64_t)

}  // namespace xspmm_b200
