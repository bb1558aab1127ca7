// pipeline.cu -- Tier-2: C = A * B for a CSR matrix A, with optional row clustering.
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
#include "ops.cuh"

namespace xspmm_b200 {

template <typename VT, typename IT>
void spmm_csr_pipeline(Handle& h, int64_t M, int64_t K, int64_t nnz, const IT* row_ptr,
                       const IT* col_ind, const VT* values, const VT* B, float* C, int64_t N,
                       int64_t hw, bool clustering, xspmm_timings_t* timings) {
    XS_REQUIRE(hw == 16, XSPMM_STATUS_UNSUPPORTED,
               "hw_block_size must be 16 (the tensor-core block size)");
    cudaStream_t s = h.stream;
    cudaEvent_t* ev = h.ev;
    auto mark = [&](int i) {
        if (timings) XS_CHECK_CUDA(cudaEventRecord(ev[i], s));
    };
    mark(0);
    const IT* arp = row_ptr;
    const IT* aci = col_ind;
    const VT* av = values;
    DevBuf<IT> perm, prp, pci;
    DevBuf<VT> pv;
    if (clustering && M > 0) {
        perm = DevBuf<IT>(M, s);
        cluster_jaccard<IT>(h, M, K, nnz, row_ptr, col_ind, 0.5f, hw, perm.get());
        mark(1);
        prp = DevBuf<IT>(M + 1, s);
        pci = DevBuf<IT>(std::max<int64_t>(nnz, 1), s);
        pv = DevBuf<VT>(std::max<int64_t>(nnz, 1), s);
        permute_rows<VT, IT>(h, M, nnz, row_ptr, col_ind, values, perm.get(), prp.get(), pci.get(),
                             pv.get(), false);
        mark(2);
        arp = prp.get();
        aci = pci.get();
        av = pv.get();
    } else {
        mark(1);
        mark(2);
    }
    const int64_t nbr = ceil_div(M, 16), nbc = ceil_div(K, 16);
    DevBuf<IT> brp(nbr + 1, s);
    const int64_t nnzb = csr_to_bcsr_count<IT>(h, M, K, nnz, arp, aci, 16, 16, brp.get());
    DevBuf<IT> bci(std::max<int64_t>(nnzb, 1), s);
    DevBuf<VT> bv(std::max<int64_t>(nnzb, 1) * 256, s);
    csr_to_bcsr_fill<VT, IT>(h, M, K, nnz, arp, aci, av, 16, 16, brp.get(), bci.get(), bv.get());
    mark(3);
    bcsr_spmm<VT, IT>(h, nbr, nbc, nnzb, brp.get(), bci.get(), bv.get(), B, C, M, K, N,
                      (clustering && M > 0) ? perm.get() : nullptr);
    mark(4);
    if (timings) {
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
    template void spmm_csr_pipeline<VT, IT>(Handle&, int64_t, int64_t, int64_t, const IT*,        \
                                            const IT*, const VT*, const VT*, float*, int64_t,     \
                                            int64_t, bool, xspmm_timings_t*);
XS_INST_PIPE(__half, int32_t)
XS_INST_PIPE(__half, int64_t)
XS_INST_PIPE(float, int32_t)
XS_INST_PIPE(float, int64_t)

}  // namespace xspmm_b200
