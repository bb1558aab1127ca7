// pipeline_example.cpp -- drives the reference-shaped C++ API (include/xspmm/xspmm.hpp) the way
// the reference's examples do (examples/01_uspmm_checkers.cpp:73-100: clustering ->
// apply_permutation -> csr_to_bcsr -> Tier 1 -> unpermute; the Tier-2 call of
// src/xspmm.cpp:137-162), on a matrix read from a binary file written by the test.
//
//   pipeline_example <in.bin> <out.bin>
// in.bin : int64 M, K, N, nnz; int32 row_ptr[M+1]; int32 col_ind[nnz]; uint16 values[nnz] (fp16);
//          uint16 B[K*N] (fp16)
// out.bin: int32 perm[M]; float C_tier2[M*N]; float C_chain[M*N]; double timings[6]
#include <cstdint>
#include <cstdio>
#include <memory>
#include <vector>

#include "xspmm/xspmm.hpp"

template <typename T>
static bool rd(std::FILE* f, T* p, size_t n) { return std::fread(p, sizeof(T), n, f) == n; }

int main(int argc, char** argv) {
    if (argc != 3) {
        std::fprintf(stderr, "usage: %s in.bin out.bin\n", argv[0]);
        return 2;
    }
    std::FILE* f = std::fopen(argv[1], "rb");
    if (!f) return 2;
    int64_t hdr[4];
    if (!rd(f, hdr, 4)) return 2;
    const int32_t M = (int32_t)hdr[0], K = (int32_t)hdr[1], N = (int32_t)hdr[2], nnz = (int32_t)hdr[3];
    std::vector<int32_t> rp(M + 1), ci(nnz);
    std::vector<__half> vals(nnz), B((size_t)K * N);
    if (!rd(f, rp.data(), rp.size()) || !rd(f, ci.data(), ci.size()) ||
        !rd(f, vals.data(), vals.size()) || !rd(f, B.data(), B.size()))
        return 2;
    std::fclose(f);

    auto exec = std::make_shared<xspmm::CudaExecutor>(0);
    xspmm::CSRMatrix<__half, int32_t> A(exec, M, K, nnz);
    A.copy_from_host(rp.data(), ci.data(), vals.data());

    __half* d_B = nullptr;
    float *d_C1 = nullptr, *d_C2 = nullptr, *d_Ctmp = nullptr;
    int32_t* d_perm = nullptr;
    exec->allocate(reinterpret_cast<void**>(&d_B), B.size() * sizeof(__half));
    exec->allocate(reinterpret_cast<void**>(&d_C1), (size_t)M * N * sizeof(float));
    exec->allocate(reinterpret_cast<void**>(&d_C2), (size_t)M * N * sizeof(float));
    exec->allocate(reinterpret_cast<void**>(&d_Ctmp), (size_t)M * N * sizeof(float));
    exec->allocate(reinterpret_cast<void**>(&d_perm), (size_t)M * sizeof(int32_t));
    exec->copy_from_host(d_B, B.data(), B.size() * sizeof(__half));

    // Tier 2 in one call
    xspmm::SpMMTimings t;
    xspmm::spmm(exec, A, d_B, d_C1, N, 16, true, &t);

    // the same pipeline through the individual calls
    xspmm::compute_1d_jaccard_clustering(exec, A, 0.5f, 16, d_perm);
    auto A_opt = xspmm::apply_permutation(exec, A, d_perm);
    auto A_bcsr = xspmm::csr_to_bcsr(exec, A_opt, 16, 16);
    xspmm::spmm(A_bcsr, d_B, d_Ctmp, N);
    xspmm::unpermute_dense_matrix(exec, d_Ctmp, d_C2, d_perm, M, N);

    // the same product from a plan (stages done once, then the Tier-1 kernel only)
    float* d_C3 = nullptr;
    exec->allocate(reinterpret_cast<void**>(&d_C3), (size_t)M * N * sizeof(float));
    {
        xspmm::SpMMPlan<__half, int32_t> plan(exec, A, 16, true);
        plan.execute(d_B, d_C3, N);
        if (plan.info().rows != M) return 4;
    }
    exec->synchronize();

    std::vector<int32_t> perm(M);
    std::vector<float> C1((size_t)M * N), C2((size_t)M * N), C3((size_t)M * N);
    exec->copy_to_host(perm.data(), d_perm, perm.size() * sizeof(int32_t));
    exec->copy_to_host(C1.data(), d_C1, C1.size() * sizeof(float));
    exec->copy_to_host(C2.data(), d_C2, C2.size() * sizeof(float));
    exec->copy_to_host(C3.data(), d_C3, C3.size() * sizeof(float));
    for (void* p : {(void*)d_B, (void*)d_C1, (void*)d_C2, (void*)d_Ctmp, (void*)d_perm, (void*)d_C3})
        exec->free(p);

    bool threw = false;  // the reference's error behaviour: bad dimensions -> invalid_argument
    try {
        xspmm::CSRMatrix<__half, int32_t> bad(exec, -1, 4, 0);
    } catch (const std::invalid_argument&) {
        threw = true;
    }
    if (!threw) return 3;

    std::FILE* o = std::fopen(argv[2], "wb");
    if (!o) return 2;
    const double tm[6] = {t.clustering_ms, t.permutation_ms, t.conversion_ms,
                          t.spmm_ms, t.unpermutation_ms, t.total_pipeline_ms};
    std::fwrite(perm.data(), sizeof(int32_t), perm.size(), o);
    std::fwrite(C1.data(), sizeof(float), C1.size(), o);
    std::fwrite(C2.data(), sizeof(float), C2.size(), o);
    std::fwrite(tm, sizeof(double), 6, o);
    std::fwrite(C3.data(), sizeof(float), C3.size(), o);
    std::fclose(o);
    std::printf("ok M=%d N=%d nnz=%d total_ms=%.3f\n", M, N, nnz, t.total_pipeline_ms);
    return 0;
}
