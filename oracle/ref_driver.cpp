// ref_driver.cpp -- C entry points over the reference xSpMM's own host code.
//
// TEST INFRASTRUCTURE. This file is compiled together with the reference's unmodified sources
// (src/xspmm.cpp, src/core/conversion.cpp, src/core/executor.cpp,
// src/cpu/clustering_sylos_labini.cpp, read where they lie) by oracle/Makefile into
// oracle/_ref/libxspmm_ref.so. It drives the reference's public functions through its
// CpuExecutor exactly as the reference's examples do (examples/01_uspmm_checkers.cpp:73-87):
//   compute_1d_jaccard_clustering -> apply_permutation -> csr_to_bcsr.
// The reference instantiates these only for float values (src/xspmm.cpp:102-114,
// src/core/conversion.cpp:106-108), so callers pass fp16 data widened to float; the functions
// only move values, so narrowing the outputs back to fp16 is exact.
#include <cstdint>
#include <cstring>
#include <memory>
#include <vector>
#include <exception>

#include "xspmm/xspmm.hpp"
#include "xspmm/clustering.hpp"
#include "xspmm/matrix/conversion.hpp"
#include "xspmm/core/executor.hpp"

namespace {

template <typename I>
std::shared_ptr<xspmm::Executor> cpu_exec() {
    return std::make_shared<xspmm::CpuExecutor>();
}

template <typename I>
int cluster(I M, I K, I nnz, const I* rp, const I* ci, float tau, I w, I* perm) {
    try {
        auto exec = cpu_exec<I>();
        std::vector<float> vals(static_cast<size_t>(nnz), 1.0f);
        xspmm::CSRMatrix<float, I> A(exec, M, K, nnz);
        A.copy_from_host(rp, ci, vals.data());
        xspmm::compute_1d_jaccard_clustering<float, I>(exec, A, tau, w, perm);
        return 0;
    } catch (const std::exception&) {
        return -1;
    }
}

template <typename I>
int permute(I M, I K, I nnz, const I* rp, const I* ci, const float* vals, const I* perm,
            I* out_rp, I* out_ci, float* out_vals) {
    try {
        auto exec = cpu_exec<I>();
        xspmm::CSRMatrix<float, I> A(exec, M, K, nnz);
        A.copy_from_host(rp, ci, vals);
        auto P = xspmm::apply_permutation<float, I>(exec, A, perm);
        std::memcpy(out_rp, P.get_row_ptr(), sizeof(I) * static_cast<size_t>(M + 1));
        if (nnz > 0) {
            std::memcpy(out_ci, P.get_col_ind(), sizeof(I) * static_cast<size_t>(nnz));
            std::memcpy(out_vals, P.get_values(), sizeof(float) * static_cast<size_t>(nnz));
        }
        return 0;
    } catch (const std::exception&) {
        return -1;
    }
}

// csr_to_bcsr returns a BCSRMatrix whose size is only known afterwards, so the result is held
// in an opaque box that the caller copies out of and frees.
template <typename I>
struct BcsrBox {
    xspmm::BCSRMatrix<float, I> m;
};

template <typename I>
void* to_bcsr(I M, I K, I nnz, const I* rp, const I* ci, const float* vals, I rb, I cb,
              int64_t* nnzb_out) {
    try {
        auto exec = cpu_exec<I>();
        xspmm::CSRMatrix<float, I> A(exec, M, K, nnz);
        A.copy_from_host(rp, ci, vals);
        auto* box = new BcsrBox<I>{xspmm::csr_to_bcsr<float, I>(exec, A, rb, cb)};
        *nnzb_out = static_cast<int64_t>(box->m.get_num_blocks());
        return box;
    } catch (const std::exception&) {
        return nullptr;
    }
}

template <typename I>
void bcsr_copy(void* h, I* brp, I* bci, float* bvals) {
    auto* box = static_cast<BcsrBox<I>*>(h);
    auto& m = box->m;
    I nbr = m.get_num_block_rows(), nnzb = m.get_num_blocks();
    std::memcpy(brp, m.get_bcsr_row_ptr(), sizeof(I) * static_cast<size_t>(nbr + 1));
    if (nnzb > 0) {
        std::memcpy(bci, m.get_bcsr_col_ind(), sizeof(I) * static_cast<size_t>(nnzb));
        size_t nv = static_cast<size_t>(nnzb) * static_cast<size_t>(m.get_r_block() * m.get_c_block());
        std::memcpy(bvals, m.get_bcsr_values(), sizeof(float) * nv);
    }
}

}  // namespace

extern "C" {

int ref_cluster_i32(int32_t M, int32_t K, int32_t nnz, const int32_t* rp, const int32_t* ci,
                    float tau, int32_t w, int32_t* perm) {
    return cluster<int32_t>(M, K, nnz, rp, ci, tau, w, perm);
}
int ref_cluster_i64(int64_t M, int64_t K, int64_t nnz, const int64_t* rp, const int64_t* ci,
                    float tau, int64_t w, int64_t* perm) {
    return cluster<int64_t>(M, K, nnz, rp, ci, tau, w, perm);
}
int ref_permute_i32(int32_t M, int32_t K, int32_t nnz, const int32_t* rp, const int32_t* ci,
                    const float* vals, const int32_t* perm, int32_t* orp, int32_t* oci,
                    float* ovals) {
    return permute<int32_t>(M, K, nnz, rp, ci, vals, perm, orp, oci, ovals);
}
int ref_permute_i64(int64_t M, int64_t K, int64_t nnz, const int64_t* rp, const int64_t* ci,
                    const float* vals, const int64_t* perm, int64_t* orp, int64_t* oci,
                    float* ovals) {
    return permute<int64_t>(M, K, nnz, rp, ci, vals, perm, orp, oci, ovals);
}
void* ref_csr_to_bcsr_i32(int32_t M, int32_t K, int32_t nnz, const int32_t* rp, const int32_t* ci,
                          const float* vals, int32_t rb, int32_t cb, int64_t* nnzb) {
    return to_bcsr<int32_t>(M, K, nnz, rp, ci, vals, rb, cb, nnzb);
}
void* ref_csr_to_bcsr_i64(int64_t M, int64_t K, int64_t nnz, const int64_t* rp, const int64_t* ci,
                          const float* vals, int64_t rb, int64_t cb, int64_t* nnzb) {
    return to_bcsr<int64_t>(M, K, nnz, rp, ci, vals, rb, cb, nnzb);
}
void ref_bcsr_copy_i32(void* h, int32_t* brp, int32_t* bci, float* bvals) {
    bcsr_copy<int32_t>(h, brp, bci, bvals);
}
void ref_bcsr_copy_i64(void* h, int64_t* brp, int64_t* bci, float* bvals) {
    bcsr_copy<int64_t>(h, brp, bci, bvals);
}
void ref_bcsr_free_i32(void* h) { delete static_cast<BcsrBox<int32_t>*>(h); }
void ref_bcsr_free_i64(void* h) { delete static_cast<BcsrBox<int64_t>*>(h); }

}  // extern "C"

// ---- Matrix Market reader (utils/matrix_io.hpp, header-only, read where it lies) -------------
#include "matrix_io.hpp"

namespace {
struct MtxBox {
    matrix_utils::io::HostCSRMatrix<float> m;
};
}  // namespace

extern "C" {

// Reads `path` with matrix_utils::io::read_mtx<float>; returns an opaque box (null if the reader
// threw) and the sizes; ref_mtx_copy copies the CSR out, ref_mtx_free releases the box.
void* ref_read_mtx(const char* path, int32_t* rows, int32_t* cols, int64_t* nnz) {
    try {
        auto* box = new MtxBox{matrix_utils::io::read_mtx<float>(path)};
        *rows = box->m.num_rows;
        *cols = box->m.num_cols;
        *nnz = static_cast<int64_t>(box->m.values.size());
        return box;
    } catch (const std::exception&) {
        return nullptr;
    }
}
void ref_mtx_copy(void* h, int32_t* rp, int32_t* ci, float* vals) {
    auto& m = static_cast<MtxBox*>(h)->m;
    std::memcpy(rp, m.row_ptr.data(), sizeof(int32_t) * m.row_ptr.size());
    if (!m.values.empty()) {
        std::memcpy(ci, m.col_ind.data(), sizeof(int32_t) * m.col_ind.size());
        std::memcpy(vals, m.values.data(), sizeof(float) * m.values.size());
    }
}
void ref_mtx_free(void* h) { delete static_cast<MtxBox*>(h); }

}  // extern "C"

// ---- generators (utils/matrix_gen.hpp, header-only, read where it lies) ----------------------
#include "matrix_gen.hpp"

namespace {
struct GenBox {
    std::vector<int32_t> rp, ci;
    std::vector<float> v;
};
}  // namespace

extern "C" {

// kind: 0 banded(a=size, b=bandwidth), 1 triangular(a, upper=b, density=f1),
// 2 hessenberg(a, upper=b, density=f1), 3 arrowhead(a, width=b), 4 checkers(rows=a, cols=b,
// block=c), 5 block_diagonal(a, block=b, density=f1), 6 near_symmetric(a, density=f1,
// drop=f2), 7 power_law(rows=a, cols=b, alpha=f1). Returns an opaque box (null on error).
void* ref_gen(int kind, int32_t a, int32_t b, int32_t c, float f1, float f2, int seed,
              int32_t* rows_out, int64_t* nnz_out) {
    namespace g = matrix_utils::generation;
    try {
        auto* box = new GenBox;
        int32_t rows = a;
        switch (kind) {
            case 0: g::generate_banded<float, int32_t>(a, b, box->rp, box->ci, box->v, seed); break;
            case 1: g::generate_triangular<float, int32_t>(a, b != 0, f1, box->rp, box->ci, box->v, seed); break;
            case 2: g::generate_hessenberg<float, int32_t>(a, b != 0, f1, box->rp, box->ci, box->v, seed); break;
            case 3: g::generate_arrowhead<float, int32_t>(a, b, box->rp, box->ci, box->v, seed); break;
            case 4: g::generate_checkers<float, int32_t>(a, b, c, box->rp, box->ci, box->v, seed); break;
            case 5: g::generate_block_diagonal<float, int32_t>(a, b, f1, box->rp, box->ci, box->v, seed); break;
            case 6: g::generate_near_symmetric<float, int32_t>(a, f1, f2, box->rp, box->ci, box->v, seed); break;
            case 7: g::generate_power_law<float, int32_t>(a, b, f1, box->rp, box->ci, box->v, seed); break;
            default: delete box; return nullptr;
        }
        *rows_out = rows;
        *nnz_out = static_cast<int64_t>(box->v.size());
        return box;
    } catch (const std::exception&) {
        return nullptr;
    }
}
void ref_gen_copy(void* h, int32_t* rp, int32_t* ci, float* v) {
    auto* box = static_cast<GenBox*>(h);
    std::memcpy(rp, box->rp.data(), sizeof(int32_t) * box->rp.size());
    if (!box->v.empty()) {
        std::memcpy(ci, box->ci.data(), sizeof(int32_t) * box->ci.size());
        std::memcpy(v, box->v.data(), sizeof(float) * box->v.size());
    }
}
void ref_gen_free(void* h) { delete static_cast<GenBox*>(h); }

}  // extern "C"
