// dist_example.cpp -- the multi-GPU C++ API (include/xspmm/dist.hpp): one matrix split by block
// rows over `nranks` GPUs of this process, one thread per GPU, NCCL communicator made through the
// library. Every rank reads the whole matrix; rank 0 holds B, broadcasts it, and gathers C in the
// caller's row order, which is written out for the test to compare with the CPU oracle.
//
//   dist_example <nranks> <in.bin> <out.bin>
// in.bin : as pipeline_example.cpp (int64 M, K, N, nnz; int32 row_ptr, col_ind; fp16 values, B)
// out.bin: float C[M*N]; int64 blocks held by each rank [nranks]; int64 blocks in all
#include <cstdint>
#include <cstdio>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "xspmm/dist.hpp"
#include "xspmm/xspmm.hpp"

template <typename T>
static bool rd(std::FILE* f, T* p, size_t n) { return std::fread(p, sizeof(T), n, f) == n; }

int main(int argc, char** argv) {
    if (argc != 4) {
        std::fprintf(stderr, "usage: %s nranks in.bin out.bin\n", argv[0]);
        return 2;
    }
    const int nranks = std::stoi(argv[1]);
    std::FILE* f = std::fopen(argv[2], "rb");
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

    unsigned char id[128];
    xspmm::dist_unique_id(id);
    std::vector<float> C((size_t)M * N);
    std::vector<int64_t> blocks(nranks, -1);
    int64_t total = -1;
    std::vector<std::string> errors(nranks);
    std::vector<std::thread> ts;
    for (int r = 0; r < nranks; ++r) {
        ts.emplace_back([&, r] {
            try {
                auto exec = std::make_shared<xspmm::CudaExecutor>(r);
                xspmm::CSRMatrix<__half, int32_t> A(exec, M, K, nnz);
                A.copy_from_host(rp.data(), ci.data(), vals.data());
                xspmm::DistComm comm(exec, nranks, r, id, 60000);
                xspmm::DistPlan<__half, int32_t> plan(comm, exec, A);
                const auto inf = plan.info();
                blocks[r] = inf.nnz_blocks;
                if (r == 0) total = inf.nnz_blocks_total;
                __half* d_B = nullptr;
                float *d_Cl = nullptr, *d_C = nullptr;
                const int64_t rows = inf.row_end - inf.row_begin;
                exec->allocate(reinterpret_cast<void**>(&d_B), B.size() * sizeof(__half));
                exec->allocate(reinterpret_cast<void**>(&d_Cl), (size_t)(rows > 0 ? rows : 1) * N * sizeof(float));
                if (r == 0) {
                    exec->allocate(reinterpret_cast<void**>(&d_C), C.size() * sizeof(float));
                    exec->copy_from_host(d_B, B.data(), B.size() * sizeof(__half));
                }
                plan.execute(d_B, d_Cl, N, /*bcast_root=*/0);
                plan.gather(d_Cl, d_C, N, /*root=*/0);
                if (r == 0) {
                    exec->copy_to_host(C.data(), d_C, C.size() * sizeof(float));
                    exec->free(d_C);
                }
                exec->free(d_B);
                exec->free(d_Cl);
            } catch (const std::exception& e) {
                errors[r] = e.what();
            }
        });
    }
    for (auto& t : ts) t.join();
    for (int r = 0; r < nranks; ++r)
        if (!errors[r].empty()) {
            std::fprintf(stderr, "rank %d: %s\n", r, errors[r].c_str());
            return 3;
        }
    std::FILE* o = std::fopen(argv[3], "wb");
    if (!o) return 2;
    std::fwrite(C.data(), sizeof(float), C.size(), o);
    std::fwrite(blocks.data(), sizeof(int64_t), blocks.size(), o);
    std::fwrite(&total, sizeof(int64_t), 1, o);
    std::fclose(o);
    std::printf("ok nranks=%d M=%d N=%d\n", nranks, M, N);
    return 0;
}
