// dist.cu -- the multi-GPU path behind the C ABI: one process (or thread) per GPU, NCCL over
// NVLink / NVSwitch, block rows of A split over the ranks.
//
// The reference runs on one device (include/xspmm/xspmm.hpp:14-32); its Tier-1 product is
// independent per block row given B (src/common/spmm_math.hpp:68-114), so the matrix splits into
// contiguous block-row ranges with one exchange step (B in) and an optional one (C out):
//
//  plan   every rank passes the whole CSR A on its own device. Clustering runs on every rank (it
//         is deterministic: every rank gets the same permutation, with no message). The permuted
//         matrix's blocks are counted once per rank (row pointer of the BCSR); block rows are
//         partitioned on that prefix of nonzero blocks (plus an optional weight per block row),
//         the same partition on every rank; each rank then copies its own rows of the permuted
//         CSR and fills only its own block rows, so its BCSR holds about 1/N of the blocks.
//  execute  optional ncclBroadcast of B from a root (in place), then the rank's Tier-1 plan writes
//         its rows of C (clustered order) into local memory.
//  gather   optional: the root receives every rank's rows (ncclSend/ncclRecv in one group) and
//         unpermutes them into C in the caller's row order (src/cuda/mtx_permutation.cu:71-85).
//
// NCCL is loaded at run time (libnccl.so.2; in a process that already loaded it -- torch does --
// the same library instance), so the library has no link-time dependency on it. Communicators are
// created non-blocking and every wait on NCCL work polls ncclCommGetAsyncError and the stream under
// a host time limit: an NCCL error returns XSPMM_STATUS_NCCL_ERROR, a limit that runs out aborts
// the communicator (ncclCommAbort) and returns XSPMM_STATUS_TIMEOUT. An aborted communicator
// refuses every later call.
#include "plan.cuh"

#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

using namespace xspmm_b200;

// ---- NCCL, loaded at run time --------------------------------------------------------------------
namespace {

struct NcclApi {
    bool ok = false;
    std::string why;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommCount)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*CommUserRank)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*Broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!lib) lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!lib) {
            api.why = std::string("libnccl.so.2 not found: ") + dlerror();
            return;
        }
        bool all = true;
        auto get = [&](auto& fn, const char* name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(lib, name));
            if (!fn) {
                all = false;
                api.why += std::string(" missing ") + name;
            }
        };
        get(api.GetUniqueId, "ncclGetUniqueId");
        get(api.CommInitRankConfig, "ncclCommInitRankConfig");
        get(api.CommGetAsyncError, "ncclCommGetAsyncError");
        get(api.CommAbort, "ncclCommAbort");
        get(api.CommDestroy, "ncclCommDestroy");
        get(api.CommCount, "ncclCommCount");
        get(api.CommUserRank, "ncclCommUserRank");
        get(api.Broadcast, "ncclBroadcast");
        get(api.Send, "ncclSend");
        get(api.Recv, "ncclRecv");
        get(api.GroupStart, "ncclGroupStart");
        get(api.GroupEnd, "ncclGroupEnd");
        get(api.GetErrorString, "ncclGetErrorString");
        api.ok = all;
    });
    XS_REQUIRE(api.ok, XSPMM_STATUS_UNSUPPORTED, "NCCL unavailable:" + api.why);
    return api;
}

}  // namespace

struct xspmm_dist_comm_s {
    ncclComm_t c = nullptr;
    int nranks = 0, rank = 0, device = 0;
    bool owned = false;    // created here (destroyed here) or wrapped
    bool aborted = false;  // after a timeout or an NCCL error: refuses every call
};

struct xspmm_dist_plan_s {
    xspmm_handle_s* owner = nullptr;
    xspmm_dist_comm_s* comm = nullptr;
    std::unique_ptr<DistPlanBase> p;
};

namespace xspmm_b200 {

using Clock = std::chrono::steady_clock;

// Polls the communicator (and the stream) until the enqueued NCCL work is done, an error shows up
// (NCCL_ERROR) or timeout_ms runs out (TIMEOUT; the communicator is aborted).
void comm_wait(xspmm_dist_comm_s* c, cudaStream_t s, int timeout_ms, bool stream_too) {
    const NcclApi& api = nccl();
    const auto t0 = Clock::now();
    const int limit = timeout_ms > 0 ? timeout_ms : 60000;
    for (;;) {
        ncclResult_t st = ncclSuccess;
        const ncclResult_t q = api.CommGetAsyncError(c->c, &st);
        if (q != ncclSuccess || (st != ncclSuccess && st != ncclInProgress)) {
            api.CommAbort(c->c);
            c->aborted = true;
            throw Error(XSPMM_STATUS_NCCL_ERROR,
                        std::string("NCCL: ") + api.GetErrorString(q != ncclSuccess ? q : st));
        }
        bool done = st == ncclSuccess;
        if (done && stream_too) {
            const cudaError_t e = cudaStreamQuery(s);
            if (e != cudaSuccess && e != cudaErrorNotReady) XS_CHECK_CUDA(e);
            done = e == cudaSuccess;
        }
        if (done) return;
        if (std::chrono::duration_cast<std::chrono::milliseconds>(Clock::now() - t0).count() > limit) {
            api.CommAbort(c->c);
            c->aborted = true;
            throw Error(XSPMM_STATUS_TIMEOUT,
                        "NCCL work did not complete within " + std::to_string(limit) +
                            " ms (a rank that never joined or stopped); communicator aborted");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

// An NCCL call on a non-blocking communicator: ncclInProgress is fine (completion is polled).
void nccl_call(xspmm_dist_comm_s* c, ncclResult_t r, const char* what) {
    if (r == ncclSuccess || r == ncclInProgress) return;
    const NcclApi& api = nccl();
    api.CommAbort(c->c);
    c->aborted = true;
    throw Error(XSPMM_STATUS_NCCL_ERROR, std::string(what) + ": " + api.GetErrorString(r));
}

// Boundaries r_0 = 0 <= ... <= r_P = nbr of P contiguous block-row ranges balancing
// blocks + row_weight * block_rows per range: r_p is the first block row whose weighted prefix
// reaches p * total / P (the same rule as xspmm_b200/shard.py).
std::vector<int64_t> partition_block_rows(const std::vector<int64_t>& brp, int parts,
                                          double row_weight) {
    const int64_t nbr = (int64_t)brp.size() - 1;
    std::vector<int64_t> b(parts + 1, 0);
    auto w = [&](int64_t i) { return (double)(brp[i] - brp[0]) + row_weight * (double)i; };
    const double total = w(nbr);
    for (int p = 0; p <= parts; ++p) {
        const double target = total * (double)p / (double)parts;
        int64_t lo = 0, hi = nbr;  // first i with w(i) >= target
        while (lo < hi) {
            const int64_t mid = lo + (hi - lo) / 2;
            if (w(mid) < target) lo = mid + 1; else hi = mid;
        }
        b[p] = lo;
    }
    b[0] = 0;
    b[parts] = nbr;
    for (int p = 1; p <= parts; ++p) b[p] = std::max(b[p], b[p - 1]);
    return b;
}

template <typename IT>
__global__ void iota_kernel(IT* out, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = (IT)i;
}

template <typename IT>
__global__ void rebase_kernel(const IT* in, IT* out, int64_t n, int64_t base) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = (IT)((int64_t)in[i] - base);
}

unsigned grid_for(Handle& h, int64_t n) {
    return (unsigned)std::max<int64_t>(
        1, std::min<int64_t>(ceil_div(n, 256), (int64_t)sm_count(h.device) * 16));
}

template <typename T>
T read_at(Handle& h, const T* dptr) {
    T v{};
    XS_CHECK_CUDA(cudaMemcpyAsync(&v, dptr, sizeof(T), cudaMemcpyDeviceToHost, h.stream));
    XS_CHECK_CUDA(cudaStreamSynchronize(h.stream));
    return v;
}

template <typename VT, typename IT>
struct DistPlan final : DistPlanBase {
    DevBuf<IT> perm;           // the clustering permutation (every rank), for the gather
    DevBuf<IT> lrp, lci;       // this rank's block rows
    DevBuf<VT> lv;
    Plan<VT, IT> plan;         // the product over them (rows in clustered order, no row map)

    void execute(Handle& h, xspmm_dist_comm_s* c, void* B, float* C_local, int64_t N, int root,
                 int timeout_ms) override {
        if (root >= 0 && K > 0 && N > 0) {
            const NcclApi& api = nccl();
            nccl_call(c, api.Broadcast(B, B, (size_t)(K * N),
                                       sizeof(VT) == 2 ? ncclFloat16 : ncclFloat32, root, c->c,
                                       h.stream),
                      "ncclBroadcast(B)");
            comm_wait(c, h.stream, timeout_ms, true);
        }
        if (row_end > row_begin && N > 0) plan.execute(h, B, C_local, N);
    }

    void gather(Handle& h, xspmm_dist_comm_s* c, const float* C_local, float* C, int64_t N,
                int root, int timeout_ms) override {
        const NcclApi& api = nccl();
        const int me = c->rank;
        if (N == 0 || M == 0) return;
        if (me == root) {
            // clustered order into a staging buffer (or straight into C without clustering)
            DevBuf<float> stage(clustered ? (size_t)(M * N) : 0, h.stream);
            float* dst = clustered ? stage.get() : C;
            nccl_call(c, api.GroupStart(), "ncclGroupStart");
            for (int r = 0; r < c->nranks; ++r) {
                const int64_t r0 = rank_rows[r], r1 = rank_rows[r + 1];
                if (r1 <= r0) continue;
                if (r == me) {
                    XS_CHECK_CUDA(cudaMemcpyAsync(dst + r0 * N, C_local,
                                                  (size_t)((r1 - r0) * N) * sizeof(float),
                                                  cudaMemcpyDeviceToDevice, h.stream));
                } else {
                    nccl_call(c, api.Recv(dst + r0 * N, (size_t)((r1 - r0) * N), ncclFloat32, r,
                                          c->c, h.stream),
                              "ncclRecv(C rows)");
                }
            }
            nccl_call(c, api.GroupEnd(), "ncclGroupEnd");
            comm_wait(c, h.stream, timeout_ms, true);
            if (clustered) {
                unpermute_dense<float, IT>(h, stage.get(), C, perm.get(), M, N, false);
                XS_CHECK_CUDA(cudaStreamSynchronize(h.stream));
            }
        } else if (row_end > row_begin) {
            nccl_call(c, api.Send(C_local, (size_t)((row_end - row_begin) * N), ncclFloat32, root,
                                  c->c, h.stream),
                      "ncclSend(C rows)");
            comm_wait(c, h.stream, timeout_ms, true);
        }
    }

    int64_t device_bytes() const override {
        return (int64_t)(perm.n + lrp.n + lci.n) * (int64_t)sizeof(IT) +
               (int64_t)lv.n * (int64_t)sizeof(VT) + plan.device_bytes();
    }
    void rebind_stream(cudaStream_t s) override {
        perm.s = lrp.s = lci.s = s;
        lv.s = s;
        plan.rebind_stream(s);
    }
};

template <typename VT, typename IT>
std::unique_ptr<DistPlanBase> dist_plan_build(Handle& h, xspmm_dist_comm_s* c, int64_t M,
                                              int64_t K, int64_t nnz, const IT* rp, const IT* ci,
                                              const VT* v, int64_t hw, bool clustering,
                                              double row_weight) {
    auto dp = std::make_unique<DistPlan<VT, IT>>();
    cudaStream_t s = h.stream;
    dp->M = M;
    dp->K = K;
    dp->clustered = clustering;
    // 1. the permutation (the same on every rank)
    dp->perm = DevBuf<IT>(std::max<int64_t>(M, 1), s);
    if (M > 0) {
        if (clustering) {
            cluster_jaccard<IT>(h, M, K, nnz, rp, ci, 0.5f, hw, dp->perm.get());
        } else {
            iota_kernel<IT><<<grid_for(h, M), 256, 0, s>>>(dp->perm.get(), M);
            after_launch(h, "dist_iota");
        }
    }
    // 2. the permuted CSR (temporary) and its block count
    DevBuf<IT> prp(M + 1, s), pci(std::max<int64_t>(nnz, 1), s);
    DevBuf<VT> pv(std::max<int64_t>(nnz, 1), s);
    if (M > 0)
        permute_rows<VT, IT>(h, M, nnz, rp, ci, v, dp->perm.get(), prp.get(), pci.get(), pv.get(),
                             true);
    const int64_t nbr = ceil_div(M, 16), nbc = ceil_div(K, 16);
    DevBuf<IT> brp(nbr + 1, s);
    const int64_t nnzb = M > 0 ? csr_to_bcsr_count<IT>(h, M, K, nnz, prp.get(), pci.get(), 16, 16,
                                                         brp.get())
                               : 0;
    std::vector<IT> hb(nbr + 1);
    XS_CHECK_CUDA(cudaMemcpyAsync(hb.data(), brp.get(), (nbr + 1) * sizeof(IT),
                                  cudaMemcpyDeviceToHost, s));
    XS_CHECK_CUDA(cudaStreamSynchronize(s));
    std::vector<int64_t> hb64(hb.begin(), hb.end());
    // 3. the partition (every rank computes the same one)
    const std::vector<int64_t> bnd = partition_block_rows(hb64, c->nranks, row_weight);
    dp->rank_rows.resize(c->nranks + 1);
    for (int r = 0; r <= c->nranks; ++r) dp->rank_rows[r] = std::min<int64_t>(M, 16 * bnd[r]);
    const int64_t b0 = bnd[c->rank], b1 = bnd[c->rank + 1];
    dp->block_begin = b0;
    dp->block_end = b1;
    dp->row_begin = dp->rank_rows[c->rank];
    dp->row_end = dp->rank_rows[c->rank + 1];
    dp->nbc = nbc;
    dp->nnzb_total = nnzb;
    const int64_t lm = dp->row_end - dp->row_begin, lnbr = b1 - b0;
    const int64_t lnnzb = hb64[b1] - hb64[b0];
    dp->nnzb = lnnzb;
    // 4. this rank's rows of the permuted CSR, then only its block rows of the BCSR
    dp->lrp = DevBuf<IT>(lnbr + 1, s);
    dp->lci = DevBuf<IT>(std::max<int64_t>(lnnzb, 1), s);
    dp->lv = DevBuf<VT>((size_t)std::max<int64_t>(lnnzb, 1) * 256, s);
    if (lnbr > 0) {
        rebase_kernel<IT><<<grid_for(h, lnbr + 1), 256, 0, s>>>(brp.get() + b0, dp->lrp.get(),
                                                                 lnbr + 1, hb64[b0]);
        after_launch(h, "dist_rebase_blocks");
        const int64_t e0 = (int64_t)read_at<IT>(h, prp.get() + dp->row_begin);
        const int64_t e1 = (int64_t)read_at<IT>(h, prp.get() + dp->row_end);
        DevBuf<IT> lrow(lm + 1, s);
        rebase_kernel<IT><<<grid_for(h, lm + 1), 256, 0, s>>>(prp.get() + dp->row_begin,
                                                               lrow.get(), lm + 1, e0);
        after_launch(h, "dist_rebase_rows");
        csr_to_bcsr_fill<VT, IT>(h, lm, K, e1 - e0, lrow.get(), pci.get() + e0, pv.get() + e0, 16,
                                 16, dp->lrp.get(), dp->lci.get(), dp->lv.get());
    }
    prp.release();
    pci.release();
    pv.release();
    brp.release();
    // 5. the rank's product plan (adopts the BCSR arrays; rows in clustered order)
    if (lnbr > 0) {
        plan_from_bcsr<VT, IT>(h, lnbr, nbc, lnnzb, dp->lrp.get(), dp->lci.get(), dp->lv.get(), lm,
                               K, dp->plan);
        if (std::is_same<VT, __half>::value && plan_wants_tc(h, lnbr, nbc, lnnzb))
            dp->plan.prepare_tc(h);
    }
    XS_CHECK_CUDA(cudaStreamSynchronize(s));
    throw_on_device_errors(h, "dist plan");
    return dp;
}

}  // namespace xspmm_b200

// ---- extern "C" ------------------------------------------------------------------------------------
namespace {

xspmm_dist_comm_s* CM(xspmm_dist_comm_t c) {
    XS_REQUIRE(c != nullptr, XSPMM_STATUS_INVALID_ARGUMENT, "null communicator");
    XS_REQUIRE(!c->aborted, XSPMM_STATUS_NCCL_ERROR,
               "communicator aborted after an earlier timeout or NCCL error");
    return c;
}

xspmm_dist_plan_s* DP(xspmm_dist_plan_t p) {
    XS_REQUIRE(p != nullptr && p->p != nullptr && p->owner != nullptr && !p->owner->destroyed,
               XSPMM_STATUS_INVALID_ARGUMENT, "null distributed plan");
    return p;
}

}  // namespace

XS_API xspmm_status_t xspmm_dist_partition(const int64_t* bcsr_row_ptr, int64_t nbr,
                                           int32_t parts, double row_weight, int64_t* bounds) {
    return guarded([&] {
        need(bcsr_row_ptr != nullptr && bounds != nullptr, "null argument");
        need(nbr >= 0 && parts >= 1 && row_weight >= 0.0, "bad argument");
        const std::vector<int64_t> brp(bcsr_row_ptr, bcsr_row_ptr + nbr + 1);
        for (int64_t i = 0; i < nbr; ++i) need(brp[i] <= brp[i + 1], "row_ptr not monotone");
        const std::vector<int64_t> b = partition_block_rows(brp, parts, row_weight);
        std::copy(b.begin(), b.end(), bounds);
    });
}

XS_API xspmm_status_t xspmm_dist_unique_id(unsigned char* id, int32_t id_bytes) {
    return guarded([&] {
        need(id != nullptr, "null id");
        need(id_bytes >= (int32_t)sizeof(ncclUniqueId), "id buffer smaller than NCCL's unique id");
        ncclUniqueId u;
        const ncclResult_t r = nccl().GetUniqueId(&u);
        XS_REQUIRE(r == ncclSuccess, XSPMM_STATUS_NCCL_ERROR,
                   std::string("ncclGetUniqueId: ") + nccl().GetErrorString(r));
        std::memcpy(id, &u, sizeof(u));
    });
}

XS_API xspmm_status_t xspmm_dist_comm_init(xspmm_handle_t hh, int32_t nranks, int32_t rank,
                                           const unsigned char* id, int32_t id_bytes,
                                           int32_t timeout_ms, xspmm_dist_comm_t* out) {
    return guarded([&] {
        need(out != nullptr, "out is null");
        *out = nullptr;
        Handle& h = H(hh);
        need(nranks >= 1 && rank >= 0 && rank < nranks, "rank outside [0, nranks)");
        need(id != nullptr && id_bytes >= (int32_t)sizeof(ncclUniqueId), "bad unique id");
        const NcclApi& api = nccl();
        DeviceGuard g(h.device);
        ncclUniqueId u;
        std::memcpy(&u, id, sizeof(u));
        ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
        cfg.blocking = 0;  // init returns at once; completion is polled under the time limit
        auto c = std::make_unique<xspmm_dist_comm_s>();
        c->nranks = nranks;
        c->rank = rank;
        c->device = h.device;
        c->owned = true;
        const ncclResult_t r = api.CommInitRankConfig(&c->c, nranks, u, rank, &cfg);
        if (r != ncclSuccess && r != ncclInProgress) {
            if (c->c) api.CommAbort(c->c);
            throw Error(XSPMM_STATUS_NCCL_ERROR,
                        std::string("ncclCommInitRankConfig: ") + api.GetErrorString(r));
        }
        comm_wait(c.get(), h.stream, timeout_ms, false);  // throws TIMEOUT / NCCL_ERROR (aborted)
        *out = c.release();
    });
}

XS_API xspmm_status_t xspmm_dist_comm_wrap(void* nccl_comm, int32_t device,
                                           xspmm_dist_comm_t* out) {
    return guarded([&] {
        need(out != nullptr && nccl_comm != nullptr, "null communicator");
        const NcclApi& api = nccl();
        auto c = std::make_unique<xspmm_dist_comm_s>();
        c->c = static_cast<ncclComm_t>(nccl_comm);
        c->device = device;
        c->owned = false;
        XS_REQUIRE(api.CommCount(c->c, &c->nranks) == ncclSuccess &&
                       api.CommUserRank(c->c, &c->rank) == ncclSuccess,
                   XSPMM_STATUS_NCCL_ERROR, "not a usable NCCL communicator");
        *out = c.release();
    });
}

XS_API xspmm_status_t xspmm_dist_comm_destroy(xspmm_dist_comm_t c) {
    return guarded([&] {
        if (!c) return;
        std::unique_ptr<xspmm_dist_comm_s> own(c);
        if (own->owned && own->c && !own->aborted) {
            DeviceGuard g(own->device);
            nccl().CommDestroy(own->c);
        }
    });
}

#define XS_DIST_PLAN(SUF, VT, IT)                                                                  \
    XS_API xspmm_status_t xspmm_dist_plan_csr_##SUF(                                               \
        xspmm_handle_t hh, xspmm_dist_comm_t cc, IT M, IT K, IT nnz, const IT* rp, const IT* ci,   \
        const void* v, IT hw, int clustering, double row_weight, xspmm_dist_plan_t* out) {         \
        return guarded([&] {                                                                       \
            need(out != nullptr, "out is null");                                                   \
            *out = nullptr;                                                                        \
            Handle& h = H(hh);                                                                     \
            xspmm_dist_comm_s* c = CM(cc);                                                         \
            need(M >= 0 && K >= 0 && nnz >= 0 && row_weight >= 0.0, "negative argument");          \
            need(hw >= 1, "hw_block_size must be at least 1");                                     \
            need(c->device == h.device, "communicator and handle on different devices");           \
            need(M == 0 || rp, "null row_ptr");                                                    \
            need(nnz == 0 || (ci && v), "null col_ind or values");                                 \
            DeviceGuard g(h.device);                                                               \
            auto ps = std::make_unique<xspmm_dist_plan_s>();                                       \
            ps->owner = hh;                                                                        \
            ps->comm = c;                                                                          \
            ps->p = dist_plan_build<VT, IT>(h, c, M, K, nnz, rp, ci, static_cast<const VT*>(v),    \
                                            hw, clustering != 0, row_weight);                      \
            ps->p->value_bytes = (int)sizeof(VT);                                                  \
            hh->live_plans += 1;                                                                   \
            *out = ps.release();                                                                   \
        });                                                                                        \
    }
XS_DIST_PLAN(f16f32_i32, __half, int32_t)
XS_DIST_PLAN(f16f32_i64, __half, int64_t)
XS_DIST_PLAN(bf16f32_i32, __nv_bfloat16, int32_t)
XS_DIST_PLAN(bf16f32_i64, __nv_bfloat16, int64_t)
XS_DIST_PLAN(f32f32_i32, float, int32_t)
XS_DIST_PLAN(f32f32_i64, float, int64_t)

XS_API xspmm_status_t xspmm_dist_plan_get_info(xspmm_dist_plan_t pp, xspmm_dist_plan_info_t* info) {
    return guarded([&] {
        need(info != nullptr, "info is null");
        const DistPlanBase& p = *DP(pp)->p;
        info->rows = p.M;
        info->cols = p.K;
        info->row_begin = p.row_begin;
        info->row_end = p.row_end;
        info->block_begin = p.block_begin;
        info->block_end = p.block_end;
        info->nnz_blocks = p.nnzb;
        info->nnz_blocks_total = p.nnzb_total;
        info->clustered = p.clustered ? 1 : 0;
        info->value_bytes = p.value_bytes;
        info->device_bytes = p.device_bytes();
    });
}

XS_API xspmm_status_t xspmm_dist_plan_execute(xspmm_dist_plan_t pp, void* B, float* C_local,
                                              int64_t N, int32_t bcast_root, int32_t timeout_ms) {
    return guarded([&] {
        xspmm_dist_plan_s* ps = DP(pp);
        Handle& h = ps->owner->h;
        xspmm_dist_comm_s* c = CM(ps->comm);
        DistPlanBase& p = *ps->p;
        need(N >= 0, "negative dimension");
        need(bcast_root < c->nranks, "broadcast root outside the communicator");
        need(p.K == 0 || N == 0 || B != nullptr, "null B");
        need(p.row_end == p.row_begin || N == 0 || C_local != nullptr, "null C_local");
        DeviceGuard g(h.device);
        p.execute(h, c, B, C_local, N, bcast_root, timeout_ms);
    });
}

XS_API xspmm_status_t xspmm_dist_gather(xspmm_dist_plan_t pp, const float* C_local, float* C,
                                        int64_t N, int32_t root, int32_t timeout_ms) {
    return guarded([&] {
        xspmm_dist_plan_s* ps = DP(pp);
        Handle& h = ps->owner->h;
        xspmm_dist_comm_s* c = CM(ps->comm);
        DistPlanBase& p = *ps->p;
        need(N >= 0, "negative dimension");
        need(root >= 0 && root < c->nranks, "root outside the communicator");
        need(c->rank != root || p.M == 0 || N == 0 || C != nullptr, "null C on the root");
        need(p.row_end == p.row_begin || N == 0 || C_local != nullptr, "null C_local");
        DeviceGuard g(h.device);
        p.gather(h, c, C_local, C, N, root, timeout_ms);
    });
}

XS_API xspmm_status_t xspmm_dist_plan_destroy(xspmm_dist_plan_t pp) {
    return guarded([&] {
        if (!pp) return;
        xspmm_dist_plan_s* ps = DP(pp);
        Handle& h = ps->owner->h;
        DeviceGuard g(h.device);
        ps->p->rebind_stream(h.stream);
        ps->p.reset();
        ps->owner->live_plans -= 1;
        delete ps;
    });
}
