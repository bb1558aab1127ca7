// capi_plan.cu -- extern "C" entry points of the plan (include/xspmm_b200.h): build once from a
// CSR matrix (the Tier-2 stages) or adopt a BCSR matrix (Tier 1), then execute many products.
#include "plan.cuh"

using namespace xspmm_b200;

namespace {

xspmm_plan_s* P(xspmm_plan_t p) {
    XS_REQUIRE(p != nullptr && p->p != nullptr && p->owner != nullptr && !p->owner->destroyed,
               XSPMM_STATUS_INVALID_ARGUMENT, "null plan");
    return p;
}

template <typename VT, typename IT>
void adopt(xspmm_handle_t hh, std::unique_ptr<Plan<VT, IT>> plan, xspmm_plan_t* out) {
    auto* ps = new xspmm_plan_s();
    ps->owner = hh;
    ps->p = std::move(plan);
    hh->live_plans += 1;
    *out = ps;
}

}  // namespace

#define XS_PLAN_CSR(SUF, VT, IT)                                                                  \
    XS_API xspmm_status_t xspmm_plan_csr_##SUF(xspmm_handle_t hh, IT M, IT K, IT nnz,             \
                                               const IT* rp, const IT* ci, const void* v, IT hw,  \
                                               int clustering, xspmm_plan_t* out,                 \
                                               xspmm_timings_t* t) {                              \
        return guarded([&] {                                                                      \
            need(out != nullptr, "out is null");                                                  \
            *out = nullptr;                                                                       \
            Handle& h = H(hh);                                                                    \
            need(M >= 0 && K >= 0 && nnz >= 0, "negative dimension");                             \
            need(hw >= 1, "hw_block_size must be at least 1");                                    \
            need(M == 0 || rp, "null row_ptr");                                                   \
            need(nnz == 0 || (ci && v), "null col_ind or values");                                \
            if (t) *t = xspmm_timings_t{0, 0, 0, 0, 0, 0};                                        \
            DeviceGuard g(h.device);                                                              \
            auto plan = std::make_unique<Plan<VT, IT>>();                                         \
            plan_from_csr<VT, IT>(h, M, K, nnz, rp, ci, static_cast<const VT*>(v), hw,            \
                                  clustering != 0, t != nullptr, *plan);                          \
            if (plan_wants_tc(h, plan->nbr, plan->nbc, plan->nnzb)) plan->prepare_tc(h);          \
            if (t) {                                                                              \
                XS_CHECK_CUDA(cudaEventRecord(h.ev[4], h.stream));                                \
                XS_CHECK_CUDA(cudaEventSynchronize(h.ev[4]));                                     \
                float ms[4];                                                                      \
                for (int i = 0; i < 4; ++i)                                                       \
                    XS_CHECK_CUDA(cudaEventElapsedTime(&ms[i], h.ev[i], h.ev[i + 1]));            \
                t->clustering_ms = ms[0];                                                         \
                t->permutation_ms = ms[1];                                                        \
                t->conversion_ms = ms[2] + ms[3];                                                 \
                t->spmm_ms = 0.0;                                                                 \
                t->unpermutation_ms = 0.0;                                                        \
                t->total_pipeline_ms = (double)ms[0] + ms[1] + ms[2] + ms[3];                     \
            }                                                                                     \
            adopt<VT, IT>(hh, std::move(plan), out);                                              \
        });                                                                                       \
    }
XS_PLAN_CSR(f16f32_i32, __half, int32_t)
XS_PLAN_CSR(f16f32_i64, __half, int64_t)
XS_PLAN_CSR(bf16f32_i32, __nv_bfloat16, int32_t)
XS_PLAN_CSR(bf16f32_i64, __nv_bfloat16, int64_t)
XS_PLAN_CSR(f32f32_i32, float, int32_t)
XS_PLAN_CSR(f32f32_i64, float, int64_t)

#define XS_PLAN_BCSR(SUF, VT, IT)                                                                 \
    XS_API xspmm_status_t xspmm_plan_bcsr_##SUF(xspmm_handle_t hh, IT nbr, IT nbc, IT nnzb,       \
                                                IT rb, IT cb, const IT* rp, const IT* ci,         \
                                                const void* v, IT M, IT K, xspmm_plan_t* out) {   \
        return guarded([&] {                                                                      \
            need(out != nullptr, "out is null");                                                  \
            *out = nullptr;                                                                       \
            Handle& h = H(hh);                                                                    \
            XS_REQUIRE(rb == 16 && cb == 16, XSPMM_STATUS_UNSUPPORTED,                            \
                       "Tier-1 SpMM supports 16x16 blocks only");                                 \
            need(nbr >= 0 && nbc >= 0 && nnzb >= 0 && M >= 0 && K >= 0, "negative dimension");    \
            need((int64_t)M <= (int64_t)nbr * 16 && (int64_t)K <= (int64_t)nbc * 16,              \
                 "M or K larger than the block grid");                                            \
            need(nbr == 0 || (int64_t)M > ((int64_t)nbr - 1) * 16,                                \
                 "M smaller than the block rows cover");                                          \
            need(nbr == 0 || rp, "null row_ptr");                                                 \
            need(nnzb == 0 || (ci && v), "null col_ind or values");                               \
            DeviceGuard g(h.device);                                                              \
            auto plan = std::make_unique<Plan<VT, IT>>();                                         \
            plan_from_bcsr<VT, IT>(h, nbr, nbc, nnzb, rp, ci, static_cast<const VT*>(v), M, K,    \
                                   *plan);                                                        \
            if (plan_wants_tc(h, nbr, nbc, nnzb) && reinterpret_cast<uintptr_t>(v) % 16 == 0)     \
                plan->prepare_tc(h);                                                              \
            adopt<VT, IT>(hh, std::move(plan), out);                                              \
        });                                                                                       \
    }
XS_PLAN_BCSR(f16f32_i32, __half, int32_t)
XS_PLAN_BCSR(f16f32_i64, __half, int64_t)
XS_PLAN_BCSR(bf16f32_i32, __nv_bfloat16, int32_t)
XS_PLAN_BCSR(bf16f32_i64, __nv_bfloat16, int64_t)
XS_PLAN_BCSR(f32f32_i32, float, int32_t)
XS_PLAN_BCSR(f32f32_i64, float, int64_t)

XS_API xspmm_status_t xspmm_plan_execute(xspmm_plan_t pp, const void* B, float* C, int64_t N) {
    return guarded([&] {
        xspmm_plan_s* ps = P(pp);
        Handle& h = ps->owner->h;
        PlanBase& p = *ps->p;
        need(N >= 0, "negative dimension");
        if (p.M == 0 || N == 0) return;
        need(C != nullptr, "null C");
        need(p.nnzb == 0 || B != nullptr, "null B");
        DeviceGuard g(h.device);
        p.execute(h, B, C, N);
    });
}

XS_API xspmm_status_t xspmm_plan_get_info(xspmm_plan_t pp, xspmm_plan_info_t* info) {
    return guarded([&] {
        need(info != nullptr, "info is null");
        const PlanBase& p = *P(pp)->p;
        info->rows = p.M;
        info->cols = p.K;
        info->block_rows = p.nbr;
        info->block_cols = p.nbc;
        info->nnz_blocks = p.nnzb;
        info->clustered = p.clustered ? 1 : 0;
        info->value_bytes = p.value_bytes;
        info->tcgen05_ready = p.tc_ready() ? 1 : 0;
        info->reserved = 0;
        info->tcgen05_tiles = p.tc_tiles();
        info->device_bytes = p.device_bytes();
    });
}

XS_API xspmm_status_t xspmm_plan_destroy(xspmm_plan_t pp) {
    return guarded([&] {
        if (!pp) return;
        xspmm_plan_s* ps = P(pp);
        Handle& h = ps->owner->h;
        DeviceGuard g(h.device);
        ps->p->rebind_stream(h.stream);  // free on the stream the handle uses now
        ps->p.reset();
        ps->owner->live_plans -= 1;
        delete ps;
    });
}
