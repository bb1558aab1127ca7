// spmm_f32.cu -- Tier-1 BCSR SpMM for fp32 blocks x fp32 B -> fp32 C on the SIMT FMA pipe.
//
// B200's tensor cores have no fp32 multiply, and TF32 (10-bit mantissa) cannot meet the 1e-5
// relative tolerance, so this instantiation (src/cuda/unstructured_mtx_mul.cu:140-141, which the
// reference cannot compile: wmma has no float A/B fragments) runs on FFMA. It skips the zero
// entries of each block: a block of an unstructured matrix is mostly zeros (1.1 % fill on the
// 4096^2 / 1 % plumbing config), so only its nonzero columns k cause a load of B row 16*col+k.
// Skipping a zero differs from the dense block product only when B holds inf or NaN
// (0 * inf = NaN); B is required to be finite for bit-level NaN parity.
//
// Accumulation is fp64: the product of two fp32 numbers is exact in fp64 and the sum then carries
// ~2^-53 relative error, so C is the exact product rounded once to fp32 except where terms cancel
// almost completely. fp32 accumulation cannot meet a 1e-5 relative bound on outputs much smaller
// than the terms that sum to them; the kernel is bound by memory, so the FP64 pipe costs nothing.
//
// Work split: a warp owns one block row and 32 columns of C (one column per lane, 16 fp64
// accumulators per lane, one per row of the block row). For each block it stages the 16x16 values
// in shared memory, finds the block's nonzero columns k with ballots, and for each of them loads
// B[16 col + k, lane] once and does 16 fused multiply-adds against the block's column read by
// broadcast -- branch-free, with no shuffles. When there are too few (block row, column tile)
// units to fill the GPU, S = 2, 4 or 8 warps share a unit, taking every S-th block, and their sums
// are added in warp order through shared memory, so results do not depend on timing.
#include "ops.cuh"

namespace xspmm_b200 {
namespace {

constexpr int F32_WARPS = 8;
constexpr int F32_TN = 32;  // columns per warp

template <typename IT, bool VEC>
__global__ void __launch_bounds__(F32_WARPS * 32, 4)
bcsr_spmm_f32_kernel(const IT* __restrict__ row_ptr, const IT* __restrict__ col_ind,
                     const float* __restrict__ vals, const float* __restrict__ B,
                     float* __restrict__ C, const IT* __restrict__ row_map,
                     const int32_t* __restrict__ br_list, int64_t M, int64_t K, int64_t N,
                     int64_t units, int64_t ntiles, int S, unsigned* __restrict__ err) {
    __shared__ float As[F32_WARPS][16][16];
    __shared__ double red[F32_WARPS][16][F32_TN];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t unit = (int64_t)blockIdx.x * (F32_WARPS / S) + warp / S;
    const int sub = warp % S;
    const bool active = unit < units;
    const int64_t br = active ? (br_list ? (int64_t)br_list[unit / ntiles] : unit / ntiles) : 0;
    const int64_t col = (active ? unit % ntiles : 0) * F32_TN + lane;

    double acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = 0.0;

    if (active) {
        const int64_t jb = row_ptr[br], je = row_ptr[br + 1];
        for (int64_t j = jb + sub; j < je; j += S) {
            const int64_t bc = (int64_t)col_ind[j];
            float v[8];  // row lane / 2, columns (lane & 1) * 8 .. + 7
            const float* src = vals + j * 256 + lane * 8;
            if constexpr (VEC) {
                const float4 x0 = __ldg(reinterpret_cast<const float4*>(src));
                const float4 x1 = __ldg(reinterpret_cast<const float4*>(src) + 1);
                v[0] = x0.x; v[1] = x0.y; v[2] = x0.z; v[3] = x0.w;
                v[4] = x1.x; v[5] = x1.y; v[6] = x1.z; v[7] = x1.w;
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] = __ldg(src + e);
            }
            uint32_t cm = 0;  // nonzero columns of the block
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const uint32_t m = __ballot_sync(0xffffffffu, v[e] != 0.0f);
                if (m & 0x55555555u) cm |= 1u << e;
                if (m & 0xAAAAAAAAu) cm |= 1u << (8 + e);
            }
            __syncwarp();
#pragma unroll
            for (int e = 0; e < 8; ++e) As[warp][lane >> 1][(lane & 1) * 8 + e] = v[e];
            __syncwarp();
            // one B row per nonzero column; more loads in flight cost more registers than they
            // save at this occupancy (measured)
            while (cm) {
                const int k = __ffs(cm) - 1;
                cm &= cm - 1u;
                const int64_t grow = bc * 16 + k;
                const double b = (grow < K && col < N) ? (double)__ldg(B + grow * N + col) : 0.0;
#pragma unroll
                for (int i = 0; i < 16; ++i) acc[i] = fma((double)As[warp][i][k], b, acc[i]);
            }
        }
    }

    if (S > 1) {  // the S warps of a unit are consecutive; sum them in warp order
#pragma unroll
        for (int i = 0; i < 16; ++i) red[warp][i][lane] = acc[i];
        __syncthreads();
        if (sub == 0 && active) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                double t = red[warp][i][lane];
                for (int q = 1; q < S; ++q) t += red[warp + q][i][lane];
                acc[i] = t;
            }
        }
    }
    if (sub == 0 && active && col < N) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int64_t r = br * 16 + i;
            if (r < M) {
                const int64_t orow = row_map ? (int64_t)row_map[r] : r;
                if (orow < 0 || orow >= M) flag_error(err, DERR_PERM_OUT_OF_RANGE);
                else C[orow * N + col] = (float)acc[i];
            }
        }
    }
}

// br_list (device, optional): the block rows to compute, nbr of them; all block rows if null.
template <typename IT>
void bcsr_spmm_f32_impl(Handle& h, const int32_t* br_list, int64_t nbr, const IT* rp,
                        const IT* ci, const float* v, const float* B, float* C, int64_t M,
                        int64_t K, int64_t N, const IT* map) {
    if (nbr == 0 || N == 0 || M == 0) return;
    const int64_t ntiles = ceil_div(N, F32_TN);
    const int64_t units = nbr * ntiles;
    // split a unit's blocks over S warps when the units alone would leave SMs short of warps
    const int64_t want = (int64_t)sm_count(h.device) * 32;
    int S = 1;
    while (S < F32_WARPS && units * S < want) S *= 2;
    const int64_t grid = ceil_div(units * S, F32_WARPS);
    XS_REQUIRE(grid < (int64_t(1) << 31), XSPMM_STATUS_UNSUPPORTED, "grid too large");
    const bool vec = reinterpret_cast<uintptr_t>(v) % 16 == 0;
    if (vec)
        bcsr_spmm_f32_kernel<IT, true><<<(unsigned)grid, F32_WARPS * 32, 0, h.stream>>>(
            rp, ci, v, B, C, map, br_list, M, K, N, units, ntiles, S, h.d_err);
    else
        bcsr_spmm_f32_kernel<IT, false><<<(unsigned)grid, F32_WARPS * 32, 0, h.stream>>>(
            rp, ci, v, B, C, map, br_list, M, K, N, units, ntiles, S, h.d_err);
    after_launch(h, "bcsr_spmm_f32");
}

}  // namespace

template <>
void bcsr_spmm<float, int32_t>(Handle& h, int64_t nbr, int64_t, int64_t, const int32_t* rp,
                               const int32_t* ci, const float* v, const float* B, float* C,
                               int64_t M, int64_t K, int64_t N, const int32_t* map) {
    bcsr_spmm_f32_impl<int32_t>(h, nullptr, nbr, rp, ci, v, B, C, M, K, N, map);
}
template <>
void bcsr_spmm<float, int64_t>(Handle& h, int64_t nbr, int64_t, int64_t, const int64_t* rp,
                               const int64_t* ci, const float* v, const float* B, float* C,
                               int64_t M, int64_t K, int64_t N, const int64_t* map) {
    bcsr_spmm_f32_impl<int64_t>(h, nullptr, nbr, rp, ci, v, B, C, M, K, N, map);
}

template <typename IT>
void bcsr_spmm_f32_rows(Handle& h, const int32_t* br_list, int64_t nlist, const IT* rp,
                        const IT* ci, const float* v, const float* B, float* C, int64_t M,
                        int64_t K, int64_t N, const IT* map) {
    bcsr_spmm_f32_impl<IT>(h, br_list, nlist, rp, ci, v, B, C, M, K, N, map);
}
template void bcsr_spmm_f32_rows<int32_t>(Handle&, const int32_t*, int64_t, const int32_t*,
                                          const int32_t*, const float*, const float*, float*,
                                          int64_t, int64_t, int64_t, const int32_t*);
template void bcsr_spmm_f32_rows<int64_t>(Handle&, const int32_t*, int64_t, const int64_t*,
                                          const int64_t*, const float*, const float*, float*,
                                          int64_t, int64_t, int64_t, const int64_t*);

}  // namespace xspmm_b200
