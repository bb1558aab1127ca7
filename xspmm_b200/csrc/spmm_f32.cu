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
// Work split: a CTA owns one block row and 64 columns (2 per lane, float2 when aligned). Its 8
// warps take the block row's blocks round-robin, each keeping 16x2 fp64 accumulators per lane, and
// reduce through shared memory in a fixed warp order, so results are deterministic.
#include "ops.cuh"

namespace xspmm_b200 {
namespace {

constexpr int F32_WARPS = 8;
constexpr int F32_TN = 64;

// Keeps the bits at even positions of x and packs them into the low 16 bits.
__device__ __forceinline__ uint32_t pack_even_bits(uint32_t x) {
    x &= 0x55555555u;
    x = (x | (x >> 1)) & 0x33333333u;
    x = (x | (x >> 2)) & 0x0F0F0F0Fu;
    x = (x | (x >> 4)) & 0x00FF00FFu;
    x = (x | (x >> 8)) & 0x0000FFFFu;
    return x;
}

template <typename IT, bool ALIGNED>
__global__ void __launch_bounds__(F32_WARPS * 32)
bcsr_spmm_f32_kernel(const IT* __restrict__ row_ptr, const IT* __restrict__ col_ind,
                     const float* __restrict__ vals, const float* __restrict__ B,
                     float* __restrict__ C, const IT* __restrict__ row_map, int64_t M, int64_t K,
                     int64_t N, unsigned* __restrict__ err) {
    __shared__ __align__(16) double red[F32_WARPS][8][F32_TN];
    const int64_t br = blockIdx.x;
    const int64_t n0 = (int64_t)blockIdx.y * F32_TN;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t col0 = n0 + 2 * lane;
    const int64_t jb = row_ptr[br], je = row_ptr[br + 1];

    double acc[16][2];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i][0] = acc[i][1] = 0.0;

    for (int64_t j = jb + warp; j < je; j += F32_WARPS) {
        const int64_t bc = (int64_t)col_ind[j];
        float v[8];
        const float* src = vals + j * 256 + lane * 8;  // row lane/2, cols (lane&1)*8 .. +7
        if constexpr (ALIGNED) {
            const float4 x0 = __ldg(reinterpret_cast<const float4*>(src));
            const float4 x1 = __ldg(reinterpret_cast<const float4*>(src) + 1);
            v[0] = x0.x; v[1] = x0.y; v[2] = x0.z; v[3] = x0.w;
            v[4] = x1.x; v[5] = x1.y; v[6] = x1.z; v[7] = x1.w;
        } else {
#pragma unroll
            for (int s = 0; s < 8; ++s) v[s] = src[s];
        }
        uint32_t colrows[16];
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            const uint32_t m = __ballot_sync(0xffffffffu, v[s] != 0.0f);
            colrows[s] = pack_even_bits(m);
            colrows[8 + s] = pack_even_bits(m >> 1);
        }
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const uint32_t rm = colrows[k];
            if (rm == 0) continue;  // warp-uniform
            const int64_t grow = bc * 16 + k;
            if (grow >= K) continue;
            double b[2];
            const float* brow = B + grow * N;
            if constexpr (ALIGNED) {
                if (col0 < N) {
                    const float2 x = __ldg(reinterpret_cast<const float2*>(brow + col0));
                    b[0] = x.x; b[1] = x.y;
                } else {
                    b[0] = b[1] = 0.0;
                }
            } else {
#pragma unroll
                for (int e = 0; e < 2; ++e) b[e] = col0 + e < N ? (double)brow[col0 + e] : 0.0;
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                if (rm & (1u << i)) {  // warp-uniform
                    const double a = __shfl_sync(0xffffffffu, v[k & 7], 2 * i + (k >> 3));
                    acc[i][0] = fma(a, b[0], acc[i][0]);
                    acc[i][1] = fma(a, b[1], acc[i][1]);
                }
            }
        }
    }

    // Deterministic cross-warp reduction, 8 rows at a time.
#pragma unroll
    for (int half = 0; half < 2; ++half) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            red[warp][i][2 * lane] = acc[8 * half + i][0];
            red[warp][i][2 * lane + 1] = acc[8 * half + i][1];
        }
        __syncthreads();
        for (int t = threadIdx.x; t < 8 * F32_TN; t += F32_WARPS * 32) {
            const int i = t / F32_TN, c = t % F32_TN;
            double s = 0.0;
#pragma unroll
            for (int w = 0; w < F32_WARPS; ++w) s += red[w][i][c];
            const int64_t r = br * 16 + 8 * half + i;
            const int64_t col = n0 + c;
            if (r < M && col < N) {
                const int64_t orow = row_map ? (int64_t)row_map[r] : r;
                if (orow < 0 || orow >= M) flag_error(err, DERR_PERM_OUT_OF_RANGE);
                else C[orow * N + col] = (float)s;
            }
        }
        __syncthreads();
    }
}

template <typename IT>
void bcsr_spmm_f32_impl(Handle& h, int64_t nbr, const IT* rp, const IT* ci, const float* v,
                        const float* B, float* C, int64_t M, int64_t K, int64_t N,
                        const IT* map) {
    if (nbr == 0 || N == 0 || M == 0) return;
    XS_REQUIRE(ceil_div(N, F32_TN) <= 65535, XSPMM_STATUS_UNSUPPORTED, "N above 4,194,240");
    const bool aligned = (N % 2 == 0) && (reinterpret_cast<uintptr_t>(B) % 8 == 0) &&
                         (reinterpret_cast<uintptr_t>(v) % 16 == 0);
    dim3 grid((unsigned)nbr, (unsigned)ceil_div(N, F32_TN));
    if (aligned)
        bcsr_spmm_f32_kernel<IT, true>
            <<<grid, F32_WARPS * 32, 0, h.stream>>>(rp, ci, v, B, C, map, M, K, N, h.d_err);
    else
        bcsr_spmm_f32_kernel<IT, false>
            <<<grid, F32_WARPS * 32, 0, h.stream>>>(rp, ci, v, B, C, map, M, K, N, h.d_err);
    after_launch(h, "bcsr_spmm_f32");
}

}  // namespace

template <>
void bcsr_spmm<float, int32_t>(Handle& h, int64_t nbr, int64_t, int64_t, const int32_t* rp,
                               const int32_t* ci, const float* v, const float* B, float* C,
                               int64_t M, int64_t K, int64_t N, const int32_t* map) {
    bcsr_spmm_f32_impl<int32_t>(h, nbr, rp, ci, v, B, C, M, K, N, map);
}
template <>
void bcsr_spmm<float, int64_t>(Handle& h, int64_t nbr, int64_t, int64_t, const int64_t* rp,
                               const int64_t* ci, const float* v, const float* B, float* C,
                               int64_t M, int64_t K, int64_t N, const int64_t* map) {
    bcsr_spmm_f32_impl<int64_t>(h, nbr, rp, ci, v, B, C, M, K, N, map);
}

}  // namespace xspmm_b200
