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
//
// Inside a plan the kernel runs over a work list of pieces (F32Work): the block rows a gather
// split leaves, with block rows far above the average length (an arrowhead's dense first block
// row: 256 blocks against ~3) cut into pieces of equal length whose fp64 partials go to a
// workspace and are added in piece order by f32_reduce_kernel. Without the cut one warp walks
// the whole long row and sets the time of the launch.
#include "ops.cuh"

#include <algorithm>
#include <vector>

namespace xspmm_b200 {
namespace {

constexpr int F32_WARPS = 8;
constexpr int F32_TN = 32;  // columns per warp

template <typename IT, bool VEC>
__global__ void __launch_bounds__(F32_WARPS * 32, 4)
bcsr_spmm_f32_kernel(const IT* __restrict__ row_ptr, const IT* __restrict__ col_ind,
                     const float* __restrict__ vals, const float* __restrict__ B,
                     float* __restrict__ C, const IT* __restrict__ row_map,
                     const F32Piece* __restrict__ pieces, double* __restrict__ ws, int64_t M,
                     int64_t K, int64_t N, int64_t units, int64_t ntiles, int S,
                     unsigned* __restrict__ err) {
    __shared__ float As[F32_WARPS][16][16];
    __shared__ double red[F32_WARPS][16][F32_TN];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t unit = (int64_t)blockIdx.x * (F32_WARPS / S) + warp / S;
    const int sub = warp % S;
    const bool active = unit < units;
    const int64_t col = (active ? unit % ntiles : 0) * F32_TN + lane;
    int64_t br = 0, jb = 0, je = 0;
    int slot = -1;
    if (active) {
        if (pieces) {
            const F32Piece pc = pieces[unit / ntiles];
            br = pc.br; jb = pc.j0; je = pc.j1; slot = pc.slot;
        } else {
            br = unit / ntiles; jb = row_ptr[br]; je = row_ptr[br + 1];
        }
    }

    double acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = 0.0;

    if (active) {
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
    if (sub == 0 && active && col < N && slot >= 0) {  // a piece of a cut block row
#pragma unroll
        for (int i = 0; i < 16; ++i) ws[((int64_t)slot * 16 + i) * N + col] = acc[i];
        return;
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

// C rows of the cut block rows: the sum of their pieces' partials in piece order, rounded once.
template <typename IT>
__global__ void f32_reduce_kernel(const int32_t* __restrict__ long_br,
                                  const int32_t* __restrict__ first, int64_t nlong,
                                  const double* __restrict__ ws, float* __restrict__ C,
                                  const IT* __restrict__ row_map, int64_t M, int64_t N,
                                  unsigned* __restrict__ err) {
    const int64_t total = nlong * 16 * N;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t li = t / N, n = t - li * N;
        const int64_t l = li >> 4, i = li & 15;
        const int64_t r = (int64_t)long_br[l] * 16 + i;
        if (r >= M) continue;
        double acc = 0.0;
        for (int q = first[l]; q < first[l + 1]; ++q) acc += ws[((int64_t)q * 16 + i) * N + n];
        const int64_t orow = row_map ? (int64_t)row_map[r] : r;
        if (orow < 0 || orow >= M) {
            flag_error(err, DERR_PERM_OUT_OF_RANGE);
            continue;
        }
        C[orow * N + n] = (float)acc;
    }
}

// pieces (device, optional): nunits_rows work items, each a block row or a piece of one; all
// block rows in order if null.
template <typename IT>
void bcsr_spmm_f32_impl(Handle& h, const F32Piece* pieces, double* ws, int64_t nrows_work,
                        const IT* rp, const IT* ci, const float* v, const float* B, float* C,
                        int64_t M, int64_t K, int64_t N, const IT* map) {
    if (nrows_work == 0 || N == 0 || M == 0) return;
    const int64_t ntiles = ceil_div(N, F32_TN);
    const int64_t units = nrows_work * ntiles;
    // split a unit's blocks over S warps when the units alone would leave SMs short of warps
    const int64_t want = (int64_t)sm_count(h.device) * 32;
    int S = 1;
    while (S < F32_WARPS && units * S < want) S *= 2;
    const int64_t grid = ceil_div(units * S, F32_WARPS);
    XS_REQUIRE(grid < (int64_t(1) << 31), XSPMM_STATUS_UNSUPPORTED, "grid too large");
    const bool vec = reinterpret_cast<uintptr_t>(v) % 16 == 0;
    if (vec)
        bcsr_spmm_f32_kernel<IT, true><<<(unsigned)grid, F32_WARPS * 32, 0, h.stream>>>(
            rp, ci, v, B, C, map, pieces, ws, M, K, N, units, ntiles, S, h.d_err);
    else
        bcsr_spmm_f32_kernel<IT, false><<<(unsigned)grid, F32_WARPS * 32, 0, h.stream>>>(
            rp, ci, v, B, C, map, pieces, ws, M, K, N, units, ntiles, S, h.d_err);
    after_launch(h, "bcsr_spmm_f32");
}

}  // namespace

template <>
void bcsr_spmm<float, int32_t>(Handle& h, int64_t nbr, int64_t, int64_t, const int32_t* rp,
                               const int32_t* ci, const float* v, const float* B, float* C,
                               int64_t M, int64_t K, int64_t N, const int32_t* map) {
    bcsr_spmm_f32_impl<int32_t>(h, nullptr, nullptr, nbr, rp, ci, v, B, C, M, K, N, map);
}
template <>
void bcsr_spmm<float, int64_t>(Handle& h, int64_t nbr, int64_t, int64_t, const int64_t* rp,
                               const int64_t* ci, const float* v, const float* B, float* C,
                               int64_t M, int64_t K, int64_t N, const int64_t* map) {
    bcsr_spmm_f32_impl<int64_t>(h, nullptr, nullptr, nbr, rp, ci, v, B, C, M, K, N, map);
}

void f32_work_build(Handle& h, int64_t nbr, const std::vector<int64_t>& hrp,
                    const std::vector<uint8_t>* keep, F32Work& out) {
    cudaStream_t s = h.stream;
    out = F32Work();
    out.built = true;
    if (nbr == 0) return;
    XS_REQUIRE(nbr < (int64_t(1) << 31) && (int64_t)hrp.size() == nbr + 1,
               XSPMM_STATUS_UNSUPPORTED, "too many block rows");
    int64_t nrows = 0, nblocks = 0;
    for (int64_t br = 0; br < nbr; ++br) {
        if (keep && !(*keep)[br]) continue;
        ++nrows;
        nblocks += (int64_t)hrp[br + 1] - hrp[br];
    }
    // Piece length: twice the average block row, at least 8 blocks, doubled while the cut rows
    // would need more than 1,024 workspace slots (a slot is 16 rows x N fp64: 32 MB at N = 256).
    int64_t P = std::max<int64_t>(8, 2 * ceil_div(nblocks, std::max<int64_t>(nrows, 1)));
    auto slots_for = [&](int64_t p) {
        int64_t n = 0;
        for (int64_t br = 0; br < nbr; ++br) {
            if (keep && !(*keep)[br]) continue;
            const int64_t nb = (int64_t)hrp[br + 1] - hrp[br];
            if (nb > p) n += ceil_div(nb, p);
        }
        return n;
    };
    while (slots_for(P) > 1024) P *= 2;
    std::vector<F32Piece> pieces;
    std::vector<int32_t> long_br, long_first;
    int32_t slot = 0;
    for (int64_t br = 0; br < nbr; ++br) {
        if (keep && !(*keep)[br]) continue;
        const int64_t j0 = hrp[br], j1 = hrp[br + 1];
        if (j1 - j0 <= P) {
            pieces.push_back(F32Piece{j0, j1, (int32_t)br, -1});
            continue;
        }
        long_br.push_back((int32_t)br);
        long_first.push_back(slot);
        const int64_t np = ceil_div(j1 - j0, P), len = ceil_div(j1 - j0, np);  // equal pieces
        for (int64_t j = j0; j < j1; j += len)
            pieces.push_back(F32Piece{j, std::min(j + len, j1), (int32_t)br, slot++});
    }
    long_first.push_back(slot);
    out.npieces = (int64_t)pieces.size();
    out.nlong = (int64_t)long_br.size();
    out.nslots = slot;
    if (out.npieces == 0) return;
    out.pieces = DevBuf<F32Piece>(pieces.size(), s);
    XS_CHECK_CUDA(cudaMemcpyAsync(out.pieces.get(), pieces.data(), pieces.size() * sizeof(F32Piece),
                                  cudaMemcpyHostToDevice, s));
    if (out.nlong > 0) {
        out.long_br = DevBuf<int32_t>(long_br.size(), s);
        out.long_first = DevBuf<int32_t>(long_first.size(), s);
        XS_CHECK_CUDA(cudaMemcpyAsync(out.long_br.get(), long_br.data(),
                                      long_br.size() * sizeof(int32_t), cudaMemcpyHostToDevice, s));
        XS_CHECK_CUDA(cudaMemcpyAsync(out.long_first.get(), long_first.data(),
                                      long_first.size() * sizeof(int32_t), cudaMemcpyHostToDevice, s));
    }
    XS_CHECK_CUDA(cudaStreamSynchronize(s));  // the host vectors go out of scope
}

template <typename IT>
void bcsr_spmm_f32_work(Handle& h, const F32Work& w, const IT* rp, const IT* ci, const float* v,
                        const float* B, float* C, int64_t M, int64_t K, int64_t N, const IT* map) {
    if (w.npieces == 0 || N == 0 || M == 0) return;
    DevBuf<double> ws(w.nslots > 0 ? (size_t)w.nslots * 16 * (size_t)N : 0, h.stream);
    bcsr_spmm_f32_impl<IT>(h, w.pieces.get(), ws.get(), w.npieces, rp, ci, v, B, C, M, K, N, map);
    if (w.nlong > 0) {
        const int64_t total = w.nlong * 16 * N;
        const unsigned grid = (unsigned)std::max<int64_t>(
            1, std::min(ceil_div(total, 256), (int64_t)sm_count(h.device) * 16));
        f32_reduce_kernel<IT><<<grid, 256, 0, h.stream>>>(w.long_br.get(), w.long_first.get(),
                                                          w.nlong, ws.get(), C, map, M, N, h.d_err);
        after_launch(h, "f32_reduce");
    }
}

#define XS_INST_F32W(IT)                                                                          \
    template void bcsr_spmm_f32_work<IT>(Handle&, const F32Work&, const IT*, const IT*,           \
                                         const float*, const float*, float*, int64_t, int64_t,    \
                                         int64_t, const IT*);
XS_INST_F32W(int32_t)
XS_INST_F32W(int64_t)

}  // namespace xspmm_b200
