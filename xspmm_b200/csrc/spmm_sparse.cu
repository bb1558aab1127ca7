// spmm_sparse.cu -- Tier-1 for block rows whose 16x16 blocks are nearly empty.
//
// The block product (src/common/spmm_math.hpp:59-122) multiplies every 16x16 block as a dense
// tile: per block it reads the block (512 bytes in fp16) and gathers a 16 x N slab of B. On graph-like
// matrices a block holds one or two nonzeros (R-MAT: ~1.4 of 256, so ~99 % of that traffic and
// of the tensor work multiplies zeros). A plan therefore splits the block rows once:
//   * block rows averaging more than a threshold of nonzeros per block stay on the block kernels
//     (SP_DENSE_NNZ_F16 for the tensor-core kernels, SP_DENSE_NNZ_F32 for the fp32 SIMT one);
//   * the others are extracted, row by row, into a compact (column, value) list in column order
//     (blocks ascending, then the column inside the block) -- the nonzeros of the BCSR values,
//     read once -- and each product then gathers one B row per nonzero: 6 + 2N bytes per
//     nonzero instead of 512 + 32N per block in fp16 (8 + 4N against 1024 + 64N in fp32).
// The result is the same sum, C[16br+i, n] = sum over the row's nonzeros a * B[col, n],
// accumulated in fp64 in column order and rounded once to fp32 (the tensor-core kernels
// accumulate in fp32; the fp32 SIMT kernel also in fp64, in the same column order). A row of a
// split block row with no nonzero is written as zeros, as the block product writes it.
//
// Kernels: a warp per row and 128-column tile (4 columns per lane) for rows of up to SP_LONG
// nonzeros; longer rows (hub rows) are cut into chunks of SP_CHUNK nonzeros, a CTA each, whose
// fp64 partials are added in chunk order afterwards -- results do not depend on timing.
#include "ops.cuh"

#include <algorithm>
#include <vector>

namespace xspmm_b200 {
namespace {

constexpr int SP_TN = 128;          // columns per warp (4 per lane)
constexpr int SP_WARPS = 8;
constexpr int64_t SP_LONG = 256;    // rows with more nonzeros are cut into chunks
constexpr int64_t SP_CHUNK = 2048;  // nonzeros per chunk of a long row
constexpr int SP_UNROLL = 8;        // B rows in flight per warp

// Value-type helpers: 8 consecutive block values of a lane (one 16x16 block row-major: lane l
// holds row l/2, columns (l&1)*8 .. +7), the nonzero test (the sign bit ignored, so -0 counts as
// zero), and 4 consecutive elements of a B row as floats.
template <typename VT> struct SpVT;
template <> struct SpVT<__half> {
    __device__ static void load8(const __half* p, __half (&o)[8]) {
        const uint4 x = *reinterpret_cast<const uint4*>(p);
        *reinterpret_cast<uint4*>(o) = x;
    }
    __device__ static bool nz(__half x) { return (__half_as_ushort(x) & 0x7FFFu) != 0; }
    __device__ static float f(__half x) { return __half2float(x); }
    __device__ static void b4(const __half* p, float (&o)[4]) {  // 8-byte aligned
        const uint2 x = __ldg(reinterpret_cast<const uint2*>(p));
        const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&x.x));
        const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&x.y));
        o[0] = f0.x; o[1] = f0.y; o[2] = f1.x; o[3] = f1.y;
    }
    static constexpr int b4_align = 8;
    using Raw = uint2;  // 4 consecutive elements of a B row, as loaded
    __device__ static Raw raw4(const __half* p) { return __ldg(reinterpret_cast<const uint2*>(p)); }
    __device__ static Raw zero4() { return make_uint2(0u, 0u); }
    __device__ static void f4(const Raw& x, float (&o)[4]) {
        const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&x.x));
        const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&x.y));
        o[0] = f0.x; o[1] = f0.y; o[2] = f1.x; o[3] = f1.y;
    }
};
template <> struct SpVT<float> {
    __device__ static void load8(const float* p, float (&o)[8]) {
        const float4 x0 = *reinterpret_cast<const float4*>(p);
        const float4 x1 = *(reinterpret_cast<const float4*>(p) + 1);
        o[0] = x0.x; o[1] = x0.y; o[2] = x0.z; o[3] = x0.w;
        o[4] = x1.x; o[5] = x1.y; o[6] = x1.z; o[7] = x1.w;
    }
    __device__ static bool nz(float x) { return (__float_as_uint(x) & 0x7FFFFFFFu) != 0; }
    __device__ static float f(float x) { return x; }
    __device__ static void b4(const float* p, float (&o)[4]) {  // 16-byte aligned
        const float4 x = __ldg(reinterpret_cast<const float4*>(p));
        o[0] = x.x; o[1] = x.y; o[2] = x.z; o[3] = x.w;
    }
    static constexpr int b4_align = 16;
    using Raw = float4;
    __device__ static Raw raw4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
    __device__ static Raw zero4() { return make_float4(0.f, 0.f, 0.f, 0.f); }
    __device__ static void f4(const Raw& x, float (&o)[4]) {
        o[0] = x.x; o[1] = x.y; o[2] = x.z; o[3] = x.w;
    }
};

// Per-row nonzero counts (rows of block row br = 16 br .. 16 br + 15), a warp per block row:
// lane 2i and 2i+1 read row i's two halves of every block (8 halves each).
template <typename VT, typename IT>
__global__ void sp_row_count_kernel(const IT* __restrict__ rp, const VT* __restrict__ v,
                                    int64_t nbr, int64_t M, int32_t* __restrict__ rowcnt) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t br = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); br < nbr;
         br += warps) {
        const int64_t j0 = rp[br], j1 = rp[br + 1];
        int c = 0;
        for (int64_t j = j0; j < j1; ++j) {
            VT h[8];
            SpVT<VT>::load8(v + j * 256 + lane * 8, h);
#pragma unroll
            for (int q = 0; q < 8; ++q) c += SpVT<VT>::nz(h[q]);
        }
        c += __shfl_xor_sync(0xffffffffu, c, 1);
        const int64_t r = br * 16 + (lane >> 1);
        if ((lane & 1) == 0 && r < M) rowcnt[r] = c;
    }
}

// Extracts the nonzeros of the listed block rows into rows [rptr[r], rptr[r+1]) in column order.
template <typename VT, typename IT>
__global__ void sp_extract_kernel(const IT* __restrict__ rp, const IT* __restrict__ ci,
                                  const VT* __restrict__ v, const int32_t* __restrict__ brs,
                                  int64_t nbrs, int64_t M, const int64_t* __restrict__ rptr,
                                  int32_t* __restrict__ col, VT* __restrict__ val) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < nbrs;
         t += warps) {
        const int64_t br = brs[t];
        const int64_t r = br * 16 + (lane >> 1);
        int64_t off = r < M ? rptr[r] : 0;  // both lanes of row r track its next slot
        const int64_t j0 = rp[br], j1 = rp[br + 1];
        for (int64_t j = j0; j < j1; ++j) {
            const int64_t bc = (int64_t)ci[j];
            VT h[8];
            SpVT<VT>::load8(v + j * 256 + lane * 8, h);
            int c = 0;
#pragma unroll
            for (int q = 0; q < 8; ++q) c += SpVT<VT>::nz(h[q]);
            const int c_lo = __shfl_sync(0xffffffffu, c, lane & ~1);  // the row's first half
            const int c_all = c_lo + __shfl_sync(0xffffffffu, c, lane | 1);
            if (r < M) {
                int64_t o = off + ((lane & 1) ? c_lo : 0);
                const int k0 = (lane & 1) * 8;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    if (SpVT<VT>::nz(h[q])) {
                        col[o] = (int32_t)(bc * 16 + k0 + q);
                        val[o] = h[q];
                        ++o;
                    }
                }
            }
            off += c_all;
        }
    }
}

// C[map(r), tile] for rows with at most SP_LONG nonzeros: a warp per (row, 128-column tile). The
// row's descriptor (first nonzero, count, row) is one 16-byte load, so the chain of dependent
// loads before the B rows is descriptor -> (column, value) pairs -> B rows. The warp loads 32
// pairs at once (coalesced), broadcasts them and keeps SP_UNROLL B rows in flight (raw fp16 in
// registers until they are used); nonzeros are still added in column order, in fp64.
template <typename VT, typename IT, bool VEC>
__global__ void __launch_bounds__(SP_WARPS * 32, sizeof(VT) == 2 ? 4 : 2)
sp_gather_short_kernel(const SpRow* __restrict__ rows, int64_t nrows,
                       const int32_t* __restrict__ col, const VT* __restrict__ val,
                       const VT* __restrict__ B, float* __restrict__ C,
                       const IT* __restrict__ row_map, int64_t M, int64_t K, int64_t N,
                       unsigned* __restrict__ err) {
    const int lane = threadIdx.x & 31;
    const int64_t t = (int64_t)blockIdx.x * SP_WARPS + (threadIdx.x >> 5);
    if (t >= nrows) return;
    const SpRow ri = rows[t];
    const int64_t r = ri.row, e0 = ri.e0;
    const int n_all = ri.cnt;
    const int64_t n0 = (int64_t)blockIdx.y * SP_TN + lane * 4;
    double acc[4] = {0.0, 0.0, 0.0, 0.0};
    for (int base = 0; base < n_all; base += 32) {
        const int cnt = min(32, n_all - base);
        const int64_t my_c = lane < cnt ? (int64_t)col[e0 + base + lane] : 0;
        const float my_a = lane < cnt ? SpVT<VT>::f(val[e0 + base + lane]) : 0.0f;
        for (int u0 = 0; u0 < cnt; u0 += SP_UNROLL) {
            typename SpVT<VT>::Raw raw[SP_UNROLL];
            float a[SP_UNROLL];
            bool lv[SP_UNROLL];
#pragma unroll
            for (int u = 0; u < SP_UNROLL; ++u) {
                const int64_t c = __shfl_sync(0xffffffffu, my_c, (u0 + u) & 31);
                a[u] = __shfl_sync(0xffffffffu, my_a, (u0 + u) & 31);
                lv[u] = u0 + u < cnt && c < K;
                const VT* src = B + c * N + n0;
                if (VEC && lv[u] && n0 + 4 <= N) {
                    raw[u] = SpVT<VT>::raw4(src);
                } else {
                    raw[u] = SpVT<VT>::zero4();
                }
            }
#pragma unroll
            for (int u = 0; u < SP_UNROLL; ++u) {
                if (u0 + u < cnt) {
                    float bb[4];
                    if (VEC) {
                        SpVT<VT>::f4(raw[u], bb);
                    } else {
                        const int64_t c = __shfl_sync(0xffffffffu, my_c, (u0 + u) & 31);
                        const VT* src = B + c * N + n0;
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            bb[q] = (lv[u] && n0 + q < N) ? SpVT<VT>::f(src[q]) : 0.0f;
                    }
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        acc[q] = fma((double)a[u], (double)bb[q], acc[q]);
                }
            }
        }
    }
    if (r >= M) return;
    const int64_t orow = row_map ? (int64_t)row_map[r] : r;
    if (orow < 0 || orow >= M) {
        if (lane == 0) flag_error(err, DERR_PERM_OUT_OF_RANGE);
        return;
    }
    float* dst = C + orow * N + n0;
    if (VEC && n0 + 4 <= N) {
        *reinterpret_cast<float4*>(dst) =
            make_float4((float)acc[0], (float)acc[1], (float)acc[2], (float)acc[3]);
    } else {
#pragma unroll
        for (int q = 0; q < 4; ++q)
            if (n0 + q < N) dst[q] = (float)acc[q];
    }
}

// Rows with more than SP_LONG nonzeros are cut into chunks of at most SP_CHUNK nonzeros: a CTA
// per (chunk, tile), warp w summing its contiguous eighth of the chunk, the 8 warp sums added in
// warp order into the chunk's fp64 partial; then sp_reduce_kernel adds a row's chunk partials in
// chunk order and rounds once. (One CTA per hub row of ~40K nonzeros set the time of the whole
// product.)
template <typename VT, bool VEC>
__global__ void __launch_bounds__(SP_WARPS * 32)
sp_gather_chunk_kernel(const SparseChunk* __restrict__ chunks, const int32_t* __restrict__ col,
                       const VT* __restrict__ val, const VT* __restrict__ B,
                       double* __restrict__ ws, int64_t K, int64_t N) {
    __shared__ double red[SP_WARPS][SP_TN];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const SparseChunk ck = chunks[blockIdx.x];
    const int64_t n0 = (int64_t)blockIdx.y * SP_TN + lane * 4;
    const int64_t len = ck.e1 - ck.e0, per = (len + SP_WARPS - 1) / SP_WARPS;
    const int64_t w0 = ck.e0 + min(len, per * warp), w1 = ck.e0 + min(len, per * (warp + 1));
    double acc[4] = {0.0, 0.0, 0.0, 0.0};
    for (int64_t base = w0; base < w1; base += 32) {
        const int cnt = (int)min((int64_t)32, w1 - base);
        const int64_t my_c = lane < cnt ? (int64_t)col[base + lane] : 0;
        const float my_a = lane < cnt ? SpVT<VT>::f(val[base + lane]) : 0.0f;
        for (int u0 = 0; u0 < cnt; u0 += SP_UNROLL) {
            typename SpVT<VT>::Raw raw[SP_UNROLL];
            float a[SP_UNROLL];
            bool lv[SP_UNROLL];
#pragma unroll
            for (int u = 0; u < SP_UNROLL; ++u) {
                const int64_t c = __shfl_sync(0xffffffffu, my_c, (u0 + u) & 31);
                a[u] = __shfl_sync(0xffffffffu, my_a, (u0 + u) & 31);
                lv[u] = u0 + u < cnt && c < K;
                raw[u] = (VEC && lv[u] && n0 + 4 <= N) ? SpVT<VT>::raw4(B + c * N + n0)
                                                        : SpVT<VT>::zero4();
            }
#pragma unroll
            for (int u = 0; u < SP_UNROLL; ++u) {
                if (u0 + u < cnt) {
                    float bb[4];
                    if (VEC) {
                        SpVT<VT>::f4(raw[u], bb);
                    } else {
                        const int64_t c = __shfl_sync(0xffffffffu, my_c, (u0 + u) & 31);
                        const VT* src = B + c * N + n0;
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            bb[q] = (lv[u] && n0 + q < N) ? SpVT<VT>::f(src[q]) : 0.0f;
                    }
#pragma unroll
                    for (int q = 0; q < 4; ++q) acc[q] = fma((double)a[u], (double)bb[q], acc[q]);
                }
            }
        }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) red[warp][lane * 4 + q] = acc[q];
    __syncthreads();
    if (warp != 0) return;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int64_t n = n0 + q;
        if (n >= N) continue;
        double t = red[0][lane * 4 + q];
        for (int w = 1; w < SP_WARPS; ++w) t += red[w][lane * 4 + q];
        ws[(int64_t)ck.slot * N + n] = t;
    }
}

// C[map(r), n] = sum of row r's chunk partials in chunk order, rounded once to fp32.
template <typename IT>
__global__ void sp_reduce_kernel(const int32_t* __restrict__ rows, const int32_t* __restrict__ first,
                                 int64_t nrows, const double* __restrict__ ws, float* __restrict__ C,
                                 const IT* __restrict__ row_map, int64_t M, int64_t N,
                                 unsigned* __restrict__ err) {
    const int64_t total = nrows * N;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t / N, n = t - i * N;
        const int64_t r = rows[i];
        if (r >= M) continue;
        double acc = 0.0;
        for (int s = first[i]; s < first[i + 1]; ++s) acc += ws[(int64_t)s * N + n];
        const int64_t orow = row_map ? (int64_t)row_map[r] : r;
        if (orow < 0 || orow >= M) {
            flag_error(err, DERR_PERM_OUT_OF_RANGE);
            continue;
        }
        C[orow * N + n] = (float)acc;
    }
}

unsigned sp_grid(Handle& h, int64_t warps_wanted) {
    const int64_t want = ceil_div(warps_wanted, 8);
    return (unsigned)std::max<int64_t>(1, std::min(want, (int64_t)sm_count(h.device) * 16));
}

}  // namespace

template <typename VT, typename IT>
void sparse_rows_build(Handle& h, int64_t nbr, int64_t M, const IT* rp, const IT* ci,
                       const VT* v, int64_t dense_nnz, SparseRows& out) {
    cudaStream_t s = h.stream;
    out = SparseRows();
    out.dense_br.assign(nbr, 1);
    if (nbr == 0 || M == 0) return;
    XS_REQUIRE(reinterpret_cast<uintptr_t>(v) % 16 == 0, XSPMM_STATUS_UNSUPPORTED,
               "block values not 16-byte aligned");
    XS_REQUIRE(M < (int64_t(1) << 31), XSPMM_STATUS_UNSUPPORTED, "too many rows");
    DevBuf<int32_t> d_cnt(M, s);
    sp_row_count_kernel<VT, IT><<<sp_grid(h, nbr), 256, 0, s>>>(rp, v, nbr, M, d_cnt.get());
    after_launch(h, "sparse_row_count");
    std::vector<int32_t> cnt(M);
    std::vector<IT> hrp(nbr + 1);
    XS_CHECK_CUDA(cudaMemcpyAsync(cnt.data(), d_cnt.get(), M * sizeof(int32_t),
                                  cudaMemcpyDeviceToHost, s));
    XS_CHECK_CUDA(cudaMemcpyAsync(hrp.data(), rp, (nbr + 1) * sizeof(IT), cudaMemcpyDeviceToHost, s));
    XS_CHECK_CUDA(cudaStreamSynchronize(s));
    out.host_rp.assign(hrp.begin(), hrp.end());
    // Block rows averaging at most dense_nnz nonzeros per block go to the gather kernels
    // (block rows with no block stay: the block kernels write their zeros); rptr is a prefix
    // over all rows, with empty ranges for the rows left on the block kernels.
    std::vector<int32_t> brs, short_ids, long_rows;
    std::vector<int64_t> rptr(M + 1, 0);
    for (int64_t br = 0; br < nbr; ++br) {
        const int64_t nb = (int64_t)hrp[br + 1] - (int64_t)hrp[br];
        const int64_t r0 = br * 16, r1 = std::min<int64_t>(M, r0 + 16);
        int64_t nz = 0;
        for (int64_t r = r0; r < r1; ++r) nz += cnt[r];
        const bool sparse = nb > 0 && nz <= dense_nnz * nb;
        out.dense_br[br] = sparse ? 0 : 1;
        if (sparse) {
            brs.push_back((int32_t)br);
            for (int64_t r = r0; r < r1; ++r)
                (cnt[r] > SP_LONG ? long_rows : short_ids).push_back((int32_t)r);
        }
        for (int64_t r = r0; r < r1; ++r) rptr[r + 1] = rptr[r] + (sparse ? cnt[r] : 0);
    }
    std::vector<SparseChunk> chunks;
    std::vector<int32_t> long_first;
    for (const int32_t r : long_rows) {
        long_first.push_back((int32_t)chunks.size());
        for (int64_t e = rptr[r]; e < rptr[r + 1]; e += SP_CHUNK)
            chunks.push_back(SparseChunk{e, std::min(e + SP_CHUNK, rptr[r + 1]), r,
                                         (int32_t)chunks.size()});
    }
    long_first.push_back((int32_t)chunks.size());
    out.nbrs = (int64_t)brs.size();
    out.nnz = rptr[M];
    std::vector<SpRow> short_rows(short_ids.size());
    for (size_t i = 0; i < short_ids.size(); ++i) {
        const int32_t r = short_ids[i];
        short_rows[i] = SpRow{rptr[r], r, (int32_t)(rptr[r + 1] - rptr[r])};
    }
    out.nshort = (int64_t)short_rows.size();
    out.nlong = (int64_t)long_rows.size();
    out.nchunks = (int64_t)chunks.size();
    if (out.nbrs == 0) return;
    out.rptr = DevBuf<int64_t>(M + 1, s);
    out.brs = DevBuf<int32_t>(brs.size(), s);
    out.short_rows = DevBuf<SpRow>(std::max<size_t>(short_rows.size(), 1), s);
    out.long_rows = DevBuf<int32_t>(std::max<size_t>(long_rows.size(), 1), s);
    out.col = DevBuf<int32_t>(std::max<int64_t>(out.nnz, 1), s);
    out.val = DevBuf<uint8_t>(std::max<int64_t>(out.nnz, 1) * sizeof(VT), s);
    XS_CHECK_CUDA(cudaMemcpyAsync(out.rptr.get(), rptr.data(), (M + 1) * sizeof(int64_t),
                                  cudaMemcpyHostToDevice, s));
    XS_CHECK_CUDA(cudaMemcpyAsync(out.brs.get(), brs.data(), brs.size() * sizeof(int32_t),
                                  cudaMemcpyHostToDevice, s));
    if (!short_rows.empty())
        XS_CHECK_CUDA(cudaMemcpyAsync(out.short_rows.get(), short_rows.data(),
                                      short_rows.size() * sizeof(SpRow), cudaMemcpyHostToDevice, s));
    if (!long_rows.empty()) {
        XS_CHECK_CUDA(cudaMemcpyAsync(out.long_rows.get(), long_rows.data(),
                                      long_rows.size() * sizeof(int32_t), cudaMemcpyHostToDevice, s));
        out.chunks = DevBuf<SparseChunk>(chunks.size(), s);
        out.long_first = DevBuf<int32_t>(long_first.size(), s);
        XS_CHECK_CUDA(cudaMemcpyAsync(out.chunks.get(), chunks.data(),
                                      chunks.size() * sizeof(SparseChunk), cudaMemcpyHostToDevice, s));
        XS_CHECK_CUDA(cudaMemcpyAsync(out.long_first.get(), long_first.data(),
                                      long_first.size() * sizeof(int32_t), cudaMemcpyHostToDevice, s));
    }
    sp_extract_kernel<VT, IT><<<sp_grid(h, out.nbrs), 256, 0, s>>>(
        rp, ci, v, out.brs.get(), out.nbrs, M, out.rptr.get(), out.col.get(),
        reinterpret_cast<VT*>(out.val.get()));
    after_launch(h, "sparse_extract");
    XS_CHECK_CUDA(cudaStreamSynchronize(s));  // the host vectors go out of scope
}

template <typename VT, typename IT>
void sparse_rows_execute(Handle& h, const SparseRows& sp, const VT* B, float* C, int64_t M,
                         int64_t K, int64_t N, const IT* map) {
    if (sp.nbrs == 0 || N == 0) return;
    const VT* val = reinterpret_cast<const VT*>(sp.val.get());
    const int64_t ntiles = ceil_div(N, SP_TN);
    XS_REQUIRE(ntiles <= 65535, XSPMM_STATUS_UNSUPPORTED, "N too large for the gather kernels");
    const bool vec = N % 4 == 0 && reinterpret_cast<uintptr_t>(B) % SpVT<VT>::b4_align == 0 &&
                     reinterpret_cast<uintptr_t>(C) % 16 == 0;
    if (sp.nshort > 0) {
        dim3 grid((unsigned)ceil_div(sp.nshort, SP_WARPS), (unsigned)ntiles);
        if (vec)
            sp_gather_short_kernel<VT, IT, true><<<grid, SP_WARPS * 32, 0, h.stream>>>(
                sp.short_rows.get(), sp.nshort, sp.col.get(), val, B, C, map, M, K, N,
                h.d_err);
        else
            sp_gather_short_kernel<VT, IT, false><<<grid, SP_WARPS * 32, 0, h.stream>>>(
                sp.short_rows.get(), sp.nshort, sp.col.get(), val, B, C, map, M, K, N,
                h.d_err);
        after_launch(h, "sparse_gather_short");
    }
    if (sp.nlong > 0) {
        DevBuf<double> ws((size_t)sp.nchunks * (size_t)N, h.stream);
        dim3 grid((unsigned)sp.nchunks, (unsigned)ntiles);
        XS_REQUIRE(sp.nchunks < (int64_t(1) << 31), XSPMM_STATUS_UNSUPPORTED, "too many chunks");
        if (vec)
            sp_gather_chunk_kernel<VT, true><<<grid, SP_WARPS * 32, 0, h.stream>>>(
                sp.chunks.get(), sp.col.get(), val, B, ws.get(), K, N);
        else
            sp_gather_chunk_kernel<VT, false><<<grid, SP_WARPS * 32, 0, h.stream>>>(
                sp.chunks.get(), sp.col.get(), val, B, ws.get(), K, N);
        after_launch(h, "sparse_gather_chunk");
        const int64_t total = sp.nlong * N;
        const unsigned rgrid = (unsigned)std::max<int64_t>(
            1, std::min(ceil_div(total, 256), (int64_t)sm_count(h.device) * 16));
        sp_reduce_kernel<IT><<<rgrid, 256, 0, h.stream>>>(sp.long_rows.get(), sp.long_first.get(),
                                                          sp.nlong, ws.get(), C, map, M, N,
                                                          h.d_err);
        after_launch(h, "sparse_reduce");
    }
}

#define XS_INST_SP(VT, IT)                                                                        \
    template void sparse_rows_build<VT, IT>(Handle&, int64_t, int64_t, const IT*, const IT*,      \
                                            const VT*, int64_t, SparseRows&);                     \
    template void sparse_rows_execute<VT, IT>(Handle&, const SparseRows&, const VT*, float*,      \
                                              int64_t, int64_t, int64_t, const IT*);
XS_INST_SP(__half, int32_t)
XS_INST_SP(__half, int64_t)
XS_INST_SP(float, int32_t)
XS_INST_SP(float, int64_t)

}  // namespace xspmm_b200
