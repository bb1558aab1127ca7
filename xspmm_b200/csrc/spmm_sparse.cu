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
// The result is the same sum, C[16br+i, n] = sum over the row's nonzeros a * B[col, n], added in
// column order. For 16-bit values every product is exact in fp32; a row of up to SP_PLAIN
// nonzeros is summed in fp32 (as the tensor-core kernels and the reference's WMMA accumulate), a
// longer one in fp32 groups of SP_UNROLL products whose sums are added in fp64, so that hub rows
// lose no accuracy to their large partial sums. fp32 values are multiplied and summed in fp64 and
// rounded once (as the fp32 SIMT block kernel does). A row of a split block row with no nonzero
// is written as zeros, as the block product writes it.
//
// Kernels. 16-bit values with N % 8 == 0 (the common case) take the tensor-core gather
// (sp_mma_kernel, below): 16 nonzeros at a time as one mma.sync per 8 columns. Otherwise the SIMT
// gather: a warp per task of consecutive short rows (up to SP_LONG nonzeros each) and 128-column
// tile (4 columns per lane); longer rows (hub rows) are cut into chunks of SP_CHUNK nonzeros, a
// CTA each, whose partials (each warp's share in column order, its SP_UNROLL-nonzero groups added
// in fp64, then the warps' sums in warp order) are added in fp64 afterwards. Both give results
// that do not depend on timing.
#include "ops.cuh"
#include "mma_sync.cuh"

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <type_traits>
#include <vector>

namespace xspmm_b200 {
namespace {

constexpr int SP_TN = 128;          // columns per warp (4 per lane)
constexpr int SP_WARPS = 8;
constexpr int64_t SP_LONG = 256;    // rows with more nonzeros are cut into chunks
constexpr int64_t SP_CHUNK = 2048;  // nonzeros per chunk of a long row
constexpr int SP_UNROLL = 8;        // B rows in flight per warp
constexpr int SP_TASK_NNZ = 128;    // nonzeros a warp task of several short rows may hold
// 16-bit values: rows of at most SP_PLAIN nonzeros are summed in fp32; in longer rows each group of
// SP_UNROLL products is summed in fp32 and the groups are added in fp64, so that a long row's
// rounding error stays at fp64 level relative to its partial sums.
constexpr int SP_PLAIN = 128;
constexpr int SP_CHUNK_MINB = 2;    // CTAs per SM the chunk kernel is compiled for

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
    using Acc = float;  // fp16 x fp16 products are exact in fp32; summed in fp32, column order
    using Raw = uint2;  // 4 consecutive elements of a B row, as loaded
    __device__ static Raw raw4(const __half* p) { return __ldg(reinterpret_cast<const uint2*>(p)); }
    __device__ static Raw zero4() { return make_uint2(0u, 0u); }
    __device__ static void f4(const Raw& x, float (&o)[4]) {
        const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&x.x));
        const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&x.y));
        o[0] = f0.x; o[1] = f0.y; o[2] = f1.x; o[3] = f1.y;
    }
};
template <> struct SpVT<__nv_bfloat16> {  // as fp16: same bits moved, bf16 -> fp32 conversions
    __device__ static void load8(const __nv_bfloat16* p, __nv_bfloat16 (&o)[8]) {
        const uint4 x = *reinterpret_cast<const uint4*>(p);
        *reinterpret_cast<uint4*>(o) = x;
    }
    __device__ static bool nz(__nv_bfloat16 x) {
        return (__bfloat16_as_ushort(x) & 0x7FFFu) != 0;
    }
    __device__ static float f(__nv_bfloat16 x) { return __bfloat162float(x); }
    static constexpr int b4_align = 8;
    using Acc = float;  // bf16 x bf16 products are exact in fp32 (8 + 8 significant bits)
    using Raw = uint2;
    __device__ static Raw raw4(const __nv_bfloat16* p) {
        return __ldg(reinterpret_cast<const uint2*>(p));
    }
    __device__ static Raw zero4() { return make_uint2(0u, 0u); }
    __device__ static void f4(const Raw& x, float (&o)[4]) {
        const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&x.x));
        const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&x.y));
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
    using Acc = double;  // fp32 products and sums in fp64, rounded once
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

// C[map(r), tile] for rows with at most SP_LONG nonzeros, a warp per (task, 128-column tile). A
// task is up to 32 consecutive short rows holding at most SP_TASK_NNZ nonzeros (or one row of up
// to SP_LONG). The warp walks the task's nonzeros as one stream, row after row: lane i holds row
// i's descriptor and the inclusive prefix of the counts, each lane finds the row of stream
// position base + lane by a 5-step search over that prefix and loads the (column, value) pair,
// and the warp keeps SP_UNROLL B rows in flight across row ends, so that rows of one to three
// nonzeros do not leave it waiting on a chain of loads per row. A row's nonzeros are still added
// in column order, in fp64, and its sum is rounded once to fp32 when the stream leaves the row;
// rows without nonzeros are written as zeros.
template <typename VT, typename IT, bool VEC, bool FLUSH>
__global__ void __launch_bounds__(SP_WARPS * 32, sizeof(VT) == 2 ? (FLUSH ? 3 : 4) : 2)
sp_gather_rows_kernel(const SpTask* __restrict__ tasks, int64_t ntasks,
                      const SpRow* __restrict__ rows, const int32_t* __restrict__ col,
                      const VT* __restrict__ val, const VT* __restrict__ B, float* __restrict__ C,
                      const IT* __restrict__ row_map, int64_t M, int64_t K, int64_t N,
                      unsigned* __restrict__ err) {
    const unsigned FULL = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    const int64_t t = (int64_t)blockIdx.x * SP_WARPS + (threadIdx.x >> 5);
    if (t >= ntasks) return;
    const SpTask tk = tasks[t];
    SpRow ri{0, -1, 0};
    if (lane < tk.nrows) ri = rows[tk.first + lane];
    // where the lane's row is stored (-1: no row, or a bad map entry)
    int64_t orow = -1;
    if (ri.row >= 0 && ri.row < M) {
        orow = row_map ? (int64_t)row_map[ri.row] : (int64_t)ri.row;
        if (orow < 0 || orow >= M) {
            flag_error(err, DERR_PERM_OUT_OF_RANGE);
            orow = -1;
        }
    }
    int incl = ri.cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(FULL, incl, o);
        if (lane >= o) incl += v;
    }
    const int total = __shfl_sync(FULL, incl, 31);
    const int64_t e_rel = ri.e0 - (int64_t)(incl - ri.cnt);  // stream position k -> k + e_rel
    const int64_t n0 = (int64_t)blockIdx.y * SP_TN + lane * 4;
    const bool full4 = VEC && n0 + 4 <= N;

    // A row's sum: products added into acc in column order; with FLUSH (tasks holding a row of
    // more than SP_PLAIN nonzeros, 16-bit values) each group of SP_UNROLL products is then moved
    // into the fp64 tot.
    using Acc = typename SpVT<VT>::Acc;
    constexpr bool flush = FLUSH && sizeof(Acc) == 4;
    auto store = [&](int j, const double (&tot)[4], const Acc (&acc)[4]) {  // j warp-uniform
        const int64_t o = __shfl_sync(FULL, orow, j);
        if (o < 0) return;
        float* dst = C + o * N + n0;
        float r[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) r[q] = flush ? (float)(tot[q] + (double)acc[q]) : (float)acc[q];
        if (full4) {
            *reinterpret_cast<float4*>(dst) = make_float4(r[0], r[1], r[2], r[3]);
        } else {
#pragma unroll
            for (int q = 0; q < 4; ++q)
                if (n0 + q < N) dst[q] = r[q];
        }
    };
    Acc acc[4] = {0, 0, 0, 0};
    double tot[4] = {0.0, 0.0, 0.0, 0.0};
    // rows without nonzeros
    {
        unsigned zm = __ballot_sync(FULL, ri.cnt == 0 && orow >= 0);
        while (zm) {
            const int j = __ffs(zm) - 1;
            zm &= zm - 1;
            store(j, tot, acc);
        }
    }
    int cur = -1;  // the row being summed
    for (int base = 0; base < total; base += 32) {
        const int cnt = min(32, total - base);
        const int k = base + lane;
        int j = 0;  // the row of stream position k: the number of rows whose prefix is <= k
#pragma unroll
        for (int step = 16; step >= 1; step >>= 1) {
            if (__shfl_sync(FULL, incl, j + step - 1) <= k) j += step;
        }
        const int64_t rel = __shfl_sync(FULL, e_rel, j);
        int my_c = 0;
        float my_a = 0.0f;
        if (lane < cnt) {
            my_c = col[rel + k];
            my_a = SpVT<VT>::f(val[rel + k]);
        }
        for (int u0 = 0; u0 < cnt; u0 += SP_UNROLL) {
            typename SpVT<VT>::Raw raw[SP_UNROLL];
            float a[SP_UNROLL];
            int ju[SP_UNROLL];
            bool lv[SP_UNROLL];
#pragma unroll
            for (int u = 0; u < SP_UNROLL; ++u) {
                const int src_lane = (u0 + u) & 31;
                const int64_t c = __shfl_sync(FULL, my_c, src_lane);
                a[u] = __shfl_sync(FULL, my_a, src_lane);
                ju[u] = __shfl_sync(FULL, j, src_lane);
                lv[u] = u0 + u < cnt && c < K;
                raw[u] = (full4 && lv[u]) ? SpVT<VT>::raw4(B + c * N + n0) : SpVT<VT>::zero4();
            }
#pragma unroll
            for (int u = 0; u < SP_UNROLL; ++u) {
                if (u0 + u < cnt) {
                    if (ju[u] != cur) {
                        if (cur >= 0) store(cur, tot, acc);
                        cur = ju[u];
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            acc[q] = 0;
                            tot[q] = 0.0;
                        }
                    }
                    float bb[4];
                    if (VEC) {  // N % 4 == 0: a lane's 4 columns are all inside N or all past it
                        SpVT<VT>::f4(raw[u], bb);
                    } else {
                        const int64_t c = __shfl_sync(FULL, my_c, (u0 + u) & 31);
                        const VT* src = B + c * N + n0;
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            bb[q] = (lv[u] && n0 + q < N) ? SpVT<VT>::f(src[q]) : 0.0f;
                    }
#pragma unroll
                    for (int q = 0; q < 4; ++q) acc[q] = fma((Acc)a[u], (Acc)bb[q], acc[q]);
                }
            }
            if (flush) {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    tot[q] += (double)acc[q];
                    acc[q] = 0;
                }
            }
        }
    }
    if (cur >= 0) store(cur, tot, acc);
}

// Rows with more than SP_LONG nonzeros are cut into chunks of at most SP_CHUNK nonzeros: a CTA
// per (chunk, tile), warp w summing its contiguous eighth of the chunk, the 8 warp sums added in
// warp order into the chunk's fp64 partial; then sp_reduce_kernel adds a row's chunk partials in
// chunk order and rounds once. (One CTA per hub row of ~40K nonzeros set the time of the whole
// product.)
template <typename VT, bool VEC>
__global__ void __launch_bounds__(SP_WARPS * 32, SP_CHUNK_MINB)
sp_gather_chunk_kernel(const SparseChunk* __restrict__ chunks, const int32_t* __restrict__ col,
                       const VT* __restrict__ val, const VT* __restrict__ B,
                       double* __restrict__ ws, int64_t K, int64_t N) {
    __shared__ double red[SP_WARPS][SP_TN];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const SparseChunk ck = chunks[blockIdx.x];
    const int64_t n0 = (int64_t)blockIdx.y * SP_TN + lane * 4;
    const int64_t len = ck.e1 - ck.e0, per = (len + SP_WARPS - 1) / SP_WARPS;
    const int64_t w0 = ck.e0 + min(len, per * warp), w1 = ck.e0 + min(len, per * (warp + 1));
    using Acc = typename SpVT<VT>::Acc;
    Acc acc[4] = {0, 0, 0, 0};
    double tot[4] = {0.0, 0.0, 0.0, 0.0};  // fp64 sum of the SP_UNROLL-nonzero groups
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
                    for (int q = 0; q < 4; ++q) acc[q] = fma((Acc)a[u], (Acc)bb[q], acc[q]);
                }
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                tot[q] += (double)acc[q];
                acc[q] = 0;
            }
        }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) red[warp][lane * 4 + q] = tot[q];
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

// C[map(r), n] = sum of row r's chunk partials, rounded once to fp32. The partials are added in
// fp64 in four interleaved running sums (slots s = 0, 1, 2, 3 mod 4, each in chunk order), then
// (s0 + s1) + (s2 + s3): the loads of a hub row's tens of partials overlap instead of forming one
// chain, and the order stays fixed.
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
        double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
        const int s1 = first[i + 1];
        int s = first[i];
        for (; s + 4 <= s1; s += 4) {
            a0 += ws[(int64_t)s * N + n];
            a1 += ws[(int64_t)(s + 1) * N + n];
            a2 += ws[(int64_t)(s + 2) * N + n];
            a3 += ws[(int64_t)(s + 3) * N + n];
        }
        if (s < s1) a0 += ws[(int64_t)s * N + n];
        if (s + 1 < s1) a1 += ws[(int64_t)(s + 1) * N + n];
        if (s + 2 < s1) a2 += ws[(int64_t)(s + 2) * N + n];
        const double acc = (a0 + a1) + (a2 + a3);
        const int64_t orow = row_map ? (int64_t)row_map[r] : r;
        if (orow < 0 || orow >= M) {
            flag_error(err, DERR_PERM_OUT_OF_RANGE);
            continue;
        }
        C[orow * N + n] = (float)acc;
    }
}

// ---- tensor-core gather (16-bit values) ------------------------------------------------------
// The SIMT kernels above spend ~48 warp instructions per nonzero (shuffles, conversions, FMAs per
// column). Here a warp takes a task of up to SPM_TASK_KS k-steps, each k-step 16 consecutive
// positions of the task's nonzero stream, and multiplies them on the tensor core as one
// mma.sync m16n8k16 per 8 columns: A (16 x 16) holds position k's value in row (its row offset
// in the block row) and column k, zeros elsewhere; B (16 x 8) holds the 16 gathered B rows.
// Sixteen times the useful multiplies, but the tensor pipe has them to spare, and the warp issues
// a few instructions per nonzero instead of ~48. The stream comes pre-arranged in 128-byte k-step
// records (built once per plan): the 16 columns, then per pair of positions their two values and
// their two one-hot rows, from which each A fragment register takes 4 ALU operations. B rows are
// staged by 16-byte cp.async in an SPM_STAGES-deep per-warp ring of 16 x TN slabs (chunks
// XOR-swizzled by k & 7, so that ldmatrix.trans reads them without bank conflicts); the records
// stream into a ring of their own by cp.async, a k-step's record landing one iteration before
// the copies that read its columns are issued. A block-row task holds the rows of one block row
// up to SPM_ROW_MAX nonzeros each; longer rows are cut into SPM_CHUNK-nonzero chunks whose fp32
// partials are added in fp64 by sp_reduce_kernel.
// Columns per warp: 64. With the grouped flush a thread holds two sets of sums per 8 columns
// (118 registers at 64 columns, 12 warps per SM); 32 columns per warp (74 registers, 24 warps)
// measured slower on cfg5 (0.78 against 0.67 ms), the per-k-step work being paid per 32 columns.
constexpr int SPM_TN = 64;
constexpr int SPM_STAGES = 4;       // B slabs in flight per warp (a power of two)
constexpr int SPM_WARPS = 4;        // warps per CTA (independent; no CTA barrier)
constexpr int SPM_TASK_KS = 32;     // k-steps a block-row task may hold
constexpr int64_t SPM_ROW_MAX = 256;  // rows with more nonzeros are cut into chunks
constexpr int64_t SPM_CHUNK = 512;  // nonzeros per chunk (32 k-steps)
constexpr int SPM_GROUP = 8;        // k-steps per tensor-core accumulation group
constexpr int SPM_MRING = 2 * SPM_STAGES;  // k-step records in flight per warp (128 B each)
constexpr int SPM_RANGES_PER_SM = 16;  // warp ranges of tasks per SM (per 64-column tile)
// Accumulation: the products of SPM_GROUP k-steps accumulate in the tensor core from zero and
// each group's result is added to fp32 running sums with round-to-nearest adds, as the block
// kernels do every 8 blocks. Without it (one accumulation per task) the ragged-rows test reached
// a guarded error of 1.2-2e-3 even with every chain cut to 8 k-steps; with it, below 1e-3.
static_assert(SPM_TASK_KS * 16 >= 2 * SPM_ROW_MAX, "a block-row task must hold any of its rows");

// Fills the k-step records of every task, a warp per task: lane i (< 16) holds row i of the
// block row (or lane 0 the chunk), each lane finds the row of stream position p by a 4-step
// search over the inclusive prefix of the counts, and padding positions get column -1, value 0.
template <typename VT>
__global__ void sp_kstep_fill_kernel(const SpMmaTask* __restrict__ tasks, int64_t ntasks,
                                     const int64_t* __restrict__ rptr,
                                     const int32_t* __restrict__ col, const VT* __restrict__ val,
                                     SpKStep* __restrict__ ks) {
    const unsigned FULL = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < ntasks;
         t += warps) {
        const SpMmaTask tk = tasks[t];
        int cnt = 0;
        int64_t e0 = 0;
        if (tk.out >= 0) {
            if (lane < 16 && ((tk.mask >> lane) & 1u)) {
                const int64_t r = (int64_t)tk.out * 16 + lane;
                e0 = rptr[r];
                cnt = (int)(rptr[r + 1] - e0);
            }
        } else if (lane == 0) {
            e0 = tk.e0;
            cnt = tk.nnz;
        }
        int incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(FULL, incl, o);
            if (lane >= o) incl += v;
        }
        const int total = __shfl_sync(FULL, incl, 31);
        const int64_t erel = e0 - (int64_t)(incl - cnt);  // position p of this lane's row -> p + erel
        const int npos = tk.nks * 16;
        SpKStep* rec = ks + tk.ks0;
        for (int p0 = 0; p0 < npos; p0 += 32) {
            const int p = p0 + lane;
            int j = 0;  // the row of position p: the number of rows whose prefix is <= p
#pragma unroll
            for (int step = 8; step >= 1; step >>= 1)
                if (__shfl_sync(FULL, incl, j + step - 1) <= p) j += step;
            const int64_t er = __shfl_sync(FULL, erel, j);
            int32_t c = -1;
            uint32_t vb = 0u, oh = 0u;  // value bits, one-hot row
            if (p < total) {
                c = col[er + p];
                vb = (uint32_t)(*reinterpret_cast<const uint16_t*>(val + er + p));
                oh = 1u << j;
            }
            const uint32_t vb1 = __shfl_down_sync(FULL, vb, 1);  // position p + 1 (p even)
            const uint32_t oh1 = __shfl_down_sync(FULL, oh, 1);
            if (p < npos) {
                rec[p >> 4].col[p & 15] = c;
                if ((p & 1) == 0) {
                    rec[p >> 4].pair[(p & 15)] = vb | (vb1 << 16);
                    rec[p >> 4].pair[(p & 15) + 1] = oh | (oh1 << 16);
                }
            }
        }
    }
}

__device__ __forceinline__ void cp_async16_sa(uint32_t dst, uint64_t src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src),
                 "r"(src_bytes));
}
__device__ __forceinline__ int4 lds128(uint32_t a) {
    int4 v;
    asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(a)
                 : "memory");
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0,%1}, [%2];\n" : "=r"(v.x), "=r"(v.y) : "r"(a) : "memory");
    return v;
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t a) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(a)
                 : "memory");
}
// The A fragment register of positions 2p, 2p+1 for C row `row`: the pair's value bits where its
// one-hot row word has bit `row` (low half) or bit `row` + 16 (high half), zeros elsewhere.
__device__ __forceinline__ uint32_t spm_afrag(uint2 w, int row) {
    return w.x & (((w.y >> row) & 0x00010001u) * 0xFFFFu);
}

// Slab geometry for TN columns per warp (64 or 128): CH 16-byte chunks per slab row, each lane
// copying RPL rows of one chunk; NT n8 tiles.
template <int TN>
struct SpmGeom {
    static constexpr int CH = TN / 8;
    static constexpr int RPL = 16 * CH / 32;
    static constexpr int ROWB = TN * 2;
    static constexpr int SLAB = 16 * ROWB;
    static constexpr int NT = TN / 8;
    static constexpr int WSMEM = SPM_STAGES * SLAB + SPM_MRING * 128;
    static constexpr int MINB = TN == 32 ? 4 : TN == 64 ? 4 : 2;  // CTAs of SPM_WARPS per SM
    // 16-byte chunk c of slab row k is stored at chunk c ^ swz(k): the 8 rows an ldmatrix matrix
    // reads then fall on 8 different 16-byte bank groups (rows of 128 bytes or more: k & 7; rows
    // of 64 bytes, two per 128-byte line: (k >> 1) & 3)
    __device__ static int swz(int k) { return TN >= 64 ? (k & 7) : ((k >> 1) & 3); }
};

// A warp job = (range of consecutive tasks, 64-column tile). The tasks' k-step records are
// consecutive, so the warp streams the range's k-steps through one ring: copies run SPM_STAGES
// k-steps ahead across task boundaries, and at a task's last k-step its sums are stored (and
// the next task starts from zero), instead of every task paying the ring's fill latency.
template <bool BF16, typename IT, int TN>
__global__ void __launch_bounds__(SPM_WARPS * 32, SpmGeom<TN>::MINB)
sp_mma_kernel(const SpMmaTask* __restrict__ tasks, const int32_t* __restrict__ ranges,
              int64_t nranges, int ntn, const SpKStep* __restrict__ ks,
              const __half* __restrict__ B, float* __restrict__ C, double* __restrict__ ws,
              const IT* __restrict__ row_map, int64_t M, int64_t K, int64_t N,
              unsigned* __restrict__ err) {
    using namespace warpmma;
    using G = SpmGeom<TN>;
    extern __shared__ __align__(128) uint8_t spm_smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t job = (int64_t)blockIdx.x * SPM_WARPS + warp;
    if (job >= nranges * ntn) return;  // warp-uniform; the warps of a CTA never wait on one another
    const int64_t rg = job / ntn;
    const int64_t n0 = (int64_t)(job % ntn) * TN;
    const int t0 = ranges[rg], t1 = ranges[rg + 1];
    const uint32_t slab0 = smem_u32(spm_smem + warp * G::WSMEM);
    const uint32_t ring0 = slab0 + SPM_STAGES * G::SLAB;  // SPM_MRING k-step records
    // the range's k-steps: [q0, q0 + nq)
    const SpMmaTask tfirst = tasks[t0];
    const SpMmaTask tlast = tasks[t1 - 1];
    const int64_t q0 = tfirst.ks0;
    const int nq = (int)(tlast.ks0 + tlast.nks - q0);
    const uint64_t rec = reinterpret_cast<uint64_t>(ks + q0);
    // copies: lane l takes the 16-byte chunk l % CH (8 columns) of slab rows kr .. kr + RPL - 1
    const int ch = lane % G::CH, kr = (lane / G::CH) * G::RPL;
    const uint32_t klim = (n0 + ch * 8 < N) ? (uint32_t)K : 0u;  // column c copied iff c < klim
    const uint64_t bl = reinterpret_cast<uint64_t>(B) + (uint64_t)(n0 + ch * 8) * 2u;
    const uint32_t rowb = (uint32_t)N * 2u;
    uint32_t doff[G::RPL];
#pragma unroll
    for (int i = 0; i < G::RPL; ++i) {
        const int k = kr + i;
        doff[i] = (uint32_t)(k * G::ROWB + ((ch ^ G::swz(k)) << 4));
    }
    // ldmatrix: lane l addresses row (mi & 1) * 8 + mr of matrix mi = l >> 3; matrices 0/1 are
    // n8 tile 2jp (k rows 0-7 / 8-15), 2/3 are n8 tile 2jp + 1
    const int mi = lane >> 3, mr = lane & 7, kk = (mi & 1) * 8 + mr;
    uint32_t loff[G::NT / 2];
#pragma unroll
    for (int jp = 0; jp < G::NT / 2; ++jp)
        loff[jp] = (uint32_t)(kk * G::ROWB + (((2 * jp + (mi >> 1)) ^ G::swz(kk)) << 4));
    const int g = lane >> 2, tq = lane & 3;
    // record q into its ring slot (lanes 0-7, 16 bytes each)
    const uint64_t rec_l = rec + lane * 16;
    const uint32_t ring_l = ring0 + lane * 16;
    auto meta_copy = [&](int q) {
        if (lane < 8 && q < nq)
            cp_async16_sa(ring_l + (uint32_t)(q & (SPM_MRING - 1)) * 128u, rec_l + (uint64_t)q * 128u,
                          16);
    };
    // k-step q's B rows, their columns read from the record in the ring; a column outside
    // [0, klim) copies nothing and zero-fills (the source given is B's first row, a valid address)
    const uint32_t ring_c = ring0 + kr * 4;
    auto issue = [&](int q) {
        if (q < nq) {
            const uint32_t st = slab0 + (uint32_t)(q & (SPM_STAGES - 1)) * G::SLAB;
            uint32_t c[G::RPL];
            const uint32_t ca = ring_c + (uint32_t)(q & (SPM_MRING - 1)) * 128u;
            if constexpr (G::RPL == 2) {
                const uint2 c2 = lds64(ca);
                c[0] = c2.x;
                c[1] = c2.y;
            } else {
#pragma unroll
                for (int i = 0; i < G::RPL; i += 4) {
                    const int4 c4 = lds128(ca + i * 4);
                    c[i] = (uint32_t)c4.x;
                    c[i + 1] = (uint32_t)c4.y;
                    c[i + 2] = (uint32_t)c4.z;
                    c[i + 3] = (uint32_t)c4.w;
                }
            }
#pragma unroll
            for (int i = 0; i < G::RPL; ++i) {
                const bool ok = c[i] < klim;
                cp_async16_sa(st + doff[i], bl + (uint64_t)(ok ? c[i] : 0u) * rowb, ok ? 16 : 0);
            }
        }
    };
    // Each group of SPM_GROUP k-steps of a task accumulates in the tensor core from zero (acc);
    // the group sums are added to sum with round-to-nearest fp32 adds.
    float acc[G::NT][4], sum[G::NT][4];
#pragma unroll
    for (int j = 0; j < G::NT; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) sum[j][q] = 0.0f;
    // the task being summed: its descriptor, its k-steps [cst, cend) in range positions
    int cur = t0;
    SpMmaTask tk = tfirst;
    int cst = (int)(tk.ks0 - q0), cend = cst + tk.nks;
    // stores task tk's sums (zeros if it has no k-step) and clears them
    auto finish = [&]() {
        if (tk.out >= 0) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int i = g + 8 * h;
                if (!((tk.mask >> i) & 1u)) continue;
                const int64_t r = (int64_t)tk.out * 16 + i;
                if (r >= M) continue;
                const int64_t o = row_map ? (int64_t)row_map[r] : r;
                if (o < 0 || o >= M) {
                    flag_error(err, DERR_PERM_OUT_OF_RANGE);
                    continue;
                }
                float* dst = C + o * N + n0;
#pragma unroll
                for (int j = 0; j < G::NT; ++j) {
                    const int n = j * 8 + 2 * tq;
                    if (n0 + n < N)
                        *reinterpret_cast<float2*>(dst + n) =
                            make_float2(sum[j][2 * h], sum[j][2 * h + 1]);
                }
            }
        } else if (g == 0) {  // a chunk: row 0 holds its partial
            double* dst = ws + (int64_t)(-(tk.out + 1)) * N + n0;
#pragma unroll
            for (int j = 0; j < G::NT; ++j) {
                const int n = j * 8 + 2 * tq;
                if (n0 + n < N) {
                    dst[n] = (double)sum[j][0];
                    dst[n + 1] = (double)sum[j][1];
                }
            }
        }
#pragma unroll
        for (int j = 0; j < G::NT; ++j)
#pragma unroll
            for (int q = 0; q < 4; ++q) sum[j][q] = 0.0f;
    };
    // moves on to the next task of the range (cur + 1 < t1)
    auto next_task = [&]() {
        ++cur;
        tk = tasks[cur];
        cst = (int)(tk.ks0 - q0);
        cend = cst + tk.nks;
    };
    // Group order: the records of k-steps 0 .. SPM_STAGES-1 first (waited for), then group g
    // holds k-step g's B rows and k-step (g + SPM_STAGES)'s record, so a record has landed one
    // iteration before the copies that read its columns are issued.
#pragma unroll
    for (int q = 0; q < SPM_STAGES; ++q) meta_copy(q);
    cp_async_commit();
    cp_async_wait<0>();
    __syncwarp();
#pragma unroll
    for (int q = 0; q < SPM_STAGES - 1; ++q) {
        issue(q);
        meta_copy(q + SPM_STAGES);
        cp_async_commit();
    }
    for (int s = 0; s < nq; ++s) {
        // tasks that ended before k-step s are stored now (their stores overlap this step's wait)
        while (cend <= s && cur + 1 < t1) {
            finish();
            next_task();
        }
        issue(s + SPM_STAGES - 1);
        meta_copy(s + 2 * SPM_STAGES - 1);
        cp_async_commit();
        cp_async_wait<SPM_STAGES - 1>();
        __syncwarp();
        const uint32_t rs = ring0 + (uint32_t)(s & (SPM_MRING - 1)) * 128u + 64u;
        const uint2 w0 = lds64(rs + 8 * tq), w1 = lds64(rs + 8 * (tq + 4));
        uint32_t a[4];
        a[0] = spm_afrag(w0, g);
        a[1] = spm_afrag(w0, g + 8);
        a[2] = spm_afrag(w1, g);
        a[3] = spm_afrag(w1, g + 8);
        const uint32_t st = slab0 + (uint32_t)(s & (SPM_STAGES - 1)) * G::SLAB;
        const int ts = s - cst;  // k-step within the task
        if ((ts & (SPM_GROUP - 1)) == 0) {
#pragma unroll
            for (int jp = 0; jp < G::NT / 2; ++jp) {
                uint32_t b[4];
                ldsm_x4_trans(b, st + loff[jp]);
                mma_16816_first<BF16>(acc[2 * jp], a, b[0], b[1]);
                mma_16816_first<BF16>(acc[2 * jp + 1], a, b[2], b[3]);
            }
        } else {
#pragma unroll
            for (int jp = 0; jp < G::NT / 2; ++jp) {
                uint32_t b[4];
                ldsm_x4_trans(b, st + loff[jp]);
                mma_16816<BF16>(acc[2 * jp], a, b[0], b[1]);
                mma_16816<BF16>(acc[2 * jp + 1], a, b[2], b[3]);
            }
        }
        if ((ts & (SPM_GROUP - 1)) == SPM_GROUP - 1 || s == cend - 1) {
#pragma unroll
            for (int j = 0; j < G::NT; ++j)
#pragma unroll
                for (int q2 = 0; q2 < 4; ++q2) sum[j][q2] = __fadd_rn(sum[j][q2], acc[j][q2]);
        }
        __syncwarp();  // every lane is done with this slot before it is refilled
    }
    cp_async_wait<0>();
    // the range's last task, and any after it without k-steps
    finish();
    while (cur + 1 < t1) {
        next_task();
        finish();
    }
}

// XSPMM_GATHER_KERNEL = simt keeps 16-bit products on the SIMT gather kernels (comparisons);
// read once per process.
enum class GatherKernel { Auto, Simt };
GatherKernel gather_kernel_choice() {
    static const GatherKernel k = [] {
        const char* e = std::getenv("XSPMM_GATHER_KERNEL");
        return (e && std::strcmp(e, "simt") == 0) ? GatherKernel::Simt : GatherKernel::Auto;
    }();
    return k;
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
    // Block rows averaging at most dense_nnz nonzeros per block, and block rows without blocks,
    // go to the gather kernels; rptr is a prefix over all rows, with empty ranges for the rows
    // left on the block kernels.
    std::vector<int32_t> brs, short_ids, long_rows;
    std::vector<int64_t> rptr(M + 1, 0);
    for (int64_t br = 0; br < nbr; ++br) {
        const int64_t nb = (int64_t)hrp[br + 1] - (int64_t)hrp[br];
        const int64_t r0 = br * 16, r1 = std::min<int64_t>(M, r0 + 16);
        int64_t nz = 0;
        for (int64_t r = r0; r < r1; ++r) nz += cnt[r];
        // (a block row without blocks is sparse too: its rows are written as zeros by the gather
        // kernels, alongside the other tasks, instead of by a launch of the block kernel)
        const bool sparse = nz <= dense_nnz * nb;
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
    // warp tasks: consecutive short rows, at most 32 of them and SP_TASK_NNZ nonzeros (a row
    // with more nonzeros is a task of its own)
    // with a 16-bit value type, tasks of rows above SP_PLAIN nonzeros (the fp64-flush kernel) are
    // kept apart from the others and listed after them
    const bool two_kinds = sizeof(VT) == 2;
    auto heavy = [&](size_t i) { return two_kinds && short_rows[i].cnt > SP_PLAIN; };
    std::vector<SpTask> tasks, heavy_tasks;
    for (size_t i = 0; i < short_rows.size();) {
        SpTask tk{(int32_t)i, 0};
        const bool hv = heavy(i);
        int64_t nz = 0;
        while (i < short_rows.size() && tk.nrows < 32 && heavy(i) == hv &&
               (tk.nrows == 0 || nz + short_rows[i].cnt <= SP_TASK_NNZ)) {
            nz += short_rows[i].cnt;
            ++tk.nrows;
            ++i;
        }
        (hv ? heavy_tasks : tasks).push_back(tk);
    }
    out.nplain_tasks = (int64_t)tasks.size();
    tasks.insert(tasks.end(), heavy_tasks.begin(), heavy_tasks.end());
    out.nshort = (int64_t)short_rows.size();
    out.ntasks = (int64_t)tasks.size();
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
    out.tasks = DevBuf<SpTask>(std::max<size_t>(tasks.size(), 1), s);
    if (!short_rows.empty()) {
        XS_CHECK_CUDA(cudaMemcpyAsync(out.short_rows.get(), short_rows.data(),
                                      short_rows.size() * sizeof(SpRow), cudaMemcpyHostToDevice, s));
        XS_CHECK_CUDA(cudaMemcpyAsync(out.tasks.get(), tasks.data(), tasks.size() * sizeof(SpTask),
                                      cudaMemcpyHostToDevice, s));
    }
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
    if constexpr (sizeof(VT) == 2) {
        // Tensor-core gather tasks: the rows of the sparse block rows above SPM_ROW_MAX nonzeros
        // cut into chunks of SPM_CHUNK, then, per sparse block row, its other rows packed in
        // order into tasks of at most SPM_TASK_KS k-steps.
        std::vector<SpMmaTask> mt;
        std::vector<int32_t> mfirst, mlong;
        for (const int32_t br : brs) {
            const int64_t r0 = (int64_t)br * 16, r1 = std::min<int64_t>(M, r0 + 16);
            for (int64_t r = r0; r < r1; ++r)
                if (cnt[r] > SPM_ROW_MAX) mlong.push_back((int32_t)r);
        }
        int64_t nks = 0, slots = 0;
        for (const int32_t r : mlong) {
            mfirst.push_back((int32_t)slots);
            for (int64_t e = rptr[r]; e < rptr[r + 1]; e += SPM_CHUNK) {
                const int64_t n = std::min<int64_t>(SPM_CHUNK, rptr[r + 1] - e);
                const int32_t k = (int32_t)((n + 15) / 16);
                mt.push_back(SpMmaTask{nks, e, k, (int32_t)(-(slots + 1)), 0u, (int32_t)n});
                nks += k;
                ++slots;
            }
        }
        mfirst.push_back((int32_t)slots);
        for (const int32_t br : brs) {
            const int64_t r0 = (int64_t)br * 16, r1 = std::min<int64_t>(M, r0 + 16);
            uint32_t mask = 0;
            int64_t pos = 0;
            auto emit = [&]() {
                const int32_t k = (int32_t)((pos + 15) / 16);
                mt.push_back(SpMmaTask{nks, 0, k, br, mask, 0});
                nks += k;
                mask = 0;
                pos = 0;
            };
            for (int64_t r = r0; r < r1; ++r) {
                if (cnt[r] > SPM_ROW_MAX) continue;
                if (mask != 0 && (pos + cnt[r] + 15) / 16 > SPM_TASK_KS) emit();
                mask |= 1u << (r - r0);
                pos += cnt[r];
            }
            if (mask != 0) emit();
        }
        XS_REQUIRE(slots < (int64_t(1) << 31) - 1, XSPMM_STATUS_UNSUPPORTED, "too many chunks");
        out.nksteps = nks;
        out.nmtasks = (int64_t)mt.size();
        out.nmslots = slots;
        out.nmlong = (int64_t)mlong.size();
        if (!mt.empty()) {
            out.mtasks = DevBuf<SpMmaTask>(mt.size(), s);
            out.ksteps = DevBuf<SpKStep>(std::max<int64_t>(nks, 1), s);
            out.mlong_first = DevBuf<int32_t>(mfirst.size(), s);
            out.mlong_rows = DevBuf<int32_t>(std::max<size_t>(mlong.size(), 1), s);
            if (!mlong.empty())
                XS_CHECK_CUDA(cudaMemcpyAsync(out.mlong_rows.get(), mlong.data(),
                                              mlong.size() * sizeof(int32_t), cudaMemcpyHostToDevice,
                                              s));
            XS_CHECK_CUDA(cudaMemcpyAsync(out.mtasks.get(), mt.data(), mt.size() * sizeof(SpMmaTask),
                                          cudaMemcpyHostToDevice, s));
            XS_CHECK_CUDA(cudaMemcpyAsync(out.mlong_first.get(), mfirst.data(),
                                          mfirst.size() * sizeof(int32_t), cudaMemcpyHostToDevice, s));
            // Warp ranges: consecutive tasks of about equal work (k-steps, plus two for a task's
            // start and store), SPM_RANGES_PER_SM per SM; a warp streams its range's k-steps
            // through one ring, so a task's first loads overlap the previous task's last steps.
            const int64_t nr = std::max<int64_t>(
                1, std::min<int64_t>((int64_t)mt.size(), (int64_t)sm_count(h.device) * SPM_RANGES_PER_SM));
            int64_t total = 0;
            for (const SpMmaTask& t : mt) total += t.nks + 2;
            std::vector<int32_t> rb(1, 0);
            int64_t acc = 0;
            for (size_t i = 0; i < mt.size(); ++i) {
                acc += mt[i].nks + 2;
                if ((int64_t)rb.size() < nr && acc * nr >= total * (int64_t)rb.size())
                    rb.push_back((int32_t)(i + 1));
            }
            if (rb.back() != (int32_t)mt.size()) rb.push_back((int32_t)mt.size());
            out.nmranges = (int64_t)rb.size() - 1;
            out.mranges = DevBuf<int32_t>(rb.size(), s);
            XS_CHECK_CUDA(cudaMemcpyAsync(out.mranges.get(), rb.data(), rb.size() * sizeof(int32_t),
                                          cudaMemcpyHostToDevice, s));
            sp_kstep_fill_kernel<VT><<<sp_grid(h, out.nmtasks), 256, 0, s>>>(
                out.mtasks.get(), out.nmtasks, out.rptr.get(), out.col.get(),
                reinterpret_cast<const VT*>(out.val.get()), out.ksteps.get());
            after_launch(h, "sparse_kstep_fill");
            out.mma_built = true;
        }
        XS_CHECK_CUDA(cudaStreamSynchronize(s));  // the host vectors go out of scope
    } else {
        XS_CHECK_CUDA(cudaStreamSynchronize(s));  // the host vectors go out of scope
    }
}

template <typename VT, typename IT>
void sparse_rows_execute(Handle& h, const SparseRows& sp, const VT* B, float* C, int64_t M,
                         int64_t K, int64_t N, const IT* map) {
    if (sp.nbrs == 0 || N == 0) return;
    const VT* val = reinterpret_cast<const VT*>(sp.val.get());
    const int64_t ntiles = ceil_div(N, SP_TN);
    XS_REQUIRE(ntiles <= 65535, XSPMM_STATUS_UNSUPPORTED, "N too large for the gather kernels");
    if constexpr (sizeof(VT) == 2) {
        // tensor-core gather: 16-byte copies of B rows need N % 8 == 0 and an aligned B
        if (sp.mma_built && gather_kernel_choice() != GatherKernel::Simt && N % 8 == 0 &&
            reinterpret_cast<uintptr_t>(B) % 16 == 0 && reinterpret_cast<uintptr_t>(C) % 8 == 0) {
            constexpr bool BF = std::is_same<VT, __nv_bfloat16>::value;
            DevBuf<double> ws((size_t)std::max<int64_t>(sp.nmslots, 1) * (size_t)N, h.stream);
            auto launch = [&](auto tn_const) {
                constexpr int TN = decltype(tn_const)::value;
                const int ntn = (int)ceil_div(N, TN);
                const int64_t blocks = ceil_div(sp.nmranges * ntn, SPM_WARPS);
                XS_REQUIRE(blocks < (int64_t(1) << 31), XSPMM_STATUS_UNSUPPORTED,
                           "too many tasks for the tensor-core gather");
                const int smem = SPM_WARPS * SpmGeom<TN>::WSMEM;
                // the shared-memory limit is a per-device attribute: set once per device (devices
                // past 63 every time; a repeated set is harmless)
                static std::atomic<uint64_t> attr_set{0};
                auto kern = sp_mma_kernel<BF, IT, TN>;
                const uint64_t bit = h.device < 64 ? (uint64_t(1) << h.device) : 0;
                if (bit == 0 || !(attr_set.load(std::memory_order_relaxed) & bit)) {
                    XS_CHECK_CUDA(cudaFuncSetAttribute(
                        kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
                    attr_set.fetch_or(bit, std::memory_order_relaxed);
                }
                kern<<<(unsigned)blocks, SPM_WARPS * 32, smem, h.stream>>>(
                    sp.mtasks.get(), sp.mranges.get(), sp.nmranges, ntn, sp.ksteps.get(),
                    reinterpret_cast<const __half*>(B), C, ws.get(), map, M, K, N, h.d_err);
            };
            launch(std::integral_constant<int, SPM_TN>());
            after_launch(h, "sparse_mma");
            if (sp.nmlong > 0) {
                const int64_t total = sp.nmlong * N;
                const unsigned rgrid = (unsigned)std::max<int64_t>(
                    1, std::min(ceil_div(total, 256), (int64_t)sm_count(h.device) * 16));
                sp_reduce_kernel<IT><<<rgrid, 256, 0, h.stream>>>(
                    sp.mlong_rows.get(), sp.mlong_first.get(), sp.nmlong, ws.get(), C, map, M, N,
                    h.d_err);
                after_launch(h, "sparse_reduce");
            }
            return;
        }
    }
    const bool vec = N % 4 == 0 && reinterpret_cast<uintptr_t>(B) % SpVT<VT>::b4_align == 0 &&
                     reinterpret_cast<uintptr_t>(C) % 16 == 0;
    auto rows_launch = [&](auto flush, int64_t t0, int64_t t1) {
        constexpr bool F = decltype(flush)::value;
        if (t1 <= t0) return;
        dim3 grid((unsigned)ceil_div(t1 - t0, SP_WARPS), (unsigned)ntiles);
        const SpTask* tk = sp.tasks.get() + t0;
        if (vec)
            sp_gather_rows_kernel<VT, IT, true, F><<<grid, SP_WARPS * 32, 0, h.stream>>>(
                tk, t1 - t0, sp.short_rows.get(), sp.col.get(), val, B, C, map, M, K, N, h.d_err);
        else
            sp_gather_rows_kernel<VT, IT, false, F><<<grid, SP_WARPS * 32, 0, h.stream>>>(
                tk, t1 - t0, sp.short_rows.get(), sp.col.get(), val, B, C, map, M, K, N, h.d_err);
        after_launch(h, "sparse_gather_rows");
    };
    rows_launch(std::false_type(), 0, sp.nplain_tasks);
    rows_launch(std::true_type(), sp.nplain_tasks, sp.ntasks);
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
XS_INST_SP(__nv_bfloat16, int32_t)
XS_INST_SP(__nv_bfloat16, int64_t)
XS_INST_SP(float, int32_t)
XS_INST_SP(float, int64_t)

}  // namespace xspmm_b200
