// spmm_f16.cu -- Tier-1 BCSR SpMM, 16-bit blocks x 16-bit B -> fp32 C (fp16, or bf16 with the bf16
// form of the instruction), on the warp-level tensor-core path (mma.sync m16n8k16 with fp32
// accumulation).
//
// Semantics follow the reference kernel (src/common/spmm_math.hpp:59-122): for block row br,
// C[16br+i, n] = sum over its blocks j (in col_ind order) of A_j[i, :] . B[16 col_j + :, n], every
// row of C written (zeros for block rows without blocks). Unlike the reference it guards the
// ragged last block row (rows >= M are not written) and block column (B rows >= K read as zero),
// takes a 1-D grid over block rows (the reference's gridDim.y = num_block_rows stops at 65,535)
// and uses 64-bit value offsets (the reference's int32 i*256 overflows past 2^31 values).
//
// Work split: a CTA owns one block row and a TN = 64*WARPS column tile; each warp owns 64 columns
// (8 n8 tiles, 32 fp32 accumulators per thread). The products of up to 8 consecutive blocks
// accumulate in the tensor core in a zeroed fragment, which is then added to the accumulators
// with IEEE round-to-nearest adds, so a long block row collects one accumulator truncation per
// group of blocks, not per block. Per block the CTA stages the 16x16 A block
// (512 B) and the 16 x TN slab of B rows 16*col .. 16*col+15 into shared memory with 16-byte
// cp.async, STAGES deep. A is read with ldmatrix.x4 (rows XOR-swizzled by (row>>2)&1), B with
// ldmatrix.x4.trans (16-byte chunks XOR-swizzled by k&7), both conflict-free. When N is not a
// multiple of 8 the B rows are not 16-byte aligned and the slab is loaded with guarded scalar
// loads instead.
#include "ops.cuh"
#include "mma_sync.cuh"

#include <cub/device/device_radix_sort.cuh>

#include <cstdlib>
#include <cstring>
#include <vector>

namespace xspmm_b200 {
namespace {

constexpr int STAGES = 4;

using namespace warpmma;

// The values and B are 16-bit (fp16, or bf16 when BF16); only the MMA instruction differs, so
// both are read through __half pointers.
template <typename IT, int WARPS, bool ALIGNED, bool BF16>
__global__ void __launch_bounds__(WARPS * 32, WARPS == 1 ? 24 : 1)
bcsr_spmm_f16_mma_kernel(const IT* __restrict__ row_ptr, const IT* __restrict__ col_ind,
                         const __half* __restrict__ vals, const __half* __restrict__ B,
                         float* __restrict__ C, const IT* __restrict__ row_map, int64_t M,
                         int64_t K, int64_t N, const MmaItem* __restrict__ items,
                         float* __restrict__ ws, unsigned* __restrict__ err) {
    constexpr int TN = 64 * WARPS;
    constexpr int A_BYTES = 512;
    constexpr int ROW_BYTES = TN * 2;
    constexpr int B_BYTES = 16 * ROW_BYTES;
    constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    constexpr int CPR = TN / 8;  // 16-byte chunks per B row
    constexpr int THREADS = WARPS * 32;
    extern __shared__ __align__(128) uint8_t smem[];

    // Work item: a block row, or a slice of a long block row whose partial sum goes to
    // workspace slot `slot` (16 x N floats) and is reduced afterwards in a fixed order.
    int64_t br, jb;
    int nblk, slot = -1;
    if (items) {
        const MmaItem it = items[blockIdx.x];
        br = it.br;
        jb = it.jb;
        nblk = it.nblk;
        slot = it.slot;
    } else {
        br = blockIdx.x;
        jb = row_ptr[br];
        nblk = (int)(row_ptr[br + 1] - jb);
    }
    const int64_t n0 = (int64_t)blockIdx.y * TN;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool warp_active = n0 + warp * 64 < N;

    // B slab chunks: every thread always copies the same ITER (row k, 16-byte chunk ch) pairs of
    // a slab, so their offsets are computed once and a stage costs one multiply-add per chunk.
    constexpr int ITER = 16 * CPR / THREADS;
    static_assert(16 * CPR % THREADS == 0, "slab chunks divide evenly over the threads");
    int64_t b_src[ITER];
    int b_dst[ITER], b_k[ITER];
    bool b_col_ok[ITER];
#pragma unroll
    for (int it = 0; it < ITER; ++it) {
        const int c = threadIdx.x + it * THREADS;
        const int k = c / CPR, ch = c % CPR;
        b_k[it] = k;
        b_src[it] = (int64_t)k * N + n0 + ch * 8;
        b_dst[it] = k * ROW_BYTES + ((ch ^ (k & 7)) * 16);
        b_col_ok[it] = n0 + ch * 8 < N;
    }

    auto load_stage = [&](int stage, int64_t j) {
        uint8_t* sA = smem + stage * STAGE_BYTES;
        uint8_t* sB = sA + A_BYTES;
        const int64_t bc = (int64_t)col_ind[j];
        if (threadIdx.x < 32) {
            const int c = threadIdx.x, row = c >> 1, ch = c & 1;
            uint8_t* dst = sA + row * 32 + ((ch ^ ((row >> 2) & 1)) * 16);
            const __half* src = vals + j * 256 + row * 16 + ch * 8;
            if constexpr (ALIGNED) {
                cp_async16(dst, src, 16);
            } else {
                __align__(16) __half t[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) t[e] = src[e];
                *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(t);
            }
        }
        if constexpr (ALIGNED) {
            const __half* Bb = B + bc * 16 * N;
            const int64_t krem = K - bc * 16;  // rows of this slab inside B
#pragma unroll
            for (int it = 0; it < ITER; ++it) {
                const bool ok = b_col_ok[it] && b_k[it] < krem;
                cp_async16(sB + b_dst[it], ok ? (const void*)(Bb + b_src[it]) : (const void*)B,
                           ok ? 16 : 0);
            }
        } else {
            for (int c = threadIdx.x; c < 16 * CPR; c += THREADS) {
                const int k = c / CPR, ch = c % CPR;
                const int64_t grow = bc * 16 + k;
                const int64_t gcol = n0 + ch * 8;
                uint8_t* dst = sB + k * ROW_BYTES + ((ch ^ (k & 7)) * 16);
                __align__(16) __half t[8];
#pragma unroll
                for (int e = 0; e < 8; ++e)
                    t[e] = (grow < K && gcol + e < N) ? B[grow * N + gcol + e] : __half(0.0f);
                *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(t);
            }
        }
    };

    // Products of up to GROUP consecutive blocks accumulate in the tensor core (fragment p); each
    // group's sum is then added to the running sum with IEEE round-to-nearest adds, so a long
    // block row collects one accumulator truncation per group of blocks, not per block.
    constexpr int GROUP = 8;
    float acc[8][4], p[8][4];
#pragma unroll
    for (int t = 0; t < 8; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[t][e] = p[t][e] = 0.0f;

#pragma unroll
    for (int s = 0; s < STAGES - 1; ++s) {
        if (s < nblk) load_stage(s, jb + s);
        cp_async_commit();
    }

    // per-lane ldmatrix offsets (bytes within a stage)
    const int mi = lane >> 3, rin = lane & 7;
    const int a_row = rin + 8 * (mi & 1);
    const int a_off = a_row * 32 + (((mi >> 1) ^ ((a_row >> 2) & 1)) * 16);
    const int b_kk = rin + 8 * (mi & 1);

    for (int i = 0; i < nblk; ++i) {
        cp_async_wait<STAGES - 2>();
        __syncthreads();
        const uint8_t* sA = smem + (i % STAGES) * STAGE_BYTES;
        const uint8_t* sB = sA + A_BYTES;
        if (warp_active) {
            uint32_t a[4];
            ldmatrix_x4(a, sA + a_off);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int chunk = (warp * 64 + j * 16) / 8 + (mi >> 1);
                uint32_t b[4];
                ldmatrix_x4_trans(b, sB + b_kk * ROW_BYTES + ((chunk ^ (b_kk & 7)) * 16));
                mma_16816<BF16>(p[2 * j], a, b[0], b[1]);
                mma_16816<BF16>(p[2 * j + 1], a, b[2], b[3]);
            }
            if ((i + 1) % GROUP == 0 || i + 1 == nblk) {
#pragma unroll
                for (int t = 0; t < 8; ++t)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        acc[t][e] = __fadd_rn(acc[t][e], p[t][e]);
                        p[t][e] = 0.0f;
                    }
            }
        }
        const int nx = i + STAGES - 1;
        if (nx < nblk) load_stage(nx % STAGES, jb + nx);
        cp_async_commit();
    }
    cp_async_wait<0>();

    if (!warp_active) return;
    const int g = lane >> 2, q = lane & 3;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        if (slot >= 0) {  // partial of a split block row: all 16 rows, no row map
            float* prow = ws + ((int64_t)slot * 16 + g + 8 * half) * N;
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                const int64_t col = n0 + warp * 64 + t * 8 + 2 * q;
                if (col < N) prow[col] = acc[t][2 * half];
                if (col + 1 < N) prow[col + 1] = acc[t][2 * half + 1];
            }
            continue;
        }
        const int64_t r = br * 16 + g + 8 * half;
        if (r >= M) continue;
        const int64_t orow = row_map ? (int64_t)row_map[r] : r;
        if (orow < 0 || orow >= M) {
            flag_error(err, DERR_PERM_OUT_OF_RANGE);
            continue;
        }
        float* crow = C + orow * N;
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            const int64_t col = n0 + warp * 64 + t * 8 + 2 * q;
            const float v0 = acc[t][2 * half], v1 = acc[t][2 * half + 1];
            if constexpr (ALIGNED) {
                if (col < N) *reinterpret_cast<float2*>(crow + col) = make_float2(v0, v1);
            } else {
                if (col < N) crow[col] = v0;
                if (col + 1 < N) crow[col + 1] = v1;
            }
        }
    }
}

template <typename IT, int WARPS, bool ALIGNED>
void launch(Handle& h, int64_t nbr, const IT* rp, const IT* ci, const __half* v, const __half* B,
            float* C, int64_t M, int64_t K, int64_t N, const IT* map, const MmaItem* items,
            float* ws, bool bf16) {
    constexpr int TN = 64 * WARPS;
    constexpr int smem = STAGES * (512 + 16 * TN * 2);
    static_assert(smem <= 48 * 1024, "stage ring must fit the default dynamic smem limit");
    auto kern = bf16 ? bcsr_spmm_f16_mma_kernel<IT, WARPS, ALIGNED, true>
                     : bcsr_spmm_f16_mma_kernel<IT, WARPS, ALIGNED, false>;
    dim3 grid((unsigned)nbr, (unsigned)ceil_div(N, TN));  // nbr = number of work items
    kern<<<grid, WARPS * 32, smem, h.stream>>>(rp, ci, v, B, C, map, M, K, N, items, ws, h.d_err);
    after_launch(h, "bcsr_spmm_f16_mma");
}

}  // namespace

Tier1Kernel tier1_kernel_choice(const Handle& h) {
    if (h.tier1_kernel == 1) return Tier1Kernel::Mma;
    if (h.tier1_kernel == 2) return Tier1Kernel::Tc;
    static const Tier1Kernel k = [] {
        const char* e = std::getenv("XSPMM_TIER1_KERNEL");
        if (e && std::strcmp(e, "mma") == 0) return Tier1Kernel::Mma;
        if (e && std::strcmp(e, "tc") == 0) return Tier1Kernel::Tc;
        return Tier1Kernel::Auto;
    }();
    return k;
}

// tcgen05 stacks 8 block rows per MMA over the union of their block columns, so it pays when the
// block grid is dense (little zero padding) and block rows are long (B tiles reused 8 times).
bool tc_preferred(int64_t nbr, int64_t nbc, int64_t nnzb) {
    const double density = (double)nnzb / ((double)nbr * (double)nbc);
    return density >= 0.25 && nnzb >= 32 * nbr;
}

template <typename IT>
static void bcsr_spmm_f16_impl(Handle& h, int64_t nbr, int64_t nbc, int64_t nnzb, const IT* rp,
                               const IT* ci, const __half* v, const __half* B, float* C,
                               int64_t M, int64_t K, int64_t N, const IT* map, bool bf16) {
    if (nbr == 0 || N == 0 || M == 0) return;
    const Tier1Kernel choice = tier1_kernel_choice(h);
    if (choice != Tier1Kernel::Mma && tc_supported(nbr, nbc, nnzb, v, B, C, N) &&
        (choice == Tier1Kernel::Tc || tc_preferred(nbr, nbc, nnzb))) {
        bcsr_spmm_tc<IT>(h, nbr, nbc, nnzb, rp, ci, v, B, C, M, K, N, map, bf16);
        return;
    }
    bcsr_spmm_mma_f16<IT>(h, nbr, rp, ci, v, B, C, M, K, N, map, nullptr, bf16);
}

// C[map(16 br + i), n] = sum over the slots of split block row br, in slot order.
template <typename IT>
__global__ void mma_split_reduce_kernel(const float* __restrict__ ws,
                                        const int32_t* __restrict__ long_rows,
                                        const int32_t* __restrict__ first_slot, int64_t nlong,
                                        float* __restrict__ C, const IT* __restrict__ row_map,
                                        int64_t M, int64_t N, unsigned* __restrict__ err) {
    const int64_t total = nlong * 16 * N;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t l = e / (16 * N), rem = e % (16 * N);
        const int i = (int)(rem / N);
        const int64_t n = rem % N;
        const int64_t r = (int64_t)long_rows[l] * 16 + i;
        if (r >= M) continue;
        const int s0 = first_slot[l], s1 = first_slot[l + 1];
        float acc = ws[((int64_t)s0 * 16 + i) * N + n];
        for (int sl = s0 + 1; sl < s1; ++sl) acc = __fadd_rn(acc, ws[((int64_t)sl * 16 + i) * N + n]);
        const int64_t orow = row_map ? (int64_t)row_map[r] : r;
        if (orow < 0 || orow >= M) {
            flag_error(err, DERR_PERM_OUT_OF_RANGE);
            continue;
        }
        C[orow * N + n] = acc;
    }
}

template <typename IT>
void bcsr_spmm_mma_f16(Handle& h, int64_t nbr, const IT* rp, const IT* ci, const __half* v,
                       const __half* B, float* C, int64_t M, int64_t K, int64_t N, const IT* map,
                       const MmaWork* work, bool bf16) {
    if (nbr == 0 || N == 0 || M == 0) return;
    const bool listed = work && work->nitems > 0;
    const int64_t nwork = listed ? work->nitems : nbr;
    const MmaItem* items = listed ? work->items.get() : nullptr;
    DevBuf<float> wsb(listed && work->nslots > 0 ? (size_t)(work->nslots * 16 * N) : 0, h.stream);
    float* ws = wsb.get();
    XS_REQUIRE(ceil_div(N, 64) <= 65535, XSPMM_STATUS_UNSUPPORTED, "N above 4,194,240 columns");
    const bool aligned = (N % 8 == 0) && (reinterpret_cast<uintptr_t>(B) % 16 == 0) &&
                         (reinterpret_cast<uintptr_t>(v) % 16 == 0) &&
                         (reinterpret_cast<uintptr_t>(C) % 8 == 0);
    const int warps = N <= 64 ? 1 : (N <= 128 ? 2 : 4);
    if (aligned) {
        if (warps == 1) launch<IT, 1, true>(h, nwork, rp, ci, v, B, C, M, K, N, map, items, ws, bf16);
        else if (warps == 2) launch<IT, 2, true>(h, nwork, rp, ci, v, B, C, M, K, N, map, items, ws, bf16);
        else launch<IT, 4, true>(h, nwork, rp, ci, v, B, C, M, K, N, map, items, ws, bf16);
    } else {
        if (warps == 1) launch<IT, 1, false>(h, nwork, rp, ci, v, B, C, M, K, N, map, items, ws, bf16);
        else if (warps == 2) launch<IT, 2, false>(h, nwork, rp, ci, v, B, C, M, K, N, map, items, ws, bf16);
        else launch<IT, 4, false>(h, nwork, rp, ci, v, B, C, M, K, N, map, items, ws, bf16);
    }
    if (listed && work->nlong > 0) {
        const int64_t total = work->nlong * 16 * N;
        const unsigned grid = (unsigned)std::max<int64_t>(
            1, std::min(ceil_div(total, 256), (int64_t)sm_count(h.device) * 16));
        mma_split_reduce_kernel<IT><<<grid, 256, 0, h.stream>>>(
            ws, work->long_rows.get(), work->first_slot.get(), work->nlong, C, map, M, N, h.d_err);
        after_launch(h, "mma_split_reduce");
    }
}

template void bcsr_spmm_mma_f16<int32_t>(Handle&, int64_t, const int32_t*, const int32_t*,
                                         const __half*, const __half*, float*, int64_t, int64_t,
                                         int64_t, const int32_t*, const MmaWork*, bool);
template void bcsr_spmm_mma_f16<int64_t>(Handle&, int64_t, const int64_t*, const int64_t*,
                                         const __half*, const __half*, float*, int64_t, int64_t,
                                         int64_t, const int64_t*, const MmaWork*, bool);

// Block rows sorted by their first block column (empty rows last): the execution order a plan
// gives the mma.sync kernel, so that CTAs running together gather nearby rows of B and the gather
// hits L2. The product of each block row does not depend on the order.
template <typename IT>
__global__ void first_col_keys_kernel(const IT* __restrict__ rp, const IT* __restrict__ ci,
                                      int64_t nbr, int64_t nbc, uint32_t* __restrict__ keys,
                                      int32_t* __restrict__ rows) {
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < nbr;
         r += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = rp[r];
        keys[r] = rp[r + 1] > b ? (uint32_t)ci[b] : (uint32_t)nbc;
        rows[r] = (int32_t)r;
    }
}

template <typename IT>
void block_row_order(Handle& h, int64_t nbr, int64_t nbc, const IT* rp, const IT* ci,
                     DevBuf<int32_t>& order) {
    XS_REQUIRE(nbr < (int64_t(1) << 31) && nbc < (int64_t(1) << 32), XSPMM_STATUS_UNSUPPORTED,
               "block grid too large to order");
    cudaStream_t s = h.stream;
    order = DevBuf<int32_t>(std::max<int64_t>(nbr, 1), s);
    if (nbr == 0) return;
    DevBuf<uint32_t> k_in(nbr, s), k_out(nbr, s);
    DevBuf<int32_t> r_in(nbr, s);
    const unsigned grid = (unsigned)std::max<int64_t>(
        1, std::min(ceil_div(nbr, 256), (int64_t)sm_count(h.device) * 8));
    first_col_keys_kernel<IT><<<grid, 256, 0, s>>>(rp, ci, nbr, nbc, k_in.get(), r_in.get());
    after_launch(h, "first_col_keys");
    int end_bit = 1;
    while (end_bit < 32 && (uint64_t(1) << end_bit) <= (uint64_t)nbc) ++end_bit;
    size_t tmp_bytes = 0;
    XS_CHECK_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, tmp_bytes, k_in.get(), k_out.get(),
                                                  r_in.get(), order.get(), (int)nbr, 0, end_bit, s));
    DevBuf<uint8_t> tmp(std::max<size_t>(tmp_bytes, 1), s);
    XS_CHECK_CUDA(cub::DeviceRadixSort::SortPairs(tmp.get(), tmp_bytes, k_in.get(), k_out.get(),
                                                  r_in.get(), order.get(), (int)nbr, 0, end_bit, s));
    h.launches += 1;
}
template <typename IT>
void mma_work_build(Handle& h, int64_t nbr, int64_t nbc, int64_t nnzb, const IT* rp,
                    const IT* ci, bool by_first_col, MmaWork& out,
                    const std::vector<uint8_t>* keep) {
    cudaStream_t s = h.stream;
    std::vector<int32_t> order(nbr);
    if (by_first_col) {
        DevBuf<int32_t> d_order;
        block_row_order<IT>(h, nbr, nbc, rp, ci, d_order);
        XS_CHECK_CUDA(cudaMemcpyAsync(order.data(), d_order.get(), nbr * sizeof(int32_t),
                                      cudaMemcpyDeviceToHost, s));
    } else {
        for (int64_t r = 0; r < nbr; ++r) order[r] = (int32_t)r;
    }
    std::vector<IT> hrp(nbr + 1);
    XS_CHECK_CUDA(cudaMemcpyAsync(hrp.data(), rp, (nbr + 1) * sizeof(IT), cudaMemcpyDeviceToHost, s));
    XS_CHECK_CUDA(cudaStreamSynchronize(s));
    // Slices of at most `chunk` blocks: one CTA walks its blocks in sequence, so a block row of
    // thousands of blocks (the hub rows of a power-law graph) would otherwise set the time of the
    // whole product.
    const int64_t chunk = std::max<int64_t>(128, ceil_div(nnzb, (int64_t)sm_count(h.device) * 64));
    std::vector<MmaItem> items;
    std::vector<int32_t> long_rows, first_slot;
    items.reserve(nbr);
    int32_t slot = 0;
    bool dropped = false;  // block rows left to another kernel (keep[r] == 0)
    for (int64_t t = 0; t < nbr; ++t) {
        const int32_t r = order[t];
        if (keep && !(*keep)[r]) {
            dropped = true;
            continue;
        }
        const int64_t j0 = (int64_t)hrp[r], len = (int64_t)hrp[r + 1] - j0;
        if (len <= chunk) {
            items.push_back(MmaItem{j0, r, (int32_t)len, -1, 0});
            continue;
        }
        long_rows.push_back(r);
        first_slot.push_back(slot);
        for (int64_t o = 0; o < len; o += chunk)
            items.push_back(MmaItem{j0 + o, r, (int32_t)std::min(chunk, len - o), slot++, 0});
    }
    first_slot.push_back(slot);
    if (long_rows.empty() && !by_first_col && !dropped) {  // every row, natural order: no list
        out.nitems = 0;
        return;
    }
    out.empty = items.empty();
    XS_REQUIRE(items.size() < (size_t(1) << 31), XSPMM_STATUS_UNSUPPORTED, "too many work items");
    out.nitems = (int64_t)items.size();
    out.nlong = (int64_t)long_rows.size();
    out.nslots = slot;
    out.items = DevBuf<MmaItem>(std::max<size_t>(items.size(), 1), s);
    XS_CHECK_CUDA(cudaMemcpyAsync(out.items.get(), items.data(), items.size() * sizeof(MmaItem),
                                  cudaMemcpyHostToDevice, s));
    out.long_rows = DevBuf<int32_t>(std::max<size_t>(long_rows.size(), 1), s);
    out.first_slot = DevBuf<int32_t>(first_slot.size(), s);
    if (!long_rows.empty())
        XS_CHECK_CUDA(cudaMemcpyAsync(out.long_rows.get(), long_rows.data(),
                                      long_rows.size() * sizeof(int32_t), cudaMemcpyHostToDevice, s));
    XS_CHECK_CUDA(cudaMemcpyAsync(out.first_slot.get(), first_slot.data(),
                                  first_slot.size() * sizeof(int32_t), cudaMemcpyHostToDevice, s));
    XS_CHECK_CUDA(cudaStreamSynchronize(s));  // the host vectors go out of scope
}

template void block_row_order<int32_t>(Handle&, int64_t, int64_t, const int32_t*, const int32_t*,
                                       DevBuf<int32_t>&);
template void mma_work_build<int32_t>(Handle&, int64_t, int64_t, int64_t, const int32_t*,
                                      const int32_t*, bool, MmaWork&, const std::vector<uint8_t>*);
template void mma_work_build<int64_t>(Handle&, int64_t, int64_t, int64_t, const int64_t*,
                                      const int64_t*, bool, MmaWork&, const std::vector<uint8_t>*);
template void block_row_order<int64_t>(Handle&, int64_t, int64_t, const int64_t*, const int64_t*,
                                       DevBuf<int32_t>&);

#define XS_BCSR_SPMM_16(VT, IT, BF)                                                               \
    template <>                                                                                   \
    void bcsr_spmm<VT, IT>(Handle & h, int64_t nbr, int64_t nbc, int64_t nnzb, const IT* rp,      \
                           const IT* ci, const VT* v, const VT* B, float* C, int64_t M,           \
                           int64_t K, int64_t N, const IT* map) {                                 \
        bcsr_spmm_f16_impl<IT>(h, nbr, nbc, nnzb, rp, ci, as_half(v), as_half(B), C, M, K, N, map, \
                               BF);                                                               \
    }
XS_BCSR_SPMM_16(__half, int32_t, false)
XS_BCSR_SPMM_16(__half, int64_t, false)
XS_BCSR_SPMM_16(__nv_bfloat16, int32_t, true)
XS_BCSR_SPMM_16(__nv_bfloat16, int64_t, true)

}  // namespace xspmm_b200
