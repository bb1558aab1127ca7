// spmm_tc.cu -- Tier-1 BCSR SpMM on the 5th-generation tensor cores: tcgen05.mma with the
// accumulator in TMEM, operands staged by TMA through an mbarrier ring.
//
// Same result as the reference kernel (src/common/spmm_math.hpp:59-122): C[16br+i, n] =
// sum over the blocks j of block row br of A_j[i, :] . B[16 col_j + :, n], every row written.
//
// Mapping (block rows stacked to M = 128): a CTA owns a group of 8 consecutive block rows and a
// 256-column tile of C. The group's block columns are merged into one sorted union list (the
// "group plan", built on the device once per matrix by a plan, or per call by the stateless
// Tier-1 entry point). For every union column u one MMA
//   D[128 x 256] += A_u[128 x 16] . B[16u .. 16u+15, n0 .. n0+255]
// is issued, where A_u stacks the 8 block rows' blocks at column u (zeros where a block row has
// no block there). One B tile therefore feeds 8 block
// rows -- the mma.sync kernel re-reads it for every block row -- and each MMA is a full-width
// 128x256x16 tcgen05 instruction. Dense-block matrices (every union column present in every
// block row) waste nothing; on scattered patterns the zero rows are wasted work, so the
// dispatcher only picks this kernel for dense block structure.
//
// Before the MMA kernel, the 8 blocks of every union entry are packed into one contiguous
// 128 x 16 tile (zeros for missing blocks), already in the shared-memory image of the K-major
// SWIZZLE_32B canonical layout, so one plain bulk copy stages it (a tensor map with 32-byte rows
// would split it into 128 requests). A pipeline stage holds four union entries: their four A tiles
// (one 16 KB bulk copy -- consecutive entries are adjacent) and their four 16 x 256 B slabs (one
// 3-D box each when N % 64 == 0, else four 64-column SWIZZLE_128B boxes; MN-major canonical
// layout). The MMAs of a stage share one tcgen05.commit: with one CTA per SM every stage costs the
// issuing thread a wait and a commit, and four MMAs per stage ran 1.35x faster than two (pruned
// LLM, N = 4096) -- a commit after every 16-deep MMA leaves the tensor pipe idle about half of the
// time.
//
// Accumulation. The tensor core's accumulation into an fp32 TMEM accumulator is not specified to
// round like IEEE FADD, and a single accumulator carried over the hundreds of union entries of a
// long block row drifts beyond the 1e-3 tolerance (an emulation with truncating additions gives
// 1.5e-2 on the 4096 x 11008 pruned-LLM matrix; IEEE fp32 in the reference's block order gives
// 1.4e-3 there). So union entries are taken in groups of TC_FLUSH_G = 16: a group accumulates in
// TMEM from zero, then its partial is added to a running fp32 sum with round-to-nearest FADD.
// TMEM holds two 128 x 256 accumulators used in turn, so the MMAs of group t+1 run while group t
// is being added.
//
// Roles (384 threads, one CTA per SM, all 512 TMEM columns): warp 0 allocates TMEM and its
// lane 0 issues tcgen05.mma and tcgen05.commit (which frees a stage once its MMAs have read it,
// and marks an accumulator full after a group); warps 1..3 are producers taking the stages in
// turn (one issuing thread cannot keep the tensor pipe busy); warps 4..11 are flushers: warp w
// reads TMEM lane quarter w % 4 (rows) and one 128-column half, keeps its 32 rows x 128 columns
// of running sums in registers, and at the end stores them to C directly, every lane one row,
// through the optional row map (so the Tier-2 unpermute stays fused). When the grid would not
// fill the GPU, the union list is split (split-K) over the CTAs of a thread-block cluster: each
// writes its partial tile to an L2-resident workspace in a store-coalesced order, and after a
// cluster barrier each CTA sums its share of the rows over the partials in rank order
// (deterministic) and stores them. Every mbarrier wait is bounded; a timeout sets an error flag
// and the CTA still waits (bounded) for its own loads and MMAs before freeing TMEM and exiting.
#include "ops.cuh"
#include "blockcols.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

namespace xspmm_b200 {
namespace {

constexpr int TC_GROUP = 8;                        // block rows per tile (M = 128)
constexpr int TC_BN = 256;                         // columns per tile = the MMA's N
constexpr int TC_KPS = 4;                          // union entries (MMAs) per stage
constexpr int TC_STAGES = 3;
constexpr int A_TILE = TC_GROUP * 512;             // 4 KB: one union entry's stacked A
constexpr int B_BOX = 16 * 128;                    // 16 rows x 64 fp16 = 2 KB
constexpr int B_SLAB = (TC_BN / 64) * B_BOX;       // 8 KB: one union entry's B rows
constexpr int A_STAGE = TC_KPS * A_TILE;           // 16 KB
constexpr int STAGE_BYTES = TC_KPS * (A_TILE + B_SLAB);  // 48 KB (multiple of 1024)
constexpr int TC_PRODUCERS = 3;                   // warps 1..3 issue the loads
constexpr int TC_FLUSHERS = 8;                    // warps 4..11 sum the TMEM partials, store C
constexpr int TC_FIRST_FLUSHER = 1 + TC_PRODUCERS;
constexpr int TC_THREADS = 32 * (1 + TC_PRODUCERS + TC_FLUSHERS);
static_assert(TC_STAGES % TC_PRODUCERS == 0, "each producer owns fixed stage slots");
static_assert(TC_FIRST_FLUSHER % 4 == 0, "flusher w reads TMEM lane quarter w % 4");
// Union entries accumulated inside the tensor core before the partial is added, with IEEE
// round-to-nearest, to the running sum in registers. The tensor core's own accumulation is not
// specified to round to nearest; a chain of hundreds of MMAs into one accumulator drifts beyond
// the 1e-3 tolerance on long block rows, a chain of 16 does not.
constexpr int TC_FLUSH_G = 16;
static_assert(TC_FLUSH_G % TC_KPS == 0, "groups end on stage boundaries");
constexpr int TC_ACC_COLS = 256;                   // one accumulator: 128 lanes x 256 fp32
constexpr int TMEM_COLS = 2 * TC_ACC_COLS;         // two accumulators, used in turn
constexpr long long WAIT_LIMIT = 1ll << 22;        // polls of an mbarrier before giving up
constexpr size_t TC_SMEM = (size_t)TC_STAGES * STAGE_BYTES + 1024 + 256;
static_assert(TC_SMEM <= 232448, "shared memory per CTA");
// full + empty per stage, acc_full[2], acc_empty[2], done, redbar, then the TMEM address
static_assert((2 * TC_STAGES + 6) * 8 + 4 <= 256, "barrier area");

// ---- PTX wrappers ---------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, P;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: false (and the error flag) if the phase did not complete.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, unsigned* err) {
    for (long long i = 0; i < WAIT_LIMIT; ++i)
        if (mbar_try_wait(b, parity)) return true;
    flag_error(err, DERR_TIMEOUT);
    return false;
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}
// Plain bulk copy (no tensor map): size and both addresses multiples of 16 bytes.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// Cluster-wide barrier (all threads of all CTAs of the cluster). Every path through the kernel
// reaches each of these the same number of times after bounded work, so it always completes.
__device__ __forceinline__ void cluster_sync_all() {
    __syncwarp();
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                     : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D (TMEM) [+]= A (smem desc) x B (smem desc), kind::f16, cta_group::1, issued by one thread.
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}
// 32 TMEM lanes (this warp's quarter) x 16 consecutive 32-bit columns, one per register.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
          "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptors (sm100 format: start>>4 [0,14), LBO>>4 [16,30), SBO>>4
// [32,46), version 1 at [46,48), layout type [61,64)).
// A: K-major, SWIZZLE_32B: rows of 32 B (16 fp16 = one MMA's K), 8-row atoms of 256 B.
__device__ __forceinline__ uint64_t desc_a(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(256 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)6 << 61);
}
// B: MN-major, SWIZZLE_128B: 64-column chunks of 16 rows x 128 B (2 KB apart = LBO), 8-row
// groups 1 KB apart (SBO).
__device__ __forceinline__ uint64_t desc_b(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)(B_BOX >> 4) << 16) |
           ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor, kind::f16: D f32 (bit 4), A/B f16 (0), A K-major (bit 15 = 0), B
// MN-major (bit 16 = 1), N >> 3 at [17,23), M >> 4 at [24,29).
constexpr uint32_t TC_IDESC = (1u << 4) | (1u << 16) | ((uint32_t)(TC_BN >> 3) << 17) |
                              ((uint32_t)(128 >> 4) << 24);
// The same with A and B in bf16 (A format at [7,10) and B format at [10,13): 1 = bf16).
constexpr uint32_t TC_IDESC_BF16 = TC_IDESC | (1u << 7) | (1u << 10);

// ---- the kernel -----------------------------------------------------------------------------------
template <typename IT, bool BF16>
__global__ void __launch_bounds__(TC_THREADS, 1)
bcsr_spmm_tc_kernel(const __half* __restrict__ apk, const __grid_constant__ CUtensorMap tmB,
                    const int64_t* __restrict__ gptr, const int32_t* __restrict__ gcol,
                    float* __restrict__ C, const IT* __restrict__ row_map, int64_t M,
                    int64_t N, int splits, int ntiles, int b3d, float4* __restrict__ ws,
                    unsigned* __restrict__ err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + TC_STAGES * STAGE_BYTES);
    uint64_t* empty = full + TC_STAGES;
    uint64_t* acc_full = empty + TC_STAGES;  // [2]: accumulator b holds a finished group
    uint64_t* acc_empty = acc_full + 2;      // [2]: accumulator b has been read by the flushers
    uint64_t* done = acc_empty + 2;          // every MMA of this CTA has completed
    uint64_t* redbar = done + 1;             // split-K bulk copies of the partials
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(redbar + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int bid = blockIdx.x;
    const int split = bid % splits;
    bid /= splits;
    const int ntile = bid % ntiles;
    const int g = bid / ntiles;
    const int64_t u0 = gptr[g], ulen = gptr[g + 1] - u0;
    const int64_t k0 = u0 + ulen * split / splits;
    const int nk = (int)(u0 + ulen * (split + 1) / splits - k0);
    const int n0 = ntile * TC_BN;

    if (threadIdx.x == 0) {
        for (int s = 0; s < TC_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], TC_FLUSHERS);
        }
        mbar_init(done, 1);
        mbar_init(redbar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // Stage j holds union entries j*KPS .. j*KPS+KPS-1 (fewer in the last stage): one MMA each,
    // and one commit per stage. Union entries form groups of TC_FLUSH_G; group t accumulates into
    // TMEM accumulator t % 2 from zero, and the flushers add it to their running sums while the
    // next group accumulates into the other one.
    const int nst = (nk + TC_KPS - 1) / TC_KPS;
    const int ngroups = (nk + TC_FLUSH_G - 1) / TC_FLUSH_G;
    if (warp == 0) {
        if (lane == 0) {  // MMA issuer
            bool ok = true;
            int mmas = 0;
            for (int j = 0; j < nst && ok; ++j) {
                const int s = j % TC_STAGES;
                if (!mbar_wait(&full[s], (j / TC_STAGES) & 1, err)) break;
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + s * STAGE_BYTES);
                const int ne = min(TC_KPS, nk - j * TC_KPS);
#pragma unroll
                for (int kk = 0; kk < TC_KPS; ++kk) {
                    if (kk >= ne) break;
                    const int e = j * TC_KPS + kk;
                    const int t = e / TC_FLUSH_G, b = t & 1;
                    const bool first = (e % TC_FLUSH_G) == 0;
                    if (first && t >= 2) {  // wait until group t-2 has left accumulator b
                        if (!mbar_wait(&acc_empty[b], ((t >> 1) - 1) & 1, err)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                    }
                    tc_mma(tmem + (uint32_t)(b * TC_ACC_COLS), desc_a(sa + kk * A_TILE),
                           desc_b(sa + A_STAGE + kk * B_SLAB), BF16 ? TC_IDESC_BF16 : TC_IDESC,
                           first ? 0u : 1u);
                    ++mmas;
                    if ((e % TC_FLUSH_G) == TC_FLUSH_G - 1 || e == nk - 1)
                        tc_commit(&acc_full[b]);
                }
                tc_commit(&empty[s]);
            }
            // arrives once every MMA issued above has completed (also after a timeout), so
            // TMEM is never freed under a running MMA
            if (mmas > 0) tc_commit(done);
            else mbar_arrive(done);
        }
    } else if (warp < TC_FIRST_FLUSHER) {
        // Warps 1..3: loads. Producer p issues the stages j = p (mod 3), so it alone refills the
        // slots s = p (mod 3) (the stage count is a multiple of 3) and its waits on them stay in
        // phase order. A single issuing thread cannot keep the tensor pipe fed; several can. Per
        // stage: one bulk copy of the stage's packed A tiles (consecutive in memory) and per
        // entry the 16 x 256 B slab (one 3-D box when N % 64 == 0, else four 64-column boxes).
        // The warp loads the union columns of 32 / KPS stages at once.
        const int p = warp - 1;
        constexpr int SPC = 32 / TC_KPS;  // stages per prefetch chunk
        int issued = 0;
        bool stop = false;
        for (int c = p; c < nst && !stop; c += SPC * TC_PRODUCERS) {
            const int e = (c + (lane / TC_KPS) * TC_PRODUCERS) * TC_KPS + lane % TC_KPS;
            const int col = e < nk ? gcol[k0 + e] : 0;
            const int cnt = min(SPC, (nst - c + TC_PRODUCERS - 1) / TC_PRODUCERS);
            for (int t = 0; t < cnt; ++t) {
                const int j = c + t * TC_PRODUCERS;
                int colt[TC_KPS];
#pragma unroll
                for (int kk = 0; kk < TC_KPS; ++kk)
                    colt[kk] = __shfl_sync(0xffffffffu, col, t * TC_KPS + kk);
                int ok = 1;
                if (lane == 0) {
                    const int s = j % TC_STAGES;
                    const int ne = min(TC_KPS, nk - j * TC_KPS);
                    if (j >= TC_STAGES && !mbar_wait(&empty[s], ((j / TC_STAGES) & 1) ^ 1, err)) {
                        ok = 0;
                    } else {
                        mbar_expect_tx(&full[s], (uint32_t)(ne * (A_TILE + B_SLAB)));
                        uint8_t* sA = smem + s * STAGE_BYTES;
                        uint8_t* sB = sA + A_STAGE;
                        bulk_load(sA, apk + (k0 + (int64_t)j * TC_KPS) * (A_TILE / 2),
                                  (uint32_t)(ne * A_TILE), &full[s]);
#pragma unroll
                        for (int kk = 0; kk < TC_KPS; ++kk) {
                            if (kk >= ne) break;
                            if (b3d) {
                                tma_load_3d(sB + kk * B_SLAB, &tmB, 0, colt[kk] * 16, n0 / 64, &full[s]);
                            } else {
#pragma unroll
                                for (int q = 0; q < TC_BN / 64; ++q)
                                    tma_load_2d(sB + kk * B_SLAB + q * B_BOX, &tmB, n0 + 64 * q,
                                                colt[kk] * 16, &full[s]);
                            }
                        }
                    }
                }
                if (!__shfl_sync(0xffffffffu, ok, 0)) {
                    stop = true;
                    break;
                }
                ++issued;
            }
        }
        // none of this producer's loads may still be in flight when the stage buffers are
        // reused for the split-K reduction or the CTA exits (bounded; they all completed unless
        // a wait timed out): its slots hold its last STAGES/PRODUCERS stages
        if (issued > 0 && lane == 0) {
            const int last = p + (issued - 1) * TC_PRODUCERS;
#pragma unroll 1
            for (int t = 0; t < TC_STAGES / TC_PRODUCERS; ++t) {
                const int j = last - t * TC_PRODUCERS;
                if (j >= p) mbar_wait(&full[j % TC_STAGES], (j / TC_STAGES) & 1, err);
            }
        }
        __syncwarp();
    } else {
        // Warps 4..11: after every group, read this warp's 32 rows x 128 columns of the
        // accumulator (lane quarter fq, column half fh) and add them to the running sums with
        // round-to-nearest FADD, then hand the accumulator back to the MMA issuer.
        const int fq = warp & 3, fh = (warp - TC_FIRST_FLUSHER) >> 2;
        float sum[TC_BN / 2];
#pragma unroll
        for (int i = 0; i < TC_BN / 2; ++i) sum[i] = 0.0f;
        bool have = true;  // every group was added
        const uint32_t lane_base = tmem + ((uint32_t)(fq * 32) << 16) + (uint32_t)(fh * (TC_BN / 2));
#pragma unroll 1
        for (int t = 0; t < ngroups; ++t) {
            const int b = t & 1;
            if (!mbar_wait(&acc_full[b], (t >> 1) & 1, err)) {
                have = false;
                break;
            }
            tc_fence_after();
            const uint32_t a = lane_base + (uint32_t)(b * TC_ACC_COLS);
#pragma unroll
            for (int c = 0; c < TC_BN / 2; c += 16) {
                uint32_t v[16];
                tmem_ld16(a + (uint32_t)c, v);
#pragma unroll
                for (int i = 0; i < 16; ++i) sum[c + i] = __fadd_rn(sum[c + i], __uint_as_float(v[i]));
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
        if (!have) {
#pragma unroll
            for (int i = 0; i < TC_BN / 2; ++i) sum[i] = 0.0f;
        }
        const int c_first = fh * (TC_BN / 2);  // this warp's first column within the tile
        if (splits == 1) {
            // Whole tile: every lane stores its row's 128 columns (through the optional row map,
            // so the Tier-2 unpermute stays fused).
            const int64_t grow = (int64_t)g * 128 + fq * 32 + lane;
            if (grow < M) {
                const int64_t orow = row_map ? (int64_t)row_map[grow] : grow;
                if (orow >= 0 && orow < M) {
                    float* dst = C + orow * N + n0 + c_first;
                    const int64_t ncol = N - (n0 + c_first);  // valid columns from dst on
                    if (ncol >= TC_BN / 2) {
                        float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
                        for (int e = 0; e < TC_BN / 8; ++e)
                            d4[e] = make_float4(sum[4 * e], sum[4 * e + 1], sum[4 * e + 2],
                                                sum[4 * e + 3]);
                    } else {
#pragma unroll
                        for (int e = 0; e < TC_BN / 2; ++e)
                            if (e < ncol) dst[e] = sum[e];
                    }
                } else {
                    flag_error(err, DERR_PERM_OUT_OF_RANGE);
                }
            }
        } else {
            // Split tile: this CTA's partial goes to the workspace, grouped by owner CTA (see
            // below): owner k's rows form one block of 64 float4 columns x nr rows, element
            // (lr, ce) at ce*nr + (lr ^ (ce & 15)).
            const int nr = 128 / splits;
            const int row = fq * 32 + lane;
            const int own = row / nr, lr = row - own * nr;
            float4* blk = ws + ((size_t)(blockIdx.x / splits) * splits + split) * 8192 +
                          (size_t)own * 64 * nr;
#pragma unroll
            for (int e = 0; e < TC_BN / 8; ++e) {
                const int ce = c_first / 4 + e;
                blk[ce * nr + (lr ^ (ce & 15))] =
                    make_float4(sum[4 * e], sum[4 * e + 1], sum[4 * e + 2], sum[4 * e + 3]);
            }
        }
    }
    __syncwarp();

    if (splits > 1) {
        // Split tile: the `splits` CTAs of the cluster (S = 2, 4 or 8) each hold a partial
        // 128 x 256 sum; rows [k*nr, (k+1)*nr) belong to CTA k (nr = 128/S). The flushers wrote
        // this CTA's partial to the workspace grouped by owner -- a warp store (32 consecutive
        // rows, one float4 column) stays within 512 bytes, and the owner's copy in shared memory
        // reads conflict-free along ce. After a cluster barrier (which publishes the stores)
        // each owner pulls its S blocks with bulk copies, in two halves of 32 float4 columns,
        // adds them in rank order (a fixed order: the result does not depend on timing) and
        // stores its rows of C, one warp per 512-byte row segment, through the row map. The
        // partials stay in L2.
        const int S = splits;
        const int nr = 128 / S;
        const int tile = blockIdx.x / S;
        float4* tile_ws = ws + (size_t)tile * S * 8192;
        // the stores above are read by other CTAs' bulk copies (async proxy)
        asm volatile("fence.proxy.async.global;" ::: "memory");
        cluster_sync_all();
        const int r0 = split * nr;
        const int nce = (int)min((int64_t)(TC_BN / 4), (N - n0 + 3) / 4);  // float4 columns of C
        float4* buf = reinterpret_cast<float4*>(smem);                    // [S][32][nr], 64 KB
        const uint32_t half_bytes = 32u * (uint32_t)nr * 16u;
#pragma unroll 1
        for (int hf = 0; hf < 2 && hf * 32 < nce; ++hf) {
            if (hf > 0) __syncthreads();  // every read of the previous half is done
            if (threadIdx.x == 32) {
                // the generic reads of this buffer come before the copy's writes
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_expect_tx(redbar, (uint32_t)S * half_bytes);
                for (int pp = 0; pp < S; ++pp)
                    bulk_load(buf + (size_t)pp * 32 * nr,
                              tile_ws + (size_t)pp * 8192 + (size_t)split * 64 * nr +
                                  (size_t)hf * 32 * nr,
                              half_bytes, redbar);
            }
            const bool ok = mbar_wait(redbar, (uint32_t)hf & 1u, err);
#pragma unroll 1
            for (int it = threadIdx.x; it < 32 * nr; it += TC_THREADS) {
                const int lr = it >> 5, cl = it & 31;  // a warp: one row, 32 float4 columns
                const int ce = hf * 32 + cl;
                const int64_t grow = (int64_t)g * 128 + r0 + lr;
                if (!ok || ce >= nce || grow >= M) continue;
                const int off = cl * nr + (lr ^ (ce & 15));
                float4 acc = buf[off];
                for (int pp = 1; pp < S; ++pp) {
                    const float4 v = buf[(size_t)pp * 32 * nr + off];
                    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
                }
                const int64_t orow = row_map ? (int64_t)row_map[grow] : grow;
                if (orow < 0 || orow >= M) {
                    flag_error(err, DERR_PERM_OUT_OF_RANGE);
                    continue;
                }
                *reinterpret_cast<float4*>(C + orow * N + n0 + (int64_t)ce * 4) = acc;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        mbar_wait(done, 0, err);  // bounded; completes once the last MMA has
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(TMEM_COLS)
                     : "memory");
    }
}

// Packs the A operand: for every union entry u, the 8 stacked blocks as one contiguous 128 x 16
// tile (4 KB, row-major; zeros for a missing block), so a stage needs one TMA load for A.
__global__ void tc_pack_kernel(const int64_t* __restrict__ gptr, int64_t ngroups,
                               const int32_t* __restrict__ gblk, const __half* __restrict__ vals,
                               __half* __restrict__ apk, int64_t bound) {
    const int64_t total = min(gptr[ngroups], bound) * 256;  // 16-byte chunks
    for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < total;
         c += (int64_t)gridDim.x * blockDim.x) {
        const int64_t u = c >> 8;
        const int within = (int)(c & 255);  // 16-byte chunk of the tile: row within>>1, half within&1
        const int b = within >> 5;          // block slot (32 chunks of 16 B per block)
        const int blk = gblk[u * TC_GROUP + b];
        uint4 v = make_uint4(0, 0, 0, 0);
        if (blk >= 0) v = reinterpret_cast<const uint4*>(vals + (int64_t)blk * 256)[within & 31];
        // stored as a SWIZZLE_32B TMA load would leave it in shared memory (16-byte half h of row
        // r at r * 32 + ((h ^ ((r >> 2) & 1)) * 16)), so one plain bulk copy stages the tile
        const int r = within >> 1, h = within & 1;
        reinterpret_cast<uint4*>(apk + u * 2048)[(r << 1) | (h ^ ((r >> 2) & 1))] = v;
    }
}

// ---- group plan: union of block columns over 8 block rows -------------------------------------
// One CTA per group: the block columns of its <= 8 block rows are marked in a shared-memory bitmap
// window (all threads), the union size is the window's population, a block's slot in the union
// is the population below its bit. Windows of 8192 columns are taken in turn.
constexpr int GP_THREADS = 256;
constexpr int GP_WORDS = 256;  // one 32-bit word per thread

__device__ __forceinline__ int64_t cta_min64(int64_t v, int64_t* red) {
    v = warp_min64(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    int64_t r = red[0];
    for (int w = 1; w < GP_THREADS / 32; ++w) r = min(r, red[w]);
    __syncthreads();
    return r;
}
__device__ __forceinline__ int64_t cta_max64(int64_t v, int64_t* red) {
    v = warp_max64(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    int64_t r = red[0];
    for (int w = 1; w < GP_THREADS / 32; ++w) r = max(r, red[w]);
    __syncthreads();
    return r;
}

// Marks the window [wb, wb + GP_WORDS*32) with the block columns of entries [e0, e1); returns
// this thread's word population, with the CTA's exclusive prefix of word populations in *pre
// and the total in *total (all after a barrier).
template <typename IT>
__device__ void gp_mark(uint32_t* win, const IT* bci, int64_t e0, int64_t e1, int64_t wb,
                        uint32_t* s_warp, uint32_t* pre_out, uint32_t* total_out) {
    const int tid = threadIdx.x;
    win[tid] = 0u;
    __syncthreads();
    const int64_t span = (int64_t)GP_WORDS * 32;
    for (int64_t e = e0 + tid; e < e1; e += GP_THREADS) {
        const int64_t d = (int64_t)bci[e] - wb;
        if (d >= 0 && d < span) atomicOr(&win[d >> 5], 1u << (d & 31));
    }
    __syncthreads();
    const uint32_t pc = __popc(win[tid]);
    const uint32_t inc = warp_inclusive_sum(pc);
    if ((tid & 31) == 31) s_warp[tid >> 5] = inc;
    __syncthreads();
    uint32_t off = 0, tot = 0;
    for (int w = 0; w < GP_THREADS / 32; ++w) {
        if (w < (tid >> 5)) off += s_warp[w];
        tot += s_warp[w];
    }
    *pre_out = off + inc - pc;
    *total_out = tot;
}

template <typename IT>
__global__ void __launch_bounds__(GP_THREADS)
tc_group_count_kernel(const IT* __restrict__ brp, const IT* __restrict__ bci, int64_t nbr,
                      int64_t ngroups, int64_t* __restrict__ cnt) {
    __shared__ uint32_t win[GP_WORDS];
    __shared__ uint32_t s_warp[GP_THREADS / 32];
    __shared__ int64_t red[GP_THREADS / 32];
    for (int64_t g = blockIdx.x; g < ngroups; g += gridDim.x) {
        const int64_t e0 = brp[g * TC_GROUP], e1 = brp[min(nbr, (g + 1) * TC_GROUP)];
        int64_t lo = INT64_MAX, hi = -1;
        for (int64_t e = e0 + threadIdx.x; e < e1; e += GP_THREADS) {
            const int64_t c = (int64_t)bci[e];
            lo = min(lo, c);
            hi = max(hi, c);
        }
        lo = cta_min64(lo, red);
        hi = cta_max64(hi, red);
        int64_t count = 0;
        for (int64_t wb = lo; wb <= hi; wb += (int64_t)GP_WORDS * 32) {
            uint32_t pre, tot;
            gp_mark(win, bci, e0, e1, wb, s_warp, &pre, &tot);
            count += tot;
            __syncthreads();
        }
        if (threadIdx.x == 0) cnt[g] = count;
    }
}

template <typename IT>
__global__ void __launch_bounds__(GP_THREADS)
tc_group_fill_kernel(const IT* __restrict__ brp, const IT* __restrict__ bci, int64_t nbr,
                     int64_t ngroups, const int64_t* __restrict__ gptr,
                     int32_t* __restrict__ gcol, int32_t* __restrict__ gblk) {
    __shared__ uint32_t win[GP_WORDS];
    __shared__ uint32_t pre_s[GP_WORDS];
    __shared__ uint32_t s_warp[GP_THREADS / 32];
    __shared__ int64_t red[GP_THREADS / 32];
    const int tid = threadIdx.x;
    for (int64_t g = blockIdx.x; g < ngroups; g += gridDim.x) {
        const int64_t r0 = g * TC_GROUP, r1 = min(nbr, r0 + TC_GROUP);
        const int64_t e0 = brp[r0], e1 = brp[r1];
        const int64_t base = gptr[g];
        int64_t lo = INT64_MAX, hi = -1;
        for (int64_t e = e0 + tid; e < e1; e += GP_THREADS) {
            const int64_t c = (int64_t)bci[e];
            lo = min(lo, c);
            hi = max(hi, c);
        }
        lo = cta_min64(lo, red);
        hi = cta_max64(hi, red);
        int64_t rank_base = 0;
        for (int64_t wb = lo; wb <= hi; wb += (int64_t)GP_WORDS * 32) {
            uint32_t pre, tot;
            gp_mark(win, bci, e0, e1, wb, s_warp, &pre, &tot);
            pre_s[tid] = pre;
            {
                uint32_t x = win[tid];
                int64_t o = base + rank_base + pre;
                while (x) {
                    const int b = __ffs(x) - 1;
                    gcol[o++] = (int32_t)(wb + (int64_t)tid * 32 + b);
                    x &= x - 1;
                }
            }
            __syncthreads();
            const int64_t span = (int64_t)GP_WORDS * 32;
            for (int64_t r = r0; r < r1; ++r) {
                const int64_t j0 = brp[r], j1 = brp[r + 1];
                for (int64_t j = j0 + tid; j < j1; j += GP_THREADS) {
                    const int64_t d = (int64_t)bci[j] - wb;
                    if (d < 0 || d >= span) continue;
                    const int64_t rank =
                        rank_base + pre_s[d >> 5] + __popc(win[d >> 5] & ((1u << (d & 31)) - 1u));
                    gblk[(base + rank) * TC_GROUP + (r - r0)] = (int32_t)j;
                }
            }
            rank_base += tot;
            __syncthreads();
        }
    }
}

// ---- host side -----------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    XS_REQUIRE(fn != nullptr, XSPMM_STATUS_CUDA_ERROR, "cuTensorMapEncodeTiled unavailable");
    return fn;
}

CUtensorMap make_map_2d(const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                        uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
    CUtensorMap m;
    std::memset(&m, 0, sizeof(m));
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base),
                                   dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    XS_REQUIRE(r == CUDA_SUCCESS, XSPMM_STATUS_CUDA_ERROR,
               "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return m;
}

// B viewed as [N/64 chunks][K rows][64 columns] (strides 128 B and N*2 B): one box of 4 chunks x
// 16 rows x 64 columns lands in shared memory as four 2 KB chunks, the MN-major SWIZZLE_128B
// canonical layout with LBO = 2 KB. Returns false if the driver rejects the view.
bool make_map_b3d(const void* B, int64_t N, int64_t K, CUtensorMap* out) {
    std::memset(out, 0, sizeof(*out));
    const cuuint64_t dims[3] = {64, (cuuint64_t)K, (cuuint64_t)(N / 64)};
    const cuuint64_t strides[2] = {(cuuint64_t)N * 2, 128};
    const cuuint32_t box[3] = {64, 16, (cuuint32_t)(TC_BN / 64)};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = encode_fn()(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(B),
                                   dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

unsigned gp_grid(Handle& h, int64_t ngroups) {
    return (unsigned)std::max<int64_t>(1, std::min(ngroups, (int64_t)sm_count(h.device) * 8));
}

}  // namespace

bool tc_supported(int64_t nbr, int64_t nbc, int64_t nnzb, const void* vals, const void* B,
                  const void* C, int64_t N) {
    return nbr > 0 && nbc > 0 && nnzb > 0 && N > 0 && N % 8 == 0 && nnzb * 16 < (int64_t(1) << 31) &&
           nbc * 16 < (int64_t(1) << 31) && reinterpret_cast<uintptr_t>(vals) % 16 == 0 &&
           reinterpret_cast<uintptr_t>(B) % 16 == 0 && reinterpret_cast<uintptr_t>(C) % 16 == 0;
}

// Stand-in with the SpMM kernel's block size and shared memory, for occupancy queries of cluster
// launches without the TMEM allocation in the way (the kernel's shared memory already limits it
// to one CTA per SM).
__global__ void __launch_bounds__(TC_THREADS, 1) tc_occupancy_stand_in(int* p) {
    if (p) p[threadIdx.x] = 0;
}

// CTAs of the tcgen05 kernel resident at once when launched in clusters of `cs` (cached per
// device and cluster size).
int64_t tc_resident_ctas(int device, int cs) {
    const void* kern = reinterpret_cast<const void*>(tc_occupancy_stand_in);
    static std::mutex mu;
    static int64_t cache[64][9] = {};
    if (device < 0 || device >= 64 || cs < 1 || cs > 8) return 0;
    std::lock_guard<std::mutex> lock(mu);
    if (cache[device][cs] == 0) {
        XS_CHECK_CUDA(cudaFuncSetAttribute(tc_occupancy_stand_in,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM));
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(cs * 64));
        cfg.blockDim = dim3(TC_THREADS);
        cfg.dynamicSmemBytes = TC_SMEM;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = (unsigned)cs;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = -1;
        }
        cache[device][cs] = n > 0 ? (int64_t)n * cs : -1;
    }
    return cache[device][cs];
}

template <typename IT>
void tc_prepare(Handle& h, int64_t nbr, int64_t nbc, int64_t nnzb, const IT* rp, const IT* ci,
                const __half* vals, TcPrep& out) {
    cudaStream_t s = h.stream;
    const int64_t ngroups = ceil_div(nbr, TC_GROUP);
    const int64_t bound = std::min(nnzb, ngroups * nbc);  // union entries, upper bound
    XS_REQUIRE(bound * 128 < (int64_t(1) << 31), XSPMM_STATUS_UNSUPPORTED, "union too large");
    out.ngroups = ngroups;
    out.bound = bound;
    out.gptr = DevBuf<int64_t>(ngroups + 1, s);
    out.gcol = DevBuf<int32_t>(std::max<int64_t>(bound, 1), s);
    DevBuf<int32_t> gblk(std::max<int64_t>(bound, 1) * TC_GROUP, s);
    XS_CHECK_CUDA(cudaMemsetAsync(gblk.get(), 0xFF, gblk.n * sizeof(int32_t), s));
    tc_group_count_kernel<IT><<<gp_grid(h, ngroups), GP_THREADS, 0, s>>>(rp, ci, nbr, ngroups,
                                                                        out.gptr.get());
    after_launch(h, "tc_group_count");
    exclusive_scan<int64_t>(h, out.gptr.get(), out.gptr.get(), ngroups);
    tc_group_fill_kernel<IT><<<gp_grid(h, ngroups), GP_THREADS, 0, s>>>(
        rp, ci, nbr, ngroups, out.gptr.get(), out.gcol.get(), gblk.get());
    after_launch(h, "tc_group_fill");
    out.apk = DevBuf<__half>((size_t)std::max<int64_t>(bound, 1) * 2048, s);
    const unsigned grid = (unsigned)std::max<int64_t>(
        1, std::min(ceil_div(bound * 256, 256), (int64_t)sm_count(h.device) * 16));
    tc_pack_kernel<<<grid, 256, 0, s>>>(out.gptr.get(), ngroups, gblk.get(), vals, out.apk.get(),
                                        bound);
    after_launch(h, "tc_pack");
}

template <typename IT>
void tc_execute(Handle& h, const TcPrep& p, const __half* B, float* C, int64_t M, int64_t K,
                int64_t N, const IT* map, bool bf16) {
    cudaStream_t s = h.stream;
    const int ntiles = (int)ceil_div(N, TC_BN);
    const int64_t tiles = p.ngroups * ntiles;
    auto kern = bf16 ? bcsr_spmm_tc_kernel<IT, true> : bcsr_spmm_tc_kernel<IT, false>;
    XS_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM));
    const int64_t avg_union = std::max<int64_t>(1, p.bound / p.ngroups);
    // Split-K factor: the CTAs of a tile form one cluster, and clusters are placed whole inside
    // a GPC, so the number resident at once depends on the cluster size. Pick the split that
    // minimises (waves) x (union entries per CTA + a fixed cost of ~30 entries for the prologue
    // and the epilogue): 1, 2, 4 or 8, never slices shorter than 32 union entries.
    int splits = 1;
    double best = 0.0;
    for (int sp = 1; sp <= 8; sp *= 2) {  // a power of two: owners get 128/sp rows
        if (sp > 1 && avg_union / sp < 32) break;
        const int64_t resident = tc_resident_ctas(h.device, sp);
        if (resident <= 0) continue;
        const int64_t waves = ceil_div(tiles * sp, resident);
        const double cost = (double)waves * ((double)avg_union / sp + 30.0);
        if (sp == 1 || cost < best * 0.97) {
            best = cost;
            splits = sp;
        }
    }
    XS_REQUIRE(tiles * splits < (int64_t(1) << 31), XSPMM_STATUS_UNSUPPORTED, "grid too large");
    int b3d = 0;
    CUtensorMap tmB;
    if (N % 64 == 0 && make_map_b3d(B, N, K, &tmB)) {
        b3d = 1;
    } else {
        tmB = make_map_2d(B, (uint64_t)N, (uint64_t)K, (uint64_t)N * 2, 64, 16,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    }
    // split-K partials: 128 x 256 fp32 per CTA (L2-resident between the two phases)
    DevBuf<float4> ws(splits > 1 ? (size_t)tiles * splits * 8192 : 0, s);
    // the CTAs of one tile (its split-K slices) form a cluster
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(tiles * splits));
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = TC_SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = splits > 1 ? 1 : 0;
    XS_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, (const __half*)p.apk.get(), tmB,
                                     (const int64_t*)p.gptr.get(), (const int32_t*)p.gcol.get(), C,
                                     map, M, N, splits, ntiles, b3d, ws.get(), h.d_err));
    after_launch(h, "bcsr_spmm_tc");
}

template <typename IT>
void bcsr_spmm_tc(Handle& h, int64_t nbr, int64_t nbc, int64_t nnzb, const IT* rp, const IT* ci,
                  const __half* vals, const __half* B, float* C, int64_t M, int64_t K, int64_t N,
                  const IT* map, bool bf16) {
    TcPrep p;
    tc_prepare<IT>(h, nbr, nbc, nnzb, rp, ci, vals, p);
    tc_execute<IT>(h, p, B, C, M, K, N, map, bf16);
}

#define XS_INST_TC(IT)                                                                            \
    template void tc_prepare<IT>(Handle&, int64_t, int64_t, int64_t, const IT*, const IT*,        \
                                 const __half*, TcPrep&);                                         \
    template void tc_execute<IT>(Handle&, const TcPrep&, const __half*, float*, int64_t, int64_t, \
                                 int64_t, const IT*, bool);                                       \
    template void bcsr_spmm_tc<IT>(Handle&, int64_t, int64_t, int64_t, const IT*, const IT*,      \
                                   const __half*, const __half*, float*, int64_t, int64_t,        \
                                   int64_t, const IT*, bool);
XS_INST_TC(int32_t)
XS_INST_TC(int64_t)

}  // namespace xspmm_b200
