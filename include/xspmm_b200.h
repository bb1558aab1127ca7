/*
 * xspmm_b200.h -- C ABI of the B200-native xSpMM hot path (libxspmm_b200.so).
 *
 * Plain pointers and sizes only. Every pointer to matrix data is a DEVICE pointer on the handle's
 * device (the reference's API takes device pointers too: include/xspmm/xspmm.hpp:14-40). Work is
 * enqueued on the handle's stream; functions that must return a size to the host (the CSR->BCSR
 * count) synchronize that stream. Every function returns an xspmm_status_t; on failure
 * xspmm_last_error() gives a message for the calling thread.
 *
 * Index types: the reference templates every function on IndexType in {int32_t, int64_t}
 * (include/xspmm/matrix/csr.hpp:12, bcsr.hpp:12); each entry point here exists with suffix _i32
 * and _i64. Value types: __half (f16) and float (f32), the instantiations the reference's CUDA
 * backend names (src/cuda/unstructured_mtx_mul.cu:137-148), and __nv_bfloat16 (bf16), which
 * takes the f16 paths with the bf16 form of the tensor-core instructions (fp32 accumulation).
 *
 * The C++ API mirroring the reference (xspmm::spmm, CudaExecutor, CSRMatrix, BCSRMatrix,
 * SpMMTimings) is header-only on top of this ABI: include/xspmm/xspmm.hpp.
 */
#ifndef XSPMM_B200_H
#define XSPMM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum xspmm_status {
    XSPMM_STATUS_OK = 0,
    XSPMM_STATUS_INVALID_ARGUMENT = 1, /* bad sizes/pointers, or a malformed CSR/permutation */
    XSPMM_STATUS_UNSUPPORTED = 2,      /* e.g. a plan over a BCSR whose blocks are not 16x16 */
    XSPMM_STATUS_CUDA_ERROR = 3,
    XSPMM_STATUS_OUT_OF_MEMORY = 4,
    XSPMM_STATUS_NCCL_ERROR = 5,
    XSPMM_STATUS_TIMEOUT = 6,
    XSPMM_STATUS_INTERNAL = 7
} xspmm_status_t;

typedef struct xspmm_handle_s* xspmm_handle_t;

/* Mirrors xspmm::SpMMTimings (include/xspmm/core/timings.hpp:7-14). Milliseconds, device time
 * measured with CUDA events on the handle's stream. */
typedef struct xspmm_timings {
    double clustering_ms;
    double permutation_ms;
    double conversion_ms;
    double spmm_ms;
    double unpermutation_ms;
    double total_pipeline_ms;
} xspmm_timings_t;

/* ---------------------------------------------------------------------------------------------
 * Environment variables. Results never depend on them (every path is exact for the structure and
 * within the SpMM tolerance for C); they select among equivalent kernels, for comparisons and
 * tests. Unset means automatic.
 *   XSPMM_CLUSTER_KERNEL = index | bits | sweep   clustering path (read at every clustering
 *       call): the inverted index, row bitsets in one SM's shared memory, or the row patterns
 *       spread over a thread-block cluster. bits and sweep return UNSUPPORTED when the matrix
 *       does not fit them.
 *   XSPMM_CLUSTER_SEED_SETS = 0                    the index path without the per-row seed sets
 *       (every pass walks the index; read at every clustering call).
 *   XSPMM_TIER1_KERNEL = mma | tc                  default fp16 Tier-1 kernel of every handle
 *       whose xspmm_set_tier1_kernel is automatic (read once per process).
 *   XSPMM_GATHER_KERNEL = simt                     16-bit plans multiply their nearly empty
 *       block rows on the SIMT gather kernels instead of the tensor-core gather (read once per
 *       process).
 * ------------------------------------------------------------------------------------------- */

/* ---------------------------------------------------------------------------------------------
 * Handle. Replaces the role of xspmm::CudaExecutor (include/xspmm/core/executor.hpp:37-51,
 * src/core/executor.cpp:80-108): it binds a device (made current inside every call, so handles on
 * different devices can be used from one thread) and a stream. stream == NULL means the legacy
 * default stream, which is what the reference launches on (src/cuda/unstructured_mtx_mul.cu:47).
 * ------------------------------------------------------------------------------------------- */
xspmm_status_t xspmm_create(int device, void* stream, xspmm_handle_t* out);
xspmm_status_t xspmm_destroy(xspmm_handle_t h);
xspmm_status_t xspmm_set_stream(xspmm_handle_t h, void* stream);
xspmm_status_t xspmm_get_device(xspmm_handle_t h, int* device);
/* Number of kernels this library has launched on the handle since creation (or the last reset). */
xspmm_status_t xspmm_get_launch_count(xspmm_handle_t h, uint64_t* count);
xspmm_status_t xspmm_reset_launch_count(xspmm_handle_t h);
/* Selects the fp16 Tier-1 kernel for this handle: 0 = automatic (tcgen05 for dense block
 * structure, mma.sync otherwise), 1 = warp-level mma.sync m16n8k16, 2 = tcgen05/TMEM with 8 block
 * rows stacked per MMA (falls back to mma.sync when N % 8 != 0 or pointers are not 16-byte
 * aligned). The reference has a single WMMA kernel; this choice exists for the comparison of the
 * two tensor-core paths. Results agree within the SpMM tolerance either way. */
xspmm_status_t xspmm_set_tier1_kernel(xspmm_handle_t h, int kind);
const char* xspmm_status_string(xspmm_status_t s);
const char* xspmm_last_error(void);
/* Device memory through the handle: replaces Executor::allocate/free/copy_*
 * (include/xspmm/core/executor.hpp:14-21). Copies are stream-ordered and synchronous w.r.t. the
 * host on return, like the reference's cudaMemcpy (src/core/executor.cpp:94-104). */
xspmm_status_t xspmm_malloc(xspmm_handle_t h, void** ptr, size_t bytes);
xspmm_status_t xspmm_free(xspmm_handle_t h, void* ptr);
xspmm_status_t xspmm_memcpy_h2d(xspmm_handle_t h, void* dst, const void* src, size_t bytes);
xspmm_status_t xspmm_memcpy_d2h(xspmm_handle_t h, void* dst, const void* src, size_t bytes);
xspmm_status_t xspmm_memcpy_d2d(xspmm_handle_t h, void* dst, const void* src, size_t bytes);
xspmm_status_t xspmm_synchronize(xspmm_handle_t h);

/* ---------------------------------------------------------------------------------------------
 * Tier-1 BCSR SpMM: C = A * B with A in BCSR (r_block x c_block blocks, row-major inside a block).
 * Replaces xspmm::spmm(const BCSRMatrix&, const In* B, Out* C, N) (include/xspmm/xspmm.hpp:14-18,
 * dispatch src/xspmm.cpp:29-52, launcher src/cuda/unstructured_mtx_mul.cu:31-51, kernel
 * src/common/spmm_math.hpp:20-146).
 *   A: num_block_rows, num_block_cols, num_blocks, row_ptr[num_block_rows+1], col_ind[num_blocks],
 *      values[num_blocks*r_block*c_block]. 16 x 16 blocks take the tensor-core kernels. Any other
 *      shape (r_block, c_block >= 1) takes a SIMT kernel that sums each row in fp64, column
 *      order, and rounds once: the reference kernel hard-codes 16 x 16
 *      (src/cuda/unstructured_mtx_mul.cu:39) and so mis-computes other shapes; this computes the
 *      product the BCSR describes.
 *   B: K x N row-major (ld = N); C: M x N row-major fp32 (ld = N), every row overwritten.
 *   M, K: true row counts of C and B. Pass num_block_rows*r_block / num_block_cols*c_block for
 *      the reference's behaviour; smaller values guard the ragged last block row / column, which the
 *      reference kernel reads and writes out of bounds (src/common/spmm_math.hpp:80, :118-122).
 *   out_row_map: NULL, or int array of M entries giving the row of C that row i of A*B goes to
 *      (fuses the Tier-2 unpermute into the store). Same index type as row_ptr.
 * ------------------------------------------------------------------------------------------- */
xspmm_status_t xspmm_bcsr_spmm_f16f32_i32(xspmm_handle_t h, int32_t num_block_rows,
    int32_t num_block_cols, int32_t num_blocks, int32_t r_block, int32_t c_block,
    const int32_t* row_ptr, const int32_t* col_ind, const void* values, const void* B, float* C,
    int32_t M, int32_t K, int32_t N, const int32_t* out_row_map);
xspmm_status_t xspmm_bcsr_spmm_f16f32_i64(xspmm_handle_t h, int64_t num_block_rows,
    int64_t num_block_cols, int64_t num_blocks, int64_t r_block, int64_t c_block,
    const int64_t* row_ptr, const int64_t* col_ind, const void* values, const void* B, float* C,
    int64_t M, int64_t K, int64_t N, const int64_t* out_row_map);
xspmm_status_t xspmm_bcsr_spmm_bf16f32_i32(xspmm_handle_t h, int32_t num_block_rows,
    int32_t num_block_cols, int32_t num_blocks, int32_t r_block, int32_t c_block,
    const int32_t* row_ptr, const int32_t* col_ind, const void* values, const void* B, float* C,
    int32_t M, int32_t K, int32_t N, const int32_t* out_row_map);
xspmm_status_t xspmm_bcsr_spmm_bf16f32_i64(xspmm_handle_t h, int64_t num_block_rows,
    int64_t num_block_cols, int64_t num_blocks, int64_t r_block, int64_t c_block,
    const int64_t* row_ptr, const int64_t* col_ind, const void* values, const void* B, float* C,
    int64_t M, int64_t K, int64_t N, const int64_t* out_row_map);
xspmm_status_t xspmm_bcsr_spmm_f32f32_i32(xspmm_handle_t h, int32_t num_block_rows,
    int32_t num_block_cols, int32_t num_blocks, int32_t r_block, int32_t c_block,
    const int32_t* row_ptr, const int32_t* col_ind, const void* values, const void* B, float* C,
    int32_t M, int32_t K, int32_t N, const int32_t* out_row_map);
xspmm_status_t xspmm_bcsr_spmm_f32f32_i64(xspmm_handle_t h, int64_t num_block_rows,
    int64_t num_block_cols, int64_t num_blocks, int64_t r_block, int64_t c_block,
    const int64_t* row_ptr, const int64_t* col_ind, const void* values, const void* B, float* C,
    int64_t M, int64_t K, int64_t N, const int64_t* out_row_map);

/* ---------------------------------------------------------------------------------------------
 * Greedy 1-D Jaccard (Sylos-Labini) row clustering. Replaces
 * xspmm::compute_1d_jaccard_clustering(exec, A, dist_thresh, block_width, perm_out)
 * (include/xspmm/clustering.hpp:19-25, src/xspmm.cpp:57-67, src/cpu/clustering_sylos_labini.cpp:
 * 51-120). Writes perm_out[M] (perm[new] = old), bit-identical to the reference. Only row_ptr and
 * col_ind are read (the reference ignores values too).
 * ------------------------------------------------------------------------------------------- */
xspmm_status_t xspmm_cluster_jaccard_i32(xspmm_handle_t h, int32_t M, int32_t K, int32_t nnz,
    const int32_t* row_ptr, const int32_t* col_ind, float dist_thresh, int32_t block_width,
    int32_t* perm_out);
xspmm_status_t xspmm_cluster_jaccard_i64(xspmm_handle_t h, int64_t M, int64_t K, int64_t nnz,
    const int64_t* row_ptr, const int64_t* col_ind, float dist_thresh, int64_t block_width,
    int64_t* perm_out);

/* ---------------------------------------------------------------------------------------------
 * CSR row permutation: out row i = row perm[i] of A, entries in their original order. Replaces
 * xspmm::apply_permutation (include/xspmm/clustering.hpp:34-38, src/cuda/mtx_permutation.cu:12-65,
 * kernels src/common/permutation.hpp:15-66). Output arrays are caller-allocated: out_row_ptr[M+1],
 * out_col_ind[nnz], out_values[nnz]. perm must be a permutation of [0, M) (checked: entries out
 * of range give INVALID_ARGUMENT).
 * ------------------------------------------------------------------------------------------- */
xspmm_status_t xspmm_permute_rows_f16_i32(xspmm_handle_t h, int32_t M, int32_t K, int32_t nnz,
    const int32_t* row_ptr, const int32_t* col_ind, const void* values, const int32_t* perm,
    int32_t* out_row_ptr, int32_t* out_col_ind, void* out_values);
xspmm_status_t xspmm_permute_rows_f16_i64(xspmm_handle_t h, int64_t M, int64_t K, int64_t nnz,
    const int64_t* row_ptr, const int64_t* col_ind, const void* values, const int64_t* perm,
    int64_t* out_row_ptr, int64_t* out_col_ind, void* out_values);
xspmm_status_t xspmm_permute_rows_bf16_i32(xspmm_handle_t h, int32_t M, int32_t K, int32_t nnz,
    const int32_t* row_ptr, const int32_t* col_ind, const void* values, const int32_t* perm,
    int32_t* out_row_ptr, int32_t* out_col_ind, void* out_values);
xspmm_status_t xspmm_permute_rows_bf16_i64(xspmm_handle_t h, int64_t M, int64_t K, int64_t nnz,
    const int64_t* row_ptr, const int64_t* col_ind, const void* values, const int64_t* perm,
    int64_t* out_row_ptr, int64_t* out_col_ind, void* out_values);
xspmm_status_t xspmm_permute_rows_f32_i32(xspmm_handle_t h, int32_t M, int32_t K, int32_t nnz,
    const int32_t* row_ptr, const int32_t* col_ind, const void* values, const int32_t* perm,
    int32_t* out_row_ptr, int32_t* out_col_ind, void* out_values);
xspmm_status_t xspmm_permute_rows_f32_i64(xspmm_handle_t h, int64_t M, int64_t K, int64_t nnz,
    const int64_t* row_ptr, const int64_t* col_ind, const void* values, const int64_t* perm,
    int64_t* out_row_ptr, int64_t* out_col_ind, void* out_values);

/* ---------------------------------------------------------------------------------------------
 * CSR row permutation that allocates no device memory. This entry point has no counterpart in the
 * reference. It is for callers that cannot allocate device memory while they run -- for example a
 * serving process whose device memory is fully reserved by its own pool, or code that must not
 * take the device-wide synchronization cudaMalloc/cudaFree can cause. Result, validation and
 * synchronization are those of xspmm_permute_rows_{f16,f32}_i32; value_bytes is 2 (fp16) or 4
 * (fp32), indices are int32.
 * Its scratch is a fixed 270,336-byte array compiled into the library (every GPU that loads the
 * library holds it until exit), so M is limited to 2,097,152 rows; larger M returns
 * INVALID_ARGUMENT. The first call on a device looks up the array's device address, so make that
 * first call before any stream capture; the address is looked up again when the device's context
 * has changed (after cudaDeviceReset), so that call too should come before a capture. All calls
 * on a device share the array: calls that overlap on the GPU race and must be serialized by the
 * caller.
 * ------------------------------------------------------------------------------------------- */
xspmm_status_t xspmm_permute_rows_noalloc_i32(xspmm_handle_t h, int32_t M, int32_t K, int32_t nnz,
    const int32_t* row_ptr, const int32_t* col_ind, const void* values, int32_t value_bytes,
    const int32_t* perm, int32_t* out_row_ptr, int32_t* out_col_ind, void* out_values);

/* ---------------------------------------------------------------------------------------------
 * CSR -> BCSR on the device, in two calls so the caller can allocate the outputs (the reference
 * builds on the host, src/core/conversion.cpp:8-100, and returns a BCSRMatrix:
 * include/xspmm/matrix/conversion.hpp:19-22).
 *   _count: writes bcsr_row_ptr[ceil(M/r_block)+1] and returns the number of blocks in
 *           *num_blocks (synchronizes). Validates the CSR (row_ptr monotone, 0 <= col < K).
 *   _fill:  given that row_ptr, writes col_ind[num_blocks] (ascending per block row) and
 *           values[num_blocks*r_block*c_block] (zero-filled blocks, a duplicate (row,col) keeps
 *           its last value in CSR order -- conversion.cpp:75-91). values may be NULL when only
 *           the structure is wanted.
 * Any r_block, c_block >= 1.
 * ------------------------------------------------------------------------------------------- */
xspmm_status_t xspmm_csr_to_bcsr_count_i32(xspmm_handle_t h, int32_t M, int32_t K, int32_t nnz,
    const int32_t* row_ptr, const int32_t* col_ind, int32_t r_block, int32_t c_block,
    int32_t* bcsr_row_ptr, int64_t* num_blocks);
xspmm_status_t xspmm_csr_to_bcsr_count_i64(xspmm_handle_t h, int64_t M, int64_t K, int64_t nnz,
    const int64_t* row_ptr, const int64_t* col_ind, int64_t r_block, int64_t c_block,
    int64_t* bcsr_row_ptr, int64_t* num_blocks);
xspmm_status_t xspmm_csr_to_bcsr_fill_f16_i32(xspmm_handle_t h, int32_t M, int32_t K, int32_t nnz,
    const int32_t* row_ptr, const int32_t* col_ind, const void* values, int32_t r_block,
    int32_t c_block, const int32_t* bcsr_row_ptr, int32_t* bcsr_col_ind, void* bcsr_values);
xspmm_status_t xspmm_csr_to_bcsr_fill_f16_i64(xspmm_handle_t h, int64_t M, int64_t K, int64_t nnz,
    const int64_t* row_ptr, const int64_t* col_ind, const void* values, int64_t r_block,
    int64_t c_block, const int64_t* bcsr_row_ptr, int64_t* bcsr_col_ind, void* bcsr_values);
xspmm_status_t xspmm_csr_to_bcsr_fill_bf16_i32(xspmm_handle_t h, int32_t M, int32_t K, int32_t nnz,
    const int32_t* row_ptr, const int32_t* col_ind, const void* values, int32_t r_block,
    int32_t c_block, const int32_t* bcsr_row_ptr, int32_t* bcsr_col_ind, void* bcsr_values);
xspmm_status_t xspmm_csr_to_bcsr_fill_bf16_i64(xspmm_handle_t h, int64_t M, int64_t K, int64_t nnz,
    const int64_t* row_ptr, const int64_t* col_ind, const void* values, int64_t r_block,
    int64_t c_block, const int64_t* bcsr_row_ptr, int64_t* bcsr_col_ind, void* bcsr_values);
xspmm_status_t xspmm_csr_to_bcsr_fill_f32_i32(xspmm_handle_t h, int32_t M, int32_t K, int32_t nnz,
    const int32_t* row_ptr, const int32_t* col_ind, const void* values, int32_t r_block,
    int32_t c_block, const int32_t* bcsr_row_ptr, int32_t* bcsr_col_ind, void* bcsr_values);
xspmm_status_t xspmm_csr_to_bcsr_fill_f32_i64(xspmm_handle_t h, int64_t M, int64_t K, int64_t nnz,
    const int64_t* row_ptr, const int64_t* col_ind, const void* values, int64_t r_block,
    int64_t c_block, const int64_t* bcsr_row_ptr, int64_t* bcsr_col_ind, void* bcsr_values);

/* ---------------------------------------------------------------------------------------------
 * Dense unpermute: out[perm[r]*N + c] = in[r*N + c]. Replaces xspmm::unpermute_dense_matrix
 * (include/xspmm/xspmm.hpp:35-40, src/xspmm.cpp:116-134, src/cuda/mtx_permutation.cu:71-85,
 * kernel src/common/permutation.hpp:89-108). in and out must not overlap.
 * ------------------------------------------------------------------------------------------- */
xspmm_status_t xspmm_unpermute_dense_f32_i32(xspmm_handle_t h, const void* in, void* out,
    const int32_t* perm, int32_t M, int32_t N);
xspmm_status_t xspmm_unpermute_dense_f32_i64(xspmm_handle_t h, const void* in, void* out,
    const int64_t* perm, int64_t M, int64_t N);
xspmm_status_t xspmm_unpermute_dense_f16_i32(xspmm_handle_t h, const void* in, void* out,
    const int32_t* perm, int32_t M, int32_t N);
xspmm_status_t xspmm_unpermute_dense_f16_i64(xspmm_handle_t h, const void* in, void* out,
    const int64_t* perm, int64_t M, int64_t N);
xspmm_status_t xspmm_unpermute_dense_bf16_i32(xspmm_handle_t h, const void* in, void* out,
    const int32_t* perm, int32_t M, int32_t N);
xspmm_status_t xspmm_unpermute_dense_bf16_i64(xspmm_handle_t h, const void* in, void* out,
    const int64_t* perm, int64_t M, int64_t N);

/* ---------------------------------------------------------------------------------------------
 * Tier-2 pipeline: C = A * B for A in CSR, with optional clustering. Replaces
 * xspmm::spmm(exec, CSR A, B, C, N, hw_block_size, optimize_pattern, timings)
 * (include/xspmm/xspmm.hpp:24-32, src/xspmm.cpp:137-162, src/cuda/unstructured_mtx_mul.cu:56-130):
 *   enable_clustering != 0: perm = cluster(A, 0.5, hw_block_size); A' = permute(A, perm);
 *   A'' = csr_to_bcsr(A', 16, 16); C[perm[i]] = (A'' * B)[i]  (the unpermute is fused into the
 *   SpMM store, so unpermutation_ms reports 0 and no M x N temporary is allocated).
 *   enable_clustering == 0: C = csr_to_bcsr(A) * B.
 * hw_block_size (>= 1) is the clustering's column block width, as in the reference; the product
 * always runs on 16 x 16 blocks, so C = A * B for every width (the reference converts to
 * hw x hw blocks, :102, and reads them as 16 x 16, so its C is wrong for hw != 16). timings may
 * be NULL; when given, the call
 * synchronizes at the end of every stage to read its events, like the reference
 * (src/cuda/unstructured_mtx_mul.cu:14-26).
 * ------------------------------------------------------------------------------------------- */
xspmm_status_t xspmm_spmm_csr_f16f32_i32(xspmm_handle_t h, int32_t M, int32_t K, int32_t nnz,
    const int32_t* row_ptr, const int32_t* col_ind, const void* values, const void* B, float* C,
    int32_t N, int32_t hw_block_size, int enable_clustering, xspmm_timings_t* timings);
xspmm_status_t xspmm_spmm_csr_f16f32_i64(xspmm_handle_t h, int64_t M, int64_t K, int64_t nnz,
    const int64_t* row_ptr, const int64_t* col_ind, const void* values, const void* B, float* C,
    int64_t N, int64_t hw_block_size, int enable_clustering, xspmm_timings_t* timings);
xspmm_status_t xspmm_spmm_csr_bf16f32_i32(xspmm_handle_t h, int32_t M, int32_t K, int32_t nnz,
    const int32_t* row_ptr, const int32_t* col_ind, const void* values, const void* B, float* C,
    int32_t N, int32_t hw_block_size, int enable_clustering, xspmm_timings_t* timings);
xspmm_status_t xspmm_spmm_csr_bf16f32_i64(xspmm_handle_t h, int64_t M, int64_t K, int64_t nnz,
    const int64_t* row_ptr, const int64_t* col_ind, const void* values, const void* B, float* C,
    int64_t N, int64_t hw_block_size, int enable_clustering, xspmm_timings_t* timings);
xspmm_status_t xspmm_spmm_csr_f32f32_i32(xspmm_handle_t h, int32_t M, int32_t K, int32_t nnz,
    const int32_t* row_ptr, const int32_t* col_ind, const void* values, const void* B, float* C,
    int32_t N, int32_t hw_block_size, int enable_clustering, xspmm_timings_t* timings);
xspmm_status_t xspmm_spmm_csr_f32f32_i64(xspmm_handle_t h, int64_t M, int64_t K, int64_t nnz,
    const int64_t* row_ptr, const int64_t* col_ind, const void* values, const void* B, float* C,
    int64_t N, int64_t hw_block_size, int enable_clustering, xspmm_timings_t* timings);

/* ---------------------------------------------------------------------------------------------
 * Plan: the Tier-2 stages run once, many products afterwards. The reference has no object for
 * this; its Tier-2 call repeats clustering, permutation and conversion every time
 * (src/cuda/unstructured_mtx_mul.cu:56-130) and it points callers who multiply one A by many B
 * to Tier 1 "for amortizing clustering time over thousands of iterations" (README.md:127). A plan
 * is that amortization done inside the library: it keeps the permutation, the permuted BCSR
 * matrix and, where the tcgen05 kernel is chosen, A's stacked tensor-core tiles on the device.
 *
 * xspmm_plan_csr_*: the stages of xspmm_spmm_csr_* up to and including CSR->BCSR, with the same
 *   arguments (any hw_block_size >= 1). build_timings (may be NULL) receives clustering_ms,
 *   permutation_ms and conversion_ms (CSR->BCSR plus the tensor-core tile packing); spmm_ms and
 *   unpermutation_ms are 0. The caller's CSR arrays may be freed once the call returns.
 * xspmm_plan_bcsr_*: adopts a BCSR matrix of 16 x 16 blocks (other shapes: UNSUPPORTED; call
 *   xspmm_bcsr_spmm_* for them) for Tier-1 products (the arguments of xspmm_bcsr_spmm_*). The
 *   plan READS the caller's arrays at every product: keep them alive and unchanged until
 *   xspmm_plan_destroy.
 * xspmm_plan_execute: C (M x N, fp32, row-major, rows in the caller's order) = A * B, B (K x N,
 *   row-major) of the plan's value type. Asynchronous on the handle's stream. Results equal
 *   xspmm_spmm_csr_* / xspmm_bcsr_spmm_* on the same inputs and kernel choice.
 * Plans belong to the handle they were built on and use its stream and kernel setting;
 * xspmm_destroy fails with INVALID_ARGUMENT while any of its plans is alive.
 * ------------------------------------------------------------------------------------------- */
typedef struct xspmm_plan_s* xspmm_plan_t;

typedef struct xspmm_plan_info {
    int64_t rows, cols;                           /* M, K */
    int64_t block_rows, block_cols, nnz_blocks;   /* the 16 x 16 BCSR matrix */
    int32_t clustered;                            /* rows permuted by the clustering */
    int32_t value_bytes;                          /* 2 (f16, bf16) or 4 (f32) */
    int32_t tcgen05_ready;                        /* stacked tiles for the tcgen05 kernel built */
    int32_t reserved;
    int64_t tcgen05_tiles;                        /* 128 x 16 tiles packed for it */
    int64_t device_bytes;                         /* device memory the plan owns */
} xspmm_plan_info_t;

xspmm_status_t xspmm_plan_csr_f16f32_i32(xspmm_handle_t h, int32_t M, int32_t K, int32_t nnz,
    const int32_t* row_ptr, const int32_t* col_ind, const void* values, int32_t hw_block_size,
    int enable_clustering, xspmm_plan_t* out, xspmm_timings_t* build_timings);
xspmm_status_t xspmm_plan_csr_f16f32_i64(xspmm_handle_t h, int64_t M, int64_t K, int64_t nnz,
    const int64_t* row_ptr, const int64_t* col_ind, const void* values, int64_t hw_block_size,
    int enable_clustering, xspmm_plan_t* out, xspmm_timings_t* build_timings);
xspmm_status_t xspmm_plan_csr_bf16f32_i32(xspmm_handle_t h, int32_t M, int32_t K, int32_t nnz,
    const int32_t* row_ptr, const int32_t* col_ind, const void* values, int32_t hw_block_size,
    int enable_clustering, xspmm_plan_t* out, xspmm_timings_t* build_timings);
xspmm_status_t xspmm_plan_csr_bf16f32_i64(xspmm_handle_t h, int64_t M, int64_t K, int64_t nnz,
    const int64_t* row_ptr, const int64_t* col_ind, const void* values, int64_t hw_block_size,
    int enable_clustering, xspmm_plan_t* out, xspmm_timings_t* build_timings);
xspmm_status_t xspmm_plan_csr_f32f32_i32(xspmm_handle_t h, int32_t M, int32_t K, int32_t nnz,
    const int32_t* row_ptr, const int32_t* col_ind, const void* values, int32_t hw_block_size,
    int enable_clustering, xspmm_plan_t* out, xspmm_timings_t* build_timings);
xspmm_status_t xspmm_plan_csr_f32f32_i64(xspmm_handle_t h, int64_t M, int64_t K, int64_t nnz,
    const int64_t* row_ptr, const int64_t* col_ind, const void* values, int64_t hw_block_size,
    int enable_clustering, xspmm_plan_t* out, xspmm_timings_t* build_timings);
xspmm_status_t xspmm_plan_bcsr_f16f32_i32(xspmm_handle_t h, int32_t nbr, int32_t nbc,
    int32_t nnzb, int32_t r_block, int32_t c_block, const int32_t* row_ptr, const int32_t* col_ind,
    const void* values, int32_t M, int32_t K, xspmm_plan_t* out);
xspmm_status_t xspmm_plan_bcsr_f16f32_i64(xspmm_handle_t h, int64_t nbr, int64_t nbc,
    int64_t nnzb, int64_t r_block, int64_t c_block, const int64_t* row_ptr, const int64_t* col_ind,
    const void* values, int64_t M, int64_t K, xspmm_plan_t* out);
xspmm_status_t xspmm_plan_bcsr_bf16f32_i32(xspmm_handle_t h, int32_t nbr, int32_t nbc,
    int32_t nnzb, int32_t r_block, int32_t c_block, const int32_t* row_ptr, const int32_t* col_ind,
    const void* values, int32_t M, int32_t K, xspmm_plan_t* out);
xspmm_status_t xspmm_plan_bcsr_bf16f32_i64(xspmm_handle_t h, int64_t nbr, int64_t nbc,
    int64_t nnzb, int64_t r_block, int64_t c_block, const int64_t* row_ptr, const int64_t* col_ind,
    const void* values, int64_t M, int64_t K, xspmm_plan_t* out);
xspmm_status_t xspmm_plan_bcsr_f32f32_i32(xspmm_handle_t h, int32_t nbr, int32_t nbc,
    int32_t nnzb, int32_t r_block, int32_t c_block, const int32_t* row_ptr, const int32_t* col_ind,
    const void* values, int32_t M, int32_t K, xspmm_plan_t* out);
xspmm_status_t xspmm_plan_bcsr_f32f32_i64(xspmm_handle_t h, int64_t nbr, int64_t nbc,
    int64_t nnzb, int64_t r_block, int64_t c_block, const int64_t* row_ptr, const int64_t* col_ind,
    const void* values, int64_t M, int64_t K, xspmm_plan_t* out);
xspmm_status_t xspmm_plan_execute(xspmm_plan_t plan, const void* B, float* C, int64_t N);
xspmm_status_t xspmm_plan_get_info(xspmm_plan_t plan, xspmm_plan_info_t* info);
xspmm_status_t xspmm_plan_destroy(xspmm_plan_t plan);

/* ---------------------------------------------------------------------------------------------
 * Multi-GPU: one matrix split by block rows over an NCCL communicator (one process or thread per
 * GPU). The reference runs on one device only; these entries replace a caller's loop of Tier-1
 * calls (xspmm::spmm(const BCSRMatrix&, B, C, N), include/xspmm/xspmm.hpp:14-18, launched in
 * src/cuda/unstructured_mtx_mul.cu:31-51) over block-row slices, with the Tier-2 preparation
 * (src/cuda/unstructured_mtx_mul.cu:56-130) done once per rank and the reference's unpermute
 * (src/cuda/mtx_permutation.cu:71-85) applied when C is gathered.
 *
 * xspmm_dist_unique_id: a new communicator's id (id_bytes >= 128), made on one rank and handed to
 *   the others by the caller (a file, a socket, MPI, torch.distributed...).
 * xspmm_dist_comm_init: joins the communicator on the handle's device (NCCL, non-blocking init).
 *   It waits at most timeout_ms (<= 0: 60 s) for every rank to join: a rank that never joins gives
 *   TIMEOUT, an NCCL failure NCCL_ERROR; the communicator is aborted in both cases.
 * xspmm_dist_comm_wrap: uses an ncclComm_t the caller created (NCCL 2.27+; not destroyed here).
 * xspmm_dist_plan_csr_*: every rank passes the whole CSR A on its own device (as for
 *   xspmm_plan_csr_*). Each rank clusters (deterministic: the same permutation everywhere),
 *   counts the permuted matrix's 16 x 16 blocks, splits the block rows into nranks contiguous
 *   ranges balanced by nonzero blocks plus row_weight per block row, and builds the BCSR of its
 *   own range only. The CSR may be freed once the call returns. Synchronizes.
 * xspmm_dist_plan_execute: C_local (rows [row_begin, row_end) of the clustered matrix, N
 *   columns, fp32) = this rank's rows of A * B. With bcast_root >= 0, B (K x N, every rank's own
 *   buffer) is first broadcast in place from that rank (waits for it, within timeout_ms); with
 *   bcast_root < 0, B must already hold the same values on every rank. The product is
 *   asynchronous on the handle's stream.
 * xspmm_dist_gather: the root receives every rank's C_local and writes C (M x N, fp32, the
 *   caller's row order); the other ranks send theirs (C may be NULL there). Synchronous, within
 *   timeout_ms. Every rank of the communicator must make the same execute / gather calls in the
 *   same order.
 * A timeout aborts the communicator (TIMEOUT); any NCCL error too (NCCL_ERROR); after that every
 * call on it or its plans returns NCCL_ERROR. hw_block_size: as for xspmm_spmm_csr_*.
 * ------------------------------------------------------------------------------------------- */
typedef struct xspmm_dist_comm_s* xspmm_dist_comm_t;
typedef struct xspmm_dist_plan_s* xspmm_dist_plan_t;

typedef struct xspmm_dist_plan_info {
    int64_t rows, cols;                   /* M, K of the whole matrix */
    int64_t row_begin, row_end;           /* this rank's rows of the clustered matrix */
    int64_t block_begin, block_end;       /* this rank's block rows */
    int64_t nnz_blocks, nnz_blocks_total; /* blocks held by this rank, by all ranks */
    int32_t clustered, value_bytes;
    int64_t device_bytes;                 /* device memory this rank's plan owns */
} xspmm_dist_plan_info_t;

/* The block-row split of xspmm_dist_plan_csr_* (host only, no device work): bounds[0..parts]
 * with bounds[0] = 0, bounds[parts] = nbr; range p is the first block row whose prefix of
 * nonzero blocks plus row_weight per block row reaches p / parts of the total. */
xspmm_status_t xspmm_dist_partition(const int64_t* bcsr_row_ptr, int64_t nbr, int32_t parts,
    double row_weight, int64_t* bounds);
xspmm_status_t xspmm_dist_unique_id(unsigned char* id, int32_t id_bytes);
xspmm_status_t xspmm_dist_comm_init(xspmm_handle_t h, int32_t nranks, int32_t rank,
    const unsigned char* id, int32_t id_bytes, int32_t timeout_ms, xspmm_dist_comm_t* comm);
xspmm_status_t xspmm_dist_comm_wrap(void* nccl_comm, int32_t device, xspmm_dist_comm_t* comm);
xspmm_status_t xspmm_dist_comm_destroy(xspmm_dist_comm_t comm);
xspmm_status_t xspmm_dist_plan_csr_f16f32_i32(xspmm_handle_t h, xspmm_dist_comm_t comm, int32_t M,
    int32_t K, int32_t nnz, const int32_t* row_ptr, const int32_t* col_ind, const void* values,
    int32_t hw_block_size, int enable_clustering, double row_weight, xspmm_dist_plan_t* out);
xspmm_status_t xspmm_dist_plan_csr_f16f32_i64(xspmm_handle_t h, xspmm_dist_comm_t comm, int64_t M,
    int64_t K, int64_t nnz, const int64_t* row_ptr, const int64_t* col_ind, const void* values,
    int64_t hw_block_size, int enable_clustering, double row_weight, xspmm_dist_plan_t* out);
xspmm_status_t xspmm_dist_plan_csr_bf16f32_i32(xspmm_handle_t h, xspmm_dist_comm_t comm, int32_t M,
    int32_t K, int32_t nnz, const int32_t* row_ptr, const int32_t* col_ind, const void* values,
    int32_t hw_block_size, int enable_clustering, double row_weight, xspmm_dist_plan_t* out);
xspmm_status_t xspmm_dist_plan_csr_bf16f32_i64(xspmm_handle_t h, xspmm_dist_comm_t comm, int64_t M,
    int64_t K, int64_t nnz, const int64_t* row_ptr, const int64_t* col_ind, const void* values,
    int64_t hw_block_size, int enable_clustering, double row_weight, xspmm_dist_plan_t* out);
xspmm_status_t xspmm_dist_plan_csr_f32f32_i32(xspmm_handle_t h, xspmm_dist_comm_t comm, int32_t M,
    int32_t K, int32_t nnz, const int32_t* row_ptr, const int32_t* col_ind, const void* values,
    int32_t hw_block_size, int enable_clustering, double row_weight, xspmm_dist_plan_t* out);
xspmm_status_t xspmm_dist_plan_csr_f32f32_i64(xspmm_handle_t h, xspmm_dist_comm_t comm, int64_t M,
    int64_t K, int64_t nnz, const int64_t* row_ptr, const int64_t* col_ind, const void* values,
    int64_t hw_block_size, int enable_clustering, double row_weight, xspmm_dist_plan_t* out);
xspmm_status_t xspmm_dist_plan_get_info(xspmm_dist_plan_t plan, xspmm_dist_plan_info_t* info);
xspmm_status_t xspmm_dist_plan_execute(xspmm_dist_plan_t plan, void* B, float* C_local, int64_t N,
    int32_t bcast_root, int32_t timeout_ms);
xspmm_status_t xspmm_dist_gather(xspmm_dist_plan_t plan, const float* C_local, float* C,
    int64_t N, int32_t root, int32_t timeout_ms);
xspmm_status_t xspmm_dist_plan_destroy(xspmm_dist_plan_t plan);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* XSPMM_B200_H */
