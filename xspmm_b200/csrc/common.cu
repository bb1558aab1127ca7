// common.cu -- error plumbing, device error word, SM count cache, device-wide exclusive scan.
#include "common.cuh"

#include <mutex>
#include <vector>

namespace xspmm_b200 {

static thread_local std::string g_last_error;

void set_last_error(const std::string& msg) { g_last_error = msg; }
const char* last_error_cstr() { return g_last_error.c_str(); }

unsigned read_device_errors(Handle& h) {
    XS_CHECK_CUDA(cudaMemcpyAsync(h.h_err, h.d_err, sizeof(unsigned), cudaMemcpyDeviceToHost,
                                  h.stream));
    XS_CHECK_CUDA(cudaStreamSynchronize(h.stream));
    unsigned e = *h.h_err;
    if (e) XS_CHECK_CUDA(cudaMemsetAsync(h.d_err, 0, sizeof(unsigned), h.stream));
    return e;
}

void throw_on_device_errors(Handle& h, const char* stage) {
    unsigned e = read_device_errors(h);
    if (!e) return;
    std::string m = std::string(stage) + ":";
    if (e & DERR_COL_OUT_OF_RANGE) m += " column index outside [0, K);";
    if (e & DERR_ROW_PTR) m += " row_ptr not monotone or outside [0, nnz];";
    if (e & DERR_PERM_OUT_OF_RANGE) m += " permutation entry outside [0, M) or not a permutation;";
    if (e & DERR_CAPACITY) m += " internal capacity exceeded;";
    if (e & DERR_INTERNAL) m += " internal consistency check failed;";
    if (e & DERR_TIMEOUT) m += " a bounded wait inside a kernel timed out;";
    xspmm_status_t s = (e & DERR_TIMEOUT) ? XSPMM_STATUS_TIMEOUT
                       : (e & (DERR_INTERNAL | DERR_CAPACITY)) ? XSPMM_STATUS_INTERNAL
                                                               : XSPMM_STATUS_INVALID_ARGUMENT;
    throw Error(s, m);
}

int sm_count(int device) {
    static std::mutex mu;
    static std::vector<int> cache;
    std::lock_guard<std::mutex> lk(mu);
    if ((int)cache.size() <= device) cache.resize(device + 1, 0);
    if (!cache[device]) {
        int v = 0;
        XS_CHECK_CUDA(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device));
        cache[device] = v;
    }
    return cache[device];
}

// ------------------------------------------------------------------------------------------------
// Exclusive scan. A tile is SCAN_THREADS * SCAN_ITEMS consecutive values; phase 1 reduces every
// tile to a partial, the partials are scanned recursively, phase 2 rescans each tile with its
// offset. The last tile also writes the total to out[n].
// ------------------------------------------------------------------------------------------------
constexpr int SCAN_THREADS = 256;
constexpr int SCAN_ITEMS = 8;
constexpr int64_t SCAN_TILE = SCAN_THREADS * SCAN_ITEMS;

template <typename T>
__device__ T block_exclusive_scan(T v, T* warp_sums, T* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    T inc = warp_inclusive_sum(v);
    if (lane == 31) warp_sums[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        T w = lane < SCAN_THREADS / 32 ? warp_sums[lane] : T(0);
        T wi = warp_inclusive_sum(w);
        if (lane < SCAN_THREADS / 32) warp_sums[lane] = wi - w;
        if (lane == SCAN_THREADS / 32 - 1) *total = wi;
    }
    __syncthreads();
    T r = warp_sums[warp] + inc - v;
    return r;
}

template <typename T>
__global__ void __launch_bounds__(SCAN_THREADS) scan_reduce_kernel(const T* in, int64_t n,
                                                                   T* partials) {
    __shared__ T warp_sums[SCAN_THREADS / 32];
    __shared__ T total;
    const int64_t base = (int64_t)blockIdx.x * SCAN_TILE + (int64_t)threadIdx.x * SCAN_ITEMS;
    T s = 0;
#pragma unroll
    for (int i = 0; i < SCAN_ITEMS; ++i)
        if (base + i < n) s += in[base + i];
    block_exclusive_scan(s, warp_sums, &total);
    if (threadIdx.x == 0) partials[blockIdx.x] = total;
}

template <typename T>
__global__ void __launch_bounds__(SCAN_THREADS) scan_down_kernel(const T* in, T* out, int64_t n,
                                                                 const T* offsets) {
    __shared__ T warp_sums[SCAN_THREADS / 32];
    __shared__ T total;
    const int64_t base = (int64_t)blockIdx.x * SCAN_TILE + (int64_t)threadIdx.x * SCAN_ITEMS;
    T v[SCAN_ITEMS];
    T s = 0;
#pragma unroll
    for (int i = 0; i < SCAN_ITEMS; ++i) {
        v[i] = base + i < n ? in[base + i] : T(0);
        s += v[i];
    }
    T off = block_exclusive_scan(s, warp_sums, &total) + (offsets ? offsets[blockIdx.x] : T(0));
#pragma unroll
    for (int i = 0; i < SCAN_ITEMS; ++i) {
        if (base + i < n) out[base + i] = off;
        off += v[i];
    }
    if (blockIdx.x == gridDim.x - 1 && threadIdx.x == 0)
        out[n] = (offsets ? offsets[blockIdx.x] : T(0)) + total;
}

template <typename T>
void exclusive_scan(Handle& h, const T* in, T* out, int64_t n) {
    if (n <= 0) {
        XS_CHECK_CUDA(cudaMemsetAsync(out, 0, sizeof(T), h.stream));
        return;
    }
    const int64_t tiles = ceil_div(n, SCAN_TILE);
    if (tiles == 1) {
        scan_down_kernel<T><<<1, SCAN_THREADS, 0, h.stream>>>(in, out, n, nullptr);
        after_launch(h, "scan_down");
        return;
    }
    DevBuf<T> part(tiles + 1, h.stream);
    scan_reduce_kernel<T><<<(unsigned)tiles, SCAN_THREADS, 0, h.stream>>>(in, n, part.get());
    after_launch(h, "scan_reduce");
    exclusive_scan<T>(h, part.get(), part.get(), tiles);
    scan_down_kernel<T><<<(unsigned)tiles, SCAN_THREADS, 0, h.stream>>>(in, out, n, part.get());
    after_launch(h, "scan_down");
}

int64_t scan_scratch_elems(int64_t n) {
    int64_t total = 0;
    while (n > SCAN_TILE) {
        const int64_t tiles = ceil_div(n, SCAN_TILE);
        total += tiles + 1;
        n = tiles;
    }
    return total;
}

template <typename T>
void exclusive_scan_scratch(Handle& h, const T* in, T* out, int64_t n, T* scratch,
                            int64_t scratch_elems) {
    if (n <= 0) {
        XS_CHECK_CUDA(cudaMemsetAsync(out, 0, sizeof(T), h.stream));
        return;
    }
    const int64_t tiles = ceil_div(n, SCAN_TILE);
    if (tiles == 1) {
        scan_down_kernel<T><<<1, SCAN_THREADS, 0, h.stream>>>(in, out, n, nullptr);
        after_launch(h, "scan_down");
        return;
    }
    XS_REQUIRE(scratch_elems >= tiles + 1, XSPMM_STATUS_INVALID_ARGUMENT,
               "scan scratch too small");
    T* part = scratch;
    scan_reduce_kernel<T><<<(unsigned)tiles, SCAN_THREADS, 0, h.stream>>>(in, n, part);
    after_launch(h, "scan_reduce");
    exclusive_scan_scratch<T>(h, part, part, tiles, scratch + tiles + 1,
                              scratch_elems - (tiles + 1));
    scan_down_kernel<T><<<(unsigned)tiles, SCAN_THREADS, 0, h.stream>>>(in, out, n, part);
    after_launch(h, "scan_down");
}

template <typename T>
T read_scalar(Handle& h, const T* dptr) {
    T v{};
    XS_CHECK_CUDA(cudaMemcpyAsync(&v, dptr, sizeof(T), cudaMemcpyDeviceToHost, h.stream));
    XS_CHECK_CUDA(cudaStreamSynchronize(h.stream));
    return v;
}

template void exclusive_scan<int32_t>(Handle&, const int32_t*, int32_t*, int64_t);
template void exclusive_scan<int64_t>(Handle&, const int64_t*, int64_t*, int64_t);
template void exclusive_scan_scratch<int32_t>(Handle&, const int32_t*, int32_t*, int64_t,
                                              int32_t*, int64_t);
template void exclusive_scan_scratch<int64_t>(Handle&, const int64_t*, int64_t*, int64_t,
                                              int64_t*, int64_t);
template int32_t read_scalar<int32_t>(Handle&, const int32_t*);
template int64_t read_scalar<int64_t>(Handle&, const int64_t*);

}  // namespace xspmm_b200
