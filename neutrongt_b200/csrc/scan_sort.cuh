// Device-wide exclusive scan and stable LSD radix sort of (u32 key, u32 value) pairs.
// Both run on caller-provided workspace and allocate nothing.
#pragma once

#include "common.cuh"

namespace ngt {
// internal linkage: every translation unit that sorts gets its own copy of these kernels
namespace {

// ------------------------------------------------------------------------------------
// exclusive scan: out[i] = sum_{j<i} in[i]   (in may equal out)
// ------------------------------------------------------------------------------------
constexpr int kScanThreads = 512;
constexpr int kScanItems = 8;
constexpr int kScanTile = kScanThreads * kScanItems;

template <typename T>
__device__ __forceinline__ T block_exclusive_scan(T x, T *total) {
    __shared__ T warp_tot[33];  // [0, 32): per-warp exclusive prefix, [32]: block total
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    T inc = x;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        T y = __shfl_up_sync(0xffffffffu, inc, off);
        if (lane >= off) inc += y;
    }
    if (lane == 31) warp_tot[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        T w = lane < nw ? warp_tot[lane] : T(0);
        T winc = w;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            T y = __shfl_up_sync(0xffffffffu, winc, off);
            if (lane >= off) winc += y;
        }
        if (lane < nw) warp_tot[lane] = winc - w;
        if (lane == nw - 1) warp_tot[32] = winc;
    }
    __syncthreads();
    const T res = inc - x + warp_tot[warp];
    if (total) *total = warp_tot[32];
    __syncthreads();
    return res;
}

template <typename T>
__global__ void __launch_bounds__(kScanThreads) scan_block_sums(const T *in, int64_t n, T *partials) {
    const int64_t base = (int64_t)blockIdx.x * kScanTile + (int64_t)threadIdx.x * kScanItems;
    T s = 0;
#pragma unroll
    for (int i = 0; i < kScanItems; i++)
        if (base + i < n) s += in[base + i];
    T tot;
    block_exclusive_scan<T>(s, &tot);
    if (threadIdx.x == 0) partials[blockIdx.x] = tot;
}

template <typename T>
__global__ void __launch_bounds__(kScanThreads) scan_partials(T *partials, int64_t m) {
    T carry = 0;
    for (int64_t b = 0; b < m; b += kScanThreads) {
        const int64_t i = b + threadIdx.x;
        const T x = i < m ? partials[i] : T(0);
        T tot;
        const T ex = block_exclusive_scan<T>(x, &tot);
        if (i < m) partials[i] = ex + carry;
        carry += tot;
    }
}

template <typename T>
__global__ void __launch_bounds__(kScanThreads)
    scan_apply(const T *in, T *out, int64_t n, const T *partials) {
    const int64_t base = (int64_t)blockIdx.x * kScanTile + (int64_t)threadIdx.x * kScanItems;
    T v[kScanItems];
    T s = 0;
#pragma unroll
    for (int i = 0; i < kScanItems; i++) {
        v[i] = (base + i < n) ? in[base + i] : T(0);
        s += v[i];
    }
    T ex = block_exclusive_scan<T>(s, nullptr) + partials[blockIdx.x];
#pragma unroll
    for (int i = 0; i < kScanItems; i++) {
        if (base + i < n) out[base + i] = ex;
        ex += v[i];
    }
}

inline int64_t scan_partials_count(int64_t n) { return (n + kScanTile - 1) / kScanTile; }

template <typename T>
int exclusive_scan(const T *in, T *out, int64_t n, T *partials, cudaStream_t st) {
    if (n <= 0) return NGT_OK;
    const int64_t nb = scan_partials_count(n);
    scan_block_sums<T><<<(unsigned)nb, kScanThreads, 0, st>>>(in, n, partials);
    scan_partials<T><<<1, kScanThreads, 0, st>>>(partials, nb);
    scan_apply<T><<<(unsigned)nb, kScanThreads, 0, st>>>(in, out, n, partials);
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}

// ------------------------------------------------------------------------------------
// stable LSD radix sort, 8-bit digits.  A tile is 256 threads x 16 rounds; within a tile
// items are visited in index order (round-major), so equal digits keep input order:
// rank = (same digit in earlier tiles) + (earlier rounds) + (earlier warps this round)
//      + (earlier lanes of this warp).
// ------------------------------------------------------------------------------------
constexpr int kSortThreads = 256;
constexpr int kSortRounds = 16;
constexpr int kSortTile = kSortThreads * kSortRounds;
constexpr int kSortWarps = kSortThreads / 32;

inline int64_t radix_tiles(int64_t n) { return (n + kSortTile - 1) / kSortTile; }

__global__ void __launch_bounds__(kSortThreads)
    radix_upsweep(const uint32_t *keys, int64_t n, int shift, int64_t ntiles, uint32_t *hist) {
    __shared__ uint32_t h[256];
    h[threadIdx.x] = 0;
    __syncthreads();
    const int64_t base = (int64_t)blockIdx.x * kSortTile;
#pragma unroll 4
    for (int r = 0; r < kSortRounds; r++) {
        const int64_t i = base + (int64_t)r * kSortThreads + threadIdx.x;
        if (i < n) atomicAdd(&h[(keys[i] >> shift) & 255u], 1u);
    }
    __syncthreads();
    hist[(int64_t)threadIdx.x * ntiles + blockIdx.x] = h[threadIdx.x];
}

__global__ void __launch_bounds__(kSortThreads)
    radix_downsweep(const uint32_t *keys_in, const uint32_t *vals_in, uint32_t *keys_out,
                    uint32_t *vals_out, int64_t n, int shift, int64_t ntiles,
                    const uint32_t *offsets) {
    __shared__ uint32_t run[256];
    __shared__ uint32_t wcnt[kSortWarps][256];
    __shared__ uint32_t base_off[256];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    run[tid] = 0;
    base_off[tid] = offsets[(int64_t)tid * ntiles + blockIdx.x];
    const int64_t base = (int64_t)blockIdx.x * kSortTile;
    const uint32_t lt_mask = (1u << lane) - 1u;
    for (int r = 0; r < kSortRounds; r++) {
#pragma unroll
        for (int w = 0; w < kSortWarps; w++) wcnt[w][tid] = 0;
        __syncthreads();
        const int64_t i = base + (int64_t)r * kSortThreads + tid;
        const bool valid = i < n;
        const uint32_t key = valid ? keys_in[i] : 0u;
        const uint32_t digit = (key >> shift) & 255u;
        // invalid lanes get a private tag (>= 256) so they never match a real digit
        const uint32_t tag = valid ? digit : 256u + (uint32_t)lane;
        const uint32_t peers = __match_any_sync(0xffffffffu, tag);
        const uint32_t rank_w = __popc(peers & lt_mask);
        if (valid && rank_w == 0) wcnt[warp][digit] = __popc(peers);
        __syncthreads();
        if (valid) {
            uint32_t pre = 0;
            for (int w = 0; w < warp; w++) pre += wcnt[w][digit];
            const uint32_t pos = base_off[digit] + run[digit] + pre + rank_w;
            keys_out[pos] = key;
            vals_out[pos] = vals_in[i];
        }
        __syncthreads();
        uint32_t add = 0;
#pragma unroll
        for (int w = 0; w < kSortWarps; w++) add += wcnt[w][tid];
        run[tid] += add;
        __syncthreads();
    }
}

// Sorts (keys, vals) by the low `bits` bits of the key, stably.  Buffers ping-pong between
// *_a and *_b; the return value says where the result is (0: *_a, 1: *_b).
// hist must hold 256 * radix_tiles(n) u32 and partials scan_partials_count(that) u32.
inline int radix_sort_pairs(uint32_t *keys_a, uint32_t *vals_a, uint32_t *keys_b, uint32_t *vals_b,
                            int64_t n, int bits, uint32_t *hist, uint32_t *partials,
                            cudaStream_t st, int *where) {
    *where = 0;
    if (n <= 1) return NGT_OK;
    const int64_t ntiles = radix_tiles(n);
    uint32_t *ki = keys_a, *vi = vals_a, *ko = keys_b, *vo = vals_b;
    for (int shift = 0; shift < bits; shift += 8) {
        radix_upsweep<<<(unsigned)ntiles, kSortThreads, 0, st>>>(ki, n, shift, ntiles, hist);
        int rc = exclusive_scan<uint32_t>(hist, hist, 256 * ntiles, partials, st);
        if (rc != NGT_OK) return rc;
        radix_downsweep<<<(unsigned)ntiles, kSortThreads, 0, st>>>(ki, vi, ko, vo, n, shift, ntiles, hist);
        NGT_CHECK_LAUNCH();
        uint32_t *t;
        t = ki; ki = ko; ko = t;
        t = vi; vi = vo; vo = t;
        *where ^= 1;
    }
    return NGT_OK;
}

inline int bits_for(int64_t max_key) {
    int b = 0;
    while (b < 32 && (max_key >> b) > 0) b++;
    return b;
}

// Workspace carving: successive 256-byte aligned slices.
struct Carver {
    char *p;
    size_t used = 0, cap;
    Carver(void *base, size_t cap_) : p(static_cast<char *>(base)), cap(cap_) {}
    template <typename T>
    T *take(int64_t count) {
        const size_t off = (used + 255) & ~size_t(255);
        used = off + sizeof(T) * (size_t)(count > 0 ? count : 0);
        return reinterpret_cast<T *>(p ? p + off : nullptr);
    }
};

}  // namespace
}  // namespace ngt
