// Shared helpers for the neutrongt_b200 kernels (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/neutrongt_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "neutrongt_b200 is built for sm_100a only"
#endif

namespace ngt {

constexpr int kWarp = 32;

#define NGT_CHECK_LAUNCH()                                   \
    do {                                                     \
        if (cudaGetLastError() != cudaSuccess) return NGT_ERR_CUDA; \
    } while (0)

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int ceil_div_i(int64_t a, int64_t b) { return static_cast<int>((a + b - 1) / b); }

// 16-byte vector of raw bits, loaded through the read-only path.
struct alignas(16) Vec16 {
    uint32_t w[4];
};

__device__ __forceinline__ Vec16 ldg16(const void *p) {
    Vec16 r;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.w[0]), "=r"(r.w[1]), "=r"(r.w[2]), "=r"(r.w[3])
                 : "l"(p));
    return r;
}

__device__ __forceinline__ void st16(void *p, const Vec16 &v) {
    asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.w[0]), "r"(v.w[1]),
                 "r"(v.w[2]), "r"(v.w[3])
                 : "memory");
}

// Element traits: how many elements a 16-byte vector holds and how to unpack/pack them.
template <typename T>
struct Elem;

template <>
struct Elem<float> {
    static constexpr int kPerVec = 4;
    __device__ __forceinline__ static void unpack(const Vec16 &v, float (&f)[4]) {
#pragma unroll
        for (int i = 0; i < 4; i++) f[i] = __uint_as_float(v.w[i]);
    }
    __device__ __forceinline__ static Vec16 pack(const float (&f)[4]) {
        Vec16 v;
#pragma unroll
        for (int i = 0; i < 4; i++) v.w[i] = __float_as_uint(f[i]);
        return v;
    }
    __device__ __forceinline__ static float load1(const float *p) { return __ldg(p); }
    __device__ __forceinline__ static void store1(float *p, float x) { *p = x; }
};

template <>
struct Elem<__nv_bfloat16> {
    static constexpr int kPerVec = 8;
    __device__ __forceinline__ static void unpack(const Vec16 &v, float (&f)[8]) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            f[2 * i] = __uint_as_float(v.w[i] << 16);
            f[2 * i + 1] = __uint_as_float(v.w[i] & 0xffff0000u);
        }
    }
    __device__ __forceinline__ static Vec16 pack(const float (&f)[8]) {
        Vec16 v;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
            v.w[i] = *reinterpret_cast<uint32_t *>(&h);
        }
        return v;
    }
    __device__ __forceinline__ static float load1(const __nv_bfloat16 *p) {
        return __bfloat162float(*p);
    }
    __device__ __forceinline__ static void store1(__nv_bfloat16 *p, float x) {
        *p = __float2bfloat16_rn(x);
    }
};

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }

}  // namespace ngt
