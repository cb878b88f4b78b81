// Device-side helper library prepended to every NVRTC-compiled Metellus kernel.
// Self-contained (NVRTC sees no system headers): fixed-width types, the by-value
// dims block, streaming vector loads/stores and warp/block reductions.
#pragma once

typedef unsigned int uint32_t;
typedef int int32_t;
typedef unsigned long long uint64_t;
typedef long long int64_t;
typedef unsigned long long uintptr_t;
#ifndef MT_SIZE_T_DEFINED
#define MT_SIZE_T_DEFINED
#endif

// Runtime dims block passed by value (replaces the reference's per-dispatch
// uint32 dims buffer). 16 slots cover every strategy.
struct mt_dims { unsigned d[16]; };

#ifndef INFINITY
#define INFINITY __int_as_float(0x7f800000)
#endif
#ifndef NAN
#define NAN __int_as_float(0x7fffffff)
#endif

// Streaming (evict-first) 128-bit load / store for data touched exactly once.
__device__ __forceinline__ float4 mt_ld_stream4(const float* p) {
    float4 v;
    asm("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ float mt_ld_stream(const float* p) {
    float v;
    asm("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ void mt_st_stream4(float* p, float4 v) {
    asm volatile("st.global.L1::no_allocate.v4.f32 [%0], {%1,%2,%3,%4};"
                 :: "l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w) : "memory");
}
__device__ __forceinline__ void mt_st_stream(float* p, float v) {
    asm volatile("st.global.L1::no_allocate.f32 [%0], %1;" :: "l"(p), "f"(v) : "memory");
}
// Read-only cached load for operands re-read by many threads (broadcast rows).
__device__ __forceinline__ float mt_ldg(const float* p) { return __ldg(p); }
__device__ __forceinline__ float4 mt_ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

// Reduction combiners. sum/product use the _rn intrinsics (no FMA contraction);
// max/min follow fmaxf/fminf (NaN-dropping).
struct mt_sum  { __device__ static float id() { return 0.0f; }
                 __device__ static float op(float a, float b) { return __fadd_rn(a, b); } };
struct mt_prod { __device__ static float id() { return 1.0f; }
                 __device__ static float op(float a, float b) { return __fmul_rn(a, b); } };
struct mt_max  { __device__ static float id() { return -INFINITY; }
                 __device__ static float op(float a, float b) { return fmaxf(a, b); } };
struct mt_min  { __device__ static float id() { return INFINITY; }
                 __device__ static float op(float a, float b) { return fminf(a, b); } };

template <class R>
__device__ __forceinline__ float mt_warp_reduce(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = R::op(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide all-reduce; every thread gets the result. `scratch` holds >= 33
// floats of shared memory. Two barriers; safe to call repeatedly with the same
// scratch.
template <class R, int NT>
__device__ __forceinline__ float mt_block_allreduce(float v, float* scratch) {
    constexpr int NW = NT / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = mt_warp_reduce<R>(v);
    if (NW == 1) return __shfl_sync(0xffffffffu, v, 0);
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float r = (lane < NW) ? scratch[lane] : R::id();
    r = mt_warp_reduce<R>(r);
    return r;
}
