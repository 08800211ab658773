// Helpers shared by the quantizer and fused-operator kernels: typed 16-element row segments, scale
// loads / stores in the caller's scale dtype, the two division flavours, FP8 packing.
#pragma once

#include "common.cuh"

namespace {

constexpr float kScaleMinThres = 1e-10f;   // SCALE_MIN_THRES, coat/activation/real_quantization/common.py:20

template <bool IEEE>
__device__ __forceinline__ float qdiv(float a, float b) {
    return IEEE ? __fdiv_rn(a, b) : coat_div_full(a, b);
}

// ---- typed 16-element row segments -------------------------------------------------------------
template <typename T> struct Seg16;
template <> struct Seg16<__nv_bfloat16> {
    static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&x)[16]) {
        const uint4 a = reinterpret_cast<const uint4*>(p)[0], b = reinterpret_cast<const uint4*>(p)[1];
        const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            x[2 * i] = __uint_as_float(w[i] << 16);
            x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
    }
    static __device__ __forceinline__ void load4(const __nv_bfloat16* p, float (&x)[4]) {
        const uint2 a = *reinterpret_cast<const uint2*>(p);
        x[0] = __uint_as_float(a.x << 16); x[1] = __uint_as_float(a.x & 0xffff0000u);
        x[2] = __uint_as_float(a.y << 16); x[3] = __uint_as_float(a.y & 0xffff0000u);
    }
    static __device__ __forceinline__ float get(const __nv_bfloat16* p) { return __bfloat162float(*p); }
};
template <> struct Seg16<__half> {
    static __device__ __forceinline__ void load(const __half* p, float (&x)[16]) {
        const uint4 a = reinterpret_cast<const uint4*>(p)[0], b = reinterpret_cast<const uint4*>(p)[1];
        const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
            x[2 * i] = f.x; x[2 * i + 1] = f.y;
        }
    }
    static __device__ __forceinline__ void load4(const __half* p, float (&x)[4]) {
        const uint2 a = *reinterpret_cast<const uint2*>(p);
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&a.x));
        const float2 g = __half22float2(*reinterpret_cast<const __half2*>(&a.y));
        x[0] = f.x; x[1] = f.y; x[2] = g.x; x[3] = g.y;
    }
    static __device__ __forceinline__ float get(const __half* p) { return __half2float(*p); }
};
template <> struct Seg16<float> {
    static __device__ __forceinline__ void load(const float* p, float (&x)[16]) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 a = reinterpret_cast<const float4*>(p)[i];
            x[4 * i] = a.x; x[4 * i + 1] = a.y; x[4 * i + 2] = a.z; x[4 * i + 3] = a.w;
        }
    }
    static __device__ __forceinline__ void load4(const float* p, float (&x)[4]) {
        const float4 a = *reinterpret_cast<const float4*>(p);
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    }
    static __device__ __forceinline__ float get(const float* p) { return *p; }
};

// scale stores / loads in the caller's scale dtype (COAT_F32 / COAT_BF16 / COAT_F16)
__device__ __forceinline__ void store_scale(void* base, int64_t idx, int dtype, float s) {
    if (dtype == COAT_F32) reinterpret_cast<float*>(base)[idx] = s;
    else if (dtype == COAT_BF16) reinterpret_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(s);
    else reinterpret_cast<__half*>(base)[idx] = __float2half_rn(s);
}
__device__ __forceinline__ float load_scale(const void* base, int64_t idx, int dtype) {
    if (dtype == COAT_F32) return reinterpret_cast<const float*>(base)[idx];
    if (dtype == COAT_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[idx]);
    return __half2float(reinterpret_cast<const __half*>(base)[idx]);
}
__device__ __forceinline__ float round_to_dtype(float s, int dtype) {
    if (dtype == COAT_F32) return s;
    if (dtype == COAT_BF16) return __bfloat162float(__float2bfloat16_rn(s));
    return __half2float(__float2half_rn(s));
}

template <int FMT>
__device__ __forceinline__ uint4 pack16(const float (&q)[16]) {
    uint4 r;
    r.x = coat_float4_to_fp8x4<FMT>(q[0], q[1], q[2], q[3]);
    r.y = coat_float4_to_fp8x4<FMT>(q[4], q[5], q[6], q[7]);
    r.z = coat_float4_to_fp8x4<FMT>(q[8], q[9], q[10], q[11]);
    r.w = coat_float4_to_fp8x4<FMT>(q[12], q[13], q[14], q[15]);
    return r;
}

// max over the `lanes` (power of two <= 8) neighbouring lanes that share a group
__device__ __forceinline__ float subgroup_max(float v, int lanes) {
    for (int o = 1; o < lanes; o <<= 1) v = fmaxf(v, __shfl_xor_sync(COAT_FULL_MASK, v, o));
    return v;
}

constexpr int kStraightThreads = 256;

inline int straight_grid(int64_t segs) {
    const int64_t blocks = (segs + kStraightThreads - 1) / kStraightThreads;
    const int64_t cap = (int64_t)coat_sm_count() * 16;   // persistent beyond 16 CTAs of 256 threads per SM
    return (int)(blocks < 1 ? 1 : (blocks < cap ? blocks : cap));
}


}  // namespace
