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

// Division of many values by one scale.  For a divisor whose magnitude lies in [2^-120, 2^120],
// div.full.f32(a, b) is bit for bit a * rcp.approx.f32(b) for every finite a (checked on sm_100 over
// 8e9 random operand pairs, divisors from 1e-36 to 1e37; outside that range div.full rescales its
// operands), so the reciprocal is taken once per scale and each element costs one multiplication.
template <bool IEEE>
struct ScaleDivider {
    float s, r;
    bool fast;
    __device__ __forceinline__ explicit ScaleDivider(float scale) : s(scale), r(0.f), fast(false) {
        if (!IEEE) {
            const float a = fabsf(scale);
            fast = a >= 7.5231638e-37f && a <= 1.3292280e36f;
            asm("rcp.approx.f32 %0, %1;" : "=f"(r) : "f"(scale));
        }
    }
    __device__ __forceinline__ float operator()(float x) const {
        if (IEEE) return __fdiv_rn(x, s);
        return fast ? x * r : coat_div_full(x, s);
    }
    template <int N>
    __device__ __forceinline__ void apply(const float (&v)[N], float (&q)[N]) const {
        if (IEEE) {
#pragma unroll
            for (int i = 0; i < N; ++i) q[i] = __fdiv_rn(v[i], s);
        } else if (fast) {
#pragma unroll
            for (int i = 0; i < N; ++i) q[i] = v[i] * r;
        } else {
#pragma unroll
            for (int i = 0; i < N; ++i) q[i] = coat_div_full(v[i], s);
        }
    }
};

// Division by a group scale that the kernel has just computed as (amax + 1e-10) / fp8_max.  Such a scale is
// never below 2e-13 and, for finite inputs, never above 8e35, i.e. always inside the range where
// div.full.f32 equals the multiplication by rcp.approx (and where the flush-to-zero form of the reciprocal
// gives the same bits); for an infinite amax both forms give 0 for finite x and NaN for infinite x.  So no
// range guard is needed, and the reciprocal is a single MUFU instruction.
template <bool IEEE>
struct GroupScaleDivider {
    float s, r;
    __device__ __forceinline__ explicit GroupScaleDivider(float scale) : s(scale), r(0.f) {
        if (!IEEE) asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(scale));
    }
    __device__ __forceinline__ float operator()(float x) const { return IEEE ? __fdiv_rn(x, s) : x * r; }
    // two quotients at once: one two-wide multiplication (each half rounds like the scalar instruction)
    __device__ __forceinline__ float2 pair(float a, float b) const {
        if (IEEE) return make_float2(__fdiv_rn(a, s), __fdiv_rn(b, s));
        return __fmul2_rn(make_float2(a, b), make_float2(r, r));
    }
    template <int N>
    __device__ __forceinline__ void apply(const float (&v)[N], float (&q)[N]) const {
#pragma unroll
        for (int i = 0; i < N; ++i) q[i] = IEEE ? __fdiv_rn(v[i], s) : v[i] * r;
    }
};

// scale = (amax + 1e-10) / fp8_max with the division by the constant hoisted (448 and 57344 are inside the
// range where div.full.f32 is the multiplication by rcp.approx)
template <int FMT, bool IEEE>
struct GroupScale {
    float r;
    __device__ __forceinline__ GroupScale() : r(0.f) {
        if (!IEEE) asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(CoatFp8Max<FMT>::value));
    }
    __device__ __forceinline__ float operator()(float amax) const {
        return IEEE ? __fdiv_rn(amax + kScaleMinThres, CoatFp8Max<FMT>::value) : (amax + kScaleMinThres) * r;
    }
};

// max |x| of 16 values as a balanced tree (depth 4 instead of a chain of 16 dependent maxima)
__device__ __forceinline__ float absmax16(const float (&x)[16]) {
    float m[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i] = fmaxf(fabsf(x[2 * i]), fabsf(x[2 * i + 1]));
#pragma unroll
    for (int i = 0; i < 4; ++i) m[i] = fmaxf(m[2 * i], m[2 * i + 1]);
    return fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
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

// 8 consecutive elements (16 bytes of a 16-bit type, 32 of fp32) as floats
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&x)[8]) {
    const uint4 a = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        x[2 * i] = __uint_as_float(w[i] << 16);
        x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}
__device__ __forceinline__ void load8(const __half* p, float (&x)[8]) {
    const uint4 a = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        x[2 * i] = f.x; x[2 * i + 1] = f.y;
    }
}
__device__ __forceinline__ void load8(const float* p, float (&x)[8]) {
    const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

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

// ---- stochastic rounding of the reference (_division.py:96-150) ---------------------------------------
// Its noise is Triton's tl.rand(0, offset): Philox-4x32 with 10 rounds (Salmon et al., SC'11), key = the two
// words of the seed (0 here), counter = (offset, 0, 0, 0), first output word w mapped to [0, 1) as
// int32 w -> (w >= 0 ? w : -w - 1) * 4.6566127342e-10.
__device__ __forceinline__ float triton_rand_seed0(uint32_t offset) {
    uint32_t c0 = offset, c1 = 0, c2 = 0, c3 = 0, k0 = 0, k1 = 0;
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint32_t a = c0, b = c2;
        c0 = __umulhi(0xCD9E8D57u, b) ^ c1 ^ k0;
        c2 = __umulhi(0xD2511F53u, a) ^ c3 ^ k1;
        c1 = 0xCD9E8D57u * b;
        c3 = 0xD2511F53u * a;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    const int32_t w = (int32_t)c0;
    return __int2float_rn(w < 0 ? -w - 1 : w) * 4.6566127342e-10f;
}

// |q| + noise * (one step of the FP8 format at q's exponent), clamped to q's binade (below the normal range:
// to [smallest subnormal, smallest normal], which also turns zeros into the smallest subnormal, as the
// reference does), with q's sign.  The saturating round-to-nearest cast follows at the caller.
template <int FMT>
__device__ __forceinline__ float stochastic_perturb(float q, float noise) {
    constexpr float kSubMin = FMT == COAT_E4M3 ? 0.001953125f : 1.52587890625e-05f;   // 2^-9, 2^-16
    constexpr float kStep = FMT == COAT_E4M3 ? 0.125f : 0.25f;                         // 2^-m
    constexpr float kSubSpan = FMT == COAT_E4M3 ? 8.f : 4.f;                           // 2^m
    const float e = fmaxf(__uint_as_float(__float_as_uint(q) & 0x7f800000u), kSubMin);
    const bool sub = e == kSubMin;
    const float a = fabsf(q) + __fmul_rn(__fmul_rn(e, noise), sub ? 1.f : kStep);
    return copysignf(fminf(fmaxf(a, e), __fmul_rn(sub ? kSubSpan : 2.f, e)), q);
}

// max over the `lanes` (power of two <= 8) neighbouring lanes that share a group
__device__ __forceinline__ float subgroup_max(float v, int lanes) {
    for (int o = 1; o < lanes; o <<= 1) v = fmaxf(v, __shfl_xor_sync(COAT_FULL_MASK, v, o));
    return v;
}

constexpr int kStraightThreads = 256;

// one thread per 16-element segment, one trip
inline unsigned straight_grid(int64_t segs) {
    const int64_t blocks = (segs + kStraightThreads - 1) / kStraightThreads;
    return (unsigned)(blocks < 1 ? 1 : blocks);
}

// Element offset of 16-element segment `seg` in a matrix of `segs_per_row` segments per row and row stride
// `ld` elements.  Contiguous rows need no division (a 64-bit division costs about as much as the rest of a
// segment's work).
__device__ __forceinline__ int64_t seg_offset(int64_t seg, int64_t segs_per_row, int64_t ld) {
    if (ld == segs_per_row * 16) return seg * 16;
    const int64_t row = seg / segs_per_row;
    return row * ld + (seg - row * segs_per_row) * 16;
}

}  // namespace
