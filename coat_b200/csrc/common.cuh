// Shared device/host helpers for the coat_b200 kernels (sm_100a only).
#pragma once

#include <cuda.h>
#include <cstdio>
#include <cstdlib>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/coat_b200.h"

#define COAT_WARP 32
#define COAT_FULL_MASK 0xffffffffu

// Number of SMs of the current device, cached per process (B200: 148).
int coat_sm_count();

// COAT_B200_DEBUG=1 in the environment prints CUDA's own message for a failed launch to stderr.
static inline int coat_launch_status() {
    const cudaError_t err = cudaGetLastError();
    if (err == cudaSuccess) return COAT_OK;
    const char* dbg = getenv("COAT_B200_DEBUG");
    if (dbg && dbg[0] == '1') fprintf(stderr, "coat_b200: launch failed: %s\n", cudaGetErrorString(err));
    return COAT_E_LAUNCH;
}

static inline bool coat_aligned(const void* p, size_t a) {
    return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

// ---- FP8 <-> float ----------------------------------------------------------
// Decoding is exact, so any route gives the same float.  Encoding uses the
// toolkit's conversion intrinsics (round-to-nearest-even, saturate-to-finite),
// the same routine `static_cast<__nv_fp8_e4m3>(float)` resolves to.

__device__ __forceinline__ float coat_e4m3_to_float(uint8_t c) {
    __half_raw h = __nv_cvt_fp8_to_halfraw(c, __NV_E4M3);
    return __half2float(__half(h));
}
__device__ __forceinline__ float coat_e5m2_to_float(uint8_t c) {
    __half_raw h = __nv_cvt_fp8_to_halfraw(c, __NV_E5M2);
    return __half2float(__half(h));
}
template <int FMT>
__device__ __forceinline__ float coat_fp8_to_float(uint8_t c) {
    return FMT == COAT_E4M3 ? coat_e4m3_to_float(c) : coat_e5m2_to_float(c);
}
// Four packed codes (little endian) -> 4 floats.
template <int FMT>
__device__ __forceinline__ void coat_fp8x4_to_float4(uint32_t w, float (&f)[4]) {
    const __nv_fp8_interpretation_t I = FMT == COAT_E4M3 ? __NV_E4M3 : __NV_E5M2;
    __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w & 0xffffu), I);
    __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w >> 16), I);
    float2 a = __half22float2(__half2(lo));
    float2 b = __half22float2(__half2(hi));
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
}
template <int FMT>
__device__ __forceinline__ uint8_t coat_float_to_fp8(float x) {
    return (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, FMT == COAT_E4M3 ? __NV_E4M3 : __NV_E5M2);
}
template <int FMT>
__device__ __forceinline__ uint32_t coat_float4_to_fp8x4(float a, float b, float c, float d) {
    const __nv_fp8_interpretation_t I = FMT == COAT_E4M3 ? __NV_E4M3 : __NV_E5M2;
    uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, I);
    uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, I);
    return lo | (hi << 16);
}

template <int FMT> struct CoatFp8Max;
template <> struct CoatFp8Max<COAT_E4M3> { static constexpr float value = 448.0f; };
template <> struct CoatFp8Max<COAT_E5M2> { static constexpr float value = 57344.0f; };

// ---- bf16 helpers -----------------------------------------------------------
__device__ __forceinline__ float coat_bf16_bits_to_float(uint16_t b) {
    return __uint_as_float(((uint32_t)b) << 16);
}
__device__ __forceinline__ uint16_t coat_float_to_bf16_bits(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// ---- division exactly as the Triton-compiled reference kernels do it --------
// Triton lowers an fp32 `/` (and tl.fdiv) to the PTX instruction div.full.f32
// (not IEEE: max 2 ulp).  The quantizers that must reproduce the reference's
// FP8 codes bit for bit issue the very same instruction.
__device__ __forceinline__ float coat_div_full(float a, float b) {
    float r;
    asm("div.full.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

__device__ __forceinline__ float coat_warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(COAT_FULL_MASK, v, o));
    return v;
}
__device__ __forceinline__ float coat_warp_min(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(COAT_FULL_MASK, v, o));
    return v;
}
