// Mixed-granularity FP8 quantizers for sm_100a: per-1xQB-group quantize, the two passes of the
// per-tensor quantize (group scales / global amax, then division by one scale), the fused
// quantize+transpose and division+transpose, byte transpose and dequantize.
//
// Arithmetic follows the reference's Triton kernels statement by statement
//   coat/activation/real_quantization/_quantize.py:74-92            scale = (max|x| + 1e-10) / fp8_max ; q = x / scale
//   coat/activation/real_quantization/_quantize_pertensor.py:80-92  same scale, stored only (pass 1)
//   coat/activation/real_quantization/_division.py:84-114           q = x / s with one scalar s
//   coat/activation/real_quantization/_quantize_transpose.py:84-145 row groups and column groups of one tile
// including the two details that decide the bits: both divisions are the PTX instruction div.full.f32
// (what Triton emits for an fp32 `/` and for tl.fdiv), and the scale is stored rounded to the scale
// dtype AFTER the un-rounded fp32 scale has divided the values.  The float->FP8 cast is round to
// nearest even, saturating (cvt.rn.satfinite), as Triton's.  COAT_QUANT_IEEE_DIV switches both
// divisions to IEEE division, which a CPU can reproduce bit for bit (used by the parity tests).
//
// Layout / mapping: the straight kernels give every thread 16 consecutive elements of a row (two or
// four 16-byte loads, one 16-byte store of codes), so a warp touches 1 KB of contiguous input; groups
// wider than 16 are reduced with shuffles among the QB/16 neighbouring lanes.  The transposing kernels
// give every thread a 4x4 block, a warp a 16(M) x 32(N) patch (lane = 8*mb + nb), so that a 1x16 row
// group is 4 neighbouring lanes (xor 1, 2) and a 16x1 column group is the 4 lanes 8 apart (xor 8, 16);
// the 4x4 byte blocks are transposed in registers and cross a padded shared tile once, so that both the
// straight and the transposed codes leave in 128-byte rows.

#include "quant_common.cuh"
#include "tma.cuh"

namespace {

__device__ int g_quant_device_status = 0;   // COAT_E_TIMEOUT if a bounded wait (a staging copy, the grid barrier) ran out

// =================================================================================================
// 1. per-1xQB-group quantize  (_quantize.py:37-118)  and pass 1 of the per-tensor quantize
//    (_quantize_pertensor.py:46-103): group scales only, plus the tensor's amax for the fused pass 2
// =================================================================================================
// MODE 0: write codes + scales.  MODE 1: write scales (if s != null) and atomically max the tensor amax.
// One 16-element segment per thread and one trip per thread: at 32 bytes loaded per thread the resident
// warps of a full grid already keep HBM busy, and a one-trip grid measured faster than a persistent
// grid-stride loop.  Contiguous rows (ld == N, the usual case) are addressed without any division.
template <typename T, int FMT, bool IEEE, int MODE>
__global__ void __launch_bounds__(kStraightThreads)
group_quantize_kernel(const T* __restrict__ x, uint8_t* __restrict__ y, void* __restrict__ s, int scale_dtype,
                      unsigned int* __restrict__ amax_bits, int64_t M, int64_t N, int64_t ldx, int64_t ldy, int QB) {
    const int64_t segs_per_row = N >> 4;
    const int64_t total = M * segs_per_row;
    const int lanes = QB >> 4;
    const int64_t seg = (int64_t)blockIdx.x * kStraightThreads + threadIdx.x;
    const bool live = seg < total;
    float v[16];
    float amax = 0.f;
    if (live) {
        Seg16<T>::load(x + seg_offset(seg, segs_per_row, ldx), v);
#pragma unroll
        for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
    }
    amax = subgroup_max(amax, lanes);   // whole warps: the grid is rounded up to blocks of 256 threads
    if (live) {
        const float scale = qdiv<IEEE>(amax + kScaleMinThres, CoatFp8Max<FMT>::value);
        if (MODE == 0) {
            float q[16];
            ScaleDivider<IEEE>(scale).apply(v, q);
            *reinterpret_cast<uint4*>(y + seg_offset(seg, segs_per_row, ldy)) = pack16<FMT>(q);
        }
        // N is a multiple of QB, so group g of row r is group r * (N / QB) + g = seg / lanes of the matrix
        if (s && (seg & (lanes - 1)) == 0) store_scale(s, seg >> (31 - __clz(lanes)), scale_dtype, scale);
    }
    if (MODE == 1) {
        float block_max = coat_warp_max(amax);
        __shared__ float wmax[kStraightThreads / 32];
        if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = block_max;
        __syncthreads();
        if (threadIdx.x < 32) {
            float m = threadIdx.x < kStraightThreads / 32 ? wmax[threadIdx.x] : 0.f;
            m = coat_warp_max(m);
            // non-negative floats order like their bit patterns
            if (threadIdx.x == 0) atomicMax(amax_bits, __float_as_uint(m));
        }
    }
}

// Tensor amax alone (pass 1 of a per-tensor quantize when the caller wants no group scales): each thread
// takes four 16-element segments, all loads issued before any is used, and for the 16-bit types the maxima
// are taken on packed pairs without converting to fp32 (max|x| of bf16 values is itself a bf16 value).
template <typename T> __device__ __forceinline__ float seg_absmax(const uint4& a, const uint4& b);
template <> __device__ __forceinline__ float seg_absmax<__nv_bfloat16>(const uint4& a, const uint4& b) {
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    __nv_bfloat162 m[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i] = __habs2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
#pragma unroll
    for (int i = 0; i < 4; ++i) m[i] = __hmax2(m[2 * i], m[2 * i + 1]);
    const __nv_bfloat162 r = __hmax2(__hmax2(m[0], m[1]), __hmax2(m[2], m[3]));
    return fmaxf(__low2float(r), __high2float(r));
}
template <> __device__ __forceinline__ float seg_absmax<__half>(const uint4& a, const uint4& b) {
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    __half2 m[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i] = __habs2(*reinterpret_cast<const __half2*>(&w[i]));
#pragma unroll
    for (int i = 0; i < 4; ++i) m[i] = __hmax2(m[2 * i], m[2 * i + 1]);
    const __half2 r = __hmax2(__hmax2(m[0], m[1]), __hmax2(m[2], m[3]));
    return fmaxf(__low2float(r), __high2float(r));
}

constexpr int kAmaxSegs = 4;
template <typename T>
__global__ void __launch_bounds__(kStraightThreads)
tensor_amax_kernel(const T* __restrict__ x, unsigned int* __restrict__ amax_bits, int64_t M, int64_t N, int64_t ldx) {
    const int64_t segs_per_row = N >> 4;
    const int64_t total = M * segs_per_row;
    const int64_t first = (int64_t)blockIdx.x * (kStraightThreads * kAmaxSegs) + threadIdx.x;
    float amax = 0.f;
    if constexpr (sizeof(T) == 2) {
        uint4 a[kAmaxSegs], b[kAmaxSegs];
#pragma unroll
        for (int k = 0; k < kAmaxSegs; ++k) {
            const int64_t seg = first + k * kStraightThreads;
            if (seg < total) {
                const uint4* p = reinterpret_cast<const uint4*>(x + seg_offset(seg, segs_per_row, ldx));
                a[k] = p[0]; b[k] = p[1];
            } else {
                a[k] = make_uint4(0, 0, 0, 0); b[k] = make_uint4(0, 0, 0, 0);
            }
        }
#pragma unroll
        for (int k = 0; k < kAmaxSegs; ++k) amax = fmaxf(amax, seg_absmax<T>(a[k], b[k]));
    } else {
#pragma unroll
        for (int k = 0; k < kAmaxSegs; ++k) {
            const int64_t seg = first + k * kStraightThreads;
            if (seg < total) {
                float v[16];
                Seg16<T>::load(x + seg_offset(seg, segs_per_row, ldx), v);
                amax = fmaxf(amax, absmax16(v));
            }
        }
    }
    amax = coat_warp_max(amax);
    __shared__ float wmax[kStraightThreads / 32];
    if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = amax;
    __syncthreads();
    if (threadIdx.x < 32) {
        float m = threadIdx.x < kStraightThreads / 32 ? wmax[threadIdx.x] : 0.f;
        m = coat_warp_max(m);
        if (threadIdx.x == 0) atomicMax(amax_bits, __float_as_uint(m));   // non-negative floats order like their bits
    }
}

// The one scale of a per-tensor quantize.  From the tensor amax it is what the reference obtains as the
// maximum of its group scales: every group scale is round_to_scale_dtype((amax_g + 1e-10) / fp8_max),
// rounding is monotone, so the maximum is the rounded scale of the largest group
// (_quantize_pertensor.py:139: s_y.max()).
template <int FMT, bool IEEE>
__device__ __forceinline__ float tensor_scale_from_amax(const unsigned int* amax_bits, int scale_dtype) {
    const float amax = __uint_as_float(*amax_bits);
    return round_to_dtype(qdiv<IEEE>(amax + kScaleMinThres, CoatFp8Max<FMT>::value), scale_dtype);
}

// =================================================================================================
// 2. division by one scale (_division.py:45-126): q = x / s
// =================================================================================================
// The scale is either a device scalar in `scale_dtype` (scale_from_amax == 0) or derived from the amax word
// of pass 1, in which case block 0 also writes it to `s_out` (in `scale_dtype`).
// STOCH: the reference's stochastic rounding; the noise of element (m, n) is drawn at offset m * ldx + n
// (32-bit arithmetic, as in the reference's kernel).
template <typename T, int FMT, bool IEEE, bool STOCH>
__global__ void __launch_bounds__(kStraightThreads)
division_kernel(const T* __restrict__ x, uint8_t* __restrict__ y, const void* __restrict__ s_in, void* __restrict__ s_out,
                int scale_dtype, const unsigned int* __restrict__ amax_bits, int64_t M, int64_t N, int64_t ldx,
                int64_t ldy) {
    const float scale = amax_bits ? tensor_scale_from_amax<FMT, IEEE>(amax_bits, scale_dtype)
                                  : load_scale(s_in, 0, scale_dtype);
    if (amax_bits && s_out && blockIdx.x == 0 && threadIdx.x == 0) store_scale(s_out, 0, scale_dtype, scale);
    const int64_t segs_per_row = N >> 4;
    const int64_t total = M * segs_per_row;
    const ScaleDivider<IEEE> divide(scale);
    const int64_t seg = (int64_t)blockIdx.x * kStraightThreads + threadIdx.x;
    if (seg >= total) return;
    float v[16], q[16];
    Seg16<T>::load(x + seg_offset(seg, segs_per_row, ldx), v);
    divide.apply(v, q);
    if (STOCH) {
        const uint32_t off0 = (uint32_t)seg_offset(seg, segs_per_row, ldx);
#pragma unroll
        for (int i = 0; i < 16; ++i) q[i] = stochastic_perturb<FMT>(q[i], triton_rand_seed0(off0 + (uint32_t)i));
    }
    *reinterpret_cast<uint4*>(y + seg_offset(seg, segs_per_row, ldy)) = pack16<FMT>(q);
}

// =================================================================================================
// 2b. per-tensor quantize in ONE cooperative launch: pass 1 (tensor amax, optional group scales), a grid
//     barrier, pass 2 (division by the one scale).  Every CTA owns one contiguous slice of the matrix and walks
//     it forwards in pass 1 and BACKWARDS in pass 2, so that the second read of x finds the lines it touched
//     last still in the L2 of its own die (two separate kernels re-read x from DRAM: the CTA-to-SM mapping
//     changes, and a forward re-scan of 67 MB meets an LRU-like L2 at its oldest lines).  Outputs are stored
//     with the streaming hint so that they do not push x out.
// =================================================================================================
#ifndef COAT_PT_FUSED_UNROLL
#define COAT_PT_FUSED_UNROLL 4
#endif
constexpr int kFusedUnroll = COAT_PT_FUSED_UNROLL;
constexpr int kBarrierLimitDefault = 1 << 20;   // polls of ~0.1-1 us each: about a second, then COAT_E_TIMEOUT
__device__ int g_barrier_limit = kBarrierLimitDefault;   // lowered only by coat_fp8_quantize_set_barrier_limit (tests)

template <typename T> struct RawSeg;      // one 16-element segment as loaded
template <> struct RawSeg<float> { uint4 q[4]; };
template <> struct RawSeg<__nv_bfloat16> { uint4 q[2]; };
template <> struct RawSeg<__half> { uint4 q[2]; };

template <typename T, bool STREAM>
__device__ __forceinline__ RawSeg<T> load_raw(const T* p) {
    RawSeg<T> r;
#pragma unroll
    for (int i = 0; i < (int)(sizeof(T) * 16 / 16); ++i)
        r.q[i] = STREAM ? __ldcs(reinterpret_cast<const uint4*>(p) + i) : __ldcg(reinterpret_cast<const uint4*>(p) + i);
    return r;
}
__device__ __forceinline__ float raw_absmax(const RawSeg<__nv_bfloat16>& r) { return seg_absmax<__nv_bfloat16>(r.q[0], r.q[1]); }
__device__ __forceinline__ float raw_absmax(const RawSeg<__half>& r) { return seg_absmax<__half>(r.q[0], r.q[1]); }
__device__ __forceinline__ float raw_absmax(const RawSeg<float>& r) {
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i)
        m = fmaxf(fmaxf(m, fmaxf(fabsf(__uint_as_float(r.q[i].x)), fabsf(__uint_as_float(r.q[i].y)))),
                  fmaxf(fabsf(__uint_as_float(r.q[i].z)), fabsf(__uint_as_float(r.q[i].w))));
    return m;
}
__device__ __forceinline__ void raw_to_float(const RawSeg<__nv_bfloat16>& r, float (&v)[16]) {
    const uint32_t w[8] = {r.q[0].x, r.q[0].y, r.q[0].z, r.q[0].w, r.q[1].x, r.q[1].y, r.q[1].z, r.q[1].w};
#pragma unroll
    for (int i = 0; i < 8; ++i) { v[2 * i] = __uint_as_float(w[i] << 16); v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u); }
}
__device__ __forceinline__ void raw_to_float(const RawSeg<__half>& r, float (&v)[16]) {
    const uint32_t w[8] = {r.q[0].x, r.q[0].y, r.q[0].z, r.q[0].w, r.q[1].x, r.q[1].y, r.q[1].z, r.q[1].w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        v[2 * i] = f.x; v[2 * i + 1] = f.y;
    }
}
__device__ __forceinline__ void raw_to_float(const RawSeg<float>& r, float (&v)[16]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[4 * i] = __uint_as_float(r.q[i].x); v[4 * i + 1] = __uint_as_float(r.q[i].y);
        v[4 * i + 2] = __uint_as_float(r.q[i].z); v[4 * i + 3] = __uint_as_float(r.q[i].w);
    }
}

__device__ __forceinline__ unsigned int ld_acquire_u32(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// All CTAs of a cooperative launch meet here once.  Bounded: returns false (in every thread of the CTA) if the
// others have not arrived after g_barrier_limit polls.  `word` receives *payload as of the barrier.
__device__ __forceinline__ bool grid_barrier_once(unsigned int* counter, const unsigned int* payload, unsigned int* word) {
    __shared__ unsigned int s_payload;
    bool ok = true;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();            // this CTA's atomicMax on the payload is ordered before its arrival
        atomicAdd(counter, 1u);
        int tries = 0;
        const int limit = g_barrier_limit;
        while (ld_acquire_u32(counter) < gridDim.x) {
            if (++tries > limit) { ok = false; break; }
            __nanosleep(100);
        }
        s_payload = ld_acquire_u32(payload);
    }
    ok = __syncthreads_and(ok);
    *word = s_payload;
    return ok;
}

// Every CTA of a one-launch per-tensor kernel leaves through here exactly once, whether it finished or gave up at a
// bounded wait: the last one out puts the three sync words back to zero, so a call that timed out leaves the words
// as clean as a call that did not and the next call on the same words starts from zero.
__device__ __forceinline__ void pertensor_depart(unsigned int* sync) {
    if (threadIdx.x == 0 && atomicAdd(&sync[2], 1u) == gridDim.x - 1) {
        sync[0] = 0u; sync[1] = 0u; sync[2] = 0u;
    }
}

#ifndef COAT_PT_FUSED_CTAS
#define COAT_PT_FUSED_CTAS 4
#endif
template <typename T, int FMT, bool IEEE>
__global__ void __launch_bounds__(kStraightThreads, COAT_PT_FUSED_CTAS)
pertensor_fused_kernel(const T* __restrict__ x, uint8_t* __restrict__ y, void* __restrict__ s_y, void* __restrict__ s_out,
                       int scale_dtype, unsigned int* __restrict__ sync /*[0] amax bits, [1] arrivals, [2] departures*/,
                       int64_t M, int64_t N, int64_t ldx, int QB, int64_t segs_per_cta) {
    constexpr int kStep = kStraightThreads * kFusedUnroll;
    const int64_t segs_per_row = N >> 4;
    const int64_t total = M * segs_per_row;
    const int lanes = QB >> 4, lane_shift = 31 - __clz(lanes);
    const int64_t begin = (int64_t)blockIdx.x * segs_per_cta;          // a multiple of 8: groups stay inside a warp
    const int64_t end = begin + segs_per_cta < total ? begin + segs_per_cta : total;
    const GroupScale<FMT, IEEE> group_scale;
    // ---- pass 1: forwards
    float amax = 0.f;
    for (int64_t base = begin; base < end; base += kStep) {
        RawSeg<T> r[kFusedUnroll];
#pragma unroll
        for (int k = 0; k < kFusedUnroll; ++k) {
            const int64_t seg = base + k * kStraightThreads + threadIdx.x;
            if (seg < end) r[k] = load_raw<T, false>(x + seg_offset(seg, segs_per_row, ldx));
        }
#pragma unroll
        for (int k = 0; k < kFusedUnroll; ++k) {
            const int64_t seg = base + k * kStraightThreads + threadIdx.x;
            float m = seg < end ? raw_absmax(r[k]) : 0.f;
            amax = fmaxf(amax, m);
            if (s_y) {   // uniform over the launch
                m = subgroup_max(m, lanes);
                if (seg < end && (seg & (lanes - 1)) == 0) store_scale(s_y, seg >> lane_shift, scale_dtype, group_scale(m));
            }
        }
    }
    amax = coat_warp_max(amax);
    __shared__ float wmax[kStraightThreads / 32];
    if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = amax;
    __syncthreads();
    if (threadIdx.x == 0) {
        float m = wmax[0];
#pragma unroll
        for (int w = 1; w < kStraightThreads / 32; ++w) m = fmaxf(m, wmax[w]);
        atomicMax(&sync[0], __float_as_uint(m));   // non-negative floats order like their bits
    }
    // ---- everyone's maximum is in
    unsigned int amax_word;
    if (!grid_barrier_once(&sync[1], &sync[0], &amax_word)) {
        if (threadIdx.x == 0) g_quant_device_status = COAT_E_TIMEOUT;
        pertensor_depart(sync);
        return;
    }
    const float scale = tensor_scale_from_amax<FMT, IEEE>(&amax_word, scale_dtype);
    if (s_out && blockIdx.x == 0 && threadIdx.x == 0) store_scale(s_out, 0, scale_dtype, scale);
    const ScaleDivider<IEEE> divide(scale);
    // ---- pass 2: backwards over the same slice
    const int64_t last = begin + ((end - begin - 1) / kStep) * kStep;
    for (int64_t base = last; base >= begin; base -= kStep) {
        RawSeg<T> r[kFusedUnroll];
#pragma unroll
        for (int k = 0; k < kFusedUnroll; ++k) {
            const int64_t seg = base + k * kStraightThreads + threadIdx.x;
            if (seg < end) r[k] = load_raw<T, true>(x + seg_offset(seg, segs_per_row, ldx));
        }
#pragma unroll
        for (int k = 0; k < kFusedUnroll; ++k) {
            const int64_t seg = base + k * kStraightThreads + threadIdx.x;
            if (seg < end) {
                float v[16], q[16];
                raw_to_float(r[k], v);
                divide.apply(v, q);
                __stcs(reinterpret_cast<uint4*>(y + seg * 16), pack16<FMT>(q));
            }
        }
    }
    // the three words go back to zero for the next call: the last CTA to leave clears them (everyone has passed
    // the barrier and has taken its copy of the amax word by then)
    pertensor_depart(sync);
}

// =================================================================================================
// 3. dequantize (_dequantize.py:44-116): y = bf16(code * group scale)
// =================================================================================================
template <int FMT>
__global__ void __launch_bounds__(kStraightThreads)
dequantize_kernel(const uint8_t* __restrict__ x, const void* __restrict__ s, int scale_dtype,
                  __nv_bfloat16* __restrict__ y, int64_t M, int64_t N, int QB) {
    const int64_t total = M * (N >> 4);
    const int64_t seg = (int64_t)blockIdx.x * kStraightThreads + threadIdx.x;
    if (seg >= total) return;
    // rows are contiguous and N is a multiple of QB: segment `seg` belongs to group seg / (QB / 16)
    const float scale = load_scale(s, seg >> (31 - __clz(QB >> 4)), scale_dtype);
    const uint4 w = *reinterpret_cast<const uint4*>(x + seg * 16);
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
    uint32_t out[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float f[4];
        coat_fp8x4_to_float4<FMT>(ww[i], f);
        out[2 * i] = (uint32_t)coat_float_to_bf16_bits(f[0] * scale) | ((uint32_t)coat_float_to_bf16_bits(f[1] * scale) << 16);
        out[2 * i + 1] = (uint32_t)coat_float_to_bf16_bits(f[2] * scale) | ((uint32_t)coat_float_to_bf16_bits(f[3] * scale) << 16);
    }
    uint4* dst = reinterpret_cast<uint4*>(y + seg * 16);
    dst[0] = make_uint4(out[0], out[1], out[2], out[3]);
    dst[1] = make_uint4(out[4], out[5], out[6], out[7]);
}

// =================================================================================================
// 4. transposing kernels: division+transpose (_division_transpose.py:48-144) and
//    quantize+transpose (_quantize_transpose.py:39-173)
// =================================================================================================
// CTA tile: 128 rows (M) x 64 columns (N), 256 threads.  Thread = 4x4 block; warp = 16(M) x 32(N) patch with
// lane = 8*mb + nb (nb: 4-column block 0..7, mb: 4-row block 0..3).  Warp w of the CTA takes the patch
// (M block w, N half h) for h = 0, 1.
constexpr int kTM = 128, kTN = 64;
constexpr int kTileThreads = 256;
constexpr int kLdT = kTM / 4 + 1;   // words per row of the transposed shared tile (+1: conflict-free scatter)

// 4x4 byte transpose in registers: in[j] holds codes (j, 0..3), out[i] holds codes (0..3, i)
__device__ __forceinline__ void transpose4x4(const uint32_t (&in)[4], uint32_t (&out)[4]) {
    const uint32_t a = __byte_perm(in[0], in[1], 0x5140);   // r0c0 r1c0 r0c1 r1c1
    const uint32_t b = __byte_perm(in[2], in[3], 0x5140);   // r2c0 r3c0 r2c1 r3c1
    const uint32_t c = __byte_perm(in[0], in[1], 0x7362);   // r0c2 r1c2 r0c3 r1c3
    const uint32_t d = __byte_perm(in[2], in[3], 0x7362);
    out[0] = __byte_perm(a, b, 0x5410);   // r0c0 r1c0 r2c0 r3c0
    out[1] = __byte_perm(a, b, 0x7632);
    out[2] = __byte_perm(c, d, 0x5410);
    out[3] = __byte_perm(c, d, 0x7632);
}

// GROUPS: true = 1x16 group scales along both directions (QB is fixed to 16 by the tile mapping);
//         false = one scalar scale.  STRAIGHT: also write the un-transposed codes.
template <typename T, int FMT, bool IEEE, bool GROUPS, bool STRAIGHT>
__global__ void __launch_bounds__(kTileThreads)
transpose_quant_kernel(const T* __restrict__ x, uint8_t* __restrict__ y, uint8_t* __restrict__ y_t,
                       void* __restrict__ s_y, void* __restrict__ s_y_t, const void* __restrict__ s_in,
                       void* __restrict__ s_out, int scale_dtype, const unsigned int* __restrict__ amax_bits,
                       int M, int N, int64_t ldx) {
    __shared__ uint32_t tile_t[kTN][kLdT];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = lane & 7, mb = lane >> 3;
    const int m_tile = blockIdx.y * kTM, n_tile = blockIdx.x * kTN;
    const float fp8_max = CoatFp8Max<FMT>::value;
    float scalar = 1.f;
    if (!GROUPS) {
        scalar = amax_bits ? tensor_scale_from_amax<FMT, IEEE>(amax_bits, scale_dtype) : load_scale(s_in, 0, scale_dtype);
        if (amax_bits && s_out && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0)
            store_scale(s_out, 0, scale_dtype, scalar);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int m_loc = warp * 16 + mb * 4, n_loc = h * 32 + nb * 4;   // inside the CTA tile
        const int m0 = m_tile + m_loc, n0 = n_tile + n_loc;
        float v[4][4];
        const bool col_ok = n0 < N;   // N is a multiple of 16, so a 4-column block is in or out as a whole
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (col_ok && m0 + j < M) Seg16<T>::load4(x + (int64_t)(m0 + j) * ldx + n0, v[j]);
            else { v[j][0] = v[j][1] = v[j][2] = v[j][3] = 0.f; }
        }
        uint32_t straight[4], transposed[4];
        if (GROUPS) {
            // row groups: 16 consecutive columns = this lane and its neighbours nb^1, nb^2
            float rs[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float a = fmaxf(fmaxf(fabsf(v[j][0]), fabsf(v[j][1])), fmaxf(fabsf(v[j][2]), fabsf(v[j][3])));
                a = fmaxf(a, __shfl_xor_sync(COAT_FULL_MASK, a, 1));
                a = fmaxf(a, __shfl_xor_sync(COAT_FULL_MASK, a, 2));
                rs[j] = qdiv<IEEE>(a + kScaleMinThres, fp8_max);
                const ScaleDivider<IEEE> dr(rs[j]);
                straight[j] = coat_float4_to_fp8x4<FMT>(dr(v[j][0]), dr(v[j][1]), dr(v[j][2]), dr(v[j][3]));
            }
            if ((nb & 3) == 0 && col_ok) {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (m0 + j < M) store_scale(s_y, (int64_t)(m0 + j) * (N >> 4) + (n0 >> 4), scale_dtype, rs[j]);
            }
            // column groups: 16 consecutive rows = the lanes mb^1, mb^2 (lane xor 8, 16)
            float cs[4];
            uint32_t qt[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float a = fmaxf(fmaxf(fabsf(v[0][i]), fabsf(v[1][i])), fmaxf(fabsf(v[2][i]), fabsf(v[3][i])));
                a = fmaxf(a, __shfl_xor_sync(COAT_FULL_MASK, a, 8));
                a = fmaxf(a, __shfl_xor_sync(COAT_FULL_MASK, a, 16));
                cs[i] = qdiv<IEEE>(a + kScaleMinThres, fp8_max);
            }
            const ScaleDivider<IEEE> d0(cs[0]), d1(cs[1]), d2(cs[2]), d3(cs[3]);
#pragma unroll
            for (int j = 0; j < 4; ++j)
                qt[j] = coat_float4_to_fp8x4<FMT>(d0(v[j][0]), d1(v[j][1]), d2(v[j][2]), d3(v[j][3]));
            transpose4x4(qt, transposed);
            if (mb == 0 && col_ok && m0 < M) {
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    store_scale(s_y_t, (int64_t)(n0 + i) * (M >> 4) + (m0 >> 4), scale_dtype, cs[i]);
            }
        } else {
            const ScaleDivider<IEEE> ds(scalar);
#pragma unroll
            for (int j = 0; j < 4; ++j)
                straight[j] = coat_float4_to_fp8x4<FMT>(ds(v[j][0]), ds(v[j][1]), ds(v[j][2]), ds(v[j][3]));
            transpose4x4(straight, transposed);
        }
        if (STRAIGHT && col_ok) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (m0 + j < M) *reinterpret_cast<uint32_t*>(y + (int64_t)(m0 + j) * N + n0) = straight[j];
        }
        // scatter into the transposed tile: row = column of x, word = 4-row block of x
#pragma unroll
        for (int i = 0; i < 4; ++i) tile_t[n_loc + i][m_loc >> 2] = transposed[i];
    }
    __syncthreads();
    // transposed rows leave as 128 contiguous bytes: one warp instruction = one row of the tile
    for (int r = warp; r < kTN; r += kTileThreads / 32) {
        const int n = n_tile + r, m = m_tile + lane * 4;
        if (n < N && m < M) *reinterpret_cast<uint32_t*>(y_t + (int64_t)n * M + m) = tile_t[r][lane];
    }
}

// TMA-staged persistent kernel for the aligned case (M a multiple of 16, 16-byte aligned outputs).
// CTA tile 128 x 128, 512 threads, thread = 4 rows x 8 columns, lane = 8*mb + nb (nb: 8-column segment 0..7,
// mb: 4-row block 0..3), so a warp is 16 rows x 64 columns and warp w sits at rows 16*(w/2), columns 64*(w%2).
// A CTA walks tiles t = blockIdx.x, + gridDim.x, ...; the 128 x 128 input tile arrives by one 2-D bulk tensor
// copy (non-multicast) into one of two shared stages while the previous tile is being converted, so loads
// stay in flight through the compute and store phases (a register-only kernel, which loads, waits, computes
// and stores in turn, stayed near 40 % of the HBM rate).  Out-of-range rows / columns of edge tiles read as
// zero.  A 1x16 row group is 2 lanes (xor 1); a 16x1 column group is the 4 lanes mb = 0..3 (xor 8, 16).
// Packing 4 rows of one column straight into a word gives the transposed word without byte permutes.  The
// transposed tile crosses shared memory once: row = column of x, 32 words of 4 rows each, rotated by
// 4 * (column / 8) words so that neither the scatter nor the 16-byte gather has bank conflicts; the
// transposed scales cross it as [column][row group].  Both are double-buffered: one barrier per tile.
// 32 warps per SM (2 CTAs) are what hides the latencies of the short dependent chains (shuffles, MUFU,
// shared memory) of this kernel; with 256 threads per CTA it issued only half of the time.
constexpr int kWT = 128;
constexpr int kTmaStages = 2;
constexpr int kTmaWaitLimit = 1 << 22;

// shared memory: input stages | two transposed tiles and two tiles of transposed scales | barriers
constexpr size_t kTileTBytes = kWT * 32 * sizeof(uint32_t);
constexpr size_t kScaleTBytes = kWT * 8 * sizeof(float);
template <typename T> constexpr size_t tma_quant_smem() {
    return (size_t)kTmaStages * kWT * kWT * sizeof(T) + 2 * kTileTBytes + 2 * kScaleTBytes + 64 + 128 /*alignment slack*/;
}

__device__ __noinline__ float div_full_outlined(float x, float s) { return coat_div_full(x, s); }

__device__ __forceinline__ void tile_coords(int t, int tiles_n, int& tm, int& tn) {
    tm = t / tiles_n;
    tn = t - tm * tiles_n;
}

// C = columns per thread: 8 (512 threads; more warps to hide latencies: best for the scalar-scale variant) or
// 16 (256 threads; a 1x16 row group is thread-local and per-column work is shared by fewer threads: best for
// the 1x16 quantize+transpose, 28.6 us against 31.3 us at 8192 x 4096).
template <int C> struct TmaShape {
    static constexpr int kThreads = kWT * kWT / (4 * C);
};

// rows / columns of the tile that a thread owns: warps tile the 128 x 128 tile in bands of 16 rows
template <int C>
__device__ __forceinline__ void tma_thread_origin(int warp, int lane, int& m_loc, int& n_loc) {
    const int nb = lane & 7, mb = lane >> 3;
    if (C == 8) { m_loc = (warp >> 1) * 16 + mb * 4; n_loc = (warp & 1) * 64 + nb * 8; }
    else { m_loc = warp * 16 + mb * 4; n_loc = nb * 16; }
}

template <typename T, int C>
__device__ __forceinline__ void load_cols(const T* p, float (&v)[C]) {
    if constexpr (C == 8) load8(p, v);
    else Seg16<T>::load(p, v);
}

template <int C>
__device__ __forceinline__ float absmax_cols(const float (&v)[C]) {
    float m[C / 2];
#pragma unroll
    for (int i = 0; i < C / 2; ++i) m[i] = fmaxf(fabsf(v[2 * i]), fabsf(v[2 * i + 1]));
#pragma unroll
    for (int w = C / 4; w >= 1; w >>= 1)
#pragma unroll
        for (int i = 0; i < w; ++i) m[i] = fmaxf(m[2 * i], m[2 * i + 1]);
    return m[0];
}

// C codes of one row, divided by `d`, to global memory (8 or 16 bytes)
template <int FMT, int C, typename Divider>
__device__ __forceinline__ void store_row_codes(uint8_t* dst, const float (&v)[C], const Divider& d) {
    uint32_t w[C / 4];
#pragma unroll
    for (int i = 0; i < C / 4; ++i) {
        const float2 lo = d.pair(v[4 * i], v[4 * i + 1]), hi = d.pair(v[4 * i + 2], v[4 * i + 3]);
        w[i] = coat_float4_to_fp8x4<FMT>(lo.x, lo.y, hi.x, hi.y);
    }
    if constexpr (C == 8) *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
    else *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
}

struct DivFullDivider {   // the division instruction itself, out of line (scales outside [2^-120, 2^120])
    float s;
    __device__ __forceinline__ float operator()(float x) const { return div_full_outlined(x, s); }
    __device__ __forceinline__ float2 pair(float a, float b) const { return make_float2((*this)(a), (*this)(b)); }
};

// FUSED (scalar-scale variant only): the kernel also finds the tensor's amax itself.  Launched cooperatively, every
// CTA first walks its tiles forwards through the same staging ring taking maxima, all CTAs meet at a bounded grid
// barrier, and the quantising pass then walks the same tiles BACKWARDS, so that its reads are served from L2
// (see pertensor_fused_kernel).  `sync` = three words, zero on entry, zero again at exit.
template <typename T, int FMT, bool IEEE, bool GROUPS, bool STRAIGHT, int C, bool FUSED = false>
__global__ void __launch_bounds__(TmaShape<C>::kThreads, sizeof(T) == 4 ? 1 : 2)
transpose_quant_tma_kernel(const __grid_constant__ CUtensorMap map_x, uint8_t* __restrict__ y,
                           uint8_t* __restrict__ y_t, void* __restrict__ s_y, void* __restrict__ s_y_t,
                           const void* __restrict__ s_in, void* __restrict__ s_out, int scale_dtype,
                           const unsigned int* __restrict__ amax_bits, int M, int N, int tiles_m, int tiles_n,
                           unsigned int* __restrict__ sync) {
    constexpr int kThreads = TmaShape<C>::kThreads;
    const int n_tiles = tiles_m * tiles_n;
    extern __shared__ unsigned char smem_dyn[];
    unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_dyn) + 127) & ~(uintptr_t)127);
    constexpr uint32_t kStageBytes = kWT * kWT * sizeof(T);
    unsigned char* after_stages = base + (size_t)kTmaStages * kStageBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(after_stages + 2 * kTileTBytes + 2 * kScaleTBytes);

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int mb = lane >> 3;
    int m_loc, n_loc;
    tma_thread_origin<C>(warp, lane, m_loc, n_loc);
    // rotated slot of this thread's 4 rows in a transposed row: 4 words further per C columns
    const int word = ((m_loc >> 2) + 4 * (n_loc / C)) & 31;
    const GroupScale<FMT, IEEE> group_scale;
    float scalar = 1.f;
    if (!GROUPS && !FUSED) {
        scalar = amax_bits ? tensor_scale_from_amax<FMT, IEEE>(amax_bits, scale_dtype) : load_scale(s_in, 0, scale_dtype);
        if (amax_bits && s_out && blockIdx.x == 0 && threadIdx.x == 0) store_scale(s_out, 0, scale_dtype, scalar);
    }
    // Uses of the staging ring are numbered k = 0, 1, ...: stage k % kTmaStages, barrier parity (k / kTmaStages) & 1.
    // Plain: use k is tile blockIdx.x + k * gridDim.x.  FUSED: the first n_mine uses are the amax pass over the
    // same tiles, the next n_mine the quantising pass over them in reverse order.
    const int n_mine = (int)blockIdx.x < n_tiles ? (n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int k_end = FUSED ? 2 * n_mine : n_mine;
    auto tile_of = [&](int use) -> int {
        const int i = (FUSED && use >= n_mine) ? 2 * n_mine - 1 - use : use;
        return (int)blockIdx.x + i * (int)gridDim.x;
    };
    auto issue = [&](int use) {   // thread 0 only
        const int st = use % kTmaStages;
        int tm, tn;
        tile_coords(tile_of(use), tiles_n, tm, tn);
        coat_tma::mbar_expect_tx(&full[st], kStageBytes);
        coat_tma::load_2d(base + (size_t)st * kStageBytes, &map_x, tn * kWT, tm * kWT, &full[st]);
    };
    auto give_up = [&](int use) {   // a wait ran out (never expected): leave only after our copies in flight have landed
        if (threadIdx.x == 0) {
            g_quant_device_status = COAT_E_TIMEOUT;
            for (int q = 0; q < kTmaStages; ++q)
                if (use + q < k_end)
                    coat_tma::mbar_wait(&full[(use + q) % kTmaStages], (uint32_t)((use + q) / kTmaStages) & 1u, kTmaWaitLimit);
        }
        __syncthreads();
        if (FUSED) pertensor_depart(sync);
    };
    if (threadIdx.x == 0) {
#pragma unroll
        for (int s = 0; s < kTmaStages; ++s) coat_tma::mbar_init(&full[s], 1);
        coat_tma::mbar_init_fence();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
#pragma unroll
        for (int s = 0; s < kTmaStages; ++s)
            if (s < k_end) issue(s);
    }
    int k = 0;
    if (FUSED) {
        float amax = 0.f;
        for (; k < n_mine; ++k) {
            const int s = k % kTmaStages;
            const T* stage = reinterpret_cast<const T*>(base + (size_t)s * kStageBytes);
            const bool arrived = coat_tma::mbar_wait(&full[s], (uint32_t)(k / kTmaStages) & 1u, kTmaWaitLimit);
            float v[4][C];
#pragma unroll
            for (int j = 0; j < 4; ++j) load_cols<T, C>(stage + (m_loc + j) * kWT + n_loc, v[j]);
#pragma unroll
            for (int j = 0; j < 4; ++j) amax = fmaxf(amax, absmax_cols<C>(v[j]));   // parts outside the matrix are zero-filled
            if (!__syncthreads_and(arrived)) { give_up(k); return; }
            if (threadIdx.x == 0 && k + kTmaStages < k_end) issue(k + kTmaStages);
        }
        amax = coat_warp_max(amax);
        float* wmax = reinterpret_cast<float*>(after_stages);   // the transposed-tile buffer is free until the second pass
        if (lane == 0) wmax[warp] = amax;
        __syncthreads();
        if (threadIdx.x == 0) {
            float m = wmax[0];
            for (int w = 1; w < kThreads / 32; ++w) m = fmaxf(m, wmax[w]);
            atomicMax(&sync[0], __float_as_uint(m));
        }
        unsigned int amax_word;
        if (!grid_barrier_once(&sync[1], &sync[0], &amax_word)) { give_up(k); return; }
        scalar = tensor_scale_from_amax<FMT, IEEE>(&amax_word, scale_dtype);
        if (s_out && blockIdx.x == 0 && threadIdx.x == 0) store_scale(s_out, 0, scale_dtype, scalar);
    }
    const ScaleDivider<IEEE> by_scalar(scalar);
    for (; k < k_end; ++k) {
        const int t = tile_of(k);
        const int s = k % kTmaStages;
        const T* stage = reinterpret_cast<const T*>(base + (size_t)s * kStageBytes);
        uint32_t (*tile_t)[32] = reinterpret_cast<uint32_t (*)[32]>(after_stages + (size_t)(k & 1) * kTileTBytes);
        float (*scale_t)[8] = reinterpret_cast<float (*)[8]>(after_stages + 2 * kTileTBytes + (size_t)(k & 1) * kScaleTBytes);
        const bool arrived = coat_tma::mbar_wait(&full[s], (uint32_t)(k / kTmaStages) & 1u, kTmaWaitLimit);
        float v[4][C];
#pragma unroll
        for (int j = 0; j < 4; ++j) load_cols<T, C>(stage + (m_loc + j) * kWT + n_loc, v[j]);
        int tm, tn;
        tile_coords(t, tiles_n, tm, tn);
        const int m_tile = tm * kWT, n_tile = tn * kWT;
        const int m0 = m_tile + m_loc, n0 = n_tile + n_loc;
        // M and N are multiples of 16 and the lanes of a 16-column group sit side by side: a 4 x 16 block is in the
        // matrix or outside it as a whole
        const bool inside = m0 < M && n0 < N;
        if (GROUPS) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {   // row groups (C = 8: this lane's columns and its neighbour's)
                float a = absmax_cols<C>(v[j]);
                if (C == 8) a = fmaxf(a, __shfl_xor_sync(COAT_FULL_MASK, a, 1));
                const float rs = group_scale(a);
                if (inside) {
                    store_row_codes<FMT, C>(y + (int64_t)(m0 + j) * N + n0, v[j], GroupScaleDivider<IEEE>(rs));
                    if (C == 16 || (lane & 1) == 0)
                        store_scale(s_y, (int64_t)(m0 + j) * (N >> 4) + (n0 >> 4), scale_dtype, rs);
                }
            }
#pragma unroll
            for (int i = 0; i < C; ++i) {   // column groups: the 4 lanes mb = 0..3
                float a = fmaxf(fmaxf(fabsf(v[0][i]), fabsf(v[1][i])), fmaxf(fabsf(v[2][i]), fabsf(v[3][i])));
                a = fmaxf(a, __shfl_xor_sync(COAT_FULL_MASK, a, 8));
                a = fmaxf(a, __shfl_xor_sync(COAT_FULL_MASK, a, 16));
                const float cs = group_scale(a);
                const GroupScaleDivider<IEEE> d(cs);
                {
                    const float2 lo = d.pair(v[0][i], v[1][i]), hi = d.pair(v[2][i], v[3][i]);
                    tile_t[n_loc + i][word] = coat_float4_to_fp8x4<FMT>(lo.x, lo.y, hi.x, hi.y);
                }
                if ((i & 3) == mb) scale_t[n_loc + i][m_loc >> 4] = cs;   // the four lanes of a group share the stores
            }
        } else if (IEEE || by_scalar.fast) {
            // the usual case, decided once per tile: one multiplication (or IEEE division) per element
            const GroupScaleDivider<IEEE> d(scalar);
            if (STRAIGHT && inside) {
#pragma unroll
                for (int j = 0; j < 4; ++j) store_row_codes<FMT, C>(y + (int64_t)(m0 + j) * N + n0, v[j], d);
            }
#pragma unroll
            for (int i = 0; i < C; ++i)
                {
                    const float2 lo = d.pair(v[0][i], v[1][i]), hi = d.pair(v[2][i], v[3][i]);
                    tile_t[n_loc + i][word] = coat_float4_to_fp8x4<FMT>(lo.x, lo.y, hi.x, hi.y);
                }
        } else {
            const DivFullDivider d{scalar};
            if (STRAIGHT && inside) {
#pragma unroll
                for (int j = 0; j < 4; ++j) store_row_codes<FMT, C>(y + (int64_t)(m0 + j) * N + n0, v[j], d);
            }
#pragma unroll
            for (int i = 0; i < C; ++i)
                {
                    const float2 lo = d.pair(v[0][i], v[1][i]), hi = d.pair(v[2][i], v[3][i]);
                    tile_t[n_loc + i][word] = coat_float4_to_fp8x4<FMT>(lo.x, lo.y, hi.x, hi.y);
                }
        }
        // The one barrier of the tile: stage s has been read by everyone (it can be refilled) and this tile's
        // transposed codes and scales are complete.  Tile k+1 writes the other pair of buffers, and nobody
        // passes the barrier of tile k+1 (after which this pair is written again) before every thread has
        // finished the readout of tile k below.
        if (!__syncthreads_and(arrived)) { give_up(k); return; }
        if (threadIdx.x == 0 && k + kTmaStages < k_end) issue(k + kTmaStages);
        // transposed rows leave in 16-byte pieces: one warp instruction = 4 rows x 128 contiguous bytes
#pragma unroll
        for (int it = 0; it < kWT * 8 / kThreads; ++it) {
            const int idx = it * kThreads + threadIdx.x;
            const int r = idx >> 3, c = idx & 7;
            const int n = n_tile + r, m = m_tile + c * 16;
            if (n < N && m < M)
                *reinterpret_cast<uint4*>(y_t + (int64_t)n * M + m) =
                    *reinterpret_cast<const uint4*>(&tile_t[r][(4 * c + 4 * (r / C)) & 31]);
        }
        if (GROUPS && threadIdx.x < kWT) {   // transposed scales: 8 consecutive row groups per column of x
            const int n = n_tile + threadIdx.x;
            const int groups_left = (M - m_tile + 15) >> 4;   // row groups of this tile that exist (1..8, or <= 0)
            if (n < N && groups_left > 0) {
                const float4 lo = reinterpret_cast<const float4*>(scale_t[threadIdx.x])[0];
                const float4 hi = reinterpret_cast<const float4*>(scale_t[threadIdx.x])[1];
                const float sc[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
                const int64_t idx0 = (int64_t)n * (M >> 4) + (m_tile >> 4);
                if (groups_left >= 8 && scale_dtype == COAT_BF16 && ((idx0 & 7) == 0) &&
                    (reinterpret_cast<uintptr_t>(s_y_t) & 15) == 0) {
                    uint4 w;
                    w.x = (uint32_t)coat_float_to_bf16_bits(sc[0]) | ((uint32_t)coat_float_to_bf16_bits(sc[1]) << 16);
                    w.y = (uint32_t)coat_float_to_bf16_bits(sc[2]) | ((uint32_t)coat_float_to_bf16_bits(sc[3]) << 16);
                    w.z = (uint32_t)coat_float_to_bf16_bits(sc[4]) | ((uint32_t)coat_float_to_bf16_bits(sc[5]) << 16);
                    w.w = (uint32_t)coat_float_to_bf16_bits(sc[6]) | ((uint32_t)coat_float_to_bf16_bits(sc[7]) << 16);
                    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(s_y_t) + idx0) = w;
                } else {
#pragma unroll
                    for (int g = 0; g < 8; ++g)
                        if (g < groups_left) store_scale(s_y_t, idx0 + g, scale_dtype, sc[g]);
                }
            }
        }
    }
    if (FUSED) pertensor_depart(sync);   // last CTA out clears the words
}

inline bool tma_tiles_fit(int64_t M, int64_t N) {   // tile counts and coordinates are 32-bit in the kernel
    return M < (1ll << 31) && N < (1ll << 31) && ((M + kWT - 1) / kWT) * ((N + kWT - 1) / kWT) < (1ll << 30);
}

// Launch of the TMA-staged kernel; COAT_E_DEVICE when the tensor map cannot be encoded.
template <typename T, int FMT, bool IEEE, bool GROUPS, bool STRAIGHT>
int launch_transpose_tma(const void* x, uint8_t* y, uint8_t* y_t, void* s_y, void* s_y_t, const void* s_in, void* s_out,
                         int scale_dtype, const unsigned int* amax, int64_t M, int64_t N, int64_t ldx, cudaStream_t st) {
    CUtensorMap map;
    if (!coat_tma::make_map_2d(&map, x, (int)sizeof(T), M, N, ldx * (int64_t)sizeof(T), kWT, kWT)) return COAT_E_DEVICE;
    constexpr int C = GROUPS ? 16 : 8;
    auto kern = transpose_quant_tma_kernel<T, FMT, IEEE, GROUPS, STRAIGHT, C>;
    constexpr size_t smem = tma_quant_smem<T>();
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return COAT_E_LAUNCH;
    const int64_t tiles_n = (N + kWT - 1) / kWT, tiles_m = (M + kWT - 1) / kWT;
    const int64_t n_tiles = tiles_n * tiles_m;
    const int64_t cap = (int64_t)coat_sm_count() * (sizeof(T) == 4 ? 1 : 2);
    const int grid = (int)(n_tiles < cap ? n_tiles : cap);
    kern<<<grid, TmaShape<C>::kThreads, smem, st>>>(map, y, y_t, s_y, s_y_t, s_in, s_out, scale_dtype, amax, (int)M, (int)N,
                                           (int)tiles_m, (int)tiles_n, nullptr);
    return coat_launch_status();
}

// The FUSED form of the scalar-scale variant (amax pass + barrier + quantising pass), launched cooperatively.
template <typename T, int FMT, bool IEEE, bool STRAIGHT>
int launch_transpose_tma_fused(const void* x, uint8_t* y, uint8_t* y_t, void* s_out, int scale_dtype, unsigned int* sync,
                               int64_t M, int64_t N, int64_t ldx, cudaStream_t st) {
    CUtensorMap map;
    if (!coat_tma::make_map_2d(&map, x, (int)sizeof(T), M, N, ldx * (int64_t)sizeof(T), kWT, kWT)) return COAT_E_DEVICE;
    constexpr int C = 8;
    auto kern = transpose_quant_tma_kernel<T, FMT, IEEE, false, STRAIGHT, C, true>;
    constexpr size_t smem = tma_quant_smem<T>();
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return COAT_E_LAUNCH;
    static int ctas_per_sm = 0;   // per instantiation
    if (ctas_per_sm == 0) {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, TmaShape<C>::kThreads, smem) != cudaSuccess || n < 1)
            return COAT_E_LAUNCH;
        ctas_per_sm = n;
    }
    const int64_t tiles_n = (N + kWT - 1) / kWT, tiles_m = (M + kWT - 1) / kWT;
    const int64_t n_tiles = tiles_n * tiles_m;
    const int64_t cap = (int64_t)coat_sm_count() * ctas_per_sm;
    const int grid = (int)(n_tiles < cap ? n_tiles : cap);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(TmaShape<C>::kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeCooperative;
    attr.val.cooperative = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, map, y, y_t, (void*)nullptr, (void*)nullptr, (const void*)nullptr, s_out, scale_dtype,
                           (const unsigned int*)nullptr, (int)M, (int)N, (int)tiles_m, (int)tiles_n, sync) != cudaSuccess) {
        cudaGetLastError();
        return COAT_E_LAUNCH;
    }
    return coat_launch_status();
}

// =================================================================================================
// 4b. fp8_mul_forward in ONE launch (mul_fwd.py:51-254: product kernel -> bf16 y + group scales, `s_y.max()`,
//     fp8_division_transpose of y)
// =================================================================================================
// The two-kernel form writes the bf16 product to memory and reads it back only because the per-tensor scale
// needs the whole tensor's maximum first: 8.4 bytes per element moved for 4.25 of inputs and outputs.  Here the
// tile kernel's one-launch pattern is applied to the product itself: every CTA walks its 128 x 128 tiles forwards
// (the codes of both operands and their 1x16 scales arrive by four bulk tensor copies per tile) taking the maximum
// of |(c1 s1)(c2 s2)|, all CTAs meet at the bounded grid barrier, and the second pass walks the same tiles
// BACKWARDS (the tail of the first pass is still in L2), recomputes the product, rounds it to bf16 as the
// reference's intermediate tensor does, divides by the per-tensor scale and writes codes and transposed codes.
// Bit-identical to the two-kernel form.  bf16 scales, QB = 16, M % 16 == 0, N % 128 == 0 (row pitch of the scale
// matrices a multiple of 16 bytes); other cases take the two kernels.
struct MulMaps { CUtensorMap q1, q2, s1, s2; };
constexpr uint32_t kMulCodeBytes = kWT * kWT, kMulScaleBytes = kWT * (kWT / 16) * 2;
constexpr uint32_t kMulStageBytes = 2 * kMulCodeBytes + 2 * kMulScaleBytes;
constexpr size_t kMulSmem = (size_t)kTmaStages * kMulStageBytes + 2 * kTileTBytes + 64 + 128;

template <int FMT, bool IEEE>
__global__ void __launch_bounds__(TmaShape<8>::kThreads, 2)
mul_pertensor_tma_kernel(const __grid_constant__ MulMaps maps, uint8_t* __restrict__ y, uint8_t* __restrict__ y_t,
                         void* __restrict__ s_out, int scale_dtype, int M, int N, int tiles_m, int tiles_n,
                         unsigned int* __restrict__ sync) {
    constexpr int C = 8;
    constexpr int kThreads = TmaShape<C>::kThreads;
    const int n_tiles = tiles_m * tiles_n;
    extern __shared__ unsigned char smem_dyn[];
    unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_dyn) + 127) & ~(uintptr_t)127);
    unsigned char* after_stages = base + (size_t)kTmaStages * kMulStageBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(after_stages + 2 * kTileTBytes);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int m_loc, n_loc;
    tma_thread_origin<C>(warp, lane, m_loc, n_loc);
    const int word = ((m_loc >> 2) + 4 * (n_loc / C)) & 31;
    const int n_mine = (int)blockIdx.x < n_tiles ? (n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int k_end = 2 * n_mine;
    auto tile_of = [&](int use) -> int {
        const int i = use >= n_mine ? 2 * n_mine - 1 - use : use;
        return (int)blockIdx.x + i * (int)gridDim.x;
    };
    auto issue = [&](int use) {   // thread 0 only
        unsigned char* st = base + (size_t)(use % kTmaStages) * kMulStageBytes;
        uint64_t* bar = &full[use % kTmaStages];
        int tm, tn;
        tile_coords(tile_of(use), tiles_n, tm, tn);
        coat_tma::mbar_expect_tx(bar, kMulStageBytes);
        coat_tma::load_2d(st, &maps.q1, tn * kWT, tm * kWT, bar);
        coat_tma::load_2d(st + kMulCodeBytes, &maps.q2, tn * kWT, tm * kWT, bar);
        coat_tma::load_2d(st + 2 * kMulCodeBytes, &maps.s1, tn * (kWT / 16), tm * kWT, bar);
        coat_tma::load_2d(st + 2 * kMulCodeBytes + kMulScaleBytes, &maps.s2, tn * (kWT / 16), tm * kWT, bar);
    };
    auto give_up = [&](int use) {   // a wait ran out (never expected): leave only after our copies in flight have landed
        if (threadIdx.x == 0) {
            g_quant_device_status = COAT_E_TIMEOUT;
            for (int q = 0; q < kTmaStages; ++q)
                if (use + q < k_end)
                    coat_tma::mbar_wait(&full[(use + q) % kTmaStages], (uint32_t)((use + q) / kTmaStages) & 1u, kTmaWaitLimit);
        }
        __syncthreads();
        pertensor_depart(sync);
    };
    // the four rows x eight columns of this thread: (c1 s1) (c2 s2) in fp32, as the reference's product kernel
    auto products = [&](const unsigned char* st, float (&v)[4][C]) {
        const __nv_bfloat16* s1 = reinterpret_cast<const __nv_bfloat16*>(st + 2 * kMulCodeBytes);
        const __nv_bfloat16* s2 = reinterpret_cast<const __nv_bfloat16*>(st + 2 * kMulCodeBytes + kMulScaleBytes);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int row = m_loc + j;
            const uint2 a = *reinterpret_cast<const uint2*>(st + row * kWT + n_loc);
            const uint2 b = *reinterpret_cast<const uint2*>(st + kMulCodeBytes + row * kWT + n_loc);
            const float sa = __bfloat162float(s1[row * (kWT / 16) + (n_loc >> 4)]);
            const float sb = __bfloat162float(s2[row * (kWT / 16) + (n_loc >> 4)]);
            float fa[8], fb[8];
            coat_fp8x4_to_float4<FMT>(a.x, *reinterpret_cast<float (*)[4]>(&fa[0]));
            coat_fp8x4_to_float4<FMT>(a.y, *reinterpret_cast<float (*)[4]>(&fa[4]));
            coat_fp8x4_to_float4<FMT>(b.x, *reinterpret_cast<float (*)[4]>(&fb[0]));
            coat_fp8x4_to_float4<FMT>(b.y, *reinterpret_cast<float (*)[4]>(&fb[4]));
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
                const float2 x1 = __fmul2_rn(make_float2(fa[i], fa[i + 1]), make_float2(sa, sa));
                const float2 x2 = __fmul2_rn(make_float2(fb[i], fb[i + 1]), make_float2(sb, sb));
                const float2 pr = __fmul2_rn(x1, x2);
                v[j][i] = pr.x; v[j][i + 1] = pr.y;
            }
        }
    };
    if (threadIdx.x == 0) {
#pragma unroll
        for (int s = 0; s < kTmaStages; ++s) coat_tma::mbar_init(&full[s], 1);
        coat_tma::mbar_init_fence();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
#pragma unroll
        for (int s = 0; s < kTmaStages; ++s)
            if (s < k_end) issue(s);
    }
    // ---- pass 1: the tensor's maximum
    int k = 0;
    float amax = 0.f;
    for (; k < n_mine; ++k) {
        const unsigned char* st = base + (size_t)(k % kTmaStages) * kMulStageBytes;
        const bool arrived = coat_tma::mbar_wait(&full[k % kTmaStages], (uint32_t)(k / kTmaStages) & 1u, kTmaWaitLimit);
        float v[4][C];
        products(st, v);
#pragma unroll
        for (int j = 0; j < 4; ++j) amax = fmaxf(amax, absmax_cols<C>(v[j]));   // parts outside the matrix are zero-filled
        if (!__syncthreads_and(arrived)) { give_up(k); return; }
        if (threadIdx.x == 0 && k + kTmaStages < k_end) issue(k + kTmaStages);
    }
    amax = coat_warp_max(amax);
    float* wmax = reinterpret_cast<float*>(after_stages);   // the transposed-tile buffer is free until the second pass
    if (lane == 0) wmax[warp] = amax;
    __syncthreads();
    if (threadIdx.x == 0) {
        float m = wmax[0];
        for (int w = 1; w < kThreads / 32; ++w) m = fmaxf(m, wmax[w]);
        atomicMax(&sync[0], __float_as_uint(m));
    }
    unsigned int amax_word;
    if (!grid_barrier_once(&sync[1], &sync[0], &amax_word)) { give_up(k); return; }
    const float scalar = tensor_scale_from_amax<FMT, IEEE>(&amax_word, scale_dtype);
    if (s_out && blockIdx.x == 0 && threadIdx.x == 0) store_scale(s_out, 0, scale_dtype, scalar);
    const ScaleDivider<IEEE> by_scalar(scalar);
    // ---- pass 2: the same tiles in reverse order
    for (; k < k_end; ++k) {
        const int t = tile_of(k);
        const unsigned char* st = base + (size_t)(k % kTmaStages) * kMulStageBytes;
        uint32_t (*tile_t)[32] = reinterpret_cast<uint32_t (*)[32]>(after_stages + (size_t)(k & 1) * kTileTBytes);
        const bool arrived = coat_tma::mbar_wait(&full[k % kTmaStages], (uint32_t)(k / kTmaStages) & 1u, kTmaWaitLimit);
        float v[4][C];
        products(st, v);
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int i = 0; i < C; ++i) v[j][i] = __bfloat162float(__float2bfloat16_rn(v[j][i]));   // the reference's bf16 y
        int tm, tn;
        tile_coords(t, tiles_n, tm, tn);
        const int m_tile = tm * kWT, n_tile = tn * kWT;
        const int m0 = m_tile + m_loc, n0 = n_tile + n_loc;
        const bool inside = m0 < M && n0 < N;
        if (IEEE || by_scalar.fast) {
            const GroupScaleDivider<IEEE> d(scalar);
            if (inside) {
#pragma unroll
                for (int j = 0; j < 4; ++j) store_row_codes<FMT, C>(y + (int64_t)(m0 + j) * N + n0, v[j], d);
            }
#pragma unroll
            for (int i = 0; i < C; ++i) {
                const float2 lo = d.pair(v[0][i], v[1][i]), hi = d.pair(v[2][i], v[3][i]);
                tile_t[n_loc + i][word] = coat_float4_to_fp8x4<FMT>(lo.x, lo.y, hi.x, hi.y);
            }
        } else {
            const DivFullDivider d{scalar};
            if (inside) {
#pragma unroll
                for (int j = 0; j < 4; ++j) store_row_codes<FMT, C>(y + (int64_t)(m0 + j) * N + n0, v[j], d);
            }
#pragma unroll
            for (int i = 0; i < C; ++i)
                tile_t[n_loc + i][word] = coat_float4_to_fp8x4<FMT>(d(v[0][i]), d(v[1][i]), d(v[2][i]), d(v[3][i]));
        }
        if (!__syncthreads_and(arrived)) { give_up(k); return; }
        if (threadIdx.x == 0 && k + kTmaStages < k_end) issue(k + kTmaStages);
#pragma unroll
        for (int it = 0; it < kWT * 8 / kThreads; ++it) {   // transposed rows leave in 16-byte pieces
            const int idx = it * kThreads + threadIdx.x;
            const int r = idx >> 3, c = idx & 7;
            const int n = n_tile + r, m = m_tile + c * 16;
            if (n < N && m < M)
                *reinterpret_cast<uint4*>(y_t + (int64_t)n * M + m) =
                    *reinterpret_cast<const uint4*>(&tile_t[r][(4 * c + 4 * (r / C)) & 31]);
        }
    }
    pertensor_depart(sync);
}

template <int FMT, bool IEEE>
int launch_mul_pertensor(const uint8_t* x1, const void* s1, const uint8_t* x2, const void* s2, uint8_t* y, uint8_t* y_t,
                         void* s_out, int scale_dtype, unsigned int* sync, int64_t M, int64_t N, cudaStream_t st) {
    MulMaps maps;
    if (!coat_tma::make_map_2d(&maps.q1, x1, 1, M, N, N, kWT, kWT) || !coat_tma::make_map_2d(&maps.q2, x2, 1, M, N, N, kWT, kWT) ||
        !coat_tma::make_map_2d(&maps.s1, s1, 2, M, N / 16, (N / 16) * 2, kWT, kWT / 16) ||
        !coat_tma::make_map_2d(&maps.s2, s2, 2, M, N / 16, (N / 16) * 2, kWT, kWT / 16))
        return COAT_E_DEVICE;
    auto kern = mul_pertensor_tma_kernel<FMT, IEEE>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMulSmem) != cudaSuccess)
        return COAT_E_LAUNCH;
    static int ctas_per_sm = 0;   // per instantiation
    if (ctas_per_sm == 0) {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, TmaShape<8>::kThreads, kMulSmem) != cudaSuccess || n < 1)
            return COAT_E_LAUNCH;
        ctas_per_sm = n;
    }
    const int64_t tiles_n = (N + kWT - 1) / kWT, tiles_m = (M + kWT - 1) / kWT;
    const int64_t n_tiles = tiles_n * tiles_m;
    const int64_t cap = (int64_t)coat_sm_count() * ctas_per_sm;
    const int grid = (int)(n_tiles < cap ? n_tiles : cap);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(TmaShape<8>::kThreads);
    cfg.dynamicSmemBytes = kMulSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeCooperative;
    attr.val.cooperative = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, maps, y, y_t, s_out, scale_dtype, (int)M, (int)N, (int)tiles_m, (int)tiles_n, sync) !=
        cudaSuccess) {
        cudaGetLastError();
        return COAT_E_LAUNCH;
    }
    return coat_launch_status();
}

// =================================================================================================
// 5. byte transpose (_transpose.py:39-82)
// =================================================================================================
__global__ void __launch_bounds__(kTileThreads)
transpose_bytes_kernel(const uint8_t* __restrict__ x, uint8_t* __restrict__ y_t, int M, int N) {
    __shared__ uint32_t tile_t[kTN][kLdT];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = lane & 7, mb = lane >> 3;
    const int m_tile = blockIdx.y * kTM, n_tile = blockIdx.x * kTN;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int m_loc = warp * 16 + mb * 4, n_loc = h * 32 + nb * 4;
        const int m0 = m_tile + m_loc, n0 = n_tile + n_loc;
        uint32_t in[4], out[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
            in[j] = (n0 < N && m0 + j < M) ? *reinterpret_cast<const uint32_t*>(x + (int64_t)(m0 + j) * N + n0) : 0u;
        transpose4x4(in, out);
#pragma unroll
        for (int i = 0; i < 4; ++i) tile_t[n_loc + i][m_loc >> 2] = out[i];
    }
    __syncthreads();
    for (int r = warp; r < kTN; r += kTileThreads / 32) {
        const int n = n_tile + r, m = m_tile + lane * 4;
        if (n < N && m < M) *reinterpret_cast<uint32_t*>(y_t + (int64_t)n * M + m) = tile_t[r][lane];
    }
}

// =================================================================================================
// host side
// =================================================================================================
bool qb_ok(int QB) { return QB == 16 || QB == 32 || QB == 64 || QB == 128; }
bool scale_dtype_ok(int d) { return d == COAT_F32 || d == COAT_BF16 || d == COAT_F16; }

// Calls f.template run<T, FMT, IEEE>() for the runtime (in_dtype, fmt, flags) triple.
template <typename F>
int dispatch(int in_dtype, int fmt, int flags, F&& f) {
    const bool ieee = flags & COAT_QUANT_IEEE_DIV;
#define COAT_CASE(T)                                                                         \
    if (fmt == COAT_E4M3) return ieee ? f.template run<T, COAT_E4M3, true>() : f.template run<T, COAT_E4M3, false>(); \
    if (fmt == COAT_E5M2) return ieee ? f.template run<T, COAT_E5M2, true>() : f.template run<T, COAT_E5M2, false>(); \
    return COAT_E_BADARG;
    switch (in_dtype) {
        case COAT_BF16: { COAT_CASE(__nv_bfloat16) }
        case COAT_F16: { COAT_CASE(__half) }
        case COAT_F32: { COAT_CASE(float) }
        default: return COAT_E_BADARG;
    }
#undef COAT_CASE
}

int elem_size(int dtype) { return dtype == COAT_F32 ? 4 : 2; }

struct GroupQuantArgs {
    const void* x; uint8_t* y; void* s; int scale_dtype; unsigned int* amax; int64_t M, N, ldx; int QB; int mode;
    cudaStream_t st;
    template <typename T, int FMT, bool IEEE> int run() const {
        const unsigned grid = straight_grid(M * (N / 16));
        if (mode == 0)
            group_quantize_kernel<T, FMT, IEEE, 0><<<grid, kStraightThreads, 0, st>>>(
                reinterpret_cast<const T*>(x), y, s, scale_dtype, nullptr, M, N, ldx, N, QB);
        else if (!s)
            tensor_amax_kernel<T><<<(unsigned)((M * (N / 16) + kStraightThreads * kAmaxSegs - 1) /
                                               (kStraightThreads * kAmaxSegs)), kStraightThreads, 0, st>>>(
                reinterpret_cast<const T*>(x), amax, M, N, ldx);
        else
            group_quantize_kernel<T, FMT, IEEE, 1><<<grid, kStraightThreads, 0, st>>>(
                reinterpret_cast<const T*>(x), nullptr, s, scale_dtype, amax, M, N, ldx, N, QB);
        return coat_launch_status();
    }
};

struct DivisionArgs {
    const void* x; uint8_t* y; uint8_t* y_t; const void* s_in; void* s_out; int scale_dtype; const unsigned int* amax;
    int64_t M, N, ldx; cudaStream_t st; bool stochastic;
    template <typename T, int FMT, bool IEEE> int run() const {
        if (stochastic) {
            // rare path: the straight kernel, then (the noise depends on the element's position only, so the
            // transposed copy holds the same codes) a byte transpose of its output
            division_kernel<T, FMT, IEEE, true><<<straight_grid(M * (N / 16)), kStraightThreads, 0, st>>>(
                reinterpret_cast<const T*>(x), y, s_in, s_out, scale_dtype, amax, M, N, ldx, N);
            if (int rc = coat_launch_status()) return rc;
            return y_t ? coat_fp8_transpose(y, y_t, M, N, st) : COAT_OK;
        }
        if (!y_t) {
            division_kernel<T, FMT, IEEE, false><<<straight_grid(M * (N / 16)), kStraightThreads, 0, st>>>(
                reinterpret_cast<const T*>(x), y, s_in, s_out, scale_dtype, amax, M, N, ldx, N);
            return coat_launch_status();
        }
        if (M % 16 == 0 && coat_aligned(y_t, 16) && (!y || coat_aligned(y, 16)) && tma_tiles_fit(M, N)) {
            if (y)
                return launch_transpose_tma<T, FMT, IEEE, false, true>(x, y, y_t, nullptr, nullptr, s_in, s_out,
                                                                       scale_dtype, amax, M, N, ldx, st);
            return launch_transpose_tma<T, FMT, IEEE, false, false>(x, nullptr, y_t, nullptr, nullptr, s_in, s_out,
                                                                    scale_dtype, amax, M, N, ldx, st);
        }
        const dim3 grid((unsigned)((N + kTN - 1) / kTN), (unsigned)((M + kTM - 1) / kTM));
        if (y)
            transpose_quant_kernel<T, FMT, IEEE, false, true><<<grid, kTileThreads, 0, st>>>(
                reinterpret_cast<const T*>(x), y, y_t, nullptr, nullptr, s_in, s_out, scale_dtype, amax, (int)M, (int)N, ldx);
        else
            transpose_quant_kernel<T, FMT, IEEE, false, false><<<grid, kTileThreads, 0, st>>>(
                reinterpret_cast<const T*>(x), nullptr, y_t, nullptr, nullptr, s_in, s_out, scale_dtype, amax, (int)M, (int)N, ldx);
        return coat_launch_status();
    }
};

struct QuantTransposeArgs {
    const void* x; uint8_t* y; uint8_t* y_t; void* s_y; void* s_y_t; int scale_dtype; int64_t M, N, ldx; cudaStream_t st;
    template <typename T, int FMT, bool IEEE> int run() const {
        if (coat_aligned(y, 16) && coat_aligned(y_t, 16) && tma_tiles_fit(M, N))   // M is a multiple of 16 here
            return launch_transpose_tma<T, FMT, IEEE, true, true>(x, y, y_t, s_y, s_y_t, nullptr, nullptr, scale_dtype,
                                                                  nullptr, M, N, ldx, st);
        const dim3 grid((unsigned)((N + kTN - 1) / kTN), (unsigned)((M + kTM - 1) / kTM));
        transpose_quant_kernel<T, FMT, IEEE, true, true><<<grid, kTileThreads, 0, st>>>(
            reinterpret_cast<const T*>(x), y, y_t, s_y, s_y_t, nullptr, nullptr, scale_dtype, nullptr, (int)M, (int)N, ldx);
        return coat_launch_status();
    }
};

struct PertensorFusedArgs {
    const void* x; uint8_t* y; uint8_t* y_t; void* s_y; void* s_out; int scale_dtype; unsigned int* sync; int64_t M, N, ldx;
    int QB; cudaStream_t st;
    template <typename T, int FMT, bool IEEE> int run() const {
        if (y_t) {
            if (y) return launch_transpose_tma_fused<T, FMT, IEEE, true>(x, y, y_t, s_out, scale_dtype, sync, M, N, ldx, st);
            return launch_transpose_tma_fused<T, FMT, IEEE, false>(x, nullptr, y_t, s_out, scale_dtype, sync, M, N, ldx, st);
        }
        auto kern = pertensor_fused_kernel<T, FMT, IEEE>;
        static int ctas_per_sm = 0;   // per instantiation; every B200 of a process gives the same answer
        if (ctas_per_sm == 0) {
            int n = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kStraightThreads, 0) != cudaSuccess || n < 1)
                return COAT_E_LAUNCH;
            ctas_per_sm = n;
        }
        constexpr int64_t kStep = (int64_t)kStraightThreads * kFusedUnroll;
        const int64_t total = M * (N / 16);
        const int64_t resident = (int64_t)coat_sm_count() * ctas_per_sm;   // every SM gets the same number of CTAs
        int64_t grid = (total + kStep - 1) / kStep;
        if (grid > resident) grid = resident;
        const int64_t segs_per_cta = ((total + grid - 1) / grid + 7) / 8 * 8;   // equal slices, group-aligned
        grid = (total + segs_per_cta - 1) / segs_per_cta;
        // cooperative: the launch fails instead of waiting at the barrier if the grid cannot be co-resident
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)grid);
        cfg.blockDim = dim3(kStraightThreads);
        cfg.stream = st;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeCooperative;
        attr.val.cooperative = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        if (cudaLaunchKernelEx(&cfg, kern, reinterpret_cast<const T*>(x), y, s_y, s_out, scale_dtype, sync, M, N, ldx, QB,
                               segs_per_cta) != cudaSuccess) {
            cudaGetLastError();
            return COAT_E_LAUNCH;
        }
        return coat_launch_status();
    }
};

int check_2d(const void* x, int64_t M, int64_t N, int64_t ldx, int in_dtype, int QB) {
    if (M < 0 || N < 0 || ldx < N) return COAT_E_BADARG;
    if (!qb_ok(QB) || N % QB != 0) return COAT_E_SHAPE;
    // 16-element row segments are moved with 16-byte vector accesses
    if (!coat_aligned(x, 16) || (ldx * elem_size(in_dtype)) % 16 != 0) return COAT_E_ALIGN;
    return COAT_OK;
}

}  // namespace

extern "C" int coat_fp8_quantize(const void* x, uint8_t* y, void* s_y, int64_t M, int64_t N, int64_t ldx, int QB,
                                 int fmt, int in_dtype, int scale_dtype, int flags, void* stream) {
    if (M == 0 || N == 0) return COAT_OK;
    if (!x || !y || !s_y || !scale_dtype_ok(scale_dtype)) return COAT_E_BADARG;
    if (int rc = check_2d(x, M, N, ldx, in_dtype, QB)) return rc;
    if (!coat_aligned(y, 16)) return COAT_E_ALIGN;
    GroupQuantArgs a{x, y, s_y, scale_dtype, nullptr, M, N, ldx, QB, 0, (cudaStream_t)stream};
    return dispatch(in_dtype, fmt, flags, a);
}

extern "C" int coat_fp8_group_scales_amax(const void* x, void* s_y, unsigned int* amax_bits, int64_t M, int64_t N,
                                          int64_t ldx, int QB, int fmt, int in_dtype, int scale_dtype, int flags,
                                          void* stream) {
    if (!amax_bits) return COAT_E_BADARG;
    if (cudaMemsetAsync(amax_bits, 0, sizeof(unsigned int), (cudaStream_t)stream) != cudaSuccess) return COAT_E_LAUNCH;
    if (M == 0 || N == 0) return COAT_OK;
    if (!x || !scale_dtype_ok(scale_dtype)) return COAT_E_BADARG;
    if (int rc = check_2d(x, M, N, ldx, in_dtype, QB)) return rc;
    GroupQuantArgs a{x, nullptr, s_y, scale_dtype, amax_bits, M, N, ldx, QB, 1, (cudaStream_t)stream};
    return dispatch(in_dtype, fmt, flags, a);
}

extern "C" int coat_fp8_division(const void* x, uint8_t* y, uint8_t* y_t, const void* s_in, void* s_out,
                                 const unsigned int* amax_bits, int64_t M, int64_t N, int64_t ldx, int fmt,
                                 int in_dtype, int scale_dtype, int flags, void* stream) {
    if (M == 0 || N == 0) return COAT_OK;
    if (!x || (!y && !y_t) || (!s_in && !amax_bits) || !scale_dtype_ok(scale_dtype)) return COAT_E_BADARG;
    if (int rc = check_2d(x, M, N, ldx, in_dtype, 16)) return rc;
    if ((y && !coat_aligned(y, 16)) || (y_t && (!coat_aligned(y_t, 4) || M % 4 != 0))) return COAT_E_ALIGN;
    const bool stochastic = flags & COAT_QUANT_STOCHASTIC;
    if (stochastic && !y) return COAT_E_BADARG;   // the transposed copy is made from y
    DivisionArgs a{x, y, y_t, s_in, s_out, scale_dtype, amax_bits, M, N, ldx, (cudaStream_t)stream, stochastic};
    return dispatch(in_dtype, fmt, flags, a);
}

extern "C" int coat_fp8_quantize_pertensor(const void* x, uint8_t* y, uint8_t* y_t, void* s_y, void* s_out,
                                           unsigned int* sync_words, int64_t M, int64_t N, int64_t ldx, int QB, int fmt,
                                           int in_dtype, int scale_dtype, int flags, void* stream) {
    if (M == 0 || N == 0) return COAT_OK;
    if (!x || (!y && !y_t) || !s_out || !sync_words || !scale_dtype_ok(scale_dtype)) return COAT_E_BADARG;
    if (int rc = check_2d(x, M, N, ldx, in_dtype, QB)) return rc;
    if ((y && !coat_aligned(y, 16)) || !coat_aligned(sync_words, 4)) return COAT_E_ALIGN;
    if (y_t) {   // the tile kernel: no group scales, 16-row granularity, 16-byte aligned transposed rows
        if (s_y) return COAT_E_BADARG;
        if (M % 16 != 0 || !tma_tiles_fit(M, N)) return COAT_E_SHAPE;
        if (!coat_aligned(y_t, 16)) return COAT_E_ALIGN;
    }
    PertensorFusedArgs a{x, y, y_t, s_y, s_out, scale_dtype, sync_words, M, N, ldx, QB, (cudaStream_t)stream};
    return dispatch(in_dtype, fmt, flags, a);
}

// Synchronises, returns and clears the quantizers' device status word (COAT_E_TIMEOUT if a bounded wait ran out).
extern "C" int coat_fp8_quantize_device_status(void) {
    int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_quant_device_status, sizeof(int)) != cudaSuccess) return COAT_E_LAUNCH;
    if (v != 0 && cudaMemcpyToSymbol(g_quant_device_status, &zero, sizeof(int)) != cudaSuccess) return COAT_E_LAUNCH;
    return v;
}

// fp8_mul_forward with a per-tensor output in one cooperative launch (see mul_pertensor_tma_kernel): q = fp8(bf16((c1 s1)(c2 s2)) / s),
// q_t its transpose, *s_out = s = the maximum of the rounded 1xQB group scales of the product.  sync_words as for
// coat_fp8_quantize_pertensor.  COAT_E_SHAPE unless QB == 16, M % 16 == 0 and N % 128 == 0 (use coat_fp8_mul_forward +
// coat_fp8_division there); scales must be bf16.
extern "C" int coat_fp8_mul_forward_pertensor(const uint8_t* x1, const void* s_x1, const uint8_t* x2, const void* s_x2,
                                              uint8_t* y, uint8_t* y_t, void* s_out, unsigned int* sync_words, int64_t M,
                                              int64_t N, int QB, int fmt, int scale_dtype, int flags, void* stream) {
    if (M < 0 || N < 0 || (fmt != COAT_E4M3 && fmt != COAT_E5M2)) return COAT_E_BADARG;
    if (M == 0 || N == 0) return COAT_OK;
    if (!x1 || !s_x1 || !x2 || !s_x2 || !y || !y_t || !s_out || !sync_words) return COAT_E_BADARG;
    if (scale_dtype != COAT_BF16 || (flags & COAT_QUANT_STOCHASTIC)) return COAT_E_BADARG;
    if (QB != 16 || M % 16 != 0 || N % 128 != 0 || !tma_tiles_fit(M, N)) return COAT_E_SHAPE;
    if (!coat_aligned(x1, 16) || !coat_aligned(x2, 16) || !coat_aligned(s_x1, 16) || !coat_aligned(s_x2, 16) ||
        !coat_aligned(y, 16) || !coat_aligned(y_t, 16)) return COAT_E_ALIGN;
    cudaStream_t st = (cudaStream_t)stream;
    const bool ieee = flags & COAT_QUANT_IEEE_DIV;
    if (fmt == COAT_E4M3)
        return ieee ? launch_mul_pertensor<COAT_E4M3, true>(x1, s_x1, x2, s_x2, y, y_t, s_out, scale_dtype, sync_words, M, N, st)
                    : launch_mul_pertensor<COAT_E4M3, false>(x1, s_x1, x2, s_x2, y, y_t, s_out, scale_dtype, sync_words, M, N, st);
    return ieee ? launch_mul_pertensor<COAT_E5M2, true>(x1, s_x1, x2, s_x2, y, y_t, s_out, scale_dtype, sync_words, M, N, st)
                : launch_mul_pertensor<COAT_E5M2, false>(x1, s_x1, x2, s_x2, y, y_t, s_out, scale_dtype, sync_words, M, N, st);
}

// Diagnostic: number of polls a CTA spends at the grid barrier of the one-launch per-tensor kernels before it gives up
// (on the current device; polls < 0 restores the default of about a second).
extern "C" int coat_fp8_quantize_set_barrier_limit(int polls) {
    const int v = polls < 0 ? kBarrierLimitDefault : polls;
    return cudaMemcpyToSymbol(g_barrier_limit, &v, sizeof(int)) == cudaSuccess ? COAT_OK : COAT_E_LAUNCH;
}

extern "C" int coat_fp8_quantize_transpose(const void* x, uint8_t* y, void* s_y, uint8_t* y_t, void* s_y_t, int64_t M,
                                           int64_t N, int64_t ldx, int QB, int fmt, int in_dtype, int scale_dtype,
                                           int flags, void* stream) {
    if (M == 0 || N == 0) return COAT_OK;
    if (!x || !y || !s_y || !y_t || !s_y_t || !scale_dtype_ok(scale_dtype)) return COAT_E_BADARG;
    if (QB != 16) return COAT_E_SHAPE;   // the tile mapping fixes 1x16 groups (the only size the models use)
    if (int rc = check_2d(x, M, N, ldx, in_dtype, QB)) return rc;
    if (M % QB != 0) return COAT_E_SHAPE;
    if (!coat_aligned(y, 4) || !coat_aligned(y_t, 4)) return COAT_E_ALIGN;
    QuantTransposeArgs a{x, y, y_t, s_y, s_y_t, scale_dtype, M, N, ldx, (cudaStream_t)stream};
    return dispatch(in_dtype, fmt, flags, a);
}

extern "C" int coat_fp8_transpose(const uint8_t* x, uint8_t* y_t, int64_t M, int64_t N, void* stream) {
    if (M == 0 || N == 0) return COAT_OK;
    if (!x || !y_t || M < 0 || N < 0) return COAT_E_BADARG;
    if (M % 4 != 0 || N % 4 != 0) return COAT_E_SHAPE;
    if (!coat_aligned(x, 4) || !coat_aligned(y_t, 4)) return COAT_E_ALIGN;
    const dim3 grid((unsigned)((N + kTN - 1) / kTN), (unsigned)((M + kTM - 1) / kTM));
    transpose_bytes_kernel<<<grid, kTileThreads, 0, (cudaStream_t)stream>>>(x, y_t, (int)M, (int)N);
    return coat_launch_status();
}

extern "C" int coat_fp8_dequantize(const uint8_t* x, const void* s_x, void* y_bf16, int64_t M, int64_t N, int QB,
                                   int fmt, int scale_dtype, void* stream) {
    if (M == 0 || N == 0) return COAT_OK;
    if (!x || !s_x || !y_bf16 || !scale_dtype_ok(scale_dtype)) return COAT_E_BADARG;
    if (!qb_ok(QB) || N % QB != 0) return COAT_E_SHAPE;
    if (!coat_aligned(x, 16) || !coat_aligned(y_bf16, 16)) return COAT_E_ALIGN;
    const unsigned grid = straight_grid(M * (N / 16));
    if (fmt == COAT_E4M3)
        dequantize_kernel<COAT_E4M3><<<grid, kStraightThreads, 0, (cudaStream_t)stream>>>(
            x, s_x, scale_dtype, reinterpret_cast<__nv_bfloat16*>(y_bf16), M, N, QB);
    else if (fmt == COAT_E5M2)
        dequantize_kernel<COAT_E5M2><<<grid, kStraightThreads, 0, (cudaStream_t)stream>>>(
            x, s_x, scale_dtype, reinterpret_cast<__nv_bfloat16*>(y_bf16), M, N, QB);
    else
        return COAT_E_BADARG;
    return coat_launch_status();
}

namespace {

// =================================================================================================
// Per-tensor quantize that allocates nothing
// =================================================================================================
// Who this is for: a host that may not allocate device memory at the point where it quantizes, and
// cannot reserve a scratch word ahead of time either.  Examples are a plugin that has been handed a
// fixed memory budget by the framework around it, a host written without a caching allocator where the
// only way to get four bytes is cudaMalloc, and code that runs in a latency-critical section between
// other GPU work, where cudaMalloc / cudaFree would synchronise the whole device.  The ordinary entry
// points above need the caller to pass a 4-byte scratch word for the tensor's amax; this one keeps its
// scratch in the library image instead.
//
// The scratch is the file-scope array below: one partial maximum per CTA of the first pass, then the
// reduced maximum in the slot after the last partial.  It is part of the loaded library, so every GPU
// that loads the library holds these ~17 KB until the process exits.  Its size fixes the largest input:
// kStaticMaxCtas CTAs of kStaticChunk elements each.
//
// Sharing: every call on a device uses the same array, and it keeps whatever the previous call left
// there.  Nothing in it has to start at zero (each call overwrites every slot it later reads: its own
// partials, then the reduced word), but two calls whose kernels overlap on the GPU - different streams,
// or different host threads - race on it and can corrupt each other's scale.  Calls on one stream are
// safe back to back.
constexpr int kStaticMaxCtas = 4096;
constexpr int kStaticSegsPerThread = 4;
constexpr int64_t kStaticChunk = (int64_t)kStraightThreads * 16 * kStaticSegsPerThread;   // 16384 elements per CTA
constexpr int64_t kStaticMaxElements = kStaticChunk * kStaticMaxCtas;                     // 67 108 864

static __device__ __align__(256) float g_pertensor_scratch[kStaticMaxCtas + 64];

// first pass: CTA b reduces |x| over its chunk of 16-element row segments into scratch[b]
template <typename T>
__global__ void __launch_bounds__(kStraightThreads)
static_partial_amax_kernel(const T* __restrict__ x, float* __restrict__ partials, int64_t M, int64_t N, int64_t ldx) {
    const int64_t segs_per_row = N >> 4;
    const int64_t total = M * segs_per_row;
    const int64_t first = (int64_t)blockIdx.x * kStraightThreads * kStaticSegsPerThread;
    float amax = 0.f;
#pragma unroll
    for (int k = 0; k < kStaticSegsPerThread; ++k) {
        const int64_t seg = first + (int64_t)k * kStraightThreads + threadIdx.x;
        if (seg < total) {
            float v[16];
            Seg16<T>::load(x + seg_offset(seg, segs_per_row, ldx), v);
#pragma unroll
            for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
        }
    }
    amax = coat_warp_max(amax);
    __shared__ float wmax[kStraightThreads / 32];
    if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = amax;
    __syncthreads();
    if (threadIdx.x < 32) {
        float m = threadIdx.x < kStraightThreads / 32 ? wmax[threadIdx.x] : 0.f;
        m = coat_warp_max(m);
        if (threadIdx.x == 0) partials[blockIdx.x] = m;
    }
}

// second step: one CTA folds the partials into the word the division kernels read (bit pattern of a
// non-negative float), stored right after the last partial slot
__global__ void __launch_bounds__(kStraightThreads)
static_reduce_amax_kernel(float* __restrict__ scratch, int n_partials) {
    float m = 0.f;
    for (int i = threadIdx.x; i < n_partials; i += kStraightThreads) m = fmaxf(m, scratch[i]);
    m = coat_warp_max(m);
    __shared__ float wmax[kStraightThreads / 32];
    if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        float r = threadIdx.x < kStraightThreads / 32 ? wmax[threadIdx.x] : 0.f;
        r = coat_warp_max(r);
        if (threadIdx.x == 0) reinterpret_cast<unsigned int*>(scratch)[kStaticMaxCtas] = __float_as_uint(r);
    }
}

// In host code the name g_pertensor_scratch is only a stand-in for the device array, not an address a
// kernel can use; the address comes from cudaGetSymbolAddress, once per device, with that device current.
int static_scratch_address(float** out) {
    static float* cached[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return COAT_E_DEVICE;
    if (!cached[dev]) {
        float* p = nullptr;
        if (cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_pertensor_scratch) != cudaSuccess || !p)
            return COAT_E_LAUNCH;
        cached[dev] = p;
    }
    *out = cached[dev];
    return COAT_OK;
}

struct StaticAmaxArgs {
    const void* x; float* scratch; int64_t M, N, ldx; int n_ctas; cudaStream_t st;
    template <typename T, int FMT, bool IEEE> int run() const {
        static_partial_amax_kernel<T><<<n_ctas, kStraightThreads, 0, st>>>(reinterpret_cast<const T*>(x), scratch, M, N, ldx);
        static_reduce_amax_kernel<<<1, kStraightThreads, 0, st>>>(scratch, n_ctas);
        return coat_launch_status();
    }
};

}  // namespace

// Per-tensor quantize (optionally with the transposed copy) without any allocation and without a
// caller-provided scratch word; see the block comment above for who needs it, the size limit and the
// sharing rules.  Same results as coat_fp8_group_scales_amax(s_y = NULL) followed by coat_fp8_division
// with that amax word.  y or y_t may be NULL (not both); *s_out receives the scale.  Returns
// COAT_E_TOOBIG if M*N exceeds 67 108 864 elements.  The first call on a device looks up the address
// of the scratch array (a runtime query, no allocation); make that first call before starting any
// stream capture on that device.
extern "C" int coat_fp8_quantize_pertensor_static(const void* x, uint8_t* y, uint8_t* y_t, void* s_out, int64_t M,
                                                  int64_t N, int64_t ldx, int fmt, int in_dtype, int scale_dtype,
                                                  int flags, void* stream) {
    if (flags & COAT_QUANT_STOCHASTIC) return COAT_E_BADARG;   // round-to-nearest only: rejected, not ignored
    if (M == 0 || N == 0) return COAT_OK;
    if (!x || (!y && !y_t) || !s_out || !scale_dtype_ok(scale_dtype)) return COAT_E_BADARG;
    if (int rc = check_2d(x, M, N, ldx, in_dtype, 16)) return rc;
    if (M * N > kStaticMaxElements) return COAT_E_TOOBIG;
    if ((y && !coat_aligned(y, 16)) || (y_t && (!coat_aligned(y_t, 4) || M % 4 != 0))) return COAT_E_ALIGN;
    float* scratch = nullptr;
    if (int rc = static_scratch_address(&scratch)) return rc;
    const int64_t segs = M * (N / 16);
    const int n_ctas = (int)((segs + kStraightThreads * kStaticSegsPerThread - 1) / (kStraightThreads * kStaticSegsPerThread));
    StaticAmaxArgs a{x, scratch, M, N, ldx, n_ctas, (cudaStream_t)stream};
    if (int rc = dispatch(in_dtype, fmt, flags, a)) return rc;
    DivisionArgs d{x, y, y_t, nullptr, s_out, scale_dtype,
                   reinterpret_cast<const unsigned int*>(scratch) + kStaticMaxCtas, M, N, ldx, (cudaStream_t)stream,
                   false};
    return dispatch(in_dtype, fmt, flags, d);
}
