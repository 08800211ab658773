// Fused FP8 AdamW step (with and without Dynamic Range Expansion) for sm_100a.
//
// What one step computes, per 128-element group of the flattened tensor, follows
// the reference kernels coat/optimizer/kernels/fp8_adamw_expand_cuda_kernel.cu:42-202
// and coat/optimizer/kernels/fp8_adamw_cuda_kernel.cu:38-124.  How it is computed
// does not: the reference runs one 128-thread block per group with one element per
// thread, scalar 1-byte loads, two block barriers, and every thread recomputing the
// group's pow/log2/sqrt.  Here a WARP owns a group: each lane holds 4 consecutive
// elements (16-byte loads of p and g, 4-byte loads of the two code arrays), group
// statistics are warp-shuffle reductions, the group's scalars are computed once (lane
// 0 for the first moment, lane 1 for the second, same instruction stream) and
// broadcast, the bias corrections are computed once per thread, and a persistent grid
// walks the groups (of one tensor or of a whole table of tensors).
//
// The arithmetic keeps the reference's expression forms (including the double-typed
// 1e-30 / 1e-20 additions and the int->float promotions) so that nvcc makes the same
// contraction decisions and the quantized state comes out bit-identical.

#include <math.h>

#include <cstddef>
#include <type_traits>

#include "common.cuh"

namespace {

constexpr int kGroup = 128;          // elements per quantization group
constexpr int kThreads = 256;        // 8 warps per CTA
constexpr int kWarpsPerCta = kThreads / COAT_WARP;

struct AdamwHyper {
    float beta1, beta2, lr, wd, eps;
    int step;
    int expand_min;
    // Broadcast of the bf16 weight copy: besides bf16_out itself, every bf16 store is repeated at
    // bf16_out + peer_delta[i] bytes (the same slot of another GPU's buffer, mapped into this process).
    int n_peers;
    long long peer_delta[COAT_MAX_PEERS];
};

// bf16 copy of 4 updated weights: the local store, then the same 8 bytes to every peer (plain stores over
// NVLink; nothing here waits on a peer)
template <bool BCAST>
__device__ __forceinline__ void store_bf16x4_bcast(__nv_bfloat16* dst, const float (&q)[4], const AdamwHyper& h) {
    uint2 t;
    const __nv_bfloat162 lo = __floats2bfloat162_rn(q[0], q[1]), hi = __floats2bfloat162_rn(q[2], q[3]);
    t.x = *reinterpret_cast<const uint32_t*>(&lo);
    t.y = *reinterpret_cast<const uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(dst) = t;
    if constexpr (BCAST)
        for (int i = 0; i < h.n_peers; ++i)
            *reinterpret_cast<uint2*>(reinterpret_cast<char*>(dst) + h.peer_delta[i]) = t;
}
template <bool BCAST>
__device__ __forceinline__ void store_bf16_bcast(__nv_bfloat16* dst, float x, const AdamwHyper& h) {
    const __nv_bfloat16 b = __float2bfloat16_rn(x);
    *dst = b;
    if constexpr (BCAST)
        for (int i = 0; i < h.n_peers; ++i)
            *reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<char*>(dst) + h.peer_delta[i]) = b;
}

// One tensor's pointers (single-tensor launch passes this by value; the table launch
// reads it from global memory).
typedef CoatAdamwTensor TensorDesc;

// ---- loads / stores of 4 consecutive parameter-typed elements -------------------

template <typename T> struct Elem4;
template <> struct Elem4<float> {
    static __device__ __forceinline__ void load(const float* p, float (&x)[4]) {
        float4 t = *reinterpret_cast<const float4*>(p);
        x[0] = t.x; x[1] = t.y; x[2] = t.z; x[3] = t.w;
    }
    static __device__ __forceinline__ void load_stream(const float* p, float (&x)[4]) {
        float4 t = __ldcs(reinterpret_cast<const float4*>(p));
        x[0] = t.x; x[1] = t.y; x[2] = t.z; x[3] = t.w;
    }
    static __device__ __forceinline__ void store(float* p, const float (&x)[4]) {
        *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
    }
    static __device__ __forceinline__ float get(const float* p) { return *p; }
    static __device__ __forceinline__ void put(float* p, float x) { *p = x; }
    static __device__ __forceinline__ float round(float x) { return x; }
    static constexpr int kVecAlign = 16;
};
template <> struct Elem4<__nv_bfloat16> {
    static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&x)[4]) {
        uint2 t = *reinterpret_cast<const uint2*>(p);
        x[0] = __uint_as_float(t.x << 16); x[1] = __uint_as_float(t.x & 0xffff0000u);
        x[2] = __uint_as_float(t.y << 16); x[3] = __uint_as_float(t.y & 0xffff0000u);
    }
    static __device__ __forceinline__ void load_stream(const __nv_bfloat16* p, float (&x)[4]) {
        uint2 t = __ldcs(reinterpret_cast<const uint2*>(p));
        x[0] = __uint_as_float(t.x << 16); x[1] = __uint_as_float(t.x & 0xffff0000u);
        x[2] = __uint_as_float(t.y << 16); x[3] = __uint_as_float(t.y & 0xffff0000u);
    }
    static __device__ __forceinline__ void store(__nv_bfloat16* p, const float (&x)[4]) {
        uint2 t;
        t.x = (uint32_t)coat_float_to_bf16_bits(x[0]) | ((uint32_t)coat_float_to_bf16_bits(x[1]) << 16);
        t.y = (uint32_t)coat_float_to_bf16_bits(x[2]) | ((uint32_t)coat_float_to_bf16_bits(x[3]) << 16);
        *reinterpret_cast<uint2*>(p) = t;
    }
    static __device__ __forceinline__ float get(const __nv_bfloat16* p) { return __bfloat162float(*p); }
    static __device__ __forceinline__ void put(__nv_bfloat16* p, float x) { *p = __float2bfloat16_rn(x); }
    static __device__ __forceinline__ float round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
    static constexpr int kVecAlign = 8;
};
template <> struct Elem4<__half> {
    static __device__ __forceinline__ void load(const __half* p, float (&x)[4]) {
        uint2 t = *reinterpret_cast<const uint2*>(p);
        float2 a = __half22float2(*reinterpret_cast<__half2*>(&t.x));
        float2 b = __half22float2(*reinterpret_cast<__half2*>(&t.y));
        x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
    }
    static __device__ __forceinline__ void load_stream(const __half* p, float (&x)[4]) { load(p, x); }
    static __device__ __forceinline__ void store(__half* p, const float (&x)[4]) {
        __half2 a = __floats2half2_rn(x[0], x[1]);
        __half2 b = __floats2half2_rn(x[2], x[3]);
        uint2 t;
        t.x = *reinterpret_cast<uint32_t*>(&a);
        t.y = *reinterpret_cast<uint32_t*>(&b);
        *reinterpret_cast<uint2*>(p) = t;
    }
    static __device__ __forceinline__ float get(const __half* p) { return __half2float(*p); }
    static __device__ __forceinline__ void put(__half* p, float x) { *p = __float2half_rn(x); }
    static __device__ __forceinline__ float round(float x) { return __half2float(__float2half_rn(x)); }
    static constexpr int kVecAlign = 8;
};

// ---- the reference's order-dependent "skip incoming zeros" minimum ---------------
// fp8_adamw_expand_cuda_kernel.cu:89-103 and :119-137 reduce with
//   own = (|incoming| > 0) ? fmin(own, |incoming|) : own
// over shfl_down trees (offsets 16..1 inside each 32-element chunk, then the four
// chunk results, sitting in lanes 0..3 of a warp whose other lanes hold 1e9, with the
// same tree).  A zero that arrives is skipped but a lane's own zero sticks, so when a
// group holds an exact zero the result depends on where it sits.  With no exact zero
// the whole thing is min(plain minimum, 1e9).
__device__ __forceinline__ float ref_min_combine(float own, float incoming) {
    float a = fabsf(incoming);
    return (a > 0) ? fminf(own, a) : own;
}

// Serial emulation of the tree over 128 values held in shared memory (one lane runs it;
// only groups that contain an exact zero come here).
__device__ float ref_min_tree_128(float* buf /*[128], clobbered*/) {
    float chunk[4];
    for (int w = 0; w < 4; ++w) {
        float* a = buf + 32 * w;
        for (int s = 16; s > 0; s >>= 1)
            for (int l = 0; l < s; ++l) a[l] = ref_min_combine(a[l], a[l + s]);
        chunk[w] = a[0];
    }
    // lanes 0..3 hold the chunk results, lanes 4..31 hold 1e9; offsets 16, 8, 4 combine
    // each of lanes 0..3 with a 1e9 lane (three times, idempotent), then 2, then 1.
    for (int w = 0; w < 4; ++w) chunk[w] = ref_min_combine(chunk[w], 1e9f);
    float a = ref_min_combine(chunk[0], chunk[2]);
    float b = ref_min_combine(chunk[1], chunk[3]);
    return ref_min_combine(a, b);
}

// m' = beta1*m + (1-beta1)*g and v' = beta2*v + ((1-beta2)*g)*g  (fp8_adamw_expand_cuda_kernel.cu:52-55)
__device__ __forceinline__ float adam_first(float beta1, float m, float om_beta1, float g) {
    return __fmaf_rn(beta1, m, __fmul_rn(om_beta1, g));
}
__device__ __forceinline__ float adam_second(float beta2, float v, float om_beta2, float g) {
    return __fmaf_rn(beta2, v, __fmul_rn(__fmul_rn(om_beta2, g), g));
}

// ---- per-group scalars of the expansion ------------------------------------------
// fp8_adamw_expand_cuda_kernel.cu:151-181.  QUANT_MIN_VAL is a double literal there, so
// the additions are done in double and rounded back to float.
#define COAT_EXPAND_MIN_VAL 1e-30
#define COAT_PLAIN_MIN_VAL 1e-20

// x + 1e-30 evaluated in double and rounded back to float, as the reference's expression does.  For x >= 2^-70 the
// addend is below a quarter of x's last place, so the rounded sum is x itself: the double-precision unit (slow on
// this GPU) is only used for smaller, zero, negative or NaN inputs.
__device__ __forceinline__ float coat_add_expand_min_val(float x) {
    if (x >= 8.4703295e-22f /* 2^-70 */ && x <= 3.0e38f) return x;
    return x + COAT_EXPAND_MIN_VAL;
}

__device__ __forceinline__ void expand_group_scalars(float absmax, float absmin, int expand_min,
                                                     float& maxv, float& sqrt_minmax, float& expo,
                                                     float& new_scale) {
    float fp8MaxVal = 448;
    float firstMaxVal = coat_add_expand_min_val(absmax);
    float firstMinVal = coat_add_expand_min_val(absmin);
    float firstRatio = firstMaxVal / firstMinVal;
    float firstSqrtMinMax = sqrt(firstMaxVal) * sqrt(firstMinVal);
    float ratioUpperBound = fp8MaxVal * fp8MaxVal / 2;
    float firstExp = floor((log2f(ratioUpperBound) / log2f(firstRatio)) * expand_min) / expand_min;
    float new_scale_exp_avg = powf(firstMaxVal / firstSqrtMinMax, firstExp) / fp8MaxVal;
    maxv = firstMaxVal;
    sqrt_minmax = firstSqrtMinMax;
    expo = firstExp;
    new_scale = new_scale_exp_avg;
}

// ---- one group, exact arithmetic ---------------------------------------------------
// `lane` owns elements [base, base+4) of the tensor; `nvalid` of them (0..4) exist.
template <typename scalar_t, bool EXPAND, bool BCAST>
__device__ __noinline__ void process_group_exact(const TensorDesc& t, int64_t group, int lane,
                                                    const AdamwHyper& h, float om_beta1,
                                                    float om_beta2, float correction1,
                                                    float correction2_sqrt, bool vec_ok,
                                                    float* smem_min /*[128] per warp*/) {
    typedef Elem4<scalar_t> E;
    const int64_t base = group * kGroup + lane * 4;
    const int64_t remaining = t.numel - base;
    const int nvalid = remaining >= 4 ? 4 : (remaining > 0 ? (int)remaining : 0);
    scalar_t* pp = reinterpret_cast<scalar_t*>(t.p) + base;
    const scalar_t* gp = reinterpret_cast<const scalar_t*>(t.g) + base;

    float p[4], g[4], fm[4], fv[4];
    uint32_t mw = 0, vw = 0;
    if (nvalid == 4 && vec_ok) {
        E::load(pp, p);
        E::load_stream(gp, g);
        mw = *reinterpret_cast<const uint32_t*>(t.m + base);
        vw = *reinterpret_cast<const uint32_t*>(t.v + base);
    } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            p[j] = 0.f; g[j] = 0.f;
            if (j < nvalid) {
                p[j] = E::get(pp + j);
                g[j] = E::get(gp + j);
                mw |= (uint32_t)t.m[base + j] << (8 * j);
                vw |= (uint32_t)t.v[base + j] << (8 * j);
            }
        }
    }
    coat_fp8x4_to_float4<COAT_E4M3>(mw, fm);
    coat_fp8x4_to_float4<COAT_E4M3>(vw, fv);

    const float scale_m = t.s_m[group];
    const float scale_v = t.s_v[group];
    float inv_km = 0.f, inv_kv = 0.f, sqm = 0.f, sqv = 0.f;
    if (EXPAND) {
        inv_km = 1 / t.k_m[group];
        inv_kv = 1 / t.k_v[group];
        sqm = t.r_m[group];
        sqv = t.r_v[group];
    }

#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float float_exp_avg = fm[j] * scale_m;
        float float_exp_avg_sq = fv[j] * scale_v;
        if (EXPAND) {
            int sign_exp_avg = 1 - 2 * signbit(float_exp_avg);
            float_exp_avg = sign_exp_avg * powf(fabsf(float_exp_avg), inv_km) * sqm;
            float_exp_avg_sq = powf(float_exp_avg_sq, inv_kv) * sqv;
        }
        // beta1*m + (1-beta1)*g etc. with the contractions nvcc applies to the reference's source
        // written out (they are verified bit for bit against the reference's compiled kernel)
        float_exp_avg = adam_first(h.beta1, float_exp_avg, om_beta1, g[j]);
        float_exp_avg_sq = adam_second(h.beta2, float_exp_avg_sq, om_beta2, g[j]);
        float denom = __fmul_rn(__fadd_rn(__fdiv_rn(__fsqrt_rn(float_exp_avg_sq), correction2_sqrt), h.eps),
                                correction1);
        float update = __fmaf_rn(h.wd, p[j], __fdiv_rn(float_exp_avg, denom));
        p[j] = __fmaf_rn(-h.lr, update, p[j]);
        if (j >= nvalid) { float_exp_avg = 0.0f; float_exp_avg_sq = 0.0f; }
        fm[j] = float_exp_avg;
        fv[j] = float_exp_avg_sq;
    }

    // updated parameters (and the optional bf16 copy)
    if (nvalid == 4 && vec_ok) {
        E::store(pp, p);
        if (t.bf16_out) {
            float q[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) q[j] = E::round(p[j]);
            store_bf16x4_bcast<BCAST>(reinterpret_cast<__nv_bfloat16*>(t.bf16_out) + base, q, h);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (j < nvalid) {
                E::put(pp + j, p[j]);
                if (t.bf16_out)
                    store_bf16_bcast<BCAST>(reinterpret_cast<__nv_bfloat16*>(t.bf16_out) + base + j, E::round(p[j]), h);
            }
    }

    // group statistics
    float mx_m = 0.f, mx_v = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        mx_m = fmaxf(mx_m, fabsf(fm[j]));
        mx_v = fmaxf(mx_v, fabsf(fv[j]));
    }
    mx_m = coat_warp_max(mx_m);
    mx_v = coat_warp_max(mx_v);

    float new_scale_m, new_scale_v;
    float k_m = 0.f, k_v = 0.f, r_m = 0.f, r_v = 0.f;
    if (EXPAND) {
        const float kFltMax = __int_as_float(0x7f7fffff);
        float am[4], av[4];
        bool has_zero = false;
        float mn_m = kFltMax, mn_v = kFltMax;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            am[j] = j < nvalid ? fabsf(fm[j]) : kFltMax;
            av[j] = j < nvalid ? fabsf(fv[j]) : kFltMax;
            // NaN compares false with > 0 as well: route it through the exact tree too
            has_zero |= !(am[j] > 0) | !(av[j] > 0);
            mn_m = fminf(mn_m, am[j]);
            mn_v = fminf(mn_v, av[j]);
        }
        if (__any_sync(COAT_FULL_MASK, has_zero)) {
            float* bm = smem_min;
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 4; ++j) bm[lane * 4 + j] = am[j];
            __syncwarp();
            if (lane == 0) mn_m = ref_min_tree_128(bm);
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 4; ++j) bm[lane * 4 + j] = av[j];
            __syncwarp();
            if (lane == 0) mn_v = ref_min_tree_128(bm);
            __syncwarp();
            mn_m = __shfl_sync(COAT_FULL_MASK, mn_m, 0);
            mn_v = __shfl_sync(COAT_FULL_MASK, mn_v, 0);
        } else {
            mn_m = fminf(coat_warp_min(mn_m), 1e9f);
            mn_v = fminf(coat_warp_min(mn_v), 1e9f);
        }
        // lane 0 derives the first moment's scalars, lane 1 the second's
        float amax = (lane & 1) ? mx_v : mx_m;
        float amin = (lane & 1) ? mn_v : mn_m;
        float maxv, sq, ex, ns;
        expand_group_scalars(amax, amin, h.expand_min, maxv, sq, ex, ns);
        r_m = __shfl_sync(COAT_FULL_MASK, sq, 0);
        r_v = __shfl_sync(COAT_FULL_MASK, sq, 1);
        k_m = __shfl_sync(COAT_FULL_MASK, ex, 0);
        k_v = __shfl_sync(COAT_FULL_MASK, ex, 1);
        new_scale_m = __shfl_sync(COAT_FULL_MASK, ns, 0);
        new_scale_v = __shfl_sync(COAT_FULL_MASK, ns, 1);
    } else {
        float fp8MaxVal = 448;
        float a = mx_m + COAT_PLAIN_MIN_VAL;
        float b = mx_v + COAT_PLAIN_MIN_VAL;
        new_scale_m = a / fp8MaxVal;
        new_scale_v = b / fp8MaxVal;
    }

    float qm[4], qv[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float float_exp_avg = fm[j];
        float float_exp_avg_sq = fv[j];
        if (EXPAND) {
            int sign_exp_avg = 1 - 2 * signbit(float_exp_avg);
            float_exp_avg = sign_exp_avg * powf(fabsf(float_exp_avg) / r_m, k_m);
            float_exp_avg_sq = powf(float_exp_avg_sq / r_v, k_v);
        }
        qm[j] = float_exp_avg / new_scale_m;
        qv[j] = float_exp_avg_sq / new_scale_v;
    }
    uint32_t cm = coat_float4_to_fp8x4<COAT_E4M3>(qm[0], qm[1], qm[2], qm[3]);
    uint32_t cv = coat_float4_to_fp8x4<COAT_E4M3>(qv[0], qv[1], qv[2], qv[3]);
    if (nvalid == 4 && vec_ok) {
        *reinterpret_cast<uint32_t*>(t.m + base) = cm;
        *reinterpret_cast<uint32_t*>(t.v + base) = cv;
    } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (j < nvalid) {
                t.m[base + j] = (uint8_t)(cm >> (8 * j));
                t.v[base + j] = (uint8_t)(cv >> (8 * j));
            }
    }
    if (lane == 0) {
        t.s_m[group] = new_scale_m;
        t.s_v[group] = new_scale_v;
        if (EXPAND) {
            t.k_m[group] = k_m;
            t.k_v[group] = k_v;
            t.r_m[group] = r_m;
            t.r_v[group] = r_v;
        }
    }
}

__device__ __forceinline__ bool desc_vec_ok(const TensorDesc& t, int align) {
    uintptr_t a = reinterpret_cast<uintptr_t>(t.p) | reinterpret_cast<uintptr_t>(t.g);
    uintptr_t c = reinterpret_cast<uintptr_t>(t.m) | reinterpret_cast<uintptr_t>(t.v);
    uintptr_t o = reinterpret_cast<uintptr_t>(t.bf16_out);
    return ((a & (uintptr_t)(align - 1)) | (c & 3) | (o & 7)) == 0;
}

// =====================================================================================
// Guarded fast path of the expansion step
// =====================================================================================
// The exact step spends ~4 libdevice powf per element (dequantise m and v with x^(1/k),
// requantise with x^k), which makes it instruction bound at ~15 % of the HBM roofline.
// The fast path evaluates those four powers as ex2.approx(k * lg2.approx(x)) and keeps
// the QUANTISED RESULT bit-identical to the exact step by bounding the error it makes:
//
//  * every approximate moment m~' carries an absolute error bound delta (from the
//    documented MUFU error bounds, the deviation allowed to libdevice's powf, and the
//    roundings in between; see fast_dequant_eps / requant constants below);
//  * the group maximum and minimum decide the stored scale, exponent and sqrt(max*min),
//    so every element whose interval [m~'-delta, m~'+delta] could hold the maximum or the
//    minimum is recomputed with the exact routine (typically 4 elements of 128), and the
//    group scalars are then computed exactly from exact inputs;
//  * an FP8 code is accepted only if the lower and the upper end of the interval of the
//    scaled value round to the same code; otherwise that element is recomputed exactly;
//  * groups that are not in the regime the bounds were derived for (fresh state, zero /
//    non-finite scales, a possible exact zero or sign change, exponents outside [1/64,64],
//    NaNs, a partial last group, unaligned pointers) take the exact path as a whole.
//
// Only the fp32 weights differ from the exact step, by the relative error of the
// approximate moments (a few 1e-6 of one update), since they are not quantised.

__device__ __forceinline__ float fast_lg2(float x) { float r; asm("lg2.approx.f32 %0, %1;" : "=f"(r) : "f"(x)); return r; }
__device__ __forceinline__ float fast_ex2(float x) { float r; asm("ex2.approx.f32 %0, %1;" : "=f"(r) : "f"(x)); return r; }
__device__ __forceinline__ float fast_rcp(float x) { float r; asm("rcp.approx.f32 %0, %1;" : "=f"(r) : "f"(x)); return r; }
__device__ __forceinline__ float fast_sqrt(float x) { float r; asm("sqrt.approx.f32 %0, %1;" : "=f"(r) : "f"(x)); return r; }

constexpr float kLn2 = 0.6931472f;
constexpr float k2m21 = 4.7683716e-07f, k2m22 = 2.3841858e-07f, k2m23 = 1.1920929e-07f, k2m24 = 5.9604645e-08f;
// lg2.approx: absolute error <= 2^-22 for arguments in [0.5, 2], relative error <= 2^-22 elsewhere;
// ex2.approx: relative error <= 2^-22.  libdevice powf is allowed 4 ulp (<= 2^-21) from the true value.
constexpr float kLgErr = k2m22, kEx2Err = k2m22, kPowDev = k2m21;
constexpr float kSafety = 1.25f;  // applied on top of every modelled bound
constexpr float kSaneLo = 8.6736174e-19f /*2^-60*/, kSaneHi = 1.1529215e+18f /*2^60*/;

struct StepConsts {
    float om_beta1, om_beta2, correction1, correction2_sqrt;
    float p_a, p_b;   // denom = sqrt(v)*p_a + p_b  ==  (sqrt(v)/correction2_sqrt + eps)*correction1
};

__device__ __forceinline__ bool sane_pos(float x) { return x >= kSaneLo && x <= kSaneHi; }

// Relative error bound of the approximate dequantisation  ex2(fma(L[c], ik, c0)) * r  against the reference's
// fl(powf(fl(c*s), ik) * r), for any E4M3 magnitude c in [2^-9, 448], where L[c] is the table of correctly rounded
// lg2(c) (|error| <= 2^-22: |lg2 c| < 8 except the exact entries -9 and -8), lgs = lg2.approx(s) and
// c0 = fl(lgs * ik).  Absolute error of the exponent handed to ex2:
//     ik * 2^-22                      table entry
//   + ik * max(|lgs|, 1) * 2^-22      lg2.approx(s) (relative 2^-22 outside [0.5, 2], absolute 2^-22 inside)
//   + 2^-24 * (|c0| + |t|)            the two roundings, |c0| <= ik |lgs|, |t| <= ik (9 + |lgs|) =: tb
// times ln 2 as a relative error of the power; plus ik * 2^-24 for the reference's rounded product c*s, ex2.approx,
// the deviation allowed to libdevice's powf, and the rounded multiplication by r.  lgs may be off by its own error
// in this bound: 1e-3 is added.
__device__ __forceinline__ float fast_dequant_eps(float ik, float lgs, float& tb) {
    const float al = fabsf(lgs) + 1e-3f;
    tb = ik * (9.0f + al);                          // |exponent handed to ex2| <= tb
    const float e_exp = ik * kLgErr * (1.0f + fmaxf(al, 1.0f)) + k2m24 * (ik * al + tb);
    return kSafety * (kLn2 * e_exp + ik * k2m24 + kEx2Err + kPowDev + k2m23);
}

template <int N>
__device__ __forceinline__ float sel4(const float (&a)[N], int j) {
    float r = a[0];
    r = j == 1 ? a[1] : r;
    r = j == 2 ? a[2] : r;
    r = j == 3 ? a[3] : r;
    return r;
}

// exact m' (or v') of one element: the statements of fp8_adamw_expand_cuda_kernel.cu:44-55
__device__ __noinline__ float exact_moment(float x, float ik, float r, float beta, float addend, bool second) {
    float pw = powf(fabsf(x), ik);
    if (!second && signbit(x)) pw = -pw;            // sign_exp_avg * powf(|x|, 1/k)
    return __fmaf_rn(beta, pw * r, addend);
}
// exact FP8 code of one element from its exact moment (:175-187)
__device__ __noinline__ uint32_t exact_code(float val, float r, float k, float scale, bool second) {
    float pw = powf(__fdiv_rn(fabsf(val), r), k);
    if (!second && signbit(val)) pw = -pw;
    return coat_float_to_fp8<COAT_E4M3>(__fdiv_rn(pw, scale));
}

__device__ __forceinline__ uint32_t redux_max_f(float v) { return __reduce_max_sync(COAT_FULL_MASK, __float_as_uint(v)); }
__device__ __forceinline__ uint32_t redux_min_f(float v) { return __reduce_min_sync(COAT_FULL_MASK, __float_as_uint(v)); }

// ---- tiled organisation ------------------------------------------------------------------
// Work that is uniform over a group costs a full warp instruction whether 1 or 32 lanes are
// busy, so a group's set-up, its exact scalars (2 log2f, a powf, sqrts, divisions) and the exact
// recomputation of single elements must not run once per group with the other lanes idle.  A
// warp therefore takes a TILE of kTile consecutive groups and runs in phases:
//   0  one lane per group: locate the tensor, read the stored scalars, 1/k, error bounds, checks
//   1  per group, lanes over elements: load, approximate dequantise, Adam, warp reductions,
//      candidate detection, weight update and store; m' and v' go to the warp's shared tile
//   2a candidate list, one entry per lane: exact moment, shared-memory atomic max/min
//   2b one lane per (group, moment): exact group scalars, stored to global and to the tile
//   3  per group, lanes over elements: requantise and store codes; an element whose interval
//      straddles a rounding boundary is appended to a pending list that outlives the tile
//   4  whenever 32 entries are pending (and at the end): exact moment + exact code per lane,
//      patched into the code arrays bytewise
#ifdef COAT_ADAMW_PROFILE
#define PHASE_CLOCK(i) do { long long now_ = clock64(); phase_cycles[i] += now_ - phase_t; phase_t = now_; } while (0)
#else
#define PHASE_CLOCK(i) do { } while (0)
#endif
#ifndef COAT_ADAMW_TILE
#define COAT_ADAMW_TILE 6
#endif
#ifndef COAT_ADAMW_TILED_THREADS
#define COAT_ADAMW_TILED_THREADS 128
#endif
constexpr int kTile = COAT_ADAMW_TILE;
constexpr int kTiledThreads = COAT_ADAMW_TILED_THREADS;
constexpr int kTiledWarps = kTiledThreads / COAT_WARP;
constexpr int kCandPerGroup = 16;
#ifndef COAT_ADAMW_PEND_CAP
#define COAT_ADAMW_PEND_CAP 32
#endif
constexpr int kPendCap = COAT_ADAMW_PEND_CAP;
constexpr float kTiny = 7.8886091e-31f;   // 2^-100: below this the flush-to-zero MUFU forms lose accuracy

struct __align__(16) WarpTile {
    // Staging buffers, filled per tile by bulk asynchronous copies (TMA, non-multicast) that complete on
    // `mbar`: the weights, later overwritten in place by m'; the gradients, later overwritten by v';
    // the old codes of both moments (kept: the exact recomputations read them).
    float4 m1[kTile][32];        // p on arrival
    float4 v1[kTile][32];        // g on arrival
    uint32_t cw_m[kTile][32];
    uint32_t cw_v[kTile][32];
    float old_sc[kTile][8];      // s_m, 1/k_m, r_m, eps_dm * max|beta1 m~|, s_v, 1/k_v, r_v, eps_dv
    float newc[kTile][2][8];     // r', k', s', 1/r', scale_lo, scale_hi, D (first moment), in-range flag
    float delta[kTile][2];       // absolute error bound of |m'| and of v' in this group
    float c0[kTile][2];          // lg2(s) / k of the stored scale and exponent, per moment: the constant part of the dequantisation's exponent
    uint32_t stat[kTile][4];     // exact max m, min m, max v, min v (float bit patterns)
    unsigned long long ptr_p[kTile], ptr_g[kTile], ptr_m[kTile], ptr_v[kTile], ptr_bf[kTile];
    unsigned long long pair_bf[kTile];   // broadcast: bf16 destinations of a pair's first tile when it is not one run
    long long local[kTile];      // group index inside its tensor
    int ti[kTile];               // tensor index
    uint32_t flags[kTile];       // bit 0: stored scalars are in the modelled range; bit 1: full, aligned group
    uint16_t cand[kTile * kCandPerGroup];
    // pending exact recomputations (structure of arrays)
    float pe_x[kPendCap], pe_ik[kPendCap], pe_r[kPendCap], pe_g[kPendCap];
    float pe_nr[kPendCap], pe_nk[kPendCap], pe_ns[kPendCap];
    unsigned long long pe_dst[kPendCap];   // byte address of the code, bit 63 = second moment
    unsigned long long mbar;               // completion barrier of the staging copies
    uint32_t n_cand, n_pend;
};

static_assert(offsetof(WarpTile, old_sc) % 16 == 0 && offsetof(WarpTile, newc) % 16 == 0 &&
              offsetof(WarpTile, v1) % 16 == 0 && offsetof(WarpTile, cw_m) % 16 == 0 &&
              offsetof(WarpTile, cw_v) % 16 == 0 && offsetof(WarpTile, mbar) % 8 == 0 && sizeof(WarpTile) % 16 == 0,
              "vector accesses and bulk copies into the tile need 16-byte aligned members");

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(unsigned long long* bar, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
// Bounded wait: gives up after ~2^24 polls and reports it (the caller sets the error flag and leaves).
__device__ __forceinline__ bool mbar_wait(unsigned long long* bar, uint32_t parity) {
    for (int tries = 0; tries < (1 << 24); ++tries) {
        uint32_t done;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
            : "=r"(done) : "r"(smem_addr(bar)), "r"(parity) : "memory");
        if (done) return true;
    }
    return false;
}
// 1-D bulk copy global -> shared of this CTA, completion counted in bytes on the mbarrier.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, unsigned long long* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar)) : "memory");
}
// 1-D bulk copy shared -> global (this GPU's memory or a mapped peer's), tracked by the thread's bulk group.
__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
                 ::"l"(dst), "r"(smem_addr(src)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the sources of this thread's committed bulk stores have been read (the staging buffer may be rewritten)
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// this thread's committed bulk stores are complete
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ int g_adamw_device_status = 0;   // set to COAT_E_TIMEOUT if a bounded wait ran out

// lg2 of the magnitudes of four packed E4M3 codes, from a 128-entry table in shared memory (entry 0 = -inf: the
// code zero dequantises to zero; entry 127 = NaN: a NaN code surfaces as a NaN moment and sends its group to the
// exact path).  One shift, one mask and one shared load per code in place of a conversion, a multiplication and
// a lg2 on the transcendental unit.
__device__ __forceinline__ void e4m3x4_lg2(const float* lut, uint32_t w, float (&f)[4]) {
    const char* base = reinterpret_cast<const char*>(lut);
    f[0] = *reinterpret_cast<const float*>(base + ((w << 2) & 0x1fcu));
    f[1] = *reinterpret_cast<const float*>(base + ((w >> 6) & 0x1fcu));
    f[2] = *reinterpret_cast<const float*>(base + ((w >> 14) & 0x1fcu));
    f[3] = *reinterpret_cast<const float*>(base + ((w >> 22) & 0x1fcu));
}

__device__ __forceinline__ float lg2_ftz(float x) { float r; asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x)); return r; }
__device__ __forceinline__ float ex2_ftz(float x) { float r; asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x)); return r; }
__device__ __forceinline__ float rcp_ftz(float x) { float r; asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x)); return r; }
__device__ __forceinline__ float sqrt_ftz(float x) { float r; asm("sqrt.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x)); return r; }
__device__ __forceinline__ float max_nan(float a, float b) { float r; asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b)); return r; }

// Two-wide fp32 arithmetic (one instruction for two lanes of a 64-bit register pair on sm_100; each half is
// rounded to nearest like the scalar instruction, so results are bit-identical to the scalar form)
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }

template <typename scalar_t>
__device__ __noinline__ void flush_pending(WarpTile& w, int lane, const AdamwHyper& h, const StepConsts& c) {
    __syncwarp();
    const uint32_t n = w.n_pend < (uint32_t)kPendCap ? w.n_pend : (uint32_t)kPendCap;
    for (uint32_t i = lane; i < n; i += 32) {
        const unsigned long long d = w.pe_dst[i];
        const bool second = d >> 63;
        const float gj = w.pe_g[i];
        const float addend = second ? __fmul_rn(__fmul_rn(c.om_beta2, gj), gj) : __fmul_rn(c.om_beta1, gj);
        const float val = exact_moment(w.pe_x[i], w.pe_ik[i], w.pe_r[i], second ? h.beta2 : h.beta1, addend, second);
        const uint32_t code = exact_code(val, w.pe_nr[i], w.pe_nk[i], w.pe_ns[i], second);
        *reinterpret_cast<uint8_t*>(d & 0x7fffffffffffffffull) = (uint8_t)code;
    }
    __syncwarp();
    if (lane == 0) w.n_pend = 0;
    __syncwarp();
}

// Rare path of phase 3: the two ends of an element's interval round to different codes.  Queue the
// exact recomputation of those bytes (the old codes are still in place: the calling lane overwrites
// its word right after this returns).  If the list is full the element is recomputed on the spot and
// patched into the word the lane is about to store.
template <typename scalar_t>
__device__ __noinline__ void queue_exact(WarpTile& w, int slot, int lane, uint32_t dm, uint32_t dv, uint32_t& cm,
                                         uint32_t& cv, const AdamwHyper& h, const StepConsts& c,
                                         unsigned long long& n_pend_total) {
    typedef Elem4<scalar_t> E;
    uint8_t* code_m = reinterpret_cast<uint8_t*>(w.ptr_m[slot]);
    uint8_t* code_v = reinterpret_cast<uint8_t*>(w.ptr_v[slot]);
    const uint32_t old_m = w.cw_m[slot][lane], old_v = w.cw_v[slot][lane];
#pragma unroll 1
    for (int b = 0; b < 8; ++b) {
        const int j = b & 3;
        const bool second = b >> 2;
        if (!(((second ? dv : dm) >> (8 * j)) & 0xffu)) continue;
        const float* sc = w.old_sc[slot] + (second ? 4 : 0);
        const float* o = w.newc[slot][second];
        const float x = coat_e4m3_to_float((uint8_t)((second ? old_v : old_m) >> (8 * j))) * sc[0];
        const float gj = E::get(reinterpret_cast<const scalar_t*>(w.ptr_g[slot]) + lane * 4 + j);
        uint8_t* dst = (second ? code_v : code_m) + lane * 4 + j;
        const uint32_t pos = atomicAdd(&w.n_pend, 1u);
        ++n_pend_total;
        if (pos < (uint32_t)kPendCap) {
            w.pe_x[pos] = x; w.pe_ik[pos] = sc[1]; w.pe_r[pos] = sc[2]; w.pe_g[pos] = gj;
            w.pe_nr[pos] = o[0]; w.pe_nk[pos] = o[1]; w.pe_ns[pos] = o[2];
            w.pe_dst[pos] = (unsigned long long)dst | (second ? (1ull << 63) : 0ull);
        } else {
            const float addend = second ? __fmul_rn(__fmul_rn(c.om_beta2, gj), gj) : __fmul_rn(c.om_beta1, gj);
            const float val = exact_moment(x, sc[1], sc[2], second ? h.beta2 : h.beta1, addend, second);
            const uint32_t code = exact_code(val, o[0], o[1], o[2], second);
            if (second) cv = (cv & ~(0xffu << (8 * j))) | (code << (8 * j));
            else cm = (cm & ~(0xffu << (8 * j))) | (code << (8 * j));
        }
    }
}

// Shared memory, not registers, limits how many CTAs share an SM; telling the compiler so lets it use the
// registers that occupancy leaves free instead of spilling.
constexpr size_t kTiledSmem = kTiledWarps * sizeof(WarpTile);
// The broadcast variant stages the bf16 weights of two adjacent tiles (256 bytes per group) per warp behind
// everything else, and sends them to this GPU's buffer and to every peer's with bulk stores of up to both tiles.
constexpr size_t kBcastStageBytes = 2 * kTile * kGroup * sizeof(__nv_bfloat16);   // two tiles: see the tile order below
constexpr size_t kTiledSmemBcast = kTiledSmem + kTiledWarps * kBcastStageBytes;
// A table launch also keeps the tensors' group offsets in (static) shared memory: the binary search that maps a
// tile to its tensor is a chain of dependent loads, 9 deep for the 291 tensors of Llama-2-7B, and from L2 that
// chain was most of the latency of a tile's set-up.
constexpr int kPrefixCap = 512;
constexpr int tiled_ctas_per_sm(bool bcast) {
    return (int)((227 * 1024) / ((bcast ? kTiledSmemBcast : kTiledSmem) + 1024 + kPrefixCap * sizeof(int) + 128 * sizeof(float)));
}
static_assert(kTiledSmem % 16 == 0 && kBcastStageBytes % 16 == 0, "bulk copies need 16-byte aligned staging");

template <typename scalar_t, bool MULTI, bool BCAST>
__global__ void __launch_bounds__(kTiledThreads, tiled_ctas_per_sm(BCAST))
fp8_adamw_expand_tiled_kernel(TensorDesc single, const TensorDesc* __restrict__ table,
                              const int64_t* __restrict__ group_prefix, int n_tensors, int64_t total_groups,
                              AdamwHyper h, unsigned long long* dbg) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    WarpTile& w = reinterpret_cast<WarpTile*>(smem_raw)[warp];
    uint2* bf_stage = reinterpret_cast<uint2*>(smem_raw + kTiledSmem + warp * kBcastStageBytes);   // BCAST only
    typedef Elem4<scalar_t> E;

    StepConsts c;
    c.om_beta1 = 1 - h.beta1;
    c.om_beta2 = 1 - h.beta2;
    c.correction1 = 1.0f - powf(h.beta1, h.step);
    c.correction2_sqrt = sqrtf(1.0f - powf(h.beta2, h.step));
    c.p_a = c.correction1 / c.correction2_sqrt;
    c.p_b = h.eps * c.correction1;
    const float kInf = __int_as_float(0x7f800000);

    const int64_t n_tiles = (total_groups + kTile - 1) / kTile;
    const int64_t warps_total = (int64_t)gridDim.x * kTiledWarps;
    unsigned long long n_fast = 0, n_exact = 0, n_cand_total = 0, n_pend_total = 0;
    __shared__ int s_prefix[MULTI ? kPrefixCap : 1];
    const bool prefix_cached = MULTI && n_tensors <= kPrefixCap && total_groups < (1ll << 31);
    if (prefix_cached)
        for (int i = threadIdx.x; i < n_tensors; i += kTiledThreads) s_prefix[i] = (int)group_prefix[i];
    // lg2 of every E4M3 magnitude, correctly rounded (through double): see e4m3x4_lg2
    __shared__ float s_lg2[128];
    for (int i = threadIdx.x; i < 128; i += kTiledThreads)
        s_lg2[i] = i == 127 ? __int_as_float(0x7fffffff)
                            : (i == 0 ? -kInf : (float)log2((double)coat_e4m3_to_float((uint8_t)i)));
    __syncthreads();
    if (lane == 0) {
        w.n_pend = 0;
        w.n_cand = 0;
        mbar_init(&w.mbar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    uint32_t mbar_parity = 0;
#ifdef COAT_ADAMW_PROFILE
    long long phase_cycles[6] = {0, 0, 0, 0, 0, 0};
    long long phase_t = clock64();
#endif

    // Tile order.  Plain: warp w of the grid takes tiles w, w + W, w + 2W, ...  Broadcast: it takes PAIRS of adjacent
    // tiles (2w, 2w+1), (2(w+W), 2(w+W)+1), ... so that the bf16 weights of a pair are one contiguous run of up to
    // 3 KB, which leaves as ONE bulk store per destination once the second tile is staged.
    const int64_t first_unit = (int64_t)blockIdx.x * kTiledWarps + warp;
    uint32_t pair_staged = 0;          // broadcast: slots of the pair's first tile that wait in bf_stage
    unsigned long long pair_ptr = 0;   // broadcast: destination of the first tile's run (0: not one contiguous run)
    int pair_slots = 0;
    int ti_cursor = 0;                 // table launches: the tensor this lane's previous group lay in
    for (int64_t it = 0;; ++it) {
        const int half = BCAST ? (int)(it & 1) : 0;
        const int64_t tile = BCAST ? 2 * (first_unit + (it >> 1) * warps_total) + half : first_unit + it * warps_total;
        if (tile >= n_tiles) break;
        const bool pair_open = BCAST && half == 0 && tile + 1 < n_tiles;   // a second tile follows: hold the stores back
        const int64_t g0 = tile * kTile;
        const int n_slots = (int)((total_groups - g0) < kTile ? (total_groups - g0) : kTile);

        // ================= phase 0: one lane per group =================
        // 0a: where the group lives
        if (lane < n_slots) {
            const int64_t gi = g0 + lane;
            int ti = 0;
            int64_t group = gi;
            if (MULTI) {
                // a lane's groups only move forward from tile to tile: start at the tensor of its previous group, and
                // search (binary, above it) only when the group has left that tensor
                int lo = ti_cursor, hi = n_tensors - 1;
                if (prefix_cached) {
                    if (lo < hi && (int64_t)s_prefix[lo + 1] <= gi) {
                        ++lo;
                        while (lo < hi) {
                            const int mid = (lo + hi + 1) >> 1;
                            if ((int64_t)s_prefix[mid] <= gi) lo = mid; else hi = mid - 1;
                        }
                    }
                    group = gi - s_prefix[lo];
                } else {
                    if (lo < hi && group_prefix[lo + 1] <= gi) {
                        ++lo;
                        while (lo < hi) {
                            const int mid = (lo + hi + 1) >> 1;
                            if (group_prefix[mid] <= gi) lo = mid; else hi = mid - 1;
                        }
                    }
                    group = gi - group_prefix[lo];
                }
                ti = lo;
                ti_cursor = lo;
            }
            const TensorDesc& t = MULTI ? table[ti] : single;
            const int64_t e0 = group * kGroup;
            w.ptr_p[lane] = (unsigned long long)(reinterpret_cast<scalar_t*>(t.p) + e0);
            w.ptr_g[lane] = (unsigned long long)(reinterpret_cast<const scalar_t*>(t.g) + e0);
            w.ptr_m[lane] = (unsigned long long)(t.m + e0);
            w.ptr_v[lane] = (unsigned long long)(t.v + e0);
            w.ptr_bf[lane] = t.bf16_out ? (unsigned long long)(reinterpret_cast<__nv_bfloat16*>(t.bf16_out) + e0) : 0ull;
            w.local[lane] = group;
            w.ti[lane] = ti;
            w.flags[lane] = (desc_vec_ok(t, E::kVecAlign) && (t.numel - e0 >= kGroup)) ? 2u : 0u;
            w.stat[lane][0] = 0u; w.stat[lane][1] = 0x7f800000u; w.stat[lane][2] = 0u; w.stat[lane][3] = 0x7f800000u;
        }
        if (lane == 0) w.n_cand = 0;
        fence_proxy_async();   // this lane's generic accesses to the staging buffers precede the next bulk write
        __syncwarp();
        // stage the tile's inputs: one bulk copy per array when the tile is one contiguous, aligned run
        const bool all_mem_ok = __ballot_sync(COAT_FULL_MASK, lane < n_slots && !(w.flags[lane] & 2u)) == 0u;
        const bool bulk = all_mem_ok && w.ti[0] == w.ti[n_slots - 1];
        if (bulk) {
            if (lane == 0) {
                const uint32_t n = (uint32_t)n_slots;
                mbar_expect_tx(&w.mbar, n * (2u * kGroup * (uint32_t)sizeof(scalar_t) + 2u * kGroup));
                bulk_g2s(&w.m1[0][0], reinterpret_cast<const void*>(w.ptr_p[0]), n * kGroup * (uint32_t)sizeof(scalar_t), &w.mbar);
                bulk_g2s(&w.v1[0][0], reinterpret_cast<const void*>(w.ptr_g[0]), n * kGroup * (uint32_t)sizeof(scalar_t), &w.mbar);
                bulk_g2s(&w.cw_m[0][0], reinterpret_cast<const void*>(w.ptr_m[0]), n * kGroup, &w.mbar);
                bulk_g2s(&w.cw_v[0][0], reinterpret_cast<const void*>(w.ptr_v[0]), n * kGroup, &w.mbar);
            }
        } else {
            for (int sl = 0; sl < n_slots; ++sl) {
                if (!(w.flags[sl] & 2u)) continue;
                w.m1[sl][lane] = reinterpret_cast<const float4*>(w.ptr_p[sl])[lane];
                w.v1[sl][lane] = reinterpret_cast<const float4*>(w.ptr_g[sl])[lane];
                w.cw_m[sl][lane] = reinterpret_cast<const uint32_t*>(w.ptr_m[sl])[lane];
                w.cw_v[sl][lane] = reinterpret_cast<const uint32_t*>(w.ptr_v[sl])[lane];
            }
        }
        // 0b: the stored scalars of each group, 1/k, error bounds, range checks (overlaps the copies); one lane per
        //     (group, moment), so that the two moments' chains of a group run side by side
        {
            const int slot = lane >> 1;
            const bool second = lane & 1;
            int ok = 1;
            if (slot < n_slots) {
                const TensorDesc& t = MULTI ? table[w.ti[slot]] : single;
                const int64_t group = w.local[slot];
                // the three loads leave before the first of them is used (each is a round trip to memory)
                const float s = (second ? t.s_v : t.s_m)[group];
                const float k = (second ? t.k_v : t.k_m)[group];
                const float r = (second ? t.r_v : t.r_m)[group];
                const float ik = __fdiv_rn(1.0f, k);
                float tb;
                const float lgs = fast_lg2(s);
                const float eps_d = fast_dequant_eps(ik, lgs, tb);
                const float c0 = __fmul_rn(lgs, ik);
                w.c0[slot][second] = c0;
                ok = sane_pos(s) && sane_pos(r) && ik >= 0.015625f && ik <= 64.0f && tb <= 60.0f;
                float* sc = w.old_sc[slot] + (second ? 4 : 0);
                // first moment: largest |beta1 * m~| any code of the group can dequantise to (the code 448; the
                // dequantisation is monotone in the code's magnitude, 2^-20 covers the approximation's own wobble), times
                // the relative bound: the absolute error the first moment inherits from the dequantisation
                const float mam = fabsf(h.beta1) * (ex2_ftz(__fmaf_rn(8.8073549f /* lg2 448 */, ik, c0)) * r) *
                                  (1.0f + 9.5367432e-07f);
                sc[0] = s; sc[1] = ik; sc[2] = r; sc[3] = second ? eps_d : eps_d * mam;
            }
            // (every lane takes part in the shuffle: it must not sit behind a short-circuiting `&&`)
            const int other = __shfl_xor_sync(COAT_FULL_MASK, ok, 1);
            if (slot < n_slots && !second && ok && other) w.flags[slot] |= 1u;
        }
        __syncwarp();
        if (bulk) {
            if (!mbar_wait(&w.mbar, mbar_parity)) {   // bounded; never expected
                g_adamw_device_status = COAT_E_TIMEOUT;
                if constexpr (BCAST) bulk_wait_all();
                return;
            }
            mbar_parity ^= 1u;
        }
        PHASE_CLOCK(0);

        // ================= phase 1: lanes over the elements of one group =================
        uint32_t live = 0;   // slots that stay on the fast path (warp-uniform)
        uint32_t staged = 0;   // BCAST: slots whose bf16 weights wait in bf_stage (warp-uniform)
        uint2* const stage = bf_stage + half * (kTile * 32);
        if constexpr (BCAST) {
            if (half == 0) bulk_wait_read();   // the previous pair's bulk stores have read bf_stage (no-op for other lanes)
            __syncwarp();
        }
#pragma unroll 1
        for (int slot = 0; slot < n_slots; ++slot) {
            bool ok = (w.flags[slot] & 3u) == 3u;
            if (ok) {
                scalar_t* pp = reinterpret_cast<scalar_t*>(w.ptr_p[slot]) + lane * 4;
                const float4 p4 = w.m1[slot][lane], g4 = w.v1[slot][lane];
                float p[4] = {p4.x, p4.y, p4.z, p4.w};
                const float g[4] = {g4.x, g4.y, g4.z, g4.w};
                const uint32_t mw = w.cw_m[slot][lane], vw = w.cw_v[slot][lane];
                float xm[4], xv[4], m1[4], v1[4];
                const float4 sa = reinterpret_cast<const float4*>(w.old_sc[slot])[0];   // s_m, 1/k_m, r_m, eps_dm * max|beta1 m~|
                const float4 sb = reinterpret_cast<const float4*>(w.old_sc[slot])[1];   // s_v, 1/k_v, r_v, eps_dv
                e4m3x4_lg2(s_lg2, mw, xm);
                e4m3x4_lg2(s_lg2, vw, xv);
                const float c0_m = w.c0[slot][0], c0_v = w.c0[slot][1];
                // a negative second-moment code sends the group to the exact path (via the NaN that max_nan carries
                // into the group maximum); a NaN code arrives as a NaN moment through the table
                float mx_a = (vw & 0x80808080u) ? __int_as_float(0x7fffffff) : 0.f;
                float mn_a = kInf, mx_v = 0.f, mn_v = kInf;
#pragma unroll
                for (int jj = 0; jj < 4; jj += 2) {
                    // |m| = (c s)^(1/k) r = ex2(lg2(c) / k + lg2(s) / k) r; the sign of the code is put back on
                    const float2 tm = __ffma2_rn(f2(xm[jj], xm[jj + 1]), f2(sa.y), f2(c0_m));
                    const float2 tv = __ffma2_rn(f2(xv[jj], xv[jj + 1]), f2(sb.y), f2(c0_v));
                    float2 mt = __fmul2_rn(f2(ex2_ftz(tm.x), ex2_ftz(tm.y)), f2(sa.z));
                    const float2 vt = __fmul2_rn(f2(ex2_ftz(tv.x), ex2_ftz(tv.y)), f2(sb.z));
                    mt.x = __uint_as_float(__float_as_uint(mt.x) | ((mw << (24 - 8 * jj)) & 0x80000000u));
                    mt.y = __uint_as_float(__float_as_uint(mt.y) | ((mw << (16 - 8 * jj)) & 0x80000000u));
                    const float2 gg = f2(g[jj], g[jj + 1]);
                    // beta1 m + (1-beta1) g  and  beta2 v + ((1-beta2) g) g, as adam_first / adam_second round them
                    const float2 m2 = __ffma2_rn(f2(h.beta1), mt, __fmul2_rn(f2(c.om_beta1), gg));
                    const float2 v2 = __ffma2_rn(f2(h.beta2), vt, __fmul2_rn(__fmul2_rn(f2(c.om_beta2), gg), gg));
                    m1[jj] = m2.x; m1[jj + 1] = m2.y; v1[jj] = v2.x; v1[jj + 1] = v2.y;
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float a1 = fabsf(m1[j]);
                    mx_a = max_nan(mx_a, a1);   // a NaN anywhere must surface in the maxima
                    mn_a = fminf(mn_a, a1);
                    mx_v = max_nan(mx_v, v1[j]);
                    mn_v = fminf(mn_v, v1[j]);
                }
                // all four are non-negative (or NaN, which orders above everything): unsigned order == float order
                const float MA = __uint_as_float(redux_max_f(mx_a)), mA = __uint_as_float(redux_min_f(mn_a));
                const float MV = __uint_as_float(redux_max_f(mx_v)), mV = __uint_as_float(redux_min_f(mn_v));
                // error bounds of the approximate moments.  First moment (the two terms may cancel), absolute
                // and uniform over the group: |m~' - m'| <= eps_dm*max|beta1*m~| + 2^-22*max|m'| = d_m (the first product comes
                // ready-made from the set-up: sa.w).
                // Second moment (both terms >= 0), relative per element: |v~' - v'| <= (eps_dv + 2^-22) * v'.
                const float d_m = __fmaf_rn(k2m22, MA, sa.w);
                const float e_v = sb.w + k2m22;
                // no possible exact zero / sign change / NaN / denormal, and nothing overflowed
                ok = (mA - d_m > kTiny) && (mV > kTiny) && (MA <= kSaneHi) && (MV <= kSaneHi);
                uint32_t cand = 0;
                if (ok) {
                    const float hi_m = MA - 2.0f * d_m, lo_m = mA + 2.0f * d_m;
                    const float hi_v = MV * (1.0f - 2.5f * e_v), lo_v = mV * (1.0f + 2.5f * e_v);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float a1 = fabsf(m1[j]);
                        if (a1 >= hi_m || a1 <= lo_m) cand |= 1u << j;
                        if (v1[j] >= hi_v || v1[j] <= lo_v) cand |= 16u << j;
                    }
                    ok = __reduce_add_sync(COAT_FULL_MASK, __popc(cand)) <= kCandPerGroup;
                }
                if (ok) {
                    // weights from the approximate moments (they are not quantised)
#pragma unroll
                    for (int jj = 0; jj < 4; jj += 2) {
                        const float2 denom = __ffma2_rn(f2(sqrt_ftz(v1[jj]), sqrt_ftz(v1[jj + 1])), f2(c.p_a), f2(c.p_b));
                        const float2 pj = f2(p[jj], p[jj + 1]);
                        const float2 update = __ffma2_rn(f2(h.wd), pj, __fmul2_rn(f2(m1[jj], m1[jj + 1]),
                                                                                  f2(rcp_ftz(denom.x), rcp_ftz(denom.y))));
                        const float2 pn = __ffma2_rn(f2(-h.lr), update, pj);
                        p[jj] = pn.x; p[jj + 1] = pn.y;
                    }
                    E::store(pp, p);
                    if (w.ptr_bf[slot]) {
                        float q[4];
#pragma unroll
                        for (int j = 0; j < 4; ++j) q[j] = E::round(p[j]);
                        if (BCAST && (w.ptr_bf[slot] & 15ull) == 0) {   // staged; sent after the loop
                            uint2 t2;
                            const __nv_bfloat162 lo = __floats2bfloat162_rn(q[0], q[1]), hi = __floats2bfloat162_rn(q[2], q[3]);
                            t2.x = *reinterpret_cast<const uint32_t*>(&lo);
                            t2.y = *reinterpret_cast<const uint32_t*>(&hi);
                            stage[slot * 32 + lane] = t2;
                            staged |= 1u << slot;
                        } else {
                            store_bf16x4_bcast<BCAST>(reinterpret_cast<__nv_bfloat16*>(w.ptr_bf[slot]) + lane * 4, q, h);
                        }
                    }
                    w.m1[slot][lane] = make_float4(m1[0], m1[1], m1[2], m1[3]);
                    w.v1[slot][lane] = make_float4(v1[0], v1[1], v1[2], v1[3]);
                    if (lane == 0) w.delta[slot][0] = d_m;
                    if (cand) {
                        uint32_t pos = atomicAdd(&w.n_cand, (uint32_t)__popc(cand));
                        while (cand) {
                            const int b = __ffs(cand) - 1;
                            cand &= cand - 1;
                            w.cand[pos++] = (uint16_t)((slot << 8) | ((lane * 4 + (b & 3)) << 1) | (b >> 2));
                        }
                    }
                    live |= 1u << slot;
                }
            }
            if (!ok) {
                const TensorDesc& t = MULTI ? table[w.ti[slot]] : single;
                // scratch of the exact minimum tree (128 floats): this slot's gradient staging, which a group that
                // leaves the fast path no longer needs (the exact routine reads its inputs from global memory)
                process_group_exact<scalar_t, true, BCAST>(t, w.local[slot], lane, h, c.om_beta1, c.om_beta2, c.correction1,
                                                    c.correction2_sqrt, desc_vec_ok(t, E::kVecAlign),
                                                    reinterpret_cast<float*>(&w.v1[slot][0]));
                ++n_exact;
            }
        }
        __syncwarp();
        if constexpr (BCAST) {
            const uint32_t group_bytes = kGroup * (uint32_t)sizeof(__nv_bfloat16);
            const bool run = bulk && staged == (1u << n_slots) - 1u;   // this tile's weights are one contiguous staged run
            if (pair_open) {   // first tile of a pair: remember it, send together with the second
                pair_staged = staged;
                pair_ptr = run ? w.ptr_bf[0] : 0ull;
                pair_slots = n_slots;
            } else if (staged | pair_staged) {
                fence_proxy_async();   // the staged words (generic stores) become visible to the bulk copies
                __syncwarp();
                if (lane <= h.n_peers) {   // lane 0: this GPU's buffer; lane i: a peer, the order rotated by warp
                    long long delta = 0ll;
                    if (lane > 0) {
                        int peer = lane - 1 + (int)(first_unit % h.n_peers);
                        if (peer >= h.n_peers) peer -= h.n_peers;
                        delta = h.peer_delta[peer];
                    }
                    const bool joined = half == 1 && pair_ptr != 0ull && run &&
                                        w.ptr_bf[0] == pair_ptr + (unsigned long long)pair_slots * group_bytes;
                    if (joined) {   // both tiles: one store per destination
                        bulk_s2g(reinterpret_cast<char*>(pair_ptr) + delta, bf_stage, (uint32_t)(pair_slots + n_slots) * group_bytes);
                    } else {
                        if (half == 1 && pair_staged) {   // the held-back first tile on its own
                            if (pair_ptr != 0ull) {
                                bulk_s2g(reinterpret_cast<char*>(pair_ptr) + delta, bf_stage, (uint32_t)pair_slots * group_bytes);
                            } else {
                                for (int slot = 0; slot < pair_slots; ++slot)
                                    if (pair_staged & (1u << slot))
                                        bulk_s2g(reinterpret_cast<char*>(w.pair_bf[slot]) + delta, bf_stage + slot * 32, group_bytes);
                            }
                        }
                        if (run) {
                            bulk_s2g(reinterpret_cast<char*>(w.ptr_bf[0]) + delta, stage, (uint32_t)n_slots * group_bytes);
                        } else {
                            for (int slot = 0; slot < n_slots; ++slot)
                                if (staged & (1u << slot))
                                    bulk_s2g(reinterpret_cast<char*>(w.ptr_bf[slot]) + delta, stage + slot * 32, group_bytes);
                        }
                    }
                    bulk_commit();
                }
                pair_staged = 0;
                pair_ptr = 0ull;
            }
            if (pair_open && !run && staged) {   // scattered first tile: its destinations are needed after ptr_bf is rewritten
                if (lane < n_slots) w.pair_bf[lane] = w.ptr_bf[lane];
            }
        }
        PHASE_CLOCK(1);
        if (live == 0) continue;
        n_fast += __popc(live);

        // ================= phase 2a: exact moments of the max/min candidates =================
        {
            const uint32_t n = w.n_cand;
            n_cand_total += n;
            for (uint32_t i = lane; i < n; i += 32) {
                const uint32_t e = w.cand[i];
                const int slot = e >> 8, elem = (e >> 1) & 127;
                const bool second = e & 1;
                const float* sc = w.old_sc[slot] + (second ? 4 : 0);
                const uint8_t code = reinterpret_cast<const uint8_t*>(second ? w.cw_v[slot] : w.cw_m[slot])[elem];
                const float gj = E::get(reinterpret_cast<const scalar_t*>(w.ptr_g[slot]) + elem);
                const float addend = second ? __fmul_rn(__fmul_rn(c.om_beta2, gj), gj) : __fmul_rn(c.om_beta1, gj);
                const float val = fabsf(exact_moment(coat_e4m3_to_float(code) * sc[0], sc[1], sc[2],
                                                     second ? h.beta2 : h.beta1, addend, second));
                if (dbg) {   // how much of the modelled error bound the approximation actually used
                    const float approx = fabsf(reinterpret_cast<const float*>(second ? w.v1[slot] : w.m1[slot])[elem]);
                    const float bound = second ? (sc[3] + k2m22) * val : w.delta[slot][0];
                    atomicMax(reinterpret_cast<unsigned int*>(dbg + (second ? 7 : 6)),
                              __float_as_uint(fabsf(approx - val) / bound));
                }
                atomicMax(&w.stat[slot][second ? 2 : 0], __float_as_uint(val));
                atomicMin(&w.stat[slot][second ? 3 : 1], __float_as_uint(val));
            }
        }
        __syncwarp();
        PHASE_CLOCK(2);

        // ================= phase 2b: exact group scalars, one lane per (group, moment) =================
        if (lane < 2 * kTile && ((live >> (lane >> 1)) & 1)) {
            const int slot = lane >> 1;
            const bool second = lane & 1;
            const float amax = __uint_as_float(w.stat[slot][second ? 2 : 0]);
            const float amin = fminf(__uint_as_float(w.stat[slot][second ? 3 : 1]), 1e9f);
            float maxv, sq, ex, ns;
            expand_group_scalars(amax, amin, h.expand_min, maxv, sq, ex, ns);
            const TensorDesc& t = MULTI ? table[w.ti[slot]] : single;
            const int64_t group = w.local[slot];
            if (second) { t.s_v[group] = ns; t.k_v[group] = ex; t.r_v[group] = sq; }
            else { t.s_m[group] = ns; t.k_m[group] = ex; t.r_m[group] = sq; }
            // |lg2(m'/r')| <= lg2(max/min)/2 (+ slack); the exponent handed to ex2 is k' times that
            const float lw = fmaxf(1.0f, fabsf(fast_lg2(__fdiv_rn(maxv, sq))) + 1e-2f);
            const float e_q = kSafety * (ex * k2m23 + kLn2 * ex * lw * (kLgErr + k2m24) + kEx2Err + kPowDev + k2m22) +
                              ex * k2m22;
            const float inv_s = __fdiv_rn(1.0f, ns);
            // relative error of the input: first moment delta/|m'| per element (D * 1/|m'| below);
            // second moment at most eps_dv + 2^-22 for every element
            const float rel_v = second ? 1.02f * ex * (w.old_sc[slot][7] + k2m22) : 0.f;
            const bool in_range = sane_pos(sq) && ex >= 0.015625f && ex <= 32.0f && ns >= 9.5367432e-07f &&
                                  ns <= 1048576.0f;
            float* o = w.newc[slot][second];
            o[0] = sq; o[1] = ex; o[2] = ns; o[3] = __fdiv_rn(1.0f, sq);
            o[4] = inv_s * (1.0f - e_q - rel_v); o[5] = inv_s * (1.0f + e_q + rel_v);
            o[6] = 1.02f * ex * inv_s * w.delta[slot][0];
            o[7] = in_range ? 1.0f : 0.0f;
        }
        __syncwarp();
        PHASE_CLOCK(3);

        // ================= phase 3: requantise; both ends of each interval must agree =================
#pragma unroll 1
        for (int slot = 0; slot < n_slots; ++slot) {
            if (!((live >> slot) & 1)) continue;
            const float4 qa_m = reinterpret_cast<const float4*>(w.newc[slot][0])[0];
            const float4 qb_m = reinterpret_cast<const float4*>(w.newc[slot][0])[1];
            const float4 qa_v = reinterpret_cast<const float4*>(w.newc[slot][1])[0];
            const float4 qb_v = reinterpret_cast<const float4*>(w.newc[slot][1])[1];
            const float4 m4 = w.m1[slot][lane], v4 = w.v1[slot][lane];
            const float m1[4] = {m4.x, m4.y, m4.z, m4.w}, v1[4] = {v4.x, v4.y, v4.z, v4.w};
            float ql[4], qh[4];
#pragma unroll
            for (int jj = 0; jj < 4; jj += 2) {
                const float2 a1 = f2(fabsf(m1[jj]), fabsf(m1[jj + 1]));
                const float2 arg = __fmul2_rn(a1, f2(qa_m.w));
                const float2 t = __fmul2_rn(f2(qa_m.y), f2(lg2_ftz(arg.x), lg2_ftz(arg.y)));
                const float2 e = f2(ex2_ftz(t.x), ex2_ftz(t.y));
                // 2^-floor(log2 a1) >= 1/a1, from the exponent field alone (a1 is a normal number here)
                const float2 ia = f2(__uint_as_float(0x7f000000u - (__float_as_uint(a1.x) & 0x7f800000u)),
                                     __uint_as_float(0x7f000000u - (__float_as_uint(a1.y) & 0x7f800000u)));
                const float2 lo = __fmul2_rn(e, __ffma2_rn(f2(-qb_m.z), ia, f2(qb_m.x)));
                const float2 hi = __fmul2_rn(e, __ffma2_rn(f2(qb_m.z), ia, f2(qb_m.y)));
                ql[jj] = lo.x; ql[jj + 1] = lo.y; qh[jj] = hi.x; qh[jj + 1] = hi.y;
            }
            uint32_t cm = coat_float4_to_fp8x4<COAT_E4M3>(ql[0], ql[1], ql[2], ql[3]);
            uint32_t dm = cm ^ coat_float4_to_fp8x4<COAT_E4M3>(qh[0], qh[1], qh[2], qh[3]);
#pragma unroll
            for (int jj = 0; jj < 4; jj += 2) {
                const float2 arg = __fmul2_rn(f2(v1[jj], v1[jj + 1]), f2(qa_v.w));
                const float2 t = __fmul2_rn(f2(qa_v.y), f2(lg2_ftz(arg.x), lg2_ftz(arg.y)));
                const float2 e = f2(ex2_ftz(t.x), ex2_ftz(t.y));
                const float2 lo = __fmul2_rn(e, f2(qb_v.x)), hi = __fmul2_rn(e, f2(qb_v.y));
                ql[jj] = lo.x; ql[jj + 1] = lo.y; qh[jj] = hi.x; qh[jj + 1] = hi.y;
            }
            uint32_t cv = coat_float4_to_fp8x4<COAT_E4M3>(ql[0], ql[1], ql[2], ql[3]);
            uint32_t dv = cv ^ coat_float4_to_fp8x4<COAT_E4M3>(qh[0], qh[1], qh[2], qh[3]);
            // sign of the first moment (certain: every interval excludes zero)
            cm |= ((__float_as_uint(m1[0]) >> 31) << 7) | ((__float_as_uint(m1[1]) >> 31) << 15) |
                  ((__float_as_uint(m1[2]) >> 31) << 23) | ((__float_as_uint(m1[3]) >> 31) << 31);
            if (qb_m.w == 0.0f) dm = 0xffffffffu;   // new scalars outside the modelled range: recompute all
            if (qb_v.w == 0.0f) dv = 0xffffffffu;
            uint8_t* code_m = reinterpret_cast<uint8_t*>(w.ptr_m[slot]);
            uint8_t* code_v = reinterpret_cast<uint8_t*>(w.ptr_v[slot]);
            if (dm | dv) queue_exact<scalar_t>(w, slot, lane, dm, dv, cm, cv, h, c, n_pend_total);
            reinterpret_cast<uint32_t*>(code_m)[lane] = cm;
            reinterpret_cast<uint32_t*>(code_v)[lane] = cv;
            __syncwarp();
            if (w.n_pend >= (uint32_t)(kPendCap < 32 ? kPendCap : 32)) { PHASE_CLOCK(4); flush_pending<scalar_t>(w, lane, h, c); PHASE_CLOCK(5); }
        }
        PHASE_CLOCK(4);
    }
    flush_pending<scalar_t>(w, lane, h, c);
#ifdef COAT_ADAMW_PROFILE
    if (dbg && lane == 0)
        for (int i = 0; i < 6; ++i) atomicAdd(dbg + 8 + i, (unsigned long long)phase_cycles[i]);
#endif
    if constexpr (BCAST) bulk_wait_all();   // this thread's bulk stores are complete before the CTA retires
    if (dbg) {
        n_pend_total = __reduce_add_sync(COAT_FULL_MASK, (unsigned)n_pend_total);
        if (lane == 0) {
            atomicAdd(dbg + 0, n_fast);
            atomicAdd(dbg + 1, n_exact);
            atomicAdd(dbg + 2, n_cand_total);
            atomicAdd(dbg + 3, n_pend_total);
        }
    }
}

template <typename scalar_t, bool EXPAND, bool MULTI, bool BCAST>
__global__ void __launch_bounds__(kThreads)
fp8_adamw_kernel(TensorDesc single, const TensorDesc* __restrict__ table,
                 const int64_t* __restrict__ group_prefix, int n_tensors, int64_t total_groups,
                 AdamwHyper h, unsigned long long* dbg) {
    __shared__ float smem_min[kWarpsPerCta][kGroup];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    // hoisted per-launch scalars, evaluated on the device with the same routines as
    // the reference (fp8_adamw_expand_cuda_kernel.cu:52-58)
    StepConsts c;
    c.om_beta1 = 1 - h.beta1;
    c.om_beta2 = 1 - h.beta2;
    c.correction1 = 1.0f - powf(h.beta1, h.step);
    c.correction2_sqrt = sqrtf(1.0f - powf(h.beta2, h.step));
    c.p_a = c.correction1 / c.correction2_sqrt;
    c.p_b = h.eps * c.correction1;

    const int64_t warps_total = (int64_t)gridDim.x * kWarpsPerCta;
    int64_t gi = (int64_t)blockIdx.x * kWarpsPerCta + warp;
    if (!MULTI) {
        const bool vec_ok = desc_vec_ok(single, Elem4<scalar_t>::kVecAlign);
        for (; gi < total_groups; gi += warps_total) {
            process_group_exact<scalar_t, EXPAND, BCAST>(single, gi, lane, h, c.om_beta1, c.om_beta2, c.correction1,
                                                  c.correction2_sqrt, vec_ok, smem_min[warp]);
            if (dbg && lane == 0) atomicAdd(dbg + 1, 1ull);
        }
    } else {
        int ti = 0;
        for (; gi < total_groups; gi += warps_total) {
            // group_prefix is sorted; successive gi only move forward
            if (gi >= group_prefix[ti + 1]) {
                int lo = ti + 1, hi = n_tensors - 1;
                while (lo < hi) {
                    int mid = (lo + hi + 1) >> 1;
                    if (group_prefix[mid] <= gi) lo = mid; else hi = mid - 1;
                }
                ti = lo;
            }
            TensorDesc t = table[ti];
            const bool vec_ok = desc_vec_ok(t, Elem4<scalar_t>::kVecAlign);
            const int64_t local = gi - group_prefix[ti];
            process_group_exact<scalar_t, EXPAND, BCAST>(t, local, lane, h, c.om_beta1, c.om_beta2, c.correction1,
                                                  c.correction2_sqrt, vec_ok, smem_min[warp]);
            if (dbg && lane == 0) atomicAdd(dbg + 1, 1ull);
        }
    }
}

// =====================================================================================
// Guarded fast path of the step WITHOUT expansion (fp8_adamw_cuda_kernel.cu:38-124)
// =====================================================================================
// Without the powers the moments cost a handful of exact fp32 operations, so m', v', the group maxima and the new
// scales are computed exactly as the reference does (same operations, same contractions).  What made the exact
// kernel instruction bound are its IEEE divisions and square root: four divisions and a square root per element,
// ~50 instructions.  Here
//   * a code is taken from m' * rcp(s') evaluated at both ends of an interval (relative half-width 2^-21) that
//     contains the reference's correctly rounded m' / s'; only if the two ends round to different codes is that
//     element divided exactly (about one element in 1e5);
//   * the weights use sqrt.approx / rcp.approx and differ from the reference's by a few 1e-7 of one update (the
//     tolerance stated for the expansion kernel's default mode); COAT_ADAMW_EXACT_POW selects the exact kernel.
// A group that is partial, unaligned, or whose maximum is not a finite number in the modelled range goes to the
// exact routine.
constexpr int kPlainThreads = 256;

template <bool MULTI>
__global__ void __launch_bounds__(kPlainThreads)
fp8_adamw_plain_fast_kernel(TensorDesc single, const TensorDesc* __restrict__ table,
                            const int64_t* __restrict__ group_prefix, int n_tensors, int64_t total_groups,
                            AdamwHyper h, unsigned long long* dbg) {
    __shared__ float smem_min[kPlainThreads / COAT_WARP][kGroup];   // scratch the exact routine's signature asks for
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    StepConsts c;
    c.om_beta1 = 1 - h.beta1;
    c.om_beta2 = 1 - h.beta2;
    c.correction1 = 1.0f - powf(h.beta1, h.step);
    c.correction2_sqrt = sqrtf(1.0f - powf(h.beta2, h.step));
    c.p_a = c.correction1 / c.correction2_sqrt;
    c.p_b = h.eps * c.correction1;
    const float kRelHalfWidth = 4.7683716e-07f;   // 2^-21: rcp.approx (2^-23) + two roundings, doubled
    const int64_t warps_total = (int64_t)gridDim.x * (kPlainThreads / COAT_WARP);
    // One group's inputs, loaded a trip ahead of their use so that a warp always has a group's worth of loads in
    // flight while it computes on the previous one.
    struct Inputs {
        float4 p4, g4;
        uint32_t mw, vw;
        float s_m, s_v;
        int64_t group;
        int ti;
        bool ok;
    };
    int ti_cursor = 0;
    auto fetch = [&](int64_t gi, Inputs& in) {
        in.group = gi;
        in.ti = 0;
        if (MULTI) {
            if (gi >= group_prefix[ti_cursor + 1]) {   // group_prefix is sorted; successive gi only move forward
                int lo = ti_cursor + 1, hi = n_tensors - 1;
                while (lo < hi) {
                    const int mid = (lo + hi + 1) >> 1;
                    if (group_prefix[mid] <= gi) lo = mid; else hi = mid - 1;
                }
                ti_cursor = lo;
            }
            in.ti = ti_cursor;
            in.group = gi - group_prefix[ti_cursor];
        }
        const TensorDesc& t = MULTI ? table[in.ti] : single;
        const int64_t base = in.group * kGroup + lane * 4;
        in.ok = desc_vec_ok(t, 16) && (t.numel - in.group * kGroup >= kGroup);
        if (in.ok) {
            in.p4 = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(t.p) + base);
            in.g4 = __ldcs(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(t.g) + base));
            in.mw = *reinterpret_cast<const uint32_t*>(t.m + base);
            in.vw = *reinterpret_cast<const uint32_t*>(t.v + base);
            in.s_m = t.s_m[in.group];
            in.s_v = t.s_v[in.group];
        }
    };
    Inputs cur, nxt;
    int64_t gi = (int64_t)blockIdx.x * (kPlainThreads / COAT_WARP) + warp;
    if (gi < total_groups) fetch(gi, cur);
    for (; gi < total_groups; gi += warps_total, cur = nxt) {
        if (gi + warps_total < total_groups) fetch(gi + warps_total, nxt);
        const TensorDesc& t = MULTI ? table[cur.ti] : single;
        const int64_t group = cur.group;
        const int64_t base = group * kGroup + lane * 4;
        bool ok = cur.ok;
        float p[4], g[4], m1[4], v1[4];
        float new_scale_m = 0.f, new_scale_v = 0.f;
        if (ok) {
            const float4 p4 = cur.p4, g4 = cur.g4;
            const uint32_t mw = cur.mw, vw = cur.vw;
            const float s_m = cur.s_m, s_v = cur.s_v;
            p[0] = p4.x; p[1] = p4.y; p[2] = p4.z; p[3] = p4.w;
            g[0] = g4.x; g[1] = g4.y; g[2] = g4.z; g[3] = g4.w;
            float fm[4], fv[4];
            coat_fp8x4_to_float4<COAT_E4M3>(mw, fm);
            coat_fp8x4_to_float4<COAT_E4M3>(vw, fv);
            float mx_m = 0.f, mx_v = 0.f;
#pragma unroll
            for (int jj = 0; jj < 4; jj += 2) {   // adam_first / adam_second, two elements per instruction
                const float2 gg = f2(g[jj], g[jj + 1]);
                const float2 m2 = __ffma2_rn(f2(h.beta1), __fmul2_rn(f2(fm[jj], fm[jj + 1]), f2(s_m)),
                                             __fmul2_rn(f2(c.om_beta1), gg));
                const float2 v2 = __ffma2_rn(f2(h.beta2), __fmul2_rn(f2(fv[jj], fv[jj + 1]), f2(s_v)),
                                             __fmul2_rn(__fmul2_rn(f2(c.om_beta2), gg), gg));
                m1[jj] = m2.x; m1[jj + 1] = m2.y; v1[jj] = v2.x; v1[jj + 1] = v2.y;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                mx_m = max_nan(mx_m, fabsf(m1[j]));
                mx_v = max_nan(mx_v, fabsf(v1[j]));
            }
            // non-negative or NaN (which orders above everything): unsigned order == float order
            mx_m = __uint_as_float(redux_max_f(mx_m));
            mx_v = __uint_as_float(redux_max_f(mx_v));
            // x + 1e-20 in double, rounded to float: x itself from 2^-40 up (the addend is below a quarter of its last place)
            const float a_m = (mx_m >= 9.094947e-13f && mx_m <= 3.0e38f) ? mx_m : (float)((double)mx_m + COAT_PLAIN_MIN_VAL);
            const float a_v = (mx_v >= 9.094947e-13f && mx_v <= 3.0e38f) ? mx_v : (float)((double)mx_v + COAT_PLAIN_MIN_VAL);
            new_scale_m = __fdiv_rn(a_m, 448.0f);
            new_scale_v = __fdiv_rn(a_v, 448.0f);
            // finite maxima and scales whose reciprocal the approximate unit handles at full accuracy
            ok = mx_m <= 1.0e30f && mx_v <= 1.0e30f && new_scale_m >= 1.0e-30f && new_scale_v >= 1.0e-30f;
        }
        if (!ok) {   // warp-uniform
            process_group_exact<float, false, false>(t, group, lane, h, c.om_beta1, c.om_beta2, c.correction1,
                                                     c.correction2_sqrt, desc_vec_ok(t, 16), smem_min[warp]);
            if (dbg && lane == 0) atomicAdd(dbg + 1, 1ull);
            continue;
        }
        // codes: both ends of the interval around m' / s'
        const float r_m = rcp_ftz(new_scale_m), r_v = rcp_ftz(new_scale_v);
        const float2 rm2 = f2(r_m * (1.0f - kRelHalfWidth), r_m * (1.0f + kRelHalfWidth));
        const float2 rv2 = f2(r_v * (1.0f - kRelHalfWidth), r_v * (1.0f + kRelHalfWidth));
        float ql[4], qh[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 q = __fmul2_rn(f2(m1[j]), rm2);
            ql[j] = q.x; qh[j] = q.y;
        }
        uint32_t cm = coat_float4_to_fp8x4<COAT_E4M3>(ql[0], ql[1], ql[2], ql[3]);
        const uint32_t dm = cm ^ coat_float4_to_fp8x4<COAT_E4M3>(qh[0], qh[1], qh[2], qh[3]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 q = __fmul2_rn(f2(v1[j]), rv2);
            ql[j] = q.x; qh[j] = q.y;
        }
        uint32_t cv = coat_float4_to_fp8x4<COAT_E4M3>(ql[0], ql[1], ql[2], ql[3]);
        const uint32_t dv = cv ^ coat_float4_to_fp8x4<COAT_E4M3>(qh[0], qh[1], qh[2], qh[3]);
        if (dm | dv) {   // rare: the exact division for the elements whose interval straddles a rounding boundary
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if ((dm >> (8 * j)) & 0xffu)
                    cm = (cm & ~(0xffu << (8 * j))) | (coat_float_to_fp8<COAT_E4M3>(__fdiv_rn(m1[j], new_scale_m)) << (8 * j));
                if ((dv >> (8 * j)) & 0xffu)
                    cv = (cv & ~(0xffu << (8 * j))) | (coat_float_to_fp8<COAT_E4M3>(__fdiv_rn(v1[j], new_scale_v)) << (8 * j));
            }
        }
        *reinterpret_cast<uint32_t*>(t.m + base) = cm;
        *reinterpret_cast<uint32_t*>(t.v + base) = cv;
        if (lane == 0) {
            t.s_m[group] = new_scale_m;
            t.s_v[group] = new_scale_v;
        }
        // weights from approximate square root and reciprocal (they are not quantised)
#pragma unroll
        for (int jj = 0; jj < 4; jj += 2) {
            const float2 denom = __ffma2_rn(f2(sqrt_ftz(v1[jj]), sqrt_ftz(v1[jj + 1])), f2(c.p_a), f2(c.p_b));
            const float2 pj = f2(p[jj], p[jj + 1]);
            const float2 update = __ffma2_rn(f2(h.wd), pj, __fmul2_rn(f2(m1[jj], m1[jj + 1]),
                                                                      f2(rcp_ftz(denom.x), rcp_ftz(denom.y))));
            const float2 pn = __ffma2_rn(f2(-h.lr), update, pj);
            p[jj] = pn.x; p[jj + 1] = pn.y;
        }
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(t.p) + base) = make_float4(p[0], p[1], p[2], p[3]);
        if (t.bf16_out) store_bf16x4_bcast<false>(reinterpret_cast<__nv_bfloat16*>(t.bf16_out) + base, p, h);
        if (dbg && lane == 0) atomicAdd(dbg + 0, 1ull);
    }
}

thread_local unsigned long long* g_debug_counters = nullptr;   // per host thread: only the caller's own launches count

int grid_for(int64_t total_groups) {
    int sms = coat_sm_count();
    int64_t ctas_needed = (total_groups + kWarpsPerCta - 1) / kWarpsPerCta;
    int64_t cap = (int64_t)sms * 8;  // persistent: up to 8 resident CTAs of 256 threads per SM
    return (int)(ctas_needed < cap ? (ctas_needed > 0 ? ctas_needed : 1) : cap);
}


template <typename scalar_t, bool EXPAND, bool MULTI>
int launch_typed(const TensorDesc& single, const TensorDesc* table, const int64_t* prefix, int n_tensors,
                 int64_t total_groups, const AdamwHyper& h, int flags, cudaStream_t st) {
    // The tiled guarded kernel serves fp32 (master) weights, the case the optimizer class supports; other
    // weight types and the COAT_ADAMW_EXACT_POW flag take the one-group-per-warp exact kernel.
    if constexpr (EXPAND && std::is_same<scalar_t, float>::value) {
        if (!(flags & COAT_ADAMW_EXACT_POW)) {
            // the broadcast variant exists for table launches only
            auto kern = (MULTI && h.n_peers > 0) ? fp8_adamw_expand_tiled_kernel<scalar_t, MULTI, MULTI>
                                                 : fp8_adamw_expand_tiled_kernel<scalar_t, MULTI, false>;
            const bool bcast = MULTI && h.n_peers > 0;
            const size_t smem = bcast ? kTiledSmemBcast : kTiledSmem;
            if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
                return COAT_E_LAUNCH;
            const int64_t tiles = (total_groups + kTile - 1) / kTile;
            const int64_t ctas_needed = (tiles + kTiledWarps - 1) / kTiledWarps;
            const int64_t cap = (int64_t)coat_sm_count() * tiled_ctas_per_sm(bcast);
            const int grid = (int)(ctas_needed < cap ? ctas_needed : cap);
            kern<<<grid, kTiledThreads, smem, st>>>(single, table, prefix, n_tensors, total_groups, h,
                                                          g_debug_counters);
            return coat_launch_status();
        }
    }
    if constexpr (!EXPAND && std::is_same<scalar_t, float>::value) {
        if (!(flags & COAT_ADAMW_EXACT_POW) && !(MULTI && h.n_peers > 0)) {
            const int64_t ctas_needed = (total_groups + kPlainThreads / COAT_WARP - 1) / (kPlainThreads / COAT_WARP);
            // persistent: exactly as many CTAs as are resident at once (a second wave would start when the first is done)
            static int per_sm = 0;
            if (per_sm == 0) {
                int n = 0;
                if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fp8_adamw_plain_fast_kernel<MULTI>, kPlainThreads, 0) !=
                    cudaSuccess || n < 1) n = 2;
                per_sm = n;
            }
            const int64_t cap = (int64_t)coat_sm_count() * per_sm;
            fp8_adamw_plain_fast_kernel<MULTI><<<(int)(ctas_needed < cap ? ctas_needed : cap), kPlainThreads, 0, st>>>(
                single, table, prefix, n_tensors, total_groups, h, g_debug_counters);
            return coat_launch_status();
        }
    }
    auto exact = (MULTI && h.n_peers > 0) ? fp8_adamw_kernel<scalar_t, EXPAND, MULTI, MULTI>
                                          : fp8_adamw_kernel<scalar_t, EXPAND, MULTI, false>;
    exact<<<grid_for(total_groups), kThreads, 0, st>>>(single, table, prefix, n_tensors, total_groups, h,
                                                       g_debug_counters);
    return coat_launch_status();
}

template <bool EXPAND, bool MULTI>
int launch(int p_dtype, const TensorDesc& single, const TensorDesc* table, const int64_t* prefix,
           int n_tensors, int64_t total_groups, const AdamwHyper& h, int flags, cudaStream_t st) {
    if (total_groups <= 0) return COAT_OK;
    switch (p_dtype) {
        case COAT_F32:
            return launch_typed<float, EXPAND, MULTI>(single, table, prefix, n_tensors, total_groups, h, flags, st);
        case COAT_BF16:
            return launch_typed<__nv_bfloat16, EXPAND, MULTI>(single, table, prefix, n_tensors, total_groups, h,
                                                             flags, st);
        case COAT_F16:
            return launch_typed<__half, EXPAND, MULTI>(single, table, prefix, n_tensors, total_groups, h, flags, st);
        default:
            return COAT_E_BADARG;
    }
}

}  // namespace

extern "C" int coat_fp8_adamw_expand_step(void* p, const void* g, uint8_t* m, float* s_m, float* k_m,
                                          float* r_m, uint8_t* v, float* s_v, float* k_v, float* r_v,
                                          float beta1, float beta2, float lr, float wd, float eps, int step,
                                          int qgroup, int expand_min, int64_t numel, int p_dtype,
                                          void* bf16_out, int flags, void* stream) {
    if (qgroup != kGroup) return COAT_E_QGROUP;
    if (numel < 0) return COAT_E_BADARG;
    if (numel == 0) return COAT_OK;
    if (!p || !g || !m || !v || !s_m || !k_m || !r_m || !s_v || !k_v || !r_v) return COAT_E_BADARG;
    TensorDesc t = {p, g, m, v, s_m, k_m, r_m, s_v, k_v, r_v, bf16_out, numel};
    AdamwHyper h = {beta1, beta2, lr, wd, eps, step, expand_min};
    return launch<true, false>(p_dtype, t, nullptr, nullptr, 1, (numel + kGroup - 1) / kGroup, h,
                               flags, (cudaStream_t)stream);
}

extern "C" int coat_fp8_adamw_step(void* p, const void* g, uint8_t* m, float* s_m, uint8_t* v, float* s_v,
                                   float beta1, float beta2, float lr, float wd, float eps, int step,
                                   int qgroup, int64_t numel, int p_dtype, void* bf16_out, int flags,
                                   void* stream) {
    if (qgroup != kGroup) return COAT_E_QGROUP;
    if (numel < 0) return COAT_E_BADARG;
    if (numel == 0) return COAT_OK;
    if (!p || !g || !m || !v || !s_m || !s_v) return COAT_E_BADARG;
    TensorDesc t = {p, g, m, v, s_m, nullptr, nullptr, s_v, nullptr, nullptr, bf16_out, numel};
    AdamwHyper h = {beta1, beta2, lr, wd, eps, step, 0};
    return launch<false, false>(p_dtype, t, nullptr, nullptr, 1, (numel + kGroup - 1) / kGroup, h,
                                flags, (cudaStream_t)stream);
}

extern "C" int coat_fp8_adamw_multi_step(const CoatAdamwTensor* table, const int64_t* group_prefix,
                                         int n_tensors, int64_t total_groups, int expand, float beta1,
                                         float beta2, float lr, float wd, float eps, int step, int qgroup,
                                         int expand_min, int p_dtype, int flags, void* stream) {
    if (qgroup != kGroup) return COAT_E_QGROUP;
    if (n_tensors < 0 || total_groups < 0) return COAT_E_BADARG;
    if (n_tensors == 0 || total_groups == 0) return COAT_OK;
    if (!table || !group_prefix) return COAT_E_BADARG;
    TensorDesc none = {};
    AdamwHyper h = {beta1, beta2, lr, wd, eps, step, expand_min};
    if (expand)
        return launch<true, true>(p_dtype, none, table, group_prefix, n_tensors, total_groups, h, flags,
                                  (cudaStream_t)stream);
    return launch<false, true>(p_dtype, none, table, group_prefix, n_tensors, total_groups, h, flags,
                               (cudaStream_t)stream);
}

// The table launch with the bf16 copy broadcast to peer GPUs: one kernel does the step and the "all-gather"
// (each GPU stores its slice into every peer's buffer while it computes).
extern "C" int coat_fp8_adamw_multi_step_bcast(const CoatAdamwTensor* table, const int64_t* group_prefix,
                                               int n_tensors, int64_t total_groups, int expand, float beta1,
                                               float beta2, float lr, float wd, float eps, int step, int qgroup,
                                               int expand_min, int p_dtype, int flags,
                                               const int64_t* peer_deltas, int n_peers, void* stream) {
    if (qgroup != kGroup) return COAT_E_QGROUP;
    if (n_tensors < 0 || total_groups < 0 || n_peers < 0 || n_peers > COAT_MAX_PEERS) return COAT_E_BADARG;
    if (n_peers > 0 && !peer_deltas) return COAT_E_BADARG;
    if (n_tensors == 0 || total_groups == 0) return COAT_OK;
    if (!table || !group_prefix) return COAT_E_BADARG;
    TensorDesc none = {};
    AdamwHyper h = {beta1, beta2, lr, wd, eps, step, expand_min};
    h.n_peers = n_peers;
    for (int i = 0; i < n_peers; ++i) {
        if (peer_deltas[i] % 16 != 0) return COAT_E_ALIGN;   // bulk stores keep their 16-byte alignment
        h.peer_delta[i] = peer_deltas[i];
    }
    if (expand)
        return launch<true, true>(p_dtype, none, table, group_prefix, n_tensors, total_groups, h, flags,
                                  (cudaStream_t)stream);
    return launch<false, true>(p_dtype, none, table, group_prefix, n_tensors, total_groups, h, flags,
                               (cudaStream_t)stream);
}

// Debug aid: six device counters (groups on the fast path, groups on the exact path, iterations of
// the max/min-candidate loop, iterations of the uncertain-rounding loop, uncertain elements, spare)
// that later launches FROM THE CALLING HOST THREAD add to; pass NULL to switch counting off.
extern "C" int coat_fp8_adamw_debug_counters(unsigned long long* device_counters) {
    g_debug_counters = device_counters;
    return COAT_OK;
}

// Reads (and clears) the device-side status word of the optimizer kernels on the current device:
// COAT_OK, or COAT_E_TIMEOUT if a bounded wait on a staging copy ever ran out.  Synchronises the device.
extern "C" int coat_fp8_adamw_device_status(void) {
    int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_adamw_device_status, sizeof(int)) != cudaSuccess) return COAT_E_LAUNCH;
    if (v != 0 && cudaMemcpyToSymbol(g_adamw_device_status, &zero, sizeof(int)) != cudaSuccess) return COAT_E_LAUNCH;
    return v;
}
