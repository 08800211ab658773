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

#include "common.cuh"

namespace {

constexpr int kGroup = 128;          // elements per quantization group
constexpr int kThreads = 256;        // 8 warps per CTA
constexpr int kWarpsPerCta = kThreads / COAT_WARP;

struct AdamwHyper {
    float beta1, beta2, lr, wd, eps;
    int step;
    int expand_min;
};

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

// ---- per-group scalars of the expansion ------------------------------------------
// fp8_adamw_expand_cuda_kernel.cu:151-181.  QUANT_MIN_VAL is a double literal there, so
// the additions are done in double and rounded back to float.
#define COAT_EXPAND_MIN_VAL 1e-30
#define COAT_PLAIN_MIN_VAL 1e-20

__device__ __forceinline__ void expand_group_scalars(float absmax, float absmin, int expand_min,
                                                     float& maxv, float& sqrt_minmax, float& expo,
                                                     float& new_scale) {
    float fp8MaxVal = 448;
    float firstMaxVal = absmax + COAT_EXPAND_MIN_VAL;
    float firstMinVal = absmin + COAT_EXPAND_MIN_VAL;
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
template <typename scalar_t, bool EXPAND>
__device__ __forceinline__ void process_group_exact(const TensorDesc& t, int64_t group, int lane,
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
        float_exp_avg = h.beta1 * float_exp_avg + om_beta1 * g[j];
        float_exp_avg_sq = h.beta2 * float_exp_avg_sq + om_beta2 * g[j] * g[j];
        float denom = (sqrtf(float_exp_avg_sq) / correction2_sqrt + h.eps) * correction1;
        float update = (float_exp_avg / denom) + (h.wd * p[j]);
        p[j] = p[j] - (h.lr * update);
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
            Elem4<__nv_bfloat16>::store(reinterpret_cast<__nv_bfloat16*>(t.bf16_out) + base, q);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (j < nvalid) {
                E::put(pp + j, p[j]);
                if (t.bf16_out)
                    reinterpret_cast<__nv_bfloat16*>(t.bf16_out)[base + j] = __float2bfloat16_rn(E::round(p[j]));
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

template <typename scalar_t, bool EXPAND, bool MULTI>
__global__ void __launch_bounds__(kThreads)
fp8_adamw_kernel(TensorDesc single, const TensorDesc* __restrict__ table,
                 const int64_t* __restrict__ group_prefix, int n_tensors, int64_t total_groups,
                 AdamwHyper h) {
    __shared__ float smem_min[kWarpsPerCta][kGroup];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    // hoisted per-launch scalars, evaluated on the device with the same routines as
    // the reference (fp8_adamw_expand_cuda_kernel.cu:52-58)
    const float om_beta1 = 1 - h.beta1;
    const float om_beta2 = 1 - h.beta2;
    const float correction1 = 1.0f - powf(h.beta1, h.step);
    const float correction2_sqrt = sqrtf(1.0f - powf(h.beta2, h.step));

    const int64_t warps_total = (int64_t)gridDim.x * kWarpsPerCta;
    int64_t gi = (int64_t)blockIdx.x * kWarpsPerCta + warp;
    if (!MULTI) {
        const bool vec_ok = desc_vec_ok(single, Elem4<scalar_t>::kVecAlign);
        for (; gi < total_groups; gi += warps_total)
            process_group_exact<scalar_t, EXPAND>(single, gi, lane, h, om_beta1, om_beta2, correction1,
                                                  correction2_sqrt, vec_ok, smem_min[warp]);
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
            process_group_exact<scalar_t, EXPAND>(t, gi - group_prefix[ti], lane, h, om_beta1, om_beta2,
                                                  correction1, correction2_sqrt, vec_ok, smem_min[warp]);
        }
    }
}

int grid_for(int64_t total_groups) {
    int sms = coat_sm_count();
    int64_t ctas_needed = (total_groups + kWarpsPerCta - 1) / kWarpsPerCta;
    int64_t cap = (int64_t)sms * 8;  // persistent: up to 8 resident CTAs of 256 threads per SM
    return (int)(ctas_needed < cap ? (ctas_needed > 0 ? ctas_needed : 1) : cap);
}

template <bool EXPAND, bool MULTI>
int launch(int p_dtype, const TensorDesc& single, const TensorDesc* table, const int64_t* prefix,
           int n_tensors, int64_t total_groups, const AdamwHyper& h, cudaStream_t st) {
    if (total_groups <= 0) return COAT_OK;
    int grid = grid_for(total_groups);
    switch (p_dtype) {
        case COAT_F32:
            fp8_adamw_kernel<float, EXPAND, MULTI><<<grid, kThreads, 0, st>>>(single, table, prefix, n_tensors,
                                                                             total_groups, h);
            break;
        case COAT_BF16:
            fp8_adamw_kernel<__nv_bfloat16, EXPAND, MULTI><<<grid, kThreads, 0, st>>>(single, table, prefix,
                                                                                     n_tensors, total_groups, h);
            break;
        case COAT_F16:
            fp8_adamw_kernel<__half, EXPAND, MULTI><<<grid, kThreads, 0, st>>>(single, table, prefix, n_tensors,
                                                                              total_groups, h);
            break;
        default:
            return COAT_E_BADARG;
    }
    return coat_launch_status();
}

}  // namespace

extern "C" int coat_fp8_adamw_expand_step(void* p, const void* g, uint8_t* m, float* s_m, float* k_m,
                                          float* r_m, uint8_t* v, float* s_v, float* k_v, float* r_v,
                                          float beta1, float beta2, float lr, float wd, float eps, int step,
                                          int qgroup, int expand_min, int64_t numel, int p_dtype,
                                          void* bf16_out, int flags, void* stream) {
    (void)flags;
    if (qgroup != kGroup) return COAT_E_QGROUP;
    if (numel < 0) return COAT_E_BADARG;
    if (numel == 0) return COAT_OK;
    if (!p || !g || !m || !v || !s_m || !k_m || !r_m || !s_v || !k_v || !r_v) return COAT_E_BADARG;
    TensorDesc t = {p, g, m, v, s_m, k_m, r_m, s_v, k_v, r_v, bf16_out, numel};
    AdamwHyper h = {beta1, beta2, lr, wd, eps, step, expand_min};
    return launch<true, false>(p_dtype, t, nullptr, nullptr, 1, (numel + kGroup - 1) / kGroup, h,
                               (cudaStream_t)stream);
}

extern "C" int coat_fp8_adamw_step(void* p, const void* g, uint8_t* m, float* s_m, uint8_t* v, float* s_v,
                                   float beta1, float beta2, float lr, float wd, float eps, int step,
                                   int qgroup, int64_t numel, int p_dtype, void* bf16_out, int flags,
                                   void* stream) {
    (void)flags;
    if (qgroup != kGroup) return COAT_E_QGROUP;
    if (numel < 0) return COAT_E_BADARG;
    if (numel == 0) return COAT_OK;
    if (!p || !g || !m || !v || !s_m || !s_v) return COAT_E_BADARG;
    TensorDesc t = {p, g, m, v, s_m, nullptr, nullptr, s_v, nullptr, nullptr, bf16_out, numel};
    AdamwHyper h = {beta1, beta2, lr, wd, eps, step, 0};
    return launch<false, false>(p_dtype, t, nullptr, nullptr, 1, (numel + kGroup - 1) / kGroup, h,
                                (cudaStream_t)stream);
}

extern "C" int coat_fp8_adamw_multi_step(const CoatAdamwTensor* table, const int64_t* group_prefix,
                                         int n_tensors, int64_t total_groups, int expand, float beta1,
                                         float beta2, float lr, float wd, float eps, int step, int qgroup,
                                         int expand_min, int p_dtype, int flags, void* stream) {
    (void)flags;
    if (qgroup != kGroup) return COAT_E_QGROUP;
    if (n_tensors < 0 || total_groups < 0) return COAT_E_BADARG;
    if (n_tensors == 0 || total_groups == 0) return COAT_OK;
    if (!table || !group_prefix) return COAT_E_BADARG;
    TensorDesc none = {};
    AdamwHyper h = {beta1, beta2, lr, wd, eps, step, expand_min};
    if (expand)
        return launch<true, true>(p_dtype, none, table, group_prefix, n_tensors, total_groups, h,
                                  (cudaStream_t)stream);
    return launch<false, true>(p_dtype, none, table, group_prefix, n_tensors, total_groups, h,
                               (cudaStream_t)stream);
}
