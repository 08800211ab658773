// Fused "quantize-on-save" element-wise operators for sm_100a: SiLU / GELU forward and backward, the
// gated product forward and backward, and the residual add, each dequantising its 1xQB-quantised FP8
// inputs on the fly, computing in fp32, and emitting a bf16 result and / or a 1xQB-quantised FP8 result,
// the per-group scales, and the tensor's amax for a following per-tensor division.
//
// Arithmetic follows the reference's Triton kernels (paths under coat/activation/real_quantization/):
//   silu_fwd.py:100-118   x = code*s ; sig = 1/(1+exp(-x)) ; y = sig*x ; group quantize
//   silu_bwd.py:112-137   (sig + x*sig*(1-sig)) * g -> bf16, group scales
//   gelu_fwd.py:100-118   0.5*(1+erf(x/sqrt 2))*x -> bf16, group scales
//   gelu_bwd.py:112-140   (cdf + x*exp(-x^2/2)/sqrt(2 pi)) * g -> bf16, group scales
//   mul_fwd.py:101-127    (c1*s1)*(c2*s2) -> bf16, group scales
//   mul_bwd.py:117-152    g*x2 -> bf16 ; g*x1 -> bf16, group scales
//   add_fwd.py:92-121     a+b -> bf16 and 1xQB FP8 + scales ;  add_bwd.py:92-113  a+b -> bf16, group scales
// Where the reference then calls `s_y.max()` and fp8_division[_transpose] on the bf16 result, the kernels
// here also leave the tensor's amax (of the fp32 values, as the group scales are) in a scratch word, so
// that coat_fp8_division can derive the same scale without a reduction pass.
//
// One thread owns 16 consecutive elements of a row (16-byte loads of codes, 32-byte loads of bf16);
// groups wider than 16 are reduced over the QB/16 neighbouring lanes.

#include <math.h>

#include "quant_common.cuh"

namespace {

enum FusedOp { OP_SILU_FWD = 0, OP_SILU_BWD, OP_GELU_FWD, OP_GELU_BWD, OP_MUL_FWD, OP_MUL_BWD, OP_ADD };

struct FusedArgs {
    const uint8_t* x1; const void* s1;      // first quantised input and its 1xQB scales
    const uint8_t* x2; const void* s2;      // second quantised input (gated product)
    const void* g;                          // bf16 upstream gradient, or first addend (add)
    const void* h;                          // second addend (add)
    __nv_bfloat16* y_bf16;                  // bf16 result (may be null)
    __nv_bfloat16* y1_bf16;                 // mul backward: g * x2
    uint8_t* y_q;                           // 1xQB FP8 result (may be null)
    void* s_y;                              // group scales of the result (may be null)
    unsigned int* amax_bits;                // tensor amax (may be null)
    int64_t M, N;
    int QB;
    int in_scale_dtype, out_scale_dtype;
    int g_dtype, h_dtype;                   // dtypes of the floating inputs
    float fp8_max;                          // largest finite value of the FP8 format the scales are for
};

template <int FMT>
// contiguous rows, N a multiple of QB: segment `seg` of the matrix belongs to group seg >> lane_shift
__device__ __forceinline__ void load_dequant16(const uint8_t* codes, const void* scales, int scale_dtype, int64_t seg,
                                               int lane_shift, float (&x)[16]) {
    const uint4 w = *reinterpret_cast<const uint4*>(codes + seg * 16);
    const float s = load_scale(scales, seg >> lane_shift, scale_dtype);
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float f[4];
        coat_fp8x4_to_float4<FMT>(ww[i], f);
#pragma unroll
        for (int j = 0; j < 4; ++j) x[4 * i + j] = f[j] * s;
    }
}

__device__ __forceinline__ void load_float16(const void* base, int dtype, int64_t off, float (&x)[16]) {
    if (dtype == COAT_BF16) Seg16<__nv_bfloat16>::load(reinterpret_cast<const __nv_bfloat16*>(base) + off, x);
    else if (dtype == COAT_F16) Seg16<__half>::load(reinterpret_cast<const __half*>(base) + off, x);
    else Seg16<float>::load(reinterpret_cast<const float*>(base) + off, x);
}

__device__ __forceinline__ void store_bf16x16(__nv_bfloat16* dst, const float (&v)[16]) {
    uint32_t o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
        o[i] = (uint32_t)coat_float_to_bf16_bits(v[2 * i]) | ((uint32_t)coat_float_to_bf16_bits(v[2 * i + 1]) << 16);
    reinterpret_cast<uint4*>(dst)[0] = make_uint4(o[0], o[1], o[2], o[3]);
    reinterpret_cast<uint4*>(dst)[1] = make_uint4(o[4], o[5], o[6], o[7]);
}

// sigmoid exactly as `1 / (1.0 + libdevice.exp(-x))` compiles: libdevice expf, then the non-IEEE division
template <bool IEEE>
__device__ __forceinline__ float sigmoid_ref(float x) { return qdiv<IEEE>(1.0f, 1.0f + expf(-x)); }

__device__ __forceinline__ float sqrt_approx(float x) { float r; asm("sqrt.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x)); return r; }
__device__ __forceinline__ float ex2_approx_noftz(float x) { float r; asm("ex2.approx.f32 %0, %1;" : "=f"(r) : "f"(x)); return r; }
// `tl.math.sqrt(2.0)` and `tl.sqrt(2 * pi)` of the GELU kernels are folded by Triton's compiler into the correctly
// rounded constants 0x3FB504F3 and 0x40206C99 (gelu_fwd.py:109, gelu_bwd.py:127-128); a run-time sqrt.approx of the
// same arguments is one step off for the second, which flips a few codes per hundred thousand.
__device__ constexpr float kSqrt2 = 1.41421353816986083984375f;     // 0x3FB504F3
__device__ constexpr float kSqrt2Pi = 2.5066282749176025390625f;    // 0x40206C99

// (no minimum number of CTAs per SM in the launch bounds: a minimum of 1 lets the compiler spend registers that cost
// occupancy, SiLU backward 219 us instead of 178 us; minima of 6 and 8 measured no better than leaving it out)
template <int OP, int FMT_IN, int FMT_OUT, bool IEEE>
__global__ void __launch_bounds__(kStraightThreads)
fused_elementwise_kernel(FusedArgs a) {
    // one 16-element segment per thread, one trip; every operand has contiguous rows, so no index division
    const int64_t total = a.M * (a.N >> 4);
    const int lanes = a.QB >> 4;
    const int lane_shift = 31 - __clz(lanes);
    const float fp8_max = a.fp8_max;
    float block_max = 0.f;
    {
        const int64_t seg = (int64_t)blockIdx.x * kStraightThreads + threadIdx.x;
        const bool live = seg < total;
        const int64_t off = seg * 16;
        float v[16];
        float amax = 0.f;
        if (live) {
            float x[16], t[16];
            if (OP == OP_ADD) {
                load_float16(a.g, a.g_dtype, off, x);
                load_float16(a.h, a.h_dtype, off, t);
#pragma unroll
                for (int i = 0; i < 16; ++i) v[i] = x[i] + t[i];
            } else {
                load_dequant16<FMT_IN>(a.x1, a.s1, a.in_scale_dtype, seg, lane_shift, x);
                if (OP == OP_SILU_FWD) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) v[i] = sigmoid_ref<IEEE>(x[i]) * x[i];
                } else if (OP == OP_SILU_BWD) {
                    load_float16(a.g, a.g_dtype, off, t);
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float sg = sigmoid_ref<IEEE>(x[i]);
                        // sigmoid + input * sigmoid * (1 - sigmoid), the outer multiply-add contracted
                        v[i] = __fmaf_rn(x[i] * sg, 1.0f - sg, sg) * t[i];
                    }
                } else if (OP == OP_GELU_FWD) {
                    const float rt2 = kSqrt2;
#pragma unroll
                    for (int i = 0; i < 16; ++i) v[i] = qdiv<IEEE>(1.0f + erff(qdiv<IEEE>(x[i], rt2)), 2.0f) * x[i];
                } else if (OP == OP_GELU_BWD) {
                    load_float16(a.g, a.g_dtype, off, t);
                    const float rt2 = kSqrt2, rt2pi = kSqrt2Pi;
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float cdf = qdiv<IEEE>(1.0f + erff(qdiv<IEEE>(x[i], rt2)), 2.0f);
                        // libdevice.pow(x, 2) is x * x; tl.exp(u) is ex2.approx(u * log2 e) without flush-to-zero
                        const float e = ex2_approx_noftz(qdiv<IEEE>(0.0f - __fmul_rn(x[i], x[i]), 2.0f) * 1.4426950408889634f);
                        v[i] = (cdf + qdiv<IEEE>(x[i] * e, rt2pi)) * t[i];
                    }
                } else {   // OP_MUL_FWD, OP_MUL_BWD
                    load_dequant16<FMT_IN>(a.x2, a.s2, a.in_scale_dtype, seg, lane_shift, t);
                    if (OP == OP_MUL_FWD) {
#pragma unroll
                        for (int i = 0; i < 16; ++i) v[i] = x[i] * t[i];
                    } else {
                        float gr[16], y1[16];
                        load_float16(a.g, a.g_dtype, off, gr);
#pragma unroll
                        for (int i = 0; i < 16; ++i) { y1[i] = gr[i] * t[i]; v[i] = gr[i] * x[i]; }
                        store_bf16x16(a.y1_bf16 + off, y1);
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
        }
        amax = subgroup_max(amax, lanes);   // whole warps: the grid is rounded up to blocks of 256 threads
        if (live) {
            const float scale = qdiv<IEEE>(amax + kScaleMinThres, fp8_max);
            if (a.y_bf16) store_bf16x16(a.y_bf16 + off, v);
            if (a.y_q) {
                float q[16];
                ScaleDivider<IEEE>(scale).apply(v, q);
                *reinterpret_cast<uint4*>(a.y_q + off) = pack16<FMT_OUT>(q);
            }
            if (a.s_y && (seg & (lanes - 1)) == 0) store_scale(a.s_y, seg >> lane_shift, a.out_scale_dtype, scale);
            block_max = amax;
        }
    }
    if (a.amax_bits) {
        block_max = coat_warp_max(block_max);
        __shared__ float wmax[kStraightThreads / 32];
        if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = block_max;
        __syncthreads();
        if (threadIdx.x < 32) {
            float m = threadIdx.x < kStraightThreads / 32 ? wmax[threadIdx.x] : 0.f;
            m = coat_warp_max(m);
            if (threadIdx.x == 0) atomicMax(a.amax_bits, __float_as_uint(m));
        }
    }
}

// =================================================================================================
// Gated-MLP backward in one kernel: fp8_mul_backward (mul_bwd.py:117-152) followed by fp8_silu_backward
// (silu_bwd.py:112-137) without the bf16 round trip of the gradient that goes from one to the other.
//   d_up   = g * silu_x                                  -> bf16 + 1xQB scales + tensor amax  (mul backward's 2nd output)
//   t      = bf16(g * up)                                 (mul backward's 1st output, as the reference rounds it)
//   d_gate = (sig + gate * sig * (1 - sig)) * t           -> bf16 + 1xQB scales + tensor amax  (silu backward)
// Same bits as the two kernels one after the other; the memory-latency-bound product and the instruction-bound
// sigmoid overlap inside one kernel, and 4 bytes per element less go through memory.
// =================================================================================================
struct MulSiluBwdArgs {
    const uint8_t* x_silu; const void* s_silu;
    const uint8_t* x_up; const void* s_up;
    const uint8_t* x_gate; const void* s_gate;
    const void* g; int g_dtype;
    __nv_bfloat16* y_up; void* sy_up; unsigned int* amax_up;
    __nv_bfloat16* y_gate; void* sy_gate; unsigned int* amax_gate;
    int64_t M, N;
    int QB, in_scale_dtype;
    float fp8_max;
};

// four CTAs per SM (64 registers): 379 us against 415 us without the bound and 390 us with five (8192 x 11008, both
// division+transpose passes included)
template <int FMT_IN, bool IEEE>
__global__ void __launch_bounds__(kStraightThreads, 4)
mul_silu_backward_kernel(MulSiluBwdArgs a) {
    const int64_t total = a.M * (a.N >> 4);
    const int lanes = a.QB >> 4;
    const int lane_shift = 31 - __clz(lanes);
    const int64_t seg = (int64_t)blockIdx.x * kStraightThreads + threadIdx.x;
    const bool live = seg < total;
    const int64_t off = seg * 16;
    float d_up[16], d_gate[16];
    float amax_up = 0.f, amax_gate = 0.f;
    if (live) {
        float xs[16], xu[16], xg[16], gr[16];
        load_dequant16<FMT_IN>(a.x_silu, a.s_silu, a.in_scale_dtype, seg, lane_shift, xs);
        load_dequant16<FMT_IN>(a.x_up, a.s_up, a.in_scale_dtype, seg, lane_shift, xu);
        load_dequant16<FMT_IN>(a.x_gate, a.s_gate, a.in_scale_dtype, seg, lane_shift, xg);
        load_float16(a.g, a.g_dtype, off, gr);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            d_up[i] = gr[i] * xs[i];
            const float t = __bfloat162float(__float2bfloat16_rn(gr[i] * xu[i]));
            const float sg = sigmoid_ref<IEEE>(xg[i]);
            d_gate[i] = __fmaf_rn(xg[i] * sg, 1.0f - sg, sg) * t;
            amax_up = fmaxf(amax_up, fabsf(d_up[i]));
            amax_gate = fmaxf(amax_gate, fabsf(d_gate[i]));
        }
    }
    amax_up = subgroup_max(amax_up, lanes);     // whole warps: the grid is rounded up to blocks of 256 threads
    amax_gate = subgroup_max(amax_gate, lanes);
    if (live) {
        store_bf16x16(a.y_up + off, d_up);
        store_bf16x16(a.y_gate + off, d_gate);
        if ((seg & (lanes - 1)) == 0) {
            store_scale(a.sy_up, seg >> lane_shift, COAT_BF16, qdiv<IEEE>(amax_up + kScaleMinThres, a.fp8_max));
            store_scale(a.sy_gate, seg >> lane_shift, COAT_BF16, qdiv<IEEE>(amax_gate + kScaleMinThres, a.fp8_max));
        }
    }
    amax_up = coat_warp_max(live ? amax_up : 0.f);
    amax_gate = coat_warp_max(live ? amax_gate : 0.f);
    __shared__ float wmax[2][kStraightThreads / 32];
    if ((threadIdx.x & 31) == 0) { wmax[0][threadIdx.x >> 5] = amax_up; wmax[1][threadIdx.x >> 5] = amax_gate; }
    __syncthreads();
    if (threadIdx.x < 64) {
        const int which = threadIdx.x >> 5, l = threadIdx.x & 31;
        float m = l < kStraightThreads / 32 ? wmax[which][l] : 0.f;
        m = coat_warp_max(m);
        if (l == 0) atomicMax(which ? a.amax_gate : a.amax_up, __float_as_uint(m));
    }
}

// =================================================================================================
// Gated-MLP forward in one kernel: fp8_silu_forward (silu_fwd.py:100-118) followed by fp8_mul_forward's kernel
// (mul_fwd.py:101-127).  silu(gate) is quantised in 1xQB groups (codes and scales are outputs: the backward pass
// needs them) and the product is formed from those codes times the ROUNDED scale, which is what the second
// operator would read back from memory; the product leaves as bf16 with its group scales and the tensor amax.
// =================================================================================================
struct SiluMulFwdArgs {
    const uint8_t* x_gate; const void* s_gate;
    const uint8_t* x_up; const void* s_up;
    uint8_t* q_silu; void* s_silu;
    __nv_bfloat16* y; void* s_y; unsigned int* amax;
    int64_t M, N;
    int QB, scale_dtype;
    float fp8_max;
};

template <int FMT, bool IEEE>
__global__ void __launch_bounds__(kStraightThreads)
silu_mul_forward_kernel(SiluMulFwdArgs a) {
    const int64_t total = a.M * (a.N >> 4);
    const int lanes = a.QB >> 4;
    const int lane_shift = 31 - __clz(lanes);
    const int64_t seg = (int64_t)blockIdx.x * kStraightThreads + threadIdx.x;
    const bool live = seg < total;
    const int64_t off = seg * 16;
    float v[16], xu[16];
    float amax = 0.f;
    if (live) {
        float xg[16];
        load_dequant16<FMT>(a.x_gate, a.s_gate, a.scale_dtype, seg, lane_shift, xg);
        load_dequant16<FMT>(a.x_up, a.s_up, a.scale_dtype, seg, lane_shift, xu);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            v[i] = sigmoid_ref<IEEE>(xg[i]) * xg[i];
            amax = fmaxf(amax, fabsf(v[i]));
        }
    }
    amax = subgroup_max(amax, lanes);   // whole warps: the grid is rounded up to blocks of 256 threads
    float pmax = 0.f;
    if (live) {
        const float scale = qdiv<IEEE>(amax + kScaleMinThres, a.fp8_max);
        float q[16];
        ScaleDivider<IEEE>(scale).apply(v, q);
        const uint4 codes = pack16<FMT>(q);
        *reinterpret_cast<uint4*>(a.q_silu + off) = codes;
        if ((seg & (lanes - 1)) == 0) store_scale(a.s_silu, seg >> lane_shift, a.scale_dtype, scale);
        const float stored = round_to_dtype(scale, a.scale_dtype);   // what the product operator reads back
        const uint32_t ww[4] = {codes.x, codes.y, codes.z, codes.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float f[4];
            coat_fp8x4_to_float4<FMT>(ww[i], f);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                v[4 * i + j] = (f[j] * stored) * xu[4 * i + j];
                pmax = fmaxf(pmax, fabsf(v[4 * i + j]));
            }
        }
    }
    pmax = subgroup_max(pmax, lanes);
    if (live) {
        store_bf16x16(a.y + off, v);
        if (a.s_y && (seg & (lanes - 1)) == 0)
            store_scale(a.s_y, seg >> lane_shift, a.scale_dtype, qdiv<IEEE>(pmax + kScaleMinThres, a.fp8_max));
    }
    pmax = coat_warp_max(live ? pmax : 0.f);
    __shared__ float wmax[kStraightThreads / 32];
    if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = pmax;
    __syncthreads();
    if (threadIdx.x < 32) {
        float m = threadIdx.x < kStraightThreads / 32 ? wmax[threadIdx.x] : 0.f;
        m = coat_warp_max(m);
        if (threadIdx.x == 0) atomicMax(a.amax, __float_as_uint(m));
    }
}

// =================================================================================================
// RMSNorm on a 1xQB-quantised input (func_rmsnorm.py:54-111 forward, :121-220 backward)
// =================================================================================================
// One CTA of 256 threads per row; thread t owns S 16-element segments (forward: S t ... S t + S - 1, the
// reference's layout; backward: t, t+256, ...) in registers, so a row of up to 16384 elements is read once.  Row sums are reduced in a fixed order
// (inside a thread, xor-shuffles inside a warp, then a tree over the 8 warp results), so the result does not
// depend on scheduling; the forward kernels use the order of the reference's compiled kernels
// (ref_order_row_sum), which makes rstd, and with it every output, bit-identical to the reference's.
constexpr int kNormThreads = 256;

// the eight warp sums combined as a butterfly over eight lanes does it (xor 4, 2, 1)
__device__ __forceinline__ float block_sum_of_warp_sums(float v, float* smem /*[8]*/) {
    __syncthreads();   // protects smem reuse between consecutive reductions
    if ((threadIdx.x & 31) == 0) smem[threadIdx.x >> 5] = v;
    __syncthreads();
    const float a0 = __fadd_rn(smem[0], smem[4]), a1 = __fadd_rn(smem[1], smem[5]);
    const float a2 = __fadd_rn(smem[2], smem[6]), a3 = __fadd_rn(smem[3], smem[7]);
    return __fadd_rn(__fadd_rn(a0, a2), __fadd_rn(a1, a3));
}
__device__ __forceinline__ float block_sum(float v, float* smem /*[8]*/) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(COAT_FULL_MASK, v, o);
    return block_sum_of_warp_sums(v, smem);
}

// Row sum of products a_i * b_i in the ORDER the reference's norm kernels use on this architecture, so that the
// forward statistics (and with them every code) come out bit-identical to the reference's.  Its Triton kernels run
// one program of 256 threads per row over the row padded with zeros to a power of two n2 (func_rmsnorm.py:82-95).
// The layouts and the contractions below are read from that compiler's own output for sm_100 (its layout
// attributes and PTX text), n2 = 256 ... 16384:
//   * thread t holds the E = max(1, n2 / 256) consecutive elements E t ... E t + E - 1; its registers hold them in
//     the order r = 0, 1, ...: element (r % G) * 16 + r / G with G = max(1, E / 16) (for E <= 16 simply in order;
//     beyond, the thread's G groups of 16 interleaved);
//   * E >= 2: p = a[r1] * b[r1]; p = fma(a[r0], b[r0], p); p = fma(a[r], b[r], p) for r = 2, 3, ... (every product
//     contracted into the running sum), then p += shfl_xor(p, 16), 8, 4, 2, 1;
//   * E == 1: p = fma(a, b, shfl_xor(a * b, 16)) (the product is contracted into the first exchange), then 8, 4, 2, 1;
//   * the eight warp sums are combined as a butterfly over eight lanes (xor 4, 2, 1).
// `f(k, i, A, B)` yields the factors of element i of this thread's k-th group of 16 (zeros in the padding).  With
// n2 >= 4096 thread t of this kernel holds the same elements as the reference's thread t (groups S t ... S t + S - 1,
// S = n2 / 4096); shorter rows go through shared memory, one slot per thread of the reference's layout.  Rows of
// fewer than 32 elements are summed in this order too, which is not the reference's there.
template <int E, class F>
__device__ __forceinline__ void ref_order_partials(F f, float* part_a, float* part_b) {
#pragma unroll
    for (int j = 0; j < 16; j += E) {
        float A, B;
        const int slot = (threadIdx.x * 16 + j) / E;
        if (E == 1) {
            f(0, j, A, B);
            part_a[slot] = A;
            part_b[slot] = B;
        } else {
            f(0, j + 1, A, B);
            float p = __fmul_rn(A, B);
            f(0, j, A, B);
            p = __fmaf_rn(A, B, p);
#pragma unroll
            for (int i = 2; i < E; ++i) {
                f(0, j + i, A, B);
                p = __fmaf_rn(A, B, p);
            }
            part_a[slot] = p;
        }
    }
}

template <int S, class F>
__device__ __forceinline__ float ref_order_row_sum(F f, int n2, float* part /*[512]*/, float* red /*[8]*/) {
    float p, A, B;
    if (n2 >= 4096) {   // S == n2 / 4096; register r = element i = r / S of group k = r % S
        f(1 % S, 1 / S, A, B);
        p = __fmul_rn(A, B);
        f(0, 0, A, B);
        p = __fmaf_rn(A, B, p);
#pragma unroll
        for (int r = 2; r < 16 * S; ++r) {
            f(r % S, r / S, A, B);
            p = __fmaf_rn(A, B, p);
        }
        p += __shfl_xor_sync(COAT_FULL_MASK, p, 16);
    } else {
        const int e = n2 >= 256 ? n2 >> 8 : 1;
        float* part_b = part + kNormThreads;
        __syncthreads();
        part[threadIdx.x] = 0.f;
        part_b[threadIdx.x] = 0.f;
        __syncthreads();
        if ((int)threadIdx.x < (n2 >> 4)) {
            if (e == 1) ref_order_partials<1>(f, part, part_b);
            else if (e == 2) ref_order_partials<2>(f, part, part_b);
            else if (e == 4) ref_order_partials<4>(f, part, part_b);
            else ref_order_partials<8>(f, part, part_b);
        }
        __syncthreads();
        if (e == 1) {
            A = part[threadIdx.x];
            B = part_b[threadIdx.x];
            p = __fmaf_rn(A, B, __shfl_xor_sync(COAT_FULL_MASK, __fmul_rn(A, B), 16));
        } else {
            p = part[threadIdx.x];
            p += __shfl_xor_sync(COAT_FULL_MASK, p, 16);
        }
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) p += __shfl_xor_sync(COAT_FULL_MASK, p, o);
    return block_sum_of_warp_sums(p, red);
}

__device__ __forceinline__ int next_pow2_at_least_16(int64_t n) {
    int p = 16;
    while (p < n) p <<= 1;
    return p;
}

__device__ __forceinline__ float block_max(float v, float* smem /*[8]*/) {
    v = coat_warp_max(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) smem[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = 0.f;
#pragma unroll
    for (int w = 0; w < kNormThreads / 32; ++w) r = fmaxf(r, smem[w]);
    return r;
}

__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

// The backward kernels walk rows one after the other and every row ends in block reductions, so only one row's
// loads are in flight per CTA: the next row's codes and gradient are pulled into L2 while this row is reduced.
template <int S>
__device__ __forceinline__ void prefetch_row(const uint8_t* x, const void* dy, int dy_dtype, int64_t row, int64_t M,
                                             int64_t N, int64_t segs) {
    if (row >= M) return;
    const int64_t dy_bytes = dy_dtype == COAT_F32 ? 4 : 2;
#pragma unroll
    for (int k = 0; k < S; ++k) {
        const int64_t c16 = threadIdx.x + (int64_t)k * kNormThreads;
        if (c16 < segs) {
            if (x && (threadIdx.x & 7) == 0) prefetch_l2(x + (row * segs + c16) * 16);   // 8 segments of codes per 128-byte line
            const char* g = reinterpret_cast<const char*>(dy) + (row * N + c16 * 16) * dy_bytes;
            if (dy_bytes == 4 || (threadIdx.x & 3) == 0) prefetch_l2(g);          // 32 (64) bytes of gradient per segment
        }
    }
}

template <int FMT, int S, bool IEEE>
__global__ void __launch_bounds__(kNormThreads)
rmsnorm_fwd_kernel(const uint8_t* __restrict__ x, const void* __restrict__ s_x, int in_scale_dtype,
                   const void* __restrict__ w, int w_dtype, __nv_bfloat16* __restrict__ y,
                   __nv_bfloat16* __restrict__ s_y, float* __restrict__ rstd_out, unsigned int* __restrict__ amax_bits,
                   int64_t M, int64_t N, int QB, float eps, int fp8_fmt_out) {
    __shared__ float red[kNormThreads / 32];
    __shared__ float part[2 * kNormThreads];
    const int64_t row = blockIdx.x;
    const int64_t segs = N >> 4;
    float v[S][16];
#pragma unroll
    for (int k = 0; k < S; ++k) {
        const int64_t c16 = (int64_t)threadIdx.x * S + k;   // the reference's layout: S consecutive groups per thread
        if (c16 < segs) {
            load_dequant16<FMT>(x, s_x, in_scale_dtype, row * segs + c16, 31 - __clz(QB >> 4), v[k]);
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) v[k][i] = 0.f;
        }
    }
    const float ss = ref_order_row_sum<S>([&](int k, int i, float& A, float& B) { A = v[k][i]; B = v[k][i]; },
                                          next_pow2_at_least_16(N), part, red);
    const float var = qdiv<IEEE>(ss, (float)N);
    const float rstd = qdiv<IEEE>(1.0f, sqrt_approx(var + eps));
    float amax = 0.f;
#pragma unroll
    for (int k = 0; k < S; ++k) {
        const int64_t c16 = (int64_t)threadIdx.x * S + k;   // the reference's layout: S consecutive groups per thread
        if (c16 < segs) {
            float wv[16];
            load_float16(w, w_dtype, c16 * 16, wv);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                v[k][i] = (v[k][i] * rstd) * wv[i];
                amax = fmaxf(amax, fabsf(v[k][i]));
            }
            store_bf16x16(y + row * N + c16 * 16, v[k]);
        }
    }
    amax = block_max(amax, red);
    if (threadIdx.x == 0) {
        const float fmax = fp8_fmt_out == COAT_E4M3 ? 448.0f : 57344.0f;
        s_y[row] = __float2bfloat16_rn(qdiv<IEEE>(amax + kScaleMinThres, fmax));
        rstd_out[row] = rstd;
        if (amax_bits) atomicMax(amax_bits, __float_as_uint(amax));
    }
}

// Backward: dx per row, and per-CTA partial sums of dW over the rows the CTA walks (rows cta, cta+P, ...),
// accumulated in fp32 registers and written to partial[cta][N]; a second kernel sums the partials in
// order.  No locks, no atomics: the result is deterministic (the reference serialises its partial sums
// behind a spin lock in arrival order, func_rmsnorm.py:186-196).
// Rows of up to 4096 elements: three CTAs per SM (80 registers, a few spilled words) measured 63 us against 102 us
// with two (8192 x 4096): the kernel lives on rows in flight.  The host side sizes n_partials to match.
template <int FMT, int S>
__global__ void __launch_bounds__(kNormThreads, S == 1 ? 3 : 1)
rmsnorm_bwd_kernel(const uint8_t* __restrict__ x, const void* __restrict__ s_x, int in_scale_dtype,
                   const void* __restrict__ dy, const void* __restrict__ dy2, const void* __restrict__ dy3,
                   int dy_dtype, const void* __restrict__ w, int w_dtype,
                   const float* __restrict__ rstd_in, __nv_bfloat16* __restrict__ dx, float* __restrict__ partial_dw,
                   int64_t M, int64_t N, int QB) {
    __shared__ float red[kNormThreads / 32];
    const int64_t segs = N >> 4;
    float acc[S][16];
    float wv[S][16];
#pragma unroll
    for (int k = 0; k < S; ++k) {
        const int64_t c16 = threadIdx.x + (int64_t)k * kNormThreads;
#pragma unroll
        for (int i = 0; i < 16; ++i) { acc[k][i] = 0.f; wv[k][i] = 0.f; }
        if (c16 < segs) load_float16(w, w_dtype, c16 * 16, wv[k]);
    }
    for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
        prefetch_row<S>(x, dy, dy_dtype, row + gridDim.x, M, N, segs);
        if (dy2) prefetch_row<S>(nullptr, dy2, dy_dtype, row + gridDim.x, M, N, segs);
        if (dy3) prefetch_row<S>(nullptr, dy3, dy_dtype, row + gridDim.x, M, N, segs);
        const float rstd = rstd_in[row];
        float xhat[S][16], wdy[S][16];
        float dot = 0.f;
#pragma unroll
        for (int k = 0; k < S; ++k) {
            const int64_t c16 = threadIdx.x + (int64_t)k * kNormThreads;
            if (c16 < segs) {
                float g[16];
                load_dequant16<FMT>(x, s_x, in_scale_dtype, row * segs + c16, 31 - __clz(QB >> 4), xhat[k]);
                load_float16(dy, dy_dtype, row * N + c16 * 16, g);
                // optional further addends of the upstream gradient (the dgrads of the projections that read the
                // norm's output), added left to right with a rounding to bf16 after each sum, as torch's bf16
                // `a + b + c` gives it: saves the separate add kernels and their round trips through memory
                if (dy2) {
                    float t[16];
                    load_float16(dy2, dy_dtype, row * N + c16 * 16, t);
#pragma unroll
                    for (int i = 0; i < 16; ++i) g[i] = __bfloat162float(__float2bfloat16_rn(g[i] + t[i]));
                    if (dy3) {
                        load_float16(dy3, dy_dtype, row * N + c16 * 16, t);
#pragma unroll
                        for (int i = 0; i < 16; ++i) g[i] = __bfloat162float(__float2bfloat16_rn(g[i] + t[i]));
                    }
                }
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    xhat[k][i] *= rstd;
                    wdy[k][i] = wv[k][i] * g[i];
                    dot += xhat[k][i] * wdy[k][i];
                    acc[k][i] += g[i] * xhat[k][i];
                }
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) { xhat[k][i] = 0.f; wdy[k][i] = 0.f; }
            }
        }
        const float c1 = block_sum(dot, red) / (float)N;
#pragma unroll
        for (int k = 0; k < S; ++k) {
            const int64_t c16 = threadIdx.x + (int64_t)k * kNormThreads;
            if (c16 < segs) {
                float o[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) o[i] = (wdy[k][i] - xhat[k][i] * c1) * rstd;
                store_bf16x16(dx + row * N + c16 * 16, o);
            }
        }
    }
#pragma unroll
    for (int k = 0; k < S; ++k) {
        const int64_t c16 = threadIdx.x + (int64_t)k * kNormThreads;
        if (c16 < segs) {
            float4* dst = reinterpret_cast<float4*>(partial_dw + (int64_t)blockIdx.x * N + c16 * 16);
#pragma unroll
            for (int i = 0; i < 4; ++i)
                dst[i] = make_float4(acc[k][4 * i], acc[k][4 * i + 1], acc[k][4 * i + 2], acc[k][4 * i + 3]);
        }
    }
}

// Column sums of `n_partials` rows of `stride` floats each (row p starts at partial + p * stride), in a fixed
// order: a CTA owns 32 columns, its 8 warps take the rows p = warp, warp + 8, ... four loads at a time, and the
// 8 warp sums are added in order.  (One thread per column with all rows in sequence left only N / 256 CTAs
// walking 300 strided loads each: a third of the backward pass's time.)
__device__ __forceinline__ float column_sum_32x8(const float* __restrict__ partial, int n_partials, int64_t stride,
                                                 int64_t col, bool live, float (*smem)[32]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
    if (live) {
        int p = warp;
        for (; p + 24 < n_partials; p += 32) {
            s0 += partial[(int64_t)p * stride + col];
            s1 += partial[(int64_t)(p + 8) * stride + col];
            s2 += partial[(int64_t)(p + 16) * stride + col];
            s3 += partial[(int64_t)(p + 24) * stride + col];
        }
        for (; p < n_partials; p += 8) s0 += partial[(int64_t)p * stride + col];
    }
    __syncthreads();
    smem[warp][lane] = (s0 + s1) + (s2 + s3);
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += smem[w][lane];
    return s;
}
__device__ __forceinline__ void store_typed(void* dst, int dtype, int64_t i, float v) {
    if (dtype == COAT_F32) reinterpret_cast<float*>(dst)[i] = v;
    else if (dtype == COAT_BF16) reinterpret_cast<__nv_bfloat16*>(dst)[i] = __float2bfloat16_rn(v);
    else reinterpret_cast<__half*>(dst)[i] = __float2half_rn(v);
}

__global__ void __launch_bounds__(256)
rmsnorm_dw_reduce_kernel(const float* __restrict__ partial_dw, int n_partials, void* __restrict__ dw, int w_dtype,
                         int64_t N) {
    __shared__ float smem[8][32];
    const int64_t col = (int64_t)blockIdx.x * 32 + (threadIdx.x & 31);
    const float s = column_sum_32x8(partial_dw, n_partials, N, col, col < N, smem);
    if (col < N && threadIdx.x < 32) store_typed(dw, w_dtype, col, s);
}

// =================================================================================================
// LayerNorm on a 1xQB-quantised input, with or without weight and bias (func_layernorm_noparam.py:54-186,
// func_layernorm_param.py:54-230; used by the OLMo blocks)
// =================================================================================================
// Same row layout and fixed-order reductions as the RMSNorm kernels above.  As in the reference, the mean is
// taken first and the variance is the mean of squared deviations from it (two sums over registers, not
// E[x^2] - mean^2), the normalised row leaves in FP32 (the per-tensor division that follows reads fp32), and the
// per-row scale is stored in bf16.
template <int FMT, int S, bool IEEE, bool AFFINE>
__global__ void __launch_bounds__(kNormThreads)
layernorm_fwd_kernel(const uint8_t* __restrict__ x, const void* __restrict__ s_x, int in_scale_dtype,
                     const void* __restrict__ w, const void* __restrict__ b, int wb_dtype, float* __restrict__ y,
                     __nv_bfloat16* __restrict__ s_y, float* __restrict__ mean_out, float* __restrict__ rstd_out,
                     unsigned int* __restrict__ amax_bits, int64_t M, int64_t N, int QB, float eps, int fp8_fmt_out) {
    __shared__ float red[kNormThreads / 32];
    __shared__ float part[2 * kNormThreads];
    const int64_t row = blockIdx.x;
    const int64_t segs = N >> 4;
    const int n2 = next_pow2_at_least_16(N);
    // raw codes as floats and the segment's scale: the reference's compiled kernel never rounds code * scale on
    // its own in this operator, every use is contracted into a multiply-add (func_layernorm_noparam.py:86-96)
    float c[S][16], sc[S];
#pragma unroll
    for (int k = 0; k < S; ++k) {
        const int64_t c16 = (int64_t)threadIdx.x * S + k;   // the reference's layout: S consecutive groups per thread
        sc[k] = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) c[k][i] = 0.f;
        if (c16 < segs) {
            const int64_t seg = row * segs + c16;
            const uint4 wq = *reinterpret_cast<const uint4*>(x + seg * 16);
            sc[k] = load_scale(s_x, seg >> (31 - __clz(QB >> 4)), in_scale_dtype);
            const uint32_t ww[4] = {wq.x, wq.y, wq.z, wq.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float f4[4];
                coat_fp8x4_to_float4<FMT>(ww[i], f4);
#pragma unroll
                for (int j = 0; j < 4; ++j) c[k][4 * i + j] = f4[j];
            }
        }
    }
    const float sum = ref_order_row_sum<S>([&](int k, int i, float& A, float& B) { A = c[k][i]; B = sc[k]; }, n2, part, red);
    const float mean = qdiv<IEEE>(sum, (float)N);
    // deviations x - mean = fma(code, scale, -mean).  As in the reference the zero padding up to the next power of
    // two is NOT masked out of the variance (each padded element adds mean^2, func_layernorm_noparam.py:92-94):
    // rows whose length is a power of two, the only ones the OLMo models have, are unaffected.
#pragma unroll
    for (int k = 0; k < S; ++k)
#pragma unroll
        for (int i = 0; i < 16; ++i) c[k][i] = __fmaf_rn(c[k][i], sc[k], -mean);
    const float ss = ref_order_row_sum<S>([&](int k, int i, float& A, float& B) { A = c[k][i]; B = c[k][i]; }, n2, part, red);
    const float var = qdiv<IEEE>(ss, (float)N);
    const float rstd = qdiv<IEEE>(1.0f, sqrt_approx(var + eps));
    float amax = 0.f;
#pragma unroll
    for (int k = 0; k < S; ++k) {
        const int64_t c16 = (int64_t)threadIdx.x * S + k;   // the reference's layout: S consecutive groups per thread
        if (c16 < segs) {
            float wv[16], bv[16];
            if (AFFINE) {
                load_float16(w, wb_dtype, c16 * 16, wv);
                load_float16(b, wb_dtype, c16 * 16, bv);
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                c[k][i] = __fmul_rn(c[k][i], rstd);
                if (AFFINE) c[k][i] = __fmaf_rn(c[k][i], wv[i], bv[i]);
                amax = fmaxf(amax, fabsf(c[k][i]));
            }
            float4* dst = reinterpret_cast<float4*>(y + row * N + c16 * 16);
#pragma unroll
            for (int i = 0; i < 4; ++i)
                dst[i] = make_float4(c[k][4 * i], c[k][4 * i + 1], c[k][4 * i + 2], c[k][4 * i + 3]);
        }
    }
    amax = block_max(amax, red);
    if (threadIdx.x == 0) {
        const float fmax = fp8_fmt_out == COAT_E4M3 ? 448.0f : 57344.0f;
        s_y[row] = __float2bfloat16_rn(qdiv<IEEE>(amax + kScaleMinThres, fmax));
        mean_out[row] = mean;
        rstd_out[row] = rstd;
        if (amax_bits) atomicMax(amax_bits, __float_as_uint(amax));
    }
}

// Backward: dx = (w*dy - (xhat * mean(xhat * w*dy) + mean(w*dy))) * rstd per row; with AFFINE also the per-CTA
// partial sums of dW = sum dy * xhat and dB = sum dy, written to partial[cta][2][N] and summed in order by
// rmsnorm_dw_reduce_kernel (deterministic; the reference serialises its partial sums behind a spin lock).
template <int FMT, int S, bool AFFINE>
__global__ void __launch_bounds__(kNormThreads)
layernorm_bwd_kernel(const uint8_t* __restrict__ x, const void* __restrict__ s_x, int in_scale_dtype,
                     const void* __restrict__ dy, int dy_dtype, const void* __restrict__ w, int w_dtype,
                     const float* __restrict__ mean_in, const float* __restrict__ rstd_in,
                     __nv_bfloat16* __restrict__ dx, float* __restrict__ partial, int64_t M, int64_t N, int QB) {
    __shared__ float red[kNormThreads / 32];
    const int64_t segs = N >> 4;
    float acc_w[AFFINE ? S : 1][16], acc_b[AFFINE ? S : 1][16], wv[AFFINE ? S : 1][16];
    if (AFFINE) {
#pragma unroll
        for (int k = 0; k < S; ++k) {
            const int64_t c16 = threadIdx.x + (int64_t)k * kNormThreads;
#pragma unroll
            for (int i = 0; i < 16; ++i) { acc_w[k][i] = 0.f; acc_b[k][i] = 0.f; wv[k][i] = 0.f; }
            if (c16 < segs) load_float16(w, w_dtype, c16 * 16, wv[k]);
        }
    }
    for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
        prefetch_row<S>(x, dy, dy_dtype, row + gridDim.x, M, N, segs);
        const float mean = mean_in[row], rstd = rstd_in[row];
        float xhat[S][16], wdy[S][16];
        float dot = 0.f, tot = 0.f;
#pragma unroll
        for (int k = 0; k < S; ++k) {
            const int64_t c16 = threadIdx.x + (int64_t)k * kNormThreads;
            if (c16 < segs) {
                load_dequant16<FMT>(x, s_x, in_scale_dtype, row * segs + c16, 31 - __clz(QB >> 4), xhat[k]);
                load_float16(dy, dy_dtype, row * N + c16 * 16, wdy[k]);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    xhat[k][i] = (xhat[k][i] - mean) * rstd;
                    if (AFFINE) {
                        acc_w[k][i] += wdy[k][i] * xhat[k][i];
                        acc_b[k][i] += wdy[k][i];
                        wdy[k][i] *= wv[k][i];
                    }
                    dot += xhat[k][i] * wdy[k][i];
                    tot += wdy[k][i];
                }
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) { xhat[k][i] = 0.f; wdy[k][i] = 0.f; }
            }
        }
        const float c1 = block_sum(dot, red) / (float)N;
        const float c2 = block_sum(tot, red) / (float)N;
#pragma unroll
        for (int k = 0; k < S; ++k) {
            const int64_t c16 = threadIdx.x + (int64_t)k * kNormThreads;
            if (c16 < segs) {
                float o[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) o[i] = (wdy[k][i] - (xhat[k][i] * c1 + c2)) * rstd;
                store_bf16x16(dx + row * N + c16 * 16, o);
            }
        }
    }
    if (AFFINE) {
#pragma unroll
        for (int k = 0; k < S; ++k) {
            const int64_t c16 = threadIdx.x + (int64_t)k * kNormThreads;
            if (c16 < segs) {
                float4* dw = reinterpret_cast<float4*>(partial + ((int64_t)blockIdx.x * 2) * N + c16 * 16);
                float4* db = reinterpret_cast<float4*>(partial + ((int64_t)blockIdx.x * 2 + 1) * N + c16 * 16);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    dw[i] = make_float4(acc_w[k][4 * i], acc_w[k][4 * i + 1], acc_w[k][4 * i + 2], acc_w[k][4 * i + 3]);
                    db[i] = make_float4(acc_b[k][4 * i], acc_b[k][4 * i + 1], acc_b[k][4 * i + 2], acc_b[k][4 * i + 3]);
                }
            }
        }
    }
}

// sums partial[p][which][col] over p (the two-row layout of layernorm_bwd_kernel)
__global__ void __launch_bounds__(256)
layernorm_dwdb_reduce_kernel(const float* __restrict__ partial, int n_partials, void* __restrict__ dw,
                             void* __restrict__ db, int w_dtype, int64_t N) {
    __shared__ float smem[8][32];
    const int64_t col = (int64_t)blockIdx.x * 32 + (threadIdx.x & 31);
    const float sw = column_sum_32x8(partial, n_partials, 2 * N, col, col < N, smem);
    const float sb = column_sum_32x8(partial + N, n_partials, 2 * N, col, col < N, smem);
    if (col < N && threadIdx.x < 32) {
        store_typed(dw, w_dtype, col, sw);
        store_typed(db, w_dtype, col, sb);
    }
}

// =================================================================================================
// host side
// =================================================================================================
bool fmt_ok(int f) { return f == COAT_E4M3 || f == COAT_E5M2; }
bool fdt_ok(int d) { return d == COAT_F32 || d == COAT_BF16 || d == COAT_F16; }
float fmt_max(int f) { return f == COAT_E4M3 ? 448.0f : 57344.0f; }

int check_shape(int64_t M, int64_t N, int QB) {
    if (M < 0 || N < 0) return COAT_E_BADARG;
    if (!(QB == 16 || QB == 32 || QB == 64 || QB == 128) || N % QB != 0) return COAT_E_SHAPE;
    return COAT_OK;
}

template <int OP>
int launch_fused(const FusedArgs& a, int fmt_in, int fmt_out, int flags, cudaStream_t st) {
    if (a.amax_bits && cudaMemsetAsync(a.amax_bits, 0, sizeof(unsigned int), st) != cudaSuccess) return COAT_E_LAUNCH;
    if (a.M == 0 || a.N == 0) return COAT_OK;
    const unsigned grid = straight_grid(a.M * (a.N / 16));
    const bool ieee = flags & COAT_QUANT_IEEE_DIV;
#define COAT_LAUNCH(FI, FO)                                                                                 \
    do {                                                                                                    \
        if (ieee) fused_elementwise_kernel<OP, FI, FO, true><<<grid, kStraightThreads, 0, st>>>(a);         \
        else fused_elementwise_kernel<OP, FI, FO, false><<<grid, kStraightThreads, 0, st>>>(a);             \
        return coat_launch_status();                                                                        \
    } while (0)
    // only the kernels that write FP8 codes depend on the output format at compile time
    const bool writes_codes = OP == OP_SILU_FWD || OP == OP_ADD;
    if (fmt_in == COAT_E4M3) {
        if (writes_codes && fmt_out == COAT_E5M2) COAT_LAUNCH(COAT_E4M3, COAT_E5M2);
        COAT_LAUNCH(COAT_E4M3, COAT_E4M3);
    } else {
        if (writes_codes && fmt_out == COAT_E4M3) COAT_LAUNCH(COAT_E5M2, COAT_E4M3);
        COAT_LAUNCH(COAT_E5M2, COAT_E5M2);
    }
#undef COAT_LAUNCH
}

FusedArgs base_args(int64_t M, int64_t N, int QB, int in_scale_dtype, int out_scale_dtype, int fmt_for_scales) {
    FusedArgs a = {};
    a.M = M; a.N = N; a.QB = QB;
    a.in_scale_dtype = in_scale_dtype; a.out_scale_dtype = out_scale_dtype;
    a.g_dtype = COAT_BF16; a.h_dtype = COAT_BF16;
    a.fp8_max = fmt_max(fmt_for_scales);
    return a;
}

}  // namespace

extern "C" int coat_fp8_silu_forward(const uint8_t* x, const void* s_x, uint8_t* y, void* s_y, int64_t M, int64_t N,
                                     int QB, int fmt, int scale_dtype, int flags, void* stream) {
    if (int rc = check_shape(M, N, QB)) return rc;
    if (M && N && (!x || !s_x || !y || !s_y)) return COAT_E_BADARG;
    if (!fmt_ok(fmt) || !fdt_ok(scale_dtype)) return COAT_E_BADARG;
    FusedArgs a = base_args(M, N, QB, scale_dtype, scale_dtype, fmt);
    a.x1 = x; a.s1 = s_x; a.y_q = y; a.s_y = s_y;
    return launch_fused<OP_SILU_FWD>(a, fmt, fmt, flags, (cudaStream_t)stream);
}

extern "C" int coat_fp8_act_backward(int gelu, const uint8_t* x, const void* s_x, const void* g, void* y_bf16,
                                     void* s_y, unsigned int* amax_bits, int64_t M, int64_t N, int QB, int fmt_in,
                                     int in_scale_dtype, int g_dtype, int fmt_out, int flags, void* stream) {
    if (int rc = check_shape(M, N, QB)) return rc;
    if (M && N && (!x || !s_x || !g || !y_bf16)) return COAT_E_BADARG;
    if (!fmt_ok(fmt_in) || !fmt_ok(fmt_out) || !fdt_ok(in_scale_dtype) || !fdt_ok(g_dtype)) return COAT_E_BADARG;
    FusedArgs a = base_args(M, N, QB, in_scale_dtype, COAT_BF16, fmt_out);
    a.x1 = x; a.s1 = s_x; a.g = g; a.g_dtype = g_dtype;
    a.y_bf16 = reinterpret_cast<__nv_bfloat16*>(y_bf16); a.s_y = s_y; a.amax_bits = amax_bits;
    return gelu ? launch_fused<OP_GELU_BWD>(a, fmt_in, fmt_out, flags, (cudaStream_t)stream)
                : launch_fused<OP_SILU_BWD>(a, fmt_in, fmt_out, flags, (cudaStream_t)stream);
}

extern "C" int coat_fp8_gelu_forward(const uint8_t* x, const void* s_x, void* y_bf16, void* s_y,
                                     unsigned int* amax_bits, int64_t M, int64_t N, int QB, int fmt, int scale_dtype,
                                     int flags, void* stream) {
    if (int rc = check_shape(M, N, QB)) return rc;
    if (M && N && (!x || !s_x || !y_bf16)) return COAT_E_BADARG;
    if (!fmt_ok(fmt) || !fdt_ok(scale_dtype)) return COAT_E_BADARG;
    FusedArgs a = base_args(M, N, QB, scale_dtype, scale_dtype, fmt);
    a.x1 = x; a.s1 = s_x; a.y_bf16 = reinterpret_cast<__nv_bfloat16*>(y_bf16); a.s_y = s_y; a.amax_bits = amax_bits;
    return launch_fused<OP_GELU_FWD>(a, fmt, fmt, flags, (cudaStream_t)stream);
}

extern "C" int coat_fp8_mul_forward(const uint8_t* x1, const void* s_x1, const uint8_t* x2, const void* s_x2,
                                    void* y_bf16, void* s_y, unsigned int* amax_bits, int64_t M, int64_t N, int QB,
                                    int fmt, int scale_dtype, int flags, void* stream) {
    if (int rc = check_shape(M, N, QB)) return rc;
    if (M && N && (!x1 || !s_x1 || !x2 || !s_x2 || !y_bf16)) return COAT_E_BADARG;
    if (!fmt_ok(fmt) || !fdt_ok(scale_dtype)) return COAT_E_BADARG;
    FusedArgs a = base_args(M, N, QB, scale_dtype, scale_dtype, fmt);
    a.x1 = x1; a.s1 = s_x1; a.x2 = x2; a.s2 = s_x2;
    a.y_bf16 = reinterpret_cast<__nv_bfloat16*>(y_bf16); a.s_y = s_y; a.amax_bits = amax_bits;
    return launch_fused<OP_MUL_FWD>(a, fmt, fmt, flags, (cudaStream_t)stream);
}

extern "C" int coat_fp8_mul_backward(const uint8_t* x1, const void* s_x1, const uint8_t* x2, const void* s_x2,
                                     const void* g, void* y1_bf16, void* y2_bf16, void* s_y2, unsigned int* amax_bits,
                                     int64_t M, int64_t N, int QB, int fmt_in, int in_scale_dtype, int g_dtype,
                                     int fmt_out, int flags, void* stream) {
    if (int rc = check_shape(M, N, QB)) return rc;
    if (M && N && (!x1 || !s_x1 || !x2 || !s_x2 || !g || !y1_bf16 || !y2_bf16)) return COAT_E_BADARG;
    if (!fmt_ok(fmt_in) || !fmt_ok(fmt_out) || !fdt_ok(in_scale_dtype) || !fdt_ok(g_dtype)) return COAT_E_BADARG;
    FusedArgs a = base_args(M, N, QB, in_scale_dtype, COAT_BF16, fmt_out);
    a.x1 = x1; a.s1 = s_x1; a.x2 = x2; a.s2 = s_x2; a.g = g; a.g_dtype = g_dtype;
    a.y1_bf16 = reinterpret_cast<__nv_bfloat16*>(y1_bf16); a.y_bf16 = reinterpret_cast<__nv_bfloat16*>(y2_bf16);
    a.s_y = s_y2; a.amax_bits = amax_bits;
    return launch_fused<OP_MUL_BWD>(a, fmt_in, fmt_out, flags, (cudaStream_t)stream);
}

extern "C" int coat_fp8_silu_mul_forward(const uint8_t* x_gate, const void* s_gate, const uint8_t* x_up, const void* s_up,
                                         uint8_t* q_silu, void* s_silu, void* y_bf16, void* s_y, unsigned int* amax_bits,
                                         int64_t M, int64_t N, int QB, int fmt, int scale_dtype, int flags,
                                         void* stream) {
    if (int rc = check_shape(M, N, QB)) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    if (!amax_bits) return COAT_E_BADARG;
    if (cudaMemsetAsync(amax_bits, 0, sizeof(unsigned int), st) != cudaSuccess) return COAT_E_LAUNCH;
    if (M == 0 || N == 0) return COAT_OK;
    if (!x_gate || !s_gate || !x_up || !s_up || !q_silu || !s_silu || !y_bf16) return COAT_E_BADARG;
    if (!fmt_ok(fmt) || !fdt_ok(scale_dtype)) return COAT_E_BADARG;
    SiluMulFwdArgs a = {x_gate, s_gate, x_up, s_up, q_silu, s_silu, reinterpret_cast<__nv_bfloat16*>(y_bf16), s_y,
                        amax_bits, M, N, QB, scale_dtype, fmt_max(fmt)};
    const unsigned grid = straight_grid(M * (N / 16));
    const bool ieee = flags & COAT_QUANT_IEEE_DIV;
    if (fmt == COAT_E4M3) {
        if (ieee) silu_mul_forward_kernel<COAT_E4M3, true><<<grid, kStraightThreads, 0, st>>>(a);
        else silu_mul_forward_kernel<COAT_E4M3, false><<<grid, kStraightThreads, 0, st>>>(a);
    } else {
        if (ieee) silu_mul_forward_kernel<COAT_E5M2, true><<<grid, kStraightThreads, 0, st>>>(a);
        else silu_mul_forward_kernel<COAT_E5M2, false><<<grid, kStraightThreads, 0, st>>>(a);
    }
    return coat_launch_status();
}

extern "C" int coat_fp8_mul_silu_backward(const uint8_t* x_silu, const void* s_silu, const uint8_t* x_up, const void* s_up,
                                          const uint8_t* x_gate, const void* s_gate, const void* g, void* y_up_bf16,
                                          void* s_y_up, unsigned int* amax_up, void* y_gate_bf16, void* s_y_gate,
                                          unsigned int* amax_gate, int64_t M, int64_t N, int QB, int fmt_in,
                                          int in_scale_dtype, int g_dtype, int fmt_out, int flags, void* stream) {
    if (int rc = check_shape(M, N, QB)) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    if (!amax_up || !amax_gate) return COAT_E_BADARG;
    if (cudaMemsetAsync(amax_up, 0, sizeof(unsigned int), st) != cudaSuccess ||
        cudaMemsetAsync(amax_gate, 0, sizeof(unsigned int), st) != cudaSuccess) return COAT_E_LAUNCH;
    if (M == 0 || N == 0) return COAT_OK;
    if (!x_silu || !s_silu || !x_up || !s_up || !x_gate || !s_gate || !g || !y_up_bf16 || !s_y_up || !y_gate_bf16 ||
        !s_y_gate) return COAT_E_BADARG;
    if (!fmt_ok(fmt_in) || !fmt_ok(fmt_out) || !fdt_ok(in_scale_dtype) || !fdt_ok(g_dtype)) return COAT_E_BADARG;
    MulSiluBwdArgs a = {x_silu, s_silu, x_up, s_up, x_gate, s_gate, g, g_dtype,
                        reinterpret_cast<__nv_bfloat16*>(y_up_bf16), s_y_up, amax_up,
                        reinterpret_cast<__nv_bfloat16*>(y_gate_bf16), s_y_gate, amax_gate, M, N, QB, in_scale_dtype,
                        fmt_max(fmt_out)};
    const unsigned grid = straight_grid(M * (N / 16));
    const bool ieee = flags & COAT_QUANT_IEEE_DIV;
    if (fmt_in == COAT_E4M3) {
        if (ieee) mul_silu_backward_kernel<COAT_E4M3, true><<<grid, kStraightThreads, 0, st>>>(a);
        else mul_silu_backward_kernel<COAT_E4M3, false><<<grid, kStraightThreads, 0, st>>>(a);
    } else {
        if (ieee) mul_silu_backward_kernel<COAT_E5M2, true><<<grid, kStraightThreads, 0, st>>>(a);
        else mul_silu_backward_kernel<COAT_E5M2, false><<<grid, kStraightThreads, 0, st>>>(a);
    }
    return coat_launch_status();
}

extern "C" int coat_fp8_add(const void* x1, const void* x2, void* y_bf16, uint8_t* y_q, void* s_y,
                            unsigned int* amax_bits, int64_t M, int64_t N, int QB, int x1_dtype, int x2_dtype,
                            int fmt_out, int flags, void* stream) {
    if (int rc = check_shape(M, N, QB)) return rc;
    if (M && N && (!x1 || !x2 || !y_bf16 || !s_y)) return COAT_E_BADARG;
    if (!fmt_ok(fmt_out) || !fdt_ok(x1_dtype) || !fdt_ok(x2_dtype)) return COAT_E_BADARG;
    FusedArgs a = base_args(M, N, QB, COAT_BF16, COAT_BF16, fmt_out);
    a.g = x1; a.h = x2; a.g_dtype = x1_dtype; a.h_dtype = x2_dtype;
    a.y_bf16 = reinterpret_cast<__nv_bfloat16*>(y_bf16); a.y_q = y_q; a.s_y = s_y; a.amax_bits = amax_bits;
    return launch_fused<OP_ADD>(a, fmt_out, fmt_out, flags, (cudaStream_t)stream);
}

extern "C" int coat_fp8_rmsnorm_forward(const uint8_t* x, const void* s_x, const void* w, void* y_bf16,
                                        void* s_y_rows_bf16, float* rstd, unsigned int* amax_bits, int64_t M,
                                        int64_t N, int QB, float eps, int fmt, int in_scale_dtype, int w_dtype,
                                        int flags, void* stream) {
    if (int rc = check_shape(M, N, QB)) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    if (amax_bits && cudaMemsetAsync(amax_bits, 0, sizeof(unsigned int), st) != cudaSuccess) return COAT_E_LAUNCH;
    if (M == 0 || N == 0) return COAT_OK;
    if (!x || !s_x || !w || !y_bf16 || !s_y_rows_bf16 || !rstd) return COAT_E_BADARG;
    if (!fmt_ok(fmt) || !fdt_ok(in_scale_dtype) || !fdt_ok(w_dtype)) return COAT_E_BADARG;
    if (N > 16384) return COAT_E_TOOBIG;
    const int S = N <= 4096 ? 1 : (N <= 8192 ? 2 : 4);
    const bool ieee = flags & COAT_QUANT_IEEE_DIV;
    __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(y_bf16);
    __nv_bfloat16* sy = reinterpret_cast<__nv_bfloat16*>(s_y_rows_bf16);
#define COAT_RMS(F, SS)                                                                                          \
    do {                                                                                                         \
        if (ieee) rmsnorm_fwd_kernel<F, SS, true><<<(unsigned)M, kNormThreads, 0, st>>>(                          \
            x, s_x, in_scale_dtype, w, w_dtype, y, sy, rstd, amax_bits, M, N, QB, eps, fmt);                     \
        else rmsnorm_fwd_kernel<F, SS, false><<<(unsigned)M, kNormThreads, 0, st>>>(                              \
            x, s_x, in_scale_dtype, w, w_dtype, y, sy, rstd, amax_bits, M, N, QB, eps, fmt);                     \
    } while (0)
    if (fmt == COAT_E4M3) { if (S == 1) COAT_RMS(COAT_E4M3, 1); else if (S == 2) COAT_RMS(COAT_E4M3, 2); else COAT_RMS(COAT_E4M3, 4); }
    else { if (S == 1) COAT_RMS(COAT_E5M2, 1); else if (S == 2) COAT_RMS(COAT_E5M2, 2); else COAT_RMS(COAT_E5M2, 4); }
#undef COAT_RMS
    return coat_launch_status();
}

extern "C" int coat_fp8_rmsnorm_backward(const uint8_t* x, const void* s_x, const void* dy, const void* dy2,
                                         const void* dy3, const void* w, const float* rstd, void* dx_bf16,
                                         float* partial_dw, int n_partials,
                                         void* dw, int64_t M, int64_t N, int QB, int fmt, int in_scale_dtype,
                                         int dy_dtype, int w_dtype, void* stream) {
    if (int rc = check_shape(M, N, QB)) return rc;
    if (M == 0 || N == 0) return COAT_OK;
    if (!x || !s_x || !dy || !w || !rstd || !dx_bf16 || !partial_dw || !dw || n_partials < 1) return COAT_E_BADARG;
    if (dy3 && !dy2) return COAT_E_BADARG;
    if ((dy2 || dy3) && dy_dtype != COAT_BF16) return COAT_E_BADARG;   // the sums are rounded to bf16
    if (!fmt_ok(fmt) || !fdt_ok(in_scale_dtype) || !fdt_ok(dy_dtype) || !fdt_ok(w_dtype)) return COAT_E_BADARG;
    if (N > 16384) return COAT_E_TOOBIG;
    cudaStream_t st = (cudaStream_t)stream;
    const int S = N <= 4096 ? 1 : (N <= 8192 ? 2 : 4);
    const unsigned grid = (unsigned)(n_partials < M ? n_partials : M);
    __nv_bfloat16* dx = reinterpret_cast<__nv_bfloat16*>(dx_bf16);
#define COAT_RMSB(F, SS) rmsnorm_bwd_kernel<F, SS><<<grid, kNormThreads, 0, st>>>(x, s_x, in_scale_dtype, dy, dy2, dy3, dy_dtype, w, w_dtype, rstd, dx, partial_dw, M, N, QB)
    if (fmt == COAT_E4M3) { if (S == 1) COAT_RMSB(COAT_E4M3, 1); else if (S == 2) COAT_RMSB(COAT_E4M3, 2); else COAT_RMSB(COAT_E4M3, 4); }
    else { if (S == 1) COAT_RMSB(COAT_E5M2, 1); else if (S == 2) COAT_RMSB(COAT_E5M2, 2); else COAT_RMSB(COAT_E5M2, 4); }
#undef COAT_RMSB
    rmsnorm_dw_reduce_kernel<<<(unsigned)((N + 31) / 32), 256, 0, st>>>(partial_dw, (int)grid, dw, w_dtype, N);
    return coat_launch_status();
}

extern "C" int coat_fp8_layernorm_forward(const uint8_t* x, const void* s_x, const void* w, const void* b, float* y_f32,
                                          void* s_y_rows_bf16, float* mean, float* rstd, unsigned int* amax_bits,
                                          int64_t M, int64_t N, int QB, float eps, int fmt, int in_scale_dtype,
                                          int wb_dtype, int flags, void* stream) {
    if (int rc = check_shape(M, N, QB)) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    if (amax_bits && cudaMemsetAsync(amax_bits, 0, sizeof(unsigned int), st) != cudaSuccess) return COAT_E_LAUNCH;
    if (M == 0 || N == 0) return COAT_OK;
    if (!x || !s_x || !y_f32 || !s_y_rows_bf16 || !mean || !rstd || ((w == nullptr) != (b == nullptr))) return COAT_E_BADARG;
    if (!fmt_ok(fmt) || !fdt_ok(in_scale_dtype) || (w && !fdt_ok(wb_dtype))) return COAT_E_BADARG;
    if (N > 16384) return COAT_E_TOOBIG;
    const int S = N <= 4096 ? 1 : (N <= 8192 ? 2 : 4);
    const bool ieee = flags & COAT_QUANT_IEEE_DIV;
    __nv_bfloat16* sy = reinterpret_cast<__nv_bfloat16*>(s_y_rows_bf16);
#define COAT_LN3(F, SS, I, A) layernorm_fwd_kernel<F, SS, I, A><<<(unsigned)M, kNormThreads, 0, st>>>( \
        x, s_x, in_scale_dtype, w, b, wb_dtype, y_f32, sy, mean, rstd, amax_bits, M, N, QB, eps, fmt)
#define COAT_LN2(F, SS) do { if (ieee) { if (w) COAT_LN3(F, SS, true, true); else COAT_LN3(F, SS, true, false); } \
                             else { if (w) COAT_LN3(F, SS, false, true); else COAT_LN3(F, SS, false, false); } } while (0)
    if (fmt == COAT_E4M3) { if (S == 1) COAT_LN2(COAT_E4M3, 1); else if (S == 2) COAT_LN2(COAT_E4M3, 2); else COAT_LN2(COAT_E4M3, 4); }
    else { if (S == 1) COAT_LN2(COAT_E5M2, 1); else if (S == 2) COAT_LN2(COAT_E5M2, 2); else COAT_LN2(COAT_E5M2, 4); }
#undef COAT_LN2
#undef COAT_LN3
    return coat_launch_status();
}

extern "C" int coat_fp8_layernorm_backward(const uint8_t* x, const void* s_x, const void* dy, const void* w,
                                           const float* mean, const float* rstd, void* dx_bf16, float* partial,
                                           int n_partials, void* dw, void* db, int64_t M, int64_t N, int QB, int fmt,
                                           int in_scale_dtype, int dy_dtype, int w_dtype, void* stream) {
    if (int rc = check_shape(M, N, QB)) return rc;
    if (M == 0 || N == 0) return COAT_OK;
    if (!x || !s_x || !dy || !mean || !rstd || !dx_bf16) return COAT_E_BADARG;
    if (w && (!partial || !dw || !db || n_partials < 1 || !fdt_ok(w_dtype))) return COAT_E_BADARG;
    if (!fmt_ok(fmt) || !fdt_ok(in_scale_dtype) || !fdt_ok(dy_dtype)) return COAT_E_BADARG;
    // with weight and bias a thread also carries the dW / dB partial sums of its columns: rows up to 8192
    if (N > (w ? 8192 : 16384)) return COAT_E_TOOBIG;
    cudaStream_t st = (cudaStream_t)stream;
    const int S = N <= 4096 ? 1 : (N <= 8192 ? 2 : 4);
    const int64_t want = w ? (int64_t)n_partials : (int64_t)4 * coat_sm_count();
    const unsigned grid = (unsigned)(want < M ? want : M);
    __nv_bfloat16* dx = reinterpret_cast<__nv_bfloat16*>(dx_bf16);
#define COAT_LNB3(F, SS, A) layernorm_bwd_kernel<F, SS, A><<<grid, kNormThreads, 0, st>>>( \
        x, s_x, in_scale_dtype, dy, dy_dtype, w, w_dtype, mean, rstd, dx, partial, M, N, QB)
#define COAT_LNB2(F, SS) do { if (w) COAT_LNB3(F, SS, true); else COAT_LNB3(F, SS, false); } while (0)
    if (fmt == COAT_E4M3) { if (S == 1) COAT_LNB2(COAT_E4M3, 1); else if (S == 2) COAT_LNB2(COAT_E4M3, 2); else COAT_LNB3(COAT_E4M3, 4, false); }
    else { if (S == 1) COAT_LNB2(COAT_E5M2, 1); else if (S == 2) COAT_LNB2(COAT_E5M2, 2); else COAT_LNB3(COAT_E5M2, 4, false); }
#undef COAT_LNB2
#undef COAT_LNB3
    if (w) layernorm_dwdb_reduce_kernel<<<(unsigned)((N + 31) / 32), 256, 0, st>>>(partial, (int)grid, dw, db, w_dtype, N);
    return coat_launch_status();
}
