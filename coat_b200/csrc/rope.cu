// Rotary position embedding on bf16 q / k of shape [B, S, H, D] (the layout the projections produce), fused
// into one pass:  y = x * cos + rotate_half(x) * sin,  rotate_half(x) = cat(-x[D/2:], x[:D/2]).
// The decoder layer's attention block (coat/models/coat_llama.py:1031-1036 through transformers'
// apply_rotary_pos_emb) does this with seven eager elementwise kernels per tensor and direction; it is not part
// of the quantization path but shows up as a fifth of the layer's time once the GEMMs are FP8.
// cos / sin are [Bc, S, D] with Bc = 1 or B (the position_embeddings the layer receives), bf16 (Llama) or fp32
// (OLMo's full-precision RoPE, examples/OLMo/olmo/model.py:254-320 of the reference's vendored trainer).  The input may
// have any strides over (b, s, h) as long as a head is contiguous (the gradient arrives as a transposed view);
// the output is contiguous [B, S, H, D].  The backward
// pass is the same kernel with the transposed rotation: dx = dy * cos + rotate_half^T(dy * sin).
// Arithmetic in fp32 with one rounding to bf16 (the eager form rounds after every operation).
#include "common.cuh"

namespace {

__device__ __forceinline__ void unpack8(const uint4& w, float (&f)[8]) {
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = __uint_as_float(u[i] << 16);
        f[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
    }
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
    uint32_t u[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
        u[i] = (uint32_t)coat_float_to_bf16_bits(f[2 * i]) | ((uint32_t)coat_float_to_bf16_bits(f[2 * i + 1]) << 16);
    return make_uint4(u[0], u[1], u[2], u[3]);
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&f)[8]) {
    unpack8(*reinterpret_cast<const uint4*>(p), f);
}
__device__ __forceinline__ void load8(const float* p, float (&f)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

// one thread per 8 elements of the first half of a head and the matching 8 of the second half
template <bool BACKWARD, typename TT>
__global__ void __launch_bounds__(256)
rope_kernel(const __nv_bfloat16* __restrict__ x, const TT* __restrict__ cos_t,
            const TT* __restrict__ sin_t, __nv_bfloat16* __restrict__ y, int64_t rows /* B*S*H */,
            int S, int H, int D, int64_t cos_batch_stride, int64_t sxb, int64_t sxs, int64_t sxh) {
    const int per_row = D >> 4;                     // threads per head row
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t row = idx / per_row;
    if (row >= rows) return;
    const int d = (int)(idx - row * per_row) * 8;
    const int64_t bs = row / H;                     // b * S + s
    const int64_t b = bs / S, s = bs - b * S;
    const int64_t h = row - bs * H;
    const int64_t xi = b * sxb + s * sxs + h * sxh + d;   // input: any strides with the head dimension contiguous
    const int64_t xo = row * D + d, co = b * cos_batch_stride + s * D + d;
    const int half = D >> 1;
    float x1[8], x2[8], c1[8], c2[8], s1[8], s2[8], o1[8], o2[8];
    unpack8(*reinterpret_cast<const uint4*>(x + xi), x1);
    unpack8(*reinterpret_cast<const uint4*>(x + xi + half), x2);
    load8(cos_t + co, c1);
    load8(cos_t + co + half, c2);
    load8(sin_t + co, s1);
    load8(sin_t + co + half, s2);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        if (!BACKWARD) {   // y1 = x1 c1 - x2 s1,  y2 = x2 c2 + x1 s2
            o1[i] = __fmaf_rn(x1[i], c1[i], -x2[i] * s1[i]);
            o2[i] = __fmaf_rn(x2[i], c2[i], x1[i] * s2[i]);
        } else {           // dx1 = dy1 c1 + dy2 s2,  dx2 = dy2 c2 - dy1 s1
            o1[i] = __fmaf_rn(x1[i], c1[i], x2[i] * s2[i]);
            o2[i] = __fmaf_rn(x2[i], c2[i], -x1[i] * s1[i]);
        }
    }
    *reinterpret_cast<uint4*>(y + xo) = pack8(o1);
    *reinterpret_cast<uint4*>(y + xo + half) = pack8(o2);
}

template <typename TT>
int launch_rope(const void* x, int64_t sxb, int64_t sxs, int64_t sxh, const void* cos_t, const void* sin_t, void* y,
                int64_t B, int64_t S, int64_t H, int64_t D, int64_t cos_batch_stride, int backward, void* stream) {
    if (B < 0 || S < 0 || H < 0 || D < 0) return COAT_E_BADARG;
    if (B == 0 || S == 0 || H == 0) return COAT_OK;
    if (!x || !cos_t || !sin_t || !y) return COAT_E_BADARG;
    if (D % 16 != 0 || D == 0) return COAT_E_SHAPE;
    if (sxb % 8 != 0 || sxs % 8 != 0 || sxh % 8 != 0) return COAT_E_ALIGN;   // 16-byte loads of the input
    if (S > 0x7fffffff || H > 0x7fffffff || D > 0x7fffffff) return COAT_E_TOOBIG;
    if (!coat_aligned(x, 16) || !coat_aligned(y, 16) || !coat_aligned(cos_t, 16) || !coat_aligned(sin_t, 16))
        return COAT_E_ALIGN;
    if (cos_batch_stride % 8 != 0) return COAT_E_ALIGN;
    const int64_t rows = B * S * H, threads = rows * (D / 16);
    const int64_t blocks = (threads + 255) / 256;
    if (blocks > 0x7fffffff) return COAT_E_TOOBIG;
    cudaStream_t st = (cudaStream_t)stream;
    const auto* xp = reinterpret_cast<const __nv_bfloat16*>(x);
    const auto* cp = reinterpret_cast<const TT*>(cos_t);
    const auto* sp = reinterpret_cast<const TT*>(sin_t);
    auto* yp = reinterpret_cast<__nv_bfloat16*>(y);
    if (backward)
        rope_kernel<true, TT><<<(unsigned)blocks, 256, 0, st>>>(xp, cp, sp, yp, rows, (int)S, (int)H, (int)D,
                                                               cos_batch_stride, sxb, sxs, sxh);
    else
        rope_kernel<false, TT><<<(unsigned)blocks, 256, 0, st>>>(xp, cp, sp, yp, rows, (int)S, (int)H, (int)D,
                                                                cos_batch_stride, sxb, sxs, sxh);
    return coat_launch_status();
}

}  // namespace

extern "C" int coat_rope_bf16(const void* x, int64_t sxb, int64_t sxs, int64_t sxh, const void* cos_t,
                              const void* sin_t, void* y, int64_t B, int64_t S, int64_t H, int64_t D,
                              int64_t cos_batch_stride, int backward, void* stream) {
    return launch_rope<__nv_bfloat16>(x, sxb, sxs, sxh, cos_t, sin_t, y, B, S, H, D, cos_batch_stride, backward, stream);
}

// The same with fp32 cos / sin tables.
extern "C" int coat_rope_bf16_f32tables(const void* x, int64_t sxb, int64_t sxs, int64_t sxh, const void* cos_t,
                                        const void* sin_t, void* y, int64_t B, int64_t S, int64_t H, int64_t D,
                                        int64_t cos_batch_stride, int backward, void* stream) {
    return launch_rope<float>(x, sxb, sxs, sxh, cos_t, sin_t, y, B, S, H, D, cos_batch_stride, backward, stream);
}
