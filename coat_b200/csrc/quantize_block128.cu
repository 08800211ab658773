// Quantizers with 128-wide granularity, the formats of the DeepSeek-style block-scaled linear layer:
//   block scales  : one scale per 128 x 128 block        (_quantize_perblock.py:33-112, the weights)
//   row groups    : one scale per 1 x 128 row segment    (_quantize_transpose.py with QB = 128 and the "per group"
//                   half of _quantize_perblock_transpose_pergroup.py:145-180, the activations / gradients)
//   column groups : one scale per 128 x 1 column segment (the transposed output of _quantize_transpose.py, QB = 128)
// and the transposed copies of the block- and column-scaled codes (_quantize_perblock_transpose.py:33-124).
// One kernel writes any subset of the four outputs from one read of the input.
//
// One CTA of 512 threads per 128 x 128 tile (which is exactly one block, one row group per row and one column
// group per column); thread = 4 rows x 8 columns, lane = 8*mb + nb as in the 1x16 transposing kernel.  Row
// maxima are reduced over the 8 lanes of a row (xor 1, 2, 4) and the two warps that share the rows (through
// shared memory), column maxima over the 4 lanes of a column (xor 8, 16) and the 8 warp rows (through shared
// memory), the block maximum from the row maxima.  Transposed codes cross shared memory once, rotated by
// 4 words per 8 columns, and leave in 16-byte pieces.
#include "quant_common.cuh"

namespace {

constexpr int kB = 128;
constexpr int kBThreads = 512;

struct Block128Args {
    const void* x;
    uint8_t* y_b; void* s_b;      // block-scaled codes [M,N], scales [M/128, N/128]
    uint8_t* y_bt; void* s_bt;    // block-scaled codes transposed [N,M], scales [N/128, M/128]
    uint8_t* y_r; void* s_r;      // row-group codes [M,N], scales [M, N/128]
    uint8_t* y_ct; void* s_ct;    // column-group codes transposed [N,M], scales [N, M/128]
    int scale_dtype;
    int64_t M, N, ldx;
};

template <typename T, int FMT, bool IEEE>
__global__ void __launch_bounds__(kBThreads)
block128_quant_kernel(Block128Args a) {
    __shared__ __align__(16) uint32_t tile_t[kB][32];   // transposed codes: [column][4-row word, rotated]
    __shared__ float row_part[kB][2];                   // per row: maxima of the two 64-column halves
    __shared__ float col_part[8][kB];                   // per column: maxima of the eight 16-row bands
    __shared__ float row_max[kB], col_max[kB];
    __shared__ float block_max_s;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = lane & 7, mb = lane >> 3;
    const int m_loc = (warp >> 1) * 16 + mb * 4, n_loc = (warp & 1) * 64 + nb * 8;
    const int64_t m_tile = (int64_t)blockIdx.y * kB, n_tile = (int64_t)blockIdx.x * kB;
    const int64_t m0 = m_tile + m_loc, n0 = n_tile + n_loc;
    const T* x = reinterpret_cast<const T*>(a.x);
    const bool want_rows = a.y_r != nullptr, want_cols = a.y_ct != nullptr;
    const bool want_block = a.y_b != nullptr || a.y_bt != nullptr;

    float v[4][8];
#pragma unroll
    for (int j = 0; j < 4; ++j) load8(x + (m0 + j) * a.ldx + n0, v[j]);

    // ---- maxima -----------------------------------------------------------------------------------
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float r = fmaxf(fmaxf(fmaxf(fabsf(v[j][0]), fabsf(v[j][1])), fmaxf(fabsf(v[j][2]), fabsf(v[j][3]))),
                        fmaxf(fmaxf(fabsf(v[j][4]), fabsf(v[j][5])), fmaxf(fabsf(v[j][6]), fabsf(v[j][7]))));
        r = fmaxf(r, __shfl_xor_sync(COAT_FULL_MASK, r, 1));
        r = fmaxf(r, __shfl_xor_sync(COAT_FULL_MASK, r, 2));
        r = fmaxf(r, __shfl_xor_sync(COAT_FULL_MASK, r, 4));
        if (nb == 0) row_part[m_loc + j][warp & 1] = r;
    }
    if (want_cols) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float c = fmaxf(fmaxf(fabsf(v[0][i]), fabsf(v[1][i])), fmaxf(fabsf(v[2][i]), fabsf(v[3][i])));
            c = fmaxf(c, __shfl_xor_sync(COAT_FULL_MASK, c, 8));
            c = fmaxf(c, __shfl_xor_sync(COAT_FULL_MASK, c, 16));
            if (mb == 0) col_part[warp >> 1][n_loc + i] = c;
        }
    }
    __syncthreads();
    if (threadIdx.x < kB) {
        const int r = threadIdx.x;
        row_max[r] = fmaxf(row_part[r][0], row_part[r][1]);
        if (want_cols) {
            float c = col_part[0][r];
#pragma unroll
            for (int b = 1; b < 8; ++b) c = fmaxf(c, col_part[b][r]);
            col_max[r] = c;
        }
    }
    __syncthreads();
    if (want_block && warp == 0) {
        float m = fmaxf(fmaxf(row_max[lane], row_max[lane + 32]), fmaxf(row_max[lane + 64], row_max[lane + 96]));
        m = coat_warp_max(m);
        if (lane == 0) block_max_s = m;
    }
    __syncthreads();

    // ---- scales and codes -------------------------------------------------------------------------
    const GroupScale<FMT, IEEE> group_scale;
    const int word = ((m_loc >> 2) + 4 * (n_loc >> 3)) & 31;
    const int64_t sn = a.N / kB, sm = a.M / kB;
    if (want_rows) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float s = group_scale(row_max[m_loc + j]);
            const GroupScaleDivider<IEEE> d(s);
            uint2 w;
            w.x = coat_float4_to_fp8x4<FMT>(d(v[j][0]), d(v[j][1]), d(v[j][2]), d(v[j][3]));
            w.y = coat_float4_to_fp8x4<FMT>(d(v[j][4]), d(v[j][5]), d(v[j][6]), d(v[j][7]));
            *reinterpret_cast<uint2*>(a.y_r + (m0 + j) * a.N + n0) = w;
            if (nb == 0 && (warp & 1) == 0) store_scale(a.s_r, (m0 + j) * sn + blockIdx.x, a.scale_dtype, s);
        }
    }
    if (want_block) {
        const float s = group_scale(block_max_s);
        const GroupScaleDivider<IEEE> d(s);
        if (a.y_b) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint2 w;
                w.x = coat_float4_to_fp8x4<FMT>(d(v[j][0]), d(v[j][1]), d(v[j][2]), d(v[j][3]));
                w.y = coat_float4_to_fp8x4<FMT>(d(v[j][4]), d(v[j][5]), d(v[j][6]), d(v[j][7]));
                *reinterpret_cast<uint2*>(a.y_b + (m0 + j) * a.N + n0) = w;
            }
            if (threadIdx.x == 0) store_scale(a.s_b, (int64_t)blockIdx.y * sn + blockIdx.x, a.scale_dtype, s);
        }
        if (a.y_bt) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
                tile_t[n_loc + i][word] = coat_float4_to_fp8x4<FMT>(d(v[0][i]), d(v[1][i]), d(v[2][i]), d(v[3][i]));
            if (threadIdx.x == 0) store_scale(a.s_bt, (int64_t)blockIdx.x * sm + blockIdx.y, a.scale_dtype, s);
            __syncthreads();
#pragma unroll
            for (int it = 0; it < kB * 8 / kBThreads; ++it) {
                const int idx = it * kBThreads + threadIdx.x;
                const int r = idx >> 3, c = idx & 7;
                *reinterpret_cast<uint4*>(a.y_bt + (n_tile + r) * a.M + m_tile + c * 16) =
                    *reinterpret_cast<const uint4*>(&tile_t[r][(4 * c + 4 * (r >> 3)) & 31]);
            }
            __syncthreads();   // the tile is reused by the column-group output below
        }
    }
    if (want_cols) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float s = group_scale(col_max[n_loc + i]);
            const GroupScaleDivider<IEEE> d(s);
            tile_t[n_loc + i][word] = coat_float4_to_fp8x4<FMT>(d(v[0][i]), d(v[1][i]), d(v[2][i]), d(v[3][i]));
        }
        if (threadIdx.x < kB)
            store_scale(a.s_ct, (n_tile + threadIdx.x) * sm + blockIdx.y, a.scale_dtype, group_scale(col_max[threadIdx.x]));
        __syncthreads();
#pragma unroll
        for (int it = 0; it < kB * 8 / kBThreads; ++it) {
            const int idx = it * kBThreads + threadIdx.x;
            const int r = idx >> 3, c = idx & 7;
            *reinterpret_cast<uint4*>(a.y_ct + (n_tile + r) * a.M + m_tile + c * 16) =
                *reinterpret_cast<const uint4*>(&tile_t[r][(4 * c + 4 * (r >> 3)) & 31]);
        }
    }
}

template <typename T>
int launch_block128(const Block128Args& a, int fmt, bool ieee, cudaStream_t st) {
    const dim3 grid((unsigned)(a.N / kB), (unsigned)(a.M / kB));
#define COAT_B128(FMT)                                                                      \
    do {                                                                                    \
        if (ieee) block128_quant_kernel<T, FMT, true><<<grid, kBThreads, 0, st>>>(a);       \
        else block128_quant_kernel<T, FMT, false><<<grid, kBThreads, 0, st>>>(a);           \
        return coat_launch_status();                                                        \
    } while (0)
    if (fmt == COAT_E4M3) COAT_B128(COAT_E4M3);
    if (fmt == COAT_E5M2) COAT_B128(COAT_E5M2);
#undef COAT_B128
    return COAT_E_BADARG;
}

}  // namespace

extern "C" int coat_fp8_quantize_block128(const void* x, int64_t M, int64_t N, int64_t ldx, uint8_t* y_b, void* s_b,
                                          uint8_t* y_bt, void* s_bt, uint8_t* y_r, void* s_r, uint8_t* y_ct,
                                          void* s_ct, int fmt, int in_dtype, int scale_dtype, int flags, void* stream) {
    if (M < 0 || N < 0 || ldx < N) return COAT_E_BADARG;
    if (M == 0 || N == 0) return COAT_OK;
    if (!x || (!y_b && !y_bt && !y_r && !y_ct)) return COAT_E_BADARG;
    if ((y_b && !s_b) || (y_bt && !s_bt) || (y_r && !s_r) || (y_ct && !s_ct)) return COAT_E_BADARG;
    if (scale_dtype != COAT_F32 && scale_dtype != COAT_BF16 && scale_dtype != COAT_F16) return COAT_E_BADARG;
    if (M % kB != 0 || N % kB != 0) return COAT_E_SHAPE;
    if (M / kB > 65535) return COAT_E_TOOBIG;   // grid.y
    const int esz = in_dtype == COAT_F32 ? 4 : 2;
    if (!coat_aligned(x, 16) || (ldx * esz) % 16 != 0) return COAT_E_ALIGN;
    if ((y_b && !coat_aligned(y_b, 16)) || (y_bt && !coat_aligned(y_bt, 16)) || (y_r && !coat_aligned(y_r, 16)) ||
        (y_ct && !coat_aligned(y_ct, 16)))
        return COAT_E_ALIGN;
    Block128Args a = {x, y_b, s_b, y_bt, s_bt, y_r, s_r, y_ct, s_ct, scale_dtype, M, N, ldx};
    const bool ieee = flags & COAT_QUANT_IEEE_DIV;
    cudaStream_t st = (cudaStream_t)stream;
    switch (in_dtype) {
        case COAT_BF16: return launch_block128<__nv_bfloat16>(a, fmt, ieee, st);
        case COAT_F16: return launch_block128<__half>(a, fmt, ieee, st);
        case COAT_F32: return launch_block128<float>(a, fmt, ieee, st);
        default: return COAT_E_BADARG;
    }
}
