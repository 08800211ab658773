// FP8 GEMM for sm_100a on the 5th-generation tensor cores: C = (A * B^T) * (s_a * s_b) [+ bias], with A [M,K]
// and B [N,K] both K-major FP8 (E4M3 or E5M2, chosen per operand), fp32 accumulation in tensor memory, and a
// bf16 result or a fused 1xQB FP8 quantisation of the result with bf16 group scales.
//
// It replaces the reference's Triton kernel _fp8matmul_kernel (coat/activation/real_quantization/linear.py:61-169)
// behind fp8matmul / fp8_linear_forward / fp8_linear_backward (:172-302).  The reference always hands that kernel
// a `.t()` view of a contiguous matrix as B (linear.py:257, :285-286), which is why both operands are K-major
// here for forward (X, W), dgrad (G, W^T) and wgrad (G^T, X^T) alike.
//
// Structure (persistent CTAs of 192 threads, one per SM, each walking 128 x 256 output tiles):
//   warp 0, one lane   TMA producer: cp.async.bulk.tensor (no multicast) of a 128x128 B A-tile and a 256x128 B B-tile
//                      per pipeline stage into 128-byte-swizzled shared memory, completion on the stage's mbarrier
//   warp 1             allocates all 512 columns of tensor memory (two accumulators, so the epilogue of one tile
//                      overlaps the main loop of the next); one lane issues tcgen05.mma.kind::f8f6f4
//                      (M=128, N=256, K=32 per instruction, 4 per stage) and commits each stage back to the producer
//   warps 2-5          epilogue: tcgen05.ld of the accumulator (lane quarter = warp index mod 4, 32 columns at a
//                      time, so one thread holds 32 consecutive columns of one row), scaling, bias, bf16 or 1xQB FP8
//                      conversion and 64-byte row-segment stores
// Every wait on an mbarrier is bounded; a wait that runs out sets a device status word, and the CTA still goes
// through its tear-down (tensor memory is released) before it returns.

#include <cuda.h>
#include <cstdlib>

#include "common.cuh"

namespace {

constexpr int kBN = 256, kBK = 128;                   // CTA tile columns; kBK bytes of K per stage (= one 128B swizzle row)
// Two tile heights.  BM = 256 (two M=128 MMAs per K step that share the B stage) halves the B traffic per flop:
// 262 flop per byte pulled from L2 instead of 170, which matters because at 2.3 PFLOP/s the 128-row tile
// draws ~13 TB/s through L2.  It uses all 512 TMEM columns for one tile, so its epilogue is not overlapped
// with the next tile's main loop; BM = 128 keeps two accumulators and overlaps them.
template <int BM> struct GemmShape {
    static constexpr int kStages = BM == 128 ? 4 : 3;
    static constexpr int kHalves = BM / 128;                 // M=128 MMAs per K step
    static constexpr int kBufs = BM == 128 ? 2 : 1;          // accumulator sets in TMEM
    static constexpr int kEpiWarps = 4 * kHalves;
    static constexpr int kThreads = 64 + 32 * kEpiWarps;
    static constexpr uint32_t kStageBytesA = BM * kBK, kStageBytesB = kBN * kBK;
    static constexpr uint32_t kStageBytes = kStageBytesA + kStageBytesB;
    // per epilogue warp: 32 rows x 128 bytes of bf16 output (64 columns), staged for a TMA store
    static constexpr uint32_t kStagingBytes = 4096 * kEpiWarps;
    static constexpr size_t kSmem = (size_t)kStages * kStageBytes + kStagingBytes + 1024 /*alignment slack*/ + 256 /*barriers*/;
};
constexpr int kMaxStages = 4;
constexpr int kUmmaK = 32;                            // K per tcgen05.mma for 8-bit operands
constexpr int kTmemCols = 512;                        // two 128 x 256 fp32 accumulators
constexpr int kWaitLimit = 1 << 20;

__device__ int g_gemm_device_status = 0;

__device__ __forceinline__ uint32_t s2u(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(s2u(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(s2u(bar)), "r"(bytes) : "memory");
}
// bounded wait for the phase with the given parity; false = gave up
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile uint32_t* abort_flag) {
    for (int i = 0; i < kWaitLimit; ++i) {
        if ((i & 63) == 63 && *abort_flag) return false;   // another role of this CTA has given up
        uint32_t done;
        asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                     : "=r"(done) : "r"(s2u(bar)), "r"(parity) : "memory");
        if (done) return true;
    }
    return false;
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
                 ::"r"(s2u(dst)), "l"(map), "r"(s2u(bar)), "r"(x), "r"(y) : "memory");
}
// 2-D tensor store shared -> global (clipped at the tensor's edges), tracked by the issuing thread's bulk group
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                 ::"l"(map), "r"(s2u(src)), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 64-bit shared-memory matrix descriptor: K-major operand, 128-byte swizzle, rows 128 B apart, 8-row groups
// 1024 B apart (stride byte offset), descriptor version 1 (Blackwell)
__device__ __forceinline__ uint64_t make_smem_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr & 0x3ffff) >> 4);          // start address, bits [0,14)
    d |= (uint64_t)1 << 16;                               // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;                     // stride byte offset, bits [32,46)
    d |= (uint64_t)1 << 46;                               // version
    d |= (uint64_t)2 << 61;                               // layout type: SWIZZLE_128B
    return d;
}
// 32-bit instruction descriptor for kind::f8f6f4: fp32 accumulator, per-operand FP8 format, both operands K-major
__host__ __device__ constexpr uint32_t make_idesc(int fmt_a, int fmt_b, int m, int n) {
    return (1u << 4) | ((uint32_t)fmt_a << 7) | ((uint32_t)fmt_b << 10) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void umma_f8(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc, uint32_t accumulate) {
    asm volatile("{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p; }"
                 ::"r"(tmem_d), "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate) : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(s2u(bar)) : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 64 consecutive accumulator columns of this thread's row in one instruction (halves the exposed load latency of
// the promotion loop of the block-scaled kernel, which waits for every load before it can use it)
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&r)[64]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, "
        "%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, "
        "%48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]),
          "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]),
          "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]),
          "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]),
          "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// The sequence of work items of one CTA.  A unit is a 128-row x 256-column block of C; tiles are numbered down
// the rows first, and CTA b takes tiles b, b + gridDim, ... so that the tiles in flight at any time are
// neighbours that share operand tiles in L2 (handing each CTA a contiguous range instead was measured 5-10 %
// slower).  BM = 128: a tile is one unit.  BM = 256: a tile is two vertically adjacent units (one at an odd
// matrix edge); when the last, partial round has at most gridDim / 2 tiles, they are split into their units
// so that the round costs half a tile.
// When the operands do not fit L2 together, tiles are numbered in bands of kGroupM tile rows: down the rows of a band
// first, then along its columns, band after band.  The tiles in flight (one per SM) then cover a few tile rows of A
// and most tile columns of B: B stays in L2 from band to band and A crosses DRAM once, where numbering down whole
// columns makes every round of tiles pull all of A again (the reference's kernel walks its tiles in GROUP_M = 8
// order for the same reason, coat/activation/real_quantization/linear.py:94-102).  Measured on the Llama-2-7B MLP
// shapes (burst TFLOP/s): dgrad 2655 -> 2777, wgrad 2589 -> 2751 with bands of 8 (4 and 16 within 1 %); the forward
// GEMM, whose operands (78 MB) stay in L2 anyway, lost 3 % with bands and keeps the column order.
#ifndef COAT_GEMM_GROUP_M
#define COAT_GEMM_GROUP_M 8
#endif
constexpr int kGroupM = COAT_GEMM_GROUP_M;
// tile number -> (tile row, tile column) in that order; band_rows = 0: down whole columns
__device__ __forceinline__ void banded_tile(int t, int tiles_m, int tiles_n, int band_rows, int& tile_m, int& tile_n) {
    if (band_rows > 0) {
        const int per_band = band_rows * tiles_n;
        const int band = t / per_band, r = t - band * per_band;
        const int rows = tiles_m - band * band_rows < band_rows ? tiles_m - band * band_rows : band_rows;
        tile_n = r / rows;
        tile_m = band * band_rows + (r - tile_n * rows);
    } else {
        tile_m = t % tiles_m;
        tile_n = t / tiles_m;
    }
}
template <int BM>
struct TileWalk {
    int k, rounds, rest, units_m, tiles_m, units_n, band_rows;
    __device__ TileWalk(int units_m_, int units_n_, int band_rows_) : k(0), units_m(units_m_), units_n(units_n_), band_rows(band_rows_) {
        tiles_m = BM == 128 ? units_m_ : (units_m_ + 1) / 2;
        const int total = tiles_m * units_n;
        rounds = total / (int)gridDim.x;
        rest = total - rounds * (int)gridDim.x;
    }
    __device__ void decode(int t, int& unit_m, int& unit_n, int& halves) const {
        int tm;
        banded_tile(t, tiles_m, units_n, band_rows, tm, unit_n);
        unit_m = BM == 128 ? tm : 2 * tm;
        halves = BM == 128 ? 1 : (units_m - unit_m >= 2 ? 2 : 1);
    }
    // false when the CTA is done; else the item's first block row, its block column and its height in units
    __device__ bool next(int& unit_m, int& unit_n, int& halves) {
        const int b = blockIdx.x, P = gridDim.x;
        if (k < rounds) {
            decode(b + k * P, unit_m, unit_n, halves);
            ++k;
            return true;
        }
        if (k > rounds || rest == 0) return false;
        ++k;
        if (BM == 256 && 2 * rest <= P) {   // split the last tiles into their units
            if (b >= 2 * rest) return false;
            decode(rounds * P + (b >> 1), unit_m, unit_n, halves);
            if ((b & 1) >= halves) return false;
            unit_m += b & 1;
            halves = 1;
            return true;
        }
        if (b >= rest) return false;
        decode(rounds * P + b, unit_m, unit_n, halves);
        return true;
    }
};

struct GemmEpilogue {
    void* c;                 // bf16 [M,N] or FP8 codes [M,N]
    void* scale_c;           // bf16 [M, N/QB] when quantising
    const void* scale_a;     // device scalars
    const void* scale_b;
    const void* bias;        // [N] or null
    int scale_dtype, bias_dtype;
    int tma_store;           // bf16 result leaves through shared memory and TMA stores (map_c is valid)
    int quantize;            // 0: bf16 result, 1: 1xQB FP8 + scales
    int QB;
    int fmt_c;
    int ieee_div;
    int M, N, K;
    int band_rows;           // tile order: 0 = down whole columns, else bands of this many tile rows (banded_tile)
};

__device__ __forceinline__ float ld_scalar(const void* p, int dtype, int64_t i = 0) {
    if (dtype == COAT_F32) return reinterpret_cast<const float*>(p)[i];
    if (dtype == COAT_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    return __half2float(reinterpret_cast<const __half*>(p)[i]);
}

// 32 consecutive columns of one row -> FP8 codes and 32 / QBV group scales.  A lane owns its row, so its stores
// never coalesce with its neighbours': the 32 codes leave as two 16-byte stores and the scales as one store
// (4-byte stores of the codes, eight per lane, made the quantising GEMM a third slower than the bf16 one).
template <int FMT_C, int QBV>
__device__ __forceinline__ void quantize_groups(const GemmEpilogue& e, int row, int col0, const float (&v)[32]) {
    const float fmax = CoatFp8Max<FMT_C>::value;
    uint8_t* dst = reinterpret_cast<uint8_t*>(e.c) + (int64_t)row * e.N + col0;
    __nv_bfloat16* sdst = reinterpret_cast<__nv_bfloat16*>(e.scale_c) + (int64_t)row * (e.N / QBV) + col0 / QBV;
    uint32_t words[8];
    uint16_t sbits[32 / QBV];
    const bool whole = col0 + 32 <= e.N;
#pragma unroll
    for (int gi = 0; gi < 32 / QBV; ++gi) {
        float m[QBV / 2];   // balanced tree: the epilogue warp has nobody to hide a 16-deep chain behind
#pragma unroll
        for (int i = 0; i < QBV / 2; ++i) m[i] = fmaxf(fabsf(v[gi * QBV + 2 * i]), fabsf(v[gi * QBV + 2 * i + 1]));
#pragma unroll
        for (int wdt = QBV / 4; wdt >= 1; wdt >>= 1)
#pragma unroll
            for (int i = 0; i < wdt; ++i) m[i] = fmaxf(m[2 * i], m[2 * i + 1]);
        const float amax = m[0];
        const float num = amax + 1e-10f;
        const float scale = e.ieee_div ? __fdiv_rn(num, fmax) : coat_div_full(num, fmax);
        sbits[gi] = coat_float_to_bf16_bits(scale);
        // div.full.f32(x, s) == x * rcp.approx.f32(s) bit for bit while |s| is in [2^-120, 2^120]
        float r;
        asm("rcp.approx.f32 %0, %1;" : "=f"(r) : "f"(scale));
        const bool fast = !e.ieee_div && scale >= 7.5231638e-37f && scale <= 1.3292280e36f;
        // one branch per group, not a three-way select per element: with the select the compiler evaluated the
        // reciprocal product, div.full and the IEEE division for every element (22 instructions per element, and the
        // epilogue warps, one per scheduler and latency-bound, took longer per tile than the tensor cores)
        if (fast) {
#pragma unroll
            for (int i = 0; i < QBV; i += 4)
                words[(gi * QBV + i) >> 2] = coat_float4_to_fp8x4<FMT_C>(v[gi * QBV + i] * r, v[gi * QBV + i + 1] * r,
                                                                         v[gi * QBV + i + 2] * r, v[gi * QBV + i + 3] * r);
        } else if (e.ieee_div) {
#pragma unroll
            for (int i = 0; i < QBV; i += 4)
                words[(gi * QBV + i) >> 2] = coat_float4_to_fp8x4<FMT_C>(
                    __fdiv_rn(v[gi * QBV + i], scale), __fdiv_rn(v[gi * QBV + i + 1], scale),
                    __fdiv_rn(v[gi * QBV + i + 2], scale), __fdiv_rn(v[gi * QBV + i + 3], scale));
        } else {
#pragma unroll
            for (int i = 0; i < QBV; i += 4)
                words[(gi * QBV + i) >> 2] = coat_float4_to_fp8x4<FMT_C>(
                    coat_div_full(v[gi * QBV + i], scale), coat_div_full(v[gi * QBV + i + 1], scale),
                    coat_div_full(v[gi * QBV + i + 2], scale), coat_div_full(v[gi * QBV + i + 3], scale));
        }
    }
    if (whole && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        reinterpret_cast<uint4*>(dst)[0] = make_uint4(words[0], words[1], words[2], words[3]);
        reinterpret_cast<uint4*>(dst)[1] = make_uint4(words[4], words[5], words[6], words[7]);
    } else {
#pragma unroll
        for (int k = 0; k < 8; ++k)
            if (col0 + 4 * k < e.N) *reinterpret_cast<uint32_t*>(dst + 4 * k) = words[k];   // N is a multiple of QBV >= 16
    }
    if (QBV == 16 && whole && (reinterpret_cast<uintptr_t>(sdst) & 3) == 0) {
        *reinterpret_cast<uint32_t*>(sdst) = (uint32_t)sbits[0] | ((uint32_t)sbits[32 / QBV - 1] << 16);
    } else {
#pragma unroll
        for (int gi = 0; gi < 32 / QBV; ++gi)
            if (col0 + gi * QBV < e.N) sdst[gi] = __ushort_as_bfloat16(sbits[gi]);
    }
}

template <int FMT_C>
__device__ __forceinline__ void epilogue_store(const GemmEpilogue& e, int row, int col0, float (&v)[32]) {
    // v: 32 consecutive columns col0.. of one row, already scaled (and biased)
    if (row >= e.M || col0 >= e.N) return;
    const bool full = col0 + 32 <= e.N;
    if (!e.quantize) {
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(e.c) + (int64_t)row * e.N + col0;
        if (full && ((e.N & 7) == 0)) {
            uint32_t o[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
                o[i] = (uint32_t)coat_float_to_bf16_bits(v[2 * i]) | ((uint32_t)coat_float_to_bf16_bits(v[2 * i + 1]) << 16);
#pragma unroll
            for (int i = 0; i < 4; ++i)
                reinterpret_cast<uint4*>(dst)[i] = make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)   // static indices: a run-time index would put v[] in local memory
                if (col0 + i < e.N) dst[i] = __float2bfloat16_rn(v[i]);
        }
    } else {
        // fused 1xQB quantisation (linear.py:139-164): QB is 16 or 32, N a multiple of QB, so groups never
        // straddle the 32 columns a thread holds
        if (e.QB == 16) quantize_groups<FMT_C, 16>(e, row, col0, v);
        else quantize_groups<FMT_C, 32>(e, row, col0, v);
    }
}

// Drains one warp's 32 rows x 256 columns of an accumulator (tensor-memory address `tmem_tile` = lane quarter
// and first column) into C, rows row0 .. row0 + 31, columns tile_col0 .. tile_col0 + 255.
//   TMA path (bf16 output): rows are staged 64 columns (128 bytes) at a time in the warp's 32 x 128-byte buffer, in
//   the 128-byte swizzle the tensor map expects (16-byte unit u of row r sits at unit u ^ (r & 7): the 8 lanes of
//   a quarter-warp hit 8 different bank groups), and one lane hands the box to the TMA unit.
//   Register path (quantising epilogue, or N not a multiple of 8): each lane writes its own row.
template <int FMT_C>
__device__ __forceinline__ void drain_accumulator(const CUtensorMap* map_c, const GemmEpilogue& e, uint8_t* stg,
                                                  uint32_t tmem_tile, int tile_col0, int row0, int lane, float sab) {
    if (e.tma_store) {
#pragma unroll 1
        for (int cc = 0; cc < kBN / 64; ++cc) {
            if (lane == 0) bulk_wait_read();   // the previous store has read the buffer
            __syncwarp();
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                uint32_t r[32];
                tmem_ld32(tmem_tile + (uint32_t)(cc * 64 + hh * 32), r);
                const int col0 = tile_col0 + cc * 64 + hh * 32;
                uint32_t o[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    float a = __uint_as_float(r[2 * i]) * sab, b = __uint_as_float(r[2 * i + 1]) * sab;
                    if (e.bias) {
                        if (col0 + 2 * i < e.N) a += ld_scalar(e.bias, e.bias_dtype, col0 + 2 * i);
                        if (col0 + 2 * i + 1 < e.N) b += ld_scalar(e.bias, e.bias_dtype, col0 + 2 * i + 1);
                    }
                    o[i] = (uint32_t)coat_float_to_bf16_bits(a) | ((uint32_t)coat_float_to_bf16_bits(b) << 16);
                }
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    *reinterpret_cast<uint4*>(stg + lane * 128 + (((hh * 4 + j) ^ (lane & 7)) << 4)) =
                        make_uint4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
            }
            fence_async_smem();   // this lane's staged words become visible to the TMA unit
            __syncwarp();
            if (lane == 0 && row0 < e.M && tile_col0 + cc * 64 < e.N) {
                tma_store_2d(map_c, stg, tile_col0 + cc * 64, row0);
                bulk_commit();
            }
        }
    } else {
#pragma unroll 1
        for (int c = 0; c < kBN / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(tmem_tile + (uint32_t)(c * 32), r);
            float v[32];
            const int col0 = tile_col0 + c * 32;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                v[i] = __uint_as_float(r[i]) * sab;
                if (e.bias && col0 + i < e.N) v[i] += ld_scalar(e.bias, e.bias_dtype, col0 + i);
            }
            epilogue_store<FMT_C>(e, row0 + lane, col0, v);
        }
    }
}

template <int FMT_C, int BM>
__global__ void __launch_bounds__(GemmShape<BM>::kThreads, 1)
fp8_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                const __grid_constant__ CUtensorMap map_c, uint32_t idesc, GemmEpilogue e, int tiles_m, int tiles_n) {
    extern __shared__ uint8_t smem_raw[];
    // 128-byte-swizzled TMA destinations and UMMA operands need 1024-byte alignment
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    typedef GemmShape<BM> S;
    constexpr int kStages = S::kStages, kHalves = S::kHalves, kBufs = S::kBufs;
    constexpr uint32_t kStageBytesA = S::kStageBytesA, kStageBytesB = S::kStageBytesB, kStageBytes = S::kStageBytes;
    uint8_t* smem_a = smem;
    uint8_t* smem_b = smem + (size_t)kStages * kStageBytesA;
    uint8_t* staging = smem + (size_t)kStages * kStageBytes;   // 1024-byte aligned: stages are multiples of 1024
    uint64_t* bars = reinterpret_cast<uint64_t*>(staging + S::kStagingBytes);
    uint64_t* full_bar = bars;                         // [kStages] TMA -> MMA
    uint64_t* empty_bar = bars + kMaxStages;           // [kStages] MMA -> TMA
    uint64_t* acc_full = bars + 2 * kMaxStages;        // [kBufs] accumulator complete -> epilogue
    uint64_t* acc_empty = bars + 2 * kMaxStages + 2;   // [kBufs] accumulator drained -> MMA (every epilogue warp arrives)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kMaxStages + 4);
    volatile uint32_t* abort_flag = tmem_slot + 1;  // set by whoever gives up waiting; makes every other wait bail out

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int k_blocks = (e.K + kBK - 1) / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) { mbar_init(&full_bar[s], 1); mbar_init(&empty_bar[s], 1); }
        for (int i = 0; i < 2; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], S::kEpiWarps); }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {   // whole warp: allocate both accumulators (all 512 columns)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s2u(tmem_slot)), "r"(kTmemCols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    bool ok = true;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int it = 0;
            TileWalk<BM> walk(tiles_m, tiles_n, e.band_rows);
            int unit_m, unit_n, halves;
            while (ok && walk.next(unit_m, unit_n, halves)) {
                for (int kb = 0; kb < k_blocks; ++kb, ++it) {
                    const int s = it % kStages;
                    if (it >= kStages) ok = mbar_wait(&empty_bar[s], ((it / kStages) - 1) & 1, abort_flag);
                    if (!ok) break;
                    mbar_expect_tx(&full_bar[s], (uint32_t)halves * (128 * kBK) + kStageBytesB);
                    for (int h = 0; h < halves; ++h)   // A arrives in 128-row boxes, one per unit of the item
                        tma_load_2d(smem_a + (size_t)s * kStageBytesA + (size_t)h * (128 * kBK), &map_a, kb * kBK,
                                    (unit_m + h) * 128, &full_bar[s]);
                    tma_load_2d(smem_b + (size_t)s * kStageBytesB, &map_b, kb * kBK, unit_n * kBN, &full_bar[s]);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            int it = 0, local = 0;
            TileWalk<BM> walk(tiles_m, tiles_n, e.band_rows);
            int unit_m, unit_n, halves;
            for (; ok && walk.next(unit_m, unit_n, halves); ++local) {
                const int buf = local % kBufs, use = local / kBufs;
                if (use >= 1) ok = mbar_wait(&acc_empty[buf], (use - 1) & 1, abort_flag);   // epilogue has drained it
                if (!ok) break;
                tc_fence_after();
                const uint32_t tmem_d = tmem_base + (uint32_t)(buf * kHalves * kBN);
                for (int kb = 0; kb < k_blocks; ++kb, ++it) {
                    const int s = it % kStages;
                    ok = mbar_wait(&full_bar[s], (it / kStages) & 1, abort_flag);
                    if (!ok) break;
                    tc_fence_after();
                    const uint64_t da = make_smem_desc(s2u(smem_a + (size_t)s * kStageBytesA));
                    const uint64_t db = make_smem_desc(s2u(smem_b + (size_t)s * kStageBytesB));
#pragma unroll
                    for (int k = 0; k < kBK / kUmmaK; ++k) {
                        // advancing K inside the 128-byte swizzle row: +32 bytes = +2 in the (>>4) address field;
                        // the second half of a 256-row A stage starts 128 rows x 128 bytes further on
#pragma unroll
                        for (int h = 0; h < kHalves; ++h)
                            if (h < halves) umma_f8(tmem_d + (uint32_t)(h * kBN),
                                    da + (uint64_t)(k * (kUmmaK >> 4)) + (uint64_t)(h * ((128 * kBK) >> 4)),
                                    db + (uint64_t)(k * (kUmmaK >> 4)), idesc, (kb | k) != 0);
                    }
                    umma_commit(&empty_bar[s]);      // frees the stage once these MMAs have read it
                }
                if (ok) umma_commit(&acc_full[buf]);  // this tile's accumulator is final once all of the above completed
            }
        }
    } else {
        // ---------------- epilogue (warps 2 .. 2 + 4*kHalves - 1) ----------------
        const int quarter = warp & 3;                         // TMEM lanes this warp may read
        const int half = (warp - 2) >> 2;                     // which M=128 accumulator of the tile
        const float sab = ld_scalar(e.scale_a, e.scale_dtype) * ld_scalar(e.scale_b, e.scale_dtype);
        int local = 0;
        TileWalk<BM> walk(tiles_m, tiles_n, e.band_rows);
        int unit_m, tile_n, halves;
        for (; ok && walk.next(unit_m, tile_n, halves); ++local) {
            const int buf = local % kBufs, use = local / kBufs;
            ok = __all_sync(COAT_FULL_MASK, mbar_wait(&acc_full[buf], use & 1, abort_flag));   // warp-uniform
            if (!ok) break;
            tc_fence_after();
            const int row0 = (unit_m + half) * 128 + quarter * 32;
            const uint32_t tmem_tile = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)((buf * kHalves + half) * kBN);
            if (half < halves)   // (a single unit: the warps of the second accumulator have nothing to drain)
                drain_accumulator<FMT_C>(&map_c, e, staging + (size_t)(warp - 2) * 4096, tmem_tile, tile_n * kBN, row0,
                                         lane, sab);
            // all of this warp's reads of the accumulator are complete (tcgen05.wait::ld inside tmem_ld32)
            tc_fence_before();
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(s2u(&acc_empty[buf])) : "memory");
        }
        if (lane == 0) bulk_wait_all();   // this warp's TMA stores are complete before the CTA retires
    }
    if (!ok) { *abort_flag = 1; g_gemm_device_status = COAT_E_TIMEOUT; }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols) : "memory");
    }
}

// =====================================================================================================
// CTA-pair kernel: two CTAs of a cluster (two SMs) work on one 256 x 256 tile with tcgen05.mma.cta_group::2.
// CTA r of the pair stages rows [128 r, 128 r + 128) of the A tile and of the B tile (so each SM writes and
// reads half of B: 128 B/clk of shared-memory traffic per SM instead of 192), its tensor memory holds rows
// [128 r, 128 r + 128) x 256 columns of the accumulator (two buffers), and its four epilogue warps drain and
// store them.  Only the leader (rank 0) issues MMAs.  Signalling:
//   full[s]      (leader's only) one expect_tx by the leader's producer for the bytes of BOTH CTAs; the peer's
//                loads complete on the leader's barrier too (TMA loads with .cta_group::2, no multicast)
//   empty[s]     in both CTAs, arrived by the leader's tcgen05.commit with a CTA mask of both
//   acc_full[b]  in both CTAs, same mechanism
//   acc_empty[b] (leader's only) 8 arrivals: the 4 epilogue warps of each CTA (the peer's arrive remotely)
// Every wait is bounded as in the single-CTA kernel; the pair synchronises (barrier.cluster) after set-up and
// before tensor memory is released, so that neither CTA leaves while its partner may still signal or read it.
// =====================================================================================================
constexpr int kPairStages = 6;
constexpr uint32_t kPairStageA = 128 * kBK, kPairStageB = 128 * kBK, kPairStageBytes = kPairStageA + kPairStageB;
constexpr uint32_t kPairStaging = 4 * 4096;
constexpr size_t kPairSmem = (size_t)kPairStages * kPairStageBytes + kPairStaging + 1024 + 256;
constexpr int kPairThreads = 192;

__device__ __forceinline__ uint32_t cluster_rank() { uint32_t r; asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r)); return r; }
__device__ __forceinline__ uint32_t map_to_cta(uint32_t smem_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// TMA load of a CTA of a pair: data into this CTA's shared memory, completion bytes onto `bar_cluster_addr`,
// which may be the partner's barrier
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int x, int y, uint32_t bar_cluster_addr) {
    asm volatile("cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
                 ::"r"(s2u(dst)), "l"(map), "r"(bar_cluster_addr), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ void umma_f8_pair(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc, uint32_t accumulate) {
    asm volatile("{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p; }"
                 ::"r"(tmem_d), "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate) : "memory");
}
// arrive on the barrier at this shared-memory offset in every CTA of `mask` once the MMAs issued so far are done
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar, uint16_t mask) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
                 ::"r"(s2u(bar)), "h"(mask) : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr) : "memory");
}

template <int FMT_C>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
fp8_gemm_pair_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                     const __grid_constant__ CUtensorMap map_c, uint32_t idesc, GemmEpilogue e, int tiles_m, int tiles_n) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* smem_a = smem;
    uint8_t* smem_b = smem + (size_t)kPairStages * kPairStageA;
    uint8_t* staging = smem + (size_t)kPairStages * kPairStageBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(staging + kPairStaging);
    uint64_t* full_bar = bars;                          // [kPairStages] used in the leader only
    uint64_t* empty_bar = bars + kPairStages;           // [kPairStages] both CTAs
    uint64_t* acc_full = bars + 2 * kPairStages;        // [2] both CTAs
    uint64_t* acc_empty = bars + 2 * kPairStages + 2;   // [2] used in the leader only
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kPairStages + 4);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
    const int k_blocks = (e.K + kBK - 1) / kBK;
    const int n_tiles = tiles_m * tiles_n;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPairStages; ++s) { mbar_init(&full_bar[s], 1); mbar_init(&empty_bar[s], 1); }
        for (int i = 0; i < 2; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], 8); }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {   // one warp of EACH CTA of the pair takes part in the allocation
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s2u(tmem_slot)), "r"(kTmemCols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();   // both CTAs' barriers exist before anything signals them
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    bool ok = true;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer (both CTAs) ----------------
            int it = 0;
            for (int t = pair; t < n_tiles && ok; t += n_pairs) {
                int tile_m, tile_n;
                banded_tile(t, tiles_m, tiles_n, e.band_rows, tile_m, tile_n);
                for (int kb = 0; kb < k_blocks; ++kb, ++it) {
                    const int s = it % kPairStages;
                    if (it >= kPairStages) ok = mbar_wait(&empty_bar[s], ((it / kPairStages) - 1) & 1, abort_flag);
                    if (!ok) break;
                    if (rank == 0) mbar_expect_tx(&full_bar[s], 2 * kPairStageBytes);
                    const uint32_t leader_full = map_to_cta(s2u(&full_bar[s]), 0);
                    tma_load_2d_pair(smem_a + (size_t)s * kPairStageA, &map_a, kb * kBK, tile_m * 256 + (int)rank * 128, leader_full);
                    tma_load_2d_pair(smem_b + (size_t)s * kPairStageB, &map_b, kb * kBK, tile_n * 256 + (int)rank * 128, leader_full);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            // ---------------- MMA issuer (leader only) ----------------
            int it = 0, local = 0;
            for (int t = pair; t < n_tiles && ok; t += n_pairs, ++local) {
                const int buf = local & 1, use = local >> 1;
                if (use >= 1) ok = mbar_wait(&acc_empty[buf], (use - 1) & 1, abort_flag);
                if (!ok) break;
                tc_fence_after();
                const uint32_t tmem_d = tmem_base + (uint32_t)(buf * kBN);
                for (int kb = 0; kb < k_blocks; ++kb, ++it) {
                    const int s = it % kPairStages;
                    ok = mbar_wait(&full_bar[s], (it / kPairStages) & 1, abort_flag);
                    if (!ok) break;
                    tc_fence_after();
                    const uint64_t da = make_smem_desc(s2u(smem_a + (size_t)s * kPairStageA));
                    const uint64_t db = make_smem_desc(s2u(smem_b + (size_t)s * kPairStageB));
#pragma unroll
                    for (int k = 0; k < kBK / kUmmaK; ++k)
                        umma_f8_pair(tmem_d, da + (uint64_t)(k * (kUmmaK >> 4)), db + (uint64_t)(k * (kUmmaK >> 4)), idesc,
                                     (kb | k) != 0);
                    umma_commit_pair(&empty_bar[s], 3);      // frees the stage in both CTAs
                }
                if (ok) umma_commit_pair(&acc_full[buf], 3);  // both CTAs' epilogues may drain their halves
            }
        }
    } else {
        // ---------------- epilogue (warps 2..5 of both CTAs) ----------------
        const int quarter = warp & 3;
        const float sab = ld_scalar(e.scale_a, e.scale_dtype) * ld_scalar(e.scale_b, e.scale_dtype);
        uint8_t* stg = staging + (size_t)(warp - 2) * 4096;
        int local = 0;
        for (int t = pair; t < n_tiles && ok; t += n_pairs, ++local) {
            int tile_m, tile_n;
                banded_tile(t, tiles_m, tiles_n, e.band_rows, tile_m, tile_n);
            const int buf = local & 1, use = local >> 1;
            ok = __all_sync(COAT_FULL_MASK, mbar_wait(&acc_full[buf], use & 1, abort_flag));
            if (!ok) break;
            tc_fence_after();
            const int row0 = tile_m * 256 + (int)rank * 128 + quarter * 32;
            const uint32_t tmem_tile = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(buf * kBN);
            drain_accumulator<FMT_C>(&map_c, e, stg, tmem_tile, tile_n * kBN, row0, lane, sab);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(map_to_cta(s2u(&acc_empty[buf]), 0));   // the leader's barrier
        }
        if (lane == 0) bulk_wait_all();
    }
    if (!ok) { *abort_flag = 1; g_gemm_device_status = COAT_E_TIMEOUT; }
    tc_fence_before();
    __syncthreads();
    cluster_sync();   // the partner has finished signalling this CTA and reading its shared memory
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols) : "memory");
    }
}

// =====================================================================================================
// Block-scaled GEMM (the DeepSeek-style recipe that the reference reaches through deep_gemm.gemm_fp8_fp8_bf16_nt,
// coat/activation/deepseek/linear.py:10-36):
//     C[m, n] = sum over K blocks kb of  sa[m, kb] * sb[n / 128, kb] * sum_{k in kb} A[m, k] * B[n, k]
// with one scale per 1 x 128 segment of A and per 128 x 128 block of B.  The tensor core cannot apply a
// scale per K block inside its accumulation, so every K block is multiplied into a FRESH 128 x 128 fp32
// buffer in tensor memory (four of them rotate) and eight "promotion" warps add it, times its two scales,
// into fp32 accumulators they hold in registers (one row per thread, 64 columns per warp of a lane quarter,
// fetched with ONE tcgen05.ld.x64 per K block: the load's latency is exposed once per K block, and a
// 128 x 256 tile with four x32 loads per K block measured 1.46 PFLOP/s for that reason) while the tensor
// core works on the next K blocks.  After the last K block the same warps convert to bf16 and store
// through shared memory and the TMA unit.  Register budget: 10 warps put 3 on one scheduler, so a thread
// may use 168 registers; 64 accumulators + 64 loaded values fit, 128 + 64 would spill.
//   warp 0      TMA producer: A and B stages of 128 rows x 128 bytes (5 stages)
//   warp 1      MMA issuer: 4 x (M128 N128 K32) per K block, commit -> stage empty, commit -> partial full
//   warps 2..9  promotion + epilogue; they arrive on `partial empty` when a buffer has been read
// Every wait is bounded as in the other kernels.
// =====================================================================================================
constexpr int kBsBN = 128, kBsStages = 5, kBsParts = 4, kBsEpiWarps = 8, kBsThreads = 64 + 32 * kBsEpiWarps;
constexpr uint32_t kBsStageA = 128 * kBK, kBsStageB = kBsBN * kBK, kBsStageBytes = kBsStageA + kBsStageB;
constexpr uint32_t kBsStaging = 4096 * kBsEpiWarps;   // per warp: 32 rows x 64 bf16 columns
constexpr size_t kBsSmem = (size_t)kBsStages * kBsStageBytes + kBsStaging + 1024 + 256;

struct BlockScaledArgs {
    const float* sa;      // [K/128][lds_a]: scale of row m for K block kb at sa[kb * lds_a + m]
    const float* sb;      // [N/128][K/128] row-major
    int64_t lds_a;
    void* c;              // bf16 [M, N]
    int tma_store;
    int M, N, K;
};

__global__ void __launch_bounds__(kBsThreads, 1)
fp8_gemm_blockscaled_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                            const __grid_constant__ CUtensorMap map_c, uint32_t idesc, BlockScaledArgs e, int tiles_m,
                            int tiles_n) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* smem_a = smem;
    uint8_t* smem_b = smem + (size_t)kBsStages * kBsStageA;
    uint8_t* staging = smem + (size_t)kBsStages * kBsStageBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(staging + kBsStaging);
    uint64_t* full_bar = bars;                               // [kBsStages] TMA -> MMA
    uint64_t* empty_bar = bars + kBsStages;                  // [kBsStages] MMA -> TMA
    uint64_t* part_full = bars + 2 * kBsStages;              // [kBsParts] K block's product complete -> promotion
    uint64_t* part_empty = bars + 2 * kBsStages + kBsParts;  // [kBsParts] promotion has read it -> MMA
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kBsStages + 2 * kBsParts);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int k_blocks = e.K / kBK;
    const int n_tiles = tiles_m * tiles_n;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kBsStages; ++s) { mbar_init(&full_bar[s], 1); mbar_init(&empty_bar[s], 1); }
        for (int i = 0; i < kBsParts; ++i) { mbar_init(&part_full[i], 1); mbar_init(&part_empty[i], kBsEpiWarps); }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s2u(tmem_slot)), "r"(kTmemCols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    bool ok = true;

    if (warp == 0) {
        if (lane == 0) {
            int it = 0;
            for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
                int tile_m, tile_n;
                banded_tile(t, tiles_m, tiles_n, kGroupM, tile_m, tile_n);
                for (int kb = 0; kb < k_blocks; ++kb, ++it) {
                    const int s = it % kBsStages;
                    if (it >= kBsStages) ok = mbar_wait(&empty_bar[s], ((it / kBsStages) - 1) & 1, abort_flag);
                    if (!ok) break;
                    mbar_expect_tx(&full_bar[s], kBsStageBytes);
                    tma_load_2d(smem_a + (size_t)s * kBsStageA, &map_a, kb * kBK, tile_m * 128, &full_bar[s]);
                    tma_load_2d(smem_b + (size_t)s * kBsStageB, &map_b, kb * kBK, tile_n * kBsBN, &full_bar[s]);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int it = 0;   // K blocks issued so far: stage it % kBsStages, partial buffer it % kBsParts
            for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
                for (int kb = 0; kb < k_blocks; ++kb, ++it) {
                    const int s = it % kBsStages, pb = it % kBsParts;
                    if (it >= kBsParts) ok = mbar_wait(&part_empty[pb], ((it / kBsParts) - 1) & 1, abort_flag);
                    if (ok) ok = mbar_wait(&full_bar[s], (it / kBsStages) & 1, abort_flag);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t tmem_d = tmem_base + (uint32_t)(pb * kBsBN);
                    const uint64_t da = make_smem_desc(s2u(smem_a + (size_t)s * kBsStageA));
                    const uint64_t db = make_smem_desc(s2u(smem_b + (size_t)s * kBsStageB));
#pragma unroll
                    for (int k = 0; k < kBK / kUmmaK; ++k)
                        umma_f8(tmem_d, da + (uint64_t)(k * (kUmmaK >> 4)), db + (uint64_t)(k * (kUmmaK >> 4)), idesc, k != 0);
                    umma_commit(&empty_bar[s]);
                    umma_commit(&part_full[pb]);
                }
            }
        }
    } else {
        // ---------------- promotion + epilogue (warps 2..9) ----------------
        const int quarter = warp & 3;            // TMEM lanes this warp may read
        const int chalf = (warp - 2) >> 2;       // which 64 of the tile's 128 columns
        uint8_t* stg = staging + (size_t)(warp - 2) * 4096;
        int it = 0;
        for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
            int tile_m, tile_n;
                banded_tile(t, tiles_m, tiles_n, kGroupM, tile_m, tile_n);
            const int row0 = tile_m * 128 + quarter * 32, row = row0 + lane;
            float acc[64];
#pragma unroll
            for (int i = 0; i < 64; ++i) acc[i] = 0.f;
            // the two scales of a K block (rows beyond M contribute nothing and are never stored) are fetched one
            // K block ahead: their global-memory latency would otherwise sit between every two promotions
            const float* sa_row = e.sa + (row < e.M ? row : 0);
            const float* sb_row = e.sb + (int64_t)tile_n * k_blocks;
            float s_next = row < e.M ? sa_row[0] * sb_row[0] : 0.f;
            for (int kb = 0; kb < k_blocks && ok; ++kb, ++it) {
                const int pb = it % kBsParts;
                const float scale = s_next;
                if (kb + 1 < k_blocks) s_next = row < e.M ? sa_row[(int64_t)(kb + 1) * e.lds_a] * sb_row[kb + 1] : 0.f;
                ok = __all_sync(COAT_FULL_MASK, mbar_wait(&part_full[pb], (it / kBsParts) & 1, abort_flag));
                if (!ok) break;
                tc_fence_after();
                uint32_t r[64];
                tmem_ld64(tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(pb * kBsBN + chalf * 64), r);
#pragma unroll
                for (int i = 0; i < 64; ++i) acc[i] = __fmaf_rn(__uint_as_float(r[i]), scale, acc[i]);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(s2u(&part_empty[pb])) : "memory");
            }
            if (!ok) break;
            const int col0 = tile_n * kBsBN + chalf * 64;
            if (e.tma_store) {
                if (lane == 0) bulk_wait_read();
                __syncwarp();
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    uint32_t o[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        o[q] = (uint32_t)coat_float_to_bf16_bits(acc[8 * j + 2 * q]) |
                               ((uint32_t)coat_float_to_bf16_bits(acc[8 * j + 2 * q + 1]) << 16);
                    *reinterpret_cast<uint4*>(stg + lane * 128 + ((j ^ (lane & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0 && row0 < e.M) {
                    tma_store_2d(&map_c, stg, col0, row0);
                    bulk_commit();
                }
            } else if (row < e.M) {
                __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(e.c) + (int64_t)row * e.N + col0;
                for (int i = 0; i < 64; ++i) dst[i] = __float2bfloat16_rn(acc[i]);
            }
        }
        if (lane == 0) bulk_wait_all();
    }
    if (!ok) { *abort_flag = 1; g_gemm_device_status = COAT_E_TIMEOUT; }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols) : "memory");
    }
}

// ---- host side ------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// Tile height for a problem.  Cost model in units of "one 128-row unit done by the 128-row kernel": that kernel
// overlaps its epilogue and takes ceil(units / SMs) rounds of one unit; the 256-row kernel does a unit in about
// 0.785 + 939 / K of that time (less shared-memory traffic per flop, but an exposed epilogue; fitted to
// measurements at K = 4096, 8192 and 11008), takes rounds of two units and, when its last round is at most half
// full, finishes it in about 1.5 units' time (a single unit still loads a whole B stage per K block).
// COAT_GEMM_BM=128|256 in the environment overrides the choice.
int coat_gemm_tile_rows(int64_t M, int64_t N, int64_t K) {
    static int forced = -1;
    if (forced < 0) {
        const char* v = getenv("COAT_GEMM_BM");
        forced = v ? atoi(v) : 0;
    }
    if (M <= 128) return 128;
    if (forced == 128 || forced == 256) return forced;
    const int64_t units_m = (M + 127) / 128, units_n = (N + kBN - 1) / kBN, sms = coat_sm_count();
    const int64_t units = units_m * units_n, tiles = ((units_m + 1) / 2) * units_n;
    const double cost128 = (double)((units + sms - 1) / sms);
    const int64_t full = tiles / sms, rest = tiles % sms;
    const double rounds256 = 2.0 * full + (rest == 0 ? 0.0 : (2 * rest <= sms ? 1.5 : 2.0));
    const double cost256 = rounds256 * (0.785 + 939.0 / (double)K);
    return cost256 < cost128 ? 256 : 128;
}

// K-major byte matrix [rows, K] with row pitch K; box = 128 bytes of K x box_rows rows, 128-byte swizzle
int make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t K, int box_rows) {
    EncodeTiledFn enc = encode_tiled();
    if (!enc) return COAT_E_DEVICE;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? COAT_OK : COAT_E_BADARG;
}

// bf16 output [M, N] (row pitch 2N bytes, a multiple of 16): box = 64 columns x 32 rows, 128-byte swizzle
int make_map_c(CUtensorMap* map, void* base, int64_t M, int64_t N) {
    EncodeTiledFn enc = encode_tiled();
    if (!enc) return COAT_E_DEVICE;
    const cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)M};
    const cuuint64_t strides[1] = {(cuuint64_t)N * 2};
    const cuuint32_t box[2] = {64, 32};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, base, dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? COAT_OK : COAT_E_BADARG;
}

// Which kernel serves a problem.  Measured on the Llama-2-7B MLP shapes (burst / sustained under the 1 kW power
// cap, TFLOP/s): forward K=4096: pair 2869 / 2551, 128-row 2798 / 2471, 256-row 2655 / 2349; dgrad K=11008:
// 256-row 2720 / 2392, pair 2640 / 2333, 128-row 2535 / 2263; wgrad K=8192: 256-row 2650 / 2330, pair 2507 /
// 2230, 128-row 2339 / 2117.  So: CTA pairs for short reductions, the 256-row tile for long ones, the 128-row
// tile for matrices of at most 128 rows.  COAT_GEMM_PAIR=0|1 and COAT_GEMM_BM=128|256 in the environment
// override the choice (experiments).
bool coat_gemm_use_pair(int64_t M, int64_t K) {
    static int pair = -2, bm = -1;
    if (pair == -2) {
        const char* v = getenv("COAT_GEMM_PAIR");
        pair = v ? atoi(v) : -1;
        const char* w = getenv("COAT_GEMM_BM");
        bm = w ? atoi(w) : 0;
    }
    if (M <= 128) return false;
    if (pair == 0 || pair == 1) return pair == 1;
    if (bm == 128 || bm == 256) return false;
    return K < 6144;
}

template <int FMT_C>
int launch_pair(const CUtensorMap& map_a, const CUtensorMap& map_b, const CUtensorMap& map_c, uint32_t idesc,
                const GemmEpilogue& e, int tiles_m, int tiles_n, int64_t tiles, cudaStream_t st) {
    auto kern = fp8_gemm_pair_kernel<FMT_C>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPairSmem) != cudaSuccess)
        return COAT_E_LAUNCH;
    // how many pairs the device can hold at once (SM counts per GPC need not be even)
    static int max_pairs[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return COAT_E_DEVICE;
    if (max_pairs[dev] == 0) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (unsigned)(coat_sm_count() / 2));
        cfg.blockDim = dim3(kPairThreads);
        cfg.dynamicSmemBytes = kPairSmem;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) { cudaGetLastError(); return COAT_E_LAUNCH; }
        max_pairs[dev] = n;
    }
    const int64_t pairs = tiles < max_pairs[dev] ? tiles : max_pairs[dev];
    kern<<<(unsigned)(2 * pairs), kPairThreads, kPairSmem, st>>>(map_a, map_b, map_c, idesc, e, tiles_m, tiles_n);
    return coat_launch_status();
}

}  // namespace

extern "C" int coat_fp8_gemm(const uint8_t* a, const uint8_t* b, void* c, void* scale_c, const void* scale_a,
                             const void* scale_b, const void* bias, int64_t M, int64_t N, int64_t K, int fmt_a,
                             int fmt_b, int scale_dtype, int bias_dtype, int output_quantize, int QB, int flags,
                             void* stream) {
    if (M < 0 || N < 0 || K < 0) return COAT_E_BADARG;
    if (M == 0 || N == 0) return COAT_OK;
    if (!a || !b || !c || !scale_a || !scale_b || (output_quantize && !scale_c)) return COAT_E_BADARG;
    if ((fmt_a != COAT_E4M3 && fmt_a != COAT_E5M2) || (fmt_b != COAT_E4M3 && fmt_b != COAT_E5M2)) return COAT_E_BADARG;
    if (K == 0 || K % 16 != 0) return COAT_E_SHAPE;            // TMA row pitch must be a multiple of 16 bytes
    if (!coat_aligned(a, 16) || !coat_aligned(b, 16) || !coat_aligned(c, 16)) return COAT_E_ALIGN;
    if (output_quantize && ((QB != 16 && QB != 32) || N % QB != 0)) return COAT_E_SHAPE;
    if (M > 0x7fffffff || N > 0x7fffffff || K > 0x7fffffff) return COAT_E_TOOBIG;
    const int bm = coat_gemm_tile_rows(M, N, K);
    CUtensorMap map_a, map_b;
    if (int rc = make_map(&map_a, a, M, K, 128)) return rc;   // A always arrives in 128-row boxes
    if (int rc = make_map(&map_b, b, N, K, kBN)) return rc;
    GemmEpilogue e = {};
    CUtensorMap map_c = map_a;   // placeholder when the TMA-store epilogue is not used
    if (!output_quantize && N % 8 == 0) {
        if (int rc = make_map_c(&map_c, c, M, N)) return rc;
        e.tma_store = 1;
    }
    e.c = c; e.scale_c = scale_c; e.scale_a = scale_a; e.scale_b = scale_b; e.bias = bias;
    e.scale_dtype = scale_dtype; e.bias_dtype = bias_dtype; e.quantize = output_quantize; e.QB = QB;
    e.fmt_c = fmt_a; e.ieee_div = (flags & COAT_QUANT_IEEE_DIV) ? 1 : 0;
    e.M = (int)M; e.N = (int)N; e.K = (int)K;
    // operands that stay in L2 together (126 MB, of which the output stream takes its share) need no bands
    e.band_rows = (M + N) * K > (int64_t)96 * 1024 * 1024 ? kGroupM : 0;
    const uint32_t idesc = make_idesc(fmt_a, fmt_b, 128, kBN);
    // work is counted in units of 128 rows x 256 columns for both tile heights
    const int tiles_m = (int)((M + 127) / 128), tiles_n = (int)((N + kBN - 1) / kBN);
    const int64_t n_units = (int64_t)tiles_m * tiles_n;
    if (n_units > 0x7fffffff) return COAT_E_TOOBIG;
    const int sms = coat_sm_count();
    const unsigned grid = (unsigned)(n_units < sms ? n_units : sms);
    cudaStream_t st = (cudaStream_t)stream;
    if (coat_gemm_use_pair(M, K)) {
        // CTA pairs: 256 x 256 tiles, A and B both in 128-row boxes, instruction shape M256 N256
        CUtensorMap map_b2;
        if (int rc = make_map(&map_b2, b, N, K, 128)) return rc;
        const uint32_t idesc2 = make_idesc(fmt_a, fmt_b, 256, kBN);
        const int tm = (int)((M + 255) / 256);
        const int64_t tiles = (int64_t)tm * tiles_n;
        int rc = COAT_E_LAUNCH;
        if (fmt_a == COAT_E4M3) rc = launch_pair<COAT_E4M3>(map_a, map_b2, map_c, idesc2, e, tm, tiles_n, tiles, st);
        else rc = launch_pair<COAT_E5M2>(map_a, map_b2, map_c, idesc2, e, tm, tiles_n, tiles, st);
        return rc;
    }
#define COAT_GEMM_LAUNCH(FMT, BMV)                                                                          \
    do {                                                                                                  \
        auto kern = fp8_gemm_kernel<FMT, BMV>;                                                            \
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,                       \
                                 (int)GemmShape<BMV>::kSmem) != cudaSuccess)                              \
            return COAT_E_LAUNCH;                                                                         \
        kern<<<grid, GemmShape<BMV>::kThreads, GemmShape<BMV>::kSmem, st>>>(map_a, map_b, map_c, idesc, e, tiles_m, tiles_n); \
    } while (0)
    if (fmt_a == COAT_E4M3) {
        if (bm == 256) COAT_GEMM_LAUNCH(COAT_E4M3, 256); else COAT_GEMM_LAUNCH(COAT_E4M3, 128);
    } else {
        if (bm == 256) COAT_GEMM_LAUNCH(COAT_E5M2, 256); else COAT_GEMM_LAUNCH(COAT_E5M2, 128);
    }
#undef COAT_GEMM_LAUNCH
    return coat_launch_status();
}

// Synchronises, returns and clears the GEMM's device status word (COAT_E_TIMEOUT if a bounded wait ran out).
extern "C" int coat_fp8_gemm_device_status(void) {
    int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_gemm_device_status, sizeof(int)) != cudaSuccess) return COAT_E_LAUNCH;
    if (v != 0 && cudaMemcpyToSymbol(g_gemm_device_status, &zero, sizeof(int)) != cudaSuccess) return COAT_E_LAUNCH;
    return v;
}

extern "C" int coat_fp8_gemm_blockscaled(const uint8_t* a, const float* scale_a, int64_t lds_a, const uint8_t* b,
                                         const float* scale_b, void* c, int64_t M, int64_t N, int64_t K, int fmt_a,
                                         int fmt_b, void* stream) {
    if (M < 0 || N < 0 || K < 0) return COAT_E_BADARG;
    if (M == 0 || N == 0) return COAT_OK;
    if (!a || !b || !c || !scale_a || !scale_b || lds_a < M) return COAT_E_BADARG;
    if ((fmt_a != COAT_E4M3 && fmt_a != COAT_E5M2) || (fmt_b != COAT_E4M3 && fmt_b != COAT_E5M2)) return COAT_E_BADARG;
    if (K == 0 || K % 128 != 0 || N % 128 != 0) return COAT_E_SHAPE;   // whole scale blocks only
    if (!coat_aligned(a, 16) || !coat_aligned(b, 16) || !coat_aligned(c, 16)) return COAT_E_ALIGN;
    if (M > 0x7fffffff || N > 0x7fffffff || K > 0x7fffffff) return COAT_E_TOOBIG;
    CUtensorMap map_a, map_b, map_c;
    if (int rc = make_map(&map_a, a, M, K, 128)) return rc;
    if (int rc = make_map(&map_b, b, N, K, kBsBN)) return rc;
    if (int rc = make_map_c(&map_c, c, M, N)) return rc;
    BlockScaledArgs e = {scale_a, scale_b, lds_a, c, 1, (int)M, (int)N, (int)K};
    const uint32_t idesc = make_idesc(fmt_a, fmt_b, 128, kBsBN);
    const int tiles_m = (int)((M + 127) / 128), tiles_n = (int)((N + kBsBN - 1) / kBsBN);
    const int64_t tiles = (int64_t)tiles_m * tiles_n;
    if (tiles > 0x7fffffff) return COAT_E_TOOBIG;
    const int sms = coat_sm_count();
    const unsigned grid = (unsigned)(tiles < sms ? tiles : sms);
    if (cudaFuncSetAttribute(fp8_gemm_blockscaled_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBsSmem) !=
        cudaSuccess)
        return COAT_E_LAUNCH;
    fp8_gemm_blockscaled_kernel<<<grid, kBsThreads, kBsSmem, (cudaStream_t)stream>>>(map_a, map_b, map_c, idesc, e,
                                                                                   tiles_m, tiles_n);
    return coat_launch_status();
}
