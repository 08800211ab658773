// Cross-entropy loss with the gradient written in place of the logits, for sm_100a.
//
// What it computes follows the loss head the reference trains with (coat/activation/liger/cross_entropy.py:25-198,
// the Liger kernel in the configuration COAT uses: hard labels, no label smoothing, no z-loss, no soft-capping):
// per row of logits x[0..V) with target y
//     lse = log sum_j exp(x_j),  loss = lse - x_y,  dloss/dx_j = softmax(x)_j - [j == y]
// both scaled by 1/n (n = number of rows whose target is not `ignore_index`) for the mean reduction; a row whose
// target is `ignore_index` gets zero loss and zero gradients.  The gradient overwrites x, so no second [rows, V]
// tensor ever exists.
//
// How: one CTA of 256 threads per row, 16-byte accesses.  Pass 1 is the online softmax (every thread keeps a
// running maximum and a sum rescaled when the maximum moves, the 256 pairs are merged through shuffles and shared
// memory), pass 2 re-reads the row (128 KB for a 32000-entry fp32 row: it comes back from L2), turns it into the
// gradient and writes it.  HBM roofline: the row is read once and written once, 8 B per logit in fp32.

#include "common.cuh"

namespace {

constexpr int kCeThreads = 256;

struct MaxSum { float m, d; };   // running maximum and sum of exp(x - m)

__device__ __forceinline__ MaxSum merge(MaxSum a, MaxSum b) {
    const float m = fmaxf(a.m, b.m);
    if (m == -INFINITY) return {m, 0.f};   // both empty
    return {m, a.d * __expf(a.m - m) + b.d * __expf(b.m - m)};
}

template <typename T> struct Vec;   // 16 bytes of logits
template <> struct Vec<float> {
    static constexpr int N = 4;
    static __device__ __forceinline__ void load(const float* p, float (&v)[4]) {
        const float4 t = *reinterpret_cast<const float4*>(p);
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    }
    static __device__ __forceinline__ void store(float* p, const float (&v)[4]) {
        *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    }
    static __device__ __forceinline__ float get(const float* p) { return *p; }
    static __device__ __forceinline__ void put(float* p, float x) { *p = x; }
};
template <> struct Vec<__nv_bfloat16> {
    static constexpr int N = 8;
    static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&v)[8]) {
        const uint4 t = *reinterpret_cast<const uint4*>(p);
        const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            v[2 * i] = __uint_as_float(w[i] << 16);
            v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
    }
    static __device__ __forceinline__ void store(__nv_bfloat16* p, const float (&v)[8]) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
            w[i] = *reinterpret_cast<const uint32_t*>(&h);
        }
        *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    static __device__ __forceinline__ float get(const __nv_bfloat16* p) { return __bfloat162float(*p); }
    static __device__ __forceinline__ void put(__nv_bfloat16* p, float x) { *p = __float2bfloat16_rn(x); }
};

template <typename T>
__global__ void __launch_bounds__(kCeThreads)
cross_entropy_inplace_kernel(T* __restrict__ x, int64_t ld, const int64_t* __restrict__ target, float* __restrict__ loss,
                             int64_t V, int64_t ignore_index, float inv_n) {
    constexpr int N = Vec<T>::N;
    __shared__ MaxSum part[kCeThreads / 32];
    __shared__ MaxSum total;
    T* row = x + (int64_t)blockIdx.x * ld;
    const int64_t y = target[blockIdx.x];
    const bool vec = (reinterpret_cast<uintptr_t>(row) & 15) == 0;   // rows 16-byte aligned: the vector path
    const int64_t v_main = vec ? V / N * N : 0;
    if (y == ignore_index) {   // no loss, no gradient
        float z[N];
#pragma unroll
        for (int i = 0; i < N; ++i) z[i] = 0.f;
        for (int64_t j = (int64_t)threadIdx.x * N; j < v_main; j += kCeThreads * N) Vec<T>::store(row + j, z);
        for (int64_t j = v_main + threadIdx.x; j < V; j += kCeThreads) Vec<T>::put(row + j, 0.f);
        if (threadIdx.x == 0) loss[blockIdx.x] = 0.f;
        return;
    }
    // ---- pass 1: online softmax
    MaxSum acc = {-INFINITY, 0.f};
    for (int64_t j = (int64_t)threadIdx.x * N; j < v_main; j += kCeThreads * N) {
        float v[N];
        Vec<T>::load(row + j, v);
        float m = v[0];
#pragma unroll
        for (int i = 1; i < N; ++i) m = fmaxf(m, v[i]);
        if (m > acc.m) { acc.d *= __expf(acc.m - m); acc.m = m; }   // exp(-inf) = 0 covers the first block
#pragma unroll
        for (int i = 0; i < N; ++i) acc.d += __expf(v[i] - acc.m);
    }
    for (int64_t j = v_main + threadIdx.x; j < V; j += kCeThreads) acc = merge(acc, MaxSum{Vec<T>::get(row + j), 1.f});
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        MaxSum other = {__shfl_xor_sync(COAT_FULL_MASK, acc.m, o), __shfl_xor_sync(COAT_FULL_MASK, acc.d, o)};
        acc = merge(acc, other);
    }
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        MaxSum t = part[0];
        for (int w = 1; w < kCeThreads / 32; ++w) t = merge(t, part[w]);
        total = t;
        const float lse = t.m + logf(t.d);
        const float xy = (y >= 0 && y < V) ? Vec<T>::get(row + y) : 0.f;
        loss[blockIdx.x] = (lse - xy) * inv_n;
    }
    __syncthreads();   // also orders thread 0's read of x_y before anyone overwrites the row
    const float m = total.m;
    const float scale = inv_n / total.d;
    // ---- pass 2: gradient in place
    for (int64_t j = (int64_t)threadIdx.x * N; j < v_main; j += kCeThreads * N) {
        float v[N];
        Vec<T>::load(row + j, v);
#pragma unroll
        for (int i = 0; i < N; ++i) v[i] = __expf(v[i] - m) * scale - ((j + i == y) ? inv_n : 0.f);
        Vec<T>::store(row + j, v);
    }
    for (int64_t j = v_main + threadIdx.x; j < V; j += kCeThreads)
        Vec<T>::put(row + j, __expf(Vec<T>::get(row + j) - m) * scale - ((j == y) ? inv_n : 0.f));
}

}  // namespace

// Cross entropy with in-place gradient: x [rows, V] (fp32 or bf16, row pitch `ld` elements) is overwritten with
// d(sum of losses)/dx, loss[r] receives row r's loss, both scaled by inv_n (1 / number of counted rows for the mean
// reduction, 1 for the sum).  Rows whose target equals ignore_index get zeros.  Targets outside [0, V) that are not
// ignore_index are a caller error; they yield the log-sum-exp as loss and a pure softmax gradient.
extern "C" int coat_cross_entropy_inplace(void* x, int x_dtype, int64_t ld, const int64_t* target, float* loss,
                                          int64_t rows, int64_t V, int64_t ignore_index, float inv_n, void* stream) {
    if (rows < 0 || V < 0 || ld < V) return COAT_E_BADARG;
    if (rows == 0 || V == 0) return COAT_OK;
    if (!x || !target || !loss) return COAT_E_BADARG;
    if (x_dtype != COAT_F32 && x_dtype != COAT_BF16) return COAT_E_BADARG;
    if (rows > 0x7fffffffLL) return COAT_E_TOOBIG;
    cudaStream_t st = (cudaStream_t)stream;
    if (x_dtype == COAT_F32)
        cross_entropy_inplace_kernel<float><<<(unsigned)rows, kCeThreads, 0, st>>>(
            reinterpret_cast<float*>(x), ld, target, loss, V, ignore_index, inv_n);
    else
        cross_entropy_inplace_kernel<__nv_bfloat16><<<(unsigned)rows, kCeThreads, 0, st>>>(
            reinterpret_cast<__nv_bfloat16*>(x), ld, target, loss, V, ignore_index, inv_n);
    return coat_launch_status();
}
