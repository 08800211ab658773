/*
 * coat_b200 — C ABI of the B200-native (sm_100a) COAT quantization hot path.
 *
 * Every compute entry point takes raw device pointers, sizes, dtype enums and a
 * CUDA stream (passed as void*, a cudaStream_t), allocates nothing, launches
 * asynchronously on that stream and returns 0 or a negative COAT_E_* code.
 * The only entry points that allocate are the set-up helpers of the sharded
 * optimizer step, coat_peer_buffer_create / _open (cudaMalloc and CUDA IPC,
 * outside any step); the status getters synchronise.
 * No C++ or torch types cross this boundary.  Tensors are dense row-major
 * unless a stride is passed explicitly.
 *
 * The comments cite the interface of the reference implementation
 * (NVlabs/COAT, paths relative to its root) that each entry point replaces.
 */
#ifndef COAT_B200_H
#define COAT_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- error codes --------------------------------------------------------- */
#define COAT_OK 0
#define COAT_E_BADARG (-1)  /* null pointer, negative size, unknown enum       */
#define COAT_E_QGROUP (-2)  /* optimizer group size other than 128             */
#define COAT_E_ALIGN (-3)   /* pointer / leading dimension alignment           */
#define COAT_E_SHAPE (-4)   /* shape not divisible as the operator requires    */
#define COAT_E_LAUNCH (-5)  /* cudaGetLastError() after the launch was not OK  */
#define COAT_E_DEVICE (-6)  /* not an sm_100 device / no device                */
#define COAT_E_TOOBIG (-7)  /* size beyond a documented static maximum         */
#define COAT_E_TIMEOUT (-8) /* a bounded device-side wait ran out              */
#define COAT_E_PEER (-9)    /* peer memory could not be allocated / mapped     */

/* ---- dtype enums --------------------------------------------------------- */
#define COAT_F32 0
#define COAT_BF16 1
#define COAT_F16 2
#define COAT_E4M3 0
#define COAT_E5M2 1

/* ---- flags for the optimizer step ---------------------------------------- */
/* Evaluate every pow() of the expansion with the exact libdevice routine, as
 * the reference kernel does (slow, the checker for the guarded fast path).   */
#define COAT_ADAMW_EXACT_POW 1

/* ---- flags for the quantizers --------------------------------------------- */
/* Use IEEE division for scale = (amax + 1e-10) / fp8_max and q = x / scale instead of the
 * PTX div.full.f32 the reference's Triton kernels compile to (a CPU can reproduce IEEE
 * division bit for bit; div.full.f32 differs from it in the last place now and then).   */
#define COAT_QUANT_IEEE_DIV 1
#define COAT_QUANT_STOCHASTIC 2   /* coat_fp8_division only: the reference's stochastic rounding */

const char* coat_b200_version(void);
const char* coat_strerror(int code);
/* 0 if the current device is sm_100, else COAT_E_DEVICE. */
int coat_check_device(void);

/*
 * Fused FP8 AdamW step with Dynamic Range Expansion, one tensor, in place.
 * Replaces qoptim_cuda.fp8_adamw_expand_step
 *   (coat/optimizer/kernels/bindings.cpp:7,
 *    coat/optimizer/kernels/include/fp8_adamw_expand.h:6-17,
 *    kernel coat/optimizer/kernels/fp8_adamw_expand_cuda_kernel.cu:21-203).
 * p, g        : numel elements of p_dtype (COAT_F32 / COAT_BF16 / COAT_F16)
 * m, v        : numel E4M3 codes (first / second moment)
 * s_*, k_*, r_* : ceil(numel/128) fp32 each: group scale, expansion exponent,
 *               sqrt(max*min) of the group
 * bf16_out    : optional (may be NULL) numel bf16 copy of the updated weights
 * qgroup must be 128 (as the reference asserts, .cu:221).
 */
int coat_fp8_adamw_expand_step(void* p, const void* g,
                               uint8_t* m, float* s_m, float* k_m, float* r_m,
                               uint8_t* v, float* s_v, float* k_v, float* r_v,
                               float beta1, float beta2, float lr, float wd, float eps,
                               int step, int qgroup, int expand_min,
                               int64_t numel, int p_dtype,
                               void* bf16_out, int flags, void* stream);

/*
 * Fused FP8 AdamW step without expansion, one tensor, in place.
 * Replaces qoptim_cuda.fp8_adamw_step
 *   (coat/optimizer/kernels/bindings.cpp:6,
 *    coat/optimizer/kernels/include/fp8_adamw.h:6-14,
 *    kernel coat/optimizer/kernels/fp8_adamw_cuda_kernel.cu:21-125).
 */
int coat_fp8_adamw_step(void* p, const void* g,
                        uint8_t* m, float* s_m, uint8_t* v, float* s_v,
                        float beta1, float beta2, float lr, float wd, float eps,
                        int step, int qgroup,
                        int64_t numel, int p_dtype,
                        void* bf16_out, int flags, void* stream);

/*
 * One launch for a list of tensors that share hyper-parameters and step
 * (what the python loop coat/optimizer/fp8_adamw.py:455-515 does with one
 * launch per tensor).  `table` is a DEVICE array of n_tensors descriptors;
 * `group_prefix` is a DEVICE array of n_tensors+1 int64: exclusive prefix sum
 * of ceil(numel/128).  k_* / r_* may be NULL when expand == 0.
 */
typedef struct CoatAdamwTensor {
    void* p;
    const void* g;
    uint8_t* m;
    uint8_t* v;
    float* s_m;
    float* k_m;
    float* r_m;
    float* s_v;
    float* k_v;
    float* r_v;
    void* bf16_out; /* may be NULL */
    int64_t numel;
} CoatAdamwTensor;

int coat_fp8_adamw_multi_step(const CoatAdamwTensor* table, const int64_t* group_prefix,
                              int n_tensors, int64_t total_groups, int expand,
                              float beta1, float beta2, float lr, float wd, float eps,
                              int step, int qgroup, int expand_min, int p_dtype,
                              int flags, void* stream);

/*
 * The table launch fused with the exchange that follows it under ZeRO-style sharding: besides
 * bf16_out itself, every bf16 store of the kernel is repeated at bf16_out + peer_deltas[i] bytes,
 * i < n_peers <= COAT_MAX_PEERS, i.e. into the same slot of peer i's copy of the gathered-weights
 * buffer (peer_deltas[i] = peer i's mapped base - this GPU's base; multiples of 16).  Bulk
 * (TMA, non-multicast) and plain stores over NVLink: the kernel never waits on a peer.  The stores have landed when the kernel has
 * completed on every GPU, so a consumer needs one cross-GPU barrier after the launch (any stream-
 * ordered collective will do).  peer_deltas is a HOST array, read during the call.  No reference
 * counterpart (the reference leaves sharding to FSDP).
 */
#define COAT_MAX_PEERS 7
int coat_fp8_adamw_multi_step_bcast(const CoatAdamwTensor* table, const int64_t* group_prefix,
                                    int n_tensors, int64_t total_groups, int expand,
                                    float beta1, float beta2, float lr, float wd, float eps,
                                    int step, int qgroup, int expand_min, int p_dtype,
                                    int flags, const int64_t* peer_deltas, int n_peers, void* stream);

/*
 * Set-up helpers for the broadcast step, the only entry points that allocate or synchronise:
 * a device buffer that other processes of the node can map (CUDA IPC; no multicast object is
 * created).  create: cudaMalloc + export a COAT_PEER_HANDLE_BYTES handle to send to the peers.
 * open: map a peer's handle into this process (enables peer access lazily); the returned pointer
 * is valid on the current device.  close / free undo them; free only after every peer closed.
 */
#define COAT_PEER_HANDLE_BYTES 64
int coat_peer_buffer_create(int64_t bytes, void** ptr_out, void* handle_out);
int coat_peer_buffer_open(const void* handle, void** ptr_out);
int coat_peer_buffer_close(void* ptr);
int coat_peer_buffer_free(void* ptr);
/* Asynchronous copy of `bytes` bytes from this GPU's memory to a mapped peer buffer (or local memory) on `stream`,
 * by the DMA engines: the transport of the bucketed "copy" exchange of the sharded step (no reference counterpart:
 * the reference leaves the weight all-gather to the host framework's FSDP). */
int coat_peer_copy_async(void* dst, const void* src, int64_t bytes, void* stream);

/* =========================== quantizers ====================================
 * x is an M x N row-major matrix of in_dtype (COAT_BF16 / COAT_F16 / COAT_F32) with row stride ldx
 * (elements); codes are dense M x N (or N x M) bytes of format fmt (COAT_E4M3 / COAT_E5M2); scales are
 * of scale_dtype (COAT_BF16, the reference's default, COAT_F32 or COAT_F16).  N must be a multiple of QB,
 * x 16-byte aligned with a 16-byte multiple row pitch.  3-D inputs are flattened by the caller, as the
 * reference's python wrappers do.
 */

/* Per-1xQB-group quantize: s = (max|x| + 1e-10) / fp8_max per group, q = x / s; QB in {16,32,64,128}.
 * Replaces fp8_quantize (coat/activation/real_quantization/_quantize.py:120-163, kernel :37-118). */
int coat_fp8_quantize(const void* x, uint8_t* y, void* s_y, int64_t M, int64_t N, int64_t ldx, int QB,
                      int fmt, int in_dtype, int scale_dtype, int flags, void* stream);

/* Pass 1 of the per-tensor quantize: the tensor's amax (as the bit pattern of a non-negative float, in the
 * 4-byte scratch word *amax_bits, which this call zeroes first on the stream) and, if s_y != NULL, the
 * per-1xQB-group scales.  Replaces the kernel of fp8_quantize_pertensor /
 * fp8_quantize_pertensor_transpose (_quantize_pertensor.py:46-103, _quantize_pertensor_transpose.py:46-103)
 * together with the torch reduction s_y.max() that follows it (:139). */
int coat_fp8_group_scales_amax(const void* x, void* s_y, unsigned int* amax_bits, int64_t M, int64_t N,
                               int64_t ldx, int QB, int fmt, int in_dtype, int scale_dtype, int flags,
                               void* stream);

/* Division by ONE scale, q = x / s, with optional transposed copy: y (M x N) and / or y_t (N x M) may be
 * NULL (y == NULL is the reference's only_transposed=True).  The scale is the device scalar *s_in of
 * scale_dtype, or, if amax_bits != NULL, round_to_scale_dtype((amax + 1e-10) / fp8_max) taken from pass 1,
 * which is then also written to *s_out.  Replaces fp8_division (_division.py:153-207, kernel :45-126) and
 * fp8_division_transpose (_division_transpose.py:147-210, kernel :48-144).  With COAT_QUANT_STOCHASTIC in
 * flags the quotient is perturbed before the cast as the reference's `stochastic=True` does
 * (_division.py:96-150: noise = Triton's rand(seed 0, offset m * ldx + n), i.e. Philox-4x32-10, scaled to one
 * step of the format and clamped to the quotient's binade); y must then be given (y_t, if wanted, is its
 * byte transpose). */
int coat_fp8_division(const void* x, uint8_t* y, uint8_t* y_t, const void* s_in, void* s_out,
                      const unsigned int* amax_bits, int64_t M, int64_t N, int64_t ldx, int fmt,
                      int in_dtype, int scale_dtype, int flags, void* stream);

/* Per-tensor quantize in ONE cooperative launch: pass 1 (tensor amax, and the 1xQB group scales if s_y != NULL), a
 * bounded grid barrier, pass 2 (q = x / s with s = round_to_scale_dtype((amax + 1e-10) / fp8_max), also written
 * to *s_out).  Every CTA re-reads, backwards, the part of x it read in pass 1, so the second read is served from
 * L2.  Same results as coat_fp8_group_scales_amax + coat_fp8_division.  Outputs: y (M x N) and / or the
 * transposed copy y_t (N x M); with y_t the tile kernel runs: s_y must be NULL, M a multiple of 16
 * (COAT_E_SHAPE otherwise: use the two calls), y_t 16-byte aligned.  sync_words: 12 bytes of caller scratch that
 * must be ZERO on entry and are zero again when the kernel ends (so one zero-initialised allocation serves all
 * calls that are ordered on a stream; two calls that may overlap on the GPU need separate words; after
 * COAT_E_TIMEOUT zero them again).  Replaces fp8_quantize_pertensor (_quantize_pertensor.py:106-147: kernel,
 * s_y.max(), fp8_division) and fp8_quantize_pertensor_transpose (_quantize_pertensor_transpose.py:106-150). */
int coat_fp8_quantize_pertensor(const void* x, uint8_t* y, uint8_t* y_t, void* s_y, void* s_out,
                                unsigned int* sync_words, int64_t M, int64_t N, int64_t ldx, int QB, int fmt,
                                int in_dtype, int scale_dtype, int flags, void* stream);

/* Synchronises, returns and clears the quantizers' device status word (COAT_E_TIMEOUT if a bounded wait on a
 * staging copy or at the grid barrier ran out; never expected).  A call that timed out has written wrong
 * codes, but it leaves the sync words of coat_fp8_quantize_pertensor zero like any other call. */
int coat_fp8_quantize_device_status(void);

/* Diagnostic (no counterpart in the reference): how many polls a CTA of the one-launch per-tensor kernels spends
 * at their grid barrier before it gives up, on the current device; polls < 0 restores the default (about one
 * second).  The tests lower it to 0 to see a timeout reported and healed without making any GPU wait. */
int coat_fp8_quantize_set_barrier_limit(int polls);

/* One pass: 1x16 groups along the rows -> (y, s_y[M, N/16]) and 1x16 groups of the transposed matrix
 * (16 consecutive rows of one column) -> (y_t[N, M], s_y_t[N, M/16]).  QB must be 16, M a multiple of 16.
 * Replaces fp8_quantize_transpose (_quantize_transpose.py:176-226, kernel :39-173). */
int coat_fp8_quantize_transpose(const void* x, uint8_t* y, void* s_y, uint8_t* y_t, void* s_y_t, int64_t M,
                                int64_t N, int64_t ldx, int QB, int fmt, int in_dtype, int scale_dtype,
                                int flags, void* stream);

/* Byte transpose of an M x N code matrix (M, N multiples of 4).
 * Replaces fp8_transpose (_transpose.py:85-115, kernel :39-82). */
int coat_fp8_transpose(const uint8_t* x, uint8_t* y_t, int64_t M, int64_t N, void* stream);

/* y = bf16(code * group scale).  Replaces fp8_dequantize (_dequantize.py:119-156, kernel :44-116). */
int coat_fp8_dequantize(const uint8_t* x, const void* s_x, void* y_bf16, int64_t M, int64_t N, int QB,
                        int fmt, int scale_dtype, void* stream);

/* Per-tensor quantize, optionally with the transposed copy, for callers that can neither allocate device
 * memory nor set aside the 4-byte amax word the two-call form above needs: a plugin living inside a
 * fixed memory budget, a host without a caching allocator, code in a section where cudaMalloc's
 * device-wide synchronisation is not acceptable.  It has no counterpart in the reference (whose wrappers
 * allocate freely through torch).  The scratch is a ~17 KB array inside the library image, which every
 * GPU that loads the library keeps until the process ends; it limits the input to 67 108 864 elements
 * (COAT_E_TOOBIG beyond that).  All calls on a device share that array: back-to-back calls on one
 * stream are fine, calls that overlap on the GPU race.  The first call on a device queries the array's
 * address and should be made before any stream capture starts.  Results are identical to
 * coat_fp8_group_scales_amax + coat_fp8_division.  y or y_t may be NULL (not both).  Round-to-nearest only:
 * COAT_QUANT_STOCHASTIC in flags is rejected with COAT_E_BADARG. */
int coat_fp8_quantize_pertensor_static(const void* x, uint8_t* y, uint8_t* y_t, void* s_out, int64_t M,
                                       int64_t N, int64_t ldx, int fmt, int in_dtype, int scale_dtype,
                                       int flags, void* stream);

/* Quantizers with 128-wide granularity (the DeepSeek-style block-scaled linear layer): from one read of x
 * (M, N multiples of 128) any subset of
 *   y_b  [M,N] + s_b  [M/128, N/128]  one scale per 128x128 block      (fp8_quantize_perblock,
 *                                      coat/activation/real_quantization/_quantize_perblock.py:115-150)
 *   y_bt [N,M] + s_bt [N/128, M/128]  the same codes transposed        (fp8_quantize_perblock_transpose,
 *                                      _quantize_perblock_transpose.py:127-190)
 *   y_r  [M,N] + s_r  [M, N/128]      one scale per 1x128 row group    (fp8_quantize_transpose with QB = 128,
 *                                      _quantize_transpose.py:39-173, and the per-group output of
 *                                      fp8_quantize_perblock_transpose_pergroup, ..._pergroup.py:145-246)
 *   y_ct [N,M] + s_ct [N, M/128]      one scale per 128x1 column group, transposed (_quantize_transpose.py)
 * Outputs not wanted are NULL (codes and scales together).  Scales are row-major in scale_dtype. */
int coat_fp8_quantize_block128(const void* x, int64_t M, int64_t N, int64_t ldx, uint8_t* y_b, void* s_b,
                               uint8_t* y_bt, void* s_bt, uint8_t* y_r, void* s_r, uint8_t* y_ct, void* s_ct,
                               int fmt, int in_dtype, int scale_dtype, int flags, void* stream);

/* =========================== fused quantize-on-save operators =================================
 * Inputs x, x1, x2 are M x N code matrices quantised in 1xQB groups with scales s_* of shape [M, N/QB];
 * g is a floating (bf16 by default) M x N matrix.  Where an amax_bits pointer is given, the call zeroes
 * that 4-byte word on the stream and leaves the bit pattern of max|result| (of the fp32 values) in it,
 * which coat_fp8_division turns into the per-tensor scale the reference gets from `s_y.max()`.
 */

/* y = 1xQB FP8 of silu(x).  Replaces fp8_silu_forward (coat/activation/real_quantization/silu_fwd.py:152-198,
 * kernel :47-149). */
int coat_fp8_silu_forward(const uint8_t* x, const void* s_x, uint8_t* y, void* s_y, int64_t M, int64_t N,
                          int QB, int fmt, int scale_dtype, int flags, void* stream);

/* y = bf16( act'(x) * g ), group scales (bf16) for FP8 format fmt_out, tensor amax.  gelu = 0: SiLU
 * (fp8_silu_backward, silu_bwd.py:170-238, kernel :47-167); gelu = 1: erf-GELU (fp8_gelu_backward,
 * gelu_bwd.py:173-230, kernel :47-170). */
int coat_fp8_act_backward(int gelu, const uint8_t* x, const void* s_x, const void* g, void* y_bf16,
                          void* s_y, unsigned int* amax_bits, int64_t M, int64_t N, int QB, int fmt_in,
                          int in_scale_dtype, int g_dtype, int fmt_out, int flags, void* stream);

/* y = bf16(gelu(x)), group scales, tensor amax.  Replaces the kernel of fp8_gelu_forward
 * (gelu_fwd.py:152-203, kernel :47-149). */
int coat_fp8_gelu_forward(const uint8_t* x, const void* s_x, void* y_bf16, void* s_y,
                          unsigned int* amax_bits, int64_t M, int64_t N, int QB, int fmt, int scale_dtype,
                          int flags, void* stream);

/* y = bf16((x1*s1) * (x2*s2)), group scales, tensor amax.  Replaces the kernel of fp8_mul_forward
 * (mul_fwd.py:191-254, kernel :51-188). */
int coat_fp8_mul_forward(const uint8_t* x1, const void* s_x1, const uint8_t* x2, const void* s_x2,
                         void* y_bf16, void* s_y, unsigned int* amax_bits, int64_t M, int64_t N, int QB,
                         int fmt, int scale_dtype, int flags, void* stream);

/* fp8_mul_forward with its per-tensor output in ONE cooperative launch (replaces the whole of fp8_mul_forward,
 * mul_fwd.py:191-254: product kernel :51-188, `s_y.max()`, fp8_division_transpose): y = fp8(bf16((c1 s1)(c2 s2)) / s)
 * [M,N], y_t its transpose [N,M], *s_out = s = the maximum of the rounded 1x16 group scales of the product.  The
 * product is recomputed from the FP8 inputs in a second pass instead of going through a bf16 tensor in memory;
 * results are bit-identical to coat_fp8_mul_forward + coat_fp8_division.  sync_words: 12 bytes of caller scratch,
 * zero on entry and zero again on return (as for coat_fp8_quantize_pertensor).  bf16 scales only; COAT_E_SHAPE unless
 * QB == 16, M % 16 == 0 and N % 128 == 0 (use the two calls there); all pointers 16-byte aligned. */
int coat_fp8_mul_forward_pertensor(const uint8_t* x1, const void* s_x1, const uint8_t* x2, const void* s_x2,
                                   uint8_t* y, uint8_t* y_t, void* s_out, unsigned int* sync_words, int64_t M,
                                   int64_t N, int QB, int fmt, int scale_dtype, int flags, void* stream);

/* y1 = bf16(g * x2), y2 = bf16(g * x1) with group scales (bf16) and tensor amax of y2.  Replaces the kernel
 * of fp8_mul_backward (mul_bwd.py:221-315, kernel :49-218). */
int coat_fp8_mul_backward(const uint8_t* x1, const void* s_x1, const uint8_t* x2, const void* s_x2,
                          const void* g, void* y1_bf16, void* y2_bf16, void* s_y2, unsigned int* amax_bits,
                          int64_t M, int64_t N, int QB, int fmt_in, int in_scale_dtype, int g_dtype,
                          int fmt_out, int flags, void* stream);

/* Forward of the gated MLP product in one kernel: coat_fp8_silu_forward(x_gate) followed by
 * coat_fp8_mul_forward(that result, x_up): q_silu / s_silu = 1xQB FP8 of silu(x_gate) (outputs, the backward pass
 * reads them), y = bf16(dequantised silu * x_up) with group scales s_y (may be NULL) and the tensor amax, bit for bit
 * what the two calls give (an extension: the reference calls fp8_silu_forward, silu_fwd.py:152-198, and
 * fp8_mul_forward, mul_fwd.py:161-254, one after the other). */
int coat_fp8_silu_mul_forward(const uint8_t* x_gate, const void* s_gate, const uint8_t* x_up, const void* s_up,
                              uint8_t* q_silu, void* s_silu, void* y_bf16, void* s_y, unsigned int* amax_bits,
                              int64_t M, int64_t N, int QB, int fmt, int scale_dtype, int flags, void* stream);

/* Backward of the gated MLP product in one kernel: coat_fp8_mul_backward(x_silu, x_up, g) followed by
 * coat_fp8_act_backward(SiLU, x_gate, its first output) without the bf16 round trip between them:
 *   y_up   = bf16(g * x_silu),                              group scales s_y_up (bf16),   tensor amax *amax_up
 *   y_gate = bf16(silu'(x_gate) * bf16(g * x_up)),          group scales s_y_gate (bf16), tensor amax *amax_gate
 * bit for bit what the two calls give (an extension: the reference calls fp8_mul_backward, mul_bwd.py:221-315, and
 * fp8_silu_backward, silu_bwd.py:170-238, one after the other).  fmt_out: the FP8 format the scales are for. */
int coat_fp8_mul_silu_backward(const uint8_t* x_silu, const void* s_silu, const uint8_t* x_up, const void* s_up,
                               const uint8_t* x_gate, const void* s_gate, const void* g, void* y_up_bf16,
                               void* s_y_up, unsigned int* amax_up, void* y_gate_bf16, void* s_y_gate,
                               unsigned int* amax_gate, int64_t M, int64_t N, int QB, int fmt_in,
                               int in_scale_dtype, int g_dtype, int fmt_out, int flags, void* stream);

/* y = bf16(x1 + x2); if y_q != NULL also its 1xQB FP8 copy; group scales (bf16); optional tensor amax.
 * Replaces fp8_add_Ifp_Ifp_Ofp_Og16 (add_fwd.py:162-213, kernel :46-159) and the kernel of
 * fp8_add_Ifp_Ifp_Ofp_Opt (add_bwd.py:147-200, kernel :48-144). */
int coat_fp8_add(const void* x1, const void* x2, void* y_bf16, uint8_t* y_q, void* s_y,
                 unsigned int* amax_bits, int64_t M, int64_t N, int QB, int x1_dtype, int x2_dtype,
                 int fmt_out, int flags, void* stream);

/* RMSNorm of a 1xQB-quantised input: y = bf16(x * rstd * w), one bf16 scale per row, rstd (fp32) per row,
 * tensor amax.  N <= 16384.  Replaces the kernel of fp8_rmsnorm_forward (func_rmsnorm.py:223-278,
 * kernel :54-111). */
int coat_fp8_rmsnorm_forward(const uint8_t* x, const void* s_x, const void* w, void* y_bf16,
                             void* s_y_rows_bf16, float* rstd, unsigned int* amax_bits, int64_t M,
                             int64_t N, int QB, float eps, int fmt, int in_scale_dtype, int w_dtype,
                             int flags, void* stream);

/* RMSNorm backward: dx (bf16) and dw (w_dtype).  partial_dw is caller-provided scratch of n_partials x N
 * fp32 (n_partials CTAs each sum their rows in registers, a second kernel adds the partials in order:
 * deterministic, no locks).  dy2 / dy3 (NULL, or bf16 like dy): further addends of the upstream gradient; the
 * kernel uses bf16(bf16(dy + dy2) + dy3), what a bf16 `dy + dy2 + dy3` in torch gives, without the add kernels
 * (an extension: the reference sums the projections' input gradients in torch before this call).  Replaces
 * fp8_rmsnorm_backward (func_rmsnorm.py:281-335, kernels :121-220). */
int coat_fp8_rmsnorm_backward(const uint8_t* x, const void* s_x, const void* dy, const void* dy2, const void* dy3,
                              const void* w, const float* rstd, void* dx_bf16, float* partial_dw, int n_partials,
                              void* dw, int64_t M, int64_t N, int QB, int fmt, int in_scale_dtype,
                              int dy_dtype, int w_dtype, void* stream);

/* LayerNorm of a 1xQB-quantised input, without (w == b == NULL) or with weight and bias: per row
 * mean = sum(x) / N, rstd = 1 / sqrt(sum((x - mean)^2) / N + eps), y = (x - mean) * rstd (* w + b), written in
 * FP32 as the reference does (its per-tensor division then reads fp32); one bf16 scale per row
 * ((max|y| + 1e-10) / fp8_max), mean and rstd (fp32) per row, tensor amax.  N <= 16384.  Replaces the kernels
 * of fp8_layernorm_noparam_forward (func_layernorm_noparam.py:188-245, kernel :54-110) and
 * fp8_layernorm_param_forward (func_layernorm_param.py:204-263, kernel :54-113). */
int coat_fp8_layernorm_forward(const uint8_t* x, const void* s_x, const void* w, const void* b, float* y_f32,
                               void* s_y_rows_bf16, float* mean, float* rstd, unsigned int* amax_bits,
                               int64_t M, int64_t N, int QB, float eps, int fmt, int in_scale_dtype,
                               int wb_dtype, int flags, void* stream);

/* LayerNorm backward: dx (bf16) = (w*dy - (xhat * mean(xhat * w*dy) + mean(w*dy))) * rstd with
 * xhat = (x - mean) * rstd; with w != NULL also dw = sum_rows dy * xhat and db = sum_rows dy (w_dtype), through
 * caller-provided scratch `partial` of n_partials x 2 x N fp32 (deterministic two-stage sum, no locks), N <= 8192;
 * with w == NULL partial, dw and db are unused and N <= 16384.  Replaces fp8_layernorm_noparam_backward
 * (func_layernorm_noparam.py:248-297, kernel :123-185; its stochastic branch names variables that do not
 * exist there and cannot run, so it has no counterpart here) and fp8_layernorm_param_backward
 * (func_layernorm_param.py:266-367, kernels :124-200). */
int coat_fp8_layernorm_backward(const uint8_t* x, const void* s_x, const void* dy, const void* w,
                                const float* mean, const float* rstd, void* dx_bf16, float* partial,
                                int n_partials, void* dw, void* db, int64_t M, int64_t N, int QB, int fmt,
                                int in_scale_dtype, int dy_dtype, int w_dtype, void* stream);

/* =========================== FP8 GEMM ==========================================================
 * C[M,N] = (A[M,K] * B[N,K]^T) * (float(*scale_a) * float(*scale_b)) (+ bias[N]), A and B FP8 codes, both with
 * K contiguous (row pitch K bytes, K a multiple of 16, 16-byte aligned bases), formats fmt_a / fmt_b chosen per
 * operand (forward E4M3 x E4M3, dgrad / wgrad E5M2 x E4M3).  fp32 accumulation on the tcgen05 tensor cores.
 * output_quantize == 0: C is bf16 [M,N].  output_quantize == 1: C is FP8 (format fmt_a) quantised in 1xQB
 * groups (QB 16 or 32, N a multiple of QB) with bf16 scales scale_c[M, N/QB].  scale_a / scale_b are device
 * scalars of scale_dtype, bias (may be NULL) is of bias_dtype.
 * Replaces fp8matmul (coat/activation/real_quantization/linear.py:172-250, kernel _fp8matmul_kernel :61-169),
 * which fp8_linear_forward (:253-258) and fp8_linear_backward (:272-302) call with B passed as a `.t()` view.
 * coat_fp8_gemm_device_status synchronises, returns and clears the kernel's status word (COAT_E_TIMEOUT if a
 * bounded wait on a pipeline barrier ever ran out). */
int coat_fp8_gemm(const uint8_t* a, const uint8_t* b, void* c, void* scale_c, const void* scale_a,
                  const void* scale_b, const void* bias, int64_t M, int64_t N, int64_t K, int fmt_a,
                  int fmt_b, int scale_dtype, int bias_dtype, int output_quantize, int QB, int flags,
                  void* stream);
int coat_fp8_gemm_device_status(void);

/* Block-scaled GEMM of the DeepSeek-style linear layer:
 *   C[m, n] = sum over K blocks kb of scale_a[m, kb] * scale_b[n / 128, kb] * sum_{k in kb} A[m, k] * B[n, k]
 * A [M,K] and B [N,K] FP8 codes with K contiguous; scale_a fp32 with one scale per 1x128 segment of A, stored
 * with the rows contiguous (element (m, kb) at scale_a[kb * lds_a + m], the layout deep_gemm asks for);
 * scale_b fp32 [N/128, K/128] row-major, one scale per 128x128 block of B; C bf16 [M,N].  K and N multiples
 * of 128.  Replaces deep_gemm.gemm_fp8_fp8_bf16_nt as called by fp8_deepseek_linear_forward / _backward
 * (coat/activation/deepseek/linear.py:10-36).  Status word shared with coat_fp8_gemm. */
int coat_fp8_gemm_blockscaled(const uint8_t* a, const float* scale_a, int64_t lds_a, const uint8_t* b,
                              const float* scale_b, void* c, int64_t M, int64_t N, int64_t K, int fmt_a,
                              int fmt_b, void* stream);

/* Rotary position embedding of bf16 q or k: x element (b, s, h, d) at x[b*sxb + s*sxs + h*sxh + d] (strides in
 * elements, multiples of 8), output y contiguous [B, S, H, D], D a multiple of 16:
 *   y = x * cos + rotate_half(x) * sin      (backward != 0: the transposed rotation, for the gradient)
 * cos / sin: bf16 [Bc, S, D], Bc = 1 (cos_batch_stride = 0) or B (cos_batch_stride = S * D).  One fused pass in
 * place of the eager apply_rotary_pos_emb of the attention block (coat/models/coat_llama.py:1031-1036); not
 * part of the quantization path.  y may equal x when x is contiguous. */
int coat_rope_bf16(const void* x, int64_t sxb, int64_t sxs, int64_t sxh, const void* cos_t, const void* sin_t,
                   void* y, int64_t B, int64_t S, int64_t H, int64_t D, int64_t cos_batch_stride, int backward,
                   void* stream);

/* coat_rope_bf16 with fp32 cos / sin tables: the rotary embedding in full precision of the OLMo blocks
 * (coat/models/coat_olmo.py:866-868 calls the host trainer's RotaryEmbedding, which multiplies in fp32 and rounds
 * once to bf16 when rope_full_precision is set). */
int coat_rope_bf16_f32tables(const void* x, int64_t sxb, int64_t sxs, int64_t sxh, const void* cos_t,
                             const void* sin_t, void* y, int64_t B, int64_t S, int64_t H, int64_t D,
                             int64_t cos_batch_stride, int backward, void* stream);

/* Cross-entropy loss with the gradient written in place of the logits: replaces liger_cross_entropy_kernel as
 * cross_entropy_forward launches it for the loss head (coat/activation/liger/cross_entropy.py:25-198, :212-278; hard
 * labels, label_smoothing = lse_square_scale = 0, no soft-capping: the configuration LigerForCausalLMLoss uses,
 * :387-410).  x [rows, V], fp32 or bf16, row pitch ld elements, is overwritten with d(sum of the returned losses)/dx;
 * loss[r] = (logsumexp(x_r) - x_r[target_r]) * inv_n; rows whose target equals ignore_index get zero loss and zero
 * gradients.  inv_n = 1 / (number of counted rows) for the mean reduction, 1 for the sum. */
int coat_cross_entropy_inplace(void* x, int x_dtype, int64_t ld, const int64_t* target, float* loss, int64_t rows,
                               int64_t V, int64_t ignore_index, float inv_n, void* stream);

/*
 * Debug / health entry points of the optimizer kernels (no counterpart in the reference).
 * coat_fp8_adamw_debug_counters: later launches made by the calling host thread add to 8 device counters (uint64): groups on the guarded
 *   fast path, groups on the exact path, exactly recomputed max/min candidates, exactly recomputed
 *   roundings, -, -, and (as float bit patterns in the low 32 bits) the largest observed fraction of the
 *   modelled error bound actually used by the first / second moment.  NULL switches counting off.
 * coat_fp8_adamw_device_status: synchronises, returns and clears the device status word
 *   (COAT_E_TIMEOUT if a bounded wait for a staging copy ever ran out).
 */
int coat_fp8_adamw_debug_counters(unsigned long long* device_counters);
int coat_fp8_adamw_device_status(void);

#ifdef __cplusplus
}
#endif
#endif /* COAT_B200_H */
