/*
 * coat_b200 — C ABI of the B200-native (sm_100a) COAT quantization hot path.
 *
 * Every entry point takes raw device pointers, sizes, dtype enums and a CUDA
 * stream (passed as void*, a cudaStream_t), allocates nothing, launches
 * asynchronously on that stream and returns 0 or a negative COAT_E_* code.
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
 * Debug / health entry points of the optimizer kernels (no counterpart in the reference).
 * coat_fp8_adamw_debug_counters: later launches add to 8 device counters (uint64): groups on the guarded
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
