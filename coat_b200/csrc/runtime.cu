// Process-wide helpers of the C ABI: version, error strings, device probing.
#include "common.cuh"

int coat_sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (cached[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

extern "C" const char* coat_b200_version(void) { return "coat_b200 0.1 (sm_100a)"; }

extern "C" const char* coat_strerror(int code) {
    switch (code) {
        case COAT_OK: return "ok";
        case COAT_E_BADARG: return "bad argument (null pointer, negative size or unknown enum)";
        case COAT_E_QGROUP: return "Only Support 128 per-group quantization currently";
        case COAT_E_ALIGN: return "pointer or leading dimension is not aligned as the kernel requires";
        case COAT_E_SHAPE: return "shape is not divisible as the operator requires";
        case COAT_E_LAUNCH: return "CUDA reported an error for the kernel launch";
        case COAT_E_DEVICE: return "the current CUDA device is not an sm_100 (B200) device";
        case COAT_E_TOOBIG: return "size exceeds the static maximum of this entry point";
        case COAT_E_TIMEOUT: return "a bounded device-side wait ran out";
        default: return "unknown coat_b200 error";
    }
}

extern "C" int coat_check_device(void) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return COAT_E_DEVICE;
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return COAT_E_DEVICE;
    return major == 10 ? COAT_OK : COAT_E_DEVICE;
}
