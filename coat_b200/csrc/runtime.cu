// Process-wide helpers of the C ABI: version, error strings, device probing.
#include "common.cuh"

#include <cstring>

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
        case COAT_E_PEER: return "peer memory could not be allocated, exported or mapped";
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

// ---- buffers that the other processes of a node can map (CUDA IPC) -----------------------------
static_assert(sizeof(cudaIpcMemHandle_t) == COAT_PEER_HANDLE_BYTES, "handle size is part of the ABI");

extern "C" int coat_peer_buffer_create(int64_t bytes, void** ptr_out, void* handle_out) {
    if (bytes <= 0 || !ptr_out || !handle_out) return COAT_E_BADARG;
    void* p = nullptr;
    if (cudaMalloc(&p, (size_t)bytes) != cudaSuccess) { cudaGetLastError(); return COAT_E_PEER; }
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(p);
        return COAT_E_PEER;
    }
    if (cudaMemset(p, 0, (size_t)bytes) != cudaSuccess) { cudaGetLastError(); cudaFree(p); return COAT_E_PEER; }
    memcpy(handle_out, &h, sizeof(h));
    *ptr_out = p;
    return COAT_OK;
}

extern "C" int coat_peer_buffer_open(const void* handle, void** ptr_out) {
    if (!handle || !ptr_out) return COAT_E_BADARG;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        return COAT_E_PEER;
    }
    *ptr_out = p;
    return COAT_OK;
}

extern "C" int coat_peer_buffer_close(void* ptr) {
    if (!ptr) return COAT_OK;
    if (cudaIpcCloseMemHandle(ptr) != cudaSuccess) { cudaGetLastError(); return COAT_E_PEER; }
    return COAT_OK;
}

extern "C" int coat_peer_buffer_free(void* ptr) {
    if (!ptr) return COAT_OK;
    if (cudaFree(ptr) != cudaSuccess) { cudaGetLastError(); return COAT_E_PEER; }
    return COAT_OK;
}

// Asynchronous device-to-device copy by raw pointers on `stream`: the source in this GPU's memory, the destination a
// mapped peer buffer (coat_peer_buffer_open) or local memory.  The DMA engines move the bytes; no SM is involved.
extern "C" int coat_peer_copy_async(void* dst, const void* src, int64_t bytes, void* stream) {
    if (bytes < 0 || (bytes > 0 && (!dst || !src))) return COAT_E_BADARG;
    if (bytes == 0) return COAT_OK;
    if (cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDeviceToDevice, (cudaStream_t)stream) != cudaSuccess) {
        cudaGetLastError();
        return COAT_E_PEER;
    }
    return COAT_OK;
}

