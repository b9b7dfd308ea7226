// capi.cu -- library-level C entry points (version, status strings, device
// error word).
#include "mi_common.cuh"

extern "C" int mi_version(void) { return 1; }

extern "C" const char* mi_status_string(int status) {
    switch (status) {
        case MI_OK: return "ok";
        case MI_ERR_INVALID: return "invalid argument";
        case MI_ERR_UNSUPPORTED: return "unsupported shape or configuration";
        case MI_ERR_CUDA: return "CUDA error";
        case MI_ERR_DEVICE: return "device error word set";
        default: return "unknown status";
    }
}

extern "C" int mi_device_error(int* out, int clear, void* stream) {
    if (!out) return MI_ERR_INVALID;
    cudaStream_t s = (cudaStream_t)stream;
    int v = 0;
    if (cudaMemcpyFromSymbolAsync(&v, mi::g_dev_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s) != cudaSuccess)
        return MI_ERR_CUDA;
    if (cudaStreamSynchronize(s) != cudaSuccess) return MI_ERR_CUDA;
    if (clear && v) {
        int z = 0;
        if (cudaMemcpyToSymbolAsync(mi::g_dev_error, &z, sizeof(int), 0, cudaMemcpyHostToDevice, s) != cudaSuccess)
            return MI_ERR_CUDA;
        if (cudaStreamSynchronize(s) != cudaSuccess) return MI_ERR_CUDA;
    }
    *out = v;
    return MI_OK;
}
