// noalloc.cu -- mi_conv_act_quant_noalloc: the conv + activation + int8
// quantisation stage with its row-absmax scratch held in a fixed device array
// of this library instead of a caller-provided workspace.
//
// Who needs it: a host that cannot call cudaMalloc for a scratch buffer --
// for example a runtime whose device memory is owned by a different
// allocator it must not bypass, or a serving loop that is not allowed to
// allocate while it runs.  Such a caller still passes its inputs and outputs
// but has no way to provide the batch*L-float workspace that
// mi_conv_act_quant needs.
//
// The scratch lives in a file-scope __device__ array of NOALLOC_MAX_ROWS
// floats (1 MiB), which every GPU that loads the library keeps until the
// process exits.  Host code cannot use the array's name as a device address,
// so the first call on each device looks the address up with
// cudaGetSymbolAddress (with that device current) and caches it for the life
// of the process.  cudaDeviceReset destroys the context the array lives in and
// the cached address with it: a process that resets a device must not call
// this entry point on that device afterwards.
#include <mutex>

#include "mi_common.cuh"

namespace mi {
namespace noalloc {

constexpr int NOALLOC_MAX_ROWS = 1 << 18;  // batch * L limit: 262144 token rows (1 MiB of fp32)
constexpr int MAX_DEVICES = 64;

static __device__ __align__(256) float g_conv_amax_scratch[NOALLOC_MAX_ROWS];

static std::mutex g_lock;
static float* g_scratch_ptr[MAX_DEVICES];  // device address of the array, per device

// Device address of the scratch array on the current device (set-up on first use).
// A failed runtime call is reported by this call only: its error is cleared from
// the runtime's last-error state so that later, unrelated entry points (which
// check cudaGetLastError after their launches) do not report it again.
static int scratch_ptr(float** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return MI_ERR_CUDA;
    }
    if (dev < 0 || dev >= MAX_DEVICES) return MI_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> guard(g_lock);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_conv_amax_scratch) != cudaSuccess || p == nullptr) {
            cudaGetLastError();
            return MI_ERR_CUDA;
        }
        g_scratch_ptr[dev] = static_cast<float*>(p);
    }
    *out = g_scratch_ptr[dev];
    return MI_OK;
}

}  // namespace noalloc
}  // namespace mi

extern "C" int mi_conv_act_quant_noalloc(const float* xz, int ldx, const float* w, const float* bias, float* act,
                                         int8_t* xq, float* xscale, int batch, int L, int D, void* stream) {
    using namespace mi::noalloc;
    if (!xq || !xscale) return MI_ERR_INVALID;
    if (batch <= 0 || L <= 0) return MI_ERR_INVALID;
    if ((long long)batch * L > NOALLOC_MAX_ROWS) return MI_ERR_UNSUPPORTED;  // more rows than the fixed scratch
    float* scratch = nullptr;
    const int rc = scratch_ptr(&scratch);
    if (rc != MI_OK) return rc;
    // mi_conv_act_quant zero-fills the absmax rows it uses before the conv
    // kernel accumulates into them, so the previous call's contents do not leak
    return mi_conv_act_quant(xz, ldx, w, bias, act, xq, xscale, scratch, batch, L, D, stream);
}
