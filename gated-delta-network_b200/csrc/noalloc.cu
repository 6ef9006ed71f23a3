// noalloc.cu -- prefill entry point for callers that cannot allocate device memory.
//
// gdn_prefill_fwd needs a caller-provided workspace (w, u, Aqk, G: about 7.2 KB per token).
// Some callers cannot provide one: a host runtime that owns every byte of device memory and
// forbids plugins from calling cudaMalloc, a serving loop whose memory budget is fixed at
// start-up, or code that must not allocate while other work is in flight.  For them this file
// keeps the workspace in a fixed, file-scope device array sized for GDN_NOALLOC_MAX_TOKENS
// tokens in at most GDN_NOALLOC_MAX_SEQS sequences; it is allocated when the library is
// loaded and held by every GPU that loads the library until the process exits.
//
// Host code may not pass the array's name to a kernel: on the host it is a stand-in symbol,
// not a device address.  The device address is looked up once per device with
// cudaGetSymbolAddress (with that device current) on the first call and cached.  The cache
// belongs to the device's primary context: a caller that resets the device (cudaDeviceReset)
// destroys the array with the context and must not call this entry point on that device again
// in the same process.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/gdn_b200.h"
#include "common.cuh"
#include "kernels.cuh"

namespace {

// Largest workspace any accepted call needs (HV = 8).  The layout grows with N and T, and the
// segmented route adds its regions for calls of few long sequences, so take the maximum over
// every accepted (N, T).
constexpr size_t noalloc_bytes() {
    size_t m = 0;
    for (int n = 0; n <= GDN_NOALLOC_MAX_SEQS; ++n)
        for (int t = 0; t <= GDN_NOALLOC_MAX_TOKENS; ++t) {
            const size_t b = gdn::prefill_layout(n, t).total;
            if (b > m) m = b;
        }
    return m;
}
constexpr size_t kNoAllocBytes = noalloc_bytes();

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

constexpr int kMaxDevices = 64;
// Device address of g_noalloc_scratch per device (nullptr until set up).  Two threads setting up
// the same device concurrently store the same value.
void* g_scratch_addr[kMaxDevices];

}  // namespace

extern "C" int gdn_prefill_fwd_noalloc(const void* q, const void* k, const void* v, const float* state,
                                       const float* A_log, const void* a, const float* dt_bias, const void* b,
                                       const void* cu_seqlens, int cu_is_int64, int N, int T, float scale, void* out,
                                       float* new_state, int H, int HV, int K, int V, void* stream, unsigned flags) {
    if (T < 0 || N < 0 || T > GDN_NOALLOC_MAX_TOKENS || N > GDN_NOALLOC_MAX_SEQS) return GDN_ERR_SIZE;
    // The device check comes before the symbol lookup: on a GPU without an sm_100a image the
    // lookup itself would fail and report a CUDA error instead of the unsupported device.
    const int drc = gdn::check_device();
    if (drc != GDN_OK) return drc;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return GDN_ERR_CUDA;
    if (dev < 0 || dev >= kMaxDevices) return GDN_ERR_DEVICE;
    if (g_scratch_addr[dev] == nullptr) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
            cudaGetLastError();
            return GDN_ERR_CUDA;
        }
        g_scratch_addr[dev] = p;
    }
    const size_t need = gdn_prefill_workspace_bytes(N, T, H, HV, K, V);
    if (need == 0) return GDN_ERR_SHAPE;
    if (need > kNoAllocBytes) return GDN_ERR_SIZE;  // the array is sized for HV = 8 v-heads
    return gdn_prefill_fwd(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, cu_is_int64, N, T, scale, out, new_state,
                           g_scratch_addr[dev], need, H, HV, K, V, stream, flags);
}
