// api.cu -- extern "C" entry points declared in include/gdn_b200.h.
//
// Host-side validation mirrors the reference's shape asserts
// (reference/gdn_decode_ref.py:32-36, reference/gdn_prefill_ref.py:33-36) and
// adds the checks the kernels rely on (alignment, workspace size, device).
// Nothing here synchronises, copies to the host or allocates device memory.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/gdn_b200.h"
#include "common.cuh"

#include "kernels.cuh"
#include "prefill_kernels.cuh"

namespace {

constexpr int kMaxDevices = 64;
// 0 = unknown, 1 = compute capability 10.0, 2 = other.  Benign race: every writer stores the same value.
int g_dev_ok[kMaxDevices];

}  // namespace

namespace gdn {

// The library holds sm_100a code only: other compute capabilities (including sm_103 parts of
// the same major) have no image to run, so they are refused here with GDN_ERR_DEVICE.
int check_device() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return GDN_ERR_CUDA;
    if (dev < 0 || dev >= kMaxDevices) return GDN_ERR_DEVICE;
    if (g_dev_ok[dev] == 0) {
        int major = 0, minor = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
            return GDN_ERR_CUDA;
        g_dev_ok[dev] = (major == 10 && minor == 0) ? 1 : 2;
    }
    return g_dev_ok[dev] == 1 ? GDN_OK : GDN_ERR_DEVICE;
}

}  // namespace gdn

namespace {

using gdn::check_device;

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Head size 128; any number of q/k heads H with HV a multiple of H (grouped v-heads).  The
// reference asserts H = 4, HV = 8 (reference/gdn_decode_ref.py:32-36); other counts are a
// superset (e.g. the qk16_v32 family, or one q/k head group of the reference's heads per GPU).
bool shape_ok(int H, int HV, int K, int V) {
    return H >= 1 && H <= GDN_MAX_QK_HEADS && HV >= H && HV <= GDN_MAX_V_HEADS && HV % H == 0 && K == GDN_HEAD_DIM &&
           V == GDN_HEAD_DIM;
}
bool prefill_shape_ok(int H, int HV, int K, int V) { return shape_ok(H, HV, K, V); }

int decode_variant(int B, int HV, unsigned flags) {
    const unsigned forced = (flags >> 8) & 0xffu;  // tuning override: variant + 1
    if (forced) return (int)forced - 1;
    // small batches: 16-row CTAs keep >= ~2 CTAs per SM in flight (measured on B200: B=16 4.00 us
    // vs 4.69 us with 32-row CTAs; from B=32 up the two are within 1%, B=64 favours 32-row CTAs)
    return B * HV <= 128 ? 2 : 0;
}

}  // namespace

extern "C" {

int gdn_decode_fwd(const void* q, const void* k, const void* v, const float* state, const float* A_log,
                   const void* a, const float* dt_bias, const void* b, float scale, void* out, float* new_state,
                   int B, int H, int HV, int K, int V, void* stream, unsigned flags) {
    if (!shape_ok(H, HV, K, V)) return GDN_ERR_SHAPE;
    if (B < 0) return GDN_ERR_SIZE;
    if (!q || !k || !v || !A_log || !a || !dt_bias || !b || !out || !new_state) return GDN_ERR_NULL;
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || !aligned16(new_state) ||
        (state && !aligned16(state)))
        return GDN_ERR_ALIGN;
    if (B == 0) return GDN_OK;
    int rc = check_device();
    if (rc != GDN_OK) return rc;
    gdn::DecodeArgs p;
    p.q = static_cast<const uint16_t*>(q);
    p.k = static_cast<const uint16_t*>(k);
    p.v = static_cast<const uint16_t*>(v);
    p.state = state;
    p.A_log = A_log;
    p.a = static_cast<const uint16_t*>(a);
    p.dt_bias = dt_bias;
    p.b = static_cast<const uint16_t*>(b);
    p.scale = scale;
    p.out = static_cast<uint16_t*>(out);
    p.new_state = new_state;
    p.B = B;
    p.H = H;
    p.HV = HV;
    p.l2norm = (flags & GDN_FLAG_QK_L2NORM) ? 1 : 0;
    const int lrc = gdn::launch_decode(p, decode_variant(B, HV, flags), static_cast<cudaStream_t>(stream));
    if (lrc == -1) return GDN_ERR_SIZE;  // unknown tuning variant
    if (lrc != 0) return GDN_ERR_CUDA;
    return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_CUDA;
}

size_t gdn_prefill_workspace_bytes(int N, int T, int H, int HV, int K, int V) {
    if (!prefill_shape_ok(H, HV, K, V) || N < 0 || T < 0) return 0;
    return gdn::prefill_layout(N, T, HV).total;
}

int gdn_prefill_fwd(const void* q, const void* k, const void* v, const float* state, const float* A_log,
                    const void* a, const float* dt_bias, const void* b, const void* cu_seqlens, int cu_is_int64,
                    int N, int T, float scale, void* out, float* new_state, void* workspace, size_t workspace_bytes,
                    int H, int HV, int K, int V, void* stream, unsigned flags) {
    if (!prefill_shape_ok(H, HV, K, V)) return GDN_ERR_SHAPE;
    if (N < 0 || T < 0) return GDN_ERR_SIZE;
    if (N == 0) return GDN_OK;
    if (!cu_seqlens || !new_state || !A_log || !dt_bias) return GDN_ERR_NULL;
    if (T > 0 && (!q || !k || !v || !a || !b || !out)) return GDN_ERR_NULL;
    // the gates are TMA tiles when HV is a multiple of 8 (16-byte rows), plain bf16 loads otherwise
    const bool gates_ok = HV % 8 == 0 ? aligned16(a) && aligned16(b)
                                      : (reinterpret_cast<uintptr_t>(a) & 1u) == 0 && (reinterpret_cast<uintptr_t>(b) & 1u) == 0;
    if ((T > 0 && (!aligned16(q) || !aligned16(k) || !aligned16(v) || !gates_ok || !aligned16(out))) ||
        !aligned16(new_state) ||
        (state && !aligned16(state)))
        return GDN_ERR_ALIGN;
    if (cu_is_int64 != 0 && cu_is_int64 != 1) return GDN_ERR_SIZE;
    const gdn::PrefillLayout lay = gdn::prefill_layout(N, T, HV);
    if (!workspace || workspace_bytes < lay.total || (reinterpret_cast<uintptr_t>(workspace) & 255u))
        return GDN_ERR_WORKSPACE;
    int rc = check_device();
    if (rc != GDN_OK) return rc;
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    gdn::PrefillArgs p;
    p.q = static_cast<const uint16_t*>(q);
    p.k = static_cast<const uint16_t*>(k);
    p.v = static_cast<const uint16_t*>(v);
    p.state = state;
    p.A_log = A_log;
    p.a = static_cast<const uint16_t*>(a);
    p.dt_bias = dt_bias;
    p.b = static_cast<const uint16_t*>(b);
    p.cu = cu_seqlens;
    p.cu64 = cu_is_int64;
    p.N = N;
    p.T = T;
    p.H = H;
    p.HV = HV;
    p.S = lay.S;
    p.small_n = N <= gdn::kSmallN ? 1 : 0;
    p.test_withhold = (flags & GDN_FLAG_TEST_WITHHOLD_CHUNK) ? 1 : 0;
    p.no_short = (flags & GDN_FLAG_NO_SHORT_PATH) ? 1 : 0;
    p.l2norm = (flags & GDN_FLAG_QK_L2NORM) ? 1 : 0;
    p.scale = scale;
    p.out = static_cast<uint16_t*>(out);
    p.new_state = new_state;
    p.status = reinterpret_cast<int*>(ws + lay.off_status);
    p.chunk_base = reinterpret_cast<int*>(ws + lay.off_base);
    p.chunk_seq = reinterpret_cast<int*>(ws + lay.off_seq);
    p.long_list = reinterpret_cast<int*>(ws + lay.off_long);
    p.w = reinterpret_cast<uint16_t*>(ws + lay.off_w);
    p.u = reinterpret_cast<float*>(ws + lay.off_u);
    p.qp = reinterpret_cast<uint16_t*>(ws + lay.off_qp);
    p.oi = reinterpret_cast<uint16_t*>(ws + lay.off_oi);
    p.g4 = reinterpret_cast<float*>(ws + lay.off_g4);
    const unsigned forced_bv = (flags >> 8) & 0xffu;
    const int bv = forced_bv ? (int)forced_bv : gdn::prefill_scan_bv(N, HV);
    if (bv != 8 && bv != 16 && bv != 32 && bv != 64) return GDN_ERR_SIZE;
    // Segmented route (only when the layout has its regions): the default for a few sequences
    // averaging >= 6144 tokens, or forced by GDN_FLAG_SEGMENTS; never with a forced scan variant or
    // GDN_FLAG_NO_SEGMENTS.  Bits 16-23 force its segment length, which must not need more segment
    // slots than the layout holds.
    const bool seg_on = ((flags & GDN_FLAG_SEGMENTS) || gdn::prefill_seg_default(N, T)) && !forced_bv &&
                        !(flags & GDN_FLAG_NO_SEGMENTS);
    p.seg_m = seg_on ? lay.seg_m : 0;
    p.SS = lay.SS;
    const unsigned forced_m = (flags >> 16) & 0xffu;
    if (p.seg_m > 0 && forced_m) {
        if ((long long)lay.S / forced_m + N > lay.SS && lay.S > lay.SS) return GDN_ERR_SIZE;
        p.seg_m = (int)forced_m;
    }
    p.seg_D = reinterpret_cast<uint16_t*>(ws + lay.off_segD);
    p.seg_B = reinterpret_cast<float*>(ws + lay.off_segB);
    p.seg_gamma = reinterpret_cast<float*>(ws + lay.off_segG);
    p.seg_hb = reinterpret_cast<uint16_t*>(ws + lay.off_seghb);
    p.qpp = reinterpret_cast<uint16_t*>(ws + lay.off_qpp);
    p.oipp = reinterpret_cast<uint16_t*>(ws + lay.off_oipp);
    if (gdn::launch_prefill(p, bv, static_cast<cudaStream_t>(stream)) != 0) return GDN_ERR_CUDA;
    return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_CUDA;
}

const char* gdn_status_string(int status) {
    switch (status) {
        case GDN_OK: return "ok";
        case GDN_ERR_NULL: return "a required pointer is NULL";
        case GDN_ERR_SHAPE: return "unsupported shape (need K=V=128, HV a multiple of H)";
        case GDN_ERR_ALIGN: return "a tensor pointer is not 16-byte aligned";
        case GDN_ERR_SIZE: return "invalid size or option";
        case GDN_ERR_WORKSPACE: return "workspace missing, misaligned (256 B) or too small";
        case GDN_ERR_CUDA: return "CUDA launch failed";
        case GDN_ERR_DEVICE: return "current device is not an sm_100 (B200) GPU";
        default: return "unknown status";
    }
}

int gdn_version(void) { return 100; }

}  // extern "C"
