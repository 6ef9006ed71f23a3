// prefill_kernels.cuh -- pieces shared by the three prefill translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.cuh"

namespace gdn {

// TMA tensor maps of one prefill call (kernel parameters, 128 B each).
struct PrefillMaps {
    CUtensorMap q;    // (128 col, 4 head, T token) bf16, box 64 x 1 x 64, SWIZZLE_128B
    CUtensorMap k;    // same
    CUtensorMap v;    // (128, 8, T) bf16, box 64 x 1 x 64, SWIZZLE_128B
    CUtensorMap w;    // (128 col, S*64 row, 8 head) bf16, box 64 x 64 x 1, SWIZZLE_128B
    CUtensorMap qp;   // (128, S*64, 8) bf16, box 64 x 64 x 1, SWIZZLE_128B
    CUtensorMap oi;   // (128, S*64, 8) bf16, box BV x 64 x 1, no swizzle
    CUtensorMap u;    // (128, S*64, 8) f32, box BV x 64 x 1, no swizzle
    CUtensorMap g4;   // (4, S*64, 8) f32, box 4 x 64 x 1, no swizzle
    CUtensorMap u_st;   // (128, S*64, 8) f32, box 32 x 64 x 1, SWIZZLE_128B (prep's stores)
    CUtensorMap oi_st;  // (128, S*64, 8) bf16, box 64 x 64 x 1, SWIZZLE_128B (prep's stores)
};

// Sequence n's token range [s, e), clamped to [0, T] (malformed cu_seqlens cannot index outside).
__device__ __forceinline__ void seq_bounds(const void* cu, int cu64, int n, int T, int& s, int& e) {
    long long a, b;
    if (cu64) {
        a = reinterpret_cast<const long long*>(cu)[n];
        b = reinterpret_cast<const long long*>(cu)[n + 1];
    } else {
        a = reinterpret_cast<const int*>(cu)[n];
        b = reinterpret_cast<const int*>(cu)[n + 1];
    }
    a = a < 0 ? 0 : (a > T ? T : a);
    b = b < a ? a : (b > T ? T : b);
    s = (int)a;
    e = (int)b;
}

bool build_prefill_maps(const PrefillArgs& p, int bv, PrefillMaps* m);
int launch_prefill_prep(const PrefillArgs& p, const PrefillMaps& maps, cudaStream_t stream);
int launch_prefill_scan(const PrefillArgs& p, const PrefillMaps& maps, int bv, cudaStream_t stream);

}  // namespace gdn
