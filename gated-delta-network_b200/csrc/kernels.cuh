// kernels.cuh -- argument blocks and launch helpers shared by decode.cu, prefill.cu and api.cu.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace gdn {

struct DecodeArgs {
    const uint16_t* q;     // [B, 4, 128] bf16
    const uint16_t* k;     // [B, 4, 128] bf16
    const uint16_t* v;     // [B, 8, 128] bf16
    const float* state;    // [B, 8, 128, 128] f32 or nullptr (zeros)
    const float* A_log;    // [8]
    const uint16_t* a;     // [B, 8] bf16
    const float* dt_bias;  // [8]
    const uint16_t* b;     // [B, 8] bf16
    float scale;
    uint16_t* out;         // [B, 8, 128] bf16
    float* new_state;      // [B, 8, 128, 128] f32 (may alias state)
    int B;
};

struct PrefillArgs {
    const uint16_t* q;     // [T, 4, 128]
    const uint16_t* k;     // [T, 4, 128]
    const uint16_t* v;     // [T, 8, 128]
    const float* state;    // [N, 8, 128, 128] or nullptr
    const float* A_log;    // [8]
    const uint16_t* a;     // [T, 8]
    const float* dt_bias;  // [8]
    const uint16_t* b;     // [T, 8]
    const void* cu;        // [N+1] int32 / int64
    int cu64;
    int N, T;
    float scale;
    uint16_t* out;         // [T, 8, 128]
    float* new_state;      // [N, 8, 128, 128]
    // workspace regions (head-major, token-indexed)
    uint16_t* w;           // [8][T][128] bf16
    float* u;              // [8][T][128] f32
    uint16_t* aqk;         // [8][T][64] bf16
    float* g;              // [8][T] f32 (chunk-local cumulative log decay)
};

int launch_decode(const DecodeArgs& p, int variant, cudaStream_t stream);
int launch_prefill(const PrefillArgs& p, int bv, cudaStream_t stream);
size_t prefill_workspace_layout(int T, size_t* off_w, size_t* off_u, size_t* off_a, size_t* off_g);
int prefill_scan_bv(int N);

}  // namespace gdn
