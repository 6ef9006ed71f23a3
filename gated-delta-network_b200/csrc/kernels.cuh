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
    int H, HV;             // q/k heads and v heads (HV a multiple of H; 4 and 8 in the reference)
    int l2norm;            // GDN_FLAG_QK_L2NORM: normalise q, k in-kernel
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
    int H, HV;             // q/k heads and v heads (HV a multiple of H; 4 and 8 in the reference)
    int gates_tma;         // 1: HV a multiple of 8, the prep loads the gates as [64 tokens][8 heads] TMA
                           //    boxes; 0: a gate row is under 16 bytes or not a whole box, plain loads
    int S;                 // chunk slots in the workspace (>= number of 64-token chunks)
    int test_withhold;     // GDN_FLAG_TEST_WITHHOLD_CHUNK: the scan skips chunk 1's copies
    int short_path;        // 1: sequences of 0..kShortLen tokens go to a short-sequence kernel, and
                           //    the chunked kernels see only the compacted list of the longer ones
    int rows;              // sequences the scan grid covers (N, or with short_path a bound on the
                           // number of longer sequences: min(N, T / (kShortLen + 1)), at least 1)
    int only_short;        // 1: T <= kShortLen, so every sequence is short: the short kernel is the only
                           //    launch and also zeroes unowned output rows and the status word
    int no_short;          // GDN_FLAG_NO_SHORT_PATH
    int l2norm;            // GDN_FLAG_QK_L2NORM: normalise q, k per token and head in-kernel
    int small_n;           // 1: N is small enough for each CTA to derive its chunk slots itself
                           //    (no chunk-table launch); 0: read chunk_base / chunk_seq
    float scale;
    uint16_t* out;         // [T, 8, 128]
    float* new_state;      // [N, 8, 128, 128]
    // workspace (slot-indexed: slot s holds one 64-token chunk of one sequence; rows past the
    // chunk end are zero / finite padding)
    int* status;           // [0] first error code of a bounded wait that gave up (0 = none); [1], [2] scan / prep work counters
    int* chunk_base;       // [N+1] first slot of each sequence (prefix sum of its chunk counts)
    int* chunk_seq;        // [S]   sequence owning each slot, -1 for unused slots
    int* long_list;        // [N+1] short_path: ids of the sequences longer than kShortLen, then their count
    uint16_t* w;           // [8][S*64][128] bf16   w = T diag(beta e^G) K
    float* u;              // [8][S][16][64][8] f32 u = beta v + (T - I) diag(beta) V, column-group major
    uint16_t* qp;          // [8][S*64][128] bf16   Q' = diag(e^G) Q - Aqk w  (output operand)
    uint16_t* oi;          // [8][S][16][64][8] bf16 oi = Aqk u (intra-chunk output), column-group major
    float* g4;             // [8][S*64][4]   f32    {G, e^G, beta, rk} (rk = 1 / |k| with the L2 norm, else 1)
    // Segmented route (seg_m > 0): each sequence's chunks are grouped into segments of seg_m
    // chunks; a segment's transition h_end = gamma h_start + D h_start + B (prefill_seg.cu).
    int seg_m;             // chunks per segment (0: the single-pass scan kernels)
    int SS;                // segment slots in the workspace (>= sum over sequences of ceil(chunks / seg_m))
    uint16_t* seg_D;       // [8][SS][128][128] bf16  D = transition - gamma I  (row = output k index)
    float* seg_B;          // [8][SS][16][128][8] f32 B (state the segment builds from zero), column-group major
    float* seg_gamma;      // [8][SS] f32           product of the segment's chunk decays
    uint16_t* seg_hb;      // [8][SS][128 K][128 V] bf16  state at the segment start (output operand)
    uint16_t* qpp;         // [8][S*64][128] bf16   Q'' = Q' Phi (Phi: transition from the segment start)
    uint16_t* oipp;        // [8][S*64][128] bf16   oi'' = oi + Q' beta  (beta: state built from zero)
};

// Byte offsets of the workspace regions for N sequences and T tokens.
struct PrefillLayout {
    int S, SS, seg_m;
    size_t off_status, off_base, off_seq, off_long, off_w, off_u, off_qp, off_oi, off_g4;
    size_t off_segD, off_segB, off_segG, off_seghb, off_qpp, off_oipp, total;
};

// GDN_OK when the current device is compute capability 10.0 (B200), else a GDN_ERR_* code.
int check_device();
int launch_decode(const DecodeArgs& p, int variant, cudaStream_t stream);
int launch_prefill(const PrefillArgs& p, int bv, cudaStream_t stream);
// Slots: one per 64-token chunk of each sequence.  sum_n ceil(len_n / 64) <= T/64 + N, and
// every chunk holds at least one token, so min(T/64 + N, T) slots always suffice.
__host__ __device__ constexpr size_t prefill_up256(size_t x) { return (x + 255) & ~(size_t)255; }
// Chunks per segment of the segmented route for a call of N sequences and T tokens, or 0 for
// the single-pass scan.  A function of (N, T, HV) only, so the workspace size is known before
// the call.  Few sequences of many chunks: the chain of one sequence is the critical path, and
// splitting it into segments whose transitions are built in parallel shortens it.  The segment
// length is the shortest that keeps the local-transition grid (two CTAs per segment and v-head)
// within one wave of 148 SMs, but not so short that the chain over segments outgrows the local
// chains: a local chunk step costs about three chain steps (B200: ~5.4 K vs ~1.8 K cycles), so
// m^2 >= chunks / 3 per sequence.  The second bound only binds with few v-heads per call (a
// sequence split over GPUs by v-head); with 8 v-heads the one-wave bound is the larger.
__host__ __device__ constexpr int prefill_seg_m(int N, int T, int HV) {
    if (N < 1 || N > 32 || HV < 1 || T < 512 * N) return 0;  // N <= kSmallN; >= 8 chunks per sequence on average
    const long long nc = ((long long)T + 63) / 64;
    int m_bal = 2;
    while (3LL * m_bal * m_bal < nc / N) ++m_bal;
    for (int m = m_bal; m <= 64; ++m) {
        const long long segs = (nc + m - 1) / m + (N - 1);  // bound on sum_n ceil(nc_n / m)
        if (segs * 2 * HV <= 148) return m;
    }
    return 0;
}
// Whether a call takes the segmented route by default (it still needs prefill_seg_m > 0).
// Measured on B200 (segmented / single-pass scan): one sequence of 8192 tokens 127 / 157 us,
// 4096 76 / 85 us, 3072 68 / 71 us, 2048 49 / 48 us; two sequences of 4096 even (129 / 128 us),
// of 2048 78 / 72 us; four of 2048 150 / 116 us.  So one sequence of at least 3072 tokens, or
// sequences averaging at least 6144.
__host__ __device__ constexpr bool prefill_seg_default(int N, int T) {
    return N >= 1 && (T >= 6144LL * N || (N == 1 && T >= 3072));
}
__host__ __device__ constexpr PrefillLayout prefill_layout(int N, int T, int HV = 8) {
    PrefillLayout L{};
    long long S = (long long)T / 64 + N;
    if (S > T) S = T;
    if (S < 1) S = 1;
    L.S = (int)S;
    const size_t rows = (size_t)S * 64;
    size_t o = 0;
    L.off_status = o;
    o = prefill_up256(o + 16);
    L.off_base = o;
    o = prefill_up256(o + sizeof(int) * ((size_t)N + 1));
    L.off_seq = o;
    o = prefill_up256(o + sizeof(int) * (size_t)S);
    L.off_long = o;
    o = prefill_up256(o + sizeof(int) * ((size_t)N + 1));
    L.off_w = o;
    o = prefill_up256(o + (size_t)HV * rows * 128 * 2);
    L.off_u = o;
    o = prefill_up256(o + (size_t)HV * rows * 128 * 4);
    L.off_qp = o;
    o = prefill_up256(o + (size_t)HV * rows * 128 * 2);
    L.off_oi = o;
    o = prefill_up256(o + (size_t)HV * rows * 128 * 2);
    L.off_g4 = o;
    o = prefill_up256(o + (size_t)HV * rows * 4 * 4);
    L.seg_m = prefill_seg_m(N, T, HV);
    L.SS = 0;
    L.off_segD = L.off_segB = L.off_segG = L.off_seghb = L.off_qpp = L.off_oipp = o;
    if (L.seg_m > 0) {
        long long SS = (long long)S / L.seg_m + N;
        if (SS > S) SS = S;
        L.SS = (int)SS;
        const size_t segs = (size_t)HV * (size_t)SS;
        L.off_segD = o;
        o = prefill_up256(o + segs * 128 * 128 * 2);
        L.off_segB = o;
        o = prefill_up256(o + segs * 128 * 128 * 4);
        L.off_segG = o;
        o = prefill_up256(o + segs * 4);
        L.off_seghb = o;
        o = prefill_up256(o + segs * 128 * 128 * 2);
        L.off_qpp = o;
        o = prefill_up256(o + (size_t)HV * rows * 128 * 2);
        L.off_oipp = o;
        o = prefill_up256(o + (size_t)HV * rows * 128 * 2);
    }
    L.total = o;
    return L;
}
int prefill_scan_bv(int N, int HV);

}  // namespace gdn
