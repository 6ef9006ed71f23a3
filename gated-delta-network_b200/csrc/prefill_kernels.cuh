// prefill_kernels.cuh -- pieces shared by the three prefill translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

namespace gdn {

// TMA tensor maps of one prefill call (kernel parameters, 128 B each).
struct PrefillMaps {
    CUtensorMap q;    // (128 col, 4 head, T token) bf16, box 64 x 1 x 64, SWIZZLE_128B
    CUtensorMap k;    // same
    CUtensorMap v;    // (128, 8, T) bf16, box 64 x 1 x 64, SWIZZLE_128B
    CUtensorMap a;    // (8 head, T token) bf16, box 8 x 64, no swizzle
    CUtensorMap b;    // same
    CUtensorMap w;    // (128 col, S*64 row, 8 head) bf16, box 64 x 64 x 1, SWIZZLE_128B
    CUtensorMap qp;   // (128, S*64, 8) bf16, box 64 x 64 x 1, SWIZZLE_128B
    // segmented route only
    CUtensorMap qpp;  // Q''  (128, S*64, 8) bf16, box 64 x 64 x 1, SWIZZLE_128B
    CUtensorMap oipp; // oi'' same
    CUtensorMap segD; // D    (128, SS*128, 8) bf16, box 64 x 128 x 1, SWIZZLE_128B
    CUtensorMap seghb;// h_s  (128, SS*128, 8) bf16, box 64 x 128 x 1, SWIZZLE_128B
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

// Up to this many sequences the prep and scan kernels derive their chunk slots from
// cu_seqlens directly (one warp, one load per lane); above it a one-CTA table kernel computes
// chunk_base / chunk_seq once per call.
constexpr int kSmallN = 32;

// Sequences of at most this many tokens take the one-chunk short-sequence kernel whenever it is
// launched (PrefillArgs::short_path): a single partial chunk done in one CTA per (sequence,
// v-head), where the chunked path would spend two launches and a workspace round trip on it.
constexpr int kShortLen = 32;

// Tokens outside [cu[0], cu[N]) belong to no sequence: their output rows are zero, as the
// reference zero-initialises the whole output (reference/gdn_prefill_ref.py:49-51).  One CTA of
// each call runs this (`tid` of `nthreads`).
__device__ __forceinline__ void zero_unowned_tokens(const PrefillArgs& p, int tid, int nthreads) {
    if (p.T <= 0) return;
    int lo, tmp, hi;
    seq_bounds(p.cu, p.cu64, 0, p.T, lo, tmp);
    seq_bounds(p.cu, p.cu64, p.N - 1, p.T, tmp, hi);
    hi = max(hi, lo);
    const size_t row_words = (size_t)p.HV * kD / 8;
    uint4* o4 = reinterpret_cast<uint4*>(p.out);
    for (size_t idx = tid; idx < (size_t)lo * row_words; idx += nthreads) o4[idx] = make_uint4(0, 0, 0, 0);
    for (size_t idx = (size_t)hi * row_words + tid; idx < (size_t)p.T * row_words; idx += nthreads)
        o4[idx] = make_uint4(0, 0, 0, 0);
}

__device__ __forceinline__ int seq_nchunks(const PrefillArgs& p, int i) {
    int s, e;
    seq_bounds(p.cu, p.cu64, i, p.T, s, e);
    return (e - s + kChunk - 1) / kChunk;
}

// Warp-wide, N <= 32: first slot of sequence `n` (chunk_base[n]) and the sequence owning
// `slot` (-1 if none, or if slot < 0).  Every lane returns the same values.
__device__ __forceinline__ void warp_chunk_lookup(const PrefillArgs& p, int n, int slot, int* base_out, int* seq_out) {
    const int lane = threadIdx.x & 31;
    const int nc = lane < p.N ? seq_nchunks(p, lane) : 0;
    int x = nc;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, off);
        if (lane >= off) x += y;
    }
    const int excl = x - nc;
    const int total = __shfl_sync(0xffffffffu, x, 31);
    *base_out = n >= p.N ? total : __shfl_sync(0xffffffffu, excl, n & 31);
    const unsigned owner = __ballot_sync(0xffffffffu, lane < p.N && nc > 0 && slot >= excl && slot < excl + nc);
    *seq_out = owner ? __ffs(owner) - 1 : -1;
}

// Warp-wide, N <= 32: the sequence with the r-th largest chunk count (ties by index).  The scan
// maps its CTA rows through this so that the longest sequences -- the critical path of a varlen
// batch -- are scheduled first.  Every lane returns the same value.
__device__ __forceinline__ int warp_seq_by_rank(const PrefillArgs& p, int r) {
    const int lane = threadIdx.x & 31;
    const int nc = lane < p.N ? seq_nchunks(p, lane) : -1;
    int rank = 0;
    for (int j = 0; j < p.N; ++j) {
        const int ncj = __shfl_sync(0xffffffffu, nc, j);
        rank += (ncj > nc || (ncj == nc && j < lane)) ? 1 : 0;
    }
    const unsigned hit = __ballot_sync(0xffffffffu, lane < p.N && rank == r);
    return hit ? __ffs(hit) - 1 : r;
}

// Chunks of one sequence that fit the workspace from its first slot.  cu_seqlens that is not
// non-decreasing (overlapping sequences) can claim more chunks in total than the S slots hold;
// the excess is skipped and reported (status word 0), so no workspace access leaves the buffer.
__device__ __forceinline__ int clamp_chunks(const PrefillArgs& p, int slot0, int nchunks, bool report) {
    const int room = p.S - slot0;
    if (nchunks <= room) return nchunks;
    if (report) atomicCAS(p.status, 0, kErrBadSeqlens);
    return room > 0 ? room : 0;
}

bool build_prefill_maps(const PrefillArgs& p, PrefillMaps* m);

// Workspace element offset of column group cg (8 state columns) of chunk slot `slot`, v-head hv,
// in the column-group-major u / oi regions: one group is a contiguous [64 rows][8] block, so a
// scan CTA's slice of BV columns is one contiguous bulk copy.
__host__ __device__ __forceinline__ size_t cg_off(int hv, int S, int slot, int cg) {
    return (((size_t)hv * S + slot) * 16 + cg) * 64 * 8;
}
int launch_prefill_prep(const PrefillArgs& p, const PrefillMaps& maps, cudaStream_t stream);
int launch_prefill_scan(const PrefillArgs& p, const PrefillMaps& maps, int bv, cudaStream_t stream);
int launch_prefill_scan_tc(const PrefillArgs& p, const PrefillMaps& maps, cudaStream_t stream);
int launch_prefill_seg(const PrefillArgs& p, const PrefillMaps& maps, cudaStream_t stream);
int launch_prefill_short(const PrefillArgs& p, cudaStream_t stream);
int launch_prefill_short_rec(const PrefillArgs& p, cudaStream_t stream);

}  // namespace gdn
