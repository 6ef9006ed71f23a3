// prefill_host.cu -- workspace layout, chunk table kernel, TMA tensor maps and the launch
// sequence of the chunked prefill (table -> prep -> scan), all on the caller's stream.
#include <algorithm>

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.cuh"
#include "prefill_kernels.cuh"

namespace gdn {

int prefill_scan_bv(int N, int HV) {
    // (128 / BV) * N * HV CTAs, one per SM.  Few (sequence, v-head) pairs: the mma.sync scan with
    // the finest slices that still fit one wave of 148 SMs (the chain of one sequence is the
    // critical path, and its per-chunk step is shortest there).  More pairs: the tcgen05 scan
    // with 64-column slices (returned as 64), whose per-chunk step is longer but covers 2-8x the
    // columns, so it wins once the scan is bound by throughput (measured on B200: 4 x 2048
    // tokens break even, 8 x 1024 is 1.6x and 64 x 4096 1.9x faster than 32-column slices).
    if (N * HV * (kD / 8) <= 148) return 8;
    if (N * HV * (kD / 16) <= 148) return 16;
    return 64;
}

// ---- chunk table ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) gdn_prefill_table_kernel(PrefillArgs p) {
    __shared__ long long s_warp[32];
    __shared__ int s_total;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    pdl_wait();
    pdl_trigger();
    if (tid == 0) {
        p.status[0] = 0;
        p.status[1] = 0;  // work-item counters of the tcgen05 scan and of the prep kernel
        p.status[2] = 0;  // (short path)
    }
    // Chunk slots go to the sequences the chunked kernels process: all of them, or with the
    // short path only those longer than kShortLen, which are also listed in order in long_list.
    int running = 0, running_long = 0;
    for (int base = 0; base < p.N; base += 1024) {
        const int i = base + tid;
        int nc = 0, lg = 0;
        if (i < p.N) {
            int s, e;
            seq_bounds(p.cu, p.cu64, i, p.T, s, e);
            lg = (!p.short_path || e - s > kShortLen) ? 1 : 0;
            nc = lg ? (e - s + kChunk - 1) / kChunk : 0;
        }
        // block-wide exclusive prefix sums of nc and lg (packed: nc < 2^20 per sequence here)
        const long long packed = ((long long)nc << 32) | (long long)lg;
        long long x = packed;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const long long y = __shfl_up_sync(0xffffffffu, x, off);
            if (lane >= off) x += y;
        }
        if (lane == 31) s_warp[warp] = x;
        __syncthreads();
        long long wpre = 0, total = 0;
        for (int w = 0; w < 32; ++w) {
            const long long c = s_warp[w];
            if (w < warp) wpre += c;
            total += c;
        }
        const long long excl = wpre + x - packed;
        if (i < p.N) {
            p.chunk_base[i] = running + (int)(excl >> 32);
            if (p.short_path && lg) p.long_list[running_long + (int)(excl & 0xffffffffll)] = i;
        }
        running += (int)(total >> 32);
        running_long += (int)(total & 0xffffffffll);
        __syncthreads();
    }
    if (tid == 0) {
        p.chunk_base[p.N] = running;
        if (p.short_path) p.long_list[p.N] = running_long;
        s_total = running;
    }
    __syncthreads();
    const int total = s_total;
    for (int i = tid; i < p.N; i += 1024) {
        const int b0 = p.chunk_base[i], nc = p.chunk_base[i + 1] - b0;
        for (int c = 0; c < nc && b0 + c < p.S; ++c) p.chunk_seq[b0 + c] = i;
    }
    for (int s = total + tid; s < p.S; s += 1024) p.chunk_seq[s] = -1;
}

// ---- TMA tensor maps -----------------------------------------------------------------------
namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn g_encode = nullptr;  // resolved once; concurrent resolution stores the same pointer

EncodeTiledFn encode_fn() {
    if (g_encode == nullptr) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return nullptr;
        g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
    return g_encode;
}

bool map3d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, uint64_t d0, uint64_t d1, uint64_t d2,
           uint64_t stride1, uint64_t stride2, uint32_t b0, uint32_t b1, uint32_t b2, CUtensorMapSwizzle sw) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[3] = {d0, d1, d2};
    const cuuint64_t strides[2] = {stride1, stride2};
    const cuuint32_t box[3] = {b0, b1, b2};
    const cuuint32_t estr[3] = {1, 1, 1};
    return enc(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
               CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool map2d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, uint64_t d0, uint64_t d1, uint64_t stride1,
           uint32_t b0, uint32_t b1) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {d0, d1};
    const cuuint64_t strides[1] = {stride1};
    const cuuint32_t box[2] = {b0, b1};
    const cuuint32_t estr[2] = {1, 1};
    return enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool build_prefill_maps(const PrefillArgs& p, PrefillMaps* m) {
    const uint64_t T = (uint64_t)p.T, R = (uint64_t)p.S * kChunk;
    const auto BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const auto SW = CU_TENSOR_MAP_SWIZZLE_128B;
    // Inputs: [T][heads][128] bf16 as (col, head, token); one box = 64 columns x 1 head x 64 tokens.
    const uint64_t H = (uint64_t)p.H, HV = (uint64_t)p.HV;
    bool ok = map3d(&m->q, p.q, BF, 128, H, T, 256, 256 * H, 64, 1, 64, SW);
    ok = ok && map3d(&m->k, p.k, BF, 128, H, T, 256, 256 * H, 64, 1, 64, SW);
    ok = ok && map3d(&m->v, p.v, BF, 128, HV, T, 256, 256 * HV, 64, 1, 64, SW);
    // Gates: [T][HV] bf16 as (head, token); one box = 8 heads (the group of v-head hv) of 64 tokens (1 KB).
    // A tensor map needs 16-byte row strides, so with HV not a multiple of 8 the prep reads the
    // gates with plain loads and no map is built.
    if (p.gates_tma) {
        ok = ok && map2d(&m->a, p.a, BF, HV, T, 2 * HV, 8, 64);
        ok = ok && map2d(&m->b, p.b, BF, HV, T, 2 * HV, 8, 64);
    }
    // Workspace: [8][R][cols] as (col, row, head); one box = one 64-row chunk slot.
    ok = ok && map3d(&m->w, p.w, BF, 128, R, HV, 256, R * 256, 64, 64, 1, SW);
    ok = ok && map3d(&m->qp, p.qp, BF, 128, R, HV, 256, R * 256, 64, 64, 1, SW);
    if (p.seg_m > 0) {
        const uint64_t RS = (uint64_t)p.SS * 128;
        ok = ok && map3d(&m->qpp, p.qpp, BF, 128, R, HV, 256, R * 256, 64, 64, 1, SW);
        ok = ok && map3d(&m->oipp, p.oipp, BF, 128, R, HV, 256, R * 256, 64, 64, 1, SW);
        ok = ok && map3d(&m->segD, p.seg_D, BF, 128, RS, HV, 256, RS * 256, 64, 128, 1, SW);
        ok = ok && map3d(&m->seghb, p.seg_hb, BF, 128, RS, HV, 256, RS * 256, 64, 128, 1, SW);
    }
    return ok;
}

// Slice width 64 selects the tcgen05 scan (prefill_scan_tc.cu), 8 / 16 / 32 the mma.sync scan.
static int launch_scan(const PrefillArgs& p, const PrefillMaps& maps, int bv, cudaStream_t stream) {
    return bv == 64 ? launch_prefill_scan_tc(p, maps, stream) : launch_prefill_scan(p, maps, bv, stream);
}

int launch_prefill(const PrefillArgs& args, int bv, cudaStream_t stream) {
    if (args.N <= 0) return 0;
    PrefillArgs p = args;
    p.gates_tma = p.HV % 8 == 0 ? 1 : 0;
    // Short sequences (0..kShortLen tokens) take a dedicated one-launch kernel in batches of many
    // sequences, where its throughput wins; with few sequences the chunked kernels process the
    // short ones off the critical path of the longest sequence, and a separate launch would only
    // add latency.  When T <= kShortLen every sequence is short, so the short kernel is the
    // call's only launch (no chunk table, prep or scan).
    p.only_short = (!p.no_short && p.T <= kShortLen) ? 1 : 0;
    p.short_path = (!p.no_short && (p.N > kSmallN || p.only_short)) ? 1 : 0;
    // Each sequence the chunked kernels see under the short path has more than kShortLen tokens,
    // so at most T / (kShortLen + 1) of them exist: the scan and prep grids are sized by that
    // bound instead of N (no CTA launches just to find its sequence is someone else's).
    p.rows = p.short_path ? (int)std::max(1, std::min(p.N, p.T / (kShortLen + 1))) : p.N;
    // Short sequences: the one-chunk tensor-core kernel, or for batches averaging at most 10 tokens
    // per sequence the token recurrence, which is cheaper for a handful of tokens (measured on
    // B200: 4000 x 6 tokens 1.14 ms vs 1.69 ms; 1000 x 16 tokens 0.61 ms vs 0.45 ms).  Both also
    // own the zero-length sequences.
    if (p.short_path &&
        ((p.T <= 10 * p.N ? launch_prefill_short_rec(p, stream) : launch_prefill_short(p, stream)) != 0))
        return -1;
    if (p.only_short) return 0;
    if (!p.small_n && launch_pdl(gdn_prefill_table_kernel, dim3(1), dim3(1024), 0, stream, p) != cudaSuccess)
        return -1;
    if (p.T > 0) {
        PrefillMaps maps;
        if (!build_prefill_maps(p, &maps)) return -3;
        if (launch_prefill_prep(p, maps, stream) != 0) return -1;
        if (p.seg_m > 0) {
            if (launch_prefill_seg(p, maps, stream) != 0) return -1;
        } else if (launch_scan(p, maps, bv, stream) != 0) {
            return -1;
        }
    } else {
        if (launch_scan(p, PrefillMaps{}, bv, stream) != 0) return -1;
    }
    return 0;
}

}  // namespace gdn
