// prefill_seg.cu -- segmented serial half of the chunked prefill (sm_100a), for calls of few long
// sequences, where the chain of one sequence's chunks is the critical path.
//
// The single-pass scans (prefill_scan.cu, prefill_scan_tc.cu) walk all chunks of a sequence in
// order: per chunk h' = A_c h + B_c with A_c = e^{G_L} I - K~^T W and B_c = K~^T u (K~ = the
// decay-weighted keys, W / u from the prep), the recurrence of
// solutions/gdn_prefill_qk4_v8_d128_k_last/solution/triton/fla_kernels.py:503-645.  Here each
// sequence is cut into segments of m chunks and the chain is rebuilt in three launches:
//
//   1. gdn_prefill_seg_local_kernel, one CTA per (segment, v-head, half), all in parallel:
//      runs the chunk recurrence over its segment on a 256-column state X = [beta | Phi] started
//      from [0 | I] (half 0 carries beta, the state the segment builds from zero, half 1 Phi, the
//      product of the chunk transitions so far).  Per chunk j it also forms the output operands
//      of every chunk against the segment's start state h_s:
//          o_j = scale (Q'_j h_j + oi_j),  h_j = Phi_j h_s + beta_j
//              = scale (Q''_j h_s + oi''_j + oi_j),  Q''_j = Q'_j Phi_j,  oi''_j = Q'_j beta_j.
//      At the end it stores the segment transition h_{s+1} = gamma h_s + D h_s + B with
//      B = beta_end, gamma = product of e^{G_L}, D = Phi_end - gamma I.
//   2. gdn_prefill_seg_chain_kernel, one CTA per (8 state columns, sequence, v-head): the short
//      serial chain over segments, h_{s+1} = gamma h_s + D h_s + B; it records each h_s (bf16,
//      the output operand) and writes the final state.
//   3. gdn_prefill_seg_out_kernel, persistent, one tcgen05 MMA per (2 chunks of a segment, v-head):
//      o_j = scale (Q''_j h_s + oi''_j + oi_j), oi_j = Aqk u from the prep.
//
// Per chunk the local kernel does what the single-pass scan does (two dependent products), on a
// state twice as wide, but every segment runs at once: the serial work per sequence drops from
// all its chunks to one segment plus one cheap step per segment.  Precision follows the scans:
// bf16 operands W, Q', K, bf16 copies of X and h as MMA operands, the decayed vn split into bf16
// hi + lo, fp32 state and accumulation; D and the Q'' / oi'' operands are stored in bf16.
#include <algorithm>

#include "prefill_kernels.cuh"
#include "sm100.cuh"
#include "dbg.cuh"

GDN_DBG_READER(gdn_debug_read_seg)

namespace gdn {

namespace segk {
constexpr int kThreads = 512;  // 16 math warps (four per TMEM lane quarter); thread kIssuer also issues the TMA
constexpr int kMath = 512;
constexpr int kIssuer = 96;    // warp 3, lane 0: an output-row warp, off the chain's critical path
constexpr int kCW = 32;        // state columns per math thread
constexpr int kStages = 2;
constexpr uint32_t kOffWQ = 0;          // [W0 | Q'0 | W1 | Q'1], 8 KB each; after MMA_P: output staging
constexpr uint32_t kOffK = 32768;       // k tile, 2 atoms of 64 tokens x 128 B
constexpr uint32_t kOffG = 49152;       // [64][4] f32 {G, e^G, beta, rk}
constexpr uint32_t kOffU = 50176;       // u f32 [16 cg][64][8] (half 0 only)
constexpr uint32_t kStage = 82944;      // 81 KB (1024-aligned)
constexpr uint32_t kTxTiles = 6 * 8192 + 1024;
constexpr uint32_t kOffX = kStages * kStage;   // X bf16, 2 column blocks of [128 rows][128 B], SW128;
                                               // between MMA_P and MMA_U: vn hi / lo [2][64][128 B] each
constexpr uint32_t kOffBar = kOffX + 32768;    // full[2], (unused)[2], mma_p, mma_u
constexpr uint32_t kSmemUsed = kOffBar + 8 * 6 + 16;
constexpr uint32_t kSmem = kSmemUsed + 1024;
constexpr uint32_t kTmemCols = 256;            // P: 0-127, D: 128-255
static_assert(kSmem <= 227 * 1024, "segment kernel shared memory");
}  // namespace segk

// Where a segment slot, chunk slot or sequence sits in the call (warp-wide, N <= 32; every lane
// returns the same values): sequence n, its first chunk slot, its first segment slot, its chunk
// count.  Chunk slots follow sequence order (prefix sums of ceil(len / 64)), and so do segment
// slots (prefix sums of ceil(chunks / m)).
struct SegSeq {
    int n, cbase, sbase, nc;
};
enum { kBySeg = 0, kByChunk = 1, kBySeq = 2 };
__device__ __forceinline__ SegSeq warp_seg_seq(const PrefillArgs& p, int kind, int key) {
    const int lane = threadIdx.x & 31;
    const int nc = lane < p.N ? seq_nchunks(p, lane) : 0;
    const int ns = (nc + p.seg_m - 1) / p.seg_m;
    int xc = nc, xs = ns;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int yc = __shfl_up_sync(0xffffffffu, xc, off);
        const int ys = __shfl_up_sync(0xffffffffu, xs, off);
        if (lane >= off) {
            xc += yc;
            xs += ys;
        }
    }
    const int ec = xc - nc, es = xs - ns;  // exclusive prefix sums
    int n;
    if (kind == kBySeq) {
        n = key;
    } else {
        const bool mine = kind == kBySeg ? (lane < p.N && key >= es && key < es + ns)
                                         : (lane < p.N && key >= ec && key < ec + nc);
        const unsigned owner = __ballot_sync(0xffffffffu, mine);
        n = owner ? __ffs(owner) - 1 : -1;
    }
    SegSeq r;
    r.n = n;
    const int src = n >= 0 ? n : 0;
    r.cbase = __shfl_sync(0xffffffffu, ec, src);
    r.sbase = __shfl_sync(0xffffffffu, es, src);
    r.nc = __shfl_sync(0xffffffffu, nc, src);
    return r;
}

// bf16 copy of X row r, columns cb .. cb + kCW - 1: MN-major SW128 B operand of MMA_P (column
// block bk, 16-byte chunks j0 ..)
#define GDN_SEG_WRITE_XB()                                                                                     \
    do {                                                                                                      \
        unsigned char* row_ = sm + kOffX + bk * 16384 + r * 128;                                               \
        _Pragma("unroll") for (int jj = 0; jj < kCW / 8; ++jj)                                                \
            *reinterpret_cast<uint4*>(row_ + (((j0 + jj) ^ (r & 7)) << 4)) =                                   \
                make_uint4(pack_bf16x2(x[8 * jj], x[8 * jj + 1]), pack_bf16x2(x[8 * jj + 2], x[8 * jj + 3]),   \
                           pack_bf16x2(x[8 * jj + 4], x[8 * jj + 5]), pack_bf16x2(x[8 * jj + 6], x[8 * jj + 7])); \
    } while (0)

// ------------------------------------------------------------------------------------------
// 1. local transitions
// ------------------------------------------------------------------------------------------
// 512 threads, 16 warps: the whole 64 K-entry register file gives 128 registers per thread.  A
// separate producer warp (17 warps, granted as 20) would cap them at 96 and spill.
__global__ void __launch_bounds__(segk::kThreads, 1)
    gdn_prefill_seg_local_kernel(PrefillArgs p, const __grid_constant__ PrefillMaps maps) {
    using namespace segk;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(sm);
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + kOffBar);
    uint64_t* bar_p = full + 2 * kStages;
    uint64_t* bar_u = bar_p + 1;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bar_u + 1);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bar_u + 1) + 1;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ss = blockIdx.x, hv = blockIdx.y, half = blockIdx.z;  // half 0: beta (with u), 1: Phi
    const int hq = hv / (p.HV / p.H);
    if (tid == kIssuer) {
        tma_prefetch_desc(&maps.w);
        tma_prefetch_desc(&maps.qp);
        tma_prefetch_desc(&maps.k);
        tma_prefetch_desc(half ? &maps.qpp : &maps.oipp);
    }
    // Set-up that reads no prep output runs before the grid-dependency wait, overlapping the prep's
    // tail: the segment lookup (cu_seqlens was complete before the prep started its work), the
    // barriers and the TMEM allocation (no prep CTA shares an SM with this 200 KB CTA).
    const SegSeq sq = warp_seg_seq(p, kBySeg, ss);
    if (sq.n < 0 || ss >= p.SS) return;  // a slot past the last segment (uniform across the CTA)
    int bos, eos;
    seq_bounds(p.cu, p.cu64, sq.n, p.T, bos, eos);
    const int seg = ss - sq.sbase;
    const int c0 = seg * p.seg_m;
    int nch = min(p.seg_m, sq.nc - c0);
    nch = max(0, min(nch, p.S - (sq.cbase + c0)));  // only a cu_seqlens that is not non-decreasing trims it
    if (nch <= 0) return;
    const int slot0 = sq.cbase + c0;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) mbar_init(full + s, 1);
        mbar_init(bar_p, 1);
        mbar_init(bar_u, 1);
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 0) tmem_alloc(tslot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    pdl_wait();  // the workspace comes from the prep kernel
    pdl_trigger();

    // Chunk c's W, Q', K tiles, gates and (half 0) u go to stage c % 2, issued by thread kIssuer:
    // chunks 0 and 1 here, chunk c + 1 at the top of chunk c once the barrier there shows that every
    // thread is done with chunk c - 1, the stage's previous contents (its output tile read by the
    // TMA store included).  n_issued counts the chunks issued (kIssuer's own count).
    int n_issued = 0;
    auto issue = [&](int c) {
        unsigned char* st = sm + (c % kStages) * kStage;
        uint64_t* bar = full + (c % kStages);
        const int slot = slot0 + c, wr = slot * kChunk, t0 = bos + (c0 + c) * kChunk;
        mbar_arrive_expect_tx(bar, kTxTiles + (half == 0 ? 32768u : 0u));
        tma_load_3d(st + kOffWQ, &maps.w, 0, wr, hv, bar);
        tma_load_3d(st + kOffWQ + 8192, &maps.qp, 0, wr, hv, bar);
        tma_load_3d(st + kOffWQ + 16384, &maps.w, 64, wr, hv, bar);
        tma_load_3d(st + kOffWQ + 24576, &maps.qp, 64, wr, hv, bar);
        tma_load_3d(st + kOffK, &maps.k, 0, hq, t0, bar);
        tma_load_3d(st + kOffK + 8192, &maps.k, 64, hq, t0, bar);
        bulk_load(st + kOffG, p.g4 + ((size_t)hv * p.S + slot) * kChunk * 4, 1024, bar);
        if (half == 0) bulk_load(st + kOffU, p.u + cg_off(hv, p.S, slot, 0), 32768, bar);
        n_issued = c + 1;
    };
    if (tid == kIssuer)
        for (int c = 0; c < min(nch, kStages); ++c) issue(c);
    {
        // ---- math warps: thread (r, cq) = TMEM lane r, state columns cb = kCW cq .. cb + kCW - 1 ----
        // (warps w, w + 4, w + 8, w + 12 share TMEM lane quarter w and split its columns)
        const int r = lane + 32 * (warp & 3), cq = warp >> 2;
        const int cb = kCW * cq, bk = cb >> 6, j0 = (cb & 63) >> 3;
        const uint32_t tl = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)cb;
        float x[kCW];  // X row r (K index), columns cb + j
#pragma unroll
        for (int j = 0; j < kCW; ++j) x[j] = (half == 1 && r == cb + j) ? 1.f : 0.f;
        GDN_SEG_WRITE_XB();
        constexpr uint32_t idesc_p = umma_idesc_bf16(128, 128, false, true);
        constexpr uint32_t idesc_u = umma_idesc_bf16(128, 128, true, true);
        const CUtensorMap* omap = half ? &maps.qpp : &maps.oipp;
        float gamma = 1.f;
        const bool dbg = true;
        long long tp = clock64();
        (void)dbg;
        int c = 0;
        for (; c < nch; ++c) {
            const uint32_t ph = (uint32_t)(c & 1);
            if (!mbar_wait(full + (c % kStages), (uint32_t)((c / kStages) & 1), p.status, kErrScanTmaTimeout))
                *abort_flag = 1;
            GDN_PH_ACC(dbg, 0, tp);
            fence_async_smem();  // this thread's X copy (generic stores) -> the tensor core
            tc_fence_before();
            named_bar_sync(1, kMath);
            GDN_PH_ACC(dbg, 1, tp);
            if (*abort_flag) break;  // written only before this barrier
            if (tid == kIssuer && c >= 1 && c + 1 < nch) issue(c + 1);
            tc_fence_after();
            const unsigned char* st = sm + (c % kStages) * kStage;
            const uint32_t sst = sbase + (uint32_t)(c % kStages) * kStage;
            const float* G4 = reinterpret_cast<const float*>(st + kOffG);
            const int slot = slot0 + c;
            const int t0 = bos + (c0 + c) * kChunk;
            const int L = min(kChunk, eos - t0);
            const float GL = G4[(L - 1) * 4];
            // MMA_P: [W; Q'] (128 x 128, K-major) x X (128 x 128, MN-major) -> TMEM columns 0-127.
            // The beta half starts from X = 0: its first product is zero and is not formed.
            const bool zeroP = half == 0 && c == 0;
            const uint32_t php = (uint32_t)((c - (half == 0 ? 1 : 0)) & 1);  // bar_p phase (one commit per product)
            if (tid == 0 && !zeroP) {
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    umma_bf16(tmem,
                              umma_desc_sw128(sst + kOffWQ + (uint32_t)(kk >> 2) * 16384u + (uint32_t)(kk & 3) * 32u, 16, 1024),
                              umma_desc_sw128(sbase + kOffX + 2048u * kk, 16384, 1024), idesc_p, kk > 0);
                umma_commit(bar_p);
            }
            bool ok = zeroP || mbar_wait(bar_p, php, p.status, kErrScanMmaTimeout);
            tc_fence_after();
            GDN_PH_ACC(dbg, 2, tp);
            if (r < 64) {
                // vn = ([u | 0] - W X) e^{G_L - G_r} / |k_r|  -> bf16 hi + lo, token row r
                bool okv = true;
                const float4 g4r = *reinterpret_cast<const float4*>(G4 + r * 4);  // {G, e^G, beta, rk}
                const float ed = __expf(GL - g4r.x) * g4r.w;
                const float* Us = reinterpret_cast<const float*>(st + kOffU);
                unsigned char* rh = sm + kOffX + bk * 8192 + r * 128;
                unsigned char* rl = rh + 16384;
                const int hA = (r >> 2) & 1;
#pragma unroll
                for (int blk = 0; blk < kCW / 16; ++blk) {
                    uint32_t d[16];
                    if (zeroP) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) d[j] = 0u;
                    } else {
                        tmem_ld16_async(tl + 16u * blk, d);
                        tmem_ld_wait();
                        tmem_regs_ready_n(d);
                    }
                    GDN_PH_ACC(dbg, 8 + 2 * (blk & 1), tp);
#pragma unroll
                    for (int q4 = 0; q4 < 2; ++q4) {
                        const int jj = 2 * blk + q4;  // 8-column group inside this thread's columns
                        float uu[8];
                        if (half == 0) {
                            const int cg = (cb >> 3) + jj;
                            const float4 x0 = *reinterpret_cast<const float4*>(Us + (cg * 64 + r) * 8 + 4 * hA);
                            const float4 x1 = *reinterpret_cast<const float4*>(Us + (cg * 64 + r) * 8 + 4 * (hA ^ 1));
                            const float4 ua = hA ? x1 : x0;
                            const float4 ub = hA ? x0 : x1;
                            uu[0] = ua.x; uu[1] = ua.y; uu[2] = ua.z; uu[3] = ua.w;
                            uu[4] = ub.x; uu[5] = ub.y; uu[6] = ub.z; uu[7] = ub.w;
                        } else {
#pragma unroll
                            for (int e = 0; e < 8; ++e) uu[e] = 0.f;
                        }
                        uint32_t hi[4], lo[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 v2 = mul2(sub2(make_float2(uu[2 * e], uu[2 * e + 1]),
                                                        make_float2(__uint_as_float(d[8 * q4 + 2 * e]),
                                                                    __uint_as_float(d[8 * q4 + 2 * e + 1]))),
                                                   make_float2(ed, ed));
                            hi[e] = pack_bf16x2(v2.x, v2.y);
                            const float2 r2 = sub2(v2, make_float2(__uint_as_float(hi[e] << 16),
                                                                   __uint_as_float(hi[e] & 0xffff0000u)));
                            lo[e] = pack_bf16x2(r2.x, r2.y);
                        }
                        *reinterpret_cast<uint4*>(rh + (((j0 + jj) ^ (r & 7)) << 4)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                        *reinterpret_cast<uint4*>(rl + (((j0 + jj) ^ (r & 7)) << 4)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                    }
                    GDN_PH_ACC(dbg, 9 + 2 * (blk & 1), tp);
                }
                // warps 0, 1, 4, 5 alone gate MMA_U
                GDN_PH_ACC(dbg, 3, tp);
                fence_async_smem();
                tc_fence_before();
                okv = named_bar_and(2, kMath / 2, ok && okv);
                tc_fence_after();
                GDN_PH_ACC(dbg, 4, tp);
                // MMA_U: K^T (128 x 64 tokens, MN-major) x (vn_hi + vn_lo) -> TMEM columns 128-255
                if (okv && tid == 0) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        umma_bf16(tmem + 128, umma_desc_sw128(sst + kOffK + 2048u * kk, 8192, 1024),
                                  umma_desc_sw128(sbase + kOffX + 2048u * kk, 8192, 1024), idesc_u, kk > 0);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        umma_bf16(tmem + 128, umma_desc_sw128(sst + kOffK + 2048u * kk, 8192, 1024),
                                  umma_desc_sw128(sbase + kOffX + 16384u + 2048u * kk, 8192, 1024), idesc_u, true);
                    umma_commit(bar_u);
                }
                ok = okv;
            } else {
                // output operand row m = r - 64: oi'' = Q' beta (half 0) or Q'' = Q' Phi (half 1),
                // staged SW128 in the stage's (consumed) W / Q' area, then one TMA store per 64 columns
                const int m = r - 64;
                unsigned char* orow = sm + (c % kStages) * kStage + kOffWQ + bk * 8192 + m * 128;
#pragma unroll
                for (int blk = 0; blk < kCW / 16; ++blk) {
                    uint32_t d[16];
                    if (zeroP) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) d[j] = 0u;
                    } else {
                        tmem_ld16_async(tl + 16u * blk, d);
                        tmem_ld_wait();
                        tmem_regs_ready_n(d);
                    }
#pragma unroll
                    for (int q4 = 0; q4 < 2; ++q4) {
                        const int jj = 2 * blk + q4;
                        uint32_t pk[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            pk[e] = pack_bf16x2(__uint_as_float(d[8 * q4 + 2 * e]), __uint_as_float(d[8 * q4 + 2 * e + 1]));
                        *reinterpret_cast<uint4*>(orow + (((j0 + jj) ^ (m & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                    }
                }
                fence_async_smem();
                named_bar_sync(3, kMath / 2);  // the output warps
                if (tid == 64) {         // warp 2, lane 0: store the 64 x 128 tile (two SW128 boxes)
                    unsigned char* ob = sm + (c % kStages) * kStage + kOffWQ;
                    tma_store_3d(omap, 0, slot * kChunk, hv, ob);
                    tma_store_3d(omap, 64, slot * kChunk, hv, ob + 8192);
                    tma_store_commit();
                }
            }
            // an MMA_U that was not issued (a wait gave up) also fails this bounded wait
            GDN_PH_ACC(dbg, 5, tp);
            if (ok) ok = mbar_wait(bar_u, ph, p.status, kErrScanMmaTimeout);
            tc_fence_after();
            GDN_PH_ACC(dbg, 6, tp);
            {
                const float eL = __expf(GL);
#pragma unroll
                for (int blk = 0; blk < kCW / 16; ++blk) {
                    uint32_t d[16];
                    tmem_ld16_async(tl + 128u + 16u * blk, d);
                    tmem_ld_wait();
                    tmem_regs_ready_n(d);
#pragma unroll
                    for (int j = 0; j < 16; j += 2) {
                        const float2 xn = fma2(make_float2(eL, eL), make_float2(x[16 * blk + j], x[16 * blk + j + 1]),
                                               make_float2(__uint_as_float(d[j]), __uint_as_float(d[j + 1])));
                        x[16 * blk + j] = xn.x;
                        x[16 * blk + j + 1] = xn.y;
                    }
                }
                gamma *= eL;
            }
            // the stage's operands are consumed (and its output tile read by the TMA store)
            if (tid == 64) tma_store_wait_read();
            if (!ok) *abort_flag = 1;
            GDN_SEG_WRITE_XB();
            GDN_PH_ACC(dbg, 7, tp);
        }
        if (c < nch) {
            // gave up: let copies already in flight land (bounded) before the CTA exits
            if (tid == kIssuer)
                for (int cc = c; cc < n_issued; ++cc)
                    mbar_wait(full + (cc % kStages), (uint32_t)((cc / kStages) & 1), nullptr, 0);
        } else {
            const size_t seg_i = (size_t)hv * p.SS + ss;
            if (half == 0) {
                // B = beta_end, column-group major [16][128][8] f32
                float* Bp = p.seg_B + seg_i * 128 * 128;
#pragma unroll
                for (int jj = 0; jj < kCW / 8; ++jj) {
                    float4* dst = reinterpret_cast<float4*>(Bp + (((cb >> 3) + jj) * 128 + r) * 8);
                    dst[0] = make_float4(x[8 * jj], x[8 * jj + 1], x[8 * jj + 2], x[8 * jj + 3]);
                    dst[1] = make_float4(x[8 * jj + 4], x[8 * jj + 5], x[8 * jj + 6], x[8 * jj + 7]);
                }
            } else {
                // D = Phi_end - gamma I, row-major [128][128] bf16 (row = output k index)
#pragma unroll
                for (int j = 0; j < kCW; ++j)
                    if (r == cb + j) x[j] -= gamma;
                uint4* dst = reinterpret_cast<uint4*>(p.seg_D + (seg_i * 128 + r) * 128 + cb);
#pragma unroll
                for (int jj = 0; jj < kCW / 8; ++jj)
                    dst[jj] = make_uint4(pack_bf16x2(x[8 * jj], x[8 * jj + 1]), pack_bf16x2(x[8 * jj + 2], x[8 * jj + 3]),
                                         pack_bf16x2(x[8 * jj + 4], x[8 * jj + 5]), pack_bf16x2(x[8 * jj + 6], x[8 * jj + 7]));
                if (tid == 0) p.seg_gamma[seg_i] = gamma;
            }
        }
        if (tid == 64) tma_store_wait_all();  // the operand stores are complete before the grid ends
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

// ------------------------------------------------------------------------------------------
// 2. chain over segments
// ------------------------------------------------------------------------------------------
namespace segc {
constexpr int BV = 8;                 // state columns per CTA
constexpr int kThreads = 288;         // 8 math warps (16 state rows each) + 1 TMA producer warp
constexpr int kMath = 256;
constexpr int kStages = 3;
constexpr int kHS = 8;                // bf16 row stride of the h copy
constexpr uint32_t kOffD = 0;         // D: 2 atoms of [128 rows][128 B], SW128
constexpr uint32_t kOffB = 32768;     // B slice [128][8] f32
constexpr uint32_t kStage = 32768 + 4096;
constexpr uint32_t kTx = 32768 + 4096;
constexpr uint32_t kOffHb = kStages * kStage;       // h bf16 [2][128][8]: step s reads copy s % 2
constexpr uint32_t kOffBar = kOffHb + 2 * 128 * kHS * 2;
constexpr uint32_t kSmemUsed = kOffBar + 16 * kStages + 16;
constexpr uint32_t kSmem = kSmemUsed + 1024;
}  // namespace segc

__global__ void __launch_bounds__(segc::kThreads, 1)
    gdn_prefill_seg_chain_kernel(PrefillArgs p, const __grid_constant__ PrefillMaps maps) {
    using namespace segc;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint16_t* Hb = reinterpret_cast<uint16_t*>(sm + kOffHb);
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + kOffBar);
    uint64_t* empty = full + kStages;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kStages);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int gq = lane >> 2, tq = lane & 3;
    const int v0 = blockIdx.x * BV, n = blockIdx.y, hv = blockIdx.z;
    if (warp == kMath / 32 && lane == 0) tma_prefetch_desc(&maps.segD);
    // Set-up that reads no output of the segment kernels runs before the grid-dependency wait, over
    // the local kernel's tail: the sequence lookup, the barriers and the initial state (inputs that
    // were complete before the prep started its work; no earlier kernel of this call writes them).
    const SegSeq sq = warp_seg_seq(p, kBySeq, n);
    int bos, eos;
    seq_bounds(p.cu, p.cu64, n, p.T, bos, eos);
    float* st_out = p.new_state + ((size_t)n * p.HV + hv) * kD * kD;
    if (eos - bos <= 0) {  // zero-length sequence: all-zero final state (reference/gdn_prefill_ref.py:52-54, 61-62)
        pdl_wait();
        pdl_trigger();
        for (int idx = tid; idx < BV * kD; idx += kThreads) st_out[(size_t)(v0 + idx / kD) * kD + idx % kD] = 0.f;
        return;
    }
    const int room = min(p.S - sq.cbase, sq.nc);  // chunks inside the workspace (all, for valid cu_seqlens)
    int nseg = room > 0 ? (room + p.seg_m - 1) / p.seg_m : 0;
    nseg = max(0, min(nseg, p.SS - sq.sbase));
    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, kMath / 32);
        }
        *abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();
    // math warp mw owns state rows 16 mw .. 16 mw + 15: h[e] = h[16 mw + gq + 8 (e >> 1)][2 tq + (e & 1)]
    const int mw = warp;
    float h[4];
    if (warp < kMath / 32) {
        const float* st_in = p.state ? p.state + ((size_t)n * p.HV + hv) * kD * kD : nullptr;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int row = 16 * mw + gq + 8 * (e >> 1), col = 2 * tq + (e & 1);
            h[e] = st_in ? st_in[(size_t)(v0 + col) * kD + row] : 0.f;
        }
    }
    pdl_wait();  // the segment transitions come from the local kernel
    pdl_trigger();
    if (warp == kMath / 32) {
        if (lane == 0) {
            for (int s = 0; s < nseg; ++s) {
                if (s >= kStages && !mbar_wait(empty + (s % kStages), (uint32_t)((s / kStages - 1) & 1), p.status,
                                               kErrScanTmaTimeout))
                    break;
                unsigned char* st = sm + (s % kStages) * kStage;
                uint64_t* bar = full + (s % kStages);
                const int row = (sq.sbase + s) * 128;
                mbar_arrive_expect_tx(bar, kTx);
                tma_load_3d(st + kOffD, &maps.segD, 0, row, hv, bar);
                tma_load_3d(st + kOffD + 16384, &maps.segD, 64, row, hv, bar);
                bulk_load(st + kOffB, p.seg_B + (((size_t)hv * p.SS + sq.sbase + s) * 16 + v0 / 8) * 128 * 8, 4096, bar);
            }
        }
        return;
    }
    // h_s (bf16) into copy s % 2 of Hb (this step's MMA operand) and into the workspace (the output
    // kernel's operand).  Two copies: a warp writes copy (s + 1) % 2 at the end of step s while
    // others may still read copy s % 2, and no warp reaches step s + 2's write before every warp has
    // passed step s + 1's barrier, i.e. finished reading copy s % 2 -- one barrier per step.
    auto put_h = [&](int step) {
        uint16_t* hb = Hb + (step & 1) * 128 * kHS;
        const size_t seg_i = (size_t)hv * p.SS + sq.sbase + step;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int row = 16 * mw + gq + 8 * hh;
            const uint32_t pk = pack_bf16x2(h[2 * hh], h[2 * hh + 1]);
            *reinterpret_cast<uint32_t*>(hb + row * kHS + 2 * tq) = pk;
            *reinterpret_cast<uint32_t*>(p.seg_hb + (seg_i * 128 + row) * 128 + v0 + 2 * tq) = pk;
        }
    };
    int s = 0;
    float gam = nseg > 0 ? p.seg_gamma[(size_t)hv * p.SS + sq.sbase] : 0.f;
    if (nseg > 0) put_h(0);
    for (; s < nseg; ++s) {
        if (!mbar_wait(full + (s % kStages), (uint32_t)((s / kStages) & 1), p.status, kErrScanTmaTimeout))
            *abort_flag = 1;
        named_bar_sync(1, kMath);  // copy s % 2 of Hb is complete
        if (*abort_flag) break;
        const unsigned char* st = sm + (s % kStages) * kStage;
        const uint16_t* hb = Hb + (s & 1) * 128 * kHS;
        // the next segment's gamma, a step ahead (a global load otherwise on the serial path)
        const float gam_next = s + 1 < nseg ? p.seg_gamma[(size_t)hv * p.SS + sq.sbase + s + 1] : 0.f;
        // P = D h_s for rows 16 mw .. +15 (even / odd k-steps in separate accumulators)
        float pa[4] = {0.f, 0.f, 0.f, 0.f}, pb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k0 = 0; k0 < 128; k0 += 16) {
            uint32_t a[4], b0, b1;
            ldsm_x4(a[0], a[1], a[2], a[3], st + kOffD + sw128_off(16 * mw + (lane & 15), k0 + ((lane >> 4) << 3), 16384));
            asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
                         : "=r"(b0), "=r"(b1)
                         : "r"(smem_u32(hb + (k0 + (lane & 15)) * kHS)));
            if ((k0 >> 4) & 1)
                mma_bf16(pb, a, b0, b1);
            else
                mma_bf16(pa, a, b0, b1);
        }
        const float* Bs = reinterpret_cast<const float*>(st + kOffB);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int row = 16 * mw + gq + 8 * (e >> 1), col = 2 * tq + (e & 1);
            h[e] = fmaf(gam, h[e], pa[e] + pb[e] + Bs[row * 8 + col]);
        }
        gam = gam_next;
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + (s % kStages));
        if (s + 1 < nseg) put_h(s + 1);
    }
    if (s < nseg) {
        if (tid == 0)
            for (int ss2 = s + 1; ss2 < min(nseg, s + kStages); ++ss2)
                mbar_wait(full + (ss2 % kStages), (uint32_t)((ss2 / kStages) & 1), nullptr, 0);
        return;
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int row = 16 * mw + gq + 8 * (e >> 1), col = 2 * tq + (e & 1);
        st_out[(size_t)(v0 + col) * kD + row] = h[e];
    }
}

// ------------------------------------------------------------------------------------------
// 3. outputs
// ------------------------------------------------------------------------------------------
namespace sego {
// Persistent: one CTA per SM walks (segment, v-head, pair of chunks) items.  Warps 0-7 run the
// epilogues, warp 8 issues the TMA loads, warp 9 the MMAs; operands and TMEM accumulators are double
// buffered, so one item's loads and product overlap the previous item's epilogue.
constexpr int kThreads = 320;
constexpr int kEpi = 256;
constexpr int kProdWarp = 8, kMmaWarp = 9;
constexpr int kPair = 2;             // chunks per item, stacked as the 128 rows of one MMA
constexpr uint32_t kBuf = 98304;     // per buffer: h_s, [Q''_a | Q''_b] (K-major A), oi'' (same arrangement)
constexpr uint32_t kOffH = 0;        // h_s: 2 column blocks of [128 K rows][128 B], SW128 (MN-major B)
constexpr uint32_t kOffQ = 32768;    // [Q''_a k0-63 | Q''_b k0-63 | Q''_a k64-127 | Q''_b k64-127]
constexpr uint32_t kOffO = 65536;
constexpr uint32_t kOffBar = 2 * kBuf;  // full[2], empty[2], mfull[2], accfree[2], TMEM slot
constexpr uint32_t kSmem = kOffBar + 8 * 8 + 16 + 1024;
}  // namespace sego

// Item w -> (segment slot, v-head, pair); false when the item holds no chunk.  Warp-wide (every lane
// of the calling warp gets the same answer), so every role walks the same sequence of items.
struct OutItem {
    int ss, hv, slot, t0, L0, L1, nch;
};
__device__ __forceinline__ bool seg_out_item(const PrefillArgs& p, int w, int npair, OutItem& it) {
    const int z = w % npair, hv = (w / npair) % p.HV, ss = w / (npair * p.HV);
    if (ss >= p.SS) return false;
    const SegSeq sq = warp_seg_seq(p, kBySeg, ss);
    if (sq.n < 0) return false;
    int bos, eos;
    seq_bounds(p.cu, p.cu64, sq.n, p.T, bos, eos);
    const int seg_c0 = (ss - sq.sbase) * p.seg_m;
    const int c0 = seg_c0 + z * sego::kPair;
    int nch = min(sego::kPair, min(seg_c0 + p.seg_m, sq.nc) - c0);
    nch = min(nch, p.S - (sq.cbase + c0));  // only a cu_seqlens that is not non-decreasing trims it
    if (nch <= 0) return false;
    it.ss = ss;
    it.hv = hv;
    it.slot = sq.cbase + c0;
    it.t0 = bos + c0 * kChunk;
    it.L0 = min(kChunk, eos - it.t0);
    it.L1 = nch > 1 ? min(kChunk, eos - it.t0 - kChunk) : 0;
    it.nch = nch;
    return true;
}

__global__ void __launch_bounds__(sego::kThreads, 1)
    gdn_prefill_seg_out_kernel(PrefillArgs p, const __grid_constant__ PrefillMaps maps) {
    using namespace sego;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(sm);
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + kOffBar);
    uint64_t* empty = full + 2;
    uint64_t* mfull = full + 4;
    uint64_t* accfree = full + 6;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(full + 8);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (warp == kProdWarp && lane == 0) {
        tma_prefetch_desc(&maps.qpp);
        tma_prefetch_desc(&maps.oipp);
        tma_prefetch_desc(&maps.seghb);
    }
    const int npair = (p.seg_m + kPair - 1) / kPair;
    const int total = p.SS * p.HV * npair;
    // barriers and TMEM before the grid-dependency wait (no chain CTA shares an SM with this one)
    if (tid == 0) {
        for (int b = 0; b < 2; ++b) {
            mbar_init(full + b, 1);
            mbar_init(empty + b, kEpi / 32);
            mbar_init(mfull + b, 1);
            mbar_init(accfree + b, kEpi / 32);
        }
        mbar_fence_init();
    }
    if (warp == 0) tmem_alloc(tslot, 256);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    pdl_wait();
    pdl_trigger();
    if (blockIdx.x == 0 && warp < kEpi / 32) zero_unowned_tokens(p, tid, kEpi);
    OutItem it;
    if (warp == kProdWarp) {
        int i = 0;
        for (int w = blockIdx.x; w < total; w += gridDim.x) {
            if (!seg_out_item(p, w, npair, it)) continue;
            const int b = i & 1;
            bool ok = true;
            if (lane == 0) {
                if (i >= 2) ok = mbar_wait(empty + b, (uint32_t)(((i >> 1) - 1) & 1), p.status, kErrScanTmaTimeout);
                if (ok) {
                    unsigned char* bf = sm + b * kBuf;
                    mbar_arrive_expect_tx(full + b, 32768u + (uint32_t)it.nch * 32768u);
                    tma_load_3d(bf + kOffH, &maps.seghb, 0, it.ss * 128, it.hv, full + b);
                    tma_load_3d(bf + kOffH + 16384, &maps.seghb, 64, it.ss * 128, it.hv, full + b);
                    for (int c = 0; c < it.nch; ++c) {
                        const int row = (it.slot + c) * kChunk;
                        tma_load_3d(bf + kOffQ + 8192 * c, &maps.qpp, 0, row, it.hv, full + b);
                        tma_load_3d(bf + kOffQ + 16384 + 8192 * c, &maps.qpp, 64, row, it.hv, full + b);
                        tma_load_3d(bf + kOffO + 8192 * c, &maps.oipp, 0, row, it.hv, full + b);
                        tma_load_3d(bf + kOffO + 16384 + 8192 * c, &maps.oipp, 64, row, it.hv, full + b);
                    }
                }
            }
            if (!__shfl_sync(0xffffffffu, (int)ok, 0)) break;
            ++i;
        }
        // the last two items' copies have landed before the CTA can leave (bounded)
        if (lane == 0)
            for (int j = max(0, i - 2); j < i; ++j) mbar_wait(full + (j & 1), (uint32_t)((j >> 1) & 1), nullptr, 0);
    } else if (warp == kMmaWarp) {
        constexpr uint32_t idesc = umma_idesc_bf16(128, 128, false, true);
        int i = 0;
        for (int w = blockIdx.x; w < total; w += gridDim.x) {
            if (!seg_out_item(p, w, npair, it)) continue;
            const int b = i & 1;
            bool ok = true;
            if (lane == 0) {
                ok = mbar_wait(full + b, (uint32_t)((i >> 1) & 1), p.status, kErrScanTmaTimeout);
                if (ok && i >= 2) ok = mbar_wait(accfree + b, (uint32_t)(((i >> 1) - 1) & 1), p.status, kErrScanMmaTimeout);
                if (ok) {
                    // [Q''_a; Q''_b] (128 x 128, K-major) x h_s (128 x 128, MN-major) -> accumulator b
                    tc_fence_after();
                    const uint32_t bf = sbase + (uint32_t)b * kBuf;
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk)
                        umma_bf16(tmem + 128u * (uint32_t)b,
                                  umma_desc_sw128(bf + kOffQ + (uint32_t)(kk >> 2) * 16384u + (uint32_t)(kk & 3) * 32u, 16, 1024),
                                  umma_desc_sw128(bf + kOffH + 2048u * kk, 16384, 1024), idesc, kk > 0);
                    umma_commit(mfull + b);
                }
            }
            if (!__shfl_sync(0xffffffffu, (int)ok, 0)) break;
            ++i;
        }
    } else {
        // epilogue: thread (r, hf) = TMEM lane r (chunk r / 64 of the pair, token row r % 64), columns
        // 64 hf .. +63: o = scale (Q'' h_s + oi'' + oi)
        const int r = lane + 32 * (warp & 3), hf = warp >> 2;
        const int ci = r >> 6, m = r & 63;
        int i = 0;
        for (int w = blockIdx.x; w < total; w += gridDim.x) {
            if (!seg_out_item(p, w, npair, it)) continue;
            const int b = i & 1;
            const bool live = ci < it.nch && m < (ci ? it.L1 : it.L0);
            const int slot = it.slot + ci;
            // oi = Aqk u of the chunk (prep, column-group major [16][64][8] bf16), loaded first so its
            // latency overlaps the wait for the product
            uint4 oc[8];
            if (live) {
                const uint16_t* oi_row = p.oi + cg_off(it.hv, p.S, slot, 8 * hf) + m * 8;
#pragma unroll
                for (int g = 0; g < 8; ++g) oc[g] = *reinterpret_cast<const uint4*>(oi_row + g * 512);
            }
            const bool ok = mbar_wait(mfull + b, (uint32_t)((i >> 1) & 1), p.status, kErrScanMmaTimeout);
            tc_fence_after();
            if (!__all_sync(0xffffffffu, ok)) break;
            uint32_t d[2][32];
            tmem_ld32_async(tmem + ((uint32_t)(32 * (warp & 3)) << 16) + 128u * (uint32_t)b + 64u * hf, d[0]);
            tmem_ld32_async(tmem + ((uint32_t)(32 * (warp & 3)) << 16) + 128u * (uint32_t)b + 64u * hf + 32u, d[1]);
            tmem_ld_wait();
            tmem_regs_ready(d[0]);
            tmem_regs_ready(d[1]);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(accfree + b);  // accumulator b may take the next product
            if (live) {
                uint16_t* dst = p.out + ((size_t)(it.t0 + ci * kChunk + m) * p.HV + it.hv) * kD + 64 * hf;
                const unsigned char* orow = sm + b * kBuf + kOffO + (uint32_t)hf * 16384u + (uint32_t)r * 128u;
#pragma unroll
                for (int g = 0; g < 8; ++g) {
                    const uint4 o2 = *reinterpret_cast<const uint4*>(orow + ((g ^ (r & 7)) << 4));
                    const uint32_t pw[4] = {o2.x, o2.y, o2.z, o2.w};
                    const uint32_t ow[4] = {oc[g].x, oc[g].y, oc[g].z, oc[g].w};
                    uint32_t pk[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const uint32_t x0 = d[g >> 2][8 * (g & 3) + 2 * e], x1 = d[g >> 2][8 * (g & 3) + 2 * e + 1];
                        const float2 x2 = add2(add2(make_float2(__uint_as_float(x0), __uint_as_float(x1)),
                                                    make_float2(__uint_as_float(pw[e] << 16), __uint_as_float(pw[e] & 0xffff0000u))),
                                               make_float2(__uint_as_float(ow[e] << 16), __uint_as_float(ow[e] & 0xffff0000u)));
                        pk[e] = pack_bf16x2(p.scale * x2.x, p.scale * x2.y);
                    }
                    *reinterpret_cast<uint4*>(dst + 8 * g) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty + b);  // buffer b (oi'') is read
            ++i;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 256);
}

int launch_prefill_seg(const PrefillArgs& p, const PrefillMaps& maps, cudaStream_t stream) {
    if (cudaFuncSetAttribute(gdn_prefill_seg_local_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, segk::kSmem) !=
            cudaSuccess ||
        cudaFuncSetAttribute(gdn_prefill_seg_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, segc::kSmem) !=
            cudaSuccess ||
        cudaFuncSetAttribute(gdn_prefill_seg_out_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, sego::kSmem) !=
            cudaSuccess)
        return -1;
    // segment slots actually used: sum_n ceil(nc_n / m) <= min(SS, ceil(T / 64 / m) + N - 1)
    const long long segs = std::min<long long>(p.SS, ((long long)p.T + 64LL * p.seg_m - 1) / (64LL * p.seg_m) + p.N - 1);
    if (launch_pdl(gdn_prefill_seg_local_kernel, dim3((unsigned)std::max<long long>(segs, 1), p.HV, 2),
                   dim3(segk::kThreads), segk::kSmem, stream, p, maps) != cudaSuccess)
        return -1;
    if (launch_pdl(gdn_prefill_seg_chain_kernel, dim3(kD / segc::BV, p.N, p.HV), dim3(segc::kThreads), segc::kSmem,
                   stream, p, maps) != cudaSuccess)
        return -1;
    {
        int dev = 0, sms = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return -1;
        const long long items = segs * p.HV * ((p.seg_m + sego::kPair - 1) / sego::kPair);
        if (launch_pdl(gdn_prefill_seg_out_kernel, dim3((unsigned)std::max<long long>(1, std::min<long long>(items, sms))),
                       dim3(sego::kThreads), sego::kSmem, stream, p, maps) != cudaSuccess)
            return -1;
    }
    return 0;
}

}  // namespace gdn
