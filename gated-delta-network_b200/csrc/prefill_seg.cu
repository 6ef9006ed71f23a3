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
//              = scale (Q''_j h_s + oi''_j),  Q''_j = Q'_j Phi_j,  oi''_j = oi_j + Q'_j beta_j.
//      At the end it stores the segment transition h_{s+1} = gamma h_s + D h_s + B with
//      B = beta_end, gamma = product of e^{G_L}, D = Phi_end - gamma I.
//   2. gdn_prefill_seg_chain_kernel, one CTA per (8 state columns, sequence, v-head): the short
//      serial chain over segments, h_{s+1} = gamma h_s + D h_s + B; it records each h_s (bf16,
//      the output operand) and writes the final state.
//   3. gdn_prefill_seg_out_kernel, one CTA per (chunk, v-head): o_j = scale (Q''_j h_s + oi''_j).
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
// One CTA per (segment, v-head): two groups of 8 math warps, group 0 carries beta (the state the
// segment builds from zero, with u), group 1 Phi (the transition, without u).  The groups share
// the chunk tiles and run independent chains, so one group's epilogues overlap the other's MMAs.
constexpr int kGroupThreads = 256;
constexpr int kThreads = 2 * kGroupThreads + 32;  // + 1 TMA producer warp
constexpr uint32_t kOffWQ = 0;              // [W0 | Q'0 | W1 | Q'1], 8 KB each (single buffer)
constexpr uint32_t kOffK = 32768;           // 2 stages of {k tile (2 atoms of 64 tokens x 128 B), G4 [64][4] f32}
constexpr uint32_t kKStage = 17408;
constexpr uint32_t kOffG = 16384;           // G4 inside a k stage
constexpr uint32_t kOffU = kOffK + 2 * kKStage;   // u f32 [16 cg][64][8] (single buffer)
constexpr uint32_t kOffX = kOffU + 32768;         // per group: X bf16, 2 column blocks of [128 rows][128 B],
                                                  // SW128; between MMA_P and MMA_U: vn hi / lo [2][64][128 B]
constexpr uint32_t kOffO = kOffX + 2 * 32768;     // per group: output tile bf16, 2 atoms of [64][128 B]
constexpr uint32_t kOffBar = kOffO + 2 * 16384;   // wq_full, wq_empty, kfull[2], kempty[2], ufull, uempty,
                                                  // bar_p[2], bar_u[2]
constexpr uint32_t kSmemUsed = kOffBar + 8 * 12 + 16;
constexpr uint32_t kSmem = kSmemUsed + 1024;
constexpr uint32_t kTmemCols = 512;         // group g: P at 256 g, X at 256 g + 128
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

// ------------------------------------------------------------------------------------------
// 1. local transitions
// ------------------------------------------------------------------------------------------
__global__ void __maxnreg__(112)
    gdn_prefill_seg_local_kernel(PrefillArgs p, const __grid_constant__ PrefillMaps maps) {
    using namespace segk;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(sm);
    uint64_t* wq_full = reinterpret_cast<uint64_t*>(sm + kOffBar);
    uint64_t* wq_empty = wq_full + 1;
    uint64_t* kfull = wq_full + 2;
    uint64_t* kempty = wq_full + 4;
    uint64_t* ufull = wq_full + 6;
    uint64_t* uempty = wq_full + 7;
    uint64_t* bar_p = wq_full + 8;
    uint64_t* bar_u = wq_full + 10;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(wq_full + 12);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ss = blockIdx.x, hv = blockIdx.y;
    const int hq = hv / (p.HV / p.H);
    const int prod_warp = 2 * kGroupThreads / 32;
    if (warp == prod_warp && lane == 0) {
        tma_prefetch_desc(&maps.w);
        tma_prefetch_desc(&maps.qp);
        tma_prefetch_desc(&maps.k);
        tma_prefetch_desc(&maps.qpp);
        tma_prefetch_desc(&maps.oipp);
    }
    pdl_wait();  // the workspace comes from the prep kernel
    pdl_trigger();
    const SegSeq sq = warp_seg_seq(p, kBySeg, ss);
    if (sq.n < 0 || ss >= p.SS) return;  // a slot past the last segment (uniform across the CTA)
    int bos, eos;
    seq_bounds(p.cu, p.cu64, sq.n, p.T, bos, eos);
    const int c0 = (ss - sq.sbase) * p.seg_m;
    int nch = min(p.seg_m, sq.nc - c0);
    nch = max(0, min(nch, p.S - (sq.cbase + c0)));  // only a cu_seqlens that is not non-decreasing trims it
    if (nch <= 0) return;
    const int slot0 = sq.cbase + c0;

    if (tid == 0) {
        mbar_init(wq_full, 1);
        mbar_init(wq_empty, 2);  // one arrival per group once its MMA_P has completed
        for (int s = 0; s < 2; ++s) {
            mbar_init(kfull + s, 1);
            mbar_init(kempty + s, 2);  // one arrival per group once its MMA_U has completed
            mbar_init(bar_p + s, 1);
            mbar_init(bar_u + s, 1);
        }
        mbar_init(ufull, 1);
        mbar_init(uempty, 4);  // the four vn warps of group 0
        mbar_fence_init();
    }
    if (warp == 0) tmem_alloc(tslot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    if (warp == prod_warp) {
        // Producer.  k stage c % 2 (k tile, gates) is refilled once both groups finished chunk c - 2;
        // the single W / Q' buffer once both groups' MMA_P of chunk c - 1 completed; the single u
        // buffer once group 0 formed chunk c - 1's vn.
        if (lane == 0) {
            for (int c = 0; c < nch; ++c) {
                const int slot = slot0 + c, wr = slot * kChunk, t0 = bos + (c0 + c) * kChunk;
                if (c >= 2 && !mbar_wait(kempty + (c & 1), (uint32_t)(((c >> 1) - 1) & 1), p.status, kErrScanTmaTimeout))
                    break;
                unsigned char* ks = sm + kOffK + (c & 1) * kKStage;
                mbar_arrive_expect_tx(kfull + (c & 1), 16384 + 1024);
                tma_load_3d(ks, &maps.k, 0, hq, t0, kfull + (c & 1));
                tma_load_3d(ks + 8192, &maps.k, 64, hq, t0, kfull + (c & 1));
                bulk_load(ks + kOffG, p.g4 + ((size_t)hv * p.S + slot) * kChunk * 4, 1024, kfull + (c & 1));
                if (c >= 1 && !mbar_wait(wq_empty, (uint32_t)((c - 1) & 1), p.status, kErrScanTmaTimeout)) break;
                mbar_arrive_expect_tx(wq_full, 32768);
                tma_load_3d(sm + kOffWQ, &maps.w, 0, wr, hv, wq_full);
                tma_load_3d(sm + kOffWQ + 8192, &maps.qp, 0, wr, hv, wq_full);
                tma_load_3d(sm + kOffWQ + 16384, &maps.w, 64, wr, hv, wq_full);
                tma_load_3d(sm + kOffWQ + 24576, &maps.qp, 64, wr, hv, wq_full);
                if (c >= 1 && !mbar_wait(uempty, (uint32_t)((c - 1) & 1), p.status, kErrScanTmaTimeout)) break;
                mbar_arrive_expect_tx(ufull, 32768);
                bulk_load(sm + kOffU, p.u + cg_off(hv, p.S, slot, 0), 32768, ufull);
            }
        }
    } else {
        // ---- math: group g, thread (r, hf) = TMEM lane r, state columns 64 hf .. 64 hf + 63 ----
        const int g = warp >> 3, gw = warp & 7;
        const int r = lane + 32 * (gw & 3), hf = gw >> 2;
        const int gt = tid - g * kGroupThreads;  // thread index inside the group
        const uint32_t lanebits = (uint32_t)(32 * (gw & 3)) << 16;
        const uint32_t tP = tmem + lanebits + 256u * g + 64u * hf;  // this thread's 64 P columns
        const uint32_t tX = tP + 128u;                                // and 64 X columns
        unsigned char* xb = sm + kOffX + g * 32768;
        const uint32_t sxb = sbase + kOffX + (uint32_t)g * 32768u;
        unsigned char* ob = sm + kOffO + g * 16384;
        const CUtensorMap* omap = g ? &maps.qpp : &maps.oipp;
        // X starts as 0 (beta) or I (Phi): in TMEM (fp32) and as the bf16 MMA operand
        {
            uint32_t z[32];
#pragma unroll
            for (int blk = 0; blk < 2; ++blk) {
#pragma unroll
                for (int j = 0; j < 32; ++j) z[j] = __float_as_uint((g == 1 && r == 64 * hf + 32 * blk + j) ? 1.f : 0.f);
                tmem_st32(tX + 32u * blk, z);
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4)
                    *reinterpret_cast<uint4*>(xb + hf * 16384 + r * 128 + (((4 * blk + q4) ^ (r & 7)) << 4)) =
                        make_uint4(pack_bf16x2(__uint_as_float(z[8 * q4]), __uint_as_float(z[8 * q4 + 1])),
                                   pack_bf16x2(__uint_as_float(z[8 * q4 + 2]), __uint_as_float(z[8 * q4 + 3])),
                                   pack_bf16x2(__uint_as_float(z[8 * q4 + 4]), __uint_as_float(z[8 * q4 + 5])),
                                   pack_bf16x2(__uint_as_float(z[8 * q4 + 6]), __uint_as_float(z[8 * q4 + 7])));
            }
            tmem_st_wait();
        }
        constexpr uint32_t idesc_p = umma_idesc_bf16(128, 128, false, true);
        constexpr uint32_t idesc_u = umma_idesc_bf16(128, 128, true, true);
        const bool dbg = g == 0;
        long long tp = clock64();
        (void)dbg;
        float gamma = 1.f;
        bool okc = true;  // every bounded wait of this thread so far succeeded
        int c = 0;
        for (; c < nch; ++c) {
            const uint32_t ph = (uint32_t)(c & 1);
            bool ok = mbar_wait(kfull + (c & 1), (uint32_t)((c >> 1) & 1), p.status, kErrScanTmaTimeout) && okc;
            ok = mbar_wait(wq_full, ph, p.status, kErrScanTmaTimeout) && ok;
            GDN_PH_ACC(dbg, 0, tp);
            if (gt == 128) tma_store_wait_read();  // the previous output tile has left the staging buffer
            fence_async_smem();                     // X copy (generic stores) -> the tensor core
            tc_fence_before();
            // a wait that gave up anywhere in the group stops the whole group (uniform break)
            if (!named_bar_and(1 + g, kGroupThreads, ok)) break;
            tc_fence_after();
            GDN_PH_ACC(dbg, 1, tp);
            const unsigned char* ks = sm + kOffK + (c & 1) * kKStage;
            const uint32_t sks = sbase + kOffK + (uint32_t)(c & 1) * kKStage;
            const float* G4 = reinterpret_cast<const float*>(ks + kOffG);
            const int slot = slot0 + c;
            const int t0 = bos + (c0 + c) * kChunk;
            const int L = min(kChunk, eos - t0);
            const float GL = G4[(L - 1) * 4];
            const float eL = __expf(GL);
            // MMA_P: [W; Q'] (128 x 128, K-major) x X (128 x 128, MN-major) -> P
            if (gt == 0) {
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    umma_bf16(tmem + 256u * g,
                              umma_desc_sw128(sbase + kOffWQ + (uint32_t)(kk >> 2) * 16384u + (uint32_t)(kk & 3) * 32u, 16, 1024),
                              umma_desc_sw128(sxb + 2048u * kk, 16384, 1024), idesc_p, kk > 0);
                umma_commit(bar_p + g);
            }
            ok = mbar_wait(bar_p + g, ph, p.status, kErrScanMmaTimeout);
            tc_fence_after();
            if (gt == 0) mbar_arrive(wq_empty);  // this group's MMA_P has read W / Q'
            GDN_PH_ACC(dbg, 2, tp);
            // X <- e^{G_L} X in TMEM: MMA_U then accumulates K^T vn onto it
#pragma unroll
            for (int blk = 0; blk < 2; ++blk) {
                uint32_t d[32];
                tmem_ld32_async(tX + 32u * blk, d);
                tmem_ld_wait();
                tmem_regs_ready(d);
#pragma unroll
                for (int j = 0; j < 32; j += 2) {
                    const float2 v2 = mul2(make_float2(eL, eL), make_float2(__uint_as_float(d[j]), __uint_as_float(d[j + 1])));
                    d[j] = __float_as_uint(v2.x);
                    d[j + 1] = __float_as_uint(v2.y);
                }
                tmem_st32(tX + 32u * blk, d);
            }
            if (r < 64) {
                // vn = ([u | 0] - W X) e^{G_L - G_r} / |k_r|  -> bf16 hi + lo, token row r
                if (g == 0 && !mbar_wait(ufull, ph, p.status, kErrScanTmaTimeout)) ok = false;
                const float4 g4r = *reinterpret_cast<const float4*>(G4 + r * 4);  // {G, e^G, beta, rk}
                const float ed = __expf(GL - g4r.x) * g4r.w;
                const float* Us = reinterpret_cast<const float*>(sm + kOffU);
                unsigned char* rh = xb + hf * 8192 + r * 128;
                unsigned char* rl = rh + 16384;
                const int hA = (r >> 2) & 1;
#pragma unroll
                for (int blk = 0; blk < 2; ++blk) {
                    uint32_t d[32];
                    tmem_ld32_async(tP + 32u * blk, d);
                    tmem_ld_wait();
                    tmem_regs_ready(d);
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        const int jj = 4 * blk + q4;  // 8-column group inside this thread's 64 columns
                        float uu[8];
                        if (g == 0) {
                            const int cg = 8 * hf + jj;
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
                        *reinterpret_cast<uint4*>(rh + ((jj ^ (r & 7)) << 4)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                        *reinterpret_cast<uint4*>(rl + ((jj ^ (r & 7)) << 4)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                    }
                }
                if (g == 0) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(uempty);  // this warp's u rows are consumed
                }
            } else {
                // output operand row m = r - 64: oi'' = Q' beta (group 0) or Q'' = Q' Phi (group 1), bf16,
                // staged SW128 for one TMA store per 64 columns
                const int m = r - 64;
                unsigned char* orow = ob + hf * 8192 + m * 128;
#pragma unroll
                for (int blk = 0; blk < 2; ++blk) {
                    uint32_t d[32];
                    tmem_ld32_async(tP + 32u * blk, d);
                    tmem_ld_wait();
                    tmem_regs_ready(d);
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        const int jj = 4 * blk + q4;
                        *reinterpret_cast<uint4*>(orow + ((jj ^ (m & 7)) << 4)) =
                            make_uint4(pack_bf16x2(__uint_as_float(d[8 * q4]), __uint_as_float(d[8 * q4 + 1])),
                                       pack_bf16x2(__uint_as_float(d[8 * q4 + 2]), __uint_as_float(d[8 * q4 + 3])),
                                       pack_bf16x2(__uint_as_float(d[8 * q4 + 4]), __uint_as_float(d[8 * q4 + 5])),
                                       pack_bf16x2(__uint_as_float(d[8 * q4 + 6]), __uint_as_float(d[8 * q4 + 7])));
                    }
                }
            }
            GDN_PH_ACC(dbg, 3, tp);
            tmem_st_wait();      // the scaled X is in TMEM
            fence_async_smem();  // vn and the output tile (generic stores) -> the tensor core / TMA
            tc_fence_before();
            ok = named_bar_and(1 + g, kGroupThreads, ok);
            tc_fence_after();
            GDN_PH_ACC(dbg, 4, tp);
            // MMA_U: K^T (128 x 64 tokens, MN-major) x (vn_hi + vn_lo), accumulated onto X
            if (ok && gt == 0) {
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_bf16(tmem + 256u * g + 128u, umma_desc_sw128(sks + 2048u * kk, 8192, 1024),
                              umma_desc_sw128(sxb + 2048u * kk, 8192, 1024), idesc_u, true);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_bf16(tmem + 256u * g + 128u, umma_desc_sw128(sks + 2048u * kk, 8192, 1024),
                              umma_desc_sw128(sxb + 16384u + 2048u * kk, 8192, 1024), idesc_u, true);
                umma_commit(bar_u + g);
            }
            if (gt == 128) {  // the output tile: two SW128 boxes of 64 columns
                tma_store_3d(omap, 0, slot * kChunk, hv, ob);
                tma_store_3d(omap, 64, slot * kChunk, hv, ob + 8192);
                tma_store_commit();
            }
            GDN_PH_ACC(dbg, 5, tp);
            // an MMA_U that was not issued (a wait gave up) also fails this bounded wait
            if (ok) ok = mbar_wait(bar_u + g, ph, p.status, kErrScanMmaTimeout);
            tc_fence_after();
            if (gt == 0) mbar_arrive(kempty + (c & 1));  // this group is done with the k tile and gates
            GDN_PH_ACC(dbg, 6, tp);
            // bf16 copy of the new X for the next MMA_P
#pragma unroll
            for (int blk = 0; blk < 2; ++blk) {
                uint32_t d[32];
                tmem_ld32_async(tX + 32u * blk, d);
                tmem_ld_wait();
                tmem_regs_ready(d);
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4)
                    *reinterpret_cast<uint4*>(xb + hf * 16384 + r * 128 + (((4 * blk + q4) ^ (r & 7)) << 4)) =
                        make_uint4(pack_bf16x2(__uint_as_float(d[8 * q4]), __uint_as_float(d[8 * q4 + 1])),
                                   pack_bf16x2(__uint_as_float(d[8 * q4 + 2]), __uint_as_float(d[8 * q4 + 3])),
                                   pack_bf16x2(__uint_as_float(d[8 * q4 + 4]), __uint_as_float(d[8 * q4 + 5])),
                                   pack_bf16x2(__uint_as_float(d[8 * q4 + 6]), __uint_as_float(d[8 * q4 + 7])));
            }
            gamma *= eL;
            okc = ok;
            GDN_PH_ACC(dbg, 7, tp);
        }
        if (c < nch) {
            // gave up: let copies already in flight land (bounded) before the CTA exits
            if (gt == 0) {
                for (int cc = c; cc < min(nch, c + 2); ++cc)
                    mbar_wait(kfull + (cc & 1), (uint32_t)((cc >> 1) & 1), nullptr, 0);
                mbar_wait(wq_full, (uint32_t)(c & 1), nullptr, 0);
                if (g == 0) mbar_wait(ufull, (uint32_t)(c & 1), nullptr, 0);
            }
        } else {
            // segment transition: B = beta_end (group 0), D = Phi_end - gamma I and gamma (group 1)
            const size_t seg_i = (size_t)hv * p.SS + ss;
#pragma unroll
            for (int blk = 0; blk < 2; ++blk) {
                uint32_t d[32];
                tmem_ld32_async(tX + 32u * blk, d);
                tmem_ld_wait();
                tmem_regs_ready(d);
                if (g == 0) {
                    float* Bp = p.seg_B + seg_i * 128 * 128;  // column-group major [16][128][8] f32
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        float4* dst = reinterpret_cast<float4*>(Bp + ((8 * hf + 4 * blk + q4) * 128 + r) * 8);
                        dst[0] = make_float4(__uint_as_float(d[8 * q4]), __uint_as_float(d[8 * q4 + 1]),
                                             __uint_as_float(d[8 * q4 + 2]), __uint_as_float(d[8 * q4 + 3]));
                        dst[1] = make_float4(__uint_as_float(d[8 * q4 + 4]), __uint_as_float(d[8 * q4 + 5]),
                                             __uint_as_float(d[8 * q4 + 6]), __uint_as_float(d[8 * q4 + 7]));
                    }
                } else {
                    float x[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        x[j] = __uint_as_float(d[j]) - ((r == 64 * hf + 32 * blk + j) ? gamma : 0.f);
                    uint4* dst = reinterpret_cast<uint4*>(p.seg_D + (seg_i * 128 + r) * 128 + 64 * hf + 32 * blk);
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4)
                        dst[q4] = make_uint4(pack_bf16x2(x[8 * q4], x[8 * q4 + 1]), pack_bf16x2(x[8 * q4 + 2], x[8 * q4 + 3]),
                                             pack_bf16x2(x[8 * q4 + 4], x[8 * q4 + 5]), pack_bf16x2(x[8 * q4 + 6], x[8 * q4 + 7]));
                }
            }
            if (g == 1 && gt == 0) p.seg_gamma[seg_i] = gamma;
        }
        if (gt == 128) tma_store_wait_all();  // the operand stores are complete before the grid ends
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
constexpr uint32_t kOffHb = kStages * kStage;       // h bf16 [128][8]
constexpr uint32_t kOffBar = kOffHb + 128 * kHS * 2;
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
    pdl_wait();  // the segment transitions come from the local kernel
    pdl_trigger();
    const SegSeq sq = warp_seg_seq(p, kBySeq, n);
    int bos, eos;
    seq_bounds(p.cu, p.cu64, n, p.T, bos, eos);
    float* st_out = p.new_state + ((size_t)n * p.HV + hv) * kD * kD;
    if (eos - bos <= 0) {  // zero-length sequence: all-zero final state (reference/gdn_prefill_ref.py:52-54, 61-62)
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
    // math warp mw owns state rows 16 mw .. 16 mw + 15: h[e] = h[16 mw + gq + 8 (e >> 1)][2 tq + (e & 1)]
    const int mw = warp;
    float h[4];
    {
        const float* st_in = p.state ? p.state + ((size_t)n * p.HV + hv) * kD * kD : nullptr;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int row = 16 * mw + gq + 8 * (e >> 1), col = 2 * tq + (e & 1);
            h[e] = st_in ? st_in[(size_t)(v0 + col) * kD + row] : 0.f;
        }
    }
    int s = 0;
    for (; s < nseg; ++s) {
        // h_s (bf16): this step's MMA operand and the output kernel's
        const size_t seg_i = (size_t)hv * p.SS + sq.sbase + s;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int row = 16 * mw + gq + 8 * hh;
            const uint32_t pk = pack_bf16x2(h[2 * hh], h[2 * hh + 1]);
            *reinterpret_cast<uint32_t*>(Hb + row * kHS + 2 * tq) = pk;
            *reinterpret_cast<uint32_t*>(p.seg_hb + (seg_i * 128 + row) * 128 + v0 + 2 * tq) = pk;
        }
        if (!mbar_wait(full + (s % kStages), (uint32_t)((s / kStages) & 1), p.status, kErrScanTmaTimeout))
            *abort_flag = 1;
        named_bar_sync(1, kMath);
        if (*abort_flag) break;
        const unsigned char* st = sm + (s % kStages) * kStage;
        const float gam = p.seg_gamma[seg_i];
        // P = D h_s for rows 16 mw .. +15 (even / odd k-steps in separate accumulators)
        float pa[4] = {0.f, 0.f, 0.f, 0.f}, pb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k0 = 0; k0 < 128; k0 += 16) {
            uint32_t a[4], b0, b1;
            ldsm_x4(a[0], a[1], a[2], a[3], st + kOffD + sw128_off(16 * mw + (lane & 15), k0 + ((lane >> 4) << 3), 16384));
            asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
                         : "=r"(b0), "=r"(b1)
                         : "r"(smem_u32(Hb + (k0 + (lane & 15)) * kHS)));
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
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + (s % kStages));
        named_bar_sync(1, kMath);  // every warp has read Hb before it is rewritten
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
constexpr int kThreads = 256;
constexpr uint32_t kOffQ = 0;        // Q'' 2 atoms [64][128 B]
constexpr uint32_t kOffO = 16384;    // oi'' 2 atoms [64][128 B]
constexpr uint32_t kOffH = 32768;    // h_s 2 atoms [128 K][128 B] (64 V columns each)
constexpr uint32_t kTx = 16384 + 16384 + 32768;
constexpr uint32_t kOffBar = 65536;
constexpr uint32_t kSmem = kOffBar + 16 + 1024;
}  // namespace sego

__global__ void __launch_bounds__(sego::kThreads)
    gdn_prefill_seg_out_kernel(PrefillArgs p, const __grid_constant__ PrefillMaps maps) {
    using namespace sego;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kOffBar);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int gq = lane >> 2, tq = lane & 3;
    const int slot = blockIdx.x, hv = blockIdx.y;
    if (tid == 0) {
        tma_prefetch_desc(&maps.qpp);
        tma_prefetch_desc(&maps.oipp);
        tma_prefetch_desc(&maps.seghb);
    }
    pdl_wait();
    pdl_trigger();
    if (slot == 0 && hv == 0) zero_unowned_tokens(p, tid, kThreads);
    const SegSeq sq = warp_seg_seq(p, kByChunk, slot);
    if (sq.n < 0) return;
    int bos, eos;
    seq_bounds(p.cu, p.cu64, sq.n, p.T, bos, eos);
    const int c = slot - sq.cbase;
    const int ss = sq.sbase + c / p.seg_m;
    if (ss >= p.SS) return;  // only a cu_seqlens that is not non-decreasing gets here
    const int t0 = bos + c * kChunk;
    const int L = min(kChunk, eos - t0);
    if (tid == 0) {
        mbar_init(bar, 1);
        mbar_fence_init();
    }
    __syncthreads();
    if (tid == 0) {
        mbar_arrive_expect_tx(bar, kTx);
        tma_load_3d(sm + kOffQ, &maps.qpp, 0, slot * kChunk, hv, bar);
        tma_load_3d(sm + kOffQ + 8192, &maps.qpp, 64, slot * kChunk, hv, bar);
        tma_load_3d(sm + kOffO, &maps.oipp, 0, slot * kChunk, hv, bar);
        tma_load_3d(sm + kOffO + 8192, &maps.oipp, 64, slot * kChunk, hv, bar);
        tma_load_3d(sm + kOffH, &maps.seghb, 0, ss * 128, hv, bar);
        tma_load_3d(sm + kOffH + 16384, &maps.seghb, 64, ss * 128, hv, bar);
    }
    if (!mbar_wait(bar, 0, p.status, kErrScanTmaTimeout)) {
        if (tid == 0) mbar_wait(bar, 0, nullptr, 0);
        return;
    }
    // oi = Aqk u of the chunk (prep kernel, column-group major [16][64][8] bf16)
    const uint16_t* oi_slot = p.oi + cg_off(hv, p.S, slot, 0);
    // warp w: output rows 16 (w & 3) .. +15, columns 64 (w >> 2) .. +63
    const int r0 = 16 * (warp & 3), n0 = 64 * (warp >> 2);
    float acc[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
#pragma unroll
    for (int k0 = 0; k0 < 128; k0 += 16) {
        uint32_t a[4];
        ldsm_x4(a[0], a[1], a[2], a[3], sm + kOffQ + sw128_off(r0 + (lane & 15), k0 + ((lane >> 4) << 3), 8192));
#pragma unroll
        for (int np = 0; np < 4; ++np) {
            uint32_t b0, b1, b2, b3;
            const int kr = k0 + (lane & 7) + (((lane >> 3) & 1) << 3);
            const int cc = n0 + 16 * np + ((lane >> 4) << 3);
            ldsm_x4_t(b0, b1, b2, b3, sm + kOffH + sw128_off(kr, cc, 16384));
            mma_bf16(acc[2 * np], a, b0, b1);
            mma_bf16(acc[2 * np + 1], a, b2, b3);
        }
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const int row = r0 + gq + 8 * hh;
        if (row >= L) continue;
        uint16_t* dst = p.out + ((size_t)(t0 + row) * p.HV + hv) * kD;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            const int col = n0 + 8 * nt + 2 * tq;
            const uint32_t oo = *reinterpret_cast<const uint32_t*>(sm + kOffO + sw128_off(row, col, 8192));
            const uint32_t oc = *reinterpret_cast<const uint32_t*>(oi_slot + (col >> 3) * 512 + row * 8 + (col & 7));
            const float2 o2 = add2(add2(make_float2(acc[nt][2 * hh], acc[nt][2 * hh + 1]),
                                        make_float2(__uint_as_float(oo << 16), __uint_as_float(oo & 0xffff0000u))),
                                   make_float2(__uint_as_float(oc << 16), __uint_as_float(oc & 0xffff0000u)));
            *reinterpret_cast<uint32_t*>(dst + col) = pack_bf16x2(p.scale * o2.x, p.scale * o2.y);
        }
    }
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
    if (launch_pdl(gdn_prefill_seg_local_kernel, dim3((unsigned)std::max<long long>(segs, 1), p.HV),
                   dim3(segk::kThreads), segk::kSmem, stream, p, maps) != cudaSuccess)
        return -1;
    if (launch_pdl(gdn_prefill_seg_chain_kernel, dim3(kD / segc::BV, p.N, p.HV), dim3(segc::kThreads), segc::kSmem,
                   stream, p, maps) != cudaSuccess)
        return -1;
    const long long chunks = std::min<long long>(p.S, ((long long)p.T + 63) / 64 + p.N - 1);
    if (launch_pdl(gdn_prefill_seg_out_kernel, dim3((unsigned)std::max<long long>(chunks, 1), p.HV),
                   dim3(sego::kThreads), sego::kSmem, stream, p, maps) != cudaSuccess)
        return -1;
    return 0;
}

}  // namespace gdn
