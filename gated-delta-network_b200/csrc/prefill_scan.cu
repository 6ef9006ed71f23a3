// prefill_scan.cu -- serial half of the chunked Gated DeltaNet prefill (sm_100a).
//
// One CTA per (slice of BV state columns, sequence n, v-head hv); it walks the chunks of
// sequence n in order and keeps its [K=128 x BV] slice of the state h in registers (fp32
// mma.sync accumulator fragments) for the whole sequence.  Per chunk (fused form of
// solutions/gdn_prefill_qk4_v8_d128_k_last/solution/triton/fla_kernels.py:411-671 chunk_h
// and 714-796 chunk_o; the per-chunk state snapshots never leave the SM):
//   vn = u - w h                                  (u, w from the prep kernel's workspace slot)
//   o  = scale (Q' h + oi)                        -> out   (Q' = e^G.Q - Aqk w, oi = Aqk u, so
//                                                  o = scale (e^G.(Q h) + Aqk vn) as in chunk_o)
//   h  = e^{G_last} h + K^T (e^{G_last - G} . vn) (vn split into bf16 hi + lo: ~16-bit mantissa)
// Each chunk's W, Q', K (SWIZZLE_128B), u / oi slices and G tiles arrive by TMA into a 3-stage
// ring of shared-memory buffers: a producer warp issues the copies as soon as the math warps
// release a stage (empty / full mbarrier pairs), so the math never waits on TMA issue.
// Eight math warps (two per SM sub-partition) split every phase: warps 0-3 form w h and vn
// while warps 4-7 form Q' h and the outputs; all eight update 16 state rows each.  The serial
// dependency (w h -> vn -> K^T vn -> h) uses warp-level mma.sync fragments: their ~20-cycle
// latency beats a tcgen05 round trip (~570 cycles) for these 64 x BV x 128 products, and the
// state never leaves the register file.
#include "prefill_kernels.cuh"
#include "sm100.cuh"
#include "dbg.cuh"

GDN_DBG_READER(gdn_debug_read_scan)

namespace gdn {

template <int BV>
struct Scan2Cfg {
    static constexpr int kThreads = 288;    // 8 math warps + 1 TMA producer warp
    static constexpr int kMath = 256;
    static constexpr int kStages = 3;
    // bf16 row stride of the [rows][BV] operand tiles: 8 consecutive rows must start in 8
    // different 16-byte bank groups for conflict-free ldmatrix (16 B for BV=8, 48 B, 80 B).
    static constexpr int kHS = BV == 8 ? 8 : BV + 8;
    static constexpr uint32_t kOffW = 0;        // 2 atoms of 64 rows x 128 B (atom stride 8 KB)
    static constexpr uint32_t kOffQ = 16384;
    static constexpr uint32_t kOffK = 32768;
    static constexpr uint32_t kOffU = 49152;                // [BV/8][64][8] f32 (u, column-group major)
    static constexpr uint32_t kOffO = kOffU + 64 * BV * 4;  // [BV/8][64][8] bf16 (oi)
    static constexpr uint32_t kOffG = kOffO + 64 * BV * 2;  // [64][4] f32 {G, e^G, beta, 0}
    static constexpr uint32_t kStage = ((kOffG + 1024) + 1023) & ~1023u;
    static constexpr uint32_t kTxBytes = 3 * 16384 + 64 * BV * 6 + 1024;
    static constexpr uint32_t kOffHb = kStages * kStage;               // [128][kHS] bf16
    static constexpr uint32_t kOffVh = kOffHb + 128 * kHS * 2;          // [64][kHS] bf16
    static constexpr uint32_t kOffVl = kOffVh + 64 * kHS * 2;
    static constexpr uint32_t kOffBar = (kOffVl + 64 * kHS * 2 + 15) & ~15u;
    static constexpr uint32_t kSmemUsed = kOffBar + 16 * kStages + 16;  // full[], empty[], abort flag
    static constexpr uint32_t kSmem = kSmemUsed + 1024;
    static_assert(kSmem <= 227 * 1024, "scan shared memory");
};

__device__ __forceinline__ void ldsm_x2_t(uint32_t& r0, uint32_t& r1, const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(smem_u32(p)));
}

// B fragments (k16 x n8 tiles nt = 0..NT8-1) of a [k][kHS] bf16 row-major tile, rows k0..k0+15.
template <int NT8, int HS>
__device__ __forceinline__ void load_b_frags(uint32_t (&b)[NT8][2], const uint16_t* tile, int k0, int lane) {
    if constexpr (NT8 == 1) {
        ldsm_x2_t(b[0][0], b[0][1], tile + (k0 + (lane & 15)) * HS);
    } else {
#pragma unroll
        for (int np = 0; np < NT8 / 2; ++np)
            ldsm_x4_t(b[2 * np][0], b[2 * np][1], b[2 * np + 1][0], b[2 * np + 1][1],
                      tile + (k0 + (lane & 7) + (((lane >> 3) & 1) << 3)) * HS + 16 * np + ((lane >> 4) << 3));
    }
}


template <int BV>
__global__ void __launch_bounds__(288, 1)
    gdn_prefill_scan2_kernel(PrefillArgs p, const __grid_constant__ PrefillMaps maps) {
    using C = Scan2Cfg<BV>;
    constexpr int NT8 = BV / 8;
    constexpr int HS = C::kHS;
    constexpr int kMathWarps = C::kMath / 32;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint16_t* Hb = reinterpret_cast<uint16_t*>(sm + C::kOffHb);
    uint16_t* VNh = reinterpret_cast<uint16_t*>(sm + C::kOffVh);
    uint16_t* VNl = reinterpret_cast<uint16_t*>(sm + C::kOffVl);
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + C::kOffBar);
    uint64_t* empty = full + C::kStages;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + C::kStages);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int gq = lane >> 2, tq = lane & 3;
    const int v0 = blockIdx.x * BV;
    const int hv = blockIdx.y % p.HV, hq = hv / (p.HV / p.H);
    pdl_wait();  // the workspace comes from the prep kernel, the inputs from earlier work
    pdl_trigger();
    // T == 0 with neither a chunk-table nor a prep launch: the scan is the call's only kernel
    if (p.T == 0 && p.small_n && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) p.status[0] = 0;
    // CTA rows: the longest sequence first (N <= 32), so the critical path starts in the first
    // wave; with the short path, the compacted list of the longer sequences.
    const int row_i = blockIdx.y / p.HV;
    const bool active = !p.short_path || row_i < p.long_list[p.N];
    const int n = p.short_path ? (active ? p.long_list[row_i] : 0)
                               : (p.small_n ? warp_seq_by_rank(p, row_i) : row_i);
    if (blockIdx.x == 0 && blockIdx.y == 0 && p.T > 0) {
        zero_unowned_tokens(p, tid, C::kThreads);
    }
    if (!active) return;
    int bos, eos;
    seq_bounds(p.cu, p.cu64, n, p.T, bos, eos);
    const int len = eos - bos;
    float* st_out = p.new_state + ((size_t)n * p.HV + hv) * kD * kD;
    if (len <= 0) {  // zero-length sequence: all-zero final state (reference/gdn_prefill_ref.py:52-54, 61-62)
        for (int idx = tid; idx < BV * kD; idx += C::kThreads) st_out[(size_t)(v0 + idx / kD) * kD + idx % kD] = 0.f;
        return;
    }
    if (p.short_path && len <= kShortLen) return;  // a short-sequence kernel owns it
    int slot0;
    if (p.small_n) {
        int dummy;
        warp_chunk_lookup(p, n, -1, &slot0, &dummy);  // every warp computes the same value
    } else {
        slot0 = p.chunk_base[n];
    }
    const int nchunks = clamp_chunks(p, slot0, (len + kChunk - 1) / kChunk, tid == 0);

    if (tid == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, kMathWarps);
        }
        *abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();
    if (warp == kMathWarps) {
        // Producer: refill stage c % 3 with chunk c once the math warps released chunk c - 3.
        if (lane == 0) {
            tma_prefetch_desc(&maps.w);
            tma_prefetch_desc(&maps.qp);
            tma_prefetch_desc(&maps.k);
            for (int c = 0; c < nchunks; ++c) {
                if (c >= C::kStages &&
                    !mbar_wait(empty + (c % C::kStages), (uint32_t)((c / C::kStages - 1) & 1), p.status,
                               kErrScanTmaTimeout))
                    break;  // the math warps stopped; they also stop waiting for more chunks
                if (p.test_withhold && c == 1) continue;  // test hook: this chunk's copies never arrive
                unsigned char* st = sm + (c % C::kStages) * C::kStage;
                uint64_t* bar = full + (c % C::kStages);
                const int wr = (slot0 + c) * kChunk, t0 = bos + c * kChunk;
                mbar_arrive_expect_tx(bar, C::kTxBytes);
                tma_load_3d(st + C::kOffW, &maps.w, 0, wr, hv, bar);
                tma_load_3d(st + C::kOffW + 8192, &maps.w, 64, wr, hv, bar);
                tma_load_3d(st + C::kOffQ, &maps.qp, 0, wr, hv, bar);
                tma_load_3d(st + C::kOffQ + 8192, &maps.qp, 64, wr, hv, bar);
                tma_load_3d(st + C::kOffK, &maps.k, 0, hq, t0, bar);
                tma_load_3d(st + C::kOffK + 8192, &maps.k, 64, hq, t0, bar);
                const int slot = slot0 + c;
                bulk_load(st + C::kOffU, p.u + cg_off(hv, p.S, slot, v0 / 8), 64 * BV * 4, bar);
                bulk_load(st + C::kOffO, p.oi + cg_off(hv, p.S, slot, v0 / 8), 64 * BV * 2, bar);
                bulk_load(st + C::kOffG, p.g4 + ((size_t)hv * p.S + slot) * kChunk * 4, 1024, bar);
            }
        }
        return;
    }

    // Math warp mw owns state rows (K dimension) 16 mw .. 16 mw + 15 as mma C fragments:
    // h[nt][e] = h[16 mw + gq + 8 (e >> 1)][8 nt + 2 tq + (e & 1)].
    const int mw = warp;
    float h[NT8][4];
    {
        const float* st_in = p.state ? p.state + ((size_t)n * p.HV + hv) * kD * kD : nullptr;
#pragma unroll
        for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int row = 16 * mw + gq + 8 * (e >> 1);
                const int col = 8 * nt + 2 * tq + (e & 1);
                h[nt][e] = st_in ? st_in[(size_t)(v0 + col) * kD + row] : 0.f;
            }
    }
    auto write_hb = [&]() {
#pragma unroll
        for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int row = 16 * mw + gq + 8 * half;
                *reinterpret_cast<uint32_t*>(Hb + row * HS + 8 * nt + 2 * tq) =
                    pack_bf16x2(h[nt][2 * half], h[nt][2 * half + 1]);
            }
    };
    write_hb();
    named_bar_sync(1, C::kMath);

    const bool dbg = blockIdx.x == 0 && blockIdx.y == 0 && mw == 0;
    long long tp = clock64();
    (void)dbg;
    const int prow0 = 16 * (mw & 3);  // rows of w h (warps 0-3) or Q' h (warps 4-7)
    const bool out_warp = mw >= 4;
    int c = 0;
    for (; c < nchunks; ++c) {
        if (!mbar_wait(full + (c % C::kStages), (uint32_t)((c / C::kStages) & 1), p.status, kErrScanTmaTimeout))
            *abort_flag = 1;  // checked by every math thread after the next barrier
        GDN_PH_ACC(dbg, 20, tp);
        const unsigned char* st = sm + (c % C::kStages) * C::kStage;
        const unsigned char* Ks = st + C::kOffK;
        const float* Us = reinterpret_cast<const float*>(st + C::kOffU);
        const uint16_t* Os = reinterpret_cast<const uint16_t*>(st + C::kOffO);
        const float* G4 = reinterpret_cast<const float*>(st + C::kOffG);
        const int t0 = bos + c * kChunk;
        const int L = min(kChunk, eos - t0);
        const float GL = G4[(L - 1) * 4];

        // (1) P = W h (warps 0-3) or Q' h (warps 4-7), rows prow0 .. +15; even / odd k-steps
        //     accumulate separately to halve the dependent-MMA chain.
        {
            const unsigned char* At = st + (out_warp ? C::kOffQ : C::kOffW);
            float pa[NT8][4], pb[NT8][4];
#pragma unroll
            for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) pa[nt][e] = pb[nt][e] = 0.f;
#pragma unroll
            for (int k0 = 0; k0 < 128; k0 += 16) {
                uint32_t a[4], b[NT8][2];
                ldsm_x4(a[0], a[1], a[2], a[3], At + sw128_off(prow0 + (lane & 15), k0 + ((lane >> 4) << 3), 8192));
                load_b_frags<NT8, HS>(b, Hb, k0, lane);
#pragma unroll
                for (int nt = 0; nt < NT8; ++nt) {
                    if ((k0 >> 4) & 1)
                        mma_bf16(pb[nt], a, b[nt][0], b[nt][1]);
                    else
                        mma_bf16(pa[nt], a, b[nt][0], b[nt][1]);
                }
            }
            GDN_PH_ACC(dbg, 21, tp);
            // (2) warps 0-3: vn = u - W h -> decayed vn (bf16 hi + lo) for the state update;
            //     warps 4-7: o = scale (Q' h + oi) -> out
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int row = prow0 + gq + 8 * half;
                if (!out_warp) {
                    // e^{G_L - G} <= 1 (padded rows have vn = 0), times 1 / |k| of the row's token
                    // with the in-kernel L2 norm (K is the raw k tile), else 1
                    const float ed = __expf(GL - G4[row * 4]) * G4[row * 4 + 3];
#pragma unroll
                    for (int nt = 0; nt < NT8; ++nt) {
                        const int col = 8 * nt + 2 * tq;
                        const float2 uu = *reinterpret_cast<const float2*>(Us + (col >> 3) * 512 + row * 8 + (col & 7));
                        const float d0 = (uu.x - (pa[nt][2 * half] + pb[nt][2 * half])) * ed;
                        const float d1 = (uu.y - (pa[nt][2 * half + 1] + pb[nt][2 * half + 1])) * ed;
                        const uint32_t hi = pack_bf16x2(d0, d1);
                        *reinterpret_cast<uint32_t*>(VNh + row * HS + col) = hi;
                        *reinterpret_cast<uint32_t*>(VNl + row * HS + col) =
                            pack_bf16x2(d0 - __uint_as_float(hi << 16), d1 - __uint_as_float(hi & 0xffff0000u));
                    }
                } else if (row < L) {
                    uint16_t* dst = p.out + ((size_t)(t0 + row) * p.HV + hv) * kD + v0;
#pragma unroll
                    for (int nt = 0; nt < NT8; ++nt) {
                        const int col = 8 * nt + 2 * tq;
                        const uint32_t oo = *reinterpret_cast<const uint32_t*>(Os + (col >> 3) * 512 + row * 8 + (col & 7));
                        *reinterpret_cast<uint32_t*>(dst + col) = pack_bf16x2(
                            p.scale * (pa[nt][2 * half] + pb[nt][2 * half] + __uint_as_float(oo << 16)),
                            p.scale * (pa[nt][2 * half + 1] + pb[nt][2 * half + 1] + __uint_as_float(oo & 0xffff0000u)));
                    }
                }
            }
        }
        GDN_PH_ACC(dbg, 22, tp);
        named_bar_sync(1, C::kMath);
        GDN_PH_ACC(dbg, 23, tp);
        if (*abort_flag) break;  // written only before this barrier: every math thread sees the same value

        // (3) h = e^{GL} h + K^T (vn_hi + vn_lo) for state rows 16 mw .. +15 (hi and lo parts
        //     accumulate separately, chain of 4 MMAs each)
        {
            float dh[NT8][4], dl[NT8][4];
#pragma unroll
            for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) dh[nt][e] = dl[nt][e] = 0.f;
#pragma unroll
            for (int k0 = 0; k0 < 64; k0 += 16) {
                uint32_t a[4], bh[NT8][2], bl[NT8][2];
                ldsm_x4_t(a[0], a[1], a[2], a[3],
                          Ks + sw128_off(k0 + (lane & 7) + ((lane >> 4) << 3), 16 * mw + (((lane >> 3) & 1) << 3), 8192));
                load_b_frags<NT8, HS>(bh, VNh, k0, lane);
                load_b_frags<NT8, HS>(bl, VNl, k0, lane);
#pragma unroll
                for (int nt = 0; nt < NT8; ++nt) {
                    mma_bf16(dh[nt], a, bh[nt][0], bh[nt][1]);
                    mma_bf16(dl[nt], a, bl[nt][0], bl[nt][1]);
                }
            }
            const float eL = __expf(GL);
#pragma unroll
            for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) h[nt][e] = fmaf(eL, h[nt][e], dh[nt][e] + dl[nt][e]);
        }
        GDN_PH_ACC(dbg, 24, tp);
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + (c % C::kStages));  // this warp is done with the stage
        write_hb();
        named_bar_sync(1, C::kMath);
        GDN_PH_ACC(dbg, 25, tp);
    }
    if (c < nchunks) {
        // A TMA wait gave up: let copies already in flight land (bounded) before the CTA exits.
        if (tid == 0)
            for (int cc = c + 1; cc < min(nchunks, c + C::kStages); ++cc)
                mbar_wait(full + (cc % C::kStages), (uint32_t)((cc / C::kStages) & 1), nullptr, 0);
        return;
    }

    // final state (k-last): new_state[n][hv][v0 + col][row]
#pragma unroll
    for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int row = 16 * mw + gq + 8 * (e >> 1);
            const int col = 8 * nt + 2 * tq + (e & 1);
            st_out[(size_t)(v0 + col) * kD + row] = h[nt][e];
        }
}

template <int BV>
static int launch_scan_bv(const PrefillArgs& p, const PrefillMaps& maps, cudaStream_t stream) {
    using C = Scan2Cfg<BV>;
    if (cudaFuncSetAttribute(gdn_prefill_scan2_kernel<BV>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem) !=
        cudaSuccess)
        return -1;
    dim3 grid(kD / BV, p.rows * p.HV);
    return launch_pdl(gdn_prefill_scan2_kernel<BV>, grid, dim3(C::kThreads), C::kSmem, stream, p, maps) ==
                   cudaSuccess
               ? 0
               : -1;
}

int launch_prefill_scan(const PrefillArgs& p, const PrefillMaps& maps, int bv, cudaStream_t stream) {
    switch (bv) {
        case 8: return launch_scan_bv<8>(p, maps, stream);
        case 16: return launch_scan_bv<16>(p, maps, stream);
        case 32: return launch_scan_bv<32>(p, maps, stream);
        default: return -2;
    }
}

}  // namespace gdn
