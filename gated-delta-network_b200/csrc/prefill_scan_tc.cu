// prefill_scan_tc.cu -- serial half of the chunked prefill on tcgen05 tensor cores, for batches
// of many sequences (throughput regime).
//
// Same recurrence as prefill_scan.cu (per chunk: vn = u - w h, o = scale (Q' h + oi),
// h = e^{G_last} h + K^T (e^{G_last - G} . vn)), one CTA per (64-column slice of the state,
// sequence, v-head).  With warp-level mma.sync every warp has to load its own copy of the
// h / vn operand fragments, and for wide slices that replicated shared-memory traffic sets the
// per-chunk time; here each product is one tcgen05 MMA that reads its operands from shared
// memory once:
//   MMA_P  [W; Q'] (128 x 128, K-major)  x  h (128 x 64, MN-major bf16)  -> TMEM P (64 columns)
//            rows 0-63 of P = w h, rows 64-127 = Q' h
//   MMA_U  K^T (128 x 64 tokens, MN-major straight from the k tile)  x  [vn_hi; vn_lo]
//            (64 tokens x 64, MN-major bf16, two accumulating MMAs)   -> TMEM D (64 columns)
// Two math warps per TMEM lane quarter split its 64 columns: thread (r, half) owns lane r and
// columns 32 half .. +31.  After MMA_P, rows r < 64 form the decayed vn (bf16 hi + lo, as in
// prefill_scan.cu) and rows r >= 64 the outputs; after MMA_U, the thread owns those 32 columns
// of state row r (fp32 registers), updates them and writes their bf16 copy (the next MMA_P's
// B operand).  A producer warp keeps a 2-stage TMA ring of the chunk operands.  Each chunk is a
// chain of two MMA round trips, so a chunk takes longer than in the mma.sync scan, but a CTA
// covers 64 state columns instead of 8-32: this kernel serves batches whose scan is bound by
// throughput rather than by the length of one sequence.
#include "prefill_kernels.cuh"
#include "sm100.cuh"
#include "dbg.cuh"

GDN_DBG_READER(gdn_debug_read_scan_tc)

namespace gdn {

namespace tcs {
constexpr int BV = 64;               // state columns per CTA
constexpr int kThreads = 288;        // 8 math warps (two per TMEM lane quarter) + 1 producer warp
constexpr int kMath = 256;
constexpr int kStages = 2;
constexpr uint32_t kOffWQ = 0;       // [W0 | Q'0 | W1 | Q'1], 8 KB each: [W; Q'] is one 128-row operand
constexpr uint32_t kOffK = 32768;    // k tile: 2 atoms (K columns 0-63, 64-127) of 64 tokens x 128 B
constexpr uint32_t kOffU = 49152;    // [8 column groups][64][8] f32
constexpr uint32_t kOffO = kOffU + 64 * BV * 4;  // [8][64][8] bf16
constexpr uint32_t kOffG = kOffO + 64 * BV * 2;  // [64][4] f32 {G, e^G, beta, rk}
constexpr uint32_t kStage = ((kOffG + 1024) + 1023) & ~1023u;
constexpr uint32_t kTxBytes = 4 * 8192 + 2 * 8192 + 64 * BV * 6 + 1024;
constexpr uint32_t kOffHb = kStages * kStage;        // h, bf16 [128 K rows][64], SW128 (MN-major B)
constexpr uint32_t kOffVh = kOffHb + 128 * 128;      // vn hi, bf16 [64 tokens][64], SW128
constexpr uint32_t kOffVl = kOffVh + 64 * 128;       // vn lo
constexpr uint32_t kOffOb = kOffVl + 64 * 128;       // output staging, bf16 [64 tokens][64], 16-byte chunks swizzled
constexpr uint32_t kOffBar = kOffOb + 64 * 128;      // full[2], empty[2], mma_p, mma_u, abort flag, TMEM slot, next item
constexpr uint32_t kSmemUsed = kOffBar + 8 * (2 * kStages + 2) + 16;
constexpr uint32_t kSmem = kSmemUsed + 1024;
constexpr uint32_t kTmemCols = 128;                  // P: columns 0-63, D: 64-127
static_assert(kSmem <= 227 * 1024, "scan shared memory");
}  // namespace tcs

__global__ void __launch_bounds__(tcs::kThreads, 1)
    gdn_prefill_scan_tc_kernel(PrefillArgs p, const __grid_constant__ PrefillMaps maps) {
    using namespace tcs;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(sm);
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + kOffBar);
    uint64_t* empty = full + kStages;
    uint64_t* bar_p = empty + kStages;
    uint64_t* bar_u = bar_p + 1;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bar_u + 1);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bar_u + 1) + 1;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    pdl_wait();  // the workspace comes from the prep kernel, the inputs from earlier work
    pdl_trigger();
    // T == 0 with neither a chunk-table nor a prep launch: the scan is the call's only kernel
    if (p.T == 0 && p.small_n && blockIdx.x == 0 && threadIdx.x == 0) p.status[0] = 0;
    if (blockIdx.x == 0) zero_unowned_tokens(p, tid, kThreads);
    // Work items: item = (row_i * HV + hv) * 2 + column half.  CTA rows are the longest sequence
    // first (N <= 32), or with the short path the compacted list of the longer sequences (as in
    // prefill_scan.cu).  Without the short path the grid holds one CTA per item; with it, the
    // number of rows is known only on the device, so a grid of at most one CTA per SM takes
    // items from a counter (status word 1, zeroed by the chunk-table kernel) until they run out,
    // instead of launching CTAs that would only find their row empty.
    const bool persistent = p.short_path != 0;
    const int rows_valid = p.short_path ? p.long_list[p.N] : p.rows;
    int* item_slot = reinterpret_cast<int*>(tslot + 1);

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, kMath / 32);
        }
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

    uint32_t cbase = 0;  // chunks this CTA has run through the ring so far
    int item = blockIdx.x;
    for (;;) {
        const int row_i = (item >> 1) / p.HV;
        if (row_i >= rows_valid) break;  // uniform across the CTA
        const int v0 = (item & 1) * BV;
        const int hv = (item >> 1) % p.HV, hq = hv / (p.HV / p.H);
        const int n = p.short_path ? p.long_list[row_i] : (p.small_n ? warp_seq_by_rank(p, row_i) : row_i);
        int bos, eos;
        seq_bounds(p.cu, p.cu64, n, p.T, bos, eos);
        const int len = eos - bos;
        float* st_out = p.new_state + ((size_t)n * p.HV + hv) * kD * kD;
        // zero-length sequence: all-zero final state (reference/gdn_prefill_ref.py:52-54, 61-62);
        // with the short path a short-sequence kernel owns the sequences of up to kShortLen tokens
        int nchunks = (len <= 0 || (p.short_path && len <= kShortLen)) ? 0 : (len + kChunk - 1) / kChunk;
        if (len <= 0)
            for (int idx = tid; idx < BV * kD; idx += kThreads) st_out[(size_t)(v0 + idx / kD) * kD + idx % kD] = 0.f;
        int slot0 = 0;
        if (nchunks > 0) {
            if (p.small_n) {
                int dummy;
                warp_chunk_lookup(p, n, -1, &slot0, &dummy);
            } else {
                slot0 = p.chunk_base[n];
            }
            nchunks = clamp_chunks(p, slot0, nchunks, tid == 0);
        }
        if (nchunks > 0) {
            if (warp == kMath / 32) {
                // Producer: refill stage c % 2 with chunk c once the math warps released chunk c - 2.
                if (lane == 0) {
                    tma_prefetch_desc(&maps.w);
                    tma_prefetch_desc(&maps.qp);
                    tma_prefetch_desc(&maps.k);
                    for (int c = 0; c < nchunks; ++c) {
                        if (cbase + c >= kStages && !mbar_wait(empty + ((cbase + c) % kStages), (uint32_t)(((cbase + c) / kStages - 1) & 1), p.status,
                                                       kErrScanTmaTimeout))
                            break;
                        if (p.test_withhold && c == 1) continue;  // test hook: this chunk's copies never arrive
                        unsigned char* st = sm + ((cbase + c) % kStages) * kStage;
                        uint64_t* bar = full + ((cbase + c) % kStages);
                        const int slot = slot0 + c, wr = slot * kChunk, t0 = bos + c * kChunk;
                        mbar_arrive_expect_tx(bar, kTxBytes);
                        tma_load_3d(st + kOffWQ, &maps.w, 0, wr, hv, bar);
                        tma_load_3d(st + kOffWQ + 8192, &maps.qp, 0, wr, hv, bar);
                        tma_load_3d(st + kOffWQ + 16384, &maps.w, 64, wr, hv, bar);
                        tma_load_3d(st + kOffWQ + 24576, &maps.qp, 64, wr, hv, bar);
                        tma_load_3d(st + kOffK, &maps.k, 0, hq, t0, bar);
                        tma_load_3d(st + kOffK + 8192, &maps.k, 64, hq, t0, bar);
                        bulk_load(st + kOffU, p.u + cg_off(hv, p.S, slot, v0 / 8), 64 * BV * 4, bar);
                        bulk_load(st + kOffO, p.oi + cg_off(hv, p.S, slot, v0 / 8), 64 * BV * 2, bar);
                        bulk_load(st + kOffG, p.g4 + ((size_t)hv * p.S + slot) * kChunk * 4, 1024, bar);
                    }
                }
            } else {
                // ---- math warps: thread (r, half) = TMEM lane r, columns 32 half .. 32 half + 31 ----
                // Warps w and w + 4 share TMEM lane quarter w (lanes 32 w .. 32 w + 31) and split its
                // 64 columns, so every per-element epilogue is spread over eight warps.
                const int r = lane + 32 * (warp & 3), half = warp >> 2;
                const uint32_t tl = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + 32u * half;
                float h[32];  // state row r (K index), columns v0 + 32 half + j
                {
                    const float* st_in = p.state ? p.state + ((size_t)n * p.HV + hv) * kD * kD : nullptr;
#pragma unroll
                    for (int j = 0; j < 32; ++j) h[j] = st_in ? st_in[(size_t)(v0 + 32 * half + j) * kD + r] : 0.f;
                }
                // bf16 copy of h into the MN-major SW128 operand: 128-byte rows, 16-byte chunks
                // XOR-swizzled by row % 8; this thread owns chunks 4 half .. 4 half + 3 of row r
                auto write_hb = [&]() {
                    unsigned char* row = sm + kOffHb + r * 128;
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj) {
                        const int j = 4 * half + jj;
                        *reinterpret_cast<uint4*>(row + ((j ^ (r & 7)) << 4)) =
                            make_uint4(pack_bf16x2(h[8 * jj], h[8 * jj + 1]), pack_bf16x2(h[8 * jj + 2], h[8 * jj + 3]),
                                       pack_bf16x2(h[8 * jj + 4], h[8 * jj + 5]), pack_bf16x2(h[8 * jj + 6], h[8 * jj + 7]));
                    }
                };
                write_hb();
                const bool dbg = blockIdx.x == 0;
                long long tp = clock64();
                (void)dbg;
                constexpr uint32_t idesc_p = umma_idesc_bf16(128, BV, false, true);
                constexpr uint32_t idesc_u = umma_idesc_bf16(128, BV, true, true);
                int c = 0;
                for (; c < nchunks; ++c) {
                    const uint32_t g = cbase + c;  // running chunk count of the CTA: ring stage and barrier phases
                    if (!mbar_wait(full + (g % kStages), (uint32_t)((g / kStages) & 1), p.status, kErrScanTmaTimeout))
                        *abort_flag = 1;
                    fence_async_smem();  // this thread's h copy (generic stores) -> the tensor core
                    tc_fence_before();
                    named_bar_sync(1, kMath);
                    if (*abort_flag) break;  // written only before this barrier
                    tc_fence_after();
                    GDN_PH_ACC(dbg, 20, tp);
                    const unsigned char* st = sm + (g % kStages) * kStage;
                    const uint32_t sst = sbase + (uint32_t)(g % kStages) * kStage;
                    const float* G4 = reinterpret_cast<const float*>(st + kOffG);
                    const int t0 = bos + c * kChunk;
                    const int L = min(kChunk, eos - t0);
                    const float GL = G4[(L - 1) * 4];
                    // MMA_P: [W; Q'] x h
                    if (tid == 0) {
#pragma unroll
                        for (int kk = 0; kk < 8; ++kk)
                            umma_bf16(tmem, umma_desc_sw128(sst + kOffWQ + (uint32_t)(kk >> 2) * 16384u + (uint32_t)(kk & 3) * 32u, 16, 1024),
                                      umma_desc_sw128(sbase + kOffHb + 2048u * kk, 8192, 1024), idesc_p, kk > 0);
                        umma_commit(bar_p);
                    }
                    bool ok = mbar_wait(bar_p, g & 1u, p.status, kErrScanMmaTimeout);
                    tc_fence_after();
                    GDN_PH_ACC(dbg, 21, tp);
                    {
                        uint32_t d[32];
                        tmem_ld32_async(tl, d);
                        tmem_ld_wait();
                        tmem_regs_ready(d);
                        GDN_PH_ACC(dbg, 25, tp);
                        if (r < 64) {
                            // vn = (u - w h) e^{G_L - G_r} / |k_r|  -> bf16 hi + lo (MN-major SW128, token row r)
                            const float4 g4r = *reinterpret_cast<const float4*>(G4 + r * 4);  // {G, e^G, beta, rk}
                            const float ed = __expf(GL - g4r.x) * g4r.w;
                            const float* Us = reinterpret_cast<const float*>(st + kOffU);
                            unsigned char* rh = sm + kOffVh + r * 128;
                            unsigned char* rl = sm + kOffVl + r * 128;
                            // Row r's 8 u values are 32 contiguous bytes.  Threads with bit 2 of r set
                            // read the upper 16 bytes first, so each 8-thread phase of a 16-byte load
                            // touches 8 different bank groups (no 2-way conflict).
                            const int hA = (r >> 2) & 1;
#pragma unroll
                            for (int jj = 0; jj < 4; ++jj) {
                                const int j = 4 * half + jj;
                                const float4 x0 = *reinterpret_cast<const float4*>(Us + (j * 64 + r) * 8 + 4 * hA);
                                const float4 x1 = *reinterpret_cast<const float4*>(Us + (j * 64 + r) * 8 + 4 * (hA ^ 1));
                                const float4 ua = hA ? x1 : x0;
                                const float4 ub = hA ? x0 : x1;
                                const float uu[8] = {ua.x, ua.y, ua.z, ua.w, ub.x, ub.y, ub.z, ub.w};
                                uint32_t hi[4], lo[4];
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    const float2 x = mul2(sub2(make_float2(uu[2 * e], uu[2 * e + 1]),
                                                               make_float2(__uint_as_float(d[8 * jj + 2 * e]),
                                                                           __uint_as_float(d[8 * jj + 2 * e + 1]))),
                                                          make_float2(ed, ed));
                                    hi[e] = pack_bf16x2(x.x, x.y);
                                    const float2 r2 = sub2(x, make_float2(__uint_as_float(hi[e] << 16), __uint_as_float(hi[e] & 0xffff0000u)));
                                    lo[e] = pack_bf16x2(r2.x, r2.y);
                                }
                                *reinterpret_cast<uint4*>(rh + ((j ^ (r & 7)) << 4)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                                *reinterpret_cast<uint4*>(rl + ((j ^ (r & 7)) << 4)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                            }
                            GDN_PH_ACC(dbg, 22, tp);
                            // warps 0, 1, 4, 5 alone gate MMA_U: the output rows are not on its path
                            fence_async_smem();  // vn (generic stores) -> the tensor core
                            tc_fence_before();
                            const bool okv = named_bar_and(2, 128, ok);
                            tc_fence_after();
                            // MMA_U: K^T x (vn_hi + vn_lo), accumulated in TMEM columns 64-127
                            if (okv && tid == 0) {
#pragma unroll
                                for (int kk = 0; kk < 4; ++kk)
                                    umma_bf16(tmem + BV, umma_desc_sw128(sst + kOffK + 2048u * kk, 8192, 1024),
                                              umma_desc_sw128(sbase + kOffVh + 2048u * kk, 8192, 1024), idesc_u, kk > 0);
#pragma unroll
                                for (int kk = 0; kk < 4; ++kk)
                                    umma_bf16(tmem + BV, umma_desc_sw128(sst + kOffK + 2048u * kk, 8192, 1024),
                                              umma_desc_sw128(sbase + kOffVl + 2048u * kk, 8192, 1024), idesc_u, true);
                                umma_commit(bar_u);
                            }
                            ok = okv;
                        } else {
                            // o = scale (Q' h + oi) for token row m = r - 64, while MMA_U runs.  Rows are
                            // staged in shared memory and then written row-contiguously (a 16-byte store
                            // per thread, eight threads per 128-byte row): one thread per row writing its
                            // own 64 bytes would spread every store instruction over 32 rows.
                            const int m = r - 64;
                            const uint16_t* Os = reinterpret_cast<const uint16_t*>(st + kOffO);
                            unsigned char* ob = sm + kOffOb + m * 128;
#pragma unroll
                            for (int jj = 0; jj < 4; ++jj) {
                                const int j = 4 * half + jj;
                                const uint4 oo = *reinterpret_cast<const uint4*>(Os + (j * 64 + m) * 8);
                                const uint32_t ow[4] = {oo.x, oo.y, oo.z, oo.w};
                                uint32_t pk[4];
#pragma unroll
                                for (int e = 0; e < 4; ++e)
                                {
                                    const float2 o2 = mul2(make_float2(p.scale, p.scale),
                                                           add2(make_float2(__uint_as_float(d[8 * jj + 2 * e]), __uint_as_float(d[8 * jj + 2 * e + 1])),
                                                                make_float2(__uint_as_float(ow[e] << 16), __uint_as_float(ow[e] & 0xffff0000u))));
                                    pk[e] = pack_bf16x2(o2.x, o2.y);
                                }
                                *reinterpret_cast<uint4*>(ob + ((j ^ (m & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                            }
                            named_bar_sync(3, 128);  // the four output warps
                            const int ot = (warp & 1) * 32 + lane + 64 * half;  // 0 .. 127
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                const int row = 16 * q + (ot >> 3), ch = ot & 7;
                                if (row < L) {
                                    const uint4 v = *reinterpret_cast<const uint4*>(sm + kOffOb + row * 128 + ((ch ^ (row & 7)) << 4));
                                    *reinterpret_cast<uint4*>(p.out + ((size_t)(t0 + row) * p.HV + hv) * kD + v0 + 8 * ch) = v;
                                }
                            }
                        }
                    }
                    // an MMA_U that was not issued (a wait gave up) also fails this bounded wait
                    if (ok) ok = mbar_wait(bar_u, g & 1u, p.status, kErrScanMmaTimeout);
                    tc_fence_after();
                    GDN_PH_ACC(dbg, 23, tp);
                    {
                        uint32_t d[32];
                        tmem_ld32_async(tl + BV, d);
                        tmem_ld_wait();
                        tmem_regs_ready(d);
                        const float eL = __expf(GL);
#pragma unroll
                        for (int j = 0; j < 32; j += 2) {  // lane-paired fp32, same values as fmaf per element
                            const float2 hn = fma2(make_float2(eL, eL), make_float2(h[j], h[j + 1]),
                                                   make_float2(__uint_as_float(d[j]), __uint_as_float(d[j + 1])));
                            h[j] = hn.x;
                            h[j + 1] = hn.y;
                        }
                    }
                    // the stage's smem operands and TMEM results are consumed: hand the stage back
                    __syncwarp();
                    if (lane == 0) mbar_arrive(empty + (g % kStages));
                    if (!ok) *abort_flag = 1;
                    write_hb();
                    GDN_PH_ACC(dbg, 24, tp);
                }
                if (c < nchunks) {
                    // gave up: let copies already in flight land (bounded) before the CTA exits
                    if (tid == 0)
                        for (int cc = c + 1; cc < min(nchunks, c + kStages); ++cc)
                            mbar_wait(full + ((cbase + cc) % kStages), (uint32_t)(((cbase + cc) / kStages) & 1), nullptr, 0);
                } else {
                    // final state (k-last): new_state[n][hv][v0 + 32 half + j][r]
#pragma unroll
                    for (int j = 0; j < 32; ++j) st_out[(size_t)(v0 + 32 * half + j) * kD + r] = h[j];
                }
            }
        }
        cbase += (uint32_t)nchunks;
        // next item: every warp is done with this one (operands, TMEM, the h copy)
        tc_fence_before();
        __syncthreads();
        if (*abort_flag || !persistent) break;
        if (tid == 0) *item_slot = (int)gridDim.x + atomicAdd(p.status + 1, 1);
        __syncthreads();
        tc_fence_after();
        item = *item_slot;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

int launch_prefill_scan_tc(const PrefillArgs& p, const PrefillMaps& maps, cudaStream_t stream) {
    using namespace tcs;
    if (cudaFuncSetAttribute(gdn_prefill_scan_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) !=
        cudaSuccess)
        return -1;
    const long long items = (long long)p.rows * p.HV * (kD / BV);
    long long ctas = items;
    if (p.short_path) {  // at most one CTA per SM, taking items from the counter
        int dev = 0, sms = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return -1;
        ctas = std::min<long long>(items, sms);
    }
    dim3 grid((unsigned)std::max<long long>(ctas, 1));
    return launch_pdl(gdn_prefill_scan_tc_kernel, grid, dim3(kThreads), kSmem, stream, p, maps) == cudaSuccess ? 0
                                                                                                                 : -1;
}

}  // namespace gdn
