// prefill_prep.cu -- chunk-parallel half of the chunked Gated DeltaNet prefill (sm_100a).
//
// One CTA per (64-token chunk slot, v-head), 256 threads, two CTAs per SM.  For the chunk's
// tokens t = bos .. bos+L-1 of v-head hv (q/k head hv/2) it computes, following the chunked
// WY form of solutions/gdn_prefill_qk4_v8_d128_k_last/solution/triton/fla_kernels.py
// (cumsum + K K^T 858-905, solve_tril 197-314, recompute_w_u 334-383):
//   G_i   = sum_{t<=i} g_t              g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b)
//   A_ij  = beta_i e^{G_i-G_j} k_i.k_j  (i > j)          Aqk_ij = e^{G_i-G_j} q_i.k_j  (i >= j)
//   T     = (I + A)^-1
//   w     = T diag(beta e^G) K          u = beta v + (T - I) diag(beta) V
// Data path:
//   * TMA (SWIZZLE_128B boxes, no multicast) brings K, Q (qk head) and V (v-head) tiles.
//   * tcgen05 MMA #1 (M=128, N=64, K=128): [K; Q] x K^T -> TMEM, rows 0-63 K K^T, 64-127 Q K^T.
//   * Epilogue: one thread per TMEM lane turns its row into a row of A (fp32, shared memory)
//     or of Aqk (bf16, shared memory, operand of MMA #3).
//   * T = (I + A)^-1: 16x16 diagonal blocks by forward substitution (one column per lane),
//     off-diagonal blocks T_ib,jb = -T_ib,ib sum_k A_ib,k T_k,jb with tf32 mma.sync.
//   * tcgen05 MMA #2 (M=128, N=256, K=64): [T diag(beta e^G); (T - I) diag(beta)] x [K | V]
//     -> TMEM; rows 0-63 / columns 0-127 are w, rows 64-127 / columns 128-255 are u - beta v.
//   * tcgen05 MMA #3 (M=128, N=256, K=64): [Aqk; Aqk] x [w | u] -> TMEM; rows 0-63 / columns
//     0-127 are Aqk w, rows 64-127 / columns 128-255 are Aqk u.  They give the chunk's output
//     operands Q' = diag(e^G) Q - Aqk w and oi = Aqk u, so the serial scan needs only
//     o = scale (Q' h + oi) (the Aqk (u - w h) term of chunk_o, fla_kernels.py:758-796).
//   * Outputs go to the chunk's workspace slot; rows past the chunk end carry zero / finite padding.
#include <algorithm>

#include "prefill_kernels.cuh"
#include "sm100.cuh"
#include "dbg.cuh"

GDN_DBG_READER(gdn_debug_read_prep)

namespace gdn {
namespace prep2 {
constexpr int kThreads = 256;  // 8 warps: warps w and w+4 share TMEM lane quarter w % 4
constexpr int kFS = 68;  // fp32 row stride of A / T (rows stay 16-byte aligned)
constexpr uint32_t kOffK0 = 0;        // K cols 0-63   (64 rows x 128 B, SW128)
constexpr uint32_t kOffQ0 = 8192;     // Q cols 0-63   -> [K;Q] is one 128-row operand
constexpr uint32_t kOffK1 = 16384;    // K cols 64-127
constexpr uint32_t kOffQ1 = 24576;    // Q cols 64-127
constexpr uint32_t kOffV0 = 32768;    // V cols 0-63   -> K0, K1, V0, V1 are 16 KB apart
constexpr uint32_t kOffMisc = 40960;  // 8 KB: scratch, gates, barriers
constexpr uint32_t kOffV1 = 49152;    // V cols 64-127
constexpr uint32_t kOffA = 57344;     // A fp32 [64][68]; later [Wb; Ub] bf16 [128][64] SW128
constexpr uint32_t kOffT = kOffA + 64 * kFS * 4;  // T fp32 [64][68]
constexpr uint32_t kOffAq = kOffT + 64 * kFS * 4;  // [Aqk; Aqk] bf16 [128][64] SW128 (1024-aligned)
constexpr uint32_t kSmemUsed = kOffAq + 16384;
constexpr uint32_t kSmem = kSmemUsed + 1024;  // slack for 1024-byte alignment
// inside the misc block
constexpr uint32_t kOffTileA = 0;                 // [64 tokens][8 heads] bf16 a tile (TMA)
constexpr uint32_t kOffTileB = 1024;             // [64][8] bf16 b tile (TMA)
constexpr uint32_t kOffG = 2048;
constexpr uint32_t kOffB = kOffG + 64 * 4;
constexpr uint32_t kOffE = kOffB + 64 * 4;
constexpr uint32_t kOffGf = kOffE + 64 * 4;    // [64] f32 final cumulative log decay
constexpr uint32_t kOffBt = kOffGf + 64 * 4;   // [64] f32 exp(G_r(j) - G_j), r(j) = last token of j's 16-block
constexpr uint32_t kOffRq = kOffBt + 64 * 4;   // [64] f32 1 / |q_t| (in-kernel L2 norm), else 1
constexpr uint32_t kOffRk = kOffRq + 64 * 4;   // [64] f32 1 / |k_t|, else 1
constexpr uint32_t kOffWf = kOffRk + 64 * 4;   // [64] f32 beta e^G / |k| (column scale of w's operand)
constexpr uint32_t kOffBar = kOffWf + 64 * 4;  // 3 mbarriers
constexpr uint32_t kOffSlot = kOffBar + 32;
static_assert(kOffSlot + 16 <= 8192, "misc block");
constexpr uint32_t kTmemCols = 256;
}  // namespace prep2

__device__ __forceinline__ uint32_t to_tf32(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}
__device__ __forceinline__ void mma_tf32(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// C += A B for 16 x 16 fp32 blocks in shared memory (row stride kFS), tf32 MMAs, one warp.
// acc[nt] is the m16n8 C fragment of columns 8 nt .. 8 nt + 7.
__device__ __forceinline__ void mma16_tf32(float (&acc)[2][4], const float* A, const float* B, int gq, int tq) {
    using prep2::kFS;
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
        const float* As_ = A + 8 * ks;
        const uint32_t a[4] = {to_tf32(As_[gq * kFS + tq]), to_tf32(As_[(gq + 8) * kFS + tq]),
                               to_tf32(As_[gq * kFS + tq + 4]), to_tf32(As_[(gq + 8) * kFS + tq + 4])};
        const float* Bm = B + (8 * ks) * kFS;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
            mma_tf32(acc[nt], a, to_tf32(Bm[tq * kFS + 8 * nt + gq]), to_tf32(Bm[(tq + 4) * kFS + 8 * nt + gq]));
    }
}

// body(cb, d) for this thread's two 32-column TMEM blocks cb0 and cb0 + 1 (taddr0 = block cb0):
// the second block's load is in flight while the first block is processed.
template <typename F>
__device__ __forceinline__ void tmem_two_blocks(uint32_t taddr0, int cb0, F&& body) {
    uint32_t da[32], db[32];
    tmem_ld32_async(taddr0, da);
    tmem_ld_wait();
    tmem_regs_ready(da);
    tmem_ld32_async(taddr0 + 32, db);
    body(cb0, da);
    tmem_ld_wait();
    tmem_regs_ready(db);
    body(cb0 + 1, db);
}

__global__ void __launch_bounds__(prep2::kThreads, 2)
    gdn_prefill_prep2_kernel(PrefillArgs p, const __grid_constant__ PrefillMaps maps) {
    using namespace prep2;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(sm);
    float* Af = reinterpret_cast<float*>(sm + kOffA);
    float* Tf = reinterpret_cast<float*>(sm + kOffT);
    unsigned char* misc = sm + kOffMisc;
    float* Gs = reinterpret_cast<float*>(misc + kOffG);
    float* Bs = reinterpret_cast<float*>(misc + kOffB);
    float* Es = reinterpret_cast<float*>(misc + kOffE);
    float* Gf = reinterpret_cast<float*>(misc + kOffGf);
    float* Bt = reinterpret_cast<float*>(misc + kOffBt);
    float* Rq = reinterpret_cast<float*>(misc + kOffRq);
    float* Rk = reinterpret_cast<float*>(misc + kOffRk);
    float* Wf = reinterpret_cast<float*>(misc + kOffWf);
    uint64_t* bar_load = reinterpret_cast<uint64_t*>(misc + kOffBar);
    uint64_t* bar_mma = bar_load + 1;
    uint64_t* bar_gate = bar_load + 2;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(misc + kOffSlot);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int gq = lane >> 2, tq = lane & 3;
    // Row-per-thread epilogues: thread rr owns TMEM lane / row rr, the two warpgroups split the
    // columns (ch_half 0 / 1).  Warp w reads TMEM lane quarter w % 4.
    const int rr = tid & 127, ch_half = tid >> 7, wq = warp & 3;
    if (tid == 0) {  // descriptors are kernel parameters: fetch them while the previous kernel drains
        tma_prefetch_desc(&maps.q);
        tma_prefetch_desc(&maps.k);
        tma_prefetch_desc(&maps.v);
        if (p.gates_tma) {
            tma_prefetch_desc(&maps.a);
            tma_prefetch_desc(&maps.b);
        }
    }
    pdl_wait();  // inputs and the chunk table come from earlier work on the stream
    // Without a chunk-table kernel this is the call's first kernel: reset the status word here,
    // before any bounded wait of this grid can record a code (a wait gives up only after 2 s,
    // and CTA 0 is in the first wave).
    if (p.small_n && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) p.status[0] = 0;
    // Work items: (chunk slot, v-head).  Without the short path the grid holds one CTA per item.
    // With it, how many slots the longer sequences own is known only on the device (the chunk
    // table's total), so a grid of at most two CTAs per SM takes items from a counter (status
    // word 2, zeroed by the chunk-table kernel), slot-major, until they run out.
    const bool persistent = p.short_path != 0;
    // (the table's total can exceed the S workspace slots only for a cu_seqlens that is not
    // non-decreasing; slots past S do not exist and are skipped)
    const int items_valid = persistent ? min(p.chunk_base[p.N], p.S) * p.HV : 0;
    int* item_slot = reinterpret_cast<int*>(tslot + 1);
    uint32_t done = 0;  // chunks this CTA has processed: phase of every mbarrier
    int item = blockIdx.x;
    for (;;) {
        int slot, hv;
        if (persistent) {
            if (item >= items_valid) break;
            slot = item / p.HV;
            hv = item % p.HV;
        } else {
            slot = blockIdx.x;
            hv = blockIdx.y;
        }
        const int hq = hv / (p.HV / p.H);
        const uint32_t ph = done & 1u;
        bool item_ok = true;
        int seq, cbase;
        if (p.small_n) {
            // warp 0 finds the slot's sequence; the result is published through shared memory
            __shared__ int s_lookup[2];
            if (warp == 0) {
                int base_dummy, sq;
                warp_chunk_lookup(p, 0, slot, &base_dummy, &sq);
                int cb = 0;
                if (sq >= 0) warp_chunk_lookup(p, sq, -1, &cb, &base_dummy);
                if (lane == 0) {
                    s_lookup[0] = sq;
                    s_lookup[1] = cb;
                }
            }
            __syncthreads();
            seq = s_lookup[0];
            cbase = s_lookup[1];
        } else {
            seq = p.chunk_seq[slot];
            cbase = seq >= 0 ? p.chunk_base[seq] : 0;
        }
        int s0 = 0, e0 = 0;
        if (seq >= 0) seq_bounds(p.cu, p.cu64, seq, p.T, s0, e0);
        // an unused slot, or (short path) a sequence that a short-sequence kernel owns: no work
        // (uniform across the CTA)
        if (seq >= 0 && !(p.short_path && e0 - s0 <= kShortLen)) {
            const int bos = s0 + (slot - cbase) * kChunk;
            const int L = min(kChunk, e0 - bos);
            const size_t row0 = (size_t)hv * p.S * kChunk + (size_t)slot * kChunk;  // workspace row of token bos
            long long tp = clock64();
            const bool dbg = true;
            (void)dbg;

            // ---- 1. barriers, TMA loads, TMEM -----------------------------------------------------
            // Thread 0 issues the tile loads first thing (the small gate tiles first, on their own
            // barrier); the other threads touch the barriers only after the block barrier below, by
            // which time their initialisation is visible.
            if (tid == 0) {
                if (done == 0) {
                    mbar_init(bar_load, 1);
                    mbar_init(bar_mma, 1);
                    mbar_init(bar_gate, 1);
                    mbar_fence_init();
                }
                if (p.gates_tma) {
                    mbar_arrive_expect_tx(bar_gate, 2 * 1024);
                    tma_load_2d(misc + kOffTileA, &maps.a, hv & ~7, bos, bar_gate);
                    tma_load_2d(misc + kOffTileB, &maps.b, hv & ~7, bos, bar_gate);
                }
                mbar_arrive_expect_tx(bar_load, 6 * 8192);
                tma_load_3d(sm + kOffK0, &maps.k, 0, hq, bos, bar_load);
                tma_load_3d(sm + kOffK1, &maps.k, 64, hq, bos, bar_load);
                tma_load_3d(sm + kOffQ0, &maps.q, 0, hq, bos, bar_load);
                tma_load_3d(sm + kOffQ1, &maps.q, 64, hq, bos, bar_load);
                tma_load_3d(sm + kOffV0, &maps.v, 0, hv, bos, bar_load);
                tma_load_3d(sm + kOffV1, &maps.v, 64, hv, bos, bar_load);
            }
            GDN_PH_ACC(dbg, 17, tp);
            pdl_trigger();
            if (warp == 1) {
                if (done == 0) tmem_alloc(tslot, kTmemCols);  // off thread 0's path: the allocation takes ~1000 cycles
            } else if (warp >= 2) {
                // zero T's six upper 16 x 16 blocks (the inverse writes every other block)
                for (int i = tid - 64; i < 6 * 256; i += kThreads - 64) {
                    const int b = i >> 8, e = i & 255;
                    const int bi = b < 3 ? 0 : (b < 5 ? 1 : 2);
                    const int bj = b < 3 ? b + 1 : (b < 5 ? b - 1 : 3);
                    Tf[(16 * bi + (e >> 4)) * kFS + 16 * bj + (e & 15)] = 0.f;
                }
            }
            GDN_PH_ACC(dbg, 18, tp);
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            const uint32_t tmem = *tslot;
            GDN_PH_ACC(dbg, 12, tp);

            // ---- 2. gates (warps 2-3) and MMA #1 (thread 0) in parallel -----------------------------
            bool ok = true;
            if (warp == 2 || warp == 3) {
                // g, beta of token t from the a / b tiles ([64 tokens][8 heads] bf16); padded tokens
                // (t >= L) carry g = 0, so their cumulative G repeats G_{L-1}, and beta = 0.
                const int t = tid - 64;
                float gl = 0.f, be = 0.f;
                if (p.gates_tma) {
                    ok = mbar_wait(bar_gate, ph, p.status, kErrPrepTmaTimeout);
                    if (ok && t < L) {
                        gl = log_decay(bf2f(reinterpret_cast<const uint16_t*>(misc + kOffTileA)[t * 8 + (hv & 7)]),
                                       p.A_log[hv], p.dt_bias[hv]);
                        be = sigmoidf_(bf2f(reinterpret_cast<const uint16_t*>(misc + kOffTileB)[t * 8 + (hv & 7)]));
                    }
                } else if (t < L) {  // [T][HV] rows narrower than a TMA box: one element per token
                    const size_t gi = (size_t)(bos + t) * p.HV + hv;
                    gl = log_decay(bf2f(p.a[gi]), p.A_log[hv], p.dt_bias[hv]);
                    be = sigmoidf_(bf2f(p.b[gi]));
                }
                float x = gl;
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
                    const float y = __shfl_up_sync(0xffffffffu, x, off);
                    if (lane >= off) x += y;
                }
                Gs[t] = x;
                Bs[t] = be;
                float rq = 1.f, rk = 1.f;
                if (p.l2norm) {
                    // in-kernel L2 norm: 1 / |q_t|, 1 / |k_t| from the tiles (16-byte chunks of a row are
                    // read in a rotated order, so the 32 rows of a warp hit different banks)
                    ok = mbar_wait(bar_load, ph, p.status, kErrPrepTmaTimeout) && ok;
                    if (ok) {
                        float ssq = 0.f, ssk = 0.f;
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            const int ch = (i + t) & 15;
                            const uint32_t off = (uint32_t)(ch >> 3) * (kOffK1 - kOffK0) + (uint32_t)t * 128u + (uint32_t)(ch & 7) * 16u;
                            const uint4 qq = *reinterpret_cast<const uint4*>(sm + kOffQ0 + off);
                            const uint4 kk = *reinterpret_cast<const uint4*>(sm + kOffK0 + off);
                            const uint32_t qw[4] = {qq.x, qq.y, qq.z, qq.w}, kw[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const float q0 = __uint_as_float(qw[e] << 16), q1 = __uint_as_float(qw[e] & 0xffff0000u);
                                const float k0 = __uint_as_float(kw[e] << 16), k1 = __uint_as_float(kw[e] & 0xffff0000u);
                                ssq = fmaf(q0, q0, fmaf(q1, q1, ssq));
                                ssk = fmaf(k0, k0, fmaf(k1, k1, ssk));
                            }
                        }
                        rq = rsqrtf(ssq + 1e-6f);
                        rk = rsqrtf(ssk + 1e-6f);
                    }
                }
                Rq[t] = rq;
                Rk[t] = rk;
                named_bar_sync(2, 64);
                // Gs holds per-warp prefix sums; the chunk prefix adds the first warp's total to tokens 32..63.
                x = Gs[t] + (t >= 32 ? Gs[31] : 0.f);
                const float xr = __shfl_sync(0xffffffffu, x, (lane & 16) | 15);  // G at the end of this 16-block
                Gf[t] = x;
                const float ex = __expf(x);
                Es[t] = ex;
                Bt[t] = __expf(fminf(xr - x, 0.f));
                Wf[t] = be * ex * rk;
            }
            if (tid == 0) {
                // MMA #1: [K; Q] (128 x 128) x K^T -> TMEM columns 0..63 (issued only if every tile
                // landed, so a CTA that gives up never leaves an MMA in flight)
                ok = (!p.gates_tma || mbar_wait(bar_gate, ph, p.status, kErrPrepTmaTimeout)) &&
                     mbar_wait(bar_load, ph, p.status, kErrPrepTmaTimeout);
                if (ok) {
                    tc_fence_after();
                    constexpr uint32_t idesc = umma_idesc_bf16(128, 64, false, false);
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint32_t koff = (uint32_t)(kk >> 2) * (kOffK1 - kOffK0) + (uint32_t)(kk & 3) * 32u;
                        umma_bf16(tmem, umma_desc_sw128(sbase + kOffK0 + koff, 16, 1024),
                                  umma_desc_sw128(sbase + kOffK0 + koff, 16, 1024), idesc, kk > 0);
                    }
                    umma_commit(bar_mma);
                }
            }
            ok = __syncthreads_and(ok);  // also publishes Gf / Es / Bt / Bs
            if (!ok) goto cleanup;
            GDN_PH_ACC(dbg, 0, tp);
            ok = mbar_wait(bar_mma, ph, p.status, kErrPrepMmaTimeout);
            ok = __syncthreads_and(ok);
            if (!ok) goto cleanup;
            tc_fence_after();

            GDN_PH_ACC(dbg, 1, tp);
            // ---- 3. epilogue #1: thread r owns TMEM lane r (rows 0-63: K K^T, rows 64-127: Q K^T) -----
            {
                long long tq3 = clock64();
                const int r = rr, i = r & 63, I = i >> 4;
                const bool qk = r >= 64;
                const float Gi = Gf[i], bi = Bs[i];
                const bool live = i < L;
                // Decay exp(G_i - G_j), j <= i.  Below row i's 16-token block it factors exactly as
                // a_i(J) * Bt[j] with a_i(J) = exp(G_i - G_r(J)), Bt[j] = exp(G_r(J) - G_j), r(J) = last token
                // of block J: both factors are <= 1, so nothing overflows and only the diagonal block needs
                // per-element exponentials.
                float aJ[3];
#pragma unroll
                for (int J = 0; J < 3; ++J) aJ[J] = __expf(fminf(Gi - Gf[16 * J + 15], 0.f));
                {
                    const int half = ch_half;
                    if (half == 1 && (wq & 1) == 0) {
                        // rows 0..31: columns 32..63 lie above the diagonal.  A's upper triangle is never
                        // read; the Aqk operand needs explicit zeros there.
                        if (qk) {
#pragma unroll
                            for (int j8 = 0; j8 < 4; ++j8) {
                                const uint32_t ch = (uint32_t)(4 + j8);
                                *reinterpret_cast<uint4*>(sm + kOffAq + i * 128 + ((ch ^ (uint32_t)(i & 7)) << 4)) =
                                    make_uint4(0, 0, 0, 0);
                                *reinterpret_cast<uint4*>(sm + kOffAq + (64 + i) * 128 + ((ch ^ (uint32_t)(i & 7)) << 4)) =
                                    make_uint4(0, 0, 0, 0);
                            }
                        }
                    } else {
                    float d[32];
                    tmem_ld32(tmem + ((uint32_t)(32 * wq) << 16) + 32 * half, d);
                    GDN_PH_ACC_T(dbg, 96, 10, tq3);
                    // v[c] = masked, decayed value of column 32*half + c (row scale beta_i for A rows)
                    float v[32];
#pragma unroll
                    for (int Jh = 0; Jh < 2; ++Jh) {
                        const int J = 2 * half + Jh;
                        if (J < I) {
                            // J depends on the runtime column half: pick the factor by compares, so aJ stays
                            // in registers (an indexed read would place it in local memory)
                            const float a = J == 0 ? aJ[0] : (J == 1 ? aJ[1] : aJ[2]);
#pragma unroll
                            for (int c = 0; c < 16; ++c) v[16 * Jh + c] = a * Bt[16 * J + c] * d[16 * Jh + c];
                        } else if (J == I) {
#pragma unroll
                            for (int c = 0; c < 16; ++c) {
                                const int j = 16 * J + c;
                                const bool keep = qk ? (j <= i) : (j < i);
                                v[16 * Jh + c] = __expf(fminf(Gi - Gf[j], 0.f)) * (keep ? d[16 * Jh + c] : 0.f);
                            }
                        } else {
#pragma unroll
                            for (int c = 0; c < 16; ++c) v[16 * Jh + c] = 0.f;
                        }
                    }
                    float rowf = 1.f;
                    if (p.l2norm) {  // k_j / |k_j| for every column, q_i / |q_i| or k_i / |k_i| for the row
#pragma unroll
                        for (int c = 0; c < 32; ++c) v[c] *= Rk[32 * half + c];
                        rowf = qk ? Rq[i] : Rk[i];
                    }
                    if (!qk) {
                        const float sc = live ? bi * rowf : 0.f;
#pragma unroll
                        for (int j4 = 0; j4 < 8; ++j4)
                            *reinterpret_cast<float4*>(Af + i * kFS + 32 * half + 4 * j4) =
                                make_float4(sc * v[4 * j4], sc * v[4 * j4 + 1], sc * v[4 * j4 + 2], sc * v[4 * j4 + 3]);
                    } else {
                        const float sc = live ? rowf : 0.f;
#pragma unroll
                        for (int j8 = 0; j8 < 4; ++j8) {
                            const uint4 q4 = make_uint4(pack_bf16x2(sc * v[8 * j8], sc * v[8 * j8 + 1]),
                                                        pack_bf16x2(sc * v[8 * j8 + 2], sc * v[8 * j8 + 3]),
                                                        pack_bf16x2(sc * v[8 * j8 + 4], sc * v[8 * j8 + 5]),
                                                        pack_bf16x2(sc * v[8 * j8 + 6], sc * v[8 * j8 + 7]));
                            const uint32_t ch = (uint32_t)(4 * half + j8);
                            *reinterpret_cast<uint4*>(sm + kOffAq + i * 128 + ((ch ^ (uint32_t)(i & 7)) << 4)) = q4;
                            *reinterpret_cast<uint4*>(sm + kOffAq + (64 + i) * 128 + ((ch ^ (uint32_t)(i & 7)) << 4)) = q4;
                        }
                    }
                    GDN_PH_ACC_T(dbg, 96, 11, tq3);
                    }
                }
                if (tid < 64) *reinterpret_cast<float4*>(p.g4 + (row0 + tid) * 4) = make_float4(Gf[tid], Es[tid], Bs[tid], Rk[tid]);
            }
            tc_fence_before();
            __syncthreads();

            GDN_PH_ACC(dbg, 2, tp);
            // ---- 4. T = (I + A)^-1 ----------------------------------------------------------------
            // 4a. diagonal 16x16 blocks: warp w (< 4) inverts block w, lanes 0..15 each own one column.
            if (warp < 4) {
                const int jb = warp;
                const float* Ab = Af + (16 * jb) * kFS + 16 * jb;
                if (lane < 16) {
                    float x[16];
#pragma unroll
                    for (int r = 0; r < 16; ++r) x[r] = (r == lane) ? 1.f : 0.f;
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float xi = x[i];
#pragma unroll
                        for (int m = i + 1; m < 16; ++m) x[m] = fmaf(-Ab[m * kFS + i], xi, x[m]);
                    }
                    float* Tb = Tf + (16 * jb) * kFS + 16 * jb;
#pragma unroll
                    for (int r = 0; r < 16; ++r) Tb[r * kFS + lane] = x[r];
                }
            }
            __syncthreads();
            GDN_PH_ACC(dbg, 13, tp);
            // 4b. off-diagonal blocks, two levels of the blocked inverse (block indices 0..3, 16 rows):
            //     level 1: T10 = -T11 (A10 T00), T32 = -T33 (A32 T22)
            //     level 2: T_LL = -T_BR (A_LL T_TL) for the lower-left 32 x 32 quadrant, i.e.
            //              X2j = A20 T0j + A21 T1j, X3j = A30 T0j + A31 T1j (j = 0, 1; T01 = 0),
            //              T2j = -T22 X2j, T3j = -(T32 X2j + T33 X3j).
            //     tf32 MMAs with fp32 accumulation.  Scratch tiles live in A's upper triangle (never read).
            {
                float acc[2][4];
                auto zero = [&]() {
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                        for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
                };
                auto blk = [&](float* base, int bi, int bj) { return base + (16 * bi) * kFS + 16 * bj; };
                auto store = [&](float* dst, float sgn) {
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt) {
                        dst[gq * kFS + 8 * nt + 2 * tq] = sgn * acc[nt][0];
                        dst[gq * kFS + 8 * nt + 2 * tq + 1] = sgn * acc[nt][1];
                        dst[(gq + 8) * kFS + 8 * nt + 2 * tq] = sgn * acc[nt][2];
                        dst[(gq + 8) * kFS + 8 * nt + 2 * tq + 1] = sgn * acc[nt][3];
                    }
                };
                float* Y0 = blk(Af, 0, 1);   // level-1 product of warp 0
                float* Y1 = blk(Af, 0, 2);   // level-1 product of warp 1
                float* X20 = blk(Af, 0, 3);
                float* X21 = blk(Af, 1, 2);
                float* X30 = blk(Af, 1, 3);
                float* X31 = blk(Af, 2, 3);
                // level 1, plus the level-2 terms that only need the diagonal blocks
                if (warp < 2) {
                    const int i = warp == 0 ? 1 : 3, j = i - 1;
                    float* Y = warp == 0 ? Y0 : Y1;
                    zero();
                    mma16_tf32(acc, blk(Af, i, j), blk(Tf, j, j), gq, tq);
                    store(Y, 1.f);
                    __syncwarp();
                    zero();
                    mma16_tf32(acc, blk(Tf, i, i), Y, gq, tq);
                    store(blk(Tf, i, j), -1.f);
                } else if (warp < 4) {
                    const int i = warp;  // X21 = A21 T11, X31 = A31 T11
                    zero();
                    mma16_tf32(acc, blk(Af, i, 1), blk(Tf, 1, 1), gq, tq);
                    store(i == 2 ? X21 : X31, 1.f);
                } else if (warp < 6) {
                    zero();
                    mma16_tf32(acc, blk(Af, warp - 2, 0), blk(Tf, 0, 0), gq, tq);  // A20 T00 / A30 T00
                }
                __syncthreads();  // T10, T32, X21, X31 visible
                if (warp == 4 || warp == 5) {
                    const int i = warp - 2;
                    mma16_tf32(acc, blk(Af, i, 1), blk(Tf, 1, 0), gq, tq);  // + A21 T10 / A31 T10
                    store(i == 2 ? X20 : X30, 1.f);
                }
                __syncthreads();  // X20, X30 visible
                if (warp < 4) {
                    const int i = 2 + (warp >> 1), j = warp & 1;
                    const float* X2 = j == 0 ? X20 : X21;
                    zero();
                    if (i == 2) {
                        mma16_tf32(acc, blk(Tf, 2, 2), X2, gq, tq);
                    } else {
                        mma16_tf32(acc, blk(Tf, 3, 2), X2, gq, tq);
                        mma16_tf32(acc, blk(Tf, 3, 3), j == 0 ? X30 : X31, gq, tq);
                    }
                    store(blk(Tf, i, j), -1.f);
                }
            }
            __syncthreads();

            GDN_PH_ACC(dbg, 3, tp);
            // ---- 5. MMA #2 operand [T diag(beta e^G); (T - I) diag(beta)]: bf16 [128][64] SW128 -----
            {
                const int r = rr, m = r & 63;
                const bool ub = r >= 64;
                const float* Trow = Tf + m * kFS;
                unsigned char* dst = sm + kOffA + r * 128;
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    const int c = 4 * ch_half + cc;
                    // two 16-byte reads per 8 columns: rows are 272 bytes apart, so the eight threads of
                    // each 128-byte phase hit disjoint bank groups (scalar reads conflicted four ways)
                    const float4 ta = *reinterpret_cast<const float4*>(Trow + 8 * c);
                    const float4 tb = *reinterpret_cast<const float4*>(Trow + 8 * c + 4);
                    const float tv[8] = {ta.x, ta.y, ta.z, ta.w, tb.x, tb.y, tb.z, tb.w};
                    uint32_t pk[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int j = 8 * c + 2 * e;
                        float t0 = tv[2 * e], t1 = tv[2 * e + 1];
                        if (ub) {
                            t0 = (j == m ? t0 - 1.f : t0) * Bs[j];
                            t1 = (j + 1 == m ? t1 - 1.f : t1) * Bs[j + 1];
                        } else {
                            t0 *= Wf[j];
                            t1 *= Wf[j + 1];
                        }
                        pk[e] = pack_bf16x2(t0, t1);
                    }
                    *reinterpret_cast<uint4*>(dst + ((c ^ (r & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                }
            }
            fence_async_smem();
            tc_fence_before();
            __syncthreads();

            GDN_PH_ACC(dbg, 4, tp);
            // ---- 6. MMA #2: [Wb; Ub] (128 x 64) x [K | V] (64 x 256, N-major) -> TMEM columns 0..255 --
            if (tid == 0) {
                tc_fence_after();
                constexpr uint32_t idesc = umma_idesc_bf16(128, 256, false, true);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_bf16(tmem, umma_desc_sw128(sbase + kOffA + 32u * kk, 16, 1024),
                              umma_desc_sw128(sbase + kOffK0 + 2048u * kk, kOffK1 - kOffK0, 1024), idesc, kk > 0);
                umma_commit(bar_mma);
            }
            ok = mbar_wait(bar_mma, ph ^ 1u, p.status, kErrPrepMmaTimeout);
            ok = __syncthreads_and(ok);
            if (!ok) goto cleanup;
            tc_fence_after();

            GDN_PH_ACC(dbg, 5, tp);
            // ---- 7. epilogue #2: rows 0-63 -> w (bf16), rows 64-127 -> u = D + beta v (f32) ---------
            {
                const int r = rr;
                const uint32_t tl = tmem + ((uint32_t)(32 * wq) << 16);
                if (r < 64) {
                    // w row r -> the (now free) K tile: MMA #3's B operand and the TMA store's source
                    tmem_two_blocks(tl + 64 * ch_half, 2 * ch_half, [&](int cb, const uint32_t(&dr)[32]) {
                        const float* d = reinterpret_cast<const float*>(dr);
#pragma unroll
                        for (int j8 = 0; j8 < 4; ++j8) {
                            const uint4 w4 =
                                make_uint4(pack_bf16x2(d[8 * j8], d[8 * j8 + 1]), pack_bf16x2(d[8 * j8 + 2], d[8 * j8 + 3]),
                                           pack_bf16x2(d[8 * j8 + 4], d[8 * j8 + 5]), pack_bf16x2(d[8 * j8 + 6], d[8 * j8 + 7]));
                            *reinterpret_cast<uint4*>(sm + kOffK0 + sw128_off(r, 32 * cb + 8 * j8, kOffK1 - kOffK0)) = w4;
                        }
                    });
                } else {
                    const int m = r - 64;
                    const float be = Bs[m];
                    unsigned char* ust = sm + kOffA;  // f32 staging of u, column-group major [16][64][8]
                    unsigned char* vt = sm + kOffV0;
                    tmem_two_blocks(tl + 128 + 64 * ch_half, 2 * ch_half, [&](int cb, const uint32_t(&dr)[32]) {
                        const float* d = reinterpret_cast<const float*>(dr);
#pragma unroll
                        for (int j4 = 0; j4 < 8; ++j4) {
                            const int c = 32 * cb + 4 * j4;
                            uint2* vp = reinterpret_cast<uint2*>(vt + sw128_off(m, c, kOffV1 - kOffV0));
                            const uint2 vv = *vp;
                            float4 o;
                            o.x = fmaf(be, __uint_as_float(vv.x << 16), d[4 * j4 + 0]);
                            o.y = fmaf(be, __uint_as_float(vv.x & 0xffff0000u), d[4 * j4 + 1]);
                            o.z = fmaf(be, __uint_as_float(vv.y << 16), d[4 * j4 + 2]);
                            o.w = fmaf(be, __uint_as_float(vv.y & 0xffff0000u), d[4 * j4 + 3]);
                            *reinterpret_cast<float4*>(ust + ((c >> 3) * 64 + m) * 32 + (c & 7) * 4) = o;
                            // u (bf16) replaces this thread's own V row in place: MMA #3's B operand
                            *vp = make_uint2(pack_bf16x2(o.x, o.y), pack_bf16x2(o.z, o.w));
                        }
                    });
                }
            }
            fence_async_smem();
            tc_fence_before();
            __syncthreads();

            GDN_PH_ACC(dbg, 6, tp);
            // ---- 8. MMA #3: [Aqk; Aqk] (128 x 64) x [w | u] (64 x 256, N-major) -> TMEM columns 0..255 --
            if (tid == 0) {
                const int wr = slot * kChunk;
                tma_store_3d(&maps.w, 0, wr, hv, sm + kOffK0);
                tma_store_3d(&maps.w, 64, wr, hv, sm + kOffK1);
                bulk_store(p.u + cg_off(hv, p.S, slot, 0), sm + kOffA, 16 * 64 * 8 * 4);
                tma_store_commit();
                tc_fence_after();
                constexpr uint32_t idesc = umma_idesc_bf16(128, 256, false, true);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_bf16(tmem, umma_desc_sw128(sbase + kOffAq + 32u * kk, 16, 1024),
                              umma_desc_sw128(sbase + kOffK0 + 2048u * kk, kOffK1 - kOffK0, 1024), idesc, kk > 0);
                umma_commit(bar_mma);
            }
            // (the w / u stores keep reading the K tile and the u staging while epilogue #3 runs: it
            // writes Q' into the Q tile and oi into MMA #3's consumed A operand)
            ok = mbar_wait(bar_mma, ph, p.status, kErrPrepMmaTimeout);
            ok = __syncthreads_and(ok);
            if (!ok) goto cleanup;
            tc_fence_after();

            GDN_PH_ACC(dbg, 7, tp);
            // ---- 9. epilogue #3: rows 0-63 -> Q' = e^G q - Aqk w, rows 64-127 -> oi = Aqk u (bf16) --------
            {
                const int r = rr;
                const uint32_t tl = tmem + ((uint32_t)(32 * wq) << 16);
                const int m = r & 63;
                const float eg = Es[m] * Rq[m];
                // Q' -> the Q tile in place (each thread reads its q chunk, then writes Q' there; SW128,
                // TMA store); oi -> staging [16][64][8] bf16 in the [Aqk; Aqk] operand area (MMA #3 is done)
                tmem_two_blocks(tl + (r < 64 ? 0 : 128) + 64 * ch_half, 2 * ch_half, [&](int cb, const uint32_t(&dr)[32]) {
                    const float* d = reinterpret_cast<const float*>(dr);
#pragma unroll
                    for (int j8 = 0; j8 < 4; ++j8) {
                        const int c = 32 * cb + 8 * j8;
                        float x[8];
                        if (r < 64) {
                            const uint4 q4 = *reinterpret_cast<const uint4*>(sm + kOffQ0 + sw128_off(m, c, kOffQ1 - kOffQ0));
                            const uint32_t qw[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                x[2 * e] = fmaf(eg, __uint_as_float(qw[e] << 16), -d[8 * j8 + 2 * e]);
                                x[2 * e + 1] = fmaf(eg, __uint_as_float(qw[e] & 0xffff0000u), -d[8 * j8 + 2 * e + 1]);
                            }
                        } else {
#pragma unroll
                            for (int e = 0; e < 8; ++e) x[e] = d[8 * j8 + e];
                        }
                        const uint4 x4 = make_uint4(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]),
                                                    pack_bf16x2(x[4], x[5]), pack_bf16x2(x[6], x[7]));
                        if (r < 64)
                            *reinterpret_cast<uint4*>(sm + kOffQ0 + sw128_off(m, c, kOffQ1 - kOffQ0)) = x4;
                        else
                            *reinterpret_cast<uint4*>(sm + kOffAq + ((c >> 3) * 64 + m) * 16) = x4;
                    }
                });
            }
            GDN_PH_ACC(dbg, 14, tp);
            fence_async_smem();
            __syncthreads();
            GDN_PH_ACC(dbg, 15, tp);
            if (tid == 0) {
                const int wr = slot * kChunk;
                tma_store_3d(&maps.qp, 0, wr, hv, sm + kOffQ0);
                tma_store_3d(&maps.qp, 64, wr, hv, sm + kOffQ1);
                bulk_store(p.oi + cg_off(hv, p.S, slot, 0), sm + kOffAq, 16 * 64 * 8 * 2);
                tma_store_commit();
            }

        cleanup:
            // Shared memory must outlive the bulk stores that read it; their global writes complete
            // before the grid does, so the scan kernel (a later launch on the stream) sees them.
            GDN_PH_ACC(dbg, 16, tp);
            if (tid == 0) tma_store_wait_read();
            GDN_PH_ACC(dbg, 8, tp);
            tc_fence_before();
            __syncthreads();
            item_ok = ok;
            ++done;
        }  // chunk work
        if (!item_ok || !persistent) break;  // (uniform) a bounded wait gave up, or one item per CTA
        __syncthreads();
        if (tid == 0) *item_slot = (int)gridDim.x + atomicAdd(p.status + 2, 1);
        __syncthreads();
        item = *item_slot;
    }  // items
    if (done > 0 && warp == 1) tmem_dealloc(*tslot, kTmemCols);  // the allocating warp
}

int launch_prefill_prep(const PrefillArgs& p, const PrefillMaps& maps, cudaStream_t stream) {
    using namespace prep2;
    if (cudaFuncSetAttribute(gdn_prefill_prep2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) !=
        cudaSuccess)
        return -1;
    dim3 grid((unsigned)std::max(p.S, 1), (unsigned)p.HV);
    if (p.short_path) {
        // only the longer sequences own slots, at most T / 64 + rows of them; at most two CTAs
        // per SM take the (slot, v-head) items from a counter
        int dev = 0, sms = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return -1;
        const long long items = (long long)std::min(p.S, p.T / kChunk + p.rows) * p.HV;
        grid = dim3((unsigned)std::max<long long>(1, std::min<long long>(items, 2LL * sms)), 1);
    }
    return launch_pdl(gdn_prefill_prep2_kernel, grid, dim3(kThreads), kSmem, stream, p, maps) == cudaSuccess ? 0 : -1;
}

}  // namespace gdn
