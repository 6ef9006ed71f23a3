// prefill.cu -- varlen chunked (C = 64) Gated DeltaNet prefill.
//
// Semantics: reference/gdn_prefill_ref.py:12-91 (token-sequential oracle).
// Algorithm: the chunked WY form of the gated delta rule, the same algebra as
// solutions/gdn_prefill_qk4_v8_d128_k_last/solution/triton/fla_kernels.py
// (cumsum+KK^T 858-905, solve_tril 197-314, recompute_w_u 334-383,
// chunk_h 411-671, chunk_o 714-796), regrouped into two kernels:
//
//   prep  (grid: chunk x qk-head; both v-heads of a qk-head share K K^T and Q K^T)
//     G_i   = cumsum_{t<=i} g_t  (log decay inside the chunk), beta_i = sigmoid(b_i)
//     A_ij  = beta_i exp(G_i - G_j) k_i.k_j      (i > j)
//     T     = (I + A)^-1                         (blocked 16x16 inverse, tf32 MMAs)
//     w     = T diag(beta e^G) K                 -> bf16  [HV][T][128]
//     u     = beta*v + (T - I) diag(beta) V      -> f32   [HV][T][128]
//     Aqk_ij= exp(G_i - G_j) q_i.k_j  (i >= j)   -> bf16  [HV][T][64]
//     G                                          -> f32   [HV][T]
//   scan  (grid: V-slice x (sequence, v-head); serial over the chunks of one sequence)
//     vn = u - w h                 (h = state at chunk start, [K x BV] slice, fp32 in registers)
//     o  = scale (e^G . (Q h) + Aqk vn)
//     h  = e^{G_last} h + K^T (e^{G_last - G} . vn)
//
// Precision plan (checked against the fp32 oracle): K, Q, V are exact bf16
// inputs; w, T, Aqk and the bf16 copy of h used as an MMA operand are rounded
// to bf16; u stays fp32 and its diagonal term beta*v is added in fp32; the
// decayed vn that feeds the state update is split into bf16 hi + lo parts
// (two MMAs against the exact K), so the state keeps ~16 mantissa bits.
// Decay exponents are only formed for i >= j, so exp never overflows.
#include "common.cuh"
#include "kernels.cuh"

namespace gdn {

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

__device__ __forceinline__ void cp_async4(void* smem, const void* gmem, bool pred) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(pred ? 4 : 0)
                 : "memory");
}

// ============================================================================================
// prep kernel
// ============================================================================================
namespace prep {
constexpr int kThreads = 256;
constexpr int kFS = 68;  // fp32 row stride of the 64x64 A / T matrices (keeps rows 16-B aligned)
// dynamic shared memory carve-up (bytes)
constexpr int kOffK = 0;                       // [64][128] bf16, swz128
constexpr int kOffQ = kOffK + 64 * 128 * 2;    // [64][128] bf16, swz128
constexpr int kOffV = kOffQ + 64 * 128 * 2;    // [2][64][128] bf16, swz128
constexpr int kOffA = kOffV + 2 * 64 * 128 * 2;  // [2][64][kFS] f32  (A, strictly lower)
constexpr int kOffT = kOffA + 2 * 64 * kFS * 4;  // [2][64][kFS] f32  (T = (I+A)^-1)
constexpr int kOffWb = kOffT + 2 * 64 * kFS * 4; // [2][64][64] bf16 swz64: T diag(beta e^G)
constexpr int kOffUb = kOffWb + 2 * 64 * 64 * 2; // [2][64][64] bf16 swz64: (T - I) diag(beta)
constexpr int kOffY = kOffUb + 2 * 64 * 64 * 2;  // [8 warps][16][17] f32 scratch
constexpr int kOffG = kOffY + 8 * 16 * 17 * 4;   // [2][64] f32 cumulative log decay
constexpr int kOffB = kOffG + 2 * 64 * 4;        // [2][64] f32 beta
constexpr int kOffE = kOffB + 2 * 64 * 4;        // [2][64] f32 exp(G)
constexpr int kSmem = kOffE + 2 * 64 * 4;
}  // namespace prep

// Locate global chunk `cid` (chunks are 64-token pieces aligned to each sequence start).
// Returns false when cid is past the last chunk.  Block-wide; all threads get the answer.
__device__ bool locate_chunk(const void* cu, int cu64, int N, int T, int cid, int& seq, int& bos, int& len) {
    __shared__ int s_warp[32];
    __shared__ int s_found[3];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
    if (tid == 0) s_found[0] = -1;
    __syncthreads();
    int running = 0;
    for (int base = 0; base < N; base += blockDim.x) {
        const int i = base + tid;
        int nc = 0, s = 0, e = 0;
        if (i < N) {
            seq_bounds(cu, cu64, i, T, s, e);
            nc = (e - s + kChunk - 1) / kChunk;
        }
        int x = nc;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, x, off);
            if (lane >= off) x += y;
        }
        if (lane == 31) s_warp[warp] = x;
        __syncthreads();
        int wpre = 0, total = 0;
        for (int w = 0; w < nwarps; ++w) {
            const int c = s_warp[w];
            if (w < warp) wpre += c;
            total += c;
        }
        const int incl = running + wpre + x, excl = incl - nc;
        if (i < N && nc > 0 && cid >= excl && cid < incl) {
            const int c = cid - excl;
            s_found[0] = i;
            s_found[1] = s + c * kChunk;
            s_found[2] = min(kChunk, e - (s + c * kChunk));
        }
        running += total;
        __syncthreads();
    }
    seq = s_found[0];
    bos = s_found[1];
    len = s_found[2];
    return seq >= 0;
}

__global__ void __launch_bounds__(prep::kThreads) gdn_prefill_prep_kernel(PrefillArgs p) {
    using namespace prep;
    extern __shared__ __align__(128) unsigned char smem[];
    uint16_t* Ks = reinterpret_cast<uint16_t*>(smem + kOffK);
    uint16_t* Qs = reinterpret_cast<uint16_t*>(smem + kOffQ);
    uint16_t* Vs = reinterpret_cast<uint16_t*>(smem + kOffV);
    float* Af = reinterpret_cast<float*>(smem + kOffA);
    float* Tf = reinterpret_cast<float*>(smem + kOffT);
    uint16_t* Wb = reinterpret_cast<uint16_t*>(smem + kOffWb);
    uint16_t* Ub = reinterpret_cast<uint16_t*>(smem + kOffUb);
    float* Ysc = reinterpret_cast<float*>(smem + kOffY);
    float* Gs = reinterpret_cast<float*>(smem + kOffG);
    float* Bs = reinterpret_cast<float*>(smem + kOffB);
    float* Es = reinterpret_cast<float*>(smem + kOffE);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int gq = lane >> 2, tq = lane & 3;  // mma fragment coordinates
    const int hq = blockIdx.y;                // qk head; v-heads 2hq, 2hq+1

    int seq, bos, L;
    if (!locate_chunk(p.cu, p.cu64, p.N, p.T, blockIdx.x, seq, bos, L)) return;

    // ---- 1. async loads of K, Q (this qk head) and V (both v-heads) -----------------------
    for (int idx = tid; idx < 64 * 16; idx += kThreads) {
        const int row = idx >> 4, ch = idx & 15;
        const bool ok = row < L;
        const size_t tok = (size_t)(bos + (ok ? row : 0));
        cp_async16(Ks + swz128(row, ch * 8), p.k + (tok * kH + hq) * kD + ch * 8, ok);
        cp_async16(Qs + swz128(row, ch * 8), p.q + (tok * kH + hq) * kD + ch * 8, ok);
#pragma unroll
        for (int h = 0; h < 2; ++h)
            cp_async16(Vs + h * 64 * 128 + swz128(row, ch * 8), p.v + (tok * kHV + 2 * hq + h) * kD + ch * 8, ok);
    }
    cp_async_commit();

    // ---- 2. gates and in-chunk cumulative log decay (threads 0..127: head = tid/64) -------
    if (tid < 128) {
        const int h = tid >> 6, t = tid & 63, hv = 2 * hq + h;
        float gl = 0.f, be = 0.f;
        if (t < L) {
            const size_t tok = (size_t)(bos + t);
            gl = log_decay(bf2f(p.a[tok * kHV + hv]), p.A_log[hv], p.dt_bias[hv]);
            be = sigmoidf_(bf2f(p.b[tok * kHV + hv]));
        }
        float x = gl;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            float y = __shfl_up_sync(0xffffffffu, x, off);
            if (lane >= off) x += y;
        }
        Gs[h * 64 + t] = x;  // partial (per warp) for now
        Bs[h * 64 + t] = be;
    }
    // zero T (its strictly-upper blocks are never written below)
    for (int idx = tid; idx < 2 * 64 * kFS; idx += kThreads) Tf[idx] = 0.f;
    __syncthreads();
    if (tid < 128) {
        const int h = tid >> 6, t = tid & 63, hv = 2 * hq + h;
        float x = Gs[h * 64 + t];
        if (t >= 32) x += Gs[h * 64 + 31];
        __syncwarp();
        // padded tokens (t >= L) carry gl = 0, so they repeat G_{L-1}
        Gs[h * 64 + t] = x;  // safe: only the second warp reads Gs[31], written back unchanged
        Es[h * 64 + t] = expf(x);
        if (t < L) p.g[(size_t)hv * p.T + bos + t] = x;
    }
    cp_async_wait<0>();
    __syncthreads();

    // ---- 3. K K^T (warps 0-3) and Q K^T (warps 4-7): rows 16*(warp&3) .. +15, all 64 cols --
    {
        const uint16_t* X = (warp < 4) ? Ks : Qs;
        const int m0 = 16 * (warp & 3);
        float acc[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll
        for (int k0 = 0; k0 < 128; k0 += 16) {
            uint32_t a[4];
            ldsm_x4(a[0], a[1], a[2], a[3], X + swz128(m0 + (lane & 15), k0 + ((lane >> 4) << 3)));
#pragma unroll
            for (int np = 0; np < 4; ++np) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4(b0, b1, b2, b3,
                        Ks + swz128(16 * np + (lane & 7) + ((lane >> 4) << 3), k0 + (((lane >> 3) & 1) << 3)));
                mma_bf16(acc[2 * np], a, b0, b1);
                mma_bf16(acc[2 * np + 1], a, b2, b3);
            }
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int hv = 2 * hq + h;
            const float* G = Gs + h * 64;
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int i = m0 + gq + 8 * half;
                    const int j0 = 8 * nt + 2 * tq;
                    float r[2];
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int j = j0 + e;
                        const float c = acc[nt][2 * half + e];
                        if (warp < 4) {
                            const bool keep = (j < i) && (i < L);
                            r[e] = keep ? Bs[h * 64 + i] * expf(G[i] - G[j]) * c : 0.f;
                        } else {
                            const bool keep = (j <= i) && (i < L);
                            r[e] = keep ? expf(G[i] - G[j]) * c : 0.f;
                        }
                    }
                    if (warp < 4) {
                        Af[(h * 64 + i) * kFS + j0] = r[0];
                        Af[(h * 64 + i) * kFS + j0 + 1] = r[1];
                    } else if (i < L) {
                        *reinterpret_cast<uint32_t*>(p.aqk + ((size_t)hv * p.T + bos + i) * 64 + j0) =
                            pack_bf16x2(r[0], r[1]);
                    }
                }
            }
        }
    }
    __syncthreads();

    // ---- 4. T = (I + A)^-1 -----------------------------------------------------------------
    // 4a. diagonal 16x16 blocks by forward substitution, one column per lane (lanes 0..15).
    {
        const int h = warp >> 2, jb = warp & 3;
        const float* Ab = Af + (h * 64 + 16 * jb) * kFS + 16 * jb;
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
            float* Tb = Tf + (h * 64 + 16 * jb) * kFS + 16 * jb;
#pragma unroll
            for (int r = 0; r < 16; ++r) Tb[r * kFS + lane] = x[r];
        }
    }
    __syncthreads();
    // 4b. off-diagonal blocks, column block jb per warp:
    //     T_ib,jb = -T_ib,ib * sum_{kb=jb}^{ib-1} A_ib,kb T_kb,jb     (tf32 MMAs, fp32 accumulate)
    {
        const int h = warp >> 2, jb = warp & 3;
        const float* Ah = Af + h * 64 * kFS;
        float* Th = Tf + h * 64 * kFS;
        float* Y = Ysc + warp * 16 * 17;
        for (int ib = jb + 1; ib < 4; ++ib) {
            float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
            for (int kb = jb; kb < ib; ++kb) {
#pragma unroll
                for (int ks = 0; ks < 2; ++ks) {
                    const float* As_ = Ah + (16 * ib) * kFS + 16 * kb + 8 * ks;
                    uint32_t a[4] = {to_tf32(As_[gq * kFS + tq]), to_tf32(As_[(gq + 8) * kFS + tq]),
                                     to_tf32(As_[gq * kFS + tq + 4]), to_tf32(As_[(gq + 8) * kFS + tq + 4])};
                    const float* Bm = Th + (16 * kb + 8 * ks) * kFS + 16 * jb;
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt)
                        mma_tf32(acc[nt], a, to_tf32(Bm[tq * kFS + 8 * nt + gq]),
                                 to_tf32(Bm[(tq + 4) * kFS + 8 * nt + gq]));
                }
            }
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                Y[gq * 17 + 8 * nt + 2 * tq] = acc[nt][0];
                Y[gq * 17 + 8 * nt + 2 * tq + 1] = acc[nt][1];
                Y[(gq + 8) * 17 + 8 * nt + 2 * tq] = acc[nt][2];
                Y[(gq + 8) * 17 + 8 * nt + 2 * tq + 1] = acc[nt][3];
            }
            __syncwarp();
            float r[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
            const float* Dm = Th + (16 * ib) * kFS + 16 * ib;
#pragma unroll
            for (int ks = 0; ks < 2; ++ks) {
                uint32_t a[4] = {to_tf32(Dm[gq * kFS + 8 * ks + tq]), to_tf32(Dm[(gq + 8) * kFS + 8 * ks + tq]),
                                 to_tf32(Dm[gq * kFS + 8 * ks + tq + 4]),
                                 to_tf32(Dm[(gq + 8) * kFS + 8 * ks + tq + 4])};
#pragma unroll
                for (int nt = 0; nt < 2; ++nt)
                    mma_tf32(r[nt], a, to_tf32(Y[(8 * ks + tq) * 17 + 8 * nt + gq]),
                             to_tf32(Y[(8 * ks + tq + 4) * 17 + 8 * nt + gq]));
            }
            float* Tout = Th + (16 * ib) * kFS + 16 * jb;
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                Tout[gq * kFS + 8 * nt + 2 * tq] = -r[nt][0];
                Tout[gq * kFS + 8 * nt + 2 * tq + 1] = -r[nt][1];
                Tout[(gq + 8) * kFS + 8 * nt + 2 * tq] = -r[nt][2];
                Tout[(gq + 8) * kFS + 8 * nt + 2 * tq + 1] = -r[nt][3];
            }
            __syncwarp();
        }
    }
    __syncthreads();

    // ---- 5. bf16 coefficient matrices for w and u ------------------------------------------
    for (int idx = tid; idx < 2 * 64 * 64; idx += kThreads) {
        const int h = idx >> 12, m = (idx >> 6) & 63, j = idx & 63;
        const float t = Tf[(h * 64 + m) * kFS + j];
        const float be = Bs[h * 64 + j];
        Wb[h * 4096 + swz64(m, j)] = f2bf(t * be * Es[h * 64 + j]);
        Ub[h * 4096 + swz64(m, j)] = f2bf((m == j ? t - 1.f : t) * be);
    }
    __syncthreads();

    // ---- 6. w = Wb K (bf16 out) and u = beta v + Ub V (f32 out); warp: head warp/4, rows 16*(warp&3)
    {
        const int h = warp >> 2, hv = 2 * hq + h, m0 = 16 * (warp & 3);
#pragma unroll 1
        for (int which = 0; which < 2; ++which) {
            const uint16_t* Cm = (which == 0 ? Wb : Ub) + h * 4096;
            const uint16_t* Bm = (which == 0) ? Ks : (Vs + h * 64 * 128);
            float acc[16][4];
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll
            for (int k0 = 0; k0 < 64; k0 += 16) {
                uint32_t a[4];
                ldsm_x4(a[0], a[1], a[2], a[3], Cm + swz64(m0 + (lane & 15), k0 + ((lane >> 4) << 3)));
#pragma unroll
                for (int np = 0; np < 8; ++np) {
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4_t(b0, b1, b2, b3,
                              Bm + swz128(k0 + (lane & 7) + (((lane >> 3) & 1) << 3), 16 * np + ((lane >> 4) << 3)));
                    mma_bf16(acc[2 * np], a, b0, b1);
                    mma_bf16(acc[2 * np + 1], a, b2, b3);
                }
            }
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int i = m0 + gq + 8 * half;
                if (i >= L) continue;
                const size_t rowoff = ((size_t)hv * p.T + bos + i) * kD;
                const float be = Bs[h * 64 + i];
#pragma unroll
                for (int nt = 0; nt < 16; ++nt) {
                    const int n = 8 * nt + 2 * tq;
                    float c0 = acc[nt][2 * half], c1 = acc[nt][2 * half + 1];
                    if (which == 0) {
                        *reinterpret_cast<uint32_t*>(p.w + rowoff + n) = pack_bf16x2(c0, c1);
                    } else {
                        const uint16_t* vr = Vs + h * 64 * 128;
                        c0 = fmaf(be, bf2f(vr[swz128(i, n)]), c0);
                        c1 = fmaf(be, bf2f(vr[swz128(i, n + 1)]), c1);
                        *reinterpret_cast<float2*>(p.u + rowoff + n) = make_float2(c0, c1);
                    }
                }
            }
        }
    }
}

// ============================================================================================
// scan kernel
// ============================================================================================
template <int BV>
struct ScanCfg {
    static constexpr int kThreads = 128;
    static constexpr int kHS = BV + 8;  // bf16 row stride of [rows][BV] operand tiles (conflict-free ldmatrix)
    static constexpr int kOffW = 0;                        // [64][128] bf16 swz128
    static constexpr int kOffQ = kOffW + 64 * 128 * 2;     // [64][128] bf16 swz128
    static constexpr int kOffK = kOffQ + 64 * 128 * 2;     // [64][128] bf16 swz128
    static constexpr int kOffA = kOffK + 64 * 128 * 2;     // [64][64] bf16 swz64
    static constexpr int kOffU = kOffA + 64 * 64 * 2;      // [64][BV] f32
    static constexpr int kOffG = kOffU + 64 * BV * 4;      // [64] f32
    static constexpr int kStage = kOffG + 64 * 4;
    static constexpr int kOffHb = 2 * kStage;              // [128][kHS] bf16
    static constexpr int kOffVn = kOffHb + 128 * kHS * 2;  // [64][kHS] bf16
    static constexpr int kOffVh = kOffVn + 64 * kHS * 2;   // [64][kHS] bf16
    static constexpr int kOffVl = kOffVh + 64 * kHS * 2;   // [64][kHS] bf16
    static constexpr int kSmem = kOffVl + 64 * kHS * 2;
};

template <int BV>
__device__ __forceinline__ void scan_issue_loads(const PrefillArgs& p, unsigned char* stage, int hv, int hq, int v0,
                                                 int t0, int L) {
    using C = ScanCfg<BV>;
    const int tid = threadIdx.x;
    uint16_t* Ws = reinterpret_cast<uint16_t*>(stage + C::kOffW);
    uint16_t* Qs = reinterpret_cast<uint16_t*>(stage + C::kOffQ);
    uint16_t* Ks = reinterpret_cast<uint16_t*>(stage + C::kOffK);
    uint16_t* As = reinterpret_cast<uint16_t*>(stage + C::kOffA);
    float* Us = reinterpret_cast<float*>(stage + C::kOffU);
    float* Gs = reinterpret_cast<float*>(stage + C::kOffG);
    for (int idx = tid; idx < 64 * 16; idx += C::kThreads) {
        const int row = idx >> 4, ch = idx & 15;
        const bool ok = row < L;
        const size_t tok = (size_t)(t0 + (ok ? row : 0));
        cp_async16(Ws + swz128(row, ch * 8), p.w + ((size_t)hv * p.T + tok) * kD + ch * 8, ok);
        cp_async16(Qs + swz128(row, ch * 8), p.q + (tok * kH + hq) * kD + ch * 8, ok);
        cp_async16(Ks + swz128(row, ch * 8), p.k + (tok * kH + hq) * kD + ch * 8, ok);
    }
    for (int idx = tid; idx < 64 * 8; idx += C::kThreads) {
        const int row = idx >> 3, ch = idx & 7;
        const bool ok = row < L;
        const size_t tok = (size_t)(t0 + (ok ? row : 0));
        cp_async16(As + swz64(row, ch * 8), p.aqk + ((size_t)hv * p.T + tok) * 64 + ch * 8, ok);
    }
    constexpr int kUch = BV / 4;  // 16-byte chunks per U row
    for (int idx = tid; idx < 64 * kUch; idx += C::kThreads) {
        const int row = idx / kUch, ch = idx % kUch;
        const bool ok = row < L;
        const size_t tok = (size_t)(t0 + (ok ? row : 0));
        cp_async16(Us + row * BV + ch * 4, p.u + ((size_t)hv * p.T + tok) * kD + v0 + ch * 4, ok);
    }
    if (tid < 64) {
        const bool ok = tid < L;
        cp_async4(Gs + tid, p.g + (size_t)hv * p.T + t0 + (ok ? tid : 0), ok);
    }
}

template <int BV>
__global__ void __launch_bounds__(128) gdn_prefill_scan_kernel(PrefillArgs p) {
    using C = ScanCfg<BV>;
    constexpr int NT8 = BV / 8;  // n-tiles of 8 columns
    extern __shared__ __align__(128) unsigned char smem[];
    uint16_t* Hb = reinterpret_cast<uint16_t*>(smem + C::kOffHb);
    uint16_t* VNb = reinterpret_cast<uint16_t*>(smem + C::kOffVn);
    uint16_t* VNh = reinterpret_cast<uint16_t*>(smem + C::kOffVh);
    uint16_t* VNl = reinterpret_cast<uint16_t*>(smem + C::kOffVl);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int gq = lane >> 2, tq = lane & 3;
    const int v0 = blockIdx.x * BV;
    const int n = blockIdx.y / kHV, hv = blockIdx.y % kHV, hq = hv / (kHV / kH);
    int bos, eos;
    seq_bounds(p.cu, p.cu64, n, p.T, bos, eos);
    const int len = eos - bos;
    float* st_out = p.new_state + ((size_t)n * kHV + hv) * kD * kD;

    if (blockIdx.x == 0 && blockIdx.y == 0) {
        // Tokens outside [cu[0], cu[N]) belong to no sequence: their output is zero, as in the
        // reference, which zero-initialises the whole output (reference/gdn_prefill_ref.py:49-51).
        int lo, tmp, hi;
        seq_bounds(p.cu, p.cu64, 0, p.T, lo, tmp);
        seq_bounds(p.cu, p.cu64, p.N - 1, p.T, tmp, hi);
        hi = max(hi, lo);
        const size_t row_words = kHV * kD / 8;  // uint4 words per token row
        uint4* o4 = reinterpret_cast<uint4*>(p.out);
        for (size_t idx = tid; idx < (size_t)lo * row_words; idx += C::kThreads) o4[idx] = make_uint4(0, 0, 0, 0);
        for (size_t idx = (size_t)hi * row_words + tid; idx < (size_t)p.T * row_words; idx += C::kThreads)
            o4[idx] = make_uint4(0, 0, 0, 0);
    }
    if (len <= 0) {  // zero-length sequence: all-zero final state (reference/gdn_prefill_ref.py:52-54,61-62)
        for (int idx = tid; idx < BV * kD; idx += C::kThreads) st_out[(size_t)(v0 + idx / kD) * kD + idx % kD] = 0.f;
        return;
    }

    // state slice h[kdim][v] as mma C fragments: warp rows 32*warp + 16*mt + gq (+8), cols 8*nt + 2*tq (+1)
    float h[2][NT8][4];
    {
        const float* st_in = p.state ? p.state + ((size_t)n * kHV + hv) * kD * kD : nullptr;
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int row = 32 * warp + 16 * mt + gq + 8 * (e >> 1);
                    const int col = 8 * nt + 2 * tq + (e & 1);
                    h[mt][nt][e] = st_in ? st_in[(size_t)(v0 + col) * kD + row] : 0.f;
                }
    }
    auto write_hb = [&]() {
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int row = 32 * warp + 16 * mt + gq + 8 * half;
                    const int col = 8 * nt + 2 * tq;
                    *reinterpret_cast<uint32_t*>(Hb + row * C::kHS + col) =
                        pack_bf16x2(h[mt][nt][2 * half], h[mt][nt][2 * half + 1]);
                }
    };
    write_hb();

    const int nchunks = (len + kChunk - 1) / kChunk;
    scan_issue_loads<BV>(p, smem, hv, hq, v0, bos, min(kChunk, len));
    cp_async_commit();

    for (int c = 0; c < nchunks; ++c) {
        const int t0 = bos + c * kChunk;
        const int L = min(kChunk, eos - t0);
        if (c + 1 < nchunks) {
            const int t1 = t0 + kChunk;
            scan_issue_loads<BV>(p, smem + ((c + 1) & 1) * C::kStage, hv, hq, v0, t1, min(kChunk, eos - t1));
        }
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();

        unsigned char* stage = smem + (c & 1) * C::kStage;
        const uint16_t* Ws = reinterpret_cast<const uint16_t*>(stage + C::kOffW);
        const uint16_t* Qs = reinterpret_cast<const uint16_t*>(stage + C::kOffQ);
        const uint16_t* Ks = reinterpret_cast<const uint16_t*>(stage + C::kOffK);
        const uint16_t* As = reinterpret_cast<const uint16_t*>(stage + C::kOffA);
        const float* Us = reinterpret_cast<const float*>(stage + C::kOffU);
        const float* Gs = reinterpret_cast<const float*>(stage + C::kOffG);
        const float GL = Gs[L - 1];

        // (1) P1 = W h, P2 = Q h   (rows 16*warp .. +15)
        float p1[NT8][4], p2[NT8][4];
#pragma unroll
        for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) p1[nt][e] = p2[nt][e] = 0.f;
#pragma unroll
        for (int k0 = 0; k0 < 128; k0 += 16) {
            uint32_t aw[4], aq[4];
            ldsm_x4(aw[0], aw[1], aw[2], aw[3], Ws + swz128(16 * warp + (lane & 15), k0 + ((lane >> 4) << 3)));
            ldsm_x4(aq[0], aq[1], aq[2], aq[3], Qs + swz128(16 * warp + (lane & 15), k0 + ((lane >> 4) << 3)));
#pragma unroll
            for (int np = 0; np < NT8 / 2; ++np) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(b0, b1, b2, b3,
                          Hb + (k0 + (lane & 7) + (((lane >> 3) & 1) << 3)) * C::kHS + 16 * np + ((lane >> 4) << 3));
                mma_bf16(p1[2 * np], aw, b0, b1);
                mma_bf16(p1[2 * np + 1], aw, b2, b3);
                mma_bf16(p2[2 * np], aq, b0, b1);
                mma_bf16(p2[2 * np + 1], aq, b2, b3);
            }
        }
        // (2) vn = u - P1; o1 = scale e^G P2; stage vn (bf16) and the decayed vn (hi + lo)
        float o[NT8][4];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int row = 16 * warp + gq + 8 * half;
            const float Gr = Gs[row];
            const float eg = expf(Gr);
            const float ed = expf(GL - Gr);  // <= 1 for every real token; padded rows have vn = 0
#pragma unroll
            for (int nt = 0; nt < NT8; ++nt) {
                const int col = 8 * nt + 2 * tq;
                const float vn0 = Us[row * BV + col] - p1[nt][2 * half];
                const float vn1 = Us[row * BV + col + 1] - p1[nt][2 * half + 1];
                o[nt][2 * half] = p.scale * eg * p2[nt][2 * half];
                o[nt][2 * half + 1] = p.scale * eg * p2[nt][2 * half + 1];
                *reinterpret_cast<uint32_t*>(VNb + row * C::kHS + col) = pack_bf16x2(vn0, vn1);
                const float d0 = vn0 * ed, d1 = vn1 * ed;
                const uint32_t hi = pack_bf16x2(d0, d1);
                const float h0 = __uint_as_float(hi << 16), h1 = __uint_as_float(hi & 0xffff0000u);
                *reinterpret_cast<uint32_t*>(VNh + row * C::kHS + col) = hi;
                *reinterpret_cast<uint32_t*>(VNl + row * C::kHS + col) = pack_bf16x2(d0 - h0, d1 - h1);
            }
        }
        __syncthreads();

        // (3a) o += scale Aqk vn
        {
            float acc[NT8][4];
#pragma unroll
            for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
#pragma unroll
            for (int k0 = 0; k0 < 64; k0 += 16) {
                uint32_t a[4];
                ldsm_x4(a[0], a[1], a[2], a[3], As + swz64(16 * warp + (lane & 15), k0 + ((lane >> 4) << 3)));
#pragma unroll
                for (int np = 0; np < NT8 / 2; ++np) {
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4_t(b0, b1, b2, b3,
                              VNb + (k0 + (lane & 7) + (((lane >> 3) & 1) << 3)) * C::kHS + 16 * np +
                                  ((lane >> 4) << 3));
                    mma_bf16(acc[2 * np], a, b0, b1);
                    mma_bf16(acc[2 * np + 1], a, b2, b3);
                }
            }
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int row = 16 * warp + gq + 8 * half;
                if (row < L) {
                    uint16_t* dst = p.out + ((size_t)(t0 + row) * kHV + hv) * kD + v0;
#pragma unroll
                    for (int nt = 0; nt < NT8; ++nt) {
                        const int col = 8 * nt + 2 * tq;
                        const float r0 = fmaf(p.scale, acc[nt][2 * half], o[nt][2 * half]);
                        const float r1 = fmaf(p.scale, acc[nt][2 * half + 1], o[nt][2 * half + 1]);
                        *reinterpret_cast<uint32_t*>(dst + col) = pack_bf16x2(r0, r1);
                    }
                }
            }
        }
        // (3b) h = e^{GL} h + K^T (vn_hi + vn_lo)   (rows 32*warp .. +31 of the K dimension)
        {
            const float eL = expf(GL);
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) h[mt][nt][e] *= eL;
#pragma unroll
            for (int k0 = 0; k0 < 64; k0 += 16) {
                uint32_t a[2][4];
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
                    ldsm_x4_t(a[mt][0], a[mt][1], a[mt][2], a[mt][3],
                              Ks + swz128(k0 + (lane & 7) + ((lane >> 4) << 3),
                                          32 * warp + 16 * mt + (((lane >> 3) & 1) << 3)));
#pragma unroll
                for (int np = 0; np < NT8 / 2; ++np) {
                    const int boff = (k0 + (lane & 7) + (((lane >> 3) & 1) << 3)) * C::kHS + 16 * np + ((lane >> 4) << 3);
                    uint32_t b0, b1, b2, b3, l0, l1, l2, l3;
                    ldsm_x4_t(b0, b1, b2, b3, VNh + boff);
                    ldsm_x4_t(l0, l1, l2, l3, VNl + boff);
#pragma unroll
                    for (int mt = 0; mt < 2; ++mt) {
                        mma_bf16(h[mt][2 * np], a[mt], b0, b1);
                        mma_bf16(h[mt][2 * np + 1], a[mt], b2, b3);
                        mma_bf16(h[mt][2 * np], a[mt], l0, l1);
                        mma_bf16(h[mt][2 * np + 1], a[mt], l2, l3);
                    }
                }
            }
        }
        write_hb();
        __syncthreads();
    }

    // final state (k-last): new_state[n][hv][v0 + col][row]
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int row = 32 * warp + 16 * mt + gq + 8 * (e >> 1);
                const int col = 8 * nt + 2 * tq + (e & 1);
                st_out[(size_t)(v0 + col) * kD + row] = h[mt][nt][e];
            }
}

// ============================================================================================
// host-side launch helpers (called from the C ABI in api.cu)
// ============================================================================================
size_t prefill_workspace_layout(int T, size_t* off_w, size_t* off_u, size_t* off_a, size_t* off_g) {
    auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
    size_t o = 0;
    *off_w = o;
    o = up(o + (size_t)kHV * T * kD * 2);
    *off_u = o;
    o = up(o + (size_t)kHV * T * kD * 4);
    *off_a = o;
    o = up(o + (size_t)kHV * T * 64 * 2);
    *off_g = o;
    o = up(o + (size_t)kHV * T * 4);
    return o;
}

int prefill_scan_bv(int N) {
    // Enough CTAs to cover the SMs: (128 / BV) * N * 8 CTAs.
    return N * kHV * (kD / 32) >= 148 ? 32 : 16;
}

int launch_prefill(const PrefillArgs& p, int bv, cudaStream_t stream) {
    static_assert(prep::kSmem <= 227 * 1024, "prep smem");
    if (p.T > 0) {
        if (cudaFuncSetAttribute(gdn_prefill_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, prep::kSmem) !=
            cudaSuccess)
            return -1;
        const long long nt_max = (long long)p.T / kChunk + p.N;
        if (nt_max > 0x7fffffffLL) return -2;
        dim3 grid((unsigned)nt_max, kH);
        gdn_prefill_prep_kernel<<<grid, prep::kThreads, prep::kSmem, stream>>>(p);
    }
    if (p.N > 0) {
        if (bv == 32) {
            if (cudaFuncSetAttribute(gdn_prefill_scan_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     ScanCfg<32>::kSmem) != cudaSuccess)
                return -1;
            dim3 grid(kD / 32, p.N * kHV);
            gdn_prefill_scan_kernel<32><<<grid, 128, ScanCfg<32>::kSmem, stream>>>(p);
        } else {
            if (cudaFuncSetAttribute(gdn_prefill_scan_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     ScanCfg<16>::kSmem) != cudaSuccess)
                return -1;
            dim3 grid(kD / 16, p.N * kHV);
            gdn_prefill_scan_kernel<16><<<grid, 128, ScanCfg<16>::kSmem, stream>>>(p);
        }
    }
    return 0;
}

}  // namespace gdn
