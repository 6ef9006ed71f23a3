// prefill_short.cu -- short prefill sequences (0 .. kShortLen tokens) in one kernel on mma.sync.
//
// A short sequence is a single partial chunk.  Its cost is the state itself -- 64 KB read and
// 64 KB written per v-head -- plus the chunk's small products, so the chunked path's two launches,
// workspace round trip and per-CTA set-up dominate it, and a token-by-token recurrence spends its
// time on scalar FMAs.  This kernel does the chunked WY algebra of one chunk
// (solutions/gdn_prefill_qk4_v8_d128_k_last/solution/triton/fla_kernels.py: cumsum + K K^T
// 858-905, solve_tril 197-314, w / u 334-383, state step 503-645, output 758-796) for one
// (sequence, v-head) per CTA, entirely in shared memory and registers, with warp-level bf16 MMAs:
//   G_t   = sum_{s<=t} g_s, gamma = e^G           A  = beta_i e^{G_i - G_j} k_i.k_j   (j < i)
//   T     = (I + A)^-1                             Aqk = e^{G_i - G_j} q_i.k_j         (j <= i)
//   W     = T diag(beta gamma) K                   U  = beta V + (T - I) diag(beta) V
//   vn    = U - W h0                               (h0 = initial state, h = S^T)
//   o     = scale (diag(gamma) Q h0 + Aqk vn)
//   S_L   = gamma_L S0 + (diag(e^{G_L - G}) vn)^T K   (vn split into bf16 hi + lo)
// with the chunk padded to 32 tokens (padded tokens have beta = 0 and g = 1).  Precision follows
// the chunked kernels: bf16 operands exactly where they use bf16 (K, Q, V exact; h0, W, T, Aqk
// rounded), fp32 accumulation, fp32 U, and the hi / lo split of vn for the state update.  With the
// in-kernel L2 norm, 1 / |q_t| and 1 / |k_t| enter as per-token scalars, as in the chunked path.
// Zero-length sequences (all-zero final state) also belong to this kernel when it runs; longer
// sequences are left to the chunked kernels, which then see only those (PrefillArgs::short_path).
//
// Mapping: 8 warps; warp w owns state rows v = 16 w .. 16 w + 15 (all 128 k) as m16n8 C fragments
// for the final update, and 16-column strips of the [token][v] products.
#include "prefill_kernels.cuh"

namespace gdn {

namespace shk {
constexpr int kThreads = 256;
constexpr int kL = 32;          // padded chunk length (kShortLen <= kL)
constexpr int kRS = 136;        // bf16 row stride of the [rows][128] tiles (272 B: conflict-free ldmatrix)
constexpr int kTS = 40;         // bf16 row stride of the [32][32] tiles (80 B)
constexpr int kFS = 33;         // fp32 row stride of the [32][32] tiles
constexpr uint32_t kOffK = 0;                               // K  bf16 [32][136]
constexpr uint32_t kOffQ = kOffK + kL * kRS * 2;            // Q
constexpr uint32_t kOffV = kOffQ + kL * kRS * 2;            // V (this v-head)
constexpr uint32_t kOffW = kOffV + kL * kRS * 2;            // W, later vn (bf16, output term)
constexpr uint32_t kOffVh = kOffW + kL * kRS * 2;           // decayed vn, bf16 hi
constexpr uint32_t kOffVl = kOffVh + kL * kRS * 2;          // decayed vn, bf16 lo
constexpr uint32_t kOffS = kOffVl + kL * kRS * 2;           // S0 bf16 [128 v][136]
constexpr uint32_t kOffA = kOffS + 128 * kRS * 2;           // A   fp32 [32][33]
constexpr uint32_t kOffT = kOffA + kL * kFS * 4;            // T   fp32 [32][33]
constexpr uint32_t kOffAq = kOffT + kL * kFS * 4;           // Aqk fp32 [32][33]
constexpr uint32_t kOffTw = kOffAq + kL * kFS * 4;          // T diag(beta gamma / |k|) bf16 [32][40]
constexpr uint32_t kOffTu = kOffTw + kL * kTS * 2;          // (T - I) diag(beta)      bf16 [32][40]
constexpr uint32_t kOffAqb = kOffTu + kL * kTS * 2;         // Aqk                     bf16 [32][40]
constexpr uint32_t kOffGate = kOffAqb + kL * kTS * 2;       // [8][32] f32: G, gamma, beta, d, rq, rk
constexpr uint32_t kSmem = kOffGate + 8 * kL * 4;
static_assert(kSmem <= 113 * 1024, "two CTAs per SM");
static_assert(kShortLen <= kL, "short sequences fit one padded chunk");
}  // namespace shk

__device__ __forceinline__ void ldsm_x4_nt(uint32_t (&r)[4], const void* p) { ldsm_x4(r[0], r[1], r[2], r[3], p); }
__device__ __forceinline__ void ldsm_x4_tr(uint32_t (&r)[4], const void* p) { ldsm_x4_t(r[0], r[1], r[2], r[3], p); }

__global__ void __launch_bounds__(shk::kThreads, 2) gdn_prefill_short_kernel(PrefillArgs p) {
    using namespace shk;
    extern __shared__ __align__(16) unsigned char sm[];
    uint16_t* Kb = reinterpret_cast<uint16_t*>(sm + kOffK);
    uint16_t* Qb = reinterpret_cast<uint16_t*>(sm + kOffQ);
    uint16_t* Vb = reinterpret_cast<uint16_t*>(sm + kOffV);
    uint16_t* Wb = reinterpret_cast<uint16_t*>(sm + kOffW);
    uint16_t* VHb = reinterpret_cast<uint16_t*>(sm + kOffVh);
    uint16_t* VLb = reinterpret_cast<uint16_t*>(sm + kOffVl);
    uint16_t* Sb = reinterpret_cast<uint16_t*>(sm + kOffS);
    float* Af = reinterpret_cast<float*>(sm + kOffA);
    float* Tf = reinterpret_cast<float*>(sm + kOffT);
    float* Aqf = reinterpret_cast<float*>(sm + kOffAq);
    uint16_t* Twb = reinterpret_cast<uint16_t*>(sm + kOffTw);
    uint16_t* Tub = reinterpret_cast<uint16_t*>(sm + kOffTu);
    uint16_t* Aqb = reinterpret_cast<uint16_t*>(sm + kOffAqb);
    float* sG = reinterpret_cast<float*>(sm + kOffGate);
    float* sGam = sG + kL;
    float* sBeta = sG + 2 * kL;
    float* sD = sG + 3 * kL;
    float* sRq = sG + 4 * kL;
    float* sRk = sG + 5 * kL;

    const int n = blockIdx.x / p.HV, hv = blockIdx.x % p.HV, hq = hv / (p.HV / p.H);
    pdl_wait();
    pdl_trigger();
    if (p.only_short && blockIdx.x == 0) {  // the call's only launch
        if (threadIdx.x == 0) p.status[0] = 0;
        zero_unowned_tokens(p, threadIdx.x, kThreads);
    }
    int bos, eos;
    seq_bounds(p.cu, p.cu64, n, p.T, bos, eos);
    const int len = eos - bos;
    if (len > kShortLen) return;  // the chunked kernels own these sequences

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int gq = lane >> 2, tq = lane & 3;
    const size_t shead = ((size_t)n * p.HV + hv) * kD * kD;
    long long tp = clock64();
    if (len <= 0) {  // zero-length sequence: all-zero final state (reference/gdn_prefill_ref.py:52-54, 61-62)
        float4* dst = reinterpret_cast<float4*>(p.new_state + shead);
        for (int i = tid; i < kD * kD / 4; i += kThreads) st_stream_f4(reinterpret_cast<float*>(dst + i), make_float4(0.f, 0.f, 0.f, 0.f));
        return;
    }

    // ---- 1-2. every global load of the CTA first (the state's 64 KB and the chunk's K, Q, V rows),
    //           then the shared-memory copies: a bf16 copy of the state S0 [v][k] (the fp32 values
    //           are read again, from L2, for the final update, so they are not held in registers
    //           through the chunk algebra) and the K, Q, V rows zero-padded to 32 tokens.
    {
        float4 x[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int idx = tid + i * kThreads, v = idx >> 5, k = 4 * (idx & 31);
            x[i] = p.state ? *reinterpret_cast<const float4*>(p.state + shead + (size_t)v * kD + k)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        // gate inputs of token `lane` (warp 0), used after the copies
        uint16_t ga = 0, gb = 0;
        if (warp == 0 && lane < len) {
            ga = p.a[(size_t)(bos + lane) * p.HV + hv];
            gb = p.b[(size_t)(bos + lane) * p.HV + hv];
        }
        uint4 kk[2], qq[2], vv[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int idx = tid + i * kThreads, t = idx >> 4, c = idx & 15;
            kk[i] = qq[i] = vv[i] = make_uint4(0, 0, 0, 0);
            if (t < len) {
                const size_t gk = ((size_t)(bos + t) * p.H + hq) * kD + 8 * c;
                kk[i] = *reinterpret_cast<const uint4*>(p.k + gk);
                qq[i] = *reinterpret_cast<const uint4*>(p.q + gk);
                vv[i] = *reinterpret_cast<const uint4*>(p.v + ((size_t)(bos + t) * p.HV + hv) * kD + 8 * c);
            }
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int idx = tid + i * kThreads, v = idx >> 5, k = 4 * (idx & 31);
            *reinterpret_cast<uint2*>(Sb + v * kRS + k) = make_uint2(pack_bf16x2(x[i].x, x[i].y), pack_bf16x2(x[i].z, x[i].w));
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int idx = tid + i * kThreads, t = idx >> 4, c = idx & 15;
            *reinterpret_cast<uint4*>(Kb + t * kRS + 8 * c) = kk[i];
            *reinterpret_cast<uint4*>(Qb + t * kRS + 8 * c) = qq[i];
            *reinterpret_cast<uint4*>(Vb + t * kRS + 8 * c) = vv[i];
        }
        if (warp == 0) {
            const int t = lane;
            float gl = 0.f, be = 0.f;
            if (t < len) {
                gl = log_decay(bf2f(ga), p.A_log[hv], p.dt_bias[hv]);
                be = sigmoidf_(bf2f(gb));
            }
            float xg = gl;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const float y = __shfl_up_sync(0xffffffffu, xg, off);
                if (lane >= off) xg += y;
            }
            const float GL = __shfl_sync(0xffffffffu, xg, len - 1);
            sG[t] = xg;
            sGam[t] = __expf(xg);
            sBeta[t] = be;
            sD[t] = __expf(fminf(GL - xg, 0.f));
        }
    }
    __syncthreads();
    if (p.l2norm) {
        // 1 / |q_t|, 1 / |k_t| (warp w: tokens w, w + 8, ...; padded tokens get 1)
        for (int t = warp; t < kL; t += kThreads / 32) {
            float ssq = 0.f, ssk = 0.f;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float qv = bf2f(Qb[t * kRS + 4 * lane + e]), kv = bf2f(Kb[t * kRS + 4 * lane + e]);
                ssq = fmaf(qv, qv, ssq);
                ssk = fmaf(kv, kv, ssk);
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                ssq += __shfl_xor_sync(0xffffffffu, ssq, off);
                ssk += __shfl_xor_sync(0xffffffffu, ssk, off);
            }
            if (lane == 0) {
                sRq[t] = t < len ? rsqrtf(ssq + 1e-6f) : 1.f;
                sRk[t] = t < len ? rsqrtf(ssk + 1e-6f) : 1.f;
            }
        }
    } else if (tid < kL) {
        sRq[tid] = 1.f;
        sRk[tid] = 1.f;
    }
    __syncthreads();

    // ---- 3. K K^T (warps 0-3) and Q K^T (warps 4-7): warp -> (m-tile (w >> 1) & 1, n-tiles 2 (w & 1) ..)
    {
        const bool isq = warp >= 4;
        const int mt = (warp >> 1) & 1, n0 = 16 * (warp & 1);
        const uint16_t* At = isq ? Qb : Kb;
        float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            uint32_t a[4], b[4];
            ldsm_x4_nt(a, At + (16 * mt + (lane & 15)) * kRS + 16 * ks + ((lane >> 4) << 3));
            ldsm_x4_nt(b, Kb + (n0 + (lane & 7) + ((lane >> 4) << 3)) * kRS + 16 * ks + (((lane >> 3) & 1) << 3));
            mma_bf16(c[0], a, b[0], b[1]);
            mma_bf16(c[1], a, b[2], b[3]);
        }
        // masked, decayed, scaled: A_ij = beta_i e^{G_i - G_j} rk_i rk_j k_i.k_j (j < i);
        // Aqk_ij = e^{G_i - G_j} rq_i rk_j q_i.k_j (j <= i)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int i = 16 * mt + gq + 8 * (e >> 1), j = n0 + 8 * nt + 2 * tq + (e & 1);
                const bool keep = isq ? (j <= i) : (j < i);
                const float dec = keep ? __expf(fminf(sG[i] - sG[j], 0.f)) : 0.f;
                const float rowf = isq ? sRq[i] : sBeta[i] * sRk[i];
                (isq ? Aqf : Af)[i * kFS + j] = keep ? c[nt][e] * dec * rowf * sRk[j] : 0.f;
            }
    }
    __syncthreads();
    // ---- 4. T = (I + A)^-1: diagonal 16 x 16 blocks by forward substitution (warps 0, 1; one
    //         column per lane), then T10 = -T11 A10 T00 (warp 0, fp32 FMAs)
    if (warp < 2) {
        const int b0 = 16 * warp;
        if (lane < 16) {
            float x[16];
#pragma unroll
            for (int r = 0; r < 16; ++r) x[r] = (r == lane) ? 1.f : 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float xi = x[i];
#pragma unroll
                for (int m = i + 1; m < 16; ++m) x[m] = fmaf(-Af[(b0 + m) * kFS + b0 + i], xi, x[m]);
            }
#pragma unroll
            for (int r = 0; r < 16; ++r) Tf[(b0 + r) * kFS + b0 + lane] = x[r];
        }
#pragma unroll
        for (int r = 0; r < 16; ++r)
            if (lane >= 16) Tf[(b0 + r) * kFS + (b0 == 0 ? 16 : 0) + lane - 16] = 0.f;  // upper block zero
    }
    __syncthreads();
    {
        // T10 = -T11 (A10 T00): warp w owns rows 16 + 2 w, 16 + 2 w + 1, lane = (row, column)
        const int r = 16 + 2 * warp + (lane >> 4), c = lane & 15;
        float y = 0.f;
#pragma unroll
        for (int m = 0; m < 16; ++m) y = fmaf(Af[r * kFS + m], Tf[m * kFS + c], y);
        __syncthreads();  // every A10 read is done: Y takes its place
        Af[r * kFS + c] = y;
        __syncthreads();
        float t = 0.f;
#pragma unroll
        for (int m = 0; m < 16; ++m) t = fmaf(Tf[r * kFS + 16 + m], Af[(16 + m) * kFS + c], t);
        Tf[r * kFS + c] = -t;
    }
    __syncthreads();
    // ---- 5. bf16 operands: Tw = T diag(beta gamma rk), Tu = (T - I) diag(beta), Aqk -----------
    for (int idx = tid; idx < kL * kL / 2; idx += kThreads) {
        const int i = idx >> 4, j = 2 * (idx & 15);
        const float t0 = Tf[i * kFS + j], t1 = Tf[i * kFS + j + 1];
        *reinterpret_cast<uint32_t*>(Twb + i * kTS + j) =
            pack_bf16x2(t0 * sBeta[j] * sGam[j] * sRk[j], t1 * sBeta[j + 1] * sGam[j + 1] * sRk[j + 1]);
        *reinterpret_cast<uint32_t*>(Tub + i * kTS + j) =
            pack_bf16x2((i == j ? t0 - 1.f : t0) * sBeta[j], (i == j + 1 ? t1 - 1.f : t1) * sBeta[j + 1]);
        *reinterpret_cast<uint32_t*>(Aqb + i * kTS + j) = pack_bf16x2(Aqf[i * kFS + j], Aqf[i * kFS + j + 1]);
    }
    __syncthreads();

    // ---- 6. W = Tw K, U = Tu V + diag(beta) V   ([token][128]; warp: m-tile w & 1, n-tiles 4 (w >> 1) ..)
    const int mt2 = warp & 1, nb = 32 * (warp >> 1);  // 16 token rows x 32 columns per warp
    float U[4][4];
    {
        float Wc[4][4];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) Wc[nt][e] = U[nt][e] = 0.f;
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
            uint32_t aw[4], au[4];
            ldsm_x4_nt(aw, Twb + (16 * mt2 + (lane & 15)) * kTS + 16 * ks + ((lane >> 4) << 3));
            ldsm_x4_nt(au, Tub + (16 * mt2 + (lane & 15)) * kTS + 16 * ks + ((lane >> 4) << 3));
#pragma unroll
            for (int np = 0; np < 2; ++np) {
                const int row = 16 * ks + (lane & 7) + (((lane >> 3) & 1) << 3), col = nb + 16 * np + ((lane >> 4) << 3);
                uint32_t bk[4], bv[4];
                ldsm_x4_tr(bk, Kb + row * kRS + col);
                ldsm_x4_tr(bv, Vb + row * kRS + col);
                mma_bf16(Wc[2 * np], aw, bk[0], bk[1]);
                mma_bf16(Wc[2 * np + 1], aw, bk[2], bk[3]);
                mma_bf16(U[2 * np], au, bv[0], bv[1]);
                mma_bf16(U[2 * np + 1], au, bv[2], bv[3]);
            }
        }
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int t = 16 * mt2 + gq + 8 * hh, col = nb + 8 * nt + 2 * tq;
                const float be = sBeta[t];
                const uint32_t vv = *reinterpret_cast<const uint32_t*>(Vb + t * kRS + col);
                U[nt][2 * hh] = fmaf(be, __uint_as_float(vv << 16), U[nt][2 * hh]);
                U[nt][2 * hh + 1] = fmaf(be, __uint_as_float(vv & 0xffff0000u), U[nt][2 * hh + 1]);
                *reinterpret_cast<uint32_t*>(Wb + t * kRS + col) = pack_bf16x2(Wc[nt][2 * hh], Wc[nt][2 * hh + 1]);
            }
    }
    __syncthreads();
    // ---- 7. P = W h0, R = Q h0 ([token][v]: B operand from S0 [v][k] bf16, K-dim = k) ----------
    float R[4][4];
    {
        float P[4][4];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) P[nt][e] = R[nt][e] = 0.f;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            uint32_t aw[4], aq[4];
            ldsm_x4_nt(aw, Wb + (16 * mt2 + (lane & 15)) * kRS + 16 * ks + ((lane >> 4) << 3));
            ldsm_x4_nt(aq, Qb + (16 * mt2 + (lane & 15)) * kRS + 16 * ks + ((lane >> 4) << 3));
#pragma unroll
            for (int np = 0; np < 2; ++np) {
                uint32_t b[4];
                ldsm_x4_nt(b, Sb + (nb + 16 * np + (lane & 7) + ((lane >> 4) << 3)) * kRS + 16 * ks + (((lane >> 3) & 1) << 3));
                mma_bf16(P[2 * np], aw, b[0], b[1]);
                mma_bf16(P[2 * np + 1], aw, b[2], b[3]);
                mma_bf16(R[2 * np], aq, b[0], b[1]);
                mma_bf16(R[2 * np + 1], aq, b[2], b[3]);
            }
        }
        __syncthreads();  // every warp is done reading W: its tile takes vn (output term)
        // vn = U - P -> vn (bf16, for Aqk vn), decayed vn d_t / |k_t| (bf16 hi + lo, state update)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int t = 16 * mt2 + gq + 8 * hh, col = nb + 8 * nt + 2 * tq;
                const float v0 = U[nt][2 * hh] - P[nt][2 * hh], v1 = U[nt][2 * hh + 1] - P[nt][2 * hh + 1];
                const float dk = sD[t] * sRk[t];
                const float d0 = v0 * dk, d1 = v1 * dk;
                const uint32_t hi = pack_bf16x2(d0, d1);
                *reinterpret_cast<uint32_t*>(Wb + t * kRS + col) = pack_bf16x2(v0, v1);
                *reinterpret_cast<uint32_t*>(VHb + t * kRS + col) = hi;
                *reinterpret_cast<uint32_t*>(VLb + t * kRS + col) =
                    pack_bf16x2(d0 - __uint_as_float(hi << 16), d1 - __uint_as_float(hi & 0xffff0000u));
            }
    }
    __syncthreads();
    // ---- 8. o = scale (gamma rq (Q h0) + Aqk vn) for the live tokens -------------------------------
    {
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
            uint32_t a[4];
            ldsm_x4_nt(a, Aqb + (16 * mt2 + (lane & 15)) * kTS + 16 * ks + ((lane >> 4) << 3));
#pragma unroll
            for (int np = 0; np < 2; ++np) {
                const int row = 16 * ks + (lane & 7) + (((lane >> 3) & 1) << 3), col = nb + 16 * np + ((lane >> 4) << 3);
                uint32_t b[4];
                ldsm_x4_tr(b, Wb + row * kRS + col);
                // R += Aqk vn / (gamma rq) would need a division; accumulate Aqk vn separately
                float o0[4] = {0.f, 0.f, 0.f, 0.f}, o1[4] = {0.f, 0.f, 0.f, 0.f};
                mma_bf16(o0, a, b[0], b[1]);
                mma_bf16(o1, a, b[2], b[3]);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int t = 16 * mt2 + gq + 8 * (e >> 1);
                    const float gr = sGam[t] * sRq[t];
                    if (ks == 0) {
                        R[2 * np][e] = fmaf(gr, R[2 * np][e], o0[e]);
                        R[2 * np + 1][e] = fmaf(gr, R[2 * np + 1][e], o1[e]);
                    } else {
                        R[2 * np][e] += o0[e];
                        R[2 * np + 1][e] += o1[e];
                    }
                }
            }
        }
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int t = 16 * mt2 + gq + 8 * hh, col = nb + 8 * nt + 2 * tq;
                if (t < len)
                    *reinterpret_cast<uint32_t*>(p.out + ((size_t)(bos + t) * p.HV + hv) * kD + col) =
                        pack_bf16x2(p.scale * R[nt][2 * hh], p.scale * R[nt][2 * hh + 1]);
            }
    }
    // ---- 9. S_L = gamma_L S0 + (decayed vn)^T K: A = vn^T from [t][v] (trans), B = K from [t][k] (trans)
    {
        const float gL = sGam[len - 1];
        const int va = 16 * warp + gq, vb = va + 8;
        uint32_t ah[2][4], al[2][4];
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
            const int arow = 16 * ks + (lane & 7) + ((lane >> 4) << 3), acol = 16 * warp + (((lane >> 3) & 1) << 3);
            ldsm_x4_tr(ah[ks], VHb + arow * kRS + acol);
            ldsm_x4_tr(al[ks], VLb + arow * kRS + acol);
        }
        // Two halves of 64 k-columns.  The half's update block (16 state rows x 64 k per warp) goes
        // through shared memory (the bf16 state copy is free by now: [128][68] fp32), so the fp32
        // state is re-read (from L2) and written back with 16-byte row-contiguous accesses instead of
        // the MMA fragment layout's 8-byte pieces spread over 8 rows.
        float* Ss = reinterpret_cast<float*>(Sb);
        constexpr int kSS = 68;  // fp32 row stride of the staging block
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            float acc[8][4];
#pragma unroll
            for (int nt = 0; nt < 8; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
#pragma unroll
            for (int ks = 0; ks < 2; ++ks)
#pragma unroll
                for (int np = 0; np < 4; ++np) {
                    const int row = 16 * ks + (lane & 7) + (((lane >> 3) & 1) << 3), col = 64 * hf + 16 * np + ((lane >> 4) << 3);
                    uint32_t b[4];
                    ldsm_x4_tr(b, Kb + row * kRS + col);
                    mma_bf16(acc[2 * np], ah[ks], b[0], b[1]);
                    mma_bf16(acc[2 * np + 1], ah[ks], b[2], b[3]);
                    mma_bf16(acc[2 * np], al[ks], b[0], b[1]);
                    mma_bf16(acc[2 * np + 1], al[ks], b[2], b[3]);
                }
            if (hf == 1) __syncwarp();  // this warp's reads of the first half's block are done
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                const int c = 8 * nt + 2 * tq;
                *reinterpret_cast<float2*>(Ss + va * kSS + c) = make_float2(acc[nt][0], acc[nt][1]);
                *reinterpret_cast<float2*>(Ss + vb * kSS + c) = make_float2(acc[nt][2], acc[nt][3]);
            }
            __syncwarp();
            // rows 16 warp .. +15, 16 float4 per row: lane covers float4 (lane & 15) of rows 2 i + (lane >> 4)
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int v = 16 * warp + 2 * i + (lane >> 4), c4 = 4 * (lane & 15);
                const size_t g = shead + (size_t)v * kD + 64 * hf + c4;
                const float4 s0 = p.state ? *reinterpret_cast<const float4*>(p.state + g) : make_float4(0.f, 0.f, 0.f, 0.f);
                const float4 d = *reinterpret_cast<const float4*>(Ss + v * kSS + c4);
                st_stream_f4(p.new_state + g, make_float4(fmaf(gL, s0.x, d.x), fmaf(gL, s0.y, d.y),
                                                          fmaf(gL, s0.z, d.z), fmaf(gL, s0.w, d.w)));
            }
        }
    }
}

int launch_prefill_short(const PrefillArgs& p, cudaStream_t stream) {
    using namespace shk;
    if (cudaFuncSetAttribute(gdn_prefill_short_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess)
        return -1;
    dim3 grid(p.N * p.HV);
    return launch_pdl(gdn_prefill_short_kernel, grid, dim3(kThreads), kSmem, stream, p) == cudaSuccess ? 0 : -1;
}

}  // namespace gdn
