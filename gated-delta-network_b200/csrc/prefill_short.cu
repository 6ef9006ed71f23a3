// prefill_short.cu -- recurrent path for short prefill sequences (1 .. kShortLen tokens).
//
// A sequence of a few tokens gains nothing from the chunked WY form: its cost is the state
// itself plus a full chunk's worth of tensor-core work.  This kernel keeps a slice of the state in registers and applies the
// token-sequential recurrence of reference/gdn_prefill_ref.py:71-87 directly (the fused form of
// the decode step, csrc/decode.cu), one token after another, so each state byte is read and
// written once and the arithmetic stays fp32 throughout.  A CTA needs 13 KB of shared memory and
// 128 threads, so about six share an SM.  Sequences longer than kShortLen (and zero-length ones) are left to the
// chunked kernels, which skip the short ones when this kernel runs (PrefillArgs::short_path).
//
// Mapping: CTA = (16-row slice of the k-last state, sequence n, v-head hv), 128 threads; the
// sequence's q, k, v and gates are staged in shared memory by one parallel load phase, then
// 8 lanes per state row (lane j holds K elements {32 i + 4 j .. +3 : i = 0..3}) step through the
// tokens reading shared memory only.  Per token:
//   sk = S.k, sq = S.q (one 3-step butterfly for both), vn = beta (v - g sk),
//   out = scale (g sq + vn (q.k)), S = g S + vn k.
#include "prefill_kernels.cuh"

namespace gdn {

constexpr int kShortRows = 16;  // state rows (V) per CTA: 128 threads, several CTAs per SM

__global__ void __launch_bounds__(kShortRows * 8) gdn_prefill_short_kernel(PrefillArgs p) {
    // The sequence's q, k (its q/k head), v (this CTA's rows) and gates, staged once.
    __shared__ __align__(16) uint16_t sq_[kShortLen][kD];
    __shared__ __align__(16) uint16_t sk_[kShortLen][kD];
    __shared__ __align__(16) uint16_t sv_[kShortLen][kShortRows];
    __shared__ float sg_[kShortLen], sb_[kShortLen];
    __shared__ float srq_[kShortLen], srk_[kShortLen];  // 1 / |q|, 1 / |k| (1 without the L2 norm)

    const int n = blockIdx.y / p.HV, hv = blockIdx.y % p.HV, hq = hv / (p.HV / p.H);
    pdl_wait();
    pdl_trigger();
    int bos, eos;
    seq_bounds(p.cu, p.cu64, n, p.T, bos, eos);
    const int len = eos - bos;
    if (len <= 0 || len > kShortLen) return;  // the chunked kernels own these sequences

    const int tid = threadIdx.x, lane = tid & 31, j = lane & 7;
    const int r0 = blockIdx.x * kShortRows;
    const int row = r0 + (tid >> 3);  // state row (V index)
    const size_t soff = (((size_t)n * p.HV + hv) * kD + row) * kD + 4 * j;

    float4 S[4];
    if (p.state) {
#pragma unroll
        for (int i = 0; i < 4; ++i) S[i] = ld_stream_f4(p.state + soff + 32 * i);
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) S[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    // stage: 16 B per load, all issued before any use
    for (int idx = tid; idx < len * (kD / 8); idx += kShortRows * 8) {
        const int t = idx / (kD / 8), c = idx % (kD / 8);
        const size_t g = ((size_t)(bos + t) * p.H + hq) * kD + 8 * c;
        *reinterpret_cast<uint4*>(&sq_[t][8 * c]) = *reinterpret_cast<const uint4*>(p.q + g);
        *reinterpret_cast<uint4*>(&sk_[t][8 * c]) = *reinterpret_cast<const uint4*>(p.k + g);
    }
    for (int idx = tid; idx < len * (kShortRows / 8); idx += kShortRows * 8) {
        const int t = idx / (kShortRows / 8), c = idx % (kShortRows / 8);
        *reinterpret_cast<uint4*>(&sv_[t][8 * c]) =
            *reinterpret_cast<const uint4*>(p.v + ((size_t)(bos + t) * p.HV + hv) * kD + r0 + 8 * c);
    }
    for (int t = tid; t < len; t += kShortRows * 8) {
        const size_t g = (size_t)(bos + t) * p.HV + hv;
        sg_[t] = expf(log_decay(bf2f(p.a[g]), p.A_log[hv], p.dt_bias[hv]));
        sb_[t] = sigmoidf_(bf2f(p.b[g]));
    }
    __syncthreads();
    if (p.l2norm) {
        // in-kernel L2 norm: warp w handles tokens w, w + 4, ...; lane l sums 4 elements
        for (int t = tid >> 5; t < len; t += (kShortRows * 8) / 32) {
            const uint2 qq = *reinterpret_cast<const uint2*>(&sq_[t][4 * lane]);
            const uint2 kk = *reinterpret_cast<const uint2*>(&sk_[t][4 * lane]);
            const float q0 = __uint_as_float(qq.x << 16), q1 = __uint_as_float(qq.x & 0xffff0000u),
                        q2 = __uint_as_float(qq.y << 16), q3 = __uint_as_float(qq.y & 0xffff0000u);
            const float k0 = __uint_as_float(kk.x << 16), k1 = __uint_as_float(kk.x & 0xffff0000u),
                        k2 = __uint_as_float(kk.y << 16), k3 = __uint_as_float(kk.y & 0xffff0000u);
            float ssq = q0 * q0 + q1 * q1 + q2 * q2 + q3 * q3;
            float ssk = k0 * k0 + k1 * k1 + k2 * k2 + k3 * k3;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                ssq += __shfl_xor_sync(0xffffffffu, ssq, off);
                ssk += __shfl_xor_sync(0xffffffffu, ssk, off);
            }
            if (lane == 0) {
                srq_[t] = rsqrtf(ssq + 1e-6f);
                srk_[t] = rsqrtf(ssk + 1e-6f);
            }
        }
        __syncthreads();
    }

    for (int t = 0; t < len; ++t) {
        float qf[16], kf[16];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint2 qq = *reinterpret_cast<const uint2*>(&sq_[t][32 * i + 4 * j]);
            const uint2 kk = *reinterpret_cast<const uint2*>(&sk_[t][32 * i + 4 * j]);
            qf[4 * i + 0] = __uint_as_float(qq.x << 16);
            qf[4 * i + 1] = __uint_as_float(qq.x & 0xffff0000u);
            qf[4 * i + 2] = __uint_as_float(qq.y << 16);
            qf[4 * i + 3] = __uint_as_float(qq.y & 0xffff0000u);
            kf[4 * i + 0] = __uint_as_float(kk.x << 16);
            kf[4 * i + 1] = __uint_as_float(kk.x & 0xffff0000u);
            kf[4 * i + 2] = __uint_as_float(kk.y << 16);
            kf[4 * i + 3] = __uint_as_float(kk.y & 0xffff0000u);
        }
        if (p.l2norm) {
            const float rq = srq_[t], rk = srk_[t];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                qf[e] *= rq;
                kf[e] *= rk;
            }
        }
        const float g = sg_[t], beta = sb_[t];
        float sk = 0.f, sq = 0.f, kq = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            sk = fmaf(S[i].x, kf[4 * i], fmaf(S[i].y, kf[4 * i + 1], fmaf(S[i].z, kf[4 * i + 2], fmaf(S[i].w, kf[4 * i + 3], sk))));
            sq = fmaf(S[i].x, qf[4 * i], fmaf(S[i].y, qf[4 * i + 1], fmaf(S[i].z, qf[4 * i + 2], fmaf(S[i].w, qf[4 * i + 3], sq))));
        }
#pragma unroll
        for (int e = 0; e < 16; ++e) kq = fmaf(kf[e], qf[e], kq);
#pragma unroll
        for (int off = 1; off < 8; off <<= 1) {
            sk += __shfl_xor_sync(0xffffffffu, sk, off);
            sq += __shfl_xor_sync(0xffffffffu, sq, off);
            kq += __shfl_xor_sync(0xffffffffu, kq, off);
        }
        const float vn = beta * (bf2f(sv_[t][tid >> 3]) - g * sk);
        const float o = p.scale * (g * sq + vn * kq);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            S[i].x = fmaf(g, S[i].x, vn * kf[4 * i + 0]);
            S[i].y = fmaf(g, S[i].y, vn * kf[4 * i + 1]);
            S[i].z = fmaf(g, S[i].z, vn * kf[4 * i + 2]);
            S[i].w = fmaf(g, S[i].w, vn * kf[4 * i + 3]);
        }
        if (j == 0) p.out[((size_t)(bos + t) * p.HV + hv) * kD + row] = f2bf(o);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) st_stream_f4(p.new_state + soff + 32 * i, S[i]);
}

int launch_prefill_short(const PrefillArgs& p, cudaStream_t stream) {
    dim3 grid(kD / kShortRows, p.N * p.HV);
    return launch_pdl(gdn_prefill_short_kernel, grid, dim3(kShortRows * 8), 0, stream, p) == cudaSuccess ? 0 : -1;
}

}  // namespace gdn
