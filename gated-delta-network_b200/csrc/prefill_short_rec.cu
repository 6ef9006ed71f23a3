// prefill_short_rec.cu -- token-recurrent path for batches of very short prefill sequences.
//
// The short-sequence kernel of prefill_short.cu spends one CTA per (sequence, v-head) on a padded
// 32-token chunk; for sequences of a handful of tokens the plain recurrence is cheaper.  This
// kernel keeps a slice of the state in registers and applies the token-sequential recurrence of
// reference/gdn_prefill_ref.py:71-87
// directly (the fused form of the decode step, csrc/decode.cu), one token after another, so each
// state byte is read and written once and the arithmetic stays fp32 throughout.  Sequences longer
// than kShortLen are left to the chunked kernels, which then see only those (PrefillArgs::
// short_path, long_list); zero-length sequences (all-zero final state) are handled here too.
//
// Mapping: CTA = (32-row slice of the k-last state, sequence n, v-head hv), 128 threads; 8 lanes
// share a pair of state rows (r and r + 16 of the slice), lane j holding K elements
// {32 i + 4 j .. +3 : i = 0..3} of both.  A parallel staging phase converts a block of up to 8 of
// the sequence's tokens' q and k (its q/k head) to fp32 in shared memory -- normalised there when
// the in-kernel L2 norm is on -- together with q.k, the gates and this slice's v, so the per-token
// loop is only
//   sk = S.k, sq = S.q (one 3-step butterfly for both rows), vn = beta (v - g sk),
//   out = scale (g sq + vn (q.k)), S = g S + vn k,
// with every q / k load shared by two state rows.  Staging 8 tokens at a time keeps shared memory at
// ~9 KB and registers at 64, so eight CTAs share an SM (64 bytes of state per thread in flight from
// 1024 threads): measured on B200, 4000 x 6 tokens 1.04 ms against 1.18 ms for a whole-sequence
// staging at six CTAs per SM; a 48- or 40-register cap (10 or 12 CTAs) spills and runs 2-3x slower.
#include "prefill_kernels.cuh"

namespace gdn {

constexpr int kRecRows = 32;                   // state rows (V) per CTA
constexpr int kRecThreads = kRecRows * 4;      // 8 lanes per row pair
constexpr int kRecBlock = 8;                   // tokens staged in shared memory at a time

__global__ void __launch_bounds__(kRecThreads, 8) gdn_prefill_short_rec_kernel(PrefillArgs p) {
    // tokens are staged kRecBlock at a time: ~9 KB of shared memory, so eight CTAs fit an SM
    __shared__ __align__(16) float sq_[kRecBlock][kD];  // q (normalised with the L2 norm), fp32
    __shared__ __align__(16) float sk_[kRecBlock][kD];  // k, likewise
    __shared__ __align__(16) uint16_t sv_[kRecBlock][kRecRows];
    __shared__ float sg_[kRecBlock], sb_[kRecBlock], skq_[kRecBlock];

    const int n = blockIdx.y / p.HV, hv = blockIdx.y % p.HV, hq = hv / (p.HV / p.H);
    pdl_wait();
    pdl_trigger();
    if (p.only_short && blockIdx.x == 0 && blockIdx.y == 0) {  // the call's only launch
        if (threadIdx.x == 0) p.status[0] = 0;
        zero_unowned_tokens(p, threadIdx.x, kRecThreads);
    }
    int bos, eos;
    seq_bounds(p.cu, p.cu64, n, p.T, bos, eos);
    const int len = eos - bos;
    if (len > kShortLen) return;  // the chunked kernels own these sequences

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, j = lane & 7;
    const int r0 = blockIdx.x * kRecRows;
    const int rowa = r0 + (tid >> 3), rowb = rowa + kRecRows / 2;  // state rows (V index)
    const size_t sbase = ((size_t)n * p.HV + hv) * kD * kD + 4 * j;
    const size_t offa = sbase + (size_t)rowa * kD, offb = sbase + (size_t)rowb * kD;

    float4 Sa[4], Sb[4];
    if (len <= 0) {  // zero-length sequence: all-zero final state (reference/gdn_prefill_ref.py:52-54, 61-62)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            st_stream_f4(p.new_state + offa + 32 * i, make_float4(0.f, 0.f, 0.f, 0.f));
            st_stream_f4(p.new_state + offb + 32 * i, make_float4(0.f, 0.f, 0.f, 0.f));
        }
        return;
    }
    if (p.state) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            Sa[i] = ld_stream_f4(p.state + offa + 32 * i);
            Sb[i] = ld_stream_f4(p.state + offb + 32 * i);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) Sa[i] = Sb[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const int ra = tid >> 3, rb = ra + kRecRows / 2;  // rows within the slice
    for (int tb = 0; tb < len; tb += kRecBlock) {
        const int nb = min(kRecBlock, len - tb);
        if (tb > 0) __syncthreads();  // the previous block's tokens are consumed
        // ---- staging: warp w takes tokens w, w + 4, ...; lane l converts elements 4 l .. 4 l + 3 ----
        for (int t = warp; t < nb; t += kRecThreads / 32) {
            const size_t g = ((size_t)(bos + tb + t) * p.H + hq) * kD + 4 * lane;
            const uint2 qq = *reinterpret_cast<const uint2*>(p.q + g);
            const uint2 kk = *reinterpret_cast<const uint2*>(p.k + g);
            float4 q4 = make_float4(__uint_as_float(qq.x << 16), __uint_as_float(qq.x & 0xffff0000u),
                                    __uint_as_float(qq.y << 16), __uint_as_float(qq.y & 0xffff0000u));
            float4 k4 = make_float4(__uint_as_float(kk.x << 16), __uint_as_float(kk.x & 0xffff0000u),
                                    __uint_as_float(kk.y << 16), __uint_as_float(kk.y & 0xffff0000u));
            if (p.l2norm) {  // x / sqrt(sum x^2 + 1e-6) per token and head
                float ssq = q4.x * q4.x + q4.y * q4.y + q4.z * q4.z + q4.w * q4.w;
                float ssk = k4.x * k4.x + k4.y * k4.y + k4.z * k4.z + k4.w * k4.w;
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
                    ssq += __shfl_xor_sync(0xffffffffu, ssq, off);
                    ssk += __shfl_xor_sync(0xffffffffu, ssk, off);
                }
                const float rq = rsqrtf(ssq + 1e-6f), rk = rsqrtf(ssk + 1e-6f);
                q4 = make_float4(q4.x * rq, q4.y * rq, q4.z * rq, q4.w * rq);
                k4 = make_float4(k4.x * rk, k4.y * rk, k4.z * rk, k4.w * rk);
            }
            *reinterpret_cast<float4*>(&sq_[t][4 * lane]) = q4;
            *reinterpret_cast<float4*>(&sk_[t][4 * lane]) = k4;
            float kq = q4.x * k4.x + q4.y * k4.y + q4.z * k4.z + q4.w * k4.w;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) kq += __shfl_xor_sync(0xffffffffu, kq, off);
            if (lane == 0) {
                const size_t gg = (size_t)(bos + tb + t) * p.HV + hv;
                skq_[t] = kq;
                sg_[t] = expf(log_decay(bf2f(p.a[gg]), p.A_log[hv], p.dt_bias[hv]));
                sb_[t] = sigmoidf_(bf2f(p.b[gg]));
            }
        }
        for (int idx = tid; idx < nb * (kRecRows / 8); idx += kRecThreads) {
            const int t = idx / (kRecRows / 8), c = idx % (kRecRows / 8);
            *reinterpret_cast<uint4*>(&sv_[t][8 * c]) =
                *reinterpret_cast<const uint4*>(p.v + ((size_t)(bos + tb + t) * p.HV + hv) * kD + r0 + 8 * c);
        }
        __syncthreads();

        for (int t = 0; t < nb; ++t) {
            float4 qv[4], kv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                qv[i] = *reinterpret_cast<const float4*>(&sq_[t][32 * i + 4 * j]);
                kv[i] = *reinterpret_cast<const float4*>(&sk_[t][32 * i + 4 * j]);
            }
            const float g = sg_[t], beta = sb_[t], kq = skq_[t];
            // Lane-paired fp32 (f32x2): the four dot products and the update run on element pairs,
            // halving the instruction count of this instruction-bound loop.
            float2 aka = make_float2(0.f, 0.f), aqa = aka, akb = aka, aqb = aka;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 k0 = make_float2(kv[i].x, kv[i].y), k1 = make_float2(kv[i].z, kv[i].w);
                const float2 q0 = make_float2(qv[i].x, qv[i].y), q1 = make_float2(qv[i].z, qv[i].w);
                const float2 a0 = make_float2(Sa[i].x, Sa[i].y), a1 = make_float2(Sa[i].z, Sa[i].w);
                const float2 b0 = make_float2(Sb[i].x, Sb[i].y), b1 = make_float2(Sb[i].z, Sb[i].w);
                aka = fma2(a1, k1, fma2(a0, k0, aka));
                aqa = fma2(a1, q1, fma2(a0, q0, aqa));
                akb = fma2(b1, k1, fma2(b0, k0, akb));
                aqb = fma2(b1, q1, fma2(b0, q0, aqb));
            }
            float ska = aka.x + aka.y, sqa = aqa.x + aqa.y, skb = akb.x + akb.y, sqb = aqb.x + aqb.y;
#pragma unroll
            for (int off = 1; off < 8; off <<= 1) {
                ska += __shfl_xor_sync(0xffffffffu, ska, off);
                sqa += __shfl_xor_sync(0xffffffffu, sqa, off);
                skb += __shfl_xor_sync(0xffffffffu, skb, off);
                sqb += __shfl_xor_sync(0xffffffffu, sqb, off);
            }
            const float vna = beta * (bf2f(sv_[t][ra]) - g * ska);
            const float vnb = beta * (bf2f(sv_[t][rb]) - g * skb);
            const float2 g2 = make_float2(g, g), va2 = make_float2(vna, vna), vb2 = make_float2(vnb, vnb);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 k0 = make_float2(kv[i].x, kv[i].y), k1 = make_float2(kv[i].z, kv[i].w);
                const float2 a0 = fma2(g2, make_float2(Sa[i].x, Sa[i].y), mul2(va2, k0));
                const float2 a1 = fma2(g2, make_float2(Sa[i].z, Sa[i].w), mul2(va2, k1));
                const float2 b0 = fma2(g2, make_float2(Sb[i].x, Sb[i].y), mul2(vb2, k0));
                const float2 b1 = fma2(g2, make_float2(Sb[i].z, Sb[i].w), mul2(vb2, k1));
                Sa[i] = make_float4(a0.x, a0.y, a1.x, a1.y);
                Sb[i] = make_float4(b0.x, b0.y, b1.x, b1.y);
            }
            if (j == 0) {
                uint16_t* o = p.out + ((size_t)(bos + tb + t) * p.HV + hv) * kD;
                o[rowa] = f2bf(p.scale * (g * sqa + vna * kq));
                o[rowb] = f2bf(p.scale * (g * sqb + vnb * kq));
            }
        }
    }  // token blocks
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        st_stream_f4(p.new_state + offa + 32 * i, Sa[i]);
        st_stream_f4(p.new_state + offb + 32 * i, Sb[i]);
    }
}

int launch_prefill_short_rec(const PrefillArgs& p, cudaStream_t stream) {
    dim3 grid(kD / kRecRows, p.N * p.HV);
    return launch_pdl(gdn_prefill_short_rec_kernel, grid, dim3(kRecThreads), 0, stream, p) == cudaSuccess ? 0 : -1;
}

}  // namespace gdn
