// decode.cu -- single-step Gated DeltaNet decode, one pass over the k-last fp32 state.
//
// Semantics: reference/gdn_decode_ref.py:12-83 (run); fused single-pass form as in
// solutions/gdn_decode_qk4_v8_d128_k_last/solution/triton/kernel.py:25-82.
// For each (batch b, v-head hv), with q,k taken from qk-head hv/2:
//   g = exp(-exp(A_log) softplus(a + dt_bias)),  beta = sigmoid(b)
//   for every state row v (S[v, :] is 128 contiguous floats, k-last):
//     sk = S[v]·k,  sq = S[v]·q                     (one butterfly for both)
//     vn = beta (v[v] - g sk)                       (delta-rule correction)
//     S'[v] = g S[v] + vn k                         (decay + rank-1 update)
//     out[v] = scale (g sq + vn (q·k))              (= scale q·S'[v])
//
// Layout and mapping.  A state row is 512 B; 8 lanes share a row, lane j of the
// row group holds K elements {32 i + 4 j .. +3 : i = 0..3} as four float4, so
// each of the four load instructions of a warp covers four full 128-B lines.
// A warp owns 4 rows per pass, a CTA of NW warps owns 4*NW*RPT rows of one
// (b, hv) head.  Every element is read and written by the same thread in the
// same pass, so new_state may alias state.  All state loads are issued before
// any arithmetic so a CTA keeps its whole slice in flight; the state is
// streamed (evict-first) because each byte is touched once.
#include "common.cuh"
#include "kernels.cuh"

namespace gdn {

template <int NW, int RPT>
__global__ void __launch_bounds__(NW * 32) gdn_decode_kernel(DecodeArgs p) {
    constexpr int kRowsPerPass = 4 * NW;
    constexpr int kRowsPerCta = kRowsPerPass * RPT;
    constexpr int kSlices = kD / kRowsPerCta;

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int j = lane & 7;     // position inside the row group
    const int rsub = lane >> 3; // row inside the warp's 4-row group
    const int slice = blockIdx.x % kSlices;
    const int bh = blockIdx.x / kSlices;
    int bi, hv, hq;
    if (p.HV == kHV && p.H == kH) {  // the reference's 4 / 8 family: shifts, no divisions
        bi = bh / kHV;
        hv = bh % kHV;
        hq = hv / (kHV / kH);
    } else {
        bi = bh / p.HV;
        hv = bh % p.HV;
        hq = hv / (p.HV / p.H);
    }

    const size_t head_off = (size_t)bh * kD * kD;
    const int row0 = slice * kRowsPerCta + warp * 4 + rsub;

    // Launched as a programmatic dependent: everything above overlapped the previous kernel's
    // tail; no input is read before that kernel has completed.
    pdl_wait();
    // 1. Issue every state load of this thread first.
    float4 S[RPT][4];
    if (p.state != nullptr) {
        const float* src = p.state + head_off + (size_t)row0 * kD + 4 * j;
#pragma unroll
        for (int r = 0; r < RPT; ++r)
#pragma unroll
            for (int i = 0; i < 4; ++i) S[r][i] = ld_stream_f4(src + (size_t)r * kRowsPerPass * kD + 32 * i);
    } else {
#pragma unroll
        for (int r = 0; r < RPT; ++r)
#pragma unroll
            for (int i = 0; i < 4; ++i) S[r][i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }

    pdl_trigger();  // the next kernel may start launching into SM slots as this grid drains
    // 2. q, k fragments (16 elements each) and the gates.
    float qf[16], kf[16];
    {
        const uint16_t* qp = p.q + ((size_t)bi * p.H + hq) * kD + 4 * j;
        const uint16_t* kp = p.k + ((size_t)bi * p.H + hq) * kD + 4 * j;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint2 qq = ld_nc_u2(qp + 32 * i);
            uint2 kk = ld_nc_u2(kp + 32 * i);
            qf[4 * i + 0] = __uint_as_float(qq.x << 16);
            qf[4 * i + 1] = __uint_as_float(qq.x & 0xffff0000u);
            qf[4 * i + 2] = __uint_as_float(qq.y << 16);
            qf[4 * i + 3] = __uint_as_float(qq.y & 0xffff0000u);
            kf[4 * i + 0] = __uint_as_float(kk.x << 16);
            kf[4 * i + 1] = __uint_as_float(kk.x & 0xffff0000u);
            kf[4 * i + 2] = __uint_as_float(kk.y << 16);
            kf[4 * i + 3] = __uint_as_float(kk.y & 0xffff0000u);
        }
    }
    if (p.l2norm) {
        // in-kernel L2 norm of q and k (the 8 lanes of a row group hold all 128 elements)
        float ssq = 0.f, ssk = 0.f;
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            ssq = fmaf(qf[e], qf[e], ssq);
            ssk = fmaf(kf[e], kf[e], ssk);
        }
#pragma unroll
        for (int off = 1; off < 8; off <<= 1) {
            ssq += __shfl_xor_sync(0xffffffffu, ssq, off);
            ssk += __shfl_xor_sync(0xffffffffu, ssk, off);
        }
        const float rq = rsqrtf(ssq + 1e-6f), rk = rsqrtf(ssk + 1e-6f);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            qf[e] *= rq;
            kf[e] *= rk;
        }
    }
    const float gl = log_decay(bf2f(p.a[bi * p.HV + hv]), p.A_log[hv], p.dt_bias[hv]);
    const float g = expf(gl);
    const float beta = sigmoidf_(bf2f(p.b[bi * p.HV + hv]));

    float kq = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e) kq = fmaf(kf[e], qf[e], kq);
    kq += __shfl_xor_sync(0xffffffffu, kq, 1);
    kq += __shfl_xor_sync(0xffffffffu, kq, 2);
    kq += __shfl_xor_sync(0xffffffffu, kq, 4);

    float vrow[RPT];
#pragma unroll
    for (int r = 0; r < RPT; ++r) vrow[r] = bf2f(p.v[(size_t)bh * kD + row0 + r * kRowsPerPass]);

    // 3. Row reductions (S·k and S·q together), update, store.
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
        float sk = 0.f, sq = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            sk = fmaf(S[r][i].x, kf[4 * i + 0], sk);
            sk = fmaf(S[r][i].y, kf[4 * i + 1], sk);
            sk = fmaf(S[r][i].z, kf[4 * i + 2], sk);
            sk = fmaf(S[r][i].w, kf[4 * i + 3], sk);
            sq = fmaf(S[r][i].x, qf[4 * i + 0], sq);
            sq = fmaf(S[r][i].y, qf[4 * i + 1], sq);
            sq = fmaf(S[r][i].z, qf[4 * i + 2], sq);
            sq = fmaf(S[r][i].w, qf[4 * i + 3], sq);
        }
#pragma unroll
        for (int off = 1; off < 8; off <<= 1) {
            sk += __shfl_xor_sync(0xffffffffu, sk, off);
            sq += __shfl_xor_sync(0xffffffffu, sq, off);
        }
        const float vn = beta * (vrow[r] - g * sk);
        const float o = p.scale * (g * sq + vn * kq);
        float* dst = p.new_state + head_off + (size_t)(row0 + r * kRowsPerPass) * kD + 4 * j;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float4 s = S[r][i];
            s.x = fmaf(g, s.x, vn * kf[4 * i + 0]);
            s.y = fmaf(g, s.y, vn * kf[4 * i + 1]);
            s.z = fmaf(g, s.z, vn * kf[4 * i + 2]);
            s.w = fmaf(g, s.w, vn * kf[4 * i + 3]);
            st_stream_f4(dst + 32 * i, s);
        }
        if (j == 0) p.out[(size_t)bh * kD + row0 + r * kRowsPerPass] = f2bf(o);
    }
}

template <int NW, int RPT>
static cudaError_t launch_variant(const DecodeArgs& p, int ctas, cudaStream_t stream) {
    return launch_pdl(gdn_decode_kernel<NW, RPT>, dim3(ctas), dim3(NW * 32), 0, stream, p);
}

// Variant table: (warps per CTA, rows per thread).  Rows per CTA = 4*NW*RPT.
int launch_decode(const DecodeArgs& p, int variant, cudaStream_t stream) {
    const int heads = p.B * p.HV;
    cudaError_t e;
    switch (variant) {
        case 0: e = launch_variant<4, 2>(p, heads * 4, stream); break;  // 32 rows / CTA, 128 threads
        case 1: e = launch_variant<4, 4>(p, heads * 2, stream); break;  // 64 rows / CTA, 128 threads
        case 2: e = launch_variant<4, 1>(p, heads * 8, stream); break;  // 16 rows / CTA (small batches)
        case 3: e = launch_variant<8, 2>(p, heads * 2, stream); break;  // 64 rows / CTA, 256 threads
        case 4: e = launch_variant<8, 4>(p, heads, stream); break;      // 128 rows / CTA: one CTA per head
        default: return -1;
    }
    return e == cudaSuccess ? 0 : -2;
}

}  // namespace gdn
