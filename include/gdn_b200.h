/*
 * gdn_b200.h -- C ABI of the B200-native Gated DeltaNet operator pair
 * (decode step and varlen chunked prefill), shape family qk4_v8_d128,
 * k-last fp32 recurrent state [*, HV, V, K].
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * passed as void*; no framework types cross this boundary.  All launches are
 * asynchronous on the given stream; no entry point synchronises the device,
 * copies device data to the host or allocates device memory, so every call
 * can be captured into a CUDA graph.
 *
 * Element types:
 *   bf16  = 16-bit brain float stored as uint16_t bits (torch.bfloat16)
 *   f32   = IEEE float
 * Return value: GDN_OK (0) or one of the GDN_ERR_* codes below; a non-zero
 * return means nothing was launched (except GDN_ERR_CUDA, which reports a
 * launch failure from the CUDA runtime).
 */
#ifndef GDN_B200_H_
#define GDN_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum gdn_status {
    GDN_OK = 0,
    GDN_ERR_NULL = 1,      /* a required pointer is NULL                          */
    GDN_ERR_SHAPE = 2,     /* head size other than 128, or head counts outside the
                              accepted family (see GDN_MAX_QK_HEADS)             */
    GDN_ERR_ALIGN = 3,     /* a pointer is not 16-byte aligned                     */
    GDN_ERR_SIZE = 4,      /* negative or inconsistent batch / token / seq counts  */
    GDN_ERR_WORKSPACE = 5, /* workspace missing, misaligned or too small           */
    GDN_ERR_CUDA = 6,      /* the CUDA runtime rejected the launch                 */
    GDN_ERR_DEVICE = 7     /* current device is not compute capability 10.0 (B200) */
};

/* Flags (bitwise OR) accepted by the entry points.
 * Bits 8-15 (value << 8) force a kernel variant for tuning: the decode CTA tiling (variant + 1)
 * or the prefill scan's state-column slice width (8, 16 or 32: mma.sync scan; 64: tcgen05 scan);
 * 0 lets the library choose. */
#define GDN_FLAG_NONE 0u
/* Failure-detection test hook for gdn_prefill_fwd: the scan kernel withholds the TMA copies of
 * each sequence's second chunk, so its bounded wait expires (after about 2 s), the call records
 * GDN_DEVSTATUS_SCAN_TMA_TIMEOUT in the workspace status word and returns without hanging.
 * Outputs of such a call are invalid.  Never set in production. */
#define GDN_FLAG_TEST_WITHHOLD_CHUNK 0x1u
/* Tuning: keep every prefill sequence on the chunked kernels (no short-sequence path). */
#define GDN_FLAG_NO_SHORT_PATH 0x2u
/* Variant for gdn_decode_fwd, gdn_prefill_fwd and gdn_prefill_fwd_noalloc: normalise q and k of every
 * token and q/k head in-kernel, x * (sum x^2 + 1e-6)^-1/2 in fp32, before the step (the in-kernel L2
 * norm of the reference's decode sweep kernel, tests/bench_decode_sweep.py:43-46, and of FLA's
 * use_qk_l2norm_in_kernel).  Without it q and k are used as given, as the reference oracles do. */
#define GDN_FLAG_QK_L2NORM 0x4u
/* Prefill route.  By default a call of one sequence of at least 3072 tokens, or of a few sequences
 * averaging at least 6144 tokens, splits every sequence into segments whose state transitions are
 * built in parallel and then chained (gdn_prefill_fwd decides from N and T).  GDN_FLAG_NO_SEGMENTS keeps the single-pass recurrence;
 * GDN_FLAG_SEGMENTS takes the segmented route for any call whose workspace has its regions (at most
 * 32 sequences averaging at least 512 tokens, see gdn_prefill_workspace_bytes).  Bits 16-23
 * (value << 16) force the segment length in 64-token chunks (it must not need more segment slots
 * than the workspace holds, else GDN_ERR_SIZE). */
#define GDN_FLAG_NO_SEGMENTS 0x8u
#define GDN_FLAG_SEGMENTS 0x10u

/* Device-side status codes written to the first int of the prefill workspace. */
#define GDN_DEVSTATUS_OK 0
#define GDN_DEVSTATUS_SCAN_TMA_TIMEOUT 1
#define GDN_DEVSTATUS_PREP_TMA_TIMEOUT 2
#define GDN_DEVSTATUS_PREP_MMA_TIMEOUT 3
#define GDN_DEVSTATUS_SCAN_MMA_TIMEOUT 4
/* cu_seqlens was not non-decreasing (overlapping or reversed sequences): the chunked kernels met
 * more 64-token chunks than the workspace holds and skipped the excess (the outputs of such a call
 * are invalid, but no access leaves the buffers). */
#define GDN_DEVSTATUS_BAD_SEQLENS 5

/* Fixed shape family (the reference asserts exactly these:
 * reference/gdn_decode_ref.py:32-36, reference/gdn_prefill_ref.py:33-36). */
#define GDN_NUM_QK_HEADS 4
#define GDN_NUM_V_HEADS 8
#define GDN_HEAD_DIM 128
/* Other head counts are accepted as a superset of the reference: H q/k heads, HV v-heads with
 * HV a multiple of H (v-head hv reads q/k head hv / (HV / H)), 1 <= H <= 64, HV <= 256, for decode
 * and prefill alike (so one q/k head group of the reference's heads, e.g. H = 1, HV = 2, runs on
 * its own GPU).  Head size stays 128.  Layouts generalise the ones below with 4 -> H and 8 -> HV. */
#define GDN_MAX_QK_HEADS 64
#define GDN_MAX_V_HEADS 256
#define GDN_CHUNK 64

/*
 * One decode step for a batch of B sequences.
 *
 * Replaces the destination-passing entry
 *   kernel(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state)
 * of solutions/gdn_decode_qk4_v8_d128_k_last/solution/triton/kernel.py:85
 * (and its CUDA twin, solutions/gdn_decode_qk4_v8_d128_k_last/solution/cuda/binding.py:195),
 * with the semantics of reference/gdn_decode_ref.py:12-83 (run).
 *
 *   q, k      [B, H=4, K=128]        bf16   (the reference's [B,1,4,128])
 *   v         [B, HV=8, V=128]       bf16
 *   state     [B, HV, V, K]          f32    k-last; NULL means an all-zero state
 *   A_log     [HV]                   f32
 *   a, b      [B, HV]                bf16
 *   dt_bias   [HV]                   f32
 *   scale     softmax-free output scale (the caller resolves None/0 to 1/sqrt(K))
 *   out       [B, HV, V]             bf16   (written)
 *   new_state [B, HV, V, K]          f32    (written; may alias `state`)
 *   H, HV, K, V are 4, 8, 128, 128 in the reference (other H / HV: see GDN_MAX_QK_HEADS).
 *   B may be 0 (no launch).
 * Pointers to q, k, v, state, out, new_state must be 16-byte aligned.
 */
int gdn_decode_fwd(const void* q, const void* k, const void* v, const float* state, const float* A_log,
                   const void* a, const float* dt_bias, const void* b, float scale, void* out, float* new_state,
                   int B, int H, int HV, int K, int V, void* stream, unsigned flags);

/*
 * Workspace bytes gdn_prefill_fwd needs for T packed tokens and N sequences.
 * Replaces the module-level buffer cache of
 * solutions/gdn_prefill_qk4_v8_d128_k_last/solution/triton/fla_kernels.py:950-957,987-1037
 * (the caller owns the memory; the library keeps no global device state).
 */
size_t gdn_prefill_workspace_bytes(int N, int T, int H, int HV, int K, int V);

/*
 * Varlen chunked prefill (chunk = 64 tokens) over N packed sequences.
 *
 * Replaces the destination-passing entry
 *   kernel(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state)
 * of solutions/gdn_prefill_qk4_v8_d128_k_last/solution/triton/fla_kernels.py:1049
 * (and the legacy FLA wrapper, solutions/gdn_prefill_qk4_v8_d128_k_last/solution/triton/kernel.py:61-104),
 * with the semantics of reference/gdn_prefill_ref.py:12-91 (run).
 *
 *   q, k        [T, H=4, K=128]      bf16
 *   v           [T, HV=8, V=128]     bf16
 *   state       [N, HV, V, K]        f32    initial state, k-last; NULL means zeros
 *   A_log       [HV] f32; a, b [T, HV] bf16; dt_bias [HV] f32
 *   cu_seqlens  [N+1]                int32 (cu_is_int64 = 0) or int64 (cu_is_int64 = 1),
 *                                    device memory; read on the device only (no host copy)
 *   out         [T, HV, V]           bf16   (written for every token covered by a sequence)
 *   new_state   [N, HV, V, K]        f32    final state; a zero-length sequence gets all zeros
 *                                    (reference/gdn_prefill_ref.py:52-54, 61-62); may alias `state`
 *   workspace   >= gdn_prefill_workspace_bytes(N, T, ...) bytes of device memory, 256-byte aligned,
 *               required even when T == 0; no contents are carried between calls.  Its first
 *               int receives 0, or the code of a bounded device-side wait that gave up
 *               (the call's outputs are then invalid); reading it is optional.
 * Pointers to q, k, v, state, out, new_state must be 16-byte aligned (the kernels read q, k, v
 * with TMA tile copies); a and b too when HV is a multiple of 8 (then also TMA tiles), else
 * 2-byte aligned.
 * Sequence bounds are clamped to [0, T] on the device, so malformed cu_seqlens
 * cannot make the kernels read or write outside the buffers.
 */
int gdn_prefill_fwd(const void* q, const void* k, const void* v, const float* state, const float* A_log,
                    const void* a, const float* dt_bias, const void* b, const void* cu_seqlens, int cu_is_int64,
                    int N, int T, float scale, void* out, float* new_state, void* workspace, size_t workspace_bytes,
                    int H, int HV, int K, int V, void* stream, unsigned flags);

/*
 * Prefill without a workspace argument, for callers that cannot allocate device memory
 * (a host runtime that owns all device memory and forbids its plugins from calling
 * cudaMalloc, or a serving loop whose memory is fixed at start-up).  This entry point has
 * no counterpart in the reference.
 *
 * Same arguments and results as gdn_prefill_fwd minus `workspace` / `workspace_bytes`: the
 * workspace is a fixed device array inside the library, sized for GDN_NOALLOC_MAX_TOKENS
 * packed tokens in at most GDN_NOALLOC_MAX_SEQS sequences (about 42 MB), which every GPU
 * that loads the library holds until the process exits.  T > GDN_NOALLOC_MAX_TOKENS or
 * N > GDN_NOALLOC_MAX_SEQS returns GDN_ERR_SIZE and launches nothing.  The array is sized for
 * HV = 8; with more v-heads a call whose workspace would not fit also returns GDN_ERR_SIZE.
 * The call itself allocates nothing (no cudaMalloc / cudaFree).
 * The first call on each device (with that device current) looks up the array's device
 * address once; make that first call before any stream capture.  That cached address dies with
 * the device's primary context: after cudaDeviceReset do not call this entry point on that device
 * again in the same process.
 * All calls share the one array: calls that can overlap on the GPU (different streams,
 * or different host threads) race on it and must be serialised by the caller.  No part of
 * the array needs to start at zero: every location a call reads was written earlier in
 * the same call.
 */
#define GDN_NOALLOC_MAX_TOKENS 2048
#define GDN_NOALLOC_MAX_SEQS 16
int gdn_prefill_fwd_noalloc(const void* q, const void* k, const void* v, const float* state, const float* A_log,
                            const void* a, const float* dt_bias, const void* b, const void* cu_seqlens,
                            int cu_is_int64, int N, int T, float scale, void* out, float* new_state, int H, int HV,
                            int K, int V, void* stream, unsigned flags);

/* Human-readable name of a status code (static storage). */
const char* gdn_status_string(int status);

/* Library version, major*10000 + minor*100 + patch. */
int gdn_version(void);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_H_ */
