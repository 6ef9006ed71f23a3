// dbg.cuh -- optional per-phase cycle counters for kernel tuning, compiled only with
// -DGDN_PHASE_TIMING (never in the shipped library).  Each translation unit that uses them
// owns one counter array and exports a reader with GDN_DBG_READER(name).
#pragma once
#ifdef GDN_PHASE_TIMING
static __device__ long long gdn_dbg_clk[64];
#define GDN_DBG_READER(name)                                                                        \
    extern "C" int name(long long* host, int n) {                                                   \
        return (int)cudaMemcpyFromSymbol(host, gdn_dbg_clk, sizeof(long long) * (n < 64 ? n : 64)); \
    }
#define GDN_PH_ACC(cond, slot, prev)              \
    do {                                          \
        if ((cond) && threadIdx.x == 0) {         \
            const long long now_ = clock64();     \
            atomicAdd((unsigned long long*)&gdn_dbg_clk[slot], (unsigned long long)(now_ - (prev))); \
            prev = now_;                          \
        }                                         \
    } while (0)
// Same, measured by thread `who` instead of thread 0.
#define GDN_PH_ACC_T(cond, who, slot, prev)       \
    do {                                          \
        if ((cond) && threadIdx.x == (who)) {     \
            const long long now_ = clock64();     \
            atomicAdd((unsigned long long*)&gdn_dbg_clk[slot], (unsigned long long)(now_ - (prev))); \
            prev = now_;                          \
        }                                         \
    } while (0)
#else
#define GDN_PH_ACC_T(cond, who, slot, prev) \
    do {                                   \
        (void)(prev);                      \
    } while (0)
#define GDN_DBG_READER(name)
#define GDN_PH_ACC(cond, slot, prev) \
    do {                             \
        (void)(prev);                \
    } while (0)
#endif
