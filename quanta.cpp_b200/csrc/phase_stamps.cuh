// Per-phase timing of the b = 1 decode layer kernels, compiled in only with -DQNT_PHASE_STAMPS (the instrumented
// library `python quanta.cpp_b200/build.py --stamps` writes to quanta.cpp_b200/lib_stamps/; the product library has
// none of it).  Thread 0 of the first CTA of each launch records the global timer at its start and end and the SM's
// cycle counter at each marked phase boundary; timeline.py turns the records into a per-phase table.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace qb {

constexpr int kPhaseMarks = 12;
struct PhaseRec {
    unsigned long long g0, g1;  // global timer (ns) at the start and the end of CTA 0
    long long c[kPhaseMarks];   // clock64 at each mark (c[0]: the start)
    int kind, n;                // kernel kind (1 attention, 2 gate|up, 3 down / o_proj residual, 4.. the rest), marks
    unsigned long long g_last;  // global timer at the end of the launch's last CTA to finish
};

#ifdef QNT_PHASE_STAMPS
namespace {
constexpr int kPhaseCap = 8192;
__device__ PhaseRec g_phase[kPhaseCap];
__device__ unsigned g_phase_n;
__device__ int g_phase_cur[16];  // the record of the latest launch of each kind (read by the launch's other CTAs)

__device__ __forceinline__ unsigned long long phase_gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
}  // namespace

struct PhaseProbe {
    int slot = -1, n = 0, kind = 0;  // the mark count stays in a register: a mark only stores (no global read)
    __device__ void begin(int k) {
        kind = k & 15;
        if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) {
            const unsigned s = atomicAdd(&g_phase_n, 1u);
            if (s < unsigned(kPhaseCap)) {
                slot = int(s);
                g_phase[s].kind = k;
                g_phase[s].g0 = phase_gtime();
                g_phase[s].g_last = 0;
                g_phase[s].c[0] = clock64();
                n = 1;
                g_phase[s].n = 1;
                __threadfence();
                *reinterpret_cast<volatile int*>(&g_phase_cur[kind]) = int(s);
            }
        }
    }
    __device__ void mark() {
        if (slot >= 0 && n < kPhaseMarks) {
            g_phase[slot].c[n] = clock64();
            g_phase[slot].n = ++n;
        }
    }
    // every CTA's thread 0 also raises the record's last end (the record is the latest of this kind: launches of one
    // kind are far apart in time, so CTA 0 has written it long before the others end)
    __device__ void end() {
        mark();
        const unsigned long long t = phase_gtime();
        if (slot >= 0) g_phase[slot].g1 = t;
        if (threadIdx.x == 0) {
            const int s = *reinterpret_cast<volatile int*>(&g_phase_cur[kind]);
            if (s >= 0 && s < kPhaseCap) atomicMax(&g_phase[s].g_last, t);
        }
    }
};

// Host side of one translation unit's records: copies up to cap of them to out, returns their count; reset clears.
#define QNT_PHASE_READER(name)                                                                             \
    extern "C" int name(void* out, int cap, int reset) {                                                   \
        unsigned n = 0;                                                                                    \
        if (cudaDeviceSynchronize() != cudaSuccess) return -2; /* the model's stream does not block */      \
        if (cudaMemcpyFromSymbol(&n, g_phase_n, sizeof n) != cudaSuccess) return -2;                       \
        const int m = int(n < unsigned(kPhaseCap) ? n : unsigned(kPhaseCap));                              \
        const int k = m < cap ? m : cap;                                                                   \
        if (out && k > 0 && cudaMemcpyFromSymbol(out, g_phase, size_t(k) * sizeof(PhaseRec)) != cudaSuccess) \
            return -2;                                                                                     \
        if (reset) {                                                                                       \
            const unsigned z = 0;                                                                          \
            if (cudaMemcpyToSymbol(g_phase_n, &z, sizeof z) != cudaSuccess) return -2;                     \
        }                                                                                                  \
        return k;                                                                                          \
    }
#else
struct PhaseProbe {
    __device__ void begin(int) {}
    __device__ void mark() {}
    __device__ void end() {}
};
#define QNT_PHASE_READER(name)
#endif

}  // namespace qb
