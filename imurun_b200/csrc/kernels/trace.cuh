// trace.cuh — optional device-time trace of kernel phases (off unless the
// host enabled it with fbk_trace_enable). Block 0 of a traced kernel records
// (globaltimer, kernel tag, event, launch number); the launch number counts
// launches of that tag since tracing was enabled. Each translation unit keeps
// its own copy of the state (kernels are compiled without relocatable device
// code); all copies point at one shared buffer.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace fb {

enum : int { TR_GEMV = 1, TR_ATTN = 2, TR_EMBED = 3, TR_KEYS = 4 };
enum : int { EV_START = 0, EV_WAITED = 1, EV_READY = 2, EV_END = 3 };
// finer GEMV events: norm scale known, first stage's weights in shared
// memory, last stage consumed (before the final reduction)
enum : int { EV_SCALE = 8, EV_FIRST = 9, EV_LOOP = 10 };

struct TraceState {
    unsigned long long* buf;   // [cap][4]
    int cap;
    int* n;                    // records written
    int* seq;                  // [8] launches per tag
};
static __device__ TraceState g_trace;

__device__ __forceinline__ bool tracing() { return g_trace.buf != nullptr; }
__device__ __forceinline__ int trace_launch(int tag) { return atomicAdd(&g_trace.seq[tag], 1); }
__device__ __forceinline__ void trace_ev(int tag, int ev, int seq) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    const int i = atomicAdd(g_trace.n, 1);
    if (i < g_trace.cap) {
        unsigned long long* r = g_trace.buf + 4 * (size_t)i;
        r[0] = t; r[1] = tag; r[2] = ev; r[3] = seq;
    }
}
// host: point this translation unit's state at the shared buffer (or null)
static inline cudaError_t trace_set(const TraceState& s) { return cudaMemcpyToSymbol(g_trace, &s, sizeof(s)); }

}  // namespace fb
