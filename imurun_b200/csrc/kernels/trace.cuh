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
// every-CTA events (when TraceState::all is set), seq = linear block id |
// block count << 20
enum : int { EV_C_START = 16, EV_C_WAITED = 17, EV_C_READY = 18, EV_C_LOOP = 19, EV_C_END = 20 };
// values: consumer thread 0's and the producer's summed barrier waits (SM cycles)
enum : int { EV_C_CWAIT = 21, EV_C_PWAIT = 22 };

struct TraceState {
    unsigned long long* buf;   // [cap][4]
    int cap;
    int* n;                    // records written
    int* seq;                  // [8] launches per tag
    int all;                   // also record EV_C_* from every CTA
};
static __device__ TraceState g_trace;

__device__ __forceinline__ bool tracing() { return g_trace.buf != nullptr; }
__device__ __forceinline__ int trace_launch(int tag) { return atomicAdd(&g_trace.seq[tag], 1); }
__device__ __forceinline__ void trace_ev(int tag, int ev, long long seq) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    const int i = atomicAdd(g_trace.n, 1);
    if (i < g_trace.cap) {
        unsigned long long* r = g_trace.buf + 4 * (size_t)i;
        r[0] = t; r[1] = tag; r[2] = ev; r[3] = seq;
    }
}
// Every-CTA events without a global round trip per event: thread 0 reserves
// n_ev records once (trace_cta_begin, -1 when not recording) and then writes
// event k of the CTA with plain stores.
#ifndef FB_TRACE_CTA
#define FB_TRACE_CTA 0   // compiled in only by a tracing build
#endif
__device__ __forceinline__ bool tracing_all() { return FB_TRACE_CTA && g_trace.buf != nullptr && g_trace.all; }
__device__ __forceinline__ int trace_cta_begin(int n_ev) {
    if (threadIdx.x != 0 || !tracing_all()) return -1;
    const int i = atomicAdd(g_trace.n, n_ev);
    return i + n_ev <= g_trace.cap ? i : -1;
}
__device__ __forceinline__ void trace_cta(int base, int k, int tag, int ev) {
    if (base < 0) return;
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    const unsigned long long b = blockIdx.x + (unsigned long long)gridDim.x * (blockIdx.y + (unsigned long long)gridDim.y * blockIdx.z);
    const unsigned long long n = (unsigned long long)gridDim.x * gridDim.y * gridDim.z;
    unsigned long long* r = g_trace.buf + 4 * (size_t)(base + k);
    r[0] = t; r[1] = tag; r[2] = ev; r[3] = b | (n << 20);
}
// a value instead of a time (ns waited, counts)
__device__ __forceinline__ void trace_cta_val(int base, int k, int tag, int ev, unsigned long long v) {
    if (base < 0) return;
    const unsigned long long b = blockIdx.x + (unsigned long long)gridDim.x * (blockIdx.y + (unsigned long long)gridDim.y * blockIdx.z);
    const unsigned long long n = (unsigned long long)gridDim.x * gridDim.y * gridDim.z;
    unsigned long long* r = g_trace.buf + 4 * (size_t)(base + k);
    r[0] = v; r[1] = tag; r[2] = ev; r[3] = b | (n << 20);
}
// host: point this translation unit's state at the shared buffer (or null)
static inline cudaError_t trace_set(const TraceState& s) { return cudaMemcpyToSymbol(g_trace, &s, sizeof(s)); }

}  // namespace fb
