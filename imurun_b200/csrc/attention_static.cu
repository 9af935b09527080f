// attention_static.cu — decode attention entry point that allocates nothing.
//
// Callers that cannot allocate device memory on the call path use this entry
// point: a serving loop that owns a fixed memory budget up front (every byte of
// HBM beyond the weights is handed to the KV page pool), code running under a
// caching allocator that must not be re-entered from a foreign library, or a
// latency-critical step that may not pay for cudaMalloc/cudaFree (both can
// synchronise the device). fbx_attention, by contrast, allocates its device
// buffers and its split-partials scratch on every call.
//
// The scratch this entry point needs (the per-split softmax partials, the
// per-token positions and an identity page table) lives in one file-scope
// __device__ array of fixed size, shared by every call on a device.
#include <cuda.h>

#include <mutex>

#include "fish/fish_kernels.h"
#include "kernels/kernels.h"

namespace {

// Limits of one call. The partials of a call take T*H*n_splits*(D+2) floats
// (fbk_attention_call_floats: n_splits = ceil((pos0+T)/32) up to 2048 keys,
// ceil((pos0+T)/128) above).
constexpr int kStaticMaxKeys = 8192;
constexpr int kStaticMaxTokens = 256;
constexpr size_t kStaticPartialFloats = size_t(2) << 20;   // 8 MiB

struct StaticScratch {
    int32_t page_table[kStaticMaxKeys];   // identity: position j lives in "page" j
    int32_t tok_seq[kStaticMaxTokens];    // all zero: one sequence slot
    int32_t tok_pos[kStaticMaxTokens];    // pos0 + t, written by every call
    float partials[kStaticPartialFloats];
};

static __device__ __align__(256) StaticScratch g_attn_scratch;

// One cached address per device, tagged with the id of the context it was
// resolved in: after cudaDeviceReset the device gets a new primary context,
// the module is loaded again (the array may move and is zeroed), and the
// id no longer matches, so the set-up runs again.
constexpr int kMaxDevices = 64;
struct Resolved {
    unsigned long long ctx_id = 0;
    StaticScratch* ptr = nullptr;
};
std::mutex g_setup_mu;
Resolved g_resolved[kMaxDevices];

using PfnCtxGetCurrent = CUresult (*)(CUcontext*);
using PfnCtxGetId = CUresult (*)(CUcontext, unsigned long long*);

// Id of the current context (driver entry points looked up through the
// runtime, so the library links no libcuda soname); 0 when unavailable.
unsigned long long current_ctx_id() {
    static PfnCtxGetCurrent get_current = nullptr;
    static PfnCtxGetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<PfnCtxGetCurrent>(f);
        f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<PfnCtxGetId>(f);
    });
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS)
        return 0;
    return id;
}

__global__ void k_static_setup(StaticScratch* s) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < kStaticMaxKeys; i += gridDim.x * blockDim.x) {
        s->page_table[i] = i;
        if (i < kStaticMaxTokens) s->tok_seq[i] = 0;
    }
}

__global__ void k_static_positions(StaticScratch* s, int pos0, int T) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t < T) s->tok_pos[t] = pos0 + t;
}

// Address of this device's scratch. The first call on a device (and the
// first after a cudaDeviceReset) resolves the symbol with the device current
// and fills the identity page table and the zero sequence slots.
int scratch_for_current_device(cudaStream_t st, StaticScratch** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= kMaxDevices) return (int)cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_setup_mu);
    Resolved& r = g_resolved[dev];
    unsigned long long id = current_ctx_id();   // 0: no context current on this thread yet
    if (r.ptr && id != 0 && r.ctx_id == id) {
        *out = r.ptr;
        return 0;
    }
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_scratch);   // makes the device's context current if needed
    if (e != cudaSuccess) return (int)e;
    if (!p) return (int)cudaErrorInvalidSymbol;
    id = current_ctx_id();
    if (p != r.ptr || id == 0 || id != r.ctx_id) {
        k_static_setup<<<(kStaticMaxKeys + 255) / 256, 256, 0, st>>>(static_cast<StaticScratch*>(p));
        e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);   // later calls may come on other streams
        if (e != cudaSuccess) return (int)e;
        r.ptr = static_cast<StaticScratch*>(p);
        r.ctx_id = id;
    }
    *out = r.ptr;
    return 0;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" FISH_API int fbx_attention_static(const float* q, const void* k, const void* v, int kv_f16, int n_keys,
                                             int H, int HKV, int D, int pos0, int T, float* out, void* stream) {
    if (!q || !k || !v || !out || T <= 0 || pos0 < 0 || HKV <= 0 || H <= 0 || H % HKV || (D != 64 && D != 128))
        return -1;
    if (n_keys < pos0 + T || pos0 + T > kStaticMaxKeys || T > kStaticMaxTokens) return -1;
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out)) return -1;
    const int max_ctx = pos0 + T;   // causal: only keys [0, pos0+T) are read
    if (fbk_attention_call_floats(T, H, D, max_ctx) > kStaticPartialFloats) return -1;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    StaticScratch* s = nullptr;
    int rc = scratch_for_current_device(st, &s);
    if (rc) return rc;
    k_static_positions<<<(T + 127) / 128, 128, 0, st>>>(s, pos0, T);
    rc = (int)cudaGetLastError();
    if (rc) return rc;
    KvView kv{};
    kv.k = const_cast<void*>(k);
    kv.v = const_cast<void*>(v);
    kv.pt = s->page_table;
    kv.pt_stride = 0;
    kv.tok_seq = s->tok_seq;
    kv.tok_pos = s->tok_pos;
    kv.page_size = 1;
    kv.page_stride = (size_t)HKV * D;
    kv.layer_stride = 0;
    kv.head_stride = (size_t)D;
    kv.f16 = kv_f16 ? 1 : 0;
    kv.n_pages = kStaticMaxKeys;
    kv.err = nullptr;
    return fbk_attention(q, H * D, T, H, HKV, D, 1.0f / sqrtf((float)D), kv, 0, out, H * D, s->partials,
                         kStaticPartialFloats, max_ctx, st);
}
