// kernel_api.cpp — host-buffer entry points for single kernels
// (include/fish/fish_kernels.h). Each call allocates its device buffers, runs
// the production kernel and copies results back; they exist for parity tests.
#include <fish/fish_kernels.h>

#include <cuda_fp16.h>
#include <cuda_profiler_api.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "engine.h"
#include "kernels/kernels.h"

using namespace fb;

namespace {

struct DevBuf {
    void* p = nullptr;
    ~DevBuf() { if (p) cudaFree(p); }
    template <class T> T* as() { return static_cast<T*>(p); }
    int alloc(size_t n) { return (int)cudaMalloc(&p, n ? n : 16); }
};

#define TRY(x) do { const int rc_ = (int)(x); if (rc_) return rc_; } while (0)

int check_device() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) return (int)cudaErrorNoDevice;
    return 0;
}

// Device activation planes for rows x K (both layouts).
struct DevAct {
    DevBuf mem;
    ActQ a{};
    int make(int rows, int K) {
        const size_t ld = (size_t)((K + 15) / 16 * 16);
        const size_t nq = (size_t)rows * ld, n32 = (size_t)rows * (K / 32 + 1), n256 = (size_t)rows * (K / 256 + 1);
        TRY(mem.alloc(2 * nq + n32 * 12 + n256 * 4 + 256));
        uint8_t* p = mem.as<uint8_t>();
        auto al = [](size_t v) { return (v + 15) / 16 * 16; };
        a.q32 = (int8_t*)p; p += al(nq);
        a.qk = (int8_t*)p; p += al(nq);
        a.d32 = (float*)p; p += al(n32 * 4);
        a.s32 = (int32_t*)p; p += al(n32 * 4);
        a.dk = (float*)p; p += al(n256 * 4);
        a.bsk = (int16_t*)p;
        a.K = K;
        a.ld = (int)ld;
        return 0;
    }
};

}  // namespace

extern "C" {

int fbx_quantize_acts(const float* x, int rows, int K, void* q8act, void* q8actk) {
    if (!x || rows <= 0 || K <= 0 || K % 32) return -1;
    TRY(check_device());
    DevBuf dx;
    DevAct da;
    TRY(dx.alloc(sizeof(float) * rows * K));
    TRY(da.make(rows, K));
    TRY(cudaMemcpy(dx.p, x, sizeof(float) * rows * K, cudaMemcpyHostToDevice));
    const int wantk = q8actk && K % 256 == 0;
    TRY(fbk_quantize_rows(dx.as<float>(), K, rows, K, &da.a, q8act ? 1 : 0, wantk, nullptr));
    TRY(cudaDeviceSynchronize());
    const size_t ld = (size_t)da.a.ld;
    std::vector<int8_t> q32((size_t)rows * ld), qk((size_t)rows * ld);
    std::vector<float> d32((size_t)rows * (K / 32)), dk((size_t)rows * (K / 256) + 1);
    std::vector<int32_t> s32((size_t)rows * (K / 32));
    std::vector<int16_t> bs((size_t)rows * (K / 32));
    TRY(cudaMemcpy(q32.data(), da.a.q32, q32.size(), cudaMemcpyDeviceToHost));
    TRY(cudaMemcpy(qk.data(), da.a.qk, qk.size(), cudaMemcpyDeviceToHost));
    TRY(cudaMemcpy(d32.data(), da.a.d32, d32.size() * 4, cudaMemcpyDeviceToHost));
    TRY(cudaMemcpy(s32.data(), da.a.s32, s32.size() * 4, cudaMemcpyDeviceToHost));
    TRY(cudaMemcpy(dk.data(), da.a.dk, dk.size() * 4, cudaMemcpyDeviceToHost));
    TRY(cudaMemcpy(bs.data(), da.a.bsk, bs.size() * 2, cudaMemcpyDeviceToHost));
    if (q8act) {
        uint8_t* o = static_cast<uint8_t*>(q8act);
        for (int r = 0; r < rows; ++r)
            for (int b = 0; b < K / 32; ++b, o += 40) {
                std::memcpy(o, &d32[(size_t)r * (K / 32) + b], 4);
                std::memcpy(o + 4, &s32[(size_t)r * (K / 32) + b], 4);
                std::memcpy(o + 8, &q32[(size_t)r * ld + 32 * b], 32);
            }
    }
    if (wantk) {
        uint8_t* o = static_cast<uint8_t*>(q8actk);
        for (int r = 0; r < rows; ++r)
            for (int b = 0; b < K / 256; ++b, o += 276) {
                std::memcpy(o, &dk[(size_t)r * (K / 256) + b], 4);
                std::memcpy(o + 4, &bs[(size_t)r * (K / 32) + 8 * b], 16);
                std::memcpy(o + 20, &qk[(size_t)r * ld + 256 * b], 256);
            }
    }
    return 0;
}

int fbx_rmsnorm(const float* x, const float* w, int rows, int K, float eps, float* out) {
    if (!x || !w || !out || rows <= 0 || K <= 0) return -1;
    TRY(check_device());
    DevBuf dx, dw, dout;
    DevAct da;
    TRY(dx.alloc(sizeof(float) * rows * K));
    TRY(dw.alloc(sizeof(float) * K));
    TRY(dout.alloc(sizeof(float) * rows * K));
    TRY(da.make(rows, K));
    TRY(cudaMemcpy(dx.p, x, sizeof(float) * rows * K, cudaMemcpyHostToDevice));
    TRY(cudaMemcpy(dw.p, w, sizeof(float) * K, cudaMemcpyHostToDevice));
    TRY(fbk_rmsnorm_quant(dx.as<float>(), K, dw.as<float>(), eps, rows, K, dout.as<float>(), K, &da.a, 0, 0, nullptr));
    TRY(cudaDeviceSynchronize());
    TRY(cudaMemcpy(out, dout.p, sizeof(float) * rows * K, cudaMemcpyDeviceToHost));
    return 0;
}

static int upload_rows(int type, const void* w, int n_in, int n_out, DevBuf& dw, size_t* stride) {
    const size_t st = dev_row_bytes(type, n_in);
    if (!st) return -1;
    std::vector<uint8_t> h(dev_matrix_bytes(type, n_in, n_out));
    repack_rows(type, static_cast<const uint8_t*>(w), n_out, n_in, h.data());
    TRY(dw.alloc(h.size()));
    TRY(cudaMemcpy(dw.p, h.data(), h.size(), cudaMemcpyHostToDevice));
    *stride = st;
    return 0;
}

int fbx_matmul(int type, const void* w, int n_in, int n_out, const float* x, int T, float* y) {
    if (!w || !x || !y || n_in <= 0 || n_out <= 0 || T <= 0 || T > kMaxBatch) return -1;
    if ((type == T_Q4_K || type == T_Q6_K) && n_in % 256) return -1;
    if (type == T_Q8_0 && n_in % 32) return -1;
    TRY(check_device());
    DevBuf dw, dx, dy;
    DevAct da;
    size_t stride = 0;
    TRY(upload_rows(type, w, n_in, n_out, dw, &stride));
    TRY(dx.alloc(sizeof(float) * T * n_in));
    TRY(dy.alloc(sizeof(float) * T * n_out));
    TRY(da.make(T + 8, n_in));
    TRY(cudaMemcpy(dx.p, x, sizeof(float) * T * n_in, cudaMemcpyHostToDevice));
    // scratch for the tensor-core kernel's K split (half-group units)
    DevBuf dpart;
    const size_t part_floats = (size_t)((n_in / 256 + 3) / 4 + 1) * T * n_out;
    TRY(dpart.alloc(sizeof(float) * part_floats));
    const bool quant = type == T_Q8_0 || type == T_Q4_K || type == T_Q6_K;
    if (quant) TRY(fbk_quantize_rows(dx.as<float>(), n_in, T, n_in, &da.a, type == T_Q8_0, type != T_Q8_0, nullptr));
    // T >= 16 quantised rows go to the tensor-core kernel in one launch,
    // otherwise GEMV launches of up to 4 (streamed) or 8 tokens
    int step = 8;
    {
        GemvArgs probe{};
        probe.nseg = 1;
        probe.K = n_in;
        probe.T = T;
        probe.act = da.a;
        probe.seg[0].type = type;
        probe.seg[0].rows = n_out;
        step = fbk_gemv_chunk(&probe);
        if (fbk_gemm_eligible(&probe)) step = T;
    }
    for (int t0 = 0; t0 < T; t0 += step) {
        GemvArgs g{};
        g.nseg = 1;
        g.K = n_in;
        g.T = T - t0 < step ? T - t0 : step;
        g.act = da.a;
        g.act.q32 = da.a.q32 + (size_t)t0 * da.a.ld;
        g.act.qk = da.a.qk + (size_t)t0 * da.a.ld;
        g.act.d32 = da.a.d32 + (size_t)t0 * (n_in / 32);
        g.act.s32 = da.a.s32 + (size_t)t0 * (n_in / 32);
        g.act.dk = da.a.dk + (size_t)t0 * (n_in / 256);
        g.act.bsk = da.a.bsk + (size_t)t0 * (n_in / 32);
        g.xf = dx.as<float>() + (size_t)t0 * n_in;
        g.ldxf = n_in;
        g.seg[0].type = type;
        g.seg[0].w = dw.as<uint8_t>();
        g.seg[0].row_stride = stride;
        g.seg[0].w_bytes = dev_matrix_bytes(type, n_in, n_out);
        g.seg[0].rows = n_out;
        g.seg[0].y = dy.as<float>() + (size_t)t0 * n_out;
        g.seg[0].ldy = n_out;
        g.seg[0].epi = EPI_STORE;
        g.part = dpart.as<float>();
        g.part_floats = part_floats;
        if (fbk_gemm_eligible(&g)) TRY(fbk_gemm(&g, nullptr));
        else TRY(fbk_gemv(&g, nullptr));
    }
    TRY(cudaDeviceSynchronize());
    TRY(cudaMemcpy(y, dy.p, sizeof(float) * T * n_out, cudaMemcpyDeviceToHost));
    return 0;
}

int fbx_profiler(int start) { return (int)(start ? cudaProfilerStart() : cudaProfilerStop()); }

int fbx_time_matmul(int type, int n_in, int n_out, int T, int iters, float* ms_per_launch, double* bytes_per_launch) {
    if (!ms_per_launch || n_in <= 0 || n_out <= 0 || T <= 0 || T > kMaxBatch || iters <= 0) return -1;
    if (type != T_Q8_0 && type != T_Q4_K && type != T_Q6_K && type != T_F32 && type != T_F16) return -1;
    TRY(check_device());
    const size_t stride = dev_row_bytes(type, n_in);
    const size_t mat = (dev_matrix_bytes(type, n_in, n_out) + 255) / 256 * 256;
    const int copies = (int)std::max<size_t>(1, ((512ull << 20) + mat - 1) / mat);
    DevBuf dw, dx, dy;
    DevAct da;
    TRY(dw.alloc(mat * copies));
    TRY(cudaMemset(dw.p, 0x11, mat * copies));
    TRY(dx.alloc(sizeof(float) * T * n_in));
    TRY(dy.alloc(sizeof(float) * T * n_out));
    TRY(da.make(T, n_in));   // planes for all T rows (the quantiser writes T rows)
    std::vector<float> hx((size_t)T * n_in);
    for (size_t i = 0; i < hx.size(); ++i) hx[i] = (float)((i * 2654435761u) % 1000) / 500.0f - 1.0f;
    TRY(cudaMemcpy(dx.p, hx.data(), hx.size() * 4, cudaMemcpyHostToDevice));
    if (type == T_Q8_0 || type == T_Q4_K || type == T_Q6_K)
        TRY(fbk_quantize_rows(dx.as<float>(), n_in, T, n_in, &da.a, type == T_Q8_0, type != T_Q8_0, nullptr));
    cudaStream_t st;
    TRY(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    GemvArgs g{};
    g.nseg = 1;
    g.K = n_in;
    g.T = T;
    g.act = da.a;
    g.xf = dx.as<float>();
    g.ldxf = n_in;
    g.seg[0].type = type;
    g.seg[0].row_stride = stride;
    g.seg[0].w_bytes = mat;
    g.seg[0].rows = n_out;
    g.seg[0].y = dy.as<float>();
    g.seg[0].ldy = n_out;
    g.seg[0].epi = EPI_STORE;
    DevBuf dpart;
    g.part_floats = (size_t)((n_in / 256 + 3) / 4 + 1) * T * n_out;
    TRY(dpart.alloc(sizeof(float) * g.part_floats));
    g.part = dpart.as<float>();
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    int rc = 0;
    const bool gemm = fbk_gemm_eligible(&g) != 0;
    const int chunk = gemm ? T : fbk_gemv_chunk(&g);   // as the engine splits a call
    for (int i = 0; i < 3 + iters && !rc; ++i) {
        if (i == 3) cudaEventRecord(e0, st);
        g.seg[0].w = dw.as<uint8_t>() + (size_t)(i % copies) * mat;
        for (int t0 = 0; t0 < T && !rc; t0 += chunk) {
            GemvArgs c = g;
            c.T = std::min(chunk, T - t0);
            if (da.a.q32) c.act.q32 = da.a.q32 + (size_t)t0 * da.a.ld;
            if (da.a.qk) c.act.qk = da.a.qk + (size_t)t0 * da.a.ld;
            if (da.a.d32) c.act.d32 = da.a.d32 + (size_t)t0 * (n_in / 32);
            if (da.a.s32) c.act.s32 = da.a.s32 + (size_t)t0 * (n_in / 32);
            if (da.a.dk) c.act.dk = da.a.dk + (size_t)t0 * (n_in / 256);
            if (da.a.bsk) c.act.bsk = da.a.bsk + (size_t)t0 * (n_in / 32);
            c.xf = dx.as<float>() + (size_t)t0 * n_in;
            c.seg[0].y = dy.as<float>() + (size_t)t0 * n_out;
            rc = gemm ? fbk_gemm(&c, st) : fbk_gemv(&c, st);
        }
    }
    cudaEventRecord(e1, st);
    const int sync = (int)cudaStreamSynchronize(st);
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaStreamDestroy(st);
    if (rc) return rc;
    if (sync) return sync;
    *ms_per_launch = ms / iters;
    if (bytes_per_launch) *bytes_per_launch = (double)ggml_row_bytes(type, (uint64_t)n_in) * n_out + 4.0 * n_out * T;
    return 0;
}

int fbx_block_sums(int type, const void* w, int n_in, int n_out, const void* acts, int32_t* sumi, int32_t* mins) {
    if (!w || !acts || !sumi || n_in <= 0 || n_out <= 0) return -1;
    if (type != T_Q8_0 && type != T_Q4_K && type != T_Q6_K) return -1;
    const bool k = type != T_Q8_0;
    if (n_in % (k ? 256 : 32)) return -1;
    TRY(check_device());
    DevBuf dw, ds, dm;
    DevAct da;
    size_t stride = 0;
    TRY(upload_rows(type, w, n_in, n_out, dw, &stride));
    TRY(da.make(1, n_in));
    // unpack the reference records into the device planes
    const uint8_t* a = static_cast<const uint8_t*>(acts);
    std::vector<int8_t> q(da.a.ld, 0);
    if (k) {
        std::vector<float> d(n_in / 256);
        std::vector<int16_t> bs(n_in / 32);
        for (int b = 0; b < n_in / 256; ++b) {
            std::memcpy(&d[b], a + 276 * b, 4);
            std::memcpy(&bs[8 * b], a + 276 * b + 4, 16);
            std::memcpy(&q[256 * b], a + 276 * b + 20, 256);
        }
        TRY(cudaMemcpy(da.a.qk, q.data(), q.size(), cudaMemcpyHostToDevice));
        TRY(cudaMemcpy(da.a.dk, d.data(), d.size() * 4, cudaMemcpyHostToDevice));
        TRY(cudaMemcpy(da.a.bsk, bs.data(), bs.size() * 2, cudaMemcpyHostToDevice));
    } else {
        std::vector<float> d(n_in / 32);
        for (int b = 0; b < n_in / 32; ++b) {
            std::memcpy(&d[b], a + 40 * b, 4);
            std::memcpy(&q[32 * b], a + 40 * b + 8, 32);
        }
        TRY(cudaMemcpy(da.a.q32, q.data(), q.size(), cudaMemcpyHostToDevice));
        TRY(cudaMemcpy(da.a.d32, d.data(), d.size() * 4, cudaMemcpyHostToDevice));
    }
    const int nb = n_in / (k ? 256 : 32);
    TRY(ds.alloc(sizeof(int32_t) * (size_t)n_out * nb));
    TRY(dm.alloc(sizeof(int32_t) * (size_t)n_out * nb));
    TRY(cudaMemset(dm.p, 0, sizeof(int32_t) * (size_t)n_out * nb));
    TRY(fbk_block_sums(type, dw.as<uint8_t>(), n_out, n_in, &da.a, ds.as<int32_t>(), dm.as<int32_t>(), nullptr));
    TRY(cudaDeviceSynchronize());
    TRY(cudaMemcpy(sumi, ds.p, sizeof(int32_t) * (size_t)n_out * nb, cudaMemcpyDeviceToHost));
    if (mins) TRY(cudaMemcpy(mins, dm.p, sizeof(int32_t) * (size_t)n_out * nb, cudaMemcpyDeviceToHost));
    return 0;
}

// A one-layer paged pool whose page i holds positions [16i, 16i+16).
struct TestPool {
    DevBuf pool, pt, seq, pos;
    KvView kv{};
    int make(int n_pos, int HKV, int D, int f16, int T, int pos0) {
        const int P = kPageSize, np = (n_pos + P - 1) / P;
        const size_t head = (size_t)P * D, vofs = (size_t)HKV * head, page = 2 * vofs;
        const size_t esz = f16 ? 2 : 4;
        TRY(pool.alloc(page * np * esz));
        TRY(cudaMemset(pool.p, 0, page * np * esz));
        std::vector<int32_t> hp(np), hs(T, 0), hq(T);
        for (int i = 0; i < np; ++i) hp[i] = i;
        for (int t = 0; t < T; ++t) hq[t] = pos0 + t;
        TRY(pt.alloc(sizeof(int32_t) * np));
        TRY(seq.alloc(sizeof(int32_t) * T));
        TRY(pos.alloc(sizeof(int32_t) * T));
        TRY(cudaMemcpy(pt.p, hp.data(), sizeof(int32_t) * np, cudaMemcpyHostToDevice));
        TRY(cudaMemcpy(seq.p, hs.data(), sizeof(int32_t) * T, cudaMemcpyHostToDevice));
        TRY(cudaMemcpy(pos.p, hq.data(), sizeof(int32_t) * T, cudaMemcpyHostToDevice));
        kv.f16 = f16;
        kv.n_pages = np;
        kv.err = fbk_gemv_error_flag();
        kv.k = pool.p;
        kv.v = static_cast<uint8_t*>(pool.p) + vofs * esz;
        kv.pt = pt.as<int32_t>();
        kv.pt_stride = np;
        kv.tok_seq = seq.as<int32_t>();
        kv.tok_pos = pos.as<int32_t>();
        kv.page_size = P;
        kv.page_stride = page;
        kv.layer_stride = page;
        kv.head_stride = head;
        return 0;
    }
};

// fbx_attention / fbx_attention_prefill: the cache built from host K/V rows,
// then the split-key kernel (tc = 0) or the tensor-core prefill kernel
static int attention_host(const float* q, const float* k, const float* v, int n_keys, int H, int HKV, int D, int pos0,
                          int T, int kv_f16, float* out, int tc) {
    if (!q || !k || !v || !out || T <= 0 || pos0 < 0 || pos0 + T > n_keys || H % HKV || (D != 64 && D != 96 && D != 128))
        return -1;
    TRY(check_device());
    TestPool tp;
    TRY(tp.make(n_keys, HKV, D, kv_f16, T, pos0));
    const int P = kPageSize, np = (n_keys + P - 1) / P;
    const size_t head = (size_t)P * D, vofs = (size_t)HKV * head, page = 2 * vofs;
    std::vector<float> hf(page * np, 0.0f);
    for (int j = 0; j < n_keys; ++j)
        for (int h = 0; h < HKV; ++h)
            for (int d = 0; d < D; ++d) {
                const size_t o = (size_t)(j / P) * page + h * head + (size_t)(j % P) * D + d;
                hf[o] = k[(size_t)j * HKV * D + h * D + d];
                hf[o + vofs] = v[(size_t)j * HKV * D + h * D + d];
            }
    if (kv_f16) {
        std::vector<__half> hh(hf.size());
        for (size_t i = 0; i < hf.size(); ++i) hh[i] = __float2half_rn(hf[i]);
        TRY(cudaMemcpy(tp.pool.p, hh.data(), hh.size() * 2, cudaMemcpyHostToDevice));
    } else {
        TRY(cudaMemcpy(tp.pool.p, hf.data(), hf.size() * 4, cudaMemcpyHostToDevice));
    }
    DevBuf dq, dout, scratch;
    const size_t sf = fbk_attention_scratch_floats(T, H, D, pos0 + T);
    TRY(dq.alloc(sizeof(float) * T * H * D));
    TRY(dout.alloc(sizeof(float) * T * H * D));
    TRY(scratch.alloc(sizeof(float) * sf));
    TRY(cudaMemcpy(dq.p, q, sizeof(float) * T * H * D, cudaMemcpyHostToDevice));
    if (tc)
        TRY(fbk_attention_prefill(dq.as<float>(), H * D, T, H, HKV, D, 1.0f / std::sqrt((float)D), tp.kv, 0,
                                  dout.as<float>(), H * D, nullptr));
    else
        TRY(fbk_attention(dq.as<float>(), H * D, T, H, HKV, D, 1.0f / std::sqrt((float)D), tp.kv, 0, dout.as<float>(),
                          H * D, scratch.as<float>(), sf, pos0 + T, nullptr));
    TRY(cudaDeviceSynchronize());
    TRY(cudaMemcpy(out, dout.p, sizeof(float) * T * H * D, cudaMemcpyDeviceToHost));
    return 0;
}

int fbx_attention(const float* q, const float* k, const float* v, int n_keys, int H, int HKV, int D, int pos0, int T,
                  int kv_f16, float* out) {
    return attention_host(q, k, v, n_keys, H, HKV, D, pos0, T, kv_f16, out, 0);
}

int fbx_attention_prefill(const float* q, const float* k, const float* v, int n_keys, int H, int HKV, int D, int pos0,
                          int T, float* out) {
    return attention_host(q, k, v, n_keys, H, HKV, D, pos0, T, 1, out, 1);
}

int fbx_attention_decode(const float* q, const float* k_cache, const float* v_cache, const float* k_new,
                         const float* v_new, int pos, int H, int HKV, int D, int rot_dim, int neox, float freq_base,
                         int kv_f16, float* out, float* k_stored, float* v_stored) {
    if (!q || !k_new || !v_new || !out || pos < 0 || (pos > 0 && (!k_cache || !v_cache)) || H % HKV ||
        (D != 64 && D != 96 && D != 128) || rot_dim <= 0 || rot_dim > D || rot_dim % 2)
        return -1;
    TRY(check_device());
    const int n_keys = pos + 1;
    TestPool tp;
    TRY(tp.make(n_keys, HKV, D, kv_f16, 1, pos));
    const int P = kPageSize, np = (n_keys + P - 1) / P;
    const size_t head = (size_t)P * D, vofs = (size_t)HKV * head, page = 2 * vofs;
    std::vector<float> hf(page * np, 0.0f);
    for (int j = 0; j < pos; ++j)
        for (int h = 0; h < HKV; ++h)
            for (int d = 0; d < D; ++d) {
                const size_t o = (size_t)(j / P) * page + h * head + (size_t)(j % P) * D + d;
                hf[o] = k_cache[(size_t)j * HKV * D + h * D + d];
                hf[o + vofs] = v_cache[(size_t)j * HKV * D + h * D + d];
            }
    if (kv_f16) {
        std::vector<__half> hh(hf.size());
        for (size_t i = 0; i < hf.size(); ++i) hh[i] = __float2half_rn(hf[i]);
        TRY(cudaMemcpy(tp.pool.p, hh.data(), hh.size() * 2, cudaMemcpyHostToDevice));
    } else {
        TRY(cudaMemcpy(tp.pool.p, hf.data(), hf.size() * 4, cudaMemcpyHostToDevice));
    }
    Config c;
    c.n_ctx = n_keys;
    c.rot_dim = rot_dim;
    c.head_dim = D;
    c.freq_base = freq_base;
    std::vector<float> cs, sn;
    build_rope_table(c, nullptr, cs, sn);
    DevBuf dq, dk, dv, dout, dc, ds;
    TRY(dq.alloc(sizeof(float) * H * D));
    TRY(dk.alloc(sizeof(float) * HKV * D));
    TRY(dv.alloc(sizeof(float) * HKV * D));
    TRY(dout.alloc(sizeof(float) * H * D));
    TRY(dc.alloc(sizeof(float) * cs.size()));
    TRY(ds.alloc(sizeof(float) * sn.size()));
    TRY(cudaMemcpy(dq.p, q, sizeof(float) * H * D, cudaMemcpyHostToDevice));
    TRY(cudaMemcpy(dk.p, k_new, sizeof(float) * HKV * D, cudaMemcpyHostToDevice));
    TRY(cudaMemcpy(dv.p, v_new, sizeof(float) * HKV * D, cudaMemcpyHostToDevice));
    TRY(cudaMemcpy(dc.p, cs.data(), sizeof(float) * cs.size(), cudaMemcpyHostToDevice));
    TRY(cudaMemcpy(ds.p, sn.data(), sizeof(float) * sn.size(), cudaMemcpyHostToDevice));
    TRY(fbk_attention_decode(dq.as<float>(), H * D, dk.as<float>(), dv.as<float>(), HKV * D, 1, H, HKV, D,
                             1.0f / std::sqrt((float)D), rot_dim, neox, dc.as<float>(), ds.as<float>(), tp.kv, 0,
                             dout.as<float>(), H * D, nullptr, 0, nullptr, nullptr, 0, nullptr));
    TRY(cudaDeviceSynchronize());
    TRY(cudaMemcpy(out, dout.p, sizeof(float) * H * D, cudaMemcpyDeviceToHost));
    if (k_stored || v_stored) {
        const size_t esz = kv_f16 ? 2 : 4;
        std::vector<uint8_t> raw(page * np * esz);
        TRY(cudaMemcpy(raw.data(), tp.pool.p, raw.size(), cudaMemcpyDeviceToHost));
        for (int h = 0; h < HKV; ++h)
            for (int d = 0; d < D; ++d) {
                const size_t o = (size_t)(pos / P) * page + h * head + (size_t)(pos % P) * D + d;
                float kx, vx;
                if (kv_f16) {
                    kx = __half2float(reinterpret_cast<const __half*>(raw.data())[o]);
                    vx = __half2float(reinterpret_cast<const __half*>(raw.data())[o + vofs]);
                } else {
                    kx = reinterpret_cast<const float*>(raw.data())[o];
                    vx = reinterpret_cast<const float*>(raw.data())[o + vofs];
                }
                if (k_stored) k_stored[h * D + d] = kx;
                if (v_stored) v_stored[h * D + d] = vx;
            }
    }
    return 0;
}

int fbx_rope(float* q, float* k, int T, int H, int HKV, int D, int rot_dim, int neox, float freq_base, int pos0) {
    if (!q || !k || T <= 0 || pos0 < 0 || rot_dim <= 0 || rot_dim > D || D % 2) return -1;
    TRY(check_device());
    Config c;
    c.n_ctx = pos0 + T;
    c.rot_dim = rot_dim;
    c.head_dim = D;
    c.freq_base = freq_base;
    std::vector<float> cs, sn;
    build_rope_table(c, nullptr, cs, sn);
    TestPool tp;
    TRY(tp.make(pos0 + T, HKV, D, 0, T, pos0));
    DevBuf dq, dk, dv, dc, ds;
    TRY(dq.alloc(sizeof(float) * T * H * D));
    TRY(dk.alloc(sizeof(float) * T * HKV * D));
    TRY(dv.alloc(sizeof(float) * T * HKV * D));
    TRY(dc.alloc(sizeof(float) * cs.size()));
    TRY(ds.alloc(sizeof(float) * sn.size()));
    TRY(cudaMemcpy(dq.p, q, sizeof(float) * T * H * D, cudaMemcpyHostToDevice));
    TRY(cudaMemcpy(dk.p, k, sizeof(float) * T * HKV * D, cudaMemcpyHostToDevice));
    TRY(cudaMemset(dv.p, 0, sizeof(float) * T * HKV * D));
    TRY(cudaMemcpy(dc.p, cs.data(), sizeof(float) * cs.size(), cudaMemcpyHostToDevice));
    TRY(cudaMemcpy(ds.p, sn.data(), sizeof(float) * sn.size(), cudaMemcpyHostToDevice));
    TRY(fbk_rope_append(dq.as<float>(), H * D, dk.as<float>(), dv.as<float>(), HKV * D, T, H, HKV, D, rot_dim, neox,
                        dc.as<float>(), ds.as<float>(), tp.kv, 0, nullptr));
    TRY(cudaDeviceSynchronize());
    TRY(cudaMemcpy(q, dq.p, sizeof(float) * T * H * D, cudaMemcpyDeviceToHost));
    const int P = kPageSize;
    const size_t head = (size_t)P * D;
    std::vector<float> pool(tp.kv.page_stride * ((pos0 + T + P - 1) / P));
    TRY(cudaMemcpy(pool.data(), tp.pool.p, pool.size() * 4, cudaMemcpyDeviceToHost));
    for (int t = 0; t < T; ++t) {
        const int j = pos0 + t;
        for (int h = 0; h < HKV; ++h)
            for (int d = 0; d < D; ++d)
                k[(size_t)t * HKV * D + h * D + d] = pool[(size_t)(j / P) * tp.kv.page_stride + h * head + (size_t)(j % P) * D + d];
    }
    return 0;
}

int fbx_argmax(const float* x, int rows, int n, int32_t* out) {
    if (!x || !out || rows <= 0 || n <= 0) return -1;
    TRY(check_device());
    DevBuf dx, dout;
    TRY(dx.alloc(sizeof(float) * (size_t)rows * n));
    TRY(dout.alloc(sizeof(int32_t) * rows));
    TRY(cudaMemcpy(dx.p, x, sizeof(float) * (size_t)rows * n, cudaMemcpyHostToDevice));
    TRY(fbk_argmax(dx.as<float>(), n, rows, n, dout.as<int32_t>(), nullptr));
    TRY(cudaDeviceSynchronize());
    TRY(cudaMemcpy(out, dout.p, sizeof(int32_t) * rows, cudaMemcpyDeviceToHost));
    return 0;
}

int fbx_argmax_penalized(const float* x, int n, const int32_t* recent, int n_recent, float penalty, int32_t* out) {
    if (!x || !out || n <= 0 || n_recent < 0 || n_recent > kMaxRecent || (n_recent > 0 && !recent)) return -1;
    TRY(check_device());
    DevBuf dx, dr, dout;
    TRY(dx.alloc(sizeof(float) * (size_t)n));
    TRY(dr.alloc(sizeof(int32_t) * (size_t)(n_recent > 0 ? n_recent : 1)));
    TRY(dout.alloc(sizeof(int32_t)));
    TRY(cudaMemcpy(dx.p, x, sizeof(float) * (size_t)n, cudaMemcpyHostToDevice));
    if (n_recent > 0) TRY(cudaMemcpy(dr.p, recent, sizeof(int32_t) * (size_t)n_recent, cudaMemcpyHostToDevice));
    TRY(fbk_argmax_penalized(dx.as<float>(), n, dr.as<int32_t>(), n_recent, penalty, dout.as<int32_t>(), nullptr));
    TRY(cudaDeviceSynchronize());
    TRY(cudaMemcpy(out, dout.p, sizeof(int32_t), cudaMemcpyDeviceToHost));
    return 0;
}

int fbx_tp_plan(int n_head, int n_head_kv, int head_dim, int n_ff, int vocab, int n_experts, int rank, int world,
                int32_t* out) {
    if (!out) return -1;
    fb::TpPlan p;
    if (!fb::tp_plan(n_head, n_head_kv, head_dim, n_ff, vocab, n_experts, rank, world, &p, nullptr)) return -1;
    const int32_t v[14] = {p.head0, p.heads, p.kv_head0, p.kv_heads, p.q_row0, p.q_rows, p.kv_row0, p.kv_rows,
                           p.ff_row0, p.ff_rows, p.expert0, p.experts, p.vocab_row0, p.vocab_rows};
    std::memcpy(out, v, sizeof(v));
    return 0;
}

int fbx_moe_localize_host(const int32_t* sel, int n, int e0, int n_local, int32_t* out) {
    if (!sel || !out || n < 0 || n_local < 0) return -1;
    for (int i = 0; i < n; ++i) out[i] = fb_localize_expert(sel[i], e0, n_local);
    return 0;
}

int fbx_embed(int type, const void* table, int E, int n_rows, const int32_t* ids, int T, float* out) {
    if (!table || !ids || !out || E <= 0 || n_rows <= 0 || T <= 0) return -1;
    for (int t = 0; t < T; ++t) if (ids[t] < 0 || ids[t] >= n_rows) return -1;
    TRY(check_device());
    DevBuf dw, di, dout;
    size_t stride = 0;
    TRY(upload_rows(type, table, E, n_rows, dw, &stride));
    TRY(di.alloc(sizeof(int32_t) * T));
    TRY(dout.alloc(sizeof(float) * (size_t)T * E));
    TRY(cudaMemcpy(di.p, ids, sizeof(int32_t) * T, cudaMemcpyHostToDevice));
    TRY(fbk_embed(type, dw.as<uint8_t>(), E, n_rows, di.as<int32_t>(), T, dout.as<float>(), E, fbk_gemv_error_flag(),
                  nullptr));
    TRY(cudaDeviceSynchronize());
    TRY(cudaMemcpy(out, dout.p, sizeof(float) * (size_t)T * E, cudaMemcpyDeviceToHost));
    return 0;
}

}  // extern "C"
