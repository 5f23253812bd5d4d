// g4_testapi.cu — single-kernel C entry points (host buffers in and out) and
// the logits top-k kernel.
//
// The g4k_* functions let parity tests drive one kernel at a time through the
// C ABI on seeded inputs; each call allocates and frees its own device
// buffers, so they are for testing, not for the hot path.
#include <cuda_runtime.h>
#include <math.h>
#include <stdio.h>

#include <mutex>
#include <vector>

#include "../../include/g4cuda.h"
#include "g4_common.cuh"
#include "g4_internal.h"

cudaError_t g4_launch_gemm_tc(const GemmArgs &a, cudaStream_t st, bool pdl);
cudaError_t g4_launch_gemm_simt(const GemmArgs &a, cudaStream_t st, bool pdl);
bool g4_gemm_tc_supported(const GemmArgs &a);
cudaError_t g4_launch_mma_peak(int iters, int *err, cudaStream_t st, double *ops);

namespace {

// Top-k in two passes: each CTA selects the k best of its slice (value
// descending, id ascending on ties, gemma4.c:544-551), then one CTA merges.
constexpr int kTopkThreads = 256;
constexpr int kTopkSlice = 4096;

__device__ void block_best(float v, int i, float *rv, int *ri, float *outv, int *outi) {
    // reduce (v desc, i asc) over the block
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float v2 = __shfl_xor_sync(0xffffffffu, v, o);
        int i2 = __shfl_xor_sync(0xffffffffu, i, o);
        if (v2 > v || (v2 == v && i2 < i)) { v = v2; i = i2; }
    }
    if (lane == 0) { rv[warp] = v; ri[warp] = i; }
    __syncthreads();
    if (threadIdx.x == 0) {
        float bv = rv[0];
        int bi = ri[0];
        for (int w = 1; w < kTopkThreads / 32; w++)
            if (rv[w] > bv || (rv[w] == bv && ri[w] < bi)) { bv = rv[w]; bi = ri[w]; }
        *outv = bv;
        *outi = bi;
    }
    __syncthreads();
}

// SLICE values per CTA; ids are explicit (xi) or the global index.
template <int SLICE>
__global__ void __launch_bounds__(kTopkThreads) k_topk_pass(const float *x, const int *xi, int n, int k, float *ov,
                                                            int *oi) {
    __shared__ float sv[SLICE];
    __shared__ int si[SLICE];
    __shared__ float rv[8];
    __shared__ int ri[8];
    __shared__ float bv;
    __shared__ int bi;
    const int base = blockIdx.x * SLICE;
    for (int j = threadIdx.x; j < SLICE; j += kTopkThreads) {
        const int g = base + j;
        sv[j] = g < n ? x[g] : -INFINITY;
        si[j] = g < n ? (xi ? xi[g] : g) : 0x7fffffff;
    }
    __syncthreads();
    for (int r = 0; r < k; r++) {
        float v = -INFINITY;
        int i = 0x7fffffff, pos = -1;
        for (int j = threadIdx.x; j < SLICE; j += kTopkThreads)
            if (sv[j] > v || (sv[j] == v && si[j] < i)) { v = sv[j]; i = si[j]; pos = j; }
        block_best(v, i, rv, ri, &bv, &bi);
        if (pos >= 0 && i == bi) { sv[pos] = -INFINITY; si[pos] = 0x7fffffff; }
        if (threadIdx.x == 0) {
            ov[blockIdx.x * k + r] = bv;
            oi[blockIdx.x * k + r] = bi;
        }
        __syncthreads();
    }
}

struct DevBuf {
    void *p = nullptr;
    ~DevBuf() { if (p) cudaFree(p); }
    cudaError_t alloc(size_t n) { return cudaMalloc(&p, n ? n : 16); }
};

#define TK(call)                                        \
    do {                                                \
        cudaError_t e_ = (call);                        \
        if (e_ != cudaSuccess) return G4_ERR_CUDA;      \
    } while (0)

int num_sms() {
    int dev = 0, n = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

}  // namespace

// ---------------------------------------------------------------------------
// Top-k without any allocation, for hosts that must not allocate device
// memory on their decode path. Its only scratch is the first pass's per-slice
// candidate list, kept in a fixed array in the library's device image: each
// GPU that loads the library reserves it (32 KB) until the process exits.
constexpr int kNoAllocSlice = 4096;
constexpr int kNoAllocMaxN = 64 * kNoAllocSlice;   // one 262144-entry vocabulary row
constexpr int kNoAllocMaxK = 64;
static __device__ __align__(256) float g_topk_cand_v[(kNoAllocMaxN / kNoAllocSlice) * kNoAllocMaxK];
static __device__ __align__(256) int g_topk_cand_i[(kNoAllocMaxN / kNoAllocSlice) * kNoAllocMaxK];

// Device addresses of the arrays above, resolved once per device. In host code
// the array names only stand in for the symbols; kernels must be given these.
struct NoAllocScratch {
    bool ready = false;
    float *v = nullptr;
    int *i = nullptr;
};
static NoAllocScratch g_noalloc[64];
static std::mutex g_noalloc_mu;

static cudaError_t noalloc_scratch(int dev, NoAllocScratch *out) {
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    NoAllocScratch &s = g_noalloc[dev];
    if (!s.ready) {
        cudaError_t e = cudaGetSymbolAddress((void **)&s.v, g_topk_cand_v);
        if (e != cudaSuccess) return e;
        e = cudaGetSymbolAddress((void **)&s.i, g_topk_cand_i);
        if (e != cudaSuccess) return e;
        s.ready = true;
    }
    *out = s;
    return cudaSuccess;
}

cudaError_t g4_launch_topk(const float *x, int n, int k, float *part_v, int *part_i, float *vals, int *ids,
                           cudaStream_t st) {
    // pass 1: 4096-value slices (64 CTAs for the vocabulary); pass 2: one CTA
    // over the <= 64 x k candidates
    constexpr int kSlice1 = 4096;
    const int blocks = (n + kSlice1 - 1) / kSlice1;
    const int m = blocks * k;
    if (k < 1 || k > 64 || m > kTopkSlice) return cudaErrorInvalidValue;
    k_topk_pass<kSlice1><<<blocks, kTopkThreads, 0, st>>>(x, nullptr, n, k, part_v, part_i);
    k_topk_pass<kTopkSlice><<<1, kTopkThreads, 0, st>>>(part_v, part_i, m, k, vals, ids);
    return cudaGetLastError();
}

// Temperature sampling over the top 64 (gemma4.c:527-561), one warp: the
// candidates are the top-64 list (value descending, id ascending on ties, as
// the reference's insertion keeps them); expf terms in parallel with the host
// library's expf, then the reference's sequential sum, 95 % prefix, xorshift
// draw and walk in one lane. temperature <= 0: the first maximum (argmax).
__global__ void k_sample64(const float *vals, const int *ids, float temperature, unsigned long long *state,
                           int *token) {
    __shared__ float e[64];
    const int lane = threadIdx.x;
    if (!(temperature > 0.0f)) {
        if (lane == 0) *token = ids[0];
        return;
    }
    const float mx = __fdiv_rn(vals[0], temperature);
    for (int i = lane; i < 64; i += 32) e[i] = expf_host(__fsub_rn(__fdiv_rn(vals[i], temperature), mx));
    __syncwarp();
    if (lane != 0) return;
    float sum = 0.0f;
    for (int i = 0; i < 64; i++) sum = __fadd_rn(sum, e[i]);
    const float lim = __fmul_rn(0.95f, sum);
    float mass = 0.0f;
    int count = 0;
    while (count < 64 && mass < lim) mass = __fadd_rn(mass, e[count++]);
    unsigned long long x = *state;   // random_uniform (gemma4.c:529-534)
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *state = x;
    const float u = __fdiv_rn((float)((x * 0x2545F4914F6CDD1DULL) >> 40), 16777216.0f);
    float th = __fmul_rn(u, mass);
    int tok = ids[count > 0 ? count - 1 : 0];
    for (int i = 0; i < count; i++) {
        th = __fsub_rn(th, e[i]);
        if (th <= 0.0f) {
            tok = ids[i];
            break;
        }
    }
    *token = tok;
}

cudaError_t g4_launch_sample64(const float *vals, const int *ids, float temperature, unsigned long long *state,
                               int *token, cudaStream_t st) {
    k_sample64<<<1, 32, 0, st>>>(vals, ids, temperature, state, token);
    return cudaGetLastError();
}

extern "C" {

int g4_topk_noalloc(const float *logits, int n, int k, float *values, int *ids, void *stream) {
    if (!logits || !values || !ids || k < 1 || k > kNoAllocMaxK || n < k) return G4_ERR_INVALID;
    if (n > kNoAllocMaxN) return G4_ERR_INVALID;   // beyond the fixed scratch
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return G4_ERR_CUDA;
    NoAllocScratch s;
    if (noalloc_scratch(dev, &s) != cudaSuccess) return G4_ERR_CUDA;
    // pass 1 writes blocks * k candidates and pass 2 reads exactly those, so
    // nothing in the shared scratch has to start at zero. Each launch reports
    // its own status (an earlier, unrelated error pending on this thread is
    // neither returned nor cleared here).
    const cudaStream_t st = (cudaStream_t)stream;
    const int blocks = (n + kNoAllocSlice - 1) / kNoAllocSlice;
    cudaError_t e = g4_launch(k_topk_pass<kNoAllocSlice>, dim3(blocks), dim3(kTopkThreads), 0, st, false, logits,
                              (const int *)nullptr, n, k, s.v, s.i);
    if (e == cudaSuccess)
        e = g4_launch(k_topk_pass<kTopkSlice>, dim3(1), dim3(kTopkThreads), 0, st, false, (const float *)s.v,
                      (const int *)s.i, blocks * k, k, values, ids);
    return e == cudaSuccess ? G4_OK : G4_ERR_CUDA;
}

int g4k_quantize(const float *x, int rows, int width, int8_t *q, float *s) {
    if (!x || !q || !s || rows < 1 || width < 64 || width % 64) return G4_ERR_INVALID;
    DevBuf dx, dq, ds;
    TK(dx.alloc((size_t)rows * width * 4));
    TK(dq.alloc((size_t)rows * width));
    TK(ds.alloc((size_t)rows * width / 64 * 4));
    TK(cudaMemcpy(dx.p, x, (size_t)rows * width * 4, cudaMemcpyHostToDevice));
    TK(g4_launch_rows_quant((const float *)dx.p, width, rows, width, (int8_t *)dq.p, (float *)ds.p, 0, false));
    TK(cudaMemcpy(q, dq.p, (size_t)rows * width, cudaMemcpyDeviceToHost));
    TK(cudaMemcpy(s, ds.p, (size_t)rows * width / 64 * 4, cudaMemcpyDeviceToHost));
    return G4_OK;
}

int g4k_rmsnorm_quant(const float *x, int rows, const float *w, float eps, float *y, int8_t *q, float *s) {
    if (!x || !w || !q || !s || rows < 1) return G4_ERR_INVALID;
    const int W = G4_HIDDEN;
    DevBuf dx, dw, dy, dq, ds;
    TK(dx.alloc((size_t)rows * W * 4));
    TK(dw.alloc((size_t)W * 4));
    TK(dy.alloc((size_t)rows * W * 4));
    TK(dq.alloc((size_t)rows * W));
    TK(ds.alloc((size_t)rows * W / 64 * 4));
    TK(cudaMemcpy(dx.p, x, (size_t)rows * W * 4, cudaMemcpyHostToDevice));
    TK(cudaMemcpy(dw.p, w, (size_t)W * 4, cudaMemcpyHostToDevice));
    TK(g4_launch_rows_norm(0, (const float *)dx.p, rows, nullptr, nullptr, nullptr, nullptr, (const float *)dw.p, eps,
                           (int8_t *)dq.p, (float *)ds.p, 0, false, (float *)dy.p));
    if (y) TK(cudaMemcpy(y, dy.p, (size_t)rows * W * 4, cudaMemcpyDeviceToHost));
    TK(cudaMemcpy(q, dq.p, (size_t)rows * W, cudaMemcpyDeviceToHost));
    TK(cudaMemcpy(s, ds.p, (size_t)rows * W / 64 * 4, cudaMemcpyDeviceToHost));
    return G4_OK;
}

int g4k_linear(const int8_t *w_packed, const uint16_t *s_packed, int N, int K, const int8_t *xq, const float *xs,
               int T, int path, float *out, int32_t *dots) {
    if (!w_packed || !s_packed || !xq || !xs || !out || N < 16 || N % 16 || K < 256 || K % 256 || T < 1 ||
        T > (path == 3 ? G4_GEMM_MAX_T : G4_BATCH))
        return G4_ERR_INVALID;
    if (path == 0) path = T <= 4 ? 1 : 2;
    if (path == 1 && T > 4) return G4_ERR_INVALID;
    const int G = K / 64;
    DevBuf pw, ps, w, s, dxq, dxs, dout, ddots, derr, dticket;
    TK(pw.alloc((size_t)N * K));
    TK(ps.alloc((size_t)N * G * 2));
    TK(w.alloc((size_t)N * K));
    TK(s.alloc((size_t)N * G * 2));
    TK(dxq.alloc((size_t)T * K));
    TK(dxs.alloc((size_t)T * G * 4));
    TK(dout.alloc((size_t)T * N * 4));
    TK(derr.alloc(64));
    TK(cudaMemset(derr.p, 0, 64));
    if (dots) TK(ddots.alloc((size_t)T * N * G * 4));
    TK(cudaMemcpy(pw.p, w_packed, (size_t)N * K, cudaMemcpyHostToDevice));
    TK(cudaMemcpy(ps.p, s_packed, (size_t)N * G * 2, cudaMemcpyHostToDevice));
    TK(cudaMemcpy(dxq.p, xq, (size_t)T * K, cudaMemcpyHostToDevice));
    TK(cudaMemcpy(dxs.p, xs, (size_t)T * G * 4, cudaMemcpyHostToDevice));
    TK(g4_launch_repack((const int8_t *)pw.p, (const uint16_t *)ps.p, N, K, (int8_t *)w.p, (uint16_t *)s.p, 0, 1, 0));
    DMat m{(const int8_t *)w.p, (const uint16_t *)s.p, nullptr, N, K};
    DevBuf sT, xsT;
    // group-major activation scales: the engine's 512-row stride, or T rounded up
    // to whole 128-row tiles for the longer tensor-core problems
    const int xs_stride = T <= G4_XST_STRIDE ? G4_XST_STRIDE : (T + 127) / 128 * 128;
    if (path == 3 || path == 4) {
        TK(sT.alloc((size_t)N * G * 4));
        TK(g4_launch_scales_t(m.s, N, K, (float *)sT.p, 0));
        m.sT = (const float *)sT.p;
        std::vector<float> h((size_t)G * xs_stride, 0.0f);
        for (int t = 0; t < T; t++)
            for (int g = 0; g < G; g++) h[(size_t)g * xs_stride + t] = xs[(size_t)t * G + g];
        TK(xsT.alloc(h.size() * 4));
        TK(cudaMemcpy(xsT.p, h.data(), h.size() * 4, cudaMemcpyHostToDevice));
    }
    if (path == 1) {
        GemvArgs a{};
        a.m = m;
        a.T = T;
        a.xq_in = (const int8_t *)dxq.p;
        a.xs_in = (const float *)dxs.p;
        a.out = (float *)dout.p;
        a.out_stride = N;
        a.dots_out = (int32_t *)ddots.p;
        a.err = (int *)derr.p;
        a.eps = G4_RMS_EPS;
        const int grid = N / 2 < num_sms() ? N / 2 : num_sms();
        g4_gemv_plan(a, grid);
        TK(g4_launch_gemv(a, PRO_LOADQ, EPI_STORE, grid, 0, false));
    } else {
        GemmArgs a{};
        a.m = m;
        a.T = T;
        a.xq = (const int8_t *)dxq.p;
        a.xs = (const float *)dxs.p;
        a.xsT = (const float *)xsT.p;
        a.xs_stride = xs_stride;
        a.epi = EPI_STORE;
        a.out = (float *)dout.p;
        a.out_stride = N;
        a.dots_out = (int32_t *)ddots.p;
        a.err = (int *)derr.p;
        if (path == 3) {
            if (!g4_gemm_tc_supported(a)) return G4_ERR_INVALID;
            TK(g4_launch_gemm_tc(a, 0, false));
        } else if (path == 4) {
            if (!g4_gemm_skinny_supported(a)) return G4_ERR_INVALID;
            TK(g4_launch_gemm_skinny(a, 0, false));
        } else {
            TK(g4_launch_gemm_simt(a, 0, false));
        }
    }
    TK(cudaDeviceSynchronize());
    int err = 0;
    TK(cudaMemcpy(&err, derr.p, 4, cudaMemcpyDeviceToHost));
    if (err) return G4_ERR_DEVICE;
    TK(cudaMemcpy(out, dout.p, (size_t)T * N * 4, cudaMemcpyDeviceToHost));
    if (dots) TK(cudaMemcpy(dots, ddots.p, (size_t)T * N * G * 4, cudaMemcpyDeviceToHost));
    return G4_OK;
}

// One attention sub-layer over an FP32 KV ring (gemma4.c:411-461), through the
// same launchers the model uses; optionally timed. See g4cuda.h.
int g4k_attention(int hd, int ring, int T, int start_pos, int mode, int splits, const float *qkv,
                  const float *q_norm, const float *k_norm, const float *rope_cos, const float *rope_sin,
                  float *kring, float *vring, float *out, int8_t *xq, float *xs, int iters, float *ms_per_call) {
    if ((hd != 256 && hd != 512) || ring < 1024 || (ring & (ring - 1)) || T < 1 || T > G4_BATCH ||
        start_pos < 0 || mode < 0 || mode > 4 || !qkv || !rope_cos || !rope_sin || !kring || !vring || !out ||
        iters < 0 || (iters > 0 && !ms_per_call))
        return G4_ERR_INVALID;
    if ((mode == 2 || mode == 3) && (splits < 1 || splits > 256)) return G4_ERR_INVALID;
    if (mode == 2 && T != 1) return G4_ERR_INVALID;
    if ((xq || xs) && ((mode != 0 && mode != 4) || !xq || !xs)) return G4_ERR_INVALID;
    const int window = hd == 256 ? G4_SLIDING_WINDOW : 0;
    const int pairs = hd == 256 ? 128 : 64;
    const int npos = start_pos + T;
    // every key a query sees must still be in the ring
    if ((window ? (T - 1 + window) : npos) > ring) return G4_ERR_INVALID;
    const int stride = 10 * hd;
    const int sms = num_sms();
    DevBuf dqkv, dqn, dkn, dcos, dsin, dk, dv, dout, dpart, dpre, dscores, derr, drs, drp, dxq, dxs, dws;
    TK(dqkv.alloc((size_t)T * stride * 4));
    TK(dqn.alloc((size_t)hd * 4));
    TK(dkn.alloc((size_t)hd * 4));
    TK(dcos.alloc((size_t)npos * pairs * 4));
    TK(dsin.alloc((size_t)npos * pairs * 4));
    TK(dk.alloc((size_t)ring * hd * 4));
    TK(dv.alloc((size_t)ring * hd * 4));
    TK(dout.alloc((size_t)T * 8 * hd * 4));
    TK(dpart.alloc((size_t)(mode == 3 ? T : 1) * (splits > 0 ? splits : 1) * 8 * (hd + 4) * 4));
    TK(dpre.alloc((size_t)2 * sms * G4_PRE_PART_SLOT * 4));
    if (mode == 1) TK(dscores.alloc((size_t)T * 8 * npos * 4));
    TK(derr.alloc(64));
    TK(cudaMemset(derr.p, 0, 64));
    std::vector<float> ones(hd, 1.0f);
    TK(cudaMemcpy(dqkv.p, qkv, (size_t)T * stride * 4, cudaMemcpyHostToDevice));
    TK(cudaMemcpy(dqn.p, q_norm ? q_norm : ones.data(), (size_t)hd * 4, cudaMemcpyHostToDevice));
    TK(cudaMemcpy(dkn.p, k_norm ? k_norm : ones.data(), (size_t)hd * 4, cudaMemcpyHostToDevice));
    TK(cudaMemcpy(dcos.p, rope_cos, (size_t)npos * pairs * 4, cudaMemcpyHostToDevice));
    TK(cudaMemcpy(dsin.p, rope_sin, (size_t)npos * pairs * 4, cudaMemcpyHostToDevice));
    TK(cudaMemcpy(dk.p, kring, (size_t)ring * hd * 4, cudaMemcpyHostToDevice));
    TK(cudaMemcpy(dv.p, vring, (size_t)ring * hd * 4, cudaMemcpyHostToDevice));
    AttnArgs a{};
    a.hd = hd;
    a.pairs = pairs;
    a.window = window;
    a.mask = ring - 1;
    a.T = T;
    a.start_pos = start_pos;
    a.qkv = (float *)dqkv.p;
    a.qkv_stride = stride;
    a.has_kv = 1;
    a.q_norm = (const float *)dqn.p;
    a.k_norm = (const float *)dkn.p;
    a.rope_cos = (const float *)dcos.p;
    a.rope_sin = (const float *)dsin.p;
    a.kcache = (float *)dk.p;
    a.vcache = (float *)dv.p;
    a.part = (float *)dpart.p;
    a.out = (float *)dout.p;
    a.err = (int *)derr.p;
    a.strict = mode == 1;
    a.scores = (float *)dscores.p;
    a.score_stride = npos;
    a.pre_part = (float *)dpre.p;
    a.pre_ctas = sms;
    if (xq) {   // the tiled kernel's fused quantisation of its output rows
        TK(dxq.alloc((size_t)T * 8 * hd));
        TK(dxs.alloc((size_t)T * 8 * hd / 64 * 4));
        a.quant_out = 1;
        a.xq = (int8_t *)dxq.p;
        a.xs = (float *)dxs.p;
    }
    if (mode == 3) {
        std::vector<int> rs(T, 0), rp(T);
        for (int t = 0; t < T; t++) rp[t] = start_pos + t;
        TK(drs.alloc((size_t)T * 4));
        TK(drp.alloc((size_t)T * 4));
        TK(cudaMemcpy(drs.p, rs.data(), (size_t)T * 4, cudaMemcpyHostToDevice));
        TK(cudaMemcpy(drp.p, rp.data(), (size_t)T * 4, cudaMemcpyHostToDevice));
        a.row_seq = (const int *)drs.p;
        a.row_pos = (const int *)drp.p;
    }
    size_t ws_bytes = 0;
    if (mode == 4) {   // the tensor-core path's workspace
        ws_bytes = g4_attn_tc_ws_bytes(a);
        if (!ws_bytes) return G4_ERR_INVALID;
        TK(dws.alloc(ws_bytes));
    }
    // q/k/v post-processing (decode does its own inside the split kernel)
    if (mode != 2) TK(g4_launch_qkv_post(a, 0, false));
    auto attend = [&]() -> cudaError_t {
        switch (mode) {
        case 0: return g4_launch_attn_prefill(a, 0, false);
        case 1: return g4_launch_attn_strict(a, 0, false);
        case 4: return g4_launch_attn_tc(a, dws.p, ws_bytes, 0, false);
        case 2: {
            cudaError_t e = g4_launch_attn_decode(a, splits, 0, false);
            return e ? e : g4_launch_attn_combine(a, splits, 0, false);
        }
        default: return g4_launch_attn_rows(a, splits, 0, false);
        }
    };
    TK(attend());
    TK(cudaDeviceSynchronize());
    int err = 0;
    TK(cudaMemcpy(&err, derr.p, 4, cudaMemcpyDeviceToHost));
    if (err) return G4_ERR_DEVICE;
    TK(cudaMemcpy(out, dout.p, (size_t)T * 8 * hd * 4, cudaMemcpyDeviceToHost));
    if (xq) {
        TK(cudaMemcpy(xq, dxq.p, (size_t)T * 8 * hd, cudaMemcpyDeviceToHost));
        TK(cudaMemcpy(xs, dxs.p, (size_t)T * 8 * hd / 64 * 4, cudaMemcpyDeviceToHost));
    }
    TK(cudaMemcpy(kring, dk.p, (size_t)ring * hd * 4, cudaMemcpyDeviceToHost));
    TK(cudaMemcpy(vring, dv.p, (size_t)ring * hd * 4, cudaMemcpyDeviceToHost));
    if (iters > 0) {
        // the attention kernels are pure functions of the post-processed q and
        // the rings, so repeating them re-does the same work
        for (int i = 0; i < 3; i++) TK(attend());
        cudaEvent_t e0, e1;
        TK(cudaEventCreate(&e0));
        TK(cudaEventCreate(&e1));
        cudaEventRecord(e0, 0);
        for (int i = 0; i < iters; i++) attend();
        cudaEventRecord(e1, 0);
        cudaError_t e = cudaEventSynchronize(e1);
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, e0, e1);
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        TK(e);
        TK(cudaGetLastError());
        *ms_per_call = ms / iters;
    }
    return G4_OK;
}

// sample() (gemma4.c:536-561) on one logits row: top-64 + temperature draw on
// the device; *state is the xorshift state before the call and receives it after.
int g4k_sample(const float *logits, int n, float temperature, unsigned long long *state, int *token) {
    if (!logits || !state || !token || n < 64 || n > 64 * 4096) return G4_ERR_INVALID;
    DevBuf dl, pv, pi, tv, ti, dst, dtok;
    TK(dl.alloc((size_t)n * 4));
    TK(pv.alloc(4096 * 4));
    TK(pi.alloc(4096 * 4));
    TK(tv.alloc(64 * 4));
    TK(ti.alloc(64 * 4));
    TK(dst.alloc(8));
    TK(dtok.alloc(4));
    TK(cudaMemcpy(dl.p, logits, (size_t)n * 4, cudaMemcpyHostToDevice));
    TK(cudaMemcpy(dst.p, state, 8, cudaMemcpyHostToDevice));
    TK(g4_launch_topk((const float *)dl.p, n, 64, (float *)pv.p, (int *)pi.p, (float *)tv.p, (int *)ti.p, 0));
    TK(g4_launch_sample64((const float *)tv.p, (const int *)ti.p, temperature, (unsigned long long *)dst.p,
                          (int *)dtok.p, 0));
    TK(cudaMemcpy(token, dtok.p, 4, cudaMemcpyDeviceToHost));
    TK(cudaMemcpy(state, dst.p, 8, cudaMemcpyDeviceToHost));
    return G4_OK;
}

// Time the decode GEMV on an N x K matrix (random device-resident weights):
// `copies` distinct weight sets are cycled so the working set exceeds L2, and
// `iters` back-to-back launches are timed with CUDA events on one stream.
// Reports the average launch duration and the algorithmic bytes per launch
// (int8 weights + FP16 scales).
int g4_bench_gemv(int N, int K, int T, int iters, int pdl, float *ms_per_launch, double *bytes_per_launch) {
    if (N < 2 || N % 2 || K % 256 || T < 1 || T > 4 || iters < 1 || !ms_per_launch) return G4_ERR_INVALID;
    const int G = K / 64;
    const size_t wbytes = (size_t)N * K + (size_t)N * G * 2;
    int copies = (int)((512ull << 20) / wbytes) + 1;
    if (copies > 64) copies = 64;
    DevBuf w, xq, xs, out, err;
    TK(w.alloc(wbytes * copies));
    TK(xq.alloc((size_t)T * K));
    TK(xs.alloc((size_t)T * G * 4));
    TK(out.alloc((size_t)T * N * 4));
    TK(err.alloc(64));
    TK(cudaMemset(w.p, 1, wbytes * copies));
    TK(cudaMemset(xq.p, 1, (size_t)T * K));
    TK(cudaMemset(xs.p, 0, (size_t)T * G * 4));
    TK(cudaMemset(err.p, 0, 64));
    TK(cudaDeviceSynchronize());   // the memsets above must land before the timed stream reads the buffers
    cudaStream_t st;
    TK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    auto launch = [&](int i) {
        const uint8_t *base = (const uint8_t *)w.p + (size_t)(i % copies) * wbytes;
        GemvArgs a{};
        a.m = DMat{(const int8_t *)base, (const uint16_t *)(base + (size_t)N * K), nullptr, N, K};
        a.T = T;
        a.xq_in = (const int8_t *)xq.p;
        a.xs_in = (const float *)xs.p;
        a.out = (float *)out.p;
        a.out_stride = N;
        a.err = (int *)err.p;
        const int grid = N / 2 < num_sms() ? N / 2 : num_sms();
        g4_gemv_plan(a, grid);
        return g4_launch_gemv(a, PRO_LOADQ, EPI_STORE, grid, st, pdl != 0);
    };
    for (int i = 0; i < 3; i++) TK(launch(i));
    // the timed launches replay as one CUDA graph, so the host's launch cost
    // (tensor-map encoding included) stays out of the device time
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    TK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    cudaError_t le = cudaSuccess;
    for (int i = 0; i < iters && le == cudaSuccess; i++) le = launch(i);
    cudaError_t ce = cudaStreamEndCapture(st, &graph);
    if (le != cudaSuccess || ce != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        cudaStreamDestroy(st);
        return G4_ERR_CUDA;
    }
    ce = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ce != cudaSuccess) {
        cudaStreamDestroy(st);
        return G4_ERR_CUDA;
    }
    TK(cudaGraphLaunch(exec, st));
    TK(cudaStreamSynchronize(st));
    cudaEvent_t e0, e1;
    TK(cudaEventCreate(&e0));
    TK(cudaEventCreate(&e1));
    TK(cudaEventRecord(e0, st));
    TK(cudaGraphLaunch(exec, st));
    TK(cudaEventRecord(e1, st));
    TK(cudaEventSynchronize(e1));
    float ms = 0;
    TK(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaGraphExecDestroy(exec);
    cudaStreamDestroy(st);
    int derr = 0;
    TK(cudaMemcpy(&derr, err.p, 4, cudaMemcpyDeviceToHost));
    if (derr) {
        fprintf(stderr, "g4_bench_gemv: device error %d stage %d block %d\n", derr & 0xff, (derr >> 8) & 0xfff,
                (unsigned)derr >> 20);
        return G4_ERR_DEVICE;
    }
    *ms_per_launch = ms / iters;
    if (bytes_per_launch) *bytes_per_launch = (double)wbytes;
    return G4_OK;
}

// Measured int8 tensor peak: k_mma_peak timed with CUDA events after one warm-up
// launch; TOP/s = ops / time.
int g4_bench_mma_i8(int iters, float *ms_per_launch, double *ops_per_launch) {
    if (iters < 1 || iters > (1 << 24) || !ms_per_launch) return G4_ERR_INVALID;
    DevBuf err;
    TK(err.alloc(64));
    TK(cudaMemset(err.p, 0, 64));
    double ops = 0;
    TK(g4_launch_mma_peak(iters, (int *)err.p, 0, &ops));
    TK(cudaDeviceSynchronize());
    cudaEvent_t e0, e1;
    TK(cudaEventCreate(&e0));
    TK(cudaEventCreate(&e1));
    TK(cudaEventRecord(e0, 0));
    TK(g4_launch_mma_peak(iters, (int *)err.p, 0, &ops));
    TK(cudaEventRecord(e1, 0));
    TK(cudaEventSynchronize(e1));
    float ms = 0;
    TK(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    int derr = 0;
    TK(cudaMemcpy(&derr, err.p, 4, cudaMemcpyDeviceToHost));
    if (derr) return G4_ERR_DEVICE;
    *ms_per_launch = ms;
    if (ops_per_launch) *ops_per_launch = ops;
    return G4_OK;
}

// Time the prefill GEMM (path 2 SIMT dp4a, 3 tcgen05, 4 small-batch mma) on a T x N x K problem
// with device-resident weights cycled over enough copies to exceed L2, and
// report the average launch duration and the int8 operations per launch
// (2 T N K).
int g4_bench_gemm(int N, int K, int T, int path, int iters, float *ms_per_launch, double *ops_per_launch) {
    if (N < 128 || N % 128 || K % 256 || T < 1 || T > (path == 3 ? G4_GEMM_MAX_T : G4_BATCH) || iters < 1 ||
        !ms_per_launch || path < 2 || path > 4 || (path == 4 && T > G4_SKINNY_MAX_T))
        return G4_ERR_INVALID;
    const int G = K / 64;
    const int xs_stride = T <= G4_XST_STRIDE ? G4_XST_STRIDE : (T + 127) / 128 * 128;
    const size_t wbytes = (size_t)N * K + (size_t)N * G * 2;
    const size_t tbytes = (size_t)N * G * 4;
    int copies = (int)((512ull << 20) / wbytes) + 1;
    if (copies > 16) copies = 16;
    DevBuf w, sT, xq, xs, xsT, out, err;
    TK(w.alloc(wbytes * copies));
    TK(sT.alloc(tbytes));
    TK(xsT.alloc((size_t)G * xs_stride * 4));
    TK(cudaMemset(xsT.p, 0, (size_t)G * xs_stride * 4));
    TK(xq.alloc((size_t)T * K));
    TK(xs.alloc((size_t)T * G * 4));
    TK(out.alloc((size_t)T * N * 4));
    TK(err.alloc(64));
    TK(cudaMemset(w.p, 1, wbytes * copies));
    TK(cudaMemset(sT.p, 0, tbytes));
    TK(cudaMemset(xq.p, 1, (size_t)T * K));
    TK(cudaMemset(xs.p, 0, (size_t)T * G * 4));
    TK(cudaMemset(err.p, 0, 64));
    TK(cudaDeviceSynchronize());
    cudaStream_t st;
    TK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    auto launch = [&](int i) {
        const uint8_t *base = (const uint8_t *)w.p + (size_t)(i % copies) * wbytes;
        GemmArgs a{};
        a.m = DMat{(const int8_t *)base, (const uint16_t *)(base + (size_t)N * K), (const float *)sT.p, N, K};
        a.T = T;
        a.xq = (const int8_t *)xq.p;
        a.xs = (const float *)xs.p;
        a.xsT = (const float *)xsT.p;
        a.xs_stride = xs_stride;
        a.epi = EPI_STORE;
        a.out = (float *)out.p;
        a.out_stride = N;
        a.err = (int *)err.p;
        return path == 4   ? g4_launch_gemm_skinny(a, st, false)
               : path == 3 ? g4_launch_gemm_tc(a, st, false)
                           : g4_launch_gemm_simt(a, st, false);
    };
    for (int i = 0; i < 3; i++) TK(launch(i));
    // the timed launches replay as one CUDA graph, so the host's launch cost
    // (tensor-map encoding included) stays out of the device time
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    TK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    cudaError_t le = cudaSuccess;
    for (int i = 0; i < iters && le == cudaSuccess; i++) le = launch(i);
    cudaError_t ce = cudaStreamEndCapture(st, &graph);
    if (le != cudaSuccess || ce != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        cudaStreamDestroy(st);
        return G4_ERR_CUDA;
    }
    ce = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ce != cudaSuccess) {
        cudaStreamDestroy(st);
        return G4_ERR_CUDA;
    }
    TK(cudaGraphLaunch(exec, st));
    TK(cudaStreamSynchronize(st));
    cudaEvent_t e0, e1;
    TK(cudaEventCreate(&e0));
    TK(cudaEventCreate(&e1));
    TK(cudaEventRecord(e0, st));
    TK(cudaGraphLaunch(exec, st));
    TK(cudaEventRecord(e1, st));
    TK(cudaEventSynchronize(e1));
    float ms = 0;
    TK(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaGraphExecDestroy(exec);
    cudaStreamDestroy(st);
    int derr = 0;
    TK(cudaMemcpy(&derr, err.p, 4, cudaMemcpyDeviceToHost));
    if (derr) return G4_ERR_DEVICE;
    *ms_per_launch = ms / iters;
    if (ops_per_launch) *ops_per_launch = 2.0 * T * (double)N * K;
    return G4_OK;
}

}  // extern "C"
