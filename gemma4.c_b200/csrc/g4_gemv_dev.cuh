// g4_gemv_dev.cuh — device building blocks of the int8 GEMV consumers, shared
// by the standalone decode GEMV (g4_gemv.cu) and the persistent decode kernel
// (g4_decode.cu).
//
// Reference: quantize (gemma4.c:265-279), rmsnorm (:360-373), add_and_scale
// (:375-378), embedding (:337-358), matmul_int8 (:192-262), geglu (:310-331),
// logits soft-cap (:519) and greedy argmax (:537-541).
#pragma once
#include "g4_common.cuh"
#include "g4_internal.h"

namespace {

constexpr int kWarps = 8;                   // consumer warps
constexpr int kConsumers = kWarps * 32;

// rows per weight stage: whole rows, an even number, ~16 KB
__host__ __device__ inline int stage_rows(int K) {
    int r = (16384 / K) & ~1;
    return r < 2 ? 2 : r;
}

G4_DEV void csync() { bar_sync(1, kConsumers); }   // consumer-only barrier

// Sum over the consumer threads; every consumer gets the result.
__device__ float block_sum(float v, float *red) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    v = warp_sum(v);
    if (lane == 0) red[warp] = v;
    csync();
    float r = 0.0f;
#pragma unroll
    for (int i = 0; i < kWarps; i++) r += red[i];
    csync();
    return r;
}

// block_sum without the trailing barrier: `red` (8 floats) must not be
// written again before the caller's next consumer barrier.
__device__ float block_sum_once(float v, float *red) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    v = warp_sum(v);
    if (lane == 0) red[warp] = v;
    csync();
    float r = 0.0f;
#pragma unroll
    for (int i = 0; i < kWarps; i++) r += red[i];
    return r;
}

// Sum of squares of the hidden row whose values this thread holds at
// e = tid + i * kConsumers: in parallel, or (strict) sequentially in index
// order through shared memory exactly as gemma4.c:367-368 does. `slot` picks
// one of two reduction buffers so that two sums in a row need no barrier in
// between (the caller's next barrier frees both).
template <int PER>
__device__ float row_sumsq(const float (&v)[PER], bool strict, float *vec, float *red, int slot) {
    const int tid = threadIdx.x;
    if (!strict) {
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < PER; i++) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
        return block_sum_once(ss, red + 16 + 8 * slot);
    }
#pragma unroll
    for (int i = 0; i < PER; i++) vec[tid + i * kConsumers] = v[i];
    csync();
    if (tid == 0) red[0] = seq_sumsq(vec, PER * kConsumers);
    csync();
    const float ss = red[0];
    csync();
    return ss;
}

// Quantise `src` (K floats, shared or global; 16-byte aligned) into xq/xs
// (gemma4.c:265-279). All consumer threads work: thread t takes the float4s at
// t + 256 j, so each 64-value group is one half-warp's 16 float4s; the group
// maximum is a 4-step shuffle reduction (exact in any order). Loads are issued
// U float4s ahead, so a global source costs ceil(K / (4 * 256 * U)) round trips:
// one for every row width of the model (K <= 12288).
__device__ __noinline__ void quantize_row(const float *src, int K, int8_t *xq, float *xs) {
    constexpr int U = 12;
    const int tid = threadIdx.x, n4 = K >> 2;   // K % 128 == 0: a warp is all in or all out
    const float4 *s4 = (const float4 *)src;
    for (int i0 = tid; i0 < n4; i0 += kConsumers * U) {
        float4 v[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int i = i0 + u * kConsumers;
            v[u] = i < n4 ? s4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int i = i0 + u * kConsumers;
            if (i - (tid & 31) >= n4) break;   // warp-uniform
            float m = fmaxf(fmaxf(fabsf(v[u].x), fabsf(v[u].y)), fmaxf(fabsf(v[u].z), fabsf(v[u].w)));
#pragma unroll
            for (int o = 1; o < 16; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            const float sc = quant_scale(m), inv = quant_inv(sc);
            const uint32_t q = (uint32_t)(quant_one(v[u].x, inv) & 0xff) | ((uint32_t)(quant_one(v[u].y, inv) & 0xff) << 8) |
                               ((uint32_t)(quant_one(v[u].z, inv) & 0xff) << 16) |
                               ((uint32_t)(quant_one(v[u].w, inv) & 0xff) << 24);
            ((uint32_t *)xq)[i] = q;
            if ((tid & 15) == 0) xs[i >> 4] = sc;
        }
    }
}

template <int T, int PRO>
__device__ void prologue(const GemvArgs &a, int8_t *xq, float *xs, float *vec, float *red) {
    const int K = a.m.K, G = K / 64, tid = threadIdx.x;
    if (PRO == PRO_LOADQ) {
        const int4 *q4 = (const int4 *)a.xq_in;
        int4 *d4 = (int4 *)xq;
        for (int i = tid; i < T * K / 16; i += kConsumers) d4[i] = q4[i];
        for (int i = tid; i < T * G; i += kConsumers) xs[i] = a.xs_in[i];
        return;
    }
    if (PRO == PRO_QUANT) {
        for (int t = 0; t < T; t++) quantize_row(a.src + (size_t)t * a.src_stride, K, xq + t * K, xs + t * G);
        return;
    }
    // K == 1536 (hidden width) for all fused-norm prologues; 6 values per thread.
    // The norm weights and the scalar do not depend on earlier work: load them
    // first, and each token row together with its residual row, so that the
    // prologue waits for one memory round trip per row rather than five.
    constexpr int PER = G4_HIDDEN / kConsumers;
    constexpr bool kRes = PRO == PRO_RES_NORM_QUANT || PRO == PRO_RES_QUANT;
    constexpr bool kPre = PRO == PRO_NORM_QUANT || PRO == PRO_RES_NORM_QUANT;
    float wpost[PER], wpre[PER];
    float sc = 1.0f;
#pragma unroll
    for (int i = 0; i < PER; i++) {
        wpost[i] = kRes ? a.w_post[tid + i * kConsumers] : 0.0f;
        wpre[i] = kPre ? a.w_pre[tid + i * kConsumers] : 0.0f;
    }
    if (kRes && a.scalar) sc = *a.scalar;
    for (int t = 0; t < T; t++) {
        float y[PER];
        if (PRO == PRO_EMBED_QUANT) {
            int tok = a.tokens[t];
            if (tok < 0 || tok >= a.embed.N) {
                g4_set_error(a.err, G4D_BAD_TOKEN);
                tok = 0;
            }
            const int8_t *wr = a.embed.w + (size_t)tok * G4_HIDDEN;
            const uint16_t *sr = a.embed.s + (size_t)tok * (G4_HIDDEN / 64);
#pragma unroll
            for (int i = 0; i < PER; i++) {
                const int e = tid + i * kConsumers;
                const float sc = __fmul_rn(h2f(sr[e >> 6]), a.embed_mult);   // gemma4.c:350
                y[i] = __fmul_rn((float)wr[e], sc);                          // gemma4.c:354
                if (blockIdx.x == 0) a.res_out[t * G4_HIDDEN + e] = y[i];
            }
            // this CTA's slice of the per-layer embedding row (x16)
            const int W = a.embed_ple.K;
            const int per = (W + gridDim.x - 1) / gridDim.x;
            const int e0 = blockIdx.x * per, e1 = min(W, e0 + per);
            const int8_t *pw = a.embed_ple.w + (size_t)tok * W;
            const uint16_t *ps = a.embed_ple.s + (size_t)tok * (W / 64);
            for (int e = e0 + tid; e < e1; e += kConsumers)
                a.ple_emb[(size_t)t * W + e] = __fmul_rn((float)pw[e], __fmul_rn(h2f(ps[e >> 6]), a.ple_mult));
        } else {
            const float *h = a.src + (size_t)t * a.src_stride;
            float hv[PER], rv[PER];
#pragma unroll
            for (int i = 0; i < PER; i++) {
                hv[i] = h[tid + i * kConsumers];
                rv[i] = kRes ? a.res_in[t * G4_HIDDEN + tid + i * kConsumers] : 0.0f;
            }
            const float ss = row_sumsq<PER>(hv, a.strict, vec, red, 0);
            const float inv = rms_inv(ss, (float)G4_HIDDEN, a.eps);
            if (PRO == PRO_NORM_QUANT) {
#pragma unroll
                for (int i = 0; i < PER; i++) y[i] = rms_apply(hv[i], inv, wpre[i]);
            } else {
                // residual update: r' = (r + rmsnorm(h, w_post)) * scalar (gemma4.c:485-486,496-497,505-506)
#pragma unroll
                for (int i = 0; i < PER; i++) {
                    const int e = tid + i * kConsumers;
                    float r = __fadd_rn(rv[i], rms_apply(hv[i], inv, wpost[i]));
                    if (a.scalar) r = __fmul_rn(r, sc);
                    y[i] = r;
                    if (blockIdx.x == 0) a.res_out[t * G4_HIDDEN + e] = r;
                }
                if (PRO == PRO_RES_NORM_QUANT) {
                    const float ss2 = row_sumsq<PER>(y, a.strict, vec, red, 1);
                    const float inv2 = rms_inv(ss2, (float)G4_HIDDEN, a.eps);
#pragma unroll
                    for (int i = 0; i < PER; i++) y[i] = rms_apply(y[i], inv2, wpre[i]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < PER; i++) vec[tid + i * kConsumers] = y[i];
        csync();
        quantize_row(vec, G4_HIDDEN, xq + t * K, xs + t * G);
        csync();
    }
}

template <int EPI>
__device__ __forceinline__ void epilogue_row(const GemvArgs &a, int t, int n, float v, float up, bool writer,
                                             float &best_v, int &best_i) {
    if (EPI == EPI_STORE) {
        if (writer) a.out[(size_t)t * a.out_stride + n] = v;
    } else if (EPI == EPI_GEGLU_PAIR) {
        if (writer && (n & 1) == 0)
            a.out[(size_t)t * a.out_stride + (n >> 1)] = geglu_one(v, up, a.gelu, 4096, -8.0f, 8.0f, 4095.0f / 16.0f);
    } else if (EPI == EPI_PLE) {
        if (writer)
            a.out[(size_t)t * a.out_stride + n] =
                geglu_one(v, a.ple_u[(size_t)t * a.u_stride + n], a.gelu, 4096, -8.0f, 8.0f, 4095.0f / 16.0f);
    } else if (EPI == EPI_LOGITS) {
        const float sv = __fmul_rn(30.0f, tanhf(__fdiv_rn(v, 30.0f)));   // gemma4.c:519
        if (writer) a.out[(size_t)t * a.out_stride + n] = sv;
        if (sv > best_v) { best_v = sv; best_i = n; }
    }
}

// Exact int32 group dots and the ordered fp32 chain of one row pair held in
// shared memory: lanes 0-15 take row A (wrow points at A + q*16 for them), lanes
// 16-31 row B; 256 bytes per row per step, four 64-groups per step.
template <int T>
G4_DEV void pair_dot(const uint8_t *wrow, const uint16_t *srow, const int8_t *xq, const float *xs, int K, float (&acc)[T],
                     int32_t *dots_row, size_t dots_t_stride) {
    const int lane = threadIdx.x & 31, q = lane & 15, G = K >> 6, NC = K >> 8;
#pragma unroll
    for (int t = 0; t < T; t++) acc[t] = 0.0f;
#pragma unroll 2
    for (int step = 0; step < NC; step++) {
        const uint4 w4 = *(const uint4 *)(wrow + step * 256);
        const uint2 s2 = *(const uint2 *)(srow + step * 4);
        const float ws0 = h2f((uint16_t)(s2.x & 0xFFFFu)), ws1 = h2f((uint16_t)(s2.x >> 16));
        const float ws2 = h2f((uint16_t)(s2.y & 0xFFFFu)), ws3 = h2f((uint16_t)(s2.y >> 16));
#pragma unroll
        for (int t = 0; t < T; t++) {
            const int4 x4 = *(const int4 *)(xq + t * K + step * 256 + q * 16);
            int d = dp4a(w4.x, (uint32_t)x4.x, 0);
            d = dp4a(w4.y, (uint32_t)x4.y, d);
            d = dp4a(w4.z, (uint32_t)x4.z, d);
            d = dp4a(w4.w, (uint32_t)x4.w, d);
            d += __shfl_xor_sync(0xffffffffu, d, 1);
            d += __shfl_xor_sync(0xffffffffu, d, 2);
            const int base = lane & 16;
            const int d0 = __shfl_sync(0xffffffffu, d, base);
            const int d1 = __shfl_sync(0xffffffffu, d, base + 4);
            const int d2 = __shfl_sync(0xffffffffu, d, base + 8);
            const int d3 = __shfl_sync(0xffffffffu, d, base + 12);
            const float4 xs4 = *(const float4 *)(xs + t * G + step * 4);
            float v = acc[t];
            v = __fmaf_rn(__int2float_rn(d0), __fmul_rn(ws0, xs4.x), v);
            v = __fmaf_rn(__int2float_rn(d1), __fmul_rn(ws1, xs4.y), v);
            v = __fmaf_rn(__int2float_rn(d2), __fmul_rn(ws2, xs4.z), v);
            v = __fmaf_rn(__int2float_rn(d3), __fmul_rn(ws3, xs4.w), v);
            acc[t] = v;
            if (dots_row && q == 0) {
                int32_t *dd = dots_row + (size_t)t * dots_t_stride + step * 4;
                dd[0] = d0; dd[1] = d1; dd[2] = d2; dd[3] = d3;
            }
        }
    }
}

}  // namespace
