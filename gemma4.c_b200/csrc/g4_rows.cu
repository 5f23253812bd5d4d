// g4_rows.cu — per-row kernels of the prefill path and the load-time repack.
//
// Reference functions restated here: quantize (gemma4.c:265-279), rmsnorm
// (:360-373), add_and_scale (:375-378), embedding (:337-358) and the
// per-layer-input preparation in forward (:469-477). The decode path runs the
// same arithmetic inside the GEMV prologues (g4_gemv.cu).
#include "g4_common.cuh"
#include "g4_internal.h"

namespace {

// Packed [N/16][G][16 chunks][16 rows][4 B] -> row-major W[N][K]; scales
// [N/16][G][16] -> S[N][G] (exporter.py:304-316). Destination row of source
// row n is row_offset + n * row_mul (row_mul 2 interleaves gate/up).
__global__ void k_repack_w(const uint32_t *__restrict__ src, int N, int K, int8_t *__restrict__ dst, int row_offset,
                           int row_mul) {
    const int G = K / 64;
    const size_t words = (size_t)N * K / 4;
    for (size_t wi = blockIdx.x * (size_t)blockDim.x + threadIdx.x; wi < words; wi += (size_t)gridDim.x * blockDim.x) {
        const size_t per_block = (size_t)G * 256;
        const size_t rb = wi / per_block, rem = wi - rb * per_block;
        const int g = (int)(rem >> 8), c = (int)((rem >> 4) & 15), r = (int)(rem & 15);
        const size_t n = rb * 16 + r;
        const size_t drow = (size_t)row_offset + n * row_mul;
        *(uint32_t *)(dst + drow * K + g * 64 + c * 4) = src[wi];
    }
}

__global__ void k_repack_s(const uint16_t *__restrict__ src, int N, int K, uint16_t *__restrict__ dst, int row_offset,
                           int row_mul) {
    const int G = K / 64;
    const size_t count = (size_t)N * G;
    for (size_t si = blockIdx.x * (size_t)blockDim.x + threadIdx.x; si < count; si += (size_t)gridDim.x * blockDim.x) {
        const size_t rb = si / ((size_t)G * 16);
        const int g = (int)((si / 16) % G), r = (int)(si & 15);
        const size_t n = rb * 16 + r;
        dst[((size_t)row_offset + n * row_mul) * G + g] = src[si];
    }
}

// Every matrix of one staging fill in one launch: CTAs walk the jobs in order,
// each job's words and scales grid-stride (the per-element mapping of
// k_repack_w / k_repack_s above).
__global__ void __launch_bounds__(256) k_repack_jobs(const RepackJob *__restrict__ jobs, int njobs) {
    const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x, nthr = (size_t)gridDim.x * blockDim.x;
    for (int j = 0; j < njobs; j++) {
        const RepackJob J = jobs[j];
        const int G = J.K / 64;
        const size_t words = (size_t)J.N * J.K / 4, per_block = (size_t)G * 256;
        const uint32_t *src = (const uint32_t *)J.src_w;
        for (size_t wi = tid; wi < words; wi += nthr) {
            const size_t rb = wi / per_block, rem = wi - rb * per_block;
            const int g = (int)(rem >> 8), c = (int)((rem >> 4) & 15), r = (int)(rem & 15);
            const size_t drow = (size_t)J.row_offset + (rb * 16 + r) * J.row_mul;
            *(uint32_t *)(J.dst_w + drow * J.K + g * 64 + c * 4) = src[wi];
        }
        const size_t count = (size_t)J.N * G;
        for (size_t si = tid; si < count; si += nthr) {
            const size_t rb = si / ((size_t)G * 16);
            const int g = (int)((si / 16) % G), r = (int)(si & 15);
            J.dst_s[((size_t)J.row_offset + (rb * 16 + r) * J.row_mul) * G + g] = J.src_s[si];
        }
    }
}

// Group-major fp32 scales of many matrices in one launch (k_scales_t per job).
__global__ void __launch_bounds__(256) k_scales_t_jobs(const ScalesJob *__restrict__ jobs, int njobs) {
    const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x, nthr = (size_t)gridDim.x * blockDim.x;
    for (int j = 0; j < njobs; j++) {
        const ScalesJob J = jobs[j];
        const size_t n = (size_t)J.N * J.G;
        for (size_t i = tid; i < n; i += nthr) {
            const int g = (int)(i / J.N), r = (int)(i % J.N);
            J.sT[i] = h2f(J.s[(size_t)r * J.G + g]);
        }
    }
}

__device__ float block_sum256(float v, float *red) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    v = warp_sum(v);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float r = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) r += red[i];
    __syncthreads();
    return r;
}

// Sum of squares of a row held as v[i] at index tid + 256*i: block tree, or
// (strict) one thread in index order through `buf` as gemma4.c:367-368 does.
template <int PER>
__device__ float sumsq_row(const float (&v)[PER], int strict, float *buf, float *red) {
    const int tid = threadIdx.x;
    if (!strict) {
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < PER; i++) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
        return block_sum256(ss, red);
    }
#pragma unroll
    for (int i = 0; i < PER; i++) buf[tid + 256 * i] = v[i];
    __syncthreads();
    if (tid == 0) red[0] = seq_sumsq(buf, PER * 256);
    __syncthreads();
    const float ss = red[0];
    __syncthreads();
    return ss;
}

// One warp per 64-group: x -> (q, scale) exactly as gemma4.c:265-279.
__device__ void quant_group_warp(const float *src, int8_t *q, float *s, float *sT = nullptr) {
    const int lane = threadIdx.x & 31;
    const float a = src[lane], b = src[32 + lane];
    const float amax = warp_max(fmaxf(fabsf(a), fabsf(b)));
    const float sc = quant_scale(amax), inv = quant_inv(sc);
    q[lane] = (int8_t)quant_one(a, inv);
    q[32 + lane] = (int8_t)quant_one(b, inv);
    if (lane == 0) {
        *s = sc;
        if (sT) *sT = sc;   // group-major copy for the tensor-core GEMM
    }
}

// residual <- embed(token) * mult; ple_emb <- embed_per_layer(token) * ple_mult
__global__ void __launch_bounds__(256) k_rows_embed(const int *tokens, DMat e, DMat ep, float mult, float ple_mult,
                                                    float *res, float *ple_emb, int *err) {
    griddep_launch();
    griddep_wait();
    const int t = blockIdx.x;
    int tok = tokens[t];
    if (tok < 0 || tok >= e.N) {
        g4_set_error(err, G4D_BAD_TOKEN);
        tok = 0;
    }
    const int W = e.K, WP = ep.K;
    for (int i = threadIdx.x; i < W; i += 256)
        res[(size_t)t * W + i] = __fmul_rn((float)e.w[(size_t)tok * W + i],
                                           __fmul_rn(h2f(e.s[(size_t)tok * (W / 64) + (i >> 6)]), mult));
    for (int i = threadIdx.x; i < WP; i += 256)
        ple_emb[(size_t)t * WP + i] = __fmul_rn((float)ep.w[(size_t)tok * WP + i],
                                                __fmul_rn(h2f(ep.s[(size_t)tok * (WP / 64) + (i >> 6)]), ple_mult));
}

// grid (T, ceil(G/8)), 8 warps, one 64-group per warp
__global__ void __launch_bounds__(256) k_rows_quant(const float *src, int src_stride, int K, int8_t *xq, float *xs,
                                                    float *xsT) {
    griddep_launch();
    griddep_wait();
    const int t = blockIdx.x, g = blockIdx.y * 8 + (threadIdx.x >> 5), G = K / 64;
    if (g >= G) return;
    quant_group_warp(src + (size_t)t * src_stride + g * 64, xq + (size_t)t * K + g * 64, xs + (size_t)t * G + g,
                     xsT ? xsT + (size_t)g * G4_XST_STRIDE + t : nullptr);
}

// Hidden-width (1536) row ops, one CTA per token row.
//   mode 0: x = rmsnorm(src, w_pre)                              -> quantise
//   mode 1: r' = (res + rmsnorm(src, w_post)) * scalar; x = rmsnorm(r', w_pre) -> quantise
//   mode 2: r' = res + rmsnorm(src, w_post); x = r'              -> quantise
//   mode 3: r' = (res + rmsnorm(src, w_post)) * scalar           (no quantisation)
__global__ void __launch_bounds__(256) k_rows_norm(int mode, const float *src, const float *w_post,
                                                   const float *res_in, float *res_out, const float *scalar,
                                                   const float *w_pre, float eps, int8_t *xq, float *xs,
                                                   float *y_out, int strict, float *xsT) {
    __shared__ float red[8];
    __shared__ __align__(16) float y[G4_HIDDEN];
    griddep_launch();
    griddep_wait();
    constexpr int PER = G4_HIDDEN / 256;
    const int t = blockIdx.x, tid = threadIdx.x;
    const float *h = src + (size_t)t * G4_HIDDEN;
    // every global operand of the row is loaded up front (one round trip, not
    // one per reduction); the arithmetic below is unchanged
    float v[PER], rin[PER], wq[PER], wp[PER];
    const bool has_res = mode != 0, has_pre = mode == 0 || mode == 1;
#pragma unroll
    for (int i = 0; i < PER; i++) {
        const int e = tid + 256 * i;
        v[i] = h[e];
        rin[i] = has_res ? res_in[(size_t)t * G4_HIDDEN + e] : 0.0f;
        wq[i] = has_res ? w_post[e] : 0.0f;
        wp[i] = has_pre ? w_pre[e] : 0.0f;
    }
    const float sc = mode != 0 && scalar ? *scalar : 1.0f;
    const float ss = sumsq_row<PER>(v, strict, y, red);
    const float inv = rms_inv(ss, (float)G4_HIDDEN, eps);
    if (mode == 0) {
#pragma unroll
        for (int i = 0; i < PER; i++) v[i] = rms_apply(v[i], inv, wp[i]);
    } else {
#pragma unroll
        for (int i = 0; i < PER; i++) {
            const int e = tid + 256 * i;
            float r = __fadd_rn(rin[i], rms_apply(v[i], inv, wq[i]));
            if (scalar) r = __fmul_rn(r, sc);
            res_out[(size_t)t * G4_HIDDEN + e] = r;
            v[i] = r;
        }
        if (mode == 3) return;
        if (mode == 1) {
            const float ss2 = sumsq_row<PER>(v, strict, y, red);
            const float inv2 = rms_inv(ss2, (float)G4_HIDDEN, eps);
#pragma unroll
            for (int i = 0; i < PER; i++) v[i] = rms_apply(v[i], inv2, wp[i]);
        }
    }
#pragma unroll
    for (int i = 0; i < PER; i++) {
        y[tid + 256 * i] = v[i];
        if (y_out) y_out[(size_t)t * G4_HIDDEN + tid + 256 * i] = v[i];
    }
    __syncthreads();
    const int warp = tid >> 5;
    for (int g = warp; g < G4_HIDDEN / 64; g += 8)
        quant_group_warp(y + g * 64, xq + (size_t)t * G4_HIDDEN + g * 64, xs + (size_t)t * (G4_HIDDEN / 64) + g,
                         xsT ? xsT + (size_t)g * G4_XST_STRIDE + t : nullptr);
}

// u[t][l][:] = (rmsnorm(pli[t][l][:], w, eps) + ple_emb[t][l][:]) * scale   (gemma4.c:474-477)
__global__ void __launch_bounds__(256) k_ple_prep(const float *pli, const float *ple_emb, const float *w, float eps,
                                                  float scale, float *u, int strict) {
    __shared__ float red[8];
    __shared__ float buf[G4_PLE];
    griddep_launch();
    griddep_wait();
    const size_t base = ((size_t)blockIdx.x * G4_NUM_LAYERS + blockIdx.y) * G4_PLE;
    const int i = threadIdx.x;
    const float xv[1] = {pli[base + i]};
    const float x = xv[0];
    const float ss = sumsq_row<1>(xv, strict, buf, red);
    const float y = rms_apply(x, rms_inv(ss, (float)G4_PLE, eps), w[i]);
    u[base + i] = __fmul_rn(__fadd_rn(y, ple_emb[base + i]), scale);
}

// sT[g][n] = fp32(s[n][g]): group-major weight scales for the tensor-core GEMM.
__global__ void k_scales_t(const uint16_t *s, int N, int G, float *sT) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)N * G) return;
    const int g = (int)(i / N), n = (int)(i % N);
    sT[i] = h2f(s[(size_t)n * G + g]);
}

// Logit soft-cap in place and the first maximum of each row (gemma4.c:519,
// :537-541): one CTA per row.
__global__ void __launch_bounds__(1024) k_softcap_argmax(float *logits, int n, int *argmax) {
    __shared__ float bvs[32];
    __shared__ int bis[32];
    float *x = logits + (size_t)blockIdx.x * n;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = __fmul_rn(30.0f, tanhf(__fdiv_rn(x[i], 30.0f)));
        x[i] = v;
        if (v > bv) { bv = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) { bvs[w] = bv; bis[w] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < (int)(blockDim.x >> 5); k++)
            if (bvs[k] > bv || (bvs[k] == bv && bis[k] < bi)) { bv = bvs[k]; bi = bis[k]; }
        argmax[blockIdx.x] = bi;
    }
}

}  // namespace

cudaError_t g4_launch_softcap_argmax(float *logits, int rows, int n, int *argmax, cudaStream_t st) {
    if (rows < 1) return cudaErrorInvalidValue;
    k_softcap_argmax<<<rows, 1024, 0, st>>>(logits, n, argmax);
    return cudaGetLastError();
}

cudaError_t g4_launch_scales_t(const uint16_t *s, int N, int K, float *sT, cudaStream_t st) {
    const size_t n = (size_t)N * (K / 64);
    k_scales_t<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(s, N, K / 64, sT);
    return cudaGetLastError();
}

cudaError_t g4_launch_repack(const int8_t *packed_w, const uint16_t *packed_s, int N, int K, int8_t *w, uint16_t *s,
                             int row_offset, int row_mul, cudaStream_t st) {
    if (N % 16 || K % 64) return cudaErrorInvalidValue;
    k_repack_w<<<1184, 256, 0, st>>>((const uint32_t *)packed_w, N, K, w, row_offset, row_mul);
    k_repack_s<<<592, 256, 0, st>>>(packed_s, N, K, s, row_offset, row_mul);
    return cudaGetLastError();
}

cudaError_t g4_launch_repack_jobs(const RepackJob *jobs_dev, int njobs, cudaStream_t st) {
    if (njobs < 1) return cudaSuccess;
    k_repack_jobs<<<2 * g4_device_sms() * 4, 256, 0, st>>>(jobs_dev, njobs);
    return cudaGetLastError();
}

cudaError_t g4_launch_scales_t_jobs(const ScalesJob *jobs_dev, int njobs, cudaStream_t st) {
    if (njobs < 1) return cudaSuccess;
    k_scales_t_jobs<<<2 * g4_device_sms() * 4, 256, 0, st>>>(jobs_dev, njobs);
    return cudaGetLastError();
}

cudaError_t g4_launch_rows_embed(const int *tokens, int T, DMat embed, DMat embed_ple, float mult, float ple_mult,
                                 float *res, float *ple_emb, int *err, cudaStream_t st, bool pdl) {
    return g4_launch(k_rows_embed, dim3(T), dim3(256), 0, st, pdl, tokens, embed, embed_ple, mult, ple_mult, res,
                     ple_emb, err);
}

cudaError_t g4_launch_rows_quant(const float *src, int src_stride, int T, int K, int8_t *xq, float *xs,
                                 cudaStream_t st, bool pdl, float *xsT) {
    const int G = K / 64;
    return g4_launch(k_rows_quant, dim3(T, (G + 7) / 8), dim3(256), 0, st, pdl, src, src_stride, K, xq, xs, xsT);
}

cudaError_t g4_launch_rows_norm(int mode, const float *src, int T, const float *w_post, const float *res_in,
                                float *res_out, const float *scalar, const float *w_pre, float eps, int8_t *xq,
                                float *xs, cudaStream_t st, bool pdl, float *y_out, int strict, float *xsT) {
    return g4_launch(k_rows_norm, dim3(T), dim3(256), 0, st, pdl, mode, src, w_post, res_in, res_out, scalar, w_pre,
                     eps, xq, xs, y_out, strict, xsT);
}

cudaError_t g4_launch_ple_prep(const float *pli, const float *ple_emb, const float *w, float eps, float scale, int T,
                               float *u, cudaStream_t st, bool pdl, int strict) {
    return g4_launch(k_ple_prep, dim3(T, G4_NUM_LAYERS), dim3(G4_PLE), 0, st, pdl, pli, ple_emb, w, eps, scale, u,
                     strict);
}
