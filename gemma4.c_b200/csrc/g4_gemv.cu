// g4_gemv.cu — decode-path int8 GEMV (T <= 4 token rows) with fused prologues
// and epilogues.
//
// Reference: matmul_int8 / matmul_block (gemma4.c:192-262) and the ops around
// each call site in forward/attention/logits (gemma4.c:411-522).
//
// Design (one persistent CTA per SM, 8 consumer warps + 1 producer warp):
//   - Each CTA owns a contiguous range of output rows. Its weight rows stream
//     HBM -> shared memory through a ring of STAGES stages with 1-D bulk async
//     copies (cp.async.bulk + mbarrier complete_tx). A stage is `rb` rows x `kc`
//     bytes; the first stage of each row batch also carries the batch's FP16
//     scales.
//   - The producer starts streaming at kernel entry, before
//     griddepcontrol.wait: with programmatic dependent launch the weight fetch
//     overlaps the tail of the previous kernel. Only the consumers wait for the
//     previous kernel's activations.
//   - Consumers first build the int8 activation (fused RMSNorm / residual /
//     embedding + dynamic quantisation, gemma4.c:265-279) in shared memory,
//     then for every stage compute the exact int32 dot of every (row, 64-group)
//     with dp4a (16-byte pieces, quad shuffles), and finally advance one fp32
//     chain per (row, token): acc = fma((float)dot_g, ws_g * xs_g, acc) with g
//     ascending — the reference's rounding sequence (gemma4.c:218), so outputs
//     are bit-exact given the same activation.
//   - Epilogues fuse GeGLU of interleaved gate/up rows, the PLE GeGLU, and the
//     logits soft-cap with a grid-wide argmax (last-CTA ticket).
#include "g4_common.cuh"
#include "g4_internal.h"

namespace {

constexpr int kConsumers = 256;
constexpr int kThreads = kConsumers + 32;
constexpr int kStages = 4;
constexpr int kMaxT = 4;

struct Layout {
    int stage_bytes, sbytes;
    int off_ring, off_sring, off_bars, off_xq, off_xs, off_dots, off_vec, off_red, total;
};

__host__ __device__ inline int round_up(int v, int a) { return (v + a - 1) / a * a; }

__host__ __device__ inline Layout make_layout(int K, int T, int rb, int kc, int pro) {
    Layout L;
    int G = K / 64, GC = kc / 64;
    L.stage_bytes = round_up(rb * kc, 128);
    L.sbytes = round_up(rb * G * 2, 16);
    int o = 0;
    L.off_ring = o;
    o += kStages * L.stage_bytes;
    L.off_sring = o;
    o += kStages * L.sbytes;
    o = round_up(o, 16);
    L.off_bars = o;
    o += 2 * kStages * 8;
    L.off_xq = round_up(o, 16);
    o = L.off_xq + round_up(T * K, 16);
    L.off_xs = o;
    o += round_up(T * G * 4, 16);
    L.off_dots = o;
    o += round_up(rb * GC * T * 4, 16);
    L.off_vec = o;
    o += (pro == PRO_NORM_QUANT || pro == PRO_RES_NORM_QUANT || pro == PRO_RES_QUANT || pro == PRO_EMBED_QUANT)
             ? G4_HIDDEN * 4
             : 0;
    L.off_red = round_up(o, 16);
    o = L.off_red + 64 * 4;
    L.total = o;
    return L;
}

// Sum over the 256 consumer threads; every consumer gets the result.
__device__ float block_sum(float v, float *red) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    v = warp_sum(v);
    if (lane == 0) red[warp] = v;
    bar_sync(1, kConsumers);
    float r = 0.0f;
#pragma unroll
    for (int i = 0; i < kConsumers / 32; i++) r += red[i];
    bar_sync(1, kConsumers);
    return r;
}

// Quantise `src` (K floats, shared or global) into xq/xs, one warp per 64-group.
__device__ void quantize_row(const float *src, int K, int8_t *xq, float *xs) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = K / 64;
    for (int g = warp; g < G; g += kConsumers / 32) {
        float a = src[g * 64 + lane], b = src[g * 64 + 32 + lane];
        float amax = warp_max(fmaxf(fabsf(a), fabsf(b)));
        float s = quant_scale(amax);
        float inv = quant_inv(s);
        xq[g * 64 + lane] = (int8_t)quant_one(a, inv);
        xq[g * 64 + 32 + lane] = (int8_t)quant_one(b, inv);
        if (lane == 0) xs[g] = s;
    }
}

template <int T, int PRO, int EPI>
__global__ void __launch_bounds__(kThreads, 1) k_gemv(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int K = a.m.K, N = a.m.N, G = K >> 6;
    const int kc = a.kc, GC = kc >> 6, nchunks = K / kc, rb = a.rb;
    const Layout L = make_layout(K, T, rb, kc, PRO);
    uint8_t *ring = smem + L.off_ring;
    uint8_t *sring = smem + L.off_sring;
    uint64_t *full = (uint64_t *)(smem + L.off_bars);
    uint64_t *empty = full + kStages;
    int8_t *xq = (int8_t *)(smem + L.off_xq);
    float *xs = (float *)(smem + L.off_xs);
    int32_t *dots = (int32_t *)(smem + L.off_dots);
    float *vec = (float *)(smem + L.off_vec);
    float *red = (float *)(smem + L.off_red);

    // Row range of this CTA (balanced in units of row_gran rows).
    const int units = N / a.row_gran;
    const int u0 = (int)((long long)blockIdx.x * units / gridDim.x);
    const int u1 = (int)((long long)(blockIdx.x + 1) * units / gridDim.x);
    const int n0 = u0 * a.row_gran, n1 = u1 * a.row_gran;
    const int nbatch = (n1 - n0 + rb - 1) / rb;
    const int nstages = nbatch * nchunks;

    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int i = 0; i < kStages; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        mbar_fence_init();
    }
    __syncthreads();
    griddep_launch();

    if (tid >= kConsumers) {
        // ---------------- producer warp ----------------
        if (tid == kConsumers) {
            const uint64_t pol = l2_policy_evict_first();
            for (int s = 0; s < nstages; s++) {
                const int slot = s % kStages, use = s / kStages;
                if (use > 0 && !mbar_wait(&empty[slot], (use - 1) & 1, a.err, G4D_TIMEOUT_EMPTY)) break;
                const int b = s / nchunks, c = s % nchunks;
                const int row0 = n0 + b * rb;
                const int rows = min(rb, n1 - row0);
                uint32_t bytes = (uint32_t)(rows * kc) + (c == 0 ? (uint32_t)(rows * G * 2) : 0u);
                mbar_arrive_expect_tx(&full[slot], bytes);
                for (int r = 0; r < rows; r++)
                    bulk_g2s(ring + slot * L.stage_bytes + r * kc, a.m.w + (size_t)(row0 + r) * K + (size_t)c * kc,
                             (uint32_t)kc, &full[slot], pol);
                if (c == 0)
                    bulk_g2s(sring + (b % kStages) * L.sbytes, a.m.s + (size_t)row0 * G, (uint32_t)(rows * G * 2),
                             &full[slot], pol);
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    const int warp = tid >> 5, lane = tid & 31;
    griddep_wait();

    // ---- prologue: build xq[T][K], xs[T][G] ----
    if (PRO == PRO_LOADQ) {
        const int4 *q4 = (const int4 *)a.xq_in;
        int4 *d4 = (int4 *)xq;
        for (int i = tid; i < T * K / 16; i += kConsumers) d4[i] = q4[i];
        for (int i = tid; i < T * G; i += kConsumers) xs[i] = a.xs_in[i];
    } else if (PRO == PRO_QUANT) {
        for (int t = 0; t < T; t++) quantize_row(a.src + (size_t)t * a.src_stride, K, xq + t * K, xs + t * G);
    } else {
        // K == 1536 (hidden width) for all fused-norm prologues; 6 values per thread.
        constexpr int PER = G4_HIDDEN / kConsumers;
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
                    int e = tid + i * kConsumers;
                    float sc = __fmul_rn(h2f(sr[e >> 6]), a.embed_mult);   // gemma4.c:350
                    y[i] = __fmul_rn((float)wr[e], sc);                     // gemma4.c:354
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
                float hv[PER];
                float ss = 0.0f;
#pragma unroll
                for (int i = 0; i < PER; i++) {
                    hv[i] = h[tid + i * kConsumers];
                    ss = __fadd_rn(ss, __fmul_rn(hv[i], hv[i]));
                }
                ss = block_sum(ss, red);
                if (PRO == PRO_NORM_QUANT) {
                    float inv = rms_inv(ss, (float)G4_HIDDEN, a.eps);
#pragma unroll
                    for (int i = 0; i < PER; i++) y[i] = rms_apply(hv[i], inv, a.w_pre[tid + i * kConsumers]);
                } else {
                    // residual update: r' = (r + rmsnorm(h, w_post)) * scalar (gemma4.c:485-486,496-497,505-506)
                    float inv = rms_inv(ss, (float)G4_HIDDEN, a.eps);
                    const float sc = a.scalar ? *a.scalar : 1.0f;
                    float ss2 = 0.0f;
#pragma unroll
                    for (int i = 0; i < PER; i++) {
                        int e = tid + i * kConsumers;
                        float hn = rms_apply(hv[i], inv, a.w_post[e]);
                        float r = __fadd_rn(a.res_in[t * G4_HIDDEN + e], hn);
                        if (a.scalar) r = __fmul_rn(r, sc);
                        y[i] = r;
                        ss2 = __fadd_rn(ss2, __fmul_rn(r, r));
                        if (blockIdx.x == 0) a.res_out[t * G4_HIDDEN + e] = r;
                    }
                    if (PRO == PRO_RES_NORM_QUANT) {
                        ss2 = block_sum(ss2, red);
                        float inv2 = rms_inv(ss2, (float)G4_HIDDEN, a.eps);
#pragma unroll
                        for (int i = 0; i < PER; i++) y[i] = rms_apply(y[i], inv2, a.w_pre[tid + i * kConsumers]);
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < PER; i++) vec[tid + i * kConsumers] = y[i];
            bar_sync(1, kConsumers);
            quantize_row(vec, G4_HIDDEN, xq + t * K, xs + t * G);
            bar_sync(1, kConsumers);
        }
    }
    bar_sync(1, kConsumers);

    // ---- main loop over stages ----
    const int ppr = kc / 16;   // 16-byte pieces per row per stage
    float acc = 0.0f;
    float best_v = -INFINITY;
    int best_i = 0x7fffffff;
    const int j = tid;         // chain owner: (r = j / T, t = j % T) for j < rows * T

    for (int s = 0; s < nstages; s++) {
        const int slot = s % kStages;
        const int b = s / nchunks, c = s % nchunks;
        const int row0 = n0 + b * rb;
        const int rows = min(rb, n1 - row0);
        if (!mbar_wait(&full[slot], (s / kStages) & 1, a.err, G4D_TIMEOUT_FULL)) return;

        // phase A: exact int32 dot of every (row, group) in the stage
        const uint8_t *st = ring + slot * L.stage_bytes;
        const int pieces = rows * ppr;
        for (int p0 = 0; p0 < pieces; p0 += kConsumers) {
            const int p = p0 + tid;
            const bool valid = p < pieces;
            int4 w4 = make_int4(0, 0, 0, 0);
            int r = 0, kb = 0;
            if (valid) {
                w4 = *(const int4 *)(st + p * 16);
                r = p / ppr;
                kb = (p - r * ppr) * 16;
            }
            int d[T];
#pragma unroll
            for (int t = 0; t < T; t++) {
                int4 x4 = make_int4(0, 0, 0, 0);
                if (valid) x4 = *(const int4 *)(xq + t * K + c * kc + kb);
                int v = dp4a((uint32_t)w4.x, (uint32_t)x4.x, 0);
                v = dp4a((uint32_t)w4.y, (uint32_t)x4.y, v);
                v = dp4a((uint32_t)w4.z, (uint32_t)x4.z, v);
                v = dp4a((uint32_t)w4.w, (uint32_t)x4.w, v);
                v += __shfl_xor_sync(0xffffffffu, v, 1);
                v += __shfl_xor_sync(0xffffffffu, v, 2);
                d[t] = v;
            }
            if (valid && (lane & 3) == 0) {
#pragma unroll
                for (int t = 0; t < T; t++) dots[(r * GC + (kb >> 6)) * T + t] = d[t];
            }
        }
        bar_sync(1, kConsumers);

        // phase B: ordered fp32 dequant chain (gemma4.c:218)
        if (j < rows * T) {
            const int r = j / T, t = j - (j / T) * T;
            const uint16_t *sc = (const uint16_t *)(sring + (b % kStages) * L.sbytes) + r * G + c * GC;
            const float *xsr = xs + t * G + c * GC;
            for (int gc = 0; gc < GC; gc++) {
                int dv = dots[(r * GC + gc) * T + t];
                float scale = __fmul_rn(h2f(sc[gc]), xsr[gc]);
                acc = __fmaf_rn(__int2float_rn(dv), scale, acc);
                if (a.dots_out) a.dots_out[((size_t)t * N + row0 + r) * G + c * GC + gc] = dv;
            }
        }
        bar_sync(1, kConsumers);
        if (tid == 0) mbar_arrive(&empty[slot]);

        // epilogue once the batch's last K-chunk is in
        if (c == nchunks - 1) {
            if (warp == 0) {
                const bool own = j < rows * T;
                const int r = j / T, t = j - (j / T) * T;
                const int n = row0 + r;
                if (EPI == EPI_STORE) {
                    if (own) a.out[(size_t)t * a.out_stride + n] = acc;
                } else if (EPI == EPI_GEGLU_PAIR) {
                    float up = __shfl_down_sync(0xffffffffu, acc, T);
                    if (own && (r & 1) == 0)
                        a.out[(size_t)t * a.out_stride + (n >> 1)] =
                            geglu_one(acc, up, a.gelu, 4096, -8.0f, 8.0f, 4095.0f / 16.0f);
                } else if (EPI == EPI_PLE) {
                    if (own)
                        a.out[(size_t)t * a.out_stride + n] =
                            geglu_one(acc, a.ple_u[(size_t)t * a.u_stride + n], a.gelu, 4096, -8.0f, 8.0f,
                                      4095.0f / 16.0f);
                } else if (EPI == EPI_LOGITS) {
                    if (own) {
                        float v = __fmul_rn(30.0f, tanhf(__fdiv_rn(acc, 30.0f)));   // gemma4.c:519
                        a.out[(size_t)t * a.out_stride + n] = v;
                        if (v > best_v) { best_v = v; best_i = n; }
                    }
                }
            }
            acc = 0.0f;
        }
    }

    if (EPI == EPI_LOGITS) {
        // per-CTA argmax (first strict maximum, gemma4.c:537-541), then last CTA reduces
        float *cand = red;  // [32][2]
        if (warp == 0) {
            cand[lane * 2] = best_v;
            cand[lane * 2 + 1] = __int_as_float(best_i);
        }
        bar_sync(1, kConsumers);
        if (tid < T) {
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int q = tid; q < 32; q += T) {
                float v = cand[q * 2];
                int i = __float_as_int(cand[q * 2 + 1]);
                if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
            }
            a.argmax_part[((size_t)blockIdx.x * T + tid) * 2] = bv;
            a.argmax_part[((size_t)blockIdx.x * T + tid) * 2 + 1] = __int_as_float(bi);
        }
        __threadfence();
        bar_sync(1, kConsumers);
        __shared__ unsigned last;
        if (tid == 0) last = atomicAdd(a.ticket, 1u) == gridDim.x - 1;
        bar_sync(1, kConsumers);
        if (last) {
            __threadfence();
            if (tid < T) {
                float bv = -INFINITY;
                int bi = 0x7fffffff;
                for (int q = 0; q < (int)gridDim.x; q++) {
                    float v = __ldcg(&a.argmax_part[((size_t)q * T + tid) * 2]);
                    int i = __float_as_int(__ldcg(&a.argmax_part[((size_t)q * T + tid) * 2 + 1]));
                    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
                }
                a.argmax_out[tid] = bi;
            }
            if (tid == 0) *a.ticket = 0u;
        }
    }
}

template <int T, int PRO, int EPI>
cudaError_t launch_t(const GemvArgs &a, int grid, cudaStream_t st, bool pdl) {
    Layout L = make_layout(a.m.K, T, a.rb, a.kc, PRO);
    auto kern = k_gemv<T, PRO, EPI>;
    static int configured = 0;
    if (configured < L.total) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
        configured = 200 * 1024;
    }
    return g4_launch(kern, dim3(grid), dim3(kThreads), (size_t)L.total, st, pdl, a);
}

template <int T>
cudaError_t launch_pe(const GemvArgs &a, int pro, int epi, int grid, cudaStream_t st, bool pdl) {
#define G4_CASE(P, E)                                              \
    if (pro == P && epi == E) return launch_t<T, P, E>(a, grid, st, pdl);
    G4_CASE(PRO_QUANT, EPI_STORE)
    G4_CASE(PRO_LOADQ, EPI_STORE)
    G4_CASE(PRO_NORM_QUANT, EPI_STORE)
    G4_CASE(PRO_RES_NORM_QUANT, EPI_STORE)
    G4_CASE(PRO_RES_NORM_QUANT, EPI_GEGLU_PAIR)
    G4_CASE(PRO_RES_QUANT, EPI_PLE)
    G4_CASE(PRO_EMBED_QUANT, EPI_STORE)
    G4_CASE(PRO_NORM_QUANT, EPI_LOGITS)
    G4_CASE(PRO_LOADQ, EPI_GEGLU_PAIR)
    G4_CASE(PRO_LOADQ, EPI_PLE)
    G4_CASE(PRO_LOADQ, EPI_LOGITS)
    G4_CASE(PRO_QUANT, EPI_GEGLU_PAIR)
    G4_CASE(PRO_QUANT, EPI_PLE)
#undef G4_CASE
    return cudaErrorInvalidValue;
}

}  // namespace

void g4_gemv_plan(GemvArgs &a, int num_sms) {
    (void)num_sms;
    const int K = a.m.K, G = K / 64;
    a.kc = K <= 2048 ? K : 2048;
    int rb = 16384 / a.kc;
    if (rb < 1) rb = 1;
    if (rb > 16) rb = 16;
    if (rb > 32 / a.T) rb = 32 / a.T;
    if (a.row_gran < 1) a.row_gran = 1;
    if (G < 8) a.row_gran = 2;
    if (a.row_gran == 2) rb = rb < 2 ? 2 : (rb & ~1);
    a.rb = rb;
}

int g4_gemv_smem_bytes(const GemvArgs &a, int pro) {
    int T = a.T <= 1 ? 1 : (a.T <= 2 ? 2 : 4);
    return make_layout(a.m.K, T, a.rb, a.kc, pro).total;
}

cudaError_t g4_launch_gemv(const GemvArgs &a, int pro, int epi, int grid, cudaStream_t st, bool pdl) {
    if (a.T < 1 || a.T > kMaxT || a.m.K % 256 != 0 || a.m.N % a.row_gran != 0) return cudaErrorInvalidValue;
    if (grid < 1) return cudaErrorInvalidValue;
    switch (a.T) {
    case 1: return launch_pe<1>(a, pro, epi, grid, st, pdl);
    case 2: return launch_pe<2>(a, pro, epi, grid, st, pdl);
    case 3: return launch_pe<3>(a, pro, epi, grid, st, pdl);
    default: return launch_pe<4>(a, pro, epi, grid, st, pdl);
    }
}
