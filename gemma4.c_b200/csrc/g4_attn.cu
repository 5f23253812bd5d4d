// g4_attn.cu — attention over the device-resident FP32 KV rings.
//
// Reference: attention (gemma4.c:411-461) with attention_scores (:281-294),
// softmax (:400-408) and weighted_value_sum (:296-307); q/k/v post-processing
// rmsnorm (:427,437,439) and apply_rope (:381-398).
//
// Semantics kept from the reference:
//   - 8 query heads share one KV head (MQA); scores are unscaled q.k;
//   - sliding layers see keys [max(0, p+1-512), p], global layers [0, p];
//   - ring slot of position p is p & (ring-1): 1024 slots for sliding caches,
//     131072 for global ones; layers 15-34 read the cache of the latest earlier
//     layer of the same kind;
//   - V is RMS-normalised without a weight; RoPE rotates (j, j + hd/2) for
//     j < pairs (all 128 pairs on sliding layers, 64 of 256 on global ones).
// The softmax is computed online (running max and rescaled sum, the same
// recurrence the reference uses) in a different summation order, so outputs
// match within floating-point tolerance, not bit-for-bit.
#include "g4_attn_dev.cuh"

namespace {

// ---------------------------------------------------------------------------
// q/k/v post-processing for a chunk of T tokens (prefill and small-T decode):
// q heads normalised + rotated in place; k, v normalised (+k rotated) and
// written to their ring slots. grid (T, heads [+2]), one warp per vector.
template <int HD>
__global__ void __launch_bounds__(32) k_qkv_post(const AttnArgs a) {
    __shared__ float x[HD];
    griddep_launch();
    griddep_wait();
    const int t = blockIdx.x, which = blockIdx.y;   // 0..7 q heads, 8 = k, 9 = v
    const int p = a.row_pos ? a.row_pos[t] : a.start_pos + t;
    const size_t so = a.row_seq ? (size_t)a.row_seq[t] * a.seq_stride : 0;
    float *src = a.qkv + (size_t)t * a.qkv_stride + which * HD;
    const int lane = threadIdx.x;
    for (int i = lane; i < HD; i += 32) x[i] = src[i];
    __syncwarp();
    const float *cosr = a.rope_cos + (size_t)p * a.pairs, *sinr = a.rope_sin + (size_t)p * a.pairs;
    const float *w = which < kHeads ? a.q_norm : (which == kHeads ? a.k_norm : nullptr);
    norm_rope_warp<HD>(x, w, cosr, sinr, a.pairs, which <= kHeads, a.strict != 0);
    float *dst = which < kHeads ? src
                 : which == kHeads ? a.kcache + so + (size_t)(p & a.mask) * HD
                                   : a.vcache + so + (size_t)(p & a.mask) * HD;
    for (int i = lane; i < HD; i += 32) dst[i] = x[i];
}

// ---------------------------------------------------------------------------
// Row-batched decode attention (g4_forward_batch): grid (splits, rows) then
// (8*HD/256, rows); the same split and combine arithmetic as single-sequence
// decode, so a batch row gives the same bits as decoding that sequence alone.
template <int HD>
__global__ void __launch_bounds__(256) k_attn_rows(const AttnArgs a, int splits) {
    extern __shared__ __align__(16) float sm[];
    griddep_launch();
    griddep_wait();
    attn_rows_split<HD, DecodeKT<HD>::value>(a, blockIdx.y, blockIdx.x, splits, sm);
}

template <int HD>
__global__ void __launch_bounds__(256) k_attn_rows_combine(const AttnArgs a, int splits) {
    __shared__ float wsm[256 + 16];
    griddep_launch();
    griddep_wait();
    const int row = blockIdx.y;
    attn_combine_part<HD>(a, a.row_pos[row], blockIdx.x, splits, wsm,
                          a.part + (size_t)row * splits * kHeads * (HD + 4), a.out + (size_t)row * kHeads * HD,
                          nullptr, nullptr);
}

// ---------------------------------------------------------------------------
// Standalone decode kernels (one launch each) around the shared bodies.
template <int HD>
struct DecodeCfg {
    static constexpr int KT = DecodeKT<HD>::value;
    static constexpr size_t smem = (size_t)decode_smem_floats(HD, KT) * 4;
};

template <int HD>
__global__ void __launch_bounds__(256) k_attn_decode(const AttnArgs a, int splits) {
    extern __shared__ __align__(16) float sm[];
    griddep_launch();
    griddep_wait();
    attn_decode_split<HD, DecodeCfg<HD>::KT>(a, a.pos_dev ? *a.pos_dev : a.start_pos, blockIdx.x, splits, sm);
}

template <int HD>
__global__ void __launch_bounds__(256) k_attn_combine(const AttnArgs a, int splits) {
    __shared__ float wsm[256 + 16];
    griddep_launch();
    griddep_wait();
    attn_combine_part<HD>(a, a.pos_dev ? *a.pos_dev : a.start_pos, blockIdx.x, splits, wsm, a.part, a.out, a.xq, a.xs);
}

// ---------------------------------------------------------------------------
// Strict attention: the reference's exact floating-point order for one
// (token, head) per CTA (gemma4.c:445-456): scores with its 16-lane FMA
// pattern and reduction tree (attention_scores, :281-294), the sequential
// running-max softmax with the host library's expf (:400-408), then every
// output dimension as an FMA chain over the keys in order (weighted_value_sum,
// :296-307). q must be post-processed (k_qkv_post, strict) and the chunk's
// keys already in the ring. Used to demonstrate whole-model parity, not speed.
template <int HD>
__global__ void __launch_bounds__(256) k_attn_strict(const AttnArgs a) {
    __shared__ float q[HD];
    __shared__ float stat[2];
    griddep_launch();
    griddep_wait();
    const int t = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
    const int p = (a.pos_dev ? *a.pos_dev : a.start_pos) + t;
    const int first = first_key(p, a.window), n = p + 1 - first;
    for (int i = tid; i < HD; i += 256) q[i] = a.qkv[(size_t)t * a.qkv_stride + h * HD + i];
    __syncthreads();
    float *sc = a.scores + ((size_t)t * kHeads + h) * a.score_stride;
    for (int i = tid; i < n; i += 256) {
        const float *k = a.kcache + (size_t)((first + i) & a.mask) * HD;
        float s0[8], s1[8];
#pragma unroll
        for (int l = 0; l < 8; l++) { s0[l] = 0.0f; s1[l] = 0.0f; }
        for (int j = 0; j < HD; j += 16) {
#pragma unroll
            for (int l = 0; l < 8; l++) {
                s0[l] = __fmaf_rn(q[j + l], k[j + l], s0[l]);
                s1[l] = __fmaf_rn(q[j + 8 + l], k[j + 8 + l], s1[l]);
            }
        }
        float s8[8], s4[4];
#pragma unroll
        for (int l = 0; l < 8; l++) s8[l] = __fadd_rn(s0[l], s1[l]);
#pragma unroll
        for (int l = 0; l < 4; l++) s4[l] = __fadd_rn(s8[l], s8[l + 4]);
        sc[i] = __fadd_rn(__fadd_rn(s4[0], s4[2]), __fadd_rn(s4[1], s4[3]));
    }
    __syncthreads();
    if (tid == 0) {
        float mx = sc[0], sum = 1.0f;
        for (int i = 1; i < n; i++) {
            const float v = sc[i];
            if (v > mx) {
                sum = __fadd_rn(__fmul_rn(sum, expf_host(__fsub_rn(mx, v))), 1.0f);
                mx = v;
            } else {
                sum = __fadd_rn(sum, expf_host(__fsub_rn(v, mx)));
            }
        }
        stat[0] = mx;
        stat[1] = sum;
    }
    __syncthreads();
    const float mx = stat[0], sum = stat[1];
    for (int i = tid; i < n; i += 256) sc[i] = __fdiv_rn(expf_host(__fsub_rn(sc[i], mx)), sum);
    __syncthreads();
    for (int d = tid; d < HD; d += 256) {
        float acc = 0.0f;
        for (int i = 0; i < n; i++) acc = __fmaf_rn(sc[i], a.vcache[(size_t)((first + i) & a.mask) * HD + d], acc);
        a.out[(size_t)t * (kHeads * HD) + h * HD + d] = acc;
    }
}

// ---------------------------------------------------------------------------
// Prefill attention: CTA = 4 query tokens x 8 heads (32 rows) against key
// tiles of 32, FP32 SIMT with online softmax. q must already be normalised and
// rotated (k_qkv_post) and the chunk's keys already in the ring.
constexpr int kTile = 32;             // keys per tile
constexpr int kQT = 4;               // tokens per CTA
constexpr int kRows = kQT * kHeads;  // 32 query rows

template <int HD>
__global__ void __launch_bounds__(256) k_attn_prefill(const AttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    float *Qs = sm;                        // [32][HD]
    float *Ks = Qs + kRows * HD;           // [32][HD + 4]
    float *Vs = Ks + kTile * (HD + 4);     // [32][HD]
    float *Ps = Vs + kTile * HD;           // [32][33]
    float *rm = Ps + kRows * 33;           // [32] running max
    float *rl = rm + kRows;                // [32] running sum
    float *rc = rl + kRows;                // [32] correction of this tile
    const int tid = threadIdx.x;
    const int t_base = blockIdx.x * kQT;

    griddep_launch();
    griddep_wait();

    // load q rows: row r = token_local * 8 + head
    for (int idx = tid; idx < kRows * (HD / 4); idx += 256) {
        const int r = idx / (HD / 4), c4 = idx - r * (HD / 4);
        const int t = t_base + r / kHeads, h = r % kHeads;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t < a.T) v = *(const float4 *)(a.qkv + (size_t)t * a.qkv_stride + h * HD + c4 * 4);
        *(float4 *)&Qs[r * HD + c4 * 4] = v;
    }
    if (tid < kRows) {
        rm[tid] = -INFINITY;
        rl[tid] = 0.0f;
    }
    const int t_last = min(a.T, t_base + kQT) - 1;
    const int p_first = a.start_pos + t_base, p_last = a.start_pos + t_last;
    const int k_lo = first_key(p_first, a.window), k_hi = p_last;   // inclusive

    // S-phase mapping: rows (2qr, 2qr+1), keys (kr, kr+16)
    const int qr = tid >> 4, kr = tid & 15;
    int prow[2], pfirst[2];
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const int r = 2 * qr + i, t = t_base + r / kHeads;
        prow[i] = t < a.T ? a.start_pos + t : -1;
        pfirst[i] = prow[i] >= 0 ? first_key(prow[i], a.window) : 0;
    }
    // PV mapping: rows 4*(tid/32) .. +3, dims 4*lane + 128*i
    const int rg = tid >> 5, lane = tid & 31;
    constexpr int NV = HD / 128;
    float4 o[4][NV];
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
        for (int i = 0; i < NV; i++) o[r][i] = make_float4(0.f, 0.f, 0.f, 0.f);

    for (int kt = k_lo; kt <= k_hi; kt += kTile) {
        const int nt = min(kTile, k_hi + 1 - kt);
        __syncthreads();
        for (int idx = tid; idx < nt * (HD / 4); idx += 256) {
            const int r = idx / (HD / 4), c4 = idx - r * (HD / 4);
            const size_t slot = (size_t)((kt + r) & a.mask) * HD;
            cp_async16(&Ks[r * (HD + 4) + c4 * 4], a.kcache + slot + c4 * 4);
            cp_async16(&Vs[r * HD + c4 * 4], a.vcache + slot + c4 * 4);
        }
        cp_async_commit();
        cp_async_wait<0>();
        __syncthreads();
        // scores
        float s[2][2];
#pragma unroll
        for (int i = 0; i < 2; i++)
#pragma unroll
            for (int jj = 0; jj < 2; jj++) s[i][jj] = 0.0f;
        const float *q0 = Qs + (2 * qr) * HD, *q1 = q0 + HD;
        const float *k0 = Ks + kr * (HD + 4), *k1 = Ks + (kr + 16) * (HD + 4);
#pragma unroll 4
        for (int d = 0; d < HD; d += 4) {
            const float4 a0 = *(const float4 *)&q0[d], a1 = *(const float4 *)&q1[d];
            const float4 b0 = *(const float4 *)&k0[d], b1 = *(const float4 *)&k1[d];
            s[0][0] = fmaf(a0.x, b0.x, fmaf(a0.y, b0.y, fmaf(a0.z, b0.z, fmaf(a0.w, b0.w, s[0][0]))));
            s[0][1] = fmaf(a0.x, b1.x, fmaf(a0.y, b1.y, fmaf(a0.z, b1.z, fmaf(a0.w, b1.w, s[0][1]))));
            s[1][0] = fmaf(a1.x, b0.x, fmaf(a1.y, b0.y, fmaf(a1.z, b0.z, fmaf(a1.w, b0.w, s[1][0]))));
            s[1][1] = fmaf(a1.x, b1.x, fmaf(a1.y, b1.y, fmaf(a1.z, b1.z, fmaf(a1.w, b1.w, s[1][1]))));
        }
        // mask + online softmax per row (16 lanes share a row pair)
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const int r = 2 * qr + i;
            float mloc = -INFINITY;
#pragma unroll
            for (int jj = 0; jj < 2; jj++) {
                const int key = kt + kr + 16 * jj;
                const bool ok = prow[i] >= 0 && (kr + 16 * jj) < nt && key <= prow[i] && key >= pfirst[i];
                if (!ok) s[i][jj] = -INFINITY;
                mloc = fmaxf(mloc, s[i][jj]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, off));
            const float mold = rm[r];
            const float mn = fmaxf(mold, mloc);
            float psum = 0.0f;
#pragma unroll
            for (int jj = 0; jj < 2; jj++) {
                const float pv = (s[i][jj] == -INFINITY) ? 0.0f : expf(s[i][jj] - mn);
                Ps[r * 33 + kr + 16 * jj] = pv;
                psum += pv;
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
            __syncwarp();
            if (kr == 0) {
                const float corr = (mold == -INFINITY) ? 0.0f : expf(mold - mn);
                rc[r] = corr;
                rl[r] = rl[r] * corr + psum;
                rm[r] = mn;
            }
        }
        __syncthreads();
        // PV
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const float corr = rc[rg * 4 + r];
#pragma unroll
            for (int i = 0; i < NV; i++) {
                o[r][i].x *= corr; o[r][i].y *= corr; o[r][i].z *= corr; o[r][i].w *= corr;
            }
        }
        for (int jk = 0; jk < nt; jk++) {
            const float *vr = Vs + jk * HD + 4 * lane;
            float4 vv[NV];
#pragma unroll
            for (int i = 0; i < NV; i++) vv[i] = *(const float4 *)&vr[128 * i];
#pragma unroll
            for (int r = 0; r < 4; r++) {
                const float pk = Ps[(rg * 4 + r) * 33 + jk];
#pragma unroll
                for (int i = 0; i < NV; i++) {
                    o[r][i].x = fmaf(pk, vv[i].x, o[r][i].x);
                    o[r][i].y = fmaf(pk, vv[i].y, o[r][i].y);
                    o[r][i].z = fmaf(pk, vv[i].z, o[r][i].z);
                    o[r][i].w = fmaf(pk, vv[i].w, o[r][i].w);
                }
            }
        }
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 4; r++) {
        const int row = rg * 4 + r, t = t_base + row / kHeads, h = row % kHeads;
        if (t >= a.T) continue;
        const float inv = 1.0f / rl[row];
        float *dst = a.out + (size_t)t * (kHeads * HD) + h * HD + 4 * lane;
#pragma unroll
        for (int i = 0; i < NV; i++)
            *(float4 *)&dst[128 * i] = make_float4(o[r][i].x * inv, o[r][i].y * inv, o[r][i].z * inv, o[r][i].w * inv);
    }
}

template <typename K>
cudaError_t set_smem(K kern, size_t bytes) {
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

size_t prefill_smem(int hd) { return (size_t)(kRows * hd + kTile * (hd + 4) + kTile * hd + kRows * 33 + 3 * kRows) * 4; }

}  // namespace

cudaError_t g4_launch_qkv_post(const AttnArgs &a, cudaStream_t st, bool pdl) {
    dim3 grid(a.T, kHeads + (a.has_kv ? 2 : 0));
    if (a.hd == 256) return g4_launch(k_qkv_post<256>, grid, dim3(32), 0, st, pdl, a);
    if (a.hd == 512) return g4_launch(k_qkv_post<512>, grid, dim3(32), 0, st, pdl, a);
    return cudaErrorInvalidValue;
}

cudaError_t g4_launch_attn_decode(const AttnArgs &a, int splits, cudaStream_t st, bool pdl) {
    if (splits < 1 || splits > 256) return cudaErrorInvalidValue;
    if (a.hd == 256) {
        const size_t smem = DecodeCfg<256>::smem;
        static bool once = false;
        if (!once) { cudaError_t e = set_smem(k_attn_decode<256>, smem); if (e) return e; once = true; }
        return g4_launch(k_attn_decode<256>, dim3(splits), dim3(256), smem, st, pdl, a, splits);
    }
    if (a.hd == 512) {
        const size_t smem = DecodeCfg<512>::smem;
        static bool once = false;
        if (!once) { cudaError_t e = set_smem(k_attn_decode<512>, smem); if (e) return e; once = true; }
        return g4_launch(k_attn_decode<512>, dim3(splits), dim3(256), smem, st, pdl, a, splits);
    }
    return cudaErrorInvalidValue;
}

cudaError_t g4_launch_attn_rows(const AttnArgs &a, int splits, cudaStream_t st, bool pdl) {
    if (splits < 1 || splits > 256 || a.T < 1 || !a.row_seq || !a.row_pos) return cudaErrorInvalidValue;
    const dim3 gs(splits, a.T), gc(kHeads * a.hd / 256, a.T);
    if (a.hd == 256) {
        const size_t smem = DecodeCfg<256>::smem;
        static bool once = false;
        if (!once) { cudaError_t e = set_smem(k_attn_rows<256>, smem); if (e) return e; once = true; }
        cudaError_t e = g4_launch(k_attn_rows<256>, gs, dim3(256), smem, st, pdl, a, splits);
        return e ? e : g4_launch(k_attn_rows_combine<256>, gc, dim3(256), 0, st, pdl, a, splits);
    }
    if (a.hd == 512) {
        const size_t smem = DecodeCfg<512>::smem;
        static bool once = false;
        if (!once) { cudaError_t e = set_smem(k_attn_rows<512>, smem); if (e) return e; once = true; }
        cudaError_t e = g4_launch(k_attn_rows<512>, gs, dim3(256), smem, st, pdl, a, splits);
        return e ? e : g4_launch(k_attn_rows_combine<512>, gc, dim3(256), 0, st, pdl, a, splits);
    }
    return cudaErrorInvalidValue;
}

cudaError_t g4_launch_attn_combine(const AttnArgs &a, int splits, cudaStream_t st, bool pdl) {
    if (splits < 1 || splits > 256) return cudaErrorInvalidValue;
    const int grid = kHeads * a.hd / 256;
    if (a.hd == 256) return g4_launch(k_attn_combine<256>, dim3(grid), dim3(256), 0, st, pdl, a, splits);
    if (a.hd == 512) return g4_launch(k_attn_combine<512>, dim3(grid), dim3(256), 0, st, pdl, a, splits);
    return cudaErrorInvalidValue;
}

cudaError_t g4_launch_attn_strict(const AttnArgs &a, cudaStream_t st, bool pdl) {
    if (!a.scores) return cudaErrorInvalidValue;
    dim3 grid(a.T, kHeads);
    if (a.hd == 256) return g4_launch(k_attn_strict<256>, grid, dim3(256), 0, st, pdl, a);
    if (a.hd == 512) return g4_launch(k_attn_strict<512>, grid, dim3(256), 0, st, pdl, a);
    return cudaErrorInvalidValue;
}

cudaError_t g4_launch_attn_prefill(const AttnArgs &a, cudaStream_t st, bool pdl) {
    const size_t smem = prefill_smem(a.hd);
    dim3 grid((a.T + kQT - 1) / kQT);
    if (a.hd == 256) {
        static bool once = false;
        if (!once) { cudaError_t e = set_smem(k_attn_prefill<256>, smem); if (e) return e; once = true; }
        return g4_launch(k_attn_prefill<256>, grid, dim3(256), smem, st, pdl, a);
    }
    if (a.hd == 512) {
        static bool once = false;
        if (!once) { cudaError_t e = set_smem(k_attn_prefill<512>, smem); if (e) return e; once = true; }
        return g4_launch(k_attn_prefill<512>, grid, dim3(256), smem, st, pdl, a);
    }
    return cudaErrorInvalidValue;
}
