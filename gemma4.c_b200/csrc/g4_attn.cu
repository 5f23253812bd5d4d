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
#include "g4_common.cuh"
#include "g4_internal.h"

namespace {

constexpr int kHeads = G4_HEADS;

G4_DEV int first_key(int p, int window) { return (window && p + 1 > window) ? p + 1 - window : 0; }

// RMS-normalise (optional weight) and rotate one head vector held in shared
// memory by one warp. x has HD floats.
template <int HD>
G4_DEV void norm_rope_warp(float *x, const float *w, const float *cosr, const float *sinr, int pairs, bool rope,
                           bool strict = false) {
    const int lane = threadIdx.x & 31;
    float v[HD / 32];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < HD / 32; i++) {
        v[i] = x[lane + 32 * i];
        ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
    }
    if (strict) {
        // reference order (gemma4.c:367-368): one lane, index order
        ss = lane == 0 ? seq_sumsq(x, HD) : 0.0f;
        ss = __shfl_sync(0xffffffffu, ss, 0);
    } else {
        ss = warp_sum(ss);
    }
    const float inv = rms_inv(ss, (float)HD, 1e-6f);
#pragma unroll
    for (int i = 0; i < HD / 32; i++) x[lane + 32 * i] = rms_apply(v[i], inv, w ? w[lane + 32 * i] : 1.0f);
    __syncwarp();
    if (rope) {
        for (int jj = lane; jj < pairs; jj += 32) {
            const float a0 = x[jj], b0 = x[jj + HD / 2], c = cosr[jj], s = sinr[jj];
            x[jj] = __fsub_rn(__fmul_rn(a0, c), __fmul_rn(b0, s));
            x[jj + HD / 2] = __fadd_rn(__fmul_rn(b0, c), __fmul_rn(a0, s));
        }
    }
    __syncwarp();
}

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
    const int p = a.start_pos + t;
    float *src = a.qkv + (size_t)t * a.qkv_stride + which * HD;
    const int lane = threadIdx.x;
    for (int i = lane; i < HD; i += 32) x[i] = src[i];
    __syncwarp();
    const float *cosr = a.rope_cos + (size_t)p * a.pairs, *sinr = a.rope_sin + (size_t)p * a.pairs;
    const float *w = which < kHeads ? a.q_norm : (which == kHeads ? a.k_norm : nullptr);
    norm_rope_warp<HD>(x, w, cosr, sinr, a.pairs, which <= kHeads, a.strict != 0);
    float *dst = which < kHeads ? src
                 : which == kHeads ? a.kcache + (size_t)(p & a.mask) * HD
                                   : a.vcache + (size_t)(p & a.mask) * HD;
    for (int i = lane; i < HD; i += 32) dst[i] = x[i];
}

// ---------------------------------------------------------------------------
// Decode (T = 1) split-KV attention. Every CTA post-processes q (all heads)
// and, on layers that own the cache, the new k/v; CTA 0 writes k/v to the
// ring, and every CTA uses its own copy for key == pos. CTA c covers a slice of
// the visible keys (at least kMinSplit keys per slice) and writes (max, sum,
// unnormalised output) per head. K/V tiles stream through a double-buffered
// cp.async pipeline; warp h owns query head h, lanes own keys for the scores
// and output dimensions for the value sum.
constexpr int kTile = 32;
constexpr int kMinSplit = 64;

G4_DEV void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
G4_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
G4_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Key range of split `s` for position p; returns the number of active splits.
G4_DEV int split_range(int p, int window, int splits, int s, int *k0, int *k1) {
    const int kf = first_key(p, window), nk = p + 1 - kf;
    int per = (nk + splits - 1) / splits;
    per = per < kMinSplit ? kMinSplit : (per + 31) / 32 * 32;
    *k0 = kf + s * per;
    *k1 = min(p + 1, *k0 + per);
    return (nk + per - 1) / per;
}

template <int HD>
struct DecodeCfg {
    static constexpr int KT = HD == 512 ? 16 : 32;   // keys per tile
    static constexpr int LPK = 32 / KT;              // lanes per key in the score phase
    static constexpr int KS = HD + 4;                // padded K row (floats)
    static constexpr size_t smem = (size_t)(kHeads * HD + 2 * HD + 2 * KT * KS + 2 * KT * HD) * 4;
};

template <int HD>
__global__ void __launch_bounds__(256) k_attn_decode(const AttnArgs a, int splits) {
    using Cfg = DecodeCfg<HD>;
    constexpr int KT = Cfg::KT, LPK = Cfg::LPK, KS = Cfg::KS;
    extern __shared__ __align__(16) float sm[];
    float *qn = sm;                       // [8][HD]
    float *kn = qn + kHeads * HD;         // [HD]
    float *vn = kn + HD;                  // [HD]
    float *Ks = vn + HD;                  // [2][KT][KS]
    float *Vs = Ks + 2 * KT * KS;         // [2][KT][HD]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    griddep_launch();
    griddep_wait();
    const int p = a.pos_dev ? *a.pos_dev : a.start_pos;
    int k0, k1;
    const int active = split_range(p, a.window, splits, blockIdx.x, &k0, &k1);
    if ((int)blockIdx.x >= active) return;

    // start streaming the first tile before the q/k/v post-processing
    auto issue = [&](int tile, int buf) {
        const int kt = k0 + tile * KT, nt = min(KT, k1 - kt);
        for (int idx = threadIdx.x; idx < nt * (HD / 4); idx += 256) {
            const int r = idx / (HD / 4), c4 = idx - r * (HD / 4);
            const size_t slot = (size_t)((kt + r) & a.mask) * HD;
            cp_async16(&Ks[(buf * KT + r) * KS + c4 * 4], a.kcache + slot + c4 * 4);
            cp_async16(&Vs[(buf * KT + r) * HD + c4 * 4], a.vcache + slot + c4 * 4);
        }
        cp_async_commit();
    };
    const int ntiles = k1 > k0 ? (k1 - k0 + KT - 1) / KT : 0;
    if (ntiles > 0) issue(0, 0);

    const float *cosr = a.rope_cos + (size_t)p * a.pairs, *sinr = a.rope_sin + (size_t)p * a.pairs;
    for (int i = lane; i < HD; i += 32) qn[warp * HD + i] = a.qkv[warp * HD + i];
    __syncwarp();
    norm_rope_warp<HD>(qn + warp * HD, a.q_norm, cosr, sinr, a.pairs, true);
    if (a.has_kv && warp < 2) {
        float *x = warp == 0 ? kn : vn;
        const float *src = a.qkv + kHeads * HD + warp * HD;
        for (int i = lane; i < HD; i += 32) x[i] = src[i];
        __syncwarp();
        norm_rope_warp<HD>(x, warp == 0 ? a.k_norm : nullptr, cosr, sinr, a.pairs, warp == 0);
        if (blockIdx.x == 0) {
            float *dst = (warp == 0 ? a.kcache : a.vcache) + (size_t)(p & a.mask) * HD;
            for (int i = lane; i < HD; i += 32) dst[i] = x[i];
        }
    }
    if ((int)blockIdx.x >= active) return;   // CTA 0 of an idle split only wrote the cache
    __syncthreads();

    constexpr int NV = HD / 128;   // float4 output slices per lane
    float4 o[NV];
#pragma unroll
    for (int i = 0; i < NV; i++) o[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    float m = -INFINITY, l = 0.0f;
    const float *q = qn + warp * HD;
    const int key_lane = lane % KT, dpart = lane / KT;   // score phase: key and dimension part

    for (int t = 0; t < ntiles; t++) {
        const int buf = t & 1, kt = k0 + t * KT, nt = min(KT, k1 - kt);
        if (t + 1 < ntiles) {
            issue(t + 1, buf ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        float *Kb = Ks + buf * KT * KS, *Vb = Vs + buf * KT * HD;
        if (a.has_kv && p >= kt && p < kt + nt) {
            // the new key/value: use this CTA's copy (CTA 0 may still be writing the ring slot)
            const int r = p - kt;
            for (int i = threadIdx.x; i < HD; i += 256) {
                Kb[r * KS + i] = kn[i];
                Vb[r * HD + i] = vn[i];
            }
            __syncthreads();
        }
        // scores: LPK lanes per key, each over HD/LPK dimensions
        float s = -INFINITY;
        {
            const float *kr = Kb + key_lane * KS + dpart * (HD / LPK);
            const float *qq = q + dpart * (HD / LPK);
            float acc = 0.0f;
#pragma unroll 8
            for (int d = 0; d < HD / LPK; d += 4) {
                const float4 a4 = *(const float4 *)&qq[d], k4 = *(const float4 *)&kr[d];
                acc = fmaf(a4.x, k4.x, acc);
                acc = fmaf(a4.y, k4.y, acc);
                acc = fmaf(a4.z, k4.z, acc);
                acc = fmaf(a4.w, k4.w, acc);
            }
            if (LPK == 2) acc += __shfl_xor_sync(0xffffffffu, acc, 16);
            if (key_lane < nt) s = acc;
        }
        const float mt = warp_max(s);
        const float mn = fmaxf(m, mt);
        const float corr = (m == -INFINITY) ? 0.0f : expf(m - mn);
        const float pj = (key_lane < nt && dpart == 0) ? expf(s - mn) : 0.0f;
        l = l * corr + warp_sum(pj);
        m = mn;
#pragma unroll
        for (int i = 0; i < NV; i++) {
            o[i].x *= corr; o[i].y *= corr; o[i].z *= corr; o[i].w *= corr;
        }
        for (int jk = 0; jk < nt; jk++) {
            const float pk = __shfl_sync(0xffffffffu, pj, jk);
            const float *vr = Vb + jk * HD + 4 * lane;
#pragma unroll
            for (int i = 0; i < NV; i++) {
                const float4 vv = *(const float4 *)&vr[128 * i];
                o[i].x = fmaf(pk, vv.x, o[i].x);
                o[i].y = fmaf(pk, vv.y, o[i].y);
                o[i].z = fmaf(pk, vv.z, o[i].z);
                o[i].w = fmaf(pk, vv.w, o[i].w);
            }
        }
        __syncthreads();
    }
    float *part = a.part + ((size_t)blockIdx.x * kHeads + warp) * (HD + 4);
    if (lane == 0) {
        part[0] = m;
        part[1] = l;
    }
#pragma unroll
    for (int i = 0; i < NV; i++) *(float4 *)&part[4 + 4 * lane + 128 * i] = o[i];
}

// Combine the active split partials into the attention output and quantise it
// for o_proj (gemma4.c:459). grid = 8*HD/256 CTAs of 256 threads; thread = one
// output dimension.
template <int HD>
__global__ void __launch_bounds__(256) k_attn_combine(const AttnArgs a, int splits) {
    __shared__ float wsm[256];
    __shared__ float red[8];
    __shared__ float tot;
    griddep_launch();
    griddep_wait();
    const int p = a.pos_dev ? *a.pos_dev : a.start_pos;
    int k0, k1;
    const int active = split_range(p, a.window, splits, 0, &k0, &k1);
    const int per_head = HD / 256;
    const int h = blockIdx.x / per_head, d = (blockIdx.x % per_head) * 256 + threadIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t stride = (size_t)kHeads * (HD + 4);
    const float *ph = a.part + (size_t)h * (HD + 4);
    if (threadIdx.x == 0) {
        float mx = -INFINITY;
        for (int s = 0; s < active; s++) mx = fmaxf(mx, ph[s * stride]);
        float lsum = 0.0f;
        for (int s = 0; s < active; s++) {
            const float w = ph[s * stride] == -INFINITY ? 0.0f : expf(ph[s * stride] - mx);
            wsm[s] = w;
            lsum += w * ph[s * stride + 1];
        }
        tot = lsum;
    }
    __syncthreads();
    float o = 0.0f;
    for (int s = 0; s < active; s++) o = fmaf(wsm[s], ph[s * stride + 4 + d], o);
    o = o / tot;
    const int col = h * HD + d;
    a.out[col] = o;
    // dynamic int8 quantisation of the 64-wide group this thread belongs to
    float amax = warp_max(fabsf(o));
    if (lane == 0) red[warp] = amax;
    __syncthreads();
    amax = fmaxf(red[warp & ~1], red[warp | 1]);
    const float sc = quant_scale(amax), inv = quant_inv(sc);
    a.xq[col] = (int8_t)quant_one(o, inv);
    if ((threadIdx.x & 63) == 0) a.xs[col >> 6] = sc;
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
