// g4_attn_dev.cuh — attention device building blocks shared by the
// standalone attention kernels (g4_attn.cu) and the persistent decode kernel
// (g4_decode.cu).
//
// Reference: attention (gemma4.c:411-461), attention_scores (:281-294),
// softmax (:400-408), weighted_value_sum (:296-307), rmsnorm of q/k/v
// (:427,437,439) and apply_rope (:381-398).
#pragma once
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


// Quantise (gemma4.c:265-279) one 64-wide group held as 4 values in each of 16
// consecutive lanes: the group's max |x| over the 16 lanes, then scale and
// rounded int8 values exactly as quantize(). All 32 lanes must call it.
G4_DEV void quant_lanes16(float4 v, int8_t *q, float *xs, float *xsT, bool leader) {
    float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    const float sc = quant_scale(m), inv = quant_inv(sc);
    *(char4 *)q = make_char4((signed char)quant_one(v.x, inv), (signed char)quant_one(v.y, inv),
                             (signed char)quant_one(v.z, inv), (signed char)quant_one(v.w, inv));
    if (leader) {
        *xs = sc;
        if (xsT) *xsT = sc;
    }
}

constexpr int kMinSplit = 8;
constexpr int kAttnThreads = 256;   // 8 warps: warp h owns query head h

G4_DEV void attn_sync() { bar_sync(1, kAttnThreads); }

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
    per = per < kMinSplit ? kMinSplit : (per + 7) / 8 * 8;
    *k0 = kf + s * per;
    *k1 = min(p + 1, *k0 + per);
    return (nk + per - 1) / per;
}

// Keys per decode tile. The standalone decode kernel and the persistent decode
// kernel use the same tile so that both give the same bits (the score lanes per
// key and the online-softmax tile steps follow KT).
template <int HD>
struct DecodeKT {
    static constexpr int value = HD == 512 ? 4 : 8;
};

// RMS-normalise (optional weight) and rotate one head vector held in
// registers by one warp: lane holds x[lane + 32 i], i < HD/32, so each rope
// pair (j, j + HD/2) sits in one lane. The weight, cos and sin loads are issued
// before any arithmetic so that they share one memory round trip with the
// caller's loads of v.
template <int HD>
G4_DEV void norm_rope_regs(float (&v)[HD / 32], const float *w, const float *cosr, const float *sinr, int pairs,
                           bool rope) {
    constexpr int NI = HD / 32, NP = HD / 64;
    const int lane = threadIdx.x & 31;
    float wv[NI], cv[NP], sv[NP];
#pragma unroll
    for (int i = 0; i < NI; i++) wv[i] = w ? w[lane + 32 * i] : 1.0f;
#pragma unroll
    for (int i = 0; i < NP; i++) {
        const int jj = lane + 32 * i;
        const bool on = rope && jj < pairs;
        cv[i] = on ? cosr[jj] : 1.0f;
        sv[i] = on ? sinr[jj] : 0.0f;
    }
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < NI; i++) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
    ss = warp_sum(ss);
    const float inv = rms_inv(ss, (float)HD, 1e-6f);
#pragma unroll
    for (int i = 0; i < NI; i++) v[i] = rms_apply(v[i], inv, wv[i]);
    if (rope) {
#pragma unroll
        for (int i = 0; i < NP; i++) {
            if (lane + 32 * i < pairs) {
                const float a0 = v[i], b0 = v[i + NP];
                v[i] = __fsub_rn(__fmul_rn(a0, cv[i]), __fmul_rn(b0, sv[i]));
                v[i + NP] = __fadd_rn(__fmul_rn(b0, cv[i]), __fmul_rn(a0, sv[i]));
            }
        }
    }
}

// Shared-memory floats of one decode split with KT-key tiles (double buffered).
// K tile row stride of the decode split: key rows land 4 (hd 256, 8 lanes per
// key phase) or 8 (hd 512, lanes of 4 keys x 2 dimension parts) banks apart, so
// the score phase's 16-byte loads are free of bank conflicts.
__host__ __device__ constexpr int dec_ks(int hd) { return hd == 512 ? hd + 8 : hd + 4; }

__host__ __device__ constexpr int decode_smem_floats(int hd, int kt) {
    return kHeads * hd + 2 * hd + 2 * kt * dec_ks(hd) + 2 * kt * hd;
}

// Decode (T = 1) split-KV attention at position p for split `split` of `splits`, run by 256
// threads (8 warps; warp h = query head h). The CTA post-processes q (all
// heads) and, on layers that own the cache, the new k/v; CTA 0 of the grid
// writes k/v to the ring, and every CTA uses its own copy for key == pos.
// K/V tiles of KT keys stream through a double-buffered cp.async pipeline.
// Writes (max, sum, unnormalised output) per head to a.part.
template <int HD, int KT>
__device__ __noinline__ void attn_decode_split(const AttnArgs &a, int p, int split, int splits, float *sm);

// The tile loop of one split: keys [k0, k1) of the ring (kc, vc) against the 8
// query heads in qn[8][HD] (shared), one warp per head. When `kn` is given,
// key `p` is taken from kn/vn (this CTA's own copy of the new key and value)
// instead of the ring. Writes (max, sum, unnormalised output) per head to part.
// first_issued: the caller already issued (and committed) tile 0 into buffer 0.
template <int HD, int KT>
G4_DEV void attn_split_core(const AttnArgs &a, const float *kc, const float *vc, int p, int k0, int k1,
                            const float *qn, const float *kn, const float *vn, float *Ks, float *Vs, float *part_base,
                            bool first_issued) {
    constexpr int LPK = 32 / KT, KS = dec_ks(HD), QC = HD / (4 * LPK);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    auto issue = [&](int tile, int buf) {
        const int kt = k0 + tile * KT, nt = min(KT, k1 - kt);
        for (int idx = tid; idx < nt * (HD / 4); idx += kAttnThreads) {
            const int r = idx / (HD / 4), c4 = idx - r * (HD / 4);
            const size_t slot = (size_t)((kt + r) & a.mask) * HD;
            cp_async16(&Ks[(buf * KT + r) * KS + c4 * 4], kc + slot + c4 * 4);
            cp_async16(&Vs[(buf * KT + r) * HD + c4 * 4], vc + slot + c4 * 4);
        }
        cp_async_commit();
    };
    const int ntiles = k1 > k0 ? (k1 - k0 + KT - 1) / KT : 0;
    if (ntiles > 0 && !first_issued) issue(0, 0);

    constexpr int NV = HD / 128;   // float4 output slices per lane
    float4 o[NV];
#pragma unroll
    for (int i = 0; i < NV; i++) o[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    float m = -INFINITY, l = 0.0f;
    const int key_lane = lane % KT, dpart = lane / KT;   // score phase: key and dimension part
    // this lane's query slice (16-byte chunks dpart, dpart + LPK, ...) stays in
    // registers for the whole split
    float4 qr[QC];
#pragma unroll
    for (int j = 0; j < QC; j++) qr[j] = *(const float4 *)&qn[warp * HD + 4 * (dpart + LPK * j)];

    for (int t = 0; t < ntiles; t++) {
        const int buf = t & 1, kt = k0 + t * KT, nt = min(KT, k1 - kt);
        if (t + 1 < ntiles) {
            issue(t + 1, buf ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        attn_sync();
        float *Kb = Ks + buf * KT * KS, *Vb = Vs + buf * KT * HD;
        if (kn && p >= kt && p < kt + nt) {
            // the new key/value: this CTA's copy (CTA 0 may still be writing the ring slot)
            const int r = p - kt;
            for (int i = tid; i < HD; i += kAttnThreads) {
                Kb[r * KS + i] = kn[i];
                Vb[r * HD + i] = vn[i];
            }
            attn_sync();
        }
        float s = -INFINITY;
        {
            const float *kr = Kb + key_lane * KS + 4 * dpart;
            float acc = 0.0f;
#pragma unroll
            for (int j = 0; j < QC; j++) {
                const float4 a4 = qr[j], k4 = *(const float4 *)&kr[4 * LPK * j];
                acc = fmaf(a4.x, k4.x, acc);
                acc = fmaf(a4.y, k4.y, acc);
                acc = fmaf(a4.z, k4.z, acc);
                acc = fmaf(a4.w, k4.w, acc);
            }
#pragma unroll
            for (int off = KT; off < 32; off <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
            if (key_lane < nt) s = acc;
        }
        // the tile's KT scores sit in lanes differing in their low log2(KT) bits, so
        // the reductions need only those levels (the dropped levels of the full
        // butterfly take maxima of equal values and add zeros: same bits)
        float mt = s;
#pragma unroll
        for (int off = KT / 2; off >= 1; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
        const float mn = fmaxf(m, mt);
        const float corr = (m == -INFINITY) ? 0.0f : expf(m - mn);
        const float pj = (key_lane < nt && dpart == 0) ? expf(s - mn) : 0.0f;
        float ps = pj;   // nonzero in lanes 0 .. KT-1 only; lane 0's sum is the one kept
#pragma unroll
        for (int off = KT / 2; off >= 1; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
        l = l * corr + ps;
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
        attn_sync();
    }
    float *part = part_base + (size_t)warp * (HD + 4);
    if (lane == 0) {
        part[0] = m;
        part[1] = l;
    }
#pragma unroll
    for (int i = 0; i < NV; i++) *(float4 *)&part[4 + 4 * lane + 128 * i] = o[i];
}

// Decode (T = 1) split-KV attention at position p for split `split` of `splits`, run by 256
// threads (8 warps; warp h = query head h). The CTA post-processes q (all
// heads) and, on layers that own the cache, the new k/v; CTA 0 of the grid
// writes k/v to the ring, and every CTA uses its own copy for key == pos.
// K/V tiles of KT keys stream through a double-buffered cp.async pipeline.
// Writes (max, sum, unnormalised output) per head to a.part.
template <int HD, int KT>
__device__ __noinline__ void attn_decode_split(const AttnArgs &a, int p, int split, int splits, float *sm) {
    float *qn = sm;                       // [8][HD]
    float *kn = qn + kHeads * HD;         // [HD]
    float *vn = kn + HD;                  // [HD]
    float *Ks = vn + HD;                  // [2][KT][dec_ks(HD)]
    float *Vs = Ks + 2 * KT * dec_ks(HD); // [2][KT][HD]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int k0, k1;
    const int active = split_range(p, a.window, splits, split, &k0, &k1);
    if (split >= active) return;
    // first K/V tile in flight while q, k and v are prepared
    {
        const int nt = min(KT, k1 - k0);
        for (int idx = tid; idx < nt * (HD / 4); idx += kAttnThreads) {
            const int r = idx / (HD / 4), c4 = idx - r * (HD / 4);
            const size_t slot = (size_t)((k0 + r) & a.mask) * HD;
            cp_async16(&Ks[r * dec_ks(HD) + c4 * 4], a.kcache + slot + c4 * 4);
            cp_async16(&Vs[r * HD + c4 * 4], a.vcache + slot + c4 * 4);
        }
        cp_async_commit();
    }

    // q of head `warp`; k and v (warps 0, 1) when the layer owns its cache. All
    // loads first, then the per-warp norm + rope in registers.
    constexpr int NI = HD / 32;
    const float *cosr = a.rope_cos + (size_t)p * a.pairs, *sinr = a.rope_sin + (size_t)p * a.pairs;
    const bool kv = a.has_kv && warp < 2;
    float qv[NI], kvv[NI];
#pragma unroll
    for (int i = 0; i < NI; i++) {
        qv[i] = a.qkv[warp * HD + lane + 32 * i];
        kvv[i] = kv ? a.qkv[(kHeads + warp) * HD + lane + 32 * i] : 0.0f;
    }
    norm_rope_regs<HD>(qv, a.q_norm, cosr, sinr, a.pairs, true);
#pragma unroll
    for (int i = 0; i < NI; i++) qn[warp * HD + lane + 32 * i] = qv[i];
    if (kv) {
        norm_rope_regs<HD>(kvv, warp == 0 ? a.k_norm : nullptr, cosr, sinr, a.pairs, warp == 0);
        float *x = warp == 0 ? kn : vn;
        float *dst = (warp == 0 ? a.kcache : a.vcache) + (size_t)(p & a.mask) * HD;
#pragma unroll
        for (int i = 0; i < NI; i++) {
            x[lane + 32 * i] = kvv[i];
            if (split == 0) dst[lane + 32 * i] = kvv[i];
        }
    }
    attn_sync();
    attn_split_core<HD, KT>(a, a.kcache, a.vcache, p, k0, k1, qn, a.has_kv ? kn : nullptr, vn, Ks, Vs,
                            a.part + (size_t)split * kHeads * (HD + 4), true);
}

// Row-batched decode attention (g4_forward_batch): row `row` of a batch, its
// sequence's ring and position from a.row_seq / a.row_pos; q already normalised
// and rotated in a.qkv and the new k/v already in the ring (k_qkv_post).
template <int HD, int KT>
G4_DEV void attn_rows_split(const AttnArgs &a, int row, int split, int splits, float *sm) {
    float *qn = sm;                       // [8][HD]
    float *Ks = qn + kHeads * HD + 2 * HD;
    float *Vs = Ks + 2 * KT * dec_ks(HD);
    const int tid = threadIdx.x;
    const int p = a.row_pos[row];
    const size_t so = (size_t)a.row_seq[row] * a.seq_stride;
    int k0, k1;
    const int active = split_range(p, a.window, splits, split, &k0, &k1);
    if (split >= active) return;
    const float *q = a.qkv + (size_t)row * a.qkv_stride;
    for (int i = tid; i < kHeads * HD / 4; i += kAttnThreads) ((float4 *)qn)[i] = ((const float4 *)q)[i];
    attn_sync();
    attn_split_core<HD, KT>(a, a.kcache + so, a.vcache + so, p, k0, k1, qn, nullptr, nullptr, Ks, Vs,
                            a.part + ((size_t)row * splits + split) * kHeads * (HD + 4), false);
}

// Combine the active split partials (part_base: [splits][8][HD + 4]) into the
// attention output out[8*HD] for 64 output dimensions (combine block `blk` of
// 8*HD/64) and, when xq is given, quantise them for o_proj (gemma4.c:459): the
// block is exactly one 64-wide quantisation group. 256 threads = 64 dimensions
// x 4 slices of the splits (slice q takes splits q, q + 4, ...); each slice's
// weighted sum runs over its splits in ascending order and the four are added
// in slice order, so the result does not depend on timing.
// smem: 256 (split weights) + 256 (slice sums) + 16 floats.
constexpr int kCombineDims = 64;
template <int HD>
__device__ __noinline__ void attn_combine_part(const AttnArgs &a, int p, int blk, int splits, float *wsm,
                                               const float *part_base, float *out, int8_t *xq, float *xs,
                                               float *xsT = nullptr) {
    float *psum = wsm + 256, *red = wsm + 512;
    const int tid = threadIdx.x;
    int k0, k1;
    const int active = split_range(p, a.window, splits, 0, &k0, &k1);
    const int col0 = blk * kCombineDims, h = col0 / HD;
    const int dl = tid & (kCombineDims - 1), sl = tid >> 6, d = col0 % HD + dl;
    const int warp = tid >> 5, lane = tid & 31;
    const size_t stride = (size_t)kHeads * (HD + 4);
    const float *ph = part_base + (size_t)h * (HD + 4);
    // this thread's values of its first splits are loaded before the weights
    // exist, so that both loads share one memory round trip
    constexpr int U = 16;
    float pv[U];
#pragma unroll
    for (int u = 0; u < U; u++) pv[u] = sl + 4 * u < active ? ph[(sl + 4 * u) * stride + 4 + d] : 0.0f;
    if (warp == 0) {
        // split weights exp(m_s - max) and the total sum, lanes over splits (active <= 256)
        float mx = -INFINITY;
        for (int s = lane; s < active; s += 32) mx = fmaxf(mx, ph[s * stride]);
        mx = warp_max(mx);
        float lsum = 0.0f;
        for (int s = lane; s < active; s += 32) {
            const float ms = ph[s * stride];
            const float w = ms == -INFINITY ? 0.0f : expf(ms - mx);
            wsm[s] = w;
            lsum = fmaf(w, ph[s * stride + 1], lsum);
        }
        lsum = warp_sum(lsum);
        if (lane == 0) red[8] = lsum;
    }
    attn_sync();
    float o = 0.0f;   // this slice's splits in ascending order
    for (int u0 = 0; sl + 4 * u0 < active; u0 += U) {
        if (u0 > 0) {
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int s = sl + 4 * (u0 + u);
                pv[u] = s < active ? ph[s * stride + 4 + d] : 0.0f;
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int s = sl + 4 * (u0 + u);
            if (s < active) o = fmaf(wsm[s], pv[u], o);
        }
    }
    psum[sl * kCombineDims + dl] = o;
    attn_sync();
    if (tid < kCombineDims) {
        o = __fadd_rn(__fadd_rn(__fadd_rn(psum[dl], psum[kCombineDims + dl]), psum[2 * kCombineDims + dl]),
                      psum[3 * kCombineDims + dl]) /
            red[8];
        out[col0 + dl] = o;
        if (xq) {
            const float amax = warp_max(fabsf(o));
            if (lane == 0) red[warp] = amax;
        }
    }
    if (!xq) {
        attn_sync();   // wsm / red are reused by the caller's next combine
        return;
    }
    attn_sync();
    if (tid < kCombineDims) {
        const float sc = quant_scale(fmaxf(red[0], red[1])), inv = quant_inv(sc);
        xq[col0 + dl] = (int8_t)quant_one(o, inv);
        if (tid == 0) {
            xs[col0 >> 6] = sc;
            if (xsT) xsT[(size_t)(col0 >> 6) * G4_XST_STRIDE] = sc;   // group-major copy (GEMM operand)
        }
    }
    attn_sync();
}

}  // namespace
