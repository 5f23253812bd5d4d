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
// written to their ring slots. One warp per vector, kQkvWarps vectors per CTA
// (vector v: token v / W, which = v % W with W = heads [+2]).
constexpr int kQkvWarps = 8;
template <int HD>
__global__ void __launch_bounds__(32 * kQkvWarps) k_qkv_post(const AttnArgs a, int W) {
    __shared__ float xs_[kQkvWarps][HD];
    griddep_launch();
    griddep_wait();
    const int vi = blockIdx.x * kQkvWarps + (threadIdx.x >> 5);
    if (vi >= a.T * W) return;   // whole warps: the vector index is warp-uniform
    float *x = xs_[threadIdx.x >> 5];
    const int t = vi / W, which = vi - t * W;   // 0..7 q heads, 8 = k, 9 = v
    const int p = a.row_pos ? a.row_pos[t] : a.start_pos + t;
    const size_t so = a.row_seq ? (size_t)a.row_seq[t] * a.seq_stride : 0;
    float *src = a.qkv + (size_t)t * a.qkv_stride + which * HD;
    const int lane = threadIdx.x & 31;
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
    __shared__ float wsm[512 + 16];
    griddep_launch();
    griddep_wait();
    const int row = blockIdx.y, W = kHeads * HD;
    // with quant_out the rows are also quantised for o_proj (one 64-wide group per block)
    attn_combine_part<HD>(a, a.row_pos[row], blockIdx.x, splits, wsm,
                          a.part + (size_t)row * splits * kHeads * (HD + 4), a.out + (size_t)row * W,
                          a.quant_out ? a.xq + (size_t)row * W : nullptr,
                          a.quant_out ? a.xs + (size_t)row * (W / 64) : nullptr,
                          a.quant_out && a.xsT ? a.xsT + row : nullptr);
}

// ---------------------------------------------------------------------------
// Standalone decode kernels (one launch each) around the shared bodies.
template <int HD>
struct DecodeCfg {
    static constexpr int KT = DecodeKT<HD>::value;
    static constexpr size_t smem = (size_t)decode_smem_floats(HD, KT) * 4;
};
static_assert(DecodeCfg<256>::smem <= 227 * 1024 && DecodeCfg<512>::smem <= 227 * 1024,
              "shared memory budget of the decode / batch-row attention CTAs");

template <int HD>
__global__ void __launch_bounds__(256) k_attn_decode(const AttnArgs a, int splits) {
    extern __shared__ __align__(16) float sm[];
    griddep_launch();
    griddep_wait();
    attn_decode_split<HD, DecodeCfg<HD>::KT>(a, a.pos_dev ? *a.pos_dev : a.start_pos, blockIdx.x, splits, sm);
}

template <int HD>
__global__ void __launch_bounds__(256) k_attn_combine(const AttnArgs a, int splits) {
    __shared__ float wsm[512 + 16];
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
// Prefill attention (fast path): FP32 on the CUDA cores, register-tiled, with
// the chunk's work split evenly over a fixed grid.
//
// A q tile is QT consecutive tokens x 8 heads = R query rows; all R rows share
// the single KV head, so one staged key/value tile serves all of them. The
// keys a q tile needs ([first_key(first token), last token]) are cut into
// units of BK keys; units are numbered q-tile-major and CTA b of G takes units
// [U b / G, U (b+1) / G). A CTA that covers a whole q tile writes its output;
// one that covers part of it writes the partial (row max, row sum, unnormalised
// output) to a slot, and k_attn_prefill_merge combines the slots of such tiles
// in CTA order (deterministic for a given T, start_pos and G).
//
// Per key tile: S = Q K^T with each thread owning 4 rows x 4 keys over a slice
// of the head dimension (packed f32x2 FMAs over even/odd dimensions), the
// online-softmax update in registers (row max / sum by warp shuffles), P
// written to shared memory duplicated as (p, p) pairs, then O += P V with each
// thread owning 8 rows (one token's 8 heads) x 8 dimensions. K of the next
// tile loads (cp.async) during P V, V of this tile during Q K^T.
template <int HD> struct PreCfg;
template <> struct PreCfg<256> { static constexpr int QT = 8, BK = 64, DS = 1, KPAD = 4; };
template <> struct PreCfg<512> { static constexpr int QT = 4, BK = 32, DS = 4, KPAD = 16; };

constexpr int kPreMaxTiles = G4_BATCH / 4;   // q tiles of a chunk at QT >= 4

template <int HD>
struct Pre {
    static constexpr int QT = PreCfg<HD>::QT, BK = PreCfg<HD>::BK, DS = PreCfg<HD>::DS;
    static constexpr int R = QT * kHeads;              // query rows per q tile
    static constexpr int KS = HD + PreCfg<HD>::KPAD;   // K row stride (bank spread)
    static constexpr int KG = BK / 4;                  // key groups of the S phase
    static constexpr int DG = HD / 8;                  // dimension groups of the P V phase
    static constexpr int PS = 2 * R;                   // P row stride: R (p, p) pairs
    static_assert((R / 4) * KG * DS == 256, "S phase covers 256 threads");
    static_assert((R / 8) * DG == 256, "PV phase covers 256 threads");
    static constexpr int kFloats = R * HD + BK * KS + BK * HD + BK * PS + 3 * R;
    static constexpr size_t kSmem = (size_t)kFloats * 4 + (kPreMaxTiles + 4) * 4;
    // key-tile units of q tile j of a chunk of T tokens starting at sp
    static G4_DEV int units(int j, int T, int sp, int window) {
        const int t0 = j * QT, t1 = min(T, t0 + QT) - 1;
        const int klo = first_key(sp + t0, window), khi = sp + t1;
        return (khi - klo + BK) / BK;
    }
    // pre[0..nq] = prefix sums of units, by warp 0
    static G4_DEV void prefix(int *pre, int nq, int T, int sp, int window) {
        const int lane = threadIdx.x & 31;
        int carry = 0;
        if (lane == 0) pre[0] = 0;
        for (int base = 0; base < nq; base += 32) {
            const int j = base + lane;
            int v = j < nq ? units(j, T, sp, window) : 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= o) v += n;
            }
            if (j < nq) pre[j + 1] = carry + v;
            carry += __shfl_sync(0xffffffffu, v, 31);
        }
    }
    // the CTA whose unit range holds unit u
    static G4_DEV int cta_of(long long u, long long U, int G) { return (int)(((u + 1) * G + U - 1) / U) - 1; }
    // CTA b has no units (more CTAs than units)
    static G4_DEV bool empty(int b, long long U, int G) { return U * b / G == U * (b + 1) / G; }
    // partial slot of q tile j written by CTA b (first tile of b: 2b, else 2b + 1)
    static G4_DEV int slot_of(int b, int j, const int *pre, long long U, int G) {
        const long long s = U * b / G;
        return s >= pre[j] ? 2 * b : 2 * b + 1;
    }
};
static_assert(Pre<256>::kSmem <= 227 * 1024 && Pre<512>::kSmem <= 227 * 1024,
              "shared memory budget of the prefill attention CTA");

// Stage BK key rows [kt, kt + nt) of a ring into shared memory (row stride
// dstride); rows past nt are zero.
template <int HD>
G4_DEV void pre_load_rows(float *dst, int dstride, const float *cache, int mask, int kt, int nt) {
    constexpr int C4 = HD / 4, BK = Pre<HD>::BK;
    for (int idx = threadIdx.x; idx < BK * C4; idx += 256) {
        const int r = idx / C4, c4 = idx - r * C4;
        float *d = dst + r * dstride + c4 * 4;
        if (r < nt) cp_async16(d, cache + (size_t)((kt + r) & mask) * HD + c4 * 4);
        else *(float4 *)d = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    cp_async_commit();
}

template <int HD>
__global__ void __launch_bounds__(256, 1) k_attn_prefill(const AttnArgs a) {
    using P = Pre<HD>;
    constexpr int QT = P::QT, BK = P::BK, DS = P::DS, R = P::R, KS = P::KS, KG = P::KG, DG = P::DG, PS = P::PS;
    extern __shared__ __align__(16) float sm[];
    float *Qs = sm;                  // [R][HD]
    float *Ks = Qs + R * HD;         // [BK][KS]
    float *Vs = Ks + BK * KS;        // [BK][HD]
    float *Pt = Vs + BK * HD;        // [BK][R] (p, p) pairs, 16-byte columns swizzled by key
    float *rc = Pt + BK * PS;        // [R] correction of the current tile
    float *rl = rc + R;              // [R] running sum
    float *rm = rl + R;              // [R] running max
    int *pre = (int *)(rm + R);      // [nq + 1]

    griddep_launch();
    griddep_wait();
    const int tid = threadIdx.x, T = a.T, sp = a.start_pos;
    const int nq = (T + QT - 1) / QT;
    if (tid < 32) P::prefix(pre, nq, T, sp, a.window);
    __syncthreads();
    const long long U = pre[nq];
    const int G = gridDim.x, b = blockIdx.x;
    const long long u0 = U * b / G, u1 = U * (b + 1) / G;
    if (u0 >= u1) return;
    int j = 0;
    {
        int lo = 0, hi = nq - 1;   // largest j with pre[j] <= u0
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (pre[mid] <= u0) lo = mid; else hi = mid - 1;
        }
        j = lo;
    }
    const int j0 = j;

    // S-phase coordinates: rows 4 ty + i, keys tx + KG jj, dimension slice sl
    const int sl = tid % DS, tx = (tid / DS) % KG, ty = tid / (DS * KG);
    // P V coordinates: rows 8 rg + r (token rg of the tile, head r), dims 4 dg + {0, HD/2}
    const int rg = tid / DG, dg = tid % DG;

    long long u = u0;
    while (u < u1) {
        const int t0 = j * QT;
        const int seg_end = (int)min(u1, (long long)pre[j + 1]);
        const int n = seg_end - (int)u;
        const int klo = first_key(sp + t0, a.window), kend = sp + min(T, t0 + QT);
        const int kt0 = klo + ((int)u - pre[j]) * BK;
        // Q tile and the first K tile
        for (int idx = tid; idx < R * (HD / 4); idx += 256) {
            const int r = idx / (HD / 4), c4 = idx - r * (HD / 4);
            const int t = t0 + (r >> 3), h = r & 7;
            float *d = Qs + r * HD + c4 * 4;
            if (t < T) cp_async16(d, a.qkv + (size_t)t * a.qkv_stride + h * HD + c4 * 4);
            else *(float4 *)d = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        pre_load_rows<HD>(Ks, KS, a.kcache, a.mask, kt0, min(BK, kend - kt0));

        // this thread's S rows all belong to token t0 + (4 ty) / 8
        const int ts = t0 + ((4 * ty) >> 3);
        const int prow = ts < T ? sp + ts : -1;
        const int pfk = prow >= 0 ? first_key(prow, a.window) : 0;
        float mrow[4], lrow[4];
#pragma unroll
        for (int i = 0; i < 4; i++) { mrow[i] = -INFINITY; lrow[i] = 0.0f; }
        uint64_t o[8][4];
#pragma unroll
        for (int r = 0; r < 8; r++)
#pragma unroll
            for (int c = 0; c < 4; c++) o[r][c] = 0ull;

        for (int it = 0; it < n; it++) {
            const int kt = kt0 + it * BK;
            const int nt = min(BK, kend - kt);
            cp_async_wait<0>();
            __syncthreads();                       // Q, K(kt) visible; V, P free
            pre_load_rows<HD>(Vs, HD, a.vcache, a.mask, kt, nt);
            // ---- S = Q K^T over this thread's dimension slice
            uint64_t acc[4][4];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int jj = 0; jj < 4; jj++) acc[i][jj] = 0ull;
            const float *qb = Qs + (4 * ty) * HD, *kb = Ks + tx * KS;
#pragma unroll 4
            for (int c = sl; c < HD / 4; c += DS) {
                ulonglong2 qv[4], kv[4];
#pragma unroll
                for (int i = 0; i < 4; i++) qv[i] = *(const ulonglong2 *)(qb + i * HD + 4 * c);
#pragma unroll
                for (int jj = 0; jj < 4; jj++) kv[jj] = *(const ulonglong2 *)(kb + jj * KG * KS + 4 * c);
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int jj = 0; jj < 4; jj++) acc[i][jj] = fma2(qv[i].x, kv[jj].x, acc[i][jj]);
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int jj = 0; jj < 4; jj++) acc[i][jj] = fma2(qv[i].y, kv[jj].y, acc[i][jj]);
            }
            float s[4][4];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int jj = 0; jj < 4; jj++) {
                    const float2 v = upk(acc[i][jj]);
                    float x = v.x + v.y;
#pragma unroll
                    for (int off = 1; off < DS; off <<= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
                    const int key = kt + tx + KG * jj;
                    const bool ok = prow >= 0 && key < kend && key <= prow && key >= pfk;
                    s[i][jj] = ok ? x : -INFINITY;
                }
            // ---- online softmax (row state replicated over the row's key lanes)
            float corr[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                float mx = fmaxf(fmaxf(s[i][0], s[i][1]), fmaxf(s[i][2], s[i][3]));
#pragma unroll
                for (int off = DS; off < DS * KG; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
                const float mn = fmaxf(mrow[i], mx);
                corr[i] = mrow[i] == -INFINITY ? 0.0f : expf(mrow[i] - mn);
                float ps = 0.0f;
#pragma unroll
                for (int jj = 0; jj < 4; jj++) {
                    s[i][jj] = s[i][jj] == -INFINITY ? 0.0f : expf(s[i][jj] - mn);
                    ps += s[i][jj];
                }
#pragma unroll
                for (int off = DS; off < DS * KG; off <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
                lrow[i] = lrow[i] * corr[i] + ps;
                mrow[i] = mn;
            }
            if (tx == 0 && sl == 0) {
                *(float4 *)&rc[4 * ty] = make_float4(corr[0], corr[1], corr[2], corr[3]);
                *(float4 *)&rl[4 * ty] = make_float4(lrow[0], lrow[1], lrow[2], lrow[3]);
                *(float4 *)&rm[4 * ty] = make_float4(mrow[0], mrow[1], mrow[2], mrow[3]);
            }
#pragma unroll
            for (int jj = 0; jj < 4; jj++) {
                if (DS > 1 && jj != sl) continue;
                const int kl = tx + KG * jj;
                const int f = (tx * DS + jj) & 7;
                float *pr = Pt + kl * PS;
                *(float4 *)&pr[4 * ((2 * ty) ^ f)] = make_float4(s[0][jj], s[0][jj], s[1][jj], s[1][jj]);
                *(float4 *)&pr[4 * ((2 * ty + 1) ^ f)] = make_float4(s[2][jj], s[2][jj], s[3][jj], s[3][jj]);
            }
            cp_async_wait<0>();
            __syncthreads();                       // V, P, rc visible; K free
            if (it + 1 < n) pre_load_rows<HD>(Ks, KS, a.kcache, a.mask, kt + BK, min(BK, kend - kt - BK));
            // ---- O = O * corr + P V
            {
                const float4 c0 = *(const float4 *)&rc[8 * rg], c1 = *(const float4 *)&rc[8 * rg + 4];
                const float cr[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
                for (int r = 0; r < 8; r++) {
                    const uint64_t c2 = pk(cr[r], cr[r]);
#pragma unroll
                    for (int c = 0; c < 4; c++) o[r][c] = mul2(o[r][c], c2);
                }
            }
            const float *vb = Vs + 4 * dg;
#pragma unroll 4
            for (int k = 0; k < BK; k++) {
                const int f = ((k % KG) * DS + k / KG) & 7;
                const float *pr = Pt + k * PS;
                const ulonglong2 va = *(const ulonglong2 *)(vb + k * HD);
                const ulonglong2 vv = *(const ulonglong2 *)(vb + k * HD + HD / 2);
#pragma unroll
                for (int m = 0; m < 4; m++) {
                    const ulonglong2 pp = *(const ulonglong2 *)&pr[4 * ((4 * rg + m) ^ f)];
                    o[2 * m][0] = fma2(pp.x, va.x, o[2 * m][0]);
                    o[2 * m][1] = fma2(pp.x, va.y, o[2 * m][1]);
                    o[2 * m][2] = fma2(pp.x, vv.x, o[2 * m][2]);
                    o[2 * m][3] = fma2(pp.x, vv.y, o[2 * m][3]);
                    o[2 * m + 1][0] = fma2(pp.y, va.x, o[2 * m + 1][0]);
                    o[2 * m + 1][1] = fma2(pp.y, va.y, o[2 * m + 1][1]);
                    o[2 * m + 1][2] = fma2(pp.y, vv.x, o[2 * m + 1][2]);
                    o[2 * m + 1][3] = fma2(pp.y, vv.y, o[2 * m + 1][3]);
                }
            }
        }
        // ---- emit: whole q tile -> output rows; part of it -> partial slot
        const int t = t0 + rg;
        const bool whole = (int)u == pre[j] && seg_end == pre[j + 1];
        if (whole) {
            if (t < T) {   // warp-uniform: the warp's lanes share rg
                constexpr int K = kHeads * HD;
                float *dst = a.out + (size_t)t * K + 4 * dg;
#pragma unroll
                for (int r = 0; r < 8; r++) {
                    const float inv = 1.0f / rl[8 * rg + r];
                    const uint64_t i2 = pk(inv, inv);
                    const float2 x0 = upk(mul2(o[r][0], i2)), x1 = upk(mul2(o[r][1], i2));
                    const float2 y0 = upk(mul2(o[r][2], i2)), y1 = upk(mul2(o[r][3], i2));
                    const float4 va = make_float4(x0.x, x0.y, x1.x, x1.y), vb = make_float4(y0.x, y0.y, y1.x, y1.y);
                    *(float4 *)&dst[r * HD] = va;
                    *(float4 *)&dst[r * HD + HD / 2] = vb;
                    if (a.quant_out) {
                        const int ca = r * HD + 4 * dg, cb2 = ca + HD / 2;   // row columns of va, vb
                        quant_lanes16(va, a.xq + (size_t)t * K + ca, a.xs + (size_t)t * (K / 64) + ca / 64,
                                      a.xsT ? a.xsT + (size_t)(ca / 64) * G4_XST_STRIDE + t : nullptr, (dg & 15) == 0);
                        quant_lanes16(vb, a.xq + (size_t)t * K + cb2, a.xs + (size_t)t * (K / 64) + cb2 / 64,
                                      a.xsT ? a.xsT + (size_t)(cb2 / 64) * G4_XST_STRIDE + t : nullptr,
                                      (dg & 15) == 0);
                    }
                }
            }
        } else {
            const int slot = j == j0 ? 2 * b : 2 * b + 1;
            float *ps = a.pre_part + (size_t)slot * G4_PRE_PART_SLOT;
#pragma unroll
            for (int r = 0; r < 8; r++) {
                float *dst = ps + (size_t)(8 * rg + r) * HD + 4 * dg;
                const float2 x0 = upk(o[r][0]), x1 = upk(o[r][1]), y0 = upk(o[r][2]), y1 = upk(o[r][3]);
                *(float4 *)&dst[0] = make_float4(x0.x, x0.y, x1.x, x1.y);
                *(float4 *)&dst[HD / 2] = make_float4(y0.x, y0.y, y1.x, y1.y);
            }
            if (dg == 0)
#pragma unroll
                for (int r = 0; r < 8; r++) {
                    ps[R * HD + 8 * rg + r] = rm[8 * rg + r];
                    ps[R * HD + R + 8 * rg + r] = rl[8 * rg + r];
                }
        }
        u = seg_end;
        j++;
    }
}

// Combine the partial slots of q tiles that k_attn_prefill split over CTAs
// (max-rescaled sums, slots in CTA order). grid (q tiles, tokens per tile):
// CTA (j, y) merges the 8 head rows of token y of q tile j.
constexpr int kMergeMaxSlots = 256;

template <int HD>
__global__ void __launch_bounds__(256) k_attn_prefill_merge(const AttnArgs a) {
    using P = Pre<HD>;
    constexpr int QT = P::QT, R = P::R;
    __shared__ int pre[kPreMaxTiles + 4];
    __shared__ int slots[kMergeMaxSlots];
    __shared__ float wgt[kHeads][kMergeMaxSlots];
    __shared__ int nslots;
    griddep_launch();
    griddep_wait();
    const int T = a.T, nq = (T + QT - 1) / QT, j = blockIdx.x, tok = j * QT + blockIdx.y;
    if (tok >= T) return;
    const int tid = threadIdx.x;
    if (tid < 32) P::prefix(pre, nq, T, a.start_pos, a.window);
    __syncthreads();
    const long long U = pre[nq];
    const int G = a.pre_ctas;
    const int bf = P::cta_of(pre[j], U, G), bl = P::cta_of(pre[j + 1] - 1, U, G);
    if (bf == bl) return;
    if (tid == 0) {
        int n = 0;
        for (int bb = bf; bb <= bl && n < kMergeMaxSlots; bb++)
            if (!P::empty(bb, U, G)) slots[n++] = P::slot_of(bb, j, pre, U, G);
        nslots = n;
    }
    __syncthreads();
    const int ns = nslots, row0 = 8 * blockIdx.y;   // tile rows of this token
    // per head: weights exp(m_s - max) / sum_s l_s exp(m_s - max); warp h = head h
    {
        const int h = tid >> 5, lane = tid & 31;
        float mx = -INFINITY;
        for (int si = lane; si < ns; si += 32)
            mx = fmaxf(mx, a.pre_part[(size_t)slots[si] * G4_PRE_PART_SLOT + R * HD + row0 + h]);
        mx = warp_max(mx);
        float l = 0.0f;
        for (int si = lane; si < ns; si += 32) {
            const float *ps = a.pre_part + (size_t)slots[si] * G4_PRE_PART_SLOT;
            const float m = ps[R * HD + row0 + h];
            const float w = m == -INFINITY ? 0.0f : expf(m - mx);
            wgt[h][si] = w;
            l = fmaf(ps[R * HD + R + row0 + h], w, l);
        }
        l = warp_sum(l);
        const float inv = 1.0f / l;
        __syncwarp();
        for (int si = lane; si < ns; si += 32) wgt[h][si] *= inv;
    }
    __syncthreads();
    for (int idx = tid; idx < kHeads * HD / 4; idx += 256) {
        const int h = idx / (HD / 4), c4 = idx - h * (HD / 4);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int si = 0; si < ns; si++) {
            const float w = wgt[h][si];
            const float4 v = *(const float4 *)&a.pre_part[(size_t)slots[si] * G4_PRE_PART_SLOT +
                                                         (size_t)(row0 + h) * HD + c4 * 4];
            acc.x = fmaf(v.x, w, acc.x);
            acc.y = fmaf(v.y, w, acc.y);
            acc.z = fmaf(v.z, w, acc.z);
            acc.w = fmaf(v.w, w, acc.w);
        }
        *(float4 *)&a.out[(size_t)tok * (kHeads * HD) + h * HD + c4 * 4] = acc;
        if (a.quant_out) {   // idx runs in whole warps: 16 consecutive lanes hold one 64-wide group
            constexpr int K = kHeads * HD;
            const int col = h * HD + c4 * 4;
            quant_lanes16(acc, a.xq + (size_t)tok * K + col, a.xs + (size_t)tok * (K / 64) + col / 64,
                          a.xsT ? a.xsT + (size_t)(col / 64) * G4_XST_STRIDE + tok : nullptr, (c4 & 15) == 0);
        }
    }
}

// Host copy of the unit schedule: does any q tile span more than one CTA?
template <int HD>
bool prefill_needs_merge(const AttnArgs &a) {
    using P = Pre<HD>;
    const int nq = (a.T + P::QT - 1) / P::QT;
    int pre[kPreMaxTiles + 1];
    pre[0] = 0;
    for (int j = 0; j < nq; j++) {
        const int t0 = j * P::QT, t1 = (a.T < t0 + P::QT ? a.T : t0 + P::QT) - 1;
        const int pf = a.start_pos + t0;
        const int klo = (a.window && pf + 1 > a.window) ? pf + 1 - a.window : 0;
        pre[j + 1] = pre[j] + (a.start_pos + t1 - klo + P::BK) / P::BK;
    }
    const long long U = pre[nq];
    const int G = a.pre_ctas;
    auto cta_of = [&](long long u) { return (int)(((u + 1) * G + U - 1) / U) - 1; };
    for (int j = 0; j < nq; j++)
        if (cta_of(pre[j]) != cta_of(pre[j + 1] - 1)) return true;
    return false;
}

template <int HD>
cudaError_t launch_prefill(const AttnArgs &a, cudaStream_t st, bool pdl) {
    {
        cudaError_t e = g4_smem_optin((const void *)k_attn_prefill<HD>, (int)Pre<HD>::kSmem);
        if (e) return e;
    }
    cudaError_t e = g4_launch(k_attn_prefill<HD>, dim3(a.pre_ctas), dim3(256), Pre<HD>::kSmem, st, pdl, a);
    if (e || !prefill_needs_merge<HD>(a)) return e;
    const int nq = (a.T + Pre<HD>::QT - 1) / Pre<HD>::QT;
    return g4_launch(k_attn_prefill_merge<HD>, dim3(nq, Pre<HD>::QT), dim3(256), 0, st, pdl, a);
}

}  // namespace

cudaError_t g4_launch_qkv_post(const AttnArgs &a, cudaStream_t st, bool pdl) {
    const int W = kHeads + (a.has_kv ? 2 : 0);
    const dim3 grid((a.T * W + kQkvWarps - 1) / kQkvWarps), block(32 * kQkvWarps);
    if (a.hd == 256) return g4_launch(k_qkv_post<256>, grid, block, 0, st, pdl, a, W);
    if (a.hd == 512) return g4_launch(k_qkv_post<512>, grid, block, 0, st, pdl, a, W);
    return cudaErrorInvalidValue;
}

cudaError_t g4_launch_attn_decode(const AttnArgs &a, int splits, cudaStream_t st, bool pdl) {
    if (splits < 1 || splits > 256) return cudaErrorInvalidValue;
    if (a.hd == 256) {
        const size_t smem = DecodeCfg<256>::smem;
        { cudaError_t e = g4_smem_optin((const void *)k_attn_decode<256>, (int)smem); if (e) return e; }
        return g4_launch(k_attn_decode<256>, dim3(splits), dim3(256), smem, st, pdl, a, splits);
    }
    if (a.hd == 512) {
        const size_t smem = DecodeCfg<512>::smem;
        { cudaError_t e = g4_smem_optin((const void *)k_attn_decode<512>, (int)smem); if (e) return e; }
        return g4_launch(k_attn_decode<512>, dim3(splits), dim3(256), smem, st, pdl, a, splits);
    }
    return cudaErrorInvalidValue;
}

cudaError_t g4_launch_attn_rows(const AttnArgs &a, int splits, cudaStream_t st, bool pdl) {
    if (splits < 1 || splits > 256 || a.T < 1 || !a.row_seq || !a.row_pos) return cudaErrorInvalidValue;
    const dim3 gs(splits, a.T), gc(kHeads * a.hd / kCombineDims, a.T);
    if (a.hd == 256) {
        const size_t smem = DecodeCfg<256>::smem;
        { cudaError_t e = g4_smem_optin((const void *)k_attn_rows<256>, (int)smem); if (e) return e; }
        cudaError_t e = g4_launch(k_attn_rows<256>, gs, dim3(256), smem, st, pdl, a, splits);
        return e ? e : g4_launch(k_attn_rows_combine<256>, gc, dim3(256), 0, st, pdl, a, splits);
    }
    if (a.hd == 512) {
        const size_t smem = DecodeCfg<512>::smem;
        { cudaError_t e = g4_smem_optin((const void *)k_attn_rows<512>, (int)smem); if (e) return e; }
        cudaError_t e = g4_launch(k_attn_rows<512>, gs, dim3(256), smem, st, pdl, a, splits);
        return e ? e : g4_launch(k_attn_rows_combine<512>, gc, dim3(256), 0, st, pdl, a, splits);
    }
    return cudaErrorInvalidValue;
}

cudaError_t g4_launch_attn_combine(const AttnArgs &a, int splits, cudaStream_t st, bool pdl) {
    if (splits < 1 || splits > 256) return cudaErrorInvalidValue;
    const int grid = kHeads * a.hd / kCombineDims;
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
    if (a.T < 1 || a.T > G4_BATCH || !a.pre_part || a.pre_ctas < 1 || a.pre_ctas > kMergeMaxSlots)
        return cudaErrorInvalidValue;
    if (a.hd == 256) return launch_prefill<256>(a, st, pdl);
    if (a.hd == 512) return launch_prefill<512>(a, st, pdl);
    return cudaErrorInvalidValue;
}
