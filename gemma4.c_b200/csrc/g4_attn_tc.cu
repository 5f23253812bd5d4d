// g4_attn_tc.cu — prefill attention on the 5th-generation tensor cores.
//
// Reference: attention (gemma4.c:411-461) for a chunk of T tokens: per query
// head, unscaled scores q.k over the visible keys (attention_scores,
// :281-294), softmax (:400-408) and the probability-weighted sum of the values
// (weighted_value_sum, :296-307). Same semantics as the CUDA-core kernel of
// g4_attn.cu (8 query heads on one KV head, causal, sliding window on the
// 256-wide layers), different floating-point order: outputs agree within fp32
// rounding, not bit for bit.
//
// Both contractions are tcgen05.mma kind::f16 on split operands: every fp32
// operand x is scaled by an exact power of two c (so |x c| < 2^15) and stored
// as hi = fp16(x c) and lo = fp16(x c - hi), round to nearest; each K step
// issues hi.hi into one fp32 TMEM accumulator and hi.lo + lo.hi into a second
// one (the accumulators add with rounding toward zero at their own magnitude,
// so the 2^-11 smaller correction products get their own), and the epilogue
// adds the two and removes the scales. 22 significant bits per operand: the
// dropped lo.lo term and the roundings leave a relative error near 2^-21 per
// product (an fp32 FMA: 2^-24). Scales: per row for Q and K (from the row's
// max |x|: q/k norm weights are unbounded), 2^15 for P (0 < p <= 1) and a
// fixed 2^(15 - ceil(log2 sqrt(HD))) for V (RMS-normalised without a weight,
// so |v| <= sqrt(HD)).
//
// The chunk's R = 8T query rows (row r = token r / 8, head r % 8) form 128-row
// tiles of 16 tokens. Five launches (four for short chunks, see 4):
//   1. k_tc_split   Q rows, the chunk's keys [kbase, npos) and their values as
//                   scaled fp16 hi/lo pairs (with the Q and K row scales); V
//                   transposed to [HD][keys] so that both GEMMs read K-major
//                   tiles;
//   2. k_tc_gemm<0> S = Q K^T per 128-row x 256-key tile (K = HD), only tiles
//                   that hold a visible key; the epilogue stores S tile-major
//                   ([row tile][key tile][key][row]: each warp store is 128
//                   contiguous bytes) and every row's max over the visible keys
//                   of each 128-key half tile;
//   3. k_tc_rowmax  per row: m = the max of its half-tile maxima;
//   4. k_tc_gemm<1> O = P V per 128-row x 256-dim tile; the K stages of all
//                   (row tile, dimension tile) pairs, in order, are cut into
//                   one even run per CTA (a CTA's run may end or start inside
//                   a pair: split K, balanced to one stage): each
//                   stage's S block (32 keys x 128 rows, one bulk copy) becomes
//                   p = exp(s - m) on visible keys (0 elsewhere) as scaled fp16
//                   hi/lo A tiles in shared memory, in place, by the epilogue
//                   warps (2^(s log2 e - m log2 e) by the hardware ex2
//                   approximation, relative error ~1e-6; fp16 pairs by packed
//                   conversions); partial O tiles and partial sums l = sum p
//                   stored per (pair, CTA) slot. Short chunks (at most 24
//                   stages per pair on average) run one CTA per pair instead,
//                   which divides by l and quantises its rows itself (no
//                   slots, no step 5);
//   5. k_tc_out     O = (sum of the slots, in CTA order) / l per token, stored and
//                   quantised for o_proj (gemma4.c:459).
// A layer that reads another layer's KV cache can reuse that layer's K/V
// split of the chunk (AttnArgs::reuse_kv): step 1 then splits only Q.
// The schedule depends only on (T, start position, SM count): deterministic.
//
// GEMM roles (10 warps, one CTA per SM, persistent over units):
//   warp 0      TMA producer: per stage the 32-wide K slice of A hi/lo (128
//               rows; for O the raw S block instead) and B hi/lo (256 rows)
//               with the 64-byte swizzle, four stages of 48 KB in flight;
//   warp 1      allocates 512 TMEM columns (the hi.hi and the correction
//               accumulator, 256 columns each); one lane issues 3 x 2 MMAs
//               (M 128, N 256, K 16) per stage;
//   warps 2-9   epilogue: thread = row (TMEM lane), two warps per lane quadrant
//               with 128 columns each; for O also the per-stage transform of S
//               into P, by two groups of four warps on alternate stages
//               (thread = row x the stage's 32 keys).
// Waits are bounded (mbar_wait); on a timeout every role leaves its loop, the
// CTA waits (bounded) for its copies and MMAs in flight, and frees TMEM.
#include <cuda.h>

#include <vector>

#include "../../include/g4cuda.h"
#include "g4_attn_dev.cuh"
#include "g4_tc.cuh"

namespace {

constexpr int kTM = 128;                  // query rows per tile (16 tokens x 8 heads)
constexpr int kTN = 256;                  // keys (S) or value dimensions (O) per tile
constexpr int kTK = 32;                   // fp16 K elements per stage: one 64-byte row
constexpr int kTStages = 4;
constexpr int kTileA = kTM * kTK * 2;     // 8 KB
constexpr int kTileB = kTN * kTK * 2;     // 16 KB
constexpr int kStageBytes = 2 * kTileA + 2 * kTileB;   // hi and lo of both operands: 48 KB
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kOffBar = kTStages * kStageBytes;
// barriers: full, empty, xready [kTStages] each, tfull, tempty [2] each, drain,
// ldone, then the TMEM address word
constexpr int kBarBytes = (3 * kTStages + 2 * 2 + 2) * 8 + 4;
constexpr int kSmem = kOffBar + 256 + 1024;          // + barriers, + 1 KB for alignment
static_assert(kBarBytes <= 256, "barrier region of the attention GEMM CTA");
constexpr int kTokTile = kTM / kHeads;                // 16 tokens per row tile
constexpr int kMaxRowTiles = G4_BATCH / kTokTile;     // 32
constexpr int kBufs = 1;                              // accumulator pairs in TMEM
// O: up to this many K stages per pair on average, one CTA takes each whole
// pair and finishes its rows (divide by l, quantise): no partial tiles and no
// combine launch. Above it the stages are cut evenly over the SMs (split K).
constexpr int kWholeMaxStages = 24;
constexpr float kPScale = 32768.0f;                   // 2^15: p in (0, 1]
// D fp32, A and B f16, both K-major, N = 256 (>> 3), M = 128 (>> 4)
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kTN >> 3) << 17) | ((uint32_t)(kTM >> 4) << 24);
static_assert(kSmem <= 227 * 1024, "shared memory budget of the attention GEMM CTA");
static_assert(kMaxRowTiles <= 32, "the unit prefix is one warp scan");

enum : int { kCodeFull = 0xa01, kCodeEmpty = 0xa02, kCodeTfull = 0xa03, kCodeTempty = 0xa04 };

// The chunk's schedule, computed the same way on the host and the device.
struct TcPlan {
    int T, sp, window, hd;
    int R, mt;        // query rows, 128-row tiles
    int kbase, nk;    // the workspace holds keys [kbase, kbase + nk)
    int kpad;         // row stride (keys) of S, P and V^T: nk rounded up to 256
    int nd;           // 256-wide value-dimension tiles: hd / 256
    int npairs;       // O: (row tile, dimension tile) pairs, row-tile major
    int u1;           // O: K stages (32 keys) of all pairs
    int g1;           // O: CTAs (each an even run of the stages, or one whole pair)
    int whole;        // O: one CTA per pair, which finishes its output rows itself
    float vscale;     // V scale 2^(15 - ceil(log2 sqrt(hd)))
};

__host__ __device__ inline int tc_first_key(int p, int window) { return (window && p + 1 > window) ? p + 1 - window : 0; }
__host__ __device__ inline int imin(int a, int b) { return a < b ? a : b; }

// Visible keys of row tile m relative to kbase: [kb, ke) (the first token's
// first key to the last token's position).
__host__ __device__ inline void tile_keys(const TcPlan &p, int m, int *kb, int *ke) {
    const int t0 = m * kTokTile, t1 = imin(p.T, t0 + kTokTile) - 1;
    *kb = tc_first_key(p.sp + t0, p.window) - p.kbase;
    *ke = p.sp + t1 + 1 - p.kbase;
}
// S units of row tile m: its 256-key tiles holding a visible key
__host__ __device__ inline int units_s(const TcPlan &p, int m) {
    int kb, ke;
    tile_keys(p, m, &kb, &ke);
    return (ke + kTN - 1) / kTN - kb / kTN;
}
// O: K stages of row tile m (each of its dimension tiles has them all)
__host__ __device__ inline int stages_o(const TcPlan &p, int m) {
    int kb, ke;
    tile_keys(p, m, &kb, &ke);
    return (ke + kTK - 1) / kTK - kb / kTK;
}
// O: the CTA whose run holds stage s (CTA b runs [u1 b / g1, u1 (b + 1) / g1))
__host__ __device__ inline int cta_of_stage(const TcPlan &p, long long s) {
    return (int)(((s + 1) * p.g1 + p.u1 - 1) / p.u1) - 1;
}

struct TcAttnArgs {
    TcPlan p;
    const float *qkv;
    int qkv_stride;
    const float *kcache, *vcache;
    int mask;
    __half *qh, *ql;      // [R][HD] scaled
    __half *kh, *kl;      // [nk][HD] scaled
    __half *vh, *vl;      // [HD][kpad] scaled
    float *qinv, *kinv;   // [R], [nk]: 1 / the row's scale
    float *s;             // [mt][kpad / 256][256 keys][128 rows] scores, tile-major
    float *smax;          // [R][kpad / 128]
    float *rmax;          // [R]
    float *lpart;         // [O slots][2][128] partial sums of p (pairs of dimension tile 0)
    float *opart;         // [O slots][128][256]; slot = pair + CTA
    float *out;           // [T][8 HD]
    int8_t *xq;
    float *xs, *xsT;
    int quant_out;
    int *err;
};

// x (already scaled, |x| < 2^15) as fp16 hi + lo, round to nearest; x - hi is exact.
G4_DEV void split_f16(float x, __half &hi, __half &lo) {
    hi = __float2half_rn(x);
    lo = __float2half_rn(__fsub_rn(x, __half2float(hi)));
}
// Two scaled values as fp16 hi and lo pairs (packed conversions: one
// instruction converts both); x - hi is exact.
G4_DEV void split2_f16(float x0, float x1, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __float22half2_rn(make_float2(x0, x1));
    const float2 hf = __half22float2(h);
    const __half2 l = __float22half2_rn(make_float2(__fsub_rn(x0, hf.x), __fsub_rn(x1, hf.y)));
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}
// 2^x by the hardware approximation (ex2.approx, relative error below 2^-22).
G4_DEV float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
constexpr float kLog2e = 1.4426950408889634f;

// The power of two c with max_abs * c in [2^14, 2^15) (1 for a zero row).
G4_DEV float row_scale(float max_abs) {
    if (!(max_abs > 0.0f)) return 1.0f;
    int e;
    frexpf(max_abs, &e);   // max_abs in [2^(e-1), 2^e)
    return ldexpf(1.0f, 15 - e);
}

// S: pre[0..mt] = prefix sums of the units of each row tile (warp 0; mt <= 32)
G4_DEV void unit_prefix_s(const TcPlan &p, int *pre) {
    const int lane = threadIdx.x & 31;
    int v = lane < p.mt ? units_s(p, lane) : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
    }
    if (lane == 0) pre[0] = 0;
    if (lane < p.mt) pre[lane + 1] = v;
}
// O: pre[0..npairs] = prefix sums of the K stages of each pair (one warp, two
// pairs a lane; npairs <= 64)
G4_DEV void pair_prefix_o(const TcPlan &p, int *pre) {
    const int lane = threadIdx.x & 31, i0 = 2 * lane, i1 = i0 + 1;
    const int v0 = i0 < p.npairs ? stages_o(p, i0 / p.nd) : 0, v1 = i1 < p.npairs ? stages_o(p, i1 / p.nd) : 0;
    int inc = v0 + v1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += n;
    }
    const int exc = inc - v0 - v1;
    if (lane == 0) pre[0] = 0;
    if (i0 < p.npairs) pre[i0 + 1] = exc + v0;
    if (i1 < p.npairs) pre[i1 + 1] = inc;
}
// O: the pair holding stage s (one warp, after pair_prefix_o): the count of pairs i >= 1 with pre[i] <= s
G4_DEV int pair_of_stage(const TcPlan &p, const int *pre, long long s) {
    const int lane = threadIdx.x & 31;
    const bool a = lane + 1 <= p.npairs && pre[lane + 1] <= s, b = lane + 33 <= p.npairs && pre[lane + 33] <= s;
    return __popc(__ballot_sync(0xffffffffu, a)) + __popc(__ballot_sync(0xffffffffu, b));
}

struct Unit {
    int m, n;     // row tile; key tile (S) or value-dimension tile (O)
    int c0, c1;   // K stages [c0, c1)
    int slot;     // O: partial slot (pair + CTA)
};
// The idx-th unit of this CTA (false: none left). S: units blockIdx.x, + gridDim.x, ...;
// O: the pairs overlapping this CTA's run of stages, from pair i0 on.
template <int MODE, int HD>
G4_DEV bool unit_at(const TcPlan &p, const int *pre, int idx, int i0, Unit &x) {
    if (MODE == 0) {
        const int u = blockIdx.x + idx * gridDim.x;
        if (u >= pre[p.mt]) return false;
        int m = 0;
        while (pre[m + 1] <= u) m++;
        int kb, ke;
        tile_keys(p, m, &kb, &ke);
        x.m = m;
        x.n = kb / kTN + (u - pre[m]);
        x.c0 = 0;
        x.c1 = HD / kTK;
        x.slot = u;
        return true;
    }
    if (p.whole) {   // CTA b: pair b, all its stages
        if (idx > 0) return false;
        int kb, ke;
        x.m = blockIdx.x / p.nd;
        x.n = blockIdx.x % p.nd;
        tile_keys(p, x.m, &kb, &ke);
        x.c0 = kb / kTK;
        x.c1 = (ke + kTK - 1) / kTK;
        x.slot = blockIdx.x;
        return true;
    }
    const int i = i0 + idx;
    const long long s0 = (long long)p.u1 * blockIdx.x / p.g1, s1 = (long long)p.u1 * (blockIdx.x + 1) / p.g1;
    if (i >= p.npairs || pre[i] >= s1) return false;
    int kb, ke;
    x.m = i / p.nd;
    x.n = i % p.nd;
    tile_keys(p, x.m, &kb, &ke);
    const int st = (int)(s0 > pre[i] ? s0 : pre[i]), en = (int)(s1 < pre[i + 1] ? s1 : pre[i + 1]);
    x.c0 = kb / kTK + (st - pre[i]);
    x.c1 = x.c0 + (en - st);
    x.slot = i + blockIdx.x;
    return true;
}

// ---------------------------------------------------------------------------
// 1. hi/lo operands. grid (blocks, 3): y = 0 Q rows, 1 key rows (one warp per
// row, scaled by the row's own power of two), 2 V^T tiles (fixed scale).
G4_DEV void store_split4(float4 x, float c, __half *dh, __half *dl) {
    uint32_t h0, l0, h1, l1;
    split2_f16(x.x * c, x.y * c, h0, l0);
    split2_f16(x.z * c, x.w * c, h1, l1);
    *(uint2 *)dh = make_uint2(h0, h1);
    *(uint2 *)dl = make_uint2(l0, l1);
}

template <int HD>
__global__ void __launch_bounds__(256) k_tc_split(const TcAttnArgs a) {
    __shared__ float tile[32][33];
    const TcPlan &p = a.p;
    griddep_launch();
    griddep_wait();   // q/k/v rows come from the previous kernel
    const int job = blockIdx.y;
    if (job < 2) {
        constexpr int V4 = HD / 128;   // float4s per lane
        const int lane = threadIdx.x & 31, rows = job == 0 ? p.R : p.nk;
        for (int r = blockIdx.x * 8 + (threadIdx.x >> 5); r < rows; r += gridDim.x * 8) {
            const float4 *src = (const float4 *)(job == 0 ? a.qkv + (size_t)(r >> 3) * a.qkv_stride + (r & 7) * HD
                                                          : a.kcache + (size_t)((p.kbase + r) & a.mask) * HD);
            float4 x[V4];
            float m = 0.0f;
#pragma unroll
            for (int i = 0; i < V4; i++) {
                x[i] = src[lane + 32 * i];
                m = fmaxf(m, fmaxf(fmaxf(fabsf(x[i].x), fabsf(x[i].y)), fmaxf(fabsf(x[i].z), fabsf(x[i].w))));
            }
            const float c = row_scale(warp_max(m));
            __half *dh = (job == 0 ? a.qh : a.kh) + (size_t)r * HD, *dl = (job == 0 ? a.ql : a.kl) + (size_t)r * HD;
#pragma unroll
            for (int i = 0; i < V4; i++) store_split4(x[i], c, dh + 4 * (lane + 32 * i), dl + 4 * (lane + 32 * i));
            if (lane == 0) (job == 0 ? a.qinv : a.kinv)[r] = 1.0f / c;   // a power of two: exact
        }
        return;
    }
    // V^T through shared memory, 32 keys x 32 dimensions per tile
    const float c = p.vscale;
    const int kt = (p.nk + 31) / 32, ntiles = kt * (HD / 32);
    for (int ti = blockIdx.x; ti < ntiles; ti += gridDim.x) {
        const int k0 = (ti / (HD / 32)) * 32, d0 = (ti % (HD / 32)) * 32;
        for (int i = threadIdx.x; i < 32 * 32; i += 256) {
            const int kr = i >> 5, dc = i & 31;
            tile[kr][dc] = k0 + kr < p.nk ? a.vcache[(size_t)((p.kbase + k0 + kr) & a.mask) * HD + d0 + dc] : 0.0f;
        }
        __syncthreads();
        for (int i = threadIdx.x; i < 32 * 32; i += 256) {
            const int dr = i >> 5, kc = i & 31;
            if (k0 + kc < p.nk) {
                __half h, l;
                split_f16(tile[kc][dr] * c, h, l);
                const size_t o = (size_t)(d0 + dr) * p.kpad + k0 + kc;
                a.vh[o] = h;
                a.vl[o] = l;
            }
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// 32 columns of this lane's hi.hi accumulator plus its correction accumulator
// (256 columns on), as fp32 bits.
G4_DEV void load_acc(uint32_t taddr, int (&v)[32]) {
    int w[32];
    tmem_ld32(taddr, v);
    tmem_ld32(taddr + kTN, w);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 32; j++) v[j] = __float_as_int(__fadd_rn(__int_as_float(v[j]), __int_as_float(w[j])));
}

// ---------------------------------------------------------------------------
// 2 and 4. The split-operand GEMMs. MODE 0: A = Q, B = K, units (row tile, key
// tile); MODE 1: A = P (made from S in shared memory), B = V^T, units (pair,
// this CTA's share of its K stages).
template <int MODE, int HD>
__global__ void __launch_bounds__(kThreads, 1)
    k_tc_gemm(const __grid_constant__ CUtensorMap map_ah, const __grid_constant__ CUtensorMap map_al,
              const __grid_constant__ CUtensorMap map_bh, const __grid_constant__ CUtensorMap map_bl,
              const TcAttnArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *full = (uint64_t *)(smem + kOffBar);
    uint64_t *empty = full + kTStages;
    uint64_t *tfull = empty + kTStages;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;
    uint64_t *xready = drain + 1;   // O: the stage's P tiles are written
    uint64_t *ldone = xready + kTStages;   // O, whole pairs: both groups' row sums are written
    uint32_t *tmem_slot = (uint32_t *)(ldone + 1);
    __shared__ int pre[2 * kMaxRowTiles + 1];
    __shared__ int fail, issued, ipair0;
    __shared__ int xfail_g[2];      // O: a transform group's wait gave up (written by that group only)
    __shared__ float lsh[2][kTM];   // O, whole pairs: the row sums of p of the two transform groups
    const TcPlan &p = a.p;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (MODE == 0 && warp == 0) unit_prefix_s(p, pre);
    if (MODE == 1 && warp == 0) {
        pair_prefix_o(p, pre);
        __syncwarp();
        // the pair holding this CTA's first stage
        const int i = pair_of_stage(p, pre, (long long)p.u1 * blockIdx.x / p.g1);
        if (lane == 0) ipair0 = i;
    }
    if (tid == 32) {
        for (int s = 0; s < kTStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < kBufs; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], kEpiWarps);
        }
        mbar_init(drain, 1);
        for (int s = 0; s < kTStages; s++) mbar_init(&xready[s], kEpiWarps / 2);
        mbar_init(ldone, kEpiWarps);
        mbar_fence_init();
        fail = 0;
        issued = 0;
        xfail_g[0] = xfail_g[1] = 0;
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(2 * kTN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // Programmatic dependent launch: the next kernel may be scheduled once
    // every CTA holds its TMEM columns (a dependent allocation then waits for
    // this grid, never the reverse); the workspace is read and written only
    // after the previous kernel has completed (the set-up above reads kernel
    // parameters only).
    griddep_launch();
    griddep_wait();
    const int ntk = p.kpad / kTN;   // key tiles per row tile in the S layout
    const int i0 = MODE == 1 ? ipair0 : 0;
    Unit x;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int k = 0;
            bool ok = true;
            for (int idx = 0; ok && unit_at<MODE, HD>(p, pre, idx, i0, x); idx++) {
                const int ay = x.m * kTM, by = x.n * kTN;
                for (int c = x.c0; c < x.c1; c++, k++) {
                    const int s = k % kTStages, use = k / kTStages;
                    if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1, a.err, G4D_TIMEOUT_EMPTY | (kCodeEmpty << 8))) {
                        ok = false;
                        break;
                    }
                    uint8_t *st = smem + s * kStageBytes;
                    mbar_arrive_expect_tx(&full[s], kStageBytes);
                    if (MODE == 0) {
                        tma_load_2d(st, &map_ah, c * kTK, ay, &full[s]);
                        tma_load_2d(st + kTileA, &map_al, c * kTK, ay, &full[s]);
                    } else {   // the S block of keys [32 c, 32 c + 32): 32 x 128 fp32, contiguous
                        constexpr int per = kTN / kTK;   // blocks per key tile
                        bulk_g2s_plain(st, a.s + (((size_t)x.m * ntk + c / per) * kTN + (c % per) * kTK) * kTM,
                                       2 * kTileA, &full[s]);
                    }
                    tma_load_2d(st + 2 * kTileA, &map_bh, c * kTK, by, &full[s]);
                    tma_load_2d(st + 2 * kTileA + kTileB, &map_bl, c * kTK, by, &full[s]);
                }
            }
            if (!ok) fail = 1;
            issued = k;
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint64_t d0 = umma_desc_sw64(smem, 0);
            int k = 0, i = 0;
            bool ok = true;
            for (; ok && unit_at<MODE, HD>(p, pre, i, i0, x); i++) {
                const int buf = i % kBufs, use = i / kBufs;
                if (use > 0 && !mbar_wait(&tempty[buf], (use - 1) & 1, a.err, G4D_TIMEOUT_EMPTY | (kCodeTempty << 8))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t td = tmem + (uint32_t)(buf * kTN), tcr = td + kTN;
                for (int c = x.c0; c < x.c1; c++, k++) {
                    const int s = k % kTStages;
                    if (!mbar_wait(MODE == 0 ? &full[s] : &xready[s], (k / kTStages) & 1, a.err,
                                   G4D_TIMEOUT_FULL | (kCodeFull << 8))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    // stage tiles: A hi, A lo, B hi, B lo (start-address field in 16-byte units)
                    const uint64_t ah = d0 + (uint64_t)((s * kStageBytes) >> 4);
                    const uint64_t al = ah + (uint64_t)(kTileA >> 4);
                    const uint64_t bh = ah + (uint64_t)((2 * kTileA) >> 4);
                    const uint64_t bl = bh + (uint64_t)(kTileB >> 4);
#pragma unroll
                    for (int kk = 0; kk < kTK / 16; kk++) {
                        const uint64_t o = (uint64_t)((kk * 32) >> 4);   // 16 fp16 = 32 bytes per MMA
                        const bool acc = c > x.c0 || kk > 0;
                        mma_f16(td, ah + o, bh + o, kIdesc, acc);
                        mma_f16(tcr, ah + o, bl + o, kIdesc, acc);
                        mma_f16(tcr, al + o, bh + o, kIdesc, true);
                    }
                    mma_commit(&empty[s]);
                }
                if (!ok) break;
                mma_commit(&tfull[buf]);
            }
            if (!ok) fail = 1;
        }
    } else {
        // ---------------- epilogue (and, for O, the S -> P transform) ----------------
        const int e = warp - 2, q = warp & 3, ch = e >> 2;
        const int row = q * 32 + lane;
        int i = 0, k = 0;
        for (; unit_at<MODE, HD>(p, pre, i, i0, x); i++) {
            if (MODE == 1) {
                // two transform groups of four warps take alternate stages (stage k:
                // group k % 2); thread = row trow x the stage's 32 keys. Each group has
                // its own named barrier and failure flag, so its exits stay uniform.
                const int g = e >> 2, trow = (e & 3) * 32 + lane;
                const int rg = x.m * kTM + trow, t = rg >> 3;
                const bool live = rg < p.R;
                const int kmin = tc_first_key(p.sp + t, p.window) - p.kbase, kmax = p.sp + t - p.kbase;
                const float mr = live ? a.rmax[rg] : 0.0f;
                const float mrl = mr * kLog2e;   // p = 2^(s log2 e - m log2 e)
                float lsum = 0.0f;
                for (int c = x.c0; c < x.c1; c++, k++) {
                    if ((k & 1) != g) continue;   // the other group's stage
                    const int s = k % kTStages;
                    const bool got = mbar_wait(&full[s], (k / kTStages) & 1, a.err, G4D_TIMEOUT_FULL | (kCodeFull << 8));
                    float v[kTK];
                    if (got) {
                        const float *raw = (const float *)(smem + s * kStageBytes);
#pragma unroll
                        for (int j = 0; j < kTK; j++) v[j] = raw[j * kTM + trow];
                    } else {
                        xfail_g[g] = 1;
                        fail = 1;
                    }
                    // every thread of the group has read the block before any writes over it
                    // (a wait that gave up still arrives here: the decision to leave is uniform)
                    bar_sync(1 + g, 32 * kEpiWarps / 2);
                    if (xfail_g[g]) break;
                    const int kb0 = c * kTK, kb1 = kb0 + kTK - 1;
                    // this row's keys all visible (the common case), none, or some
                    const bool all_vis = live && kb0 >= kmin && kb1 <= kmax;
                    const bool none_vis = !live || kb0 > kmax || kb1 < kmin;
                    uint32_t hw[kTK / 2], lw[kTK / 2];
#pragma unroll
                    for (int j = 0; j < kTK; j += 2) {
                        float p0, p1;
                        if (all_vis) {
                            p0 = ex2_approx(__fmaf_rn(v[j], kLog2e, -mrl));
                            p1 = ex2_approx(__fmaf_rn(v[j + 1], kLog2e, -mrl));
                        } else if (none_vis) {
                            p0 = p1 = 0.0f;
                        } else {
                            p0 = kb0 + j >= kmin && kb0 + j <= kmax ? ex2_approx(__fmaf_rn(v[j], kLog2e, -mrl)) : 0.0f;
                            p1 = kb0 + j + 1 >= kmin && kb0 + j + 1 <= kmax
                                     ? ex2_approx(__fmaf_rn(v[j + 1], kLog2e, -mrl)) : 0.0f;
                        }
                        lsum += p0;
                        lsum += p1;
                        split2_f16(p0 * kPScale, p1 * kPScale, hw[j / 2], lw[j / 2]);
                    }
                    // K-major fp16 rows of 64 bytes with the 64-byte swizzle: logical 16-byte
                    // chunk j of row r sits at chunk j ^ ((r / 2) % 4)
                    uint8_t *th = smem + s * kStageBytes, *tl = th + kTileA;
#pragma unroll
                    for (int c4 = 0; c4 < kTK / 8; c4++) {
                        const int off = trow * (kTK * 2) + ((c4 ^ ((trow >> 1) & 3)) << 4);
                        *(uint4 *)(th + off) = make_uint4(hw[4 * c4], hw[4 * c4 + 1], hw[4 * c4 + 2], hw[4 * c4 + 3]);
                        *(uint4 *)(tl + off) = make_uint4(lw[4 * c4], lw[4 * c4 + 1], lw[4 * c4 + 2], lw[4 * c4 + 3]);
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // visible to the tensor core
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&xready[s]);
                }
                if (xfail_g[g]) break;
                if (p.whole) {   // the row sums of both groups meet in shared memory
                    lsh[g][trow] = lsum;
                    __syncwarp();
                    if (lane == 0) mbar_arrive(ldone);
                } else if (x.n == 0) {
                    a.lpart[((size_t)x.slot * 2 + g) * kTM + trow] = lsum;
                }
            }
            const int buf = i % kBufs;
            const bool got = mbar_wait(&tfull[buf], (i / kBufs) & 1, a.err, G4D_TIMEOUT_FULL | (kCodeTfull << 8));
            if (!__all_sync(0xffffffffu, got)) {
                // (for O the warp goes on to the next unit with its group: its transform
                // waits then give up on their own, keeping the group's barriers uniform)
                if (lane == 0) fail = 1;
                if (MODE == 0) break;
                continue;
            }
            tc_fence_after();
            const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * kTN + ch * 128);
            const int rg = x.m * kTM + row;
            if (MODE == 0) {
                const int t = rg >> 3;
                const int kmin = tc_first_key(p.sp + t, p.window) - p.kbase, kmax = p.sp + t - p.kbase;
                const int j0 = x.n * kTN + ch * 128;
                float *blk = a.s + ((size_t)x.m * ntk + x.n) * kTN * kTM;   // [256 keys][128 rows]
                const float qi = rg < p.R ? __ldg(a.qinv + rg) : 0.0f;
                float mx = -INFINITY;
#pragma unroll 1
                for (int c = 0; c < 4; c++) {
                    const int jb = j0 + c * 32;
                    // the chunk's key scales, loaded before the accumulator read (one
                    // round trip, not one per key between the stores below)
                    float kv[32];
#pragma unroll
                    for (int j = 0; j < 32; j++) kv[j] = jb + j < p.nk ? __ldg(a.kinv + jb + j) : 0.0f;
                    int v[32];
                    load_acc(ta + (uint32_t)(c * 32), v);
                    if (c == 3) {   // the accumulator is read: free it for the unit after next
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&tempty[buf]);
                    }
#pragma unroll
                    for (int j = 0; j < 32; j++) {
                        const int key = jb + j;
                        // the row and key scales are powers of two: exact
                        const float sv = __int_as_float(v[j]) * qi * kv[j];
                        if (key >= kmin && key <= kmax) mx = fmaxf(mx, sv);
                        blk[(size_t)(ch * 128 + c * 32 + j) * kTM + row] = sv;   // the warp: 128 contiguous bytes
                    }
                }
                if (rg < p.R) a.smax[(size_t)rg * (p.kpad / 128) + j0 / 128] = mx;
            } else if (p.whole) {
                // the finished rows: O = acc / l with the P and V scales removed (powers of
                // two: exact), stored and quantised per 64-wide group (quantize,
                // gemma4.c:265-279) for o_proj; the same arithmetic as k_tc_out's
                if (!__all_sync(0xffffffffu, mbar_wait(ldone, 0, a.err, G4D_TIMEOUT_FULL | (kCodeTfull << 8)))) {
                    if (lane == 0) fail = 1;
                    continue;
                }
                const float inv = (1.0f / (lsh[0][row] + lsh[1][row])) * (1.0f / (kPScale * p.vscale));
                const int t = rg >> 3;
#pragma unroll 1
                for (int c = 0; c < 4; c += 2) {
                    float o[64];
                    {
                        int v[32];
                        load_acc(ta + (uint32_t)(c * 32), v);
#pragma unroll
                        for (int j = 0; j < 32; j++) o[j] = __int_as_float(v[j]) * inv;
                        load_acc(ta + (uint32_t)(c * 32 + 32), v);
#pragma unroll
                        for (int j = 0; j < 32; j++) o[32 + j] = __int_as_float(v[j]) * inv;
                    }
                    if (c == 2) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&tempty[buf]);
                    }
                    if (rg >= p.R) continue;
                    const int d0 = x.n * kTN + ch * 128 + c * 32;   // 64-aligned
                    float *orow = a.out + (size_t)rg * HD + d0;
#pragma unroll
                    for (int j = 0; j < 64; j += 4) *(float4 *)(orow + j) = make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]);
                    if (a.quant_out) {
                        float mx = 0.0f;
#pragma unroll
                        for (int j = 0; j < 64; j++) mx = fmaxf(mx, fabsf(o[j]));
                        const float sc = quant_scale(mx), qv = quant_inv(sc);
                        uint32_t w[16];
#pragma unroll
                        for (int j = 0; j < 16; j++)
                            w[j] = (uint32_t)(uint8_t)quant_one(o[4 * j], qv) |
                                   ((uint32_t)(uint8_t)quant_one(o[4 * j + 1], qv) << 8) |
                                   ((uint32_t)(uint8_t)quant_one(o[4 * j + 2], qv) << 16) |
                                   ((uint32_t)(uint8_t)quant_one(o[4 * j + 3], qv) << 24);
                        uint4 *qrow = (uint4 *)(a.xq + (size_t)rg * HD + d0);
#pragma unroll
                        for (int j = 0; j < 4; j++) qrow[j] = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
                        const int gcol = ((rg & 7) * HD + d0) / 64;   // the group's column in the token's row
                        a.xs[(size_t)t * (kHeads * HD / 64) + gcol] = sc;
                        if (a.xsT) a.xsT[(size_t)gcol * G4_XST_STRIDE + t] = sc;
                    }
                }
            } else {
                float *dst = a.opart + ((size_t)x.slot * kTM + row) * kTN + ch * 128;
#pragma unroll 1
                for (int c = 0; c < 4; c++) {
                    int v[32];
                    load_acc(ta + (uint32_t)(c * 32), v);
                    if (c == 3) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&tempty[buf]);
                    }
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        *(float4 *)(dst + c * 32 + j) = make_float4(__int_as_float(v[j]), __int_as_float(v[j + 1]),
                                                                    __int_as_float(v[j + 2]), __int_as_float(v[j + 3]));
                }
            }
        }
    }

    // ---------------- teardown ----------------
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (tid == 32) {
        // every MMA this lane issued has retired (bounded: after a failure some never ran)
        mma_commit(drain);
        mbar_wait(drain, 0, nullptr, 0);
    }
    if (fail && tid == 0) {
        // copies in flight still write shared memory: let them land
        const uint64_t t0n = g4_globaltimer();
        for (int k = issued > kTStages ? issued - kTStages : 0; k < issued; k++)
            while (!mbar_try_wait(&full[k % kTStages], (k / kTStages) & 1) && g4_globaltimer() - t0n < G4_WAIT_NS) {
            }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kTN) : "memory");
    }
}

// ---------------------------------------------------------------------------
// 3. Row maxima of the scores: one warp per query row.
__global__ void __launch_bounds__(256) k_tc_rowmax(const TcAttnArgs a) {
    const TcPlan &p = a.p;
    const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    griddep_launch();
    griddep_wait();
    if (r >= p.R) return;
    int kb, ke;
    tile_keys(p, r / kTM, &kb, &ke);
    const int h0 = (kb / kTN) * 2, h1 = ((ke + kTN - 1) / kTN) * 2;
    float mx = -INFINITY;
    for (int h = h0 + lane; h < h1; h += 32) mx = fmaxf(mx, a.smax[(size_t)r * (p.kpad / 128) + h]);
    mx = warp_max(mx);
    if (lane == 0) a.rmax[r] = mx;
}

// ---------------------------------------------------------------------------
// 5. Output rows: one CTA per token (its 8 heads), pieces summed in order.
template <int HD>
__global__ void __launch_bounds__(256) k_tc_out(const TcAttnArgs a) {
    __shared__ int pre[2 * kMaxRowTiles + 1];
    __shared__ int bfirst[2], blast[2];
    __shared__ float inv[kHeads];
    const TcPlan &p = a.p;
    const int t = blockIdx.x, tid = threadIdx.x;
    const int m = t / kTokTile;
    griddep_launch();
    griddep_wait();
    if (tid < 32) {
        pair_prefix_o(p, pre);
        __syncwarp();
        if (tid < p.nd) {   // the CTAs whose runs cover pair (m, n)
            const int i = m * p.nd + tid;
            bfirst[tid] = cta_of_stage(p, pre[i]);
            blast[tid] = cta_of_stage(p, pre[i + 1] - 1);
        }
    }
    __syncthreads();
    if (tid < kHeads) {
        // l = the partial sums of the CTAs in order; 1 / l, then the P and V scales
        // (powers of two: exact)
        const int rl = (t * kHeads + tid) % kTM, i = m * p.nd;
        float l = 0.0f;
        for (int b = bfirst[0]; b <= blast[0]; b++) {
            const size_t sl = (size_t)(i + b);
            l += a.lpart[(sl * 2) * kTM + rl];
            l += a.lpart[(sl * 2 + 1) * kTM + rl];
        }
        inv[tid] = (1.0f / l) * (1.0f / (kPScale * p.vscale));
    }
    __syncthreads();
    constexpr int W = kHeads * HD;
    for (int idx = tid; idx < W / 4; idx += 256) {
        const int h = idx / (HD / 4), c4 = idx % (HD / 4), d = c4 * 4;
        const int n = d / kTN, dl = d % kTN, rl = (t * kHeads + h) % kTM;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int b = bfirst[n]; b <= blast[n]; b++) {
            const float4 v = *(const float4 *)(a.opart + ((size_t)(m * p.nd + n + b) * kTM + rl) * kTN + dl);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        const float s = inv[h];
        acc = make_float4(acc.x * s, acc.y * s, acc.z * s, acc.w * s);
        const int col = h * HD + d;
        *(float4 *)(a.out + (size_t)t * W + col) = acc;
        if (a.quant_out)   // 16 consecutive lanes hold one 64-wide group
            quant_lanes16(acc, a.xq + (size_t)t * W + col, a.xs + (size_t)t * (W / 64) + col / 64,
                          a.xsT ? a.xsT + (size_t)(col / 64) * G4_XST_STRIDE + t : nullptr, (c4 & 15) == 0);
    }
}

// ---- host side ----------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// fp16 [rows][cols] (row stride `stride` bytes), boxes of box_rows x 32 with
// the 64-byte swizzle; elements outside [rows][cols] read as zero.
bool make_map_f16(CUtensorMap *m, const __half *base, int cols, int rows, size_t stride, int box_rows) {
    EncodeTiledFn fn = (EncodeTiledFn)g4_tmap_encoder();
    if (!fn || ((uintptr_t)base & 15) || (stride & 15) || cols < 1 || rows < 1) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)stride};
    const cuuint32_t box[2] = {(cuuint32_t)kTK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void *)base, dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

TcPlan make_plan(const AttnArgs &a, int sms, int *nunits_s, int *nunits_o) {
    TcPlan p{};
    p.T = a.T;
    p.sp = a.start_pos;
    p.window = a.window;
    p.hd = a.hd;
    p.R = kHeads * a.T;
    p.mt = (p.R + kTM - 1) / kTM;
    p.kbase = tc_first_key(a.start_pos, a.window);
    p.nk = a.start_pos + a.T - p.kbase;
    p.kpad = (p.nk + kTN - 1) / kTN * kTN;
    p.nd = a.hd / kTN;
    {   // |v| <= sqrt(hd): the largest power of two c with sqrt(hd) c < 2^15
        int e;
        frexpf(sqrtf((float)a.hd), &e);
        p.vscale = ldexpf(1.0f, 15 - e);
    }
    int us = 0, u1 = 0;
    for (int m = 0; m < p.mt; m++) {
        us += units_s(p, m);
        u1 += p.nd * stages_o(p, m);
    }
    p.npairs = p.mt * p.nd;
    p.u1 = u1;
    p.whole = u1 <= kWholeMaxStages * p.npairs ? 1 : 0;
    // one run per SM even when runs are short: a unit's epilogue and pipeline
    // refill (~6-8 us: the two accumulators fill TMEM, so nothing overlaps
    // them) cost more in sequence on fewer SMs (measured: 36 runs of 8 stages
    // 71 us, 148 runs of 2 stages 25 us, global chunk at position 0)
    p.g1 = p.whole ? p.npairs : (u1 < sms ? u1 : sms);
    *nunits_s = us;
    *nunits_o = p.whole ? 0 : p.npairs + p.g1;   // O partial slots (pair + CTA)
    return p;
}

// Workspace pieces, 1 KB aligned (float offsets).
struct TcWs {   // byte offsets
    size_t qh, ql, kh, kl, vh, vl, qinv, kinv, s, smax, rmax, lpart, opart, total;
};
TcWs ws_layout(const TcPlan &p, int nunits_o) {
    TcWs w{};
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += (bytes + 1023) / 1024 * 1024;
        return o;
    };
    const size_t R = (size_t)p.R, HD = (size_t)p.hd, kp = (size_t)p.kpad, nk = (size_t)p.nk;
    w.qh = take(R * HD * 2);
    w.ql = take(R * HD * 2);
    w.kh = take(nk * HD * 2);
    w.kl = take(nk * HD * 2);
    w.vh = take(HD * kp * 2);
    w.vl = take(HD * kp * 2);
    w.qinv = take(R * 4);
    w.kinv = take(nk * 4);
    w.s = take((size_t)p.mt * kTM * kp * 4);
    w.smax = take(R * (kp / 128) * 4);
    w.rmax = take(R * 4);
    w.lpart = take((size_t)nunits_o * 2 * kTM * 4);
    w.opart = take((size_t)nunits_o * kTM * kTN * 4);
    w.total = off;
    return w;
}

bool tc_args_ok(const AttnArgs &a) {
    return (a.hd == 256 || a.hd == 512) && a.T >= 1 && a.T <= G4_BATCH && !a.row_seq && !a.strict &&
           a.start_pos >= 0 && a.qkv && a.kcache && a.vcache && a.out &&
           // the keys of the chunk must not wrap around the ring
           a.start_pos + a.T - tc_first_key(a.start_pos, a.window) <= a.mask + 1;
}

template <int HD>
cudaError_t launch_tc(const AttnArgs &a, void *ws, size_t ws_bytes, cudaStream_t st, bool pdl) {
    const int sms = g4_device_sms();
    int nus = 0, nuo = 0;
    const TcPlan p = make_plan(a, sms, &nus, &nuo);
    const TcWs w = ws_layout(p, nuo);
    if (!ws || ws_bytes < w.total || ((uintptr_t)ws & 255)) return cudaErrorInvalidValue;
    uint8_t *b = (uint8_t *)ws;
    TcAttnArgs x{};
    x.p = p;
    x.qkv = a.qkv;
    x.qkv_stride = a.qkv_stride;
    x.kcache = a.kcache;
    x.vcache = a.vcache;
    x.mask = a.mask;
    x.qh = (__half *)(b + w.qh);
    x.ql = (__half *)(b + w.ql);
    x.kh = (__half *)(b + w.kh);
    x.kl = (__half *)(b + w.kl);
    x.vh = (__half *)(b + w.vh);
    x.vl = (__half *)(b + w.vl);
    x.qinv = (float *)(b + w.qinv);
    x.kinv = (float *)(b + w.kinv);
    x.s = (float *)(b + w.s);
    x.smax = (float *)(b + w.smax);
    x.rmax = (float *)(b + w.rmax);
    x.lpart = (float *)(b + w.lpart);
    x.opart = (float *)(b + w.opart);
    x.out = a.out;
    x.quant_out = a.quant_out;
    x.xq = a.xq;
    x.xs = a.xs;
    x.xsT = a.xsT;
    x.err = a.err;
    if (a.quant_out && (!a.xq || !a.xs)) return cudaErrorInvalidValue;
    CUtensorMap qh, ql, kh, kl, vh, vl;
    const size_t rs = (size_t)HD * 2, ks = (size_t)p.kpad * 2;
    if (!make_map_f16(&qh, x.qh, HD, p.R, rs, kTM) || !make_map_f16(&ql, x.ql, HD, p.R, rs, kTM) ||
        !make_map_f16(&kh, x.kh, HD, p.nk, rs, kTN) || !make_map_f16(&kl, x.kl, HD, p.nk, rs, kTN) ||
        !make_map_f16(&vh, x.vh, p.nk, HD, ks, kTN) || !make_map_f16(&vl, x.vl, p.nk, HD, ks, kTN))
        return cudaErrorInvalidValue;
    cudaError_t e = g4_smem_optin((const void *)k_tc_gemm<0, HD>, kSmem);
    if (e == cudaSuccess) e = g4_smem_optin((const void *)k_tc_gemm<1, HD>, kSmem);
    if (e) return e;
    // job 0 splits Q; jobs 1 and 2 K and V, unless the workspace holds them already
    e = g4_launch(k_tc_split<HD>, dim3(4 * sms, a.reuse_kv ? 1 : 3), dim3(256), 0, st, pdl, x);
    if (e == cudaSuccess)
        e = g4_launch(k_tc_gemm<0, HD>, dim3(nus < sms ? nus : sms), dim3(kThreads), (size_t)kSmem, st, pdl, qh, ql,
                      kh, kl, x);
    if (e == cudaSuccess) e = g4_launch(k_tc_rowmax, dim3((p.R + 7) / 8), dim3(256), 0, st, pdl, x);
    // the A maps are unused for O (its A tiles are made from S in shared memory)
    if (e == cudaSuccess)
        e = g4_launch(k_tc_gemm<1, HD>, dim3(p.g1), dim3(kThreads), (size_t)kSmem, st, pdl, vh, vl, vh, vl, x);
    if (e == cudaSuccess && !p.whole) e = g4_launch(k_tc_out<HD>, dim3(p.T), dim3(256), 0, st, pdl, x);
    return e;
}

}  // namespace

// Host check of the tensor-core attention schedule for a chunk (no GPU work):
// every S unit's key tile inside the workspace and every row tile's visible
// keys inside its units; the P V stages of every (row tile, dimension tile)
// pair covered exactly once by the CTA runs; partial slots distinct and below
// npairs + g1; the combine's CTA range of each pair equal to the CTAs that ran
// it. Returns 0, or the number of the first failed check.
extern "C" int g4k_attn_tc_plan(int hd, int T, int start_pos, int sms, int *units_s_out, int *stages_o_out,
                                int *ctas_o_out, unsigned long long *ws_bytes_out) {
    if ((hd != 256 && hd != 512) || T < 1 || T > G4_BATCH || start_pos < 0 || sms < 1 ||
        start_pos + T > G4_MAX_CONTEXT)
        return G4_ERR_INVALID;
    AttnArgs a{};
    a.hd = hd;
    a.window = hd == 256 ? G4_SLIDING_WINDOW : 0;
    a.mask = (hd == 256 ? 1024 : G4_MAX_CONTEXT) - 1;
    a.T = T;
    a.start_pos = start_pos;
    a.qkv = a.kcache = a.vcache = a.out = (float *)&a;   // placeholders: nothing is read
    if (!tc_args_ok(a)) return 1;
    int nus = 0, nslots = 0;
    const TcPlan p = make_plan(a, sms, &nus, &nslots);
    if (p.mt > kMaxRowTiles || p.npairs > 2 * kMaxRowTiles || p.kpad % kTN || p.nk < 1 || p.nk > p.kpad) return 2;
    // S units and row tiles
    int us = 0;
    for (int m = 0; m < p.mt; m++) {
        int kb, ke;
        tile_keys(p, m, &kb, &ke);
        if (kb < 0 || kb >= ke || ke > p.nk) return 3;
        for (int t = m * kTokTile; t < imin(T, m * kTokTile + kTokTile); t++) {
            const int kmin = tc_first_key(start_pos + t, a.window) - p.kbase, kmax = start_pos + t - p.kbase;
            if (kmin < kb || kmax >= ke) return 4;
        }
        const int n0 = kb / kTN, n1 = (ke + kTN - 1) / kTN;
        if (n1 * kTN > p.kpad || n1 - n0 != units_s(p, m)) return 5;
        // the P V stages of the row tile and the S tiles that hold them
        const int c0 = kb / kTK, c1 = (ke + kTK - 1) / kTK;
        if (c1 * kTK > p.kpad || c0 * kTK < n0 * kTN || c1 * kTK > n1 * kTN || c1 - c0 != stages_o(p, m)) return 6;
        us += n1 - n0;
    }
    if (us != nus) return 7;
    // P V runs: CTA b takes stages [u1 b / g1, u1 (b + 1) / g1) of the pairs in order
    std::vector<int> pre(p.npairs + 1, 0), cover(p.u1, 0), slot_used(p.npairs + p.g1, 0);
    for (int i = 0; i < p.npairs; i++) pre[i + 1] = pre[i] + stages_o(p, i / p.nd);
    if (p.whole) {   // CTA b takes pair b whole and finishes its rows: no slots, no combine
        if (pre[p.npairs] != p.u1 || p.g1 != p.npairs || nslots != 0 || p.u1 > kWholeMaxStages * p.npairs) return 14;
        if (units_s_out) *units_s_out = nus;
        if (stages_o_out) *stages_o_out = p.u1;
        if (ctas_o_out) *ctas_o_out = p.g1;
        if (ws_bytes_out) *ws_bytes_out = ws_layout(p, nslots).total;
        return 0;
    }
    if (pre[p.npairs] != p.u1 || p.g1 < 1 || p.g1 > sms || p.g1 > p.u1) return 8;
    std::vector<int> first_cta(p.npairs, -1), last_cta(p.npairs, -1);
    for (int b = 0; b < p.g1; b++) {
        const long long s0 = (long long)p.u1 * b / p.g1, s1 = (long long)p.u1 * (b + 1) / p.g1;
        if (s1 <= s0) return 9;
        int i = 0;
        while (pre[i + 1] <= s0) i++;
        for (; i < p.npairs && pre[i] < s1; i++) {
            const long long st = s0 > pre[i] ? s0 : pre[i], en = s1 < pre[i + 1] ? s1 : pre[i + 1];
            if (en <= st) return 10;
            for (long long s = st; s < en; s++) cover[s]++;
            const int slot = i + b;
            if (slot >= p.npairs + p.g1 || slot_used[slot]++) return 11;
            if (first_cta[i] < 0) first_cta[i] = b;
            last_cta[i] = b;
        }
    }
    for (int s = 0; s < p.u1; s++)
        if (cover[s] != 1) return 12;
    for (int i = 0; i < p.npairs; i++)
        if (cta_of_stage(p, pre[i]) != first_cta[i] || cta_of_stage(p, pre[i + 1] - 1) != last_cta[i]) return 13;
    if (units_s_out) *units_s_out = nus;
    if (stages_o_out) *stages_o_out = p.u1;
    if (ctas_o_out) *ctas_o_out = p.g1;
    if (ws_bytes_out) *ws_bytes_out = ws_layout(p, nslots).total;
    return 0;
}

size_t g4_attn_tc_ws_bytes(const AttnArgs &a) {
    if (!tc_args_ok(a)) return 0;
    int nus = 0, nuo = 0;
    const TcPlan p = make_plan(a, g4_device_sms(), &nus, &nuo);
    return ws_layout(p, nuo).total;
}

cudaError_t g4_launch_attn_tc(const AttnArgs &a, void *ws, size_t ws_bytes, cudaStream_t st, bool pdl) {
    if (!tc_args_ok(a) || !g4_tmap_encoder()) return cudaErrorInvalidValue;
    if (a.hd == 256) return launch_tc<256>(a, ws, ws_bytes, st, pdl);
    return launch_tc<512>(a, ws, ws_bytes, st, pdl);
}
