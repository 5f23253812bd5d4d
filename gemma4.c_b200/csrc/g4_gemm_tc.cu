// g4_gemm_tc.cu — prefill int8 GEMM on the 5th-generation tensor cores.
//
// Reference: matmul_int8 / matmul_block (gemma4.c:192-262) over T token rows:
//   out[t][n] = fma-chain over groups g ascending of
//               (float)(sum_{k in g} xq[t][k] * w[n][k])  *  (ws[n][g] * xs[t][g])
// The int32 dot of every 64-wide group is exact on the tensor core; the fp32
// chain runs on CUDA cores in the reference's order, so the result is
// bit-identical to the GEMV and SIMT GEMM paths.
//
// Persistent CTAs (one per SM) walk 128 (tokens) x 128 (outputs) tiles; the
// ring, the TMEM buffers and their barrier phases carry over from tile to
// tile, so one tile's epilogue overlaps the next tile's loads and MMAs.
// Roles (10 warps):
//   warp 0      TMA producer: per K step of 128 bytes, a 128x128 int8 tile of
//               the activations and of the weights (2-D tensor maps, 128-byte
//               swizzle) plus the step's two groups of weight scales
//               (transposed fp32 [G][N], 1-D bulk copies) into a 4-stage ring;
//   warp 1      allocates all 512 TMEM columns; one lane issues tcgen05.mma
//               kind::i8 (M 128, N 128, K 32): two per 64-wide group, into one
//               of four TMEM accumulators (int32), and commits each group;
//   warps 2-17  epilogue: thread = token row (TMEM lane), warp w owns the
//               32 columns (w - 2) / 4 of its lane quadrant (four warps per
//               quadrant, so each scheduler has four to hide the TMEM-load and
//               conversion latencies); per group it reads the int32 dots from
//               TMEM (one 32-column load), frees the accumulator and advances
//               its 32 fp32 chains with the weight and activation scales
//               staged by the producer, then applies the output epilogue
//               (store, GEGLU pair, PLE gate).
// Up to 64 token rows the roles are transposed (TcArgs::swap): A is a tile of
// 128 weight rows and B the token rows padded to BN = 32 or 64, so a TMEM
// lane is an output and a column a token; the stage's column scales are then
// the activations' and the row scales the weights' (the chain's product
// xs * ws equals ws * xs), and the epilogue stores per (token, output).
// Waits are bounded (mbar_wait); on a timeout every role leaves its loop, the
// CTA drains the copies and MMAs it issued, and TMEM is freed.
#include <cuda.h>

#include "g4_common.cuh"
#include "g4_internal.h"
#include "g4_tc.cuh"

namespace {

constexpr int kBM = 128, kBK = 128;   // tile: tokens x K bytes per stage (outputs: BN below)
constexpr int kStages = 6;
constexpr int kTileBytesA = kBM * kBK;            // 16 KB
constexpr int kGeluSize = 4096;                   // GELU table (GEGLU / PLE epilogues), staged once
constexpr int kEpiWarps = 16;                     // 4 per TMEM lane quadrant, BN / 4 columns each
constexpr int kThreads = 64 + 32 * kEpiWarps;

// Output-tile width BN (128, 64 or 32): narrower tiles give GEMMs with few
// output columns (N = 1536, 256) enough tiles for every SM.
template <int BN>
struct TcCfg {
    static constexpr int kTmemBufs = 512 / BN > 8 ? 8 : 512 / BN;   // int32 group accumulators in flight
    static constexpr int kTmemCols = kTmemBufs * BN;                 // 512 / 512 / 256
    static constexpr int kTileBytesB = BN * kBK;
    static constexpr int kScaleBytes = 2 * BN * 4 + 2 * kBM * 4;     // two groups of weight and activation scales
    static constexpr int kOffA = 0;
    static constexpr int kOffB = kOffA + kStages * kTileBytesA;
    static constexpr int kOffS = kOffB + kStages * kTileBytesB;
    static constexpr int kOffBar = kOffS + kStages * kScaleBytes;
    // barriers: full[S], empty[S], tfull[B], tempty[B], then the TMEM address word
    static constexpr int kOffGelu = (kOffBar + (2 * kStages + 2 * kTmemBufs) * 8 + 16 + 127) & ~127;
    // GEGLU quantisation: per lane quadrant an mbarrier (its four warps) and
    // per tile parity x column block x row the row's max |x| over 16 outputs
    static constexpr int kOffQbar = kOffGelu + kGeluSize * 4;
    static constexpr int kOffAmax = kOffQbar + 64;
    static constexpr int kSmemBytes = kOffAmax + 2 * 4 * kBM * 4 + 1024;   // + 1 KB for alignment
    static constexpr int CW = BN / 4;                                    // columns per epilogue warp
    // Instruction descriptor: S32 accumulate, signed int8 A and B, both K-major,
    // N = BN (>> 3), M = 128 (>> 4).
    static constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                       ((uint32_t)(kBM >> 4) << 24);
};

static_assert(TcCfg<128>::kSmemBytes <= 227 * 1024 && TcCfg<64>::kSmemBytes <= 227 * 1024 &&
                  TcCfg<32>::kSmemBytes <= 227 * 1024,
              "shared memory budget of the GEMM tiles");

// One group's step of CW columns of the chain: acc = fma((float)d, ws * xs, acc).
template <int CW>
G4_DEV void chain(uint64_t *acc, const int (&d)[CW], const float *ws, float xv) {
    const uint64_t x2 = pk(xv, xv);
#pragma unroll
    for (int j = 0; j < CW; j += 4) {
        const float4 w4 = *(const float4 *)(ws + j);
        const uint64_t w01 = mul2(pk(w4.x, w4.y), x2), w23 = mul2(pk(w4.z, w4.w), x2);
        acc[j / 2] = fma2(pk(__int2float_rn(d[j]), __int2float_rn(d[j + 1])), w01, acc[j / 2]);
        acc[j / 2 + 1] = fma2(pk(__int2float_rn(d[j + 2]), __int2float_rn(d[j + 3])), w23, acc[j / 2 + 1]);
    }
}

struct TcArgs {
    int T, N, K;
    const float *xsT;       // [K/64][xs_stride] activation scales, group-major
    int xs_stride;          // row stride of xsT (and qsT), >= T
    const float *wsT;       // [K/64][N] weight scales, fp32
    int epi;
    float *out;
    int out_stride;
    const float *ple_u;
    int u_stride;
    const float *gelu;
    int *err;
    int8_t *qout;           // GEGLU rows quantised (BN 128 only), or NULL
    float *qs, *qsT;
    // Transposed roles (few token rows): A = 128 weight rows, B = the BN >= T
    // token rows; a TMEM lane is then an output and a column a token
    int swap;
};

template <int BN>
// 18 warps, one CTA per SM: at most 96 registers a thread (five warps share one
// scheduler's quarter of the register file)
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, const TcArgs p) {
    using C = TcCfg<BN>;
    // TMEM holds kPairs pairs of group accumulators: a K step's two groups
    // are committed, waited for and released together
    constexpr int kTmemBufs = C::kTmemBufs, kPairs = kTmemBufs / 2, CW = C::CW;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the swizzled tiles
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *full = (uint64_t *)(smem + C::kOffBar);
    uint64_t *empty = full + kStages;
    uint64_t *tfull = empty + kStages;
    uint64_t *tempty = tfull + kTmemBufs;
    uint32_t *tmem_slot = (uint32_t *)(tempty + kTmemBufs);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int steps = p.K / kBK;
    const int mt = (p.T + kBM - 1) / kBM, tiles = p.swap ? p.N / kBM : (p.N / BN) * mt;
    // persistent: this CTA takes tiles blockIdx.x, + gridDim.x, ...; the m tiles of
    // one n tile are consecutive, so CTAs sharing weights run together (L2 reuse)
    __shared__ int fail, issued, committed;

    if (tid == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1 + kEpiWarps);   // the MMA commit and every epilogue warp
        }
        for (int b = 0; b < kPairs; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], kEpiWarps);
        }
        for (int qd = 0; qd < 4; qd++) mbar_init((uint64_t *)(smem + C::kOffQbar) + qd, 4);
        mbar_fence_init();
        fail = 0;
        issued = 0;
        committed = 0;
    }
    float *gelu_s = (float *)(smem + C::kOffGelu);
    if (p.epi != EPI_STORE)
        for (int i = tid; i < kGeluSize; i += kThreads) gelu_s[i] = p.gelu[i];
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(C::kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // Programmatic dependent launch. The next kernel may be scheduled from
    // here: every CTA of this grid holds its TMEM columns already, so a
    // dependent kernel's allocation can only wait for this one, never the
    // reverse. Nothing the previous kernel writes or reads is touched before
    // it has completed (the set-up above reads only the GELU table, a model
    // constant).
    griddep_launch();
    griddep_wait();

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int k = 0;   // steps issued so far (all tiles)
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
                // A rows (token rows, or weight rows when swapped) and B rows
                const int ra = p.swap ? tile * kBM : (tile % mt) * kBM, rb = p.swap ? 0 : (tile / mt) * BN;
                // per group: BN column scales then 128 row scales (weight / activation,
                // or activation / weight when swapped)
                const float *colT = p.swap ? p.xsT + rb : p.wsT + rb, *rowT = p.swap ? p.wsT + ra : p.xsT + ra;
                const size_t colS = p.swap ? (size_t)p.xs_stride : p.N, rowS = p.swap ? p.N : (size_t)p.xs_stride;
                for (int ks = 0; ks < steps; ks++, k++) {
                    const int s = k % kStages, use = k / kStages;
                    if (use > 0 &&
                        !mbar_wait(&empty[s], (use - 1) & 1, p.err, G4D_TIMEOUT_EMPTY | ((k & 0xfff) << 8))) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], kTileBytesA + C::kTileBytesB + C::kScaleBytes);
                    tma_load_2d(smem + C::kOffA + s * kTileBytesA, &map_a, ks * kBK, ra, &full[s]);
                    tma_load_2d(smem + C::kOffB + s * C::kTileBytesB, &map_b, ks * kBK, rb, &full[s]);
                    for (int gi = 0; gi < 2; gi++) {
                        bulk_g2s_plain(smem + C::kOffS + s * C::kScaleBytes + gi * BN * 4,
                                       colT + (size_t)(2 * ks + gi) * colS, BN * 4, &full[s]);
                        bulk_g2s_plain(smem + C::kOffS + s * C::kScaleBytes + 2 * BN * 4 + gi * kBM * 4,
                                       rowT + (size_t)(2 * ks + gi) * rowS, kBM * 4, &full[s]);
                    }
                }
            }
            if (!ok) fail = 1;
            issued = k;
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint64_t dA0 = umma_desc(smem + C::kOffA, 0), dB0 = umma_desc(smem + C::kOffB, 0);
            int k = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
                for (int ks = 0; ks < steps; ks++, k++) {
                    const int s = k % kStages, pb = k % kPairs, use = k / kPairs;
                    if (!mbar_wait(&full[s], (k / kStages) & 1, p.err, G4D_TIMEOUT_FULL | ((k & 0xfff) << 8)) ||
                        (use > 0 &&
                         !mbar_wait(&tempty[pb], (use - 1) & 1, p.err, G4D_TIMEOUT_EMPTY | (0xffe << 8)))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    // descriptors: the stage's tile base plus the K offset, in 16-byte units
                    // of the start-address field (addresses stay below 2^18, so no carry)
                    const uint64_t da = dA0 + (uint64_t)((s * kTileBytesA) >> 4);
                    const uint64_t db = dB0 + (uint64_t)((s * C::kTileBytesB) >> 4);
#pragma unroll
                    for (int gi = 0; gi < 2; gi++)
#pragma unroll
                        for (int kk = 0; kk < 2; kk++) {
                            const int kb = (gi * 64 + kk * 32) >> 4;
                            mma_i8(tmem + (pb * 2 + gi) * BN, da + kb, db + kb, C::kIdesc, kk != 0);
                        }
                    mma_commit(&tfull[pb]);
                    mma_commit(&empty[s]);
                }
            }
            if (!ok) fail = 1;
            committed = k;
        }
    } else {
        // ---------------- epilogue ----------------
        // warp w: TMEM lane quadrant w % 4 (token rows), CW-column block (w - 2) / 4.
        const int e = warp - 2, q = warp & 3, cb = e >> 2;
        const int row = q * 32 + lane;
        const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(cb * CW);
        int kidx = 0;   // K steps consumed so far (all tiles)
        bool ok = true;
        int tcount = -1;   // tiles of this CTA so far (parity of the quantisation exchange)
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
            tcount++;
            const int n0 = p.swap ? tile * kBM + row : (tile / mt) * BN;   // swapped: this lane's output
            const int t = p.swap ? 0 : (tile % mt) * kBM + row;
            uint64_t acc[CW / 2];
#pragma unroll
            for (int j = 0; j < CW / 2; j++) acc[j] = 0ull;
            int d[CW];
            for (int ks = 0; ks < steps; ks++, kidx++) {
                const int pb = kidx % kPairs, s = kidx % kStages;
                // wait until the step's two groups of dots are in TMEM and its scales in smem
                const bool got =
                    mbar_wait(&tfull[pb], (kidx / kPairs) & 1, p.err, G4D_TIMEOUT_FULL | (0xffd << 8)) &&
                    mbar_wait(&full[s], (kidx / kStages) & 1, p.err, G4D_TIMEOUT_FULL | (0xffc << 8));
                if (!__all_sync(0xffffffffu, got)) {
                    if (lane == 0) fail = 1;
                    ok = false;
                    break;
                }
                tc_fence_after();
                const float *sc = (const float *)(smem + C::kOffS + s * C::kScaleBytes);
#pragma unroll 1
                for (int gi = 0; gi < 2; gi++) {
                    tmem_ld<CW>(tbase + (uint32_t)((pb * 2 + gi) * BN), d);
                    tmem_wait_ld();
                    if (gi == 1) {   // both groups read: the pair of accumulators is free
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&tempty[pb]);
                    }
                    chain<CW>(acc, d, sc + gi * BN + cb * CW, sc[2 * BN + gi * kBM + row]);
                }
                __syncwarp();   // the step's scales are consumed: release its stage
                if (lane == 0) mbar_arrive(&empty[s]);
            }
            if (!ok) continue;
            if (p.swap) {
                // lane = output n0, columns = token rows cb * CW + j (the chain's product
                // xs * ws equals ws * xs: IEEE multiplication commutes)
                const int n = n0, tb = cb * CW;
                if (p.epi == EPI_GEGLU_PAIR) {
#pragma unroll
                    for (int j = 0; j < CW / 2; j++) {
                        const float2 a = upk(acc[j]);
                        const float u0 = __shfl_down_sync(0xffffffffu, a.x, 1);   // row n + 1 = the up row
                        const float u1 = __shfl_down_sync(0xffffffffu, a.y, 1);
                        if (n & 1) continue;
                        const int t0 = tb + 2 * j;
                        if (t0 < p.T)
                            p.out[(size_t)t0 * p.out_stride + (n >> 1)] =
                                geglu_one(a.x, u0, gelu_s, kGeluSize, -8.0f, 8.0f, 4095.0f / 16.0f);
                        if (t0 + 1 < p.T)
                            p.out[(size_t)(t0 + 1) * p.out_stride + (n >> 1)] =
                                geglu_one(a.y, u1, gelu_s, kGeluSize, -8.0f, 8.0f, 4095.0f / 16.0f);
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < CW / 2; j++) {
                        const float2 a = upk(acc[j]);
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const int tt = tb + 2 * j + h;
                            if (tt >= p.T) continue;
                            float v = h ? a.y : a.x;
                            if (p.epi == EPI_PLE)
                                v = geglu_one(v, p.ple_u[(size_t)tt * p.u_stride + n], gelu_s, kGeluSize, -8.0f,
                                              8.0f, 4095.0f / 16.0f);
                            p.out[(size_t)tt * p.out_stride + n] = v;
                        }
                    }
                }
                continue;
            }
            const int nb = n0 + cb * CW;
            const bool qexch = p.epi == EPI_GEGLU_PAIR && BN == 128 && p.qout;   // every lane takes part
            if (t >= p.T && !qexch) continue;
            if (p.epi == EPI_STORE) {
                float4 *o = (float4 *)(p.out + (size_t)t * p.out_stride + nb);
#pragma unroll
                for (int j = 0; j < CW / 4; j++) {
                    const float2 a = upk(acc[2 * j]), b2 = upk(acc[2 * j + 1]);
                    o[j] = make_float4(a.x, a.y, b2.x, b2.y);
                }
            } else if (qexch) {
              if constexpr (BN == 128) {
                // this tile's 64 GEGLU outputs of a row form one quantisation group,
                // spread over the quadrant's four warps (16 each): exchange the
                // row maxima through shared memory under the quadrant's mbarrier
                float r[CW / 2];
                float m = 0.0f;
#pragma unroll
                for (int j = 0; j < CW / 2; j++) {
                    const float2 a = upk(acc[j]);
                    r[j] = geglu_one(a.x, a.y, gelu_s, kGeluSize, -8.0f, 8.0f, 4095.0f / 16.0f);
                    m = fmaxf(m, fabsf(r[j]));
                }
                float *amax = (float *)(smem + C::kOffAmax) + (tcount & 1) * 4 * kBM;
                uint64_t *qbar = (uint64_t *)(smem + C::kOffQbar) + q;
                amax[cb * kBM + row] = m;
                __syncwarp();
                if (lane == 0) mbar_arrive(qbar);
                const bool got = mbar_wait(qbar, tcount & 1, p.err, G4D_TIMEOUT_FULL | (0xffb << 8));
                if (!__all_sync(0xffffffffu, got)) {
                    if (lane == 0) fail = 1;
                    ok = false;
                    continue;
                }
                const float gm = fmaxf(fmaxf(amax[row], amax[kBM + row]), fmaxf(amax[2 * kBM + row], amax[3 * kBM + row]));
                const float sc = quant_scale(gm), inv = quant_inv(sc);
                if (t < p.T) {
                    const int K2 = p.N >> 1, g = n0 >> 7;   // 64 outputs per 128-column tile
                    uint32_t w4[CW / 8];
#pragma unroll
                    for (int j = 0; j < CW / 8; j++)
                        w4[j] = (uint32_t)(uint8_t)quant_one(r[4 * j], inv) |
                                ((uint32_t)(uint8_t)quant_one(r[4 * j + 1], inv) << 8) |
                                ((uint32_t)(uint8_t)quant_one(r[4 * j + 2], inv) << 16) |
                                ((uint32_t)(uint8_t)quant_one(r[4 * j + 3], inv) << 24);
                    *(uint4 *)(p.qout + (size_t)t * K2 + (nb >> 1)) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                    if (cb == 0) {
                        p.qs[(size_t)t * (K2 / 64) + g] = sc;
                        if (p.qsT) p.qsT[(size_t)g * p.xs_stride + t] = sc;
                    }
                }
              }
            } else if (p.epi == EPI_GEGLU_PAIR) {
                float4 *o = (float4 *)(p.out + (size_t)t * p.out_stride + (nb >> 1));
#pragma unroll
                for (int j = 0; j < CW / 8; j++) {
                    float r[4];
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const float2 a = upk(acc[4 * j + i]);
                        r[i] = geglu_one(a.x, a.y, gelu_s, kGeluSize, -8.0f, 8.0f, 4095.0f / 16.0f);
                    }
                    o[j] = make_float4(r[0], r[1], r[2], r[3]);
                }
            } else {
                float4 *o = (float4 *)(p.out + (size_t)t * p.out_stride + nb);
                const float4 *u = (const float4 *)(p.ple_u + (size_t)t * p.u_stride + nb);
#pragma unroll
                for (int j = 0; j < CW / 4; j++) {
                    const float4 u4 = u[j];
                    const float2 a = upk(acc[2 * j]), b2 = upk(acc[2 * j + 1]);
                    o[j] = make_float4(geglu_one(a.x, u4.x, gelu_s, kGeluSize, -8.0f, 8.0f, 4095.0f / 16.0f),
                                       geglu_one(a.y, u4.y, gelu_s, kGeluSize, -8.0f, 8.0f, 4095.0f / 16.0f),
                                       geglu_one(b2.x, u4.z, gelu_s, kGeluSize, -8.0f, 8.0f, 4095.0f / 16.0f),
                                       geglu_one(b2.y, u4.w, gelu_s, kGeluSize, -8.0f, 8.0f, 4095.0f / 16.0f));
                }
            }
        }
    }

    // ---------------- teardown ----------------
    __syncwarp();   // the producer and MMA lanes rejoin their warps
    tc_fence_before();
    __syncthreads();
    if (fail && tid == 0) {
        // let issued copies and committed MMAs finish before the CTA exits
        const uint64_t t0n = g4_globaltimer();
        for (int k = issued > kStages ? issued - kStages : 0; k < issued; k++)
            while (!mbar_try_wait(&full[k % kStages], (k / kStages) & 1) && g4_globaltimer() - t0n < G4_WAIT_NS) {
            }
        for (int g = committed > kPairs ? committed - kPairs : 0; g < committed; g++)
            while (!mbar_try_wait(&tfull[g % kPairs], (g / kPairs) & 1) &&
                   g4_globaltimer() - t0n < G4_WAIT_NS) {
            }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kTmemCols) : "memory");
    }
}

// ---- peak of the int8 tensor pipe -----------------------------------------------
// Back-to-back tcgen05.mma kind::i8 (M 128, N 256, K 32) from two zero tiles in
// shared memory (128-byte swizzle, as the GEMM's) into one TMEM accumulator,
// committed once at the end; one CTA per SM. Throughput does not depend on the
// operand values, so this is the measured denominator for the GEMM's int8 rate.
constexpr int kPeakN = 256;
constexpr uint32_t kPeakIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kPeakN >> 3) << 17) |
                                ((uint32_t)(kBM >> 4) << 24);
constexpr int kPeakSmem = kBM * kBK + kPeakN * kBK + 64 + 1024;

__global__ void __launch_bounds__(128, 1) k_mma_peak(int iters, int *err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *A = smem, *B = smem + kBM * kBK;
    uint64_t *bar = (uint64_t *)(B + kPeakN * kBK);
    uint32_t *slot = (uint32_t *)(bar + 1);
    const int tid = threadIdx.x, warp = tid >> 5;
    for (int i = tid; i < (kBM + kPeakN) * kBK / 16; i += 128) ((int4 *)smem)[i] = make_int4(0, 0, 0, 0);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // the zeros, visible to the tensor core
    if (tid == 0) {
        mbar_init(bar, 1);
        mbar_fence_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                     "r"(kPeakN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *slot;
    if (tid == 0) {
        const uint64_t da = umma_desc(A, 0), db = umma_desc(B, 0);
        for (int i = 0; i < iters; i++) {
            const uint64_t kb = (uint64_t)((i & 3) * 32) >> 4;   // the four 32-byte K chunks of a row
            mma_i8(tmem, da + kb, db + kb, kPeakIdesc, i != 0);
        }
        mma_commit(bar);
    }
    __syncwarp();
    mbar_wait(bar, 0, err, G4D_TIMEOUT_FULL | (0xffa << 8));   // bounded; all MMAs retired
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPeakN) : "memory");
    }
}

// ---- host side ----------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    }
    return fn;
}

// int8 [rows][K] row-major, boxes of box_rows x 128 bytes, 128-byte swizzle.
bool make_map(CUtensorMap *m, const void *base, int K, int rows, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || ((uintptr_t)base & 15) || K % 128) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void *)base, dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Output-tile width for an N-column GEMM over mt token tiles: the widest whose
// waves of tiles over the SMs cost least, counting each tile as its width plus
// a fixed per-tile overhead of about 64 columns.
int pick_bn(int N, int mt, int sms) {
    int best = 128;
    long best_cost = -1;
    for (int bn = 128; bn >= 32; bn >>= 1) {
        if (N % bn) continue;
        const long tiles = (long)(N / bn) * mt, waves = (tiles + sms - 1) / sms;
        const long cost = waves * (bn + 64);
        if (best_cost < 0 || cost < best_cost) { best = bn; best_cost = cost; }
    }
    return best;
}

template <int BN>
cudaError_t launch_bn(const CUtensorMap &ma, const CUtensorMap &mb, const TcArgs &p, int sms, cudaStream_t st,
                      bool pdl) {
    {
        cudaError_t e = g4_smem_optin((const void *)k_gemm_tc<BN>, TcCfg<BN>::kSmemBytes);
        if (e != cudaSuccess) return e;
    }
    const int tiles = p.swap ? p.N / kBM : (p.N / BN) * ((p.T + kBM - 1) / kBM);
    return g4_launch(k_gemm_tc<BN>, dim3(tiles < sms ? tiles : sms), dim3(kThreads), (size_t)TcCfg<BN>::kSmemBytes,
                     st, pdl, ma, mb, p);
}

}  // namespace

void *g4_tmap_encoder() { return (void *)encode_fn(); }

bool g4_gemm_tc_supported(const GemmArgs &a) {
    const int xs_stride = a.xs_stride > 0 ? a.xs_stride : G4_XST_STRIDE;
    return a.m.sT != nullptr && a.xsT != nullptr && a.T <= xs_stride && a.m.K % kBK == 0 && a.m.N % 32 == 0 &&
           a.T >= 1 && encode_fn() != nullptr && (a.epi == EPI_STORE || a.epi == EPI_GEGLU_PAIR || a.epi == EPI_PLE) &&
           a.dots_out == nullptr;
}

cudaError_t g4_launch_mma_peak(int iters, int *err, cudaStream_t st, double *ops) {
    if (iters < 1) return cudaErrorInvalidValue;
    cudaError_t e = g4_smem_optin((const void *)k_mma_peak, kPeakSmem);
    if (e != cudaSuccess) return e;
    const int sms = g4_device_sms();
    if (ops) *ops = 2.0 * kBM * kPeakN * 32 * (double)iters * sms;
    k_mma_peak<<<sms, 128, kPeakSmem, st>>>(iters, err);
    return cudaGetLastError();
}

bool g4_gemm_tc_swapped(const GemmArgs &a) {
    // up to 64 token rows: the weights fill the MMA's 128 rows and the tokens its N
    return g4_gemm_tc_supported(a) && a.T <= 64 && a.m.N % kBM == 0 && !a.qout;
}

cudaError_t g4_launch_gemm_tc(const GemmArgs &a, cudaStream_t st, bool pdl) {
    if (!g4_gemm_tc_supported(a)) return cudaErrorNotSupported;
    const int sms = g4_device_sms();
    const bool swap = g4_gemm_tc_swapped(a);
    const bool fuse_q = !swap && a.epi == EPI_GEGLU_PAIR && a.qout && a.qs && a.m.N % 128 == 0;
    const int bn = swap ? (a.T <= 32 ? 32 : 64) : fuse_q ? 128 : pick_bn(a.m.N, (a.T + kBM - 1) / kBM, sms);
    CUtensorMap ma, mb;
    // rows of either operand beyond its extent read as zero and are not stored
    if (swap ? (!make_map(&ma, a.m.w, a.m.K, a.m.N, kBM) || !make_map(&mb, a.xq, a.m.K, a.T, bn))
             : (!make_map(&ma, a.xq, a.m.K, a.T, kBM) || !make_map(&mb, a.m.w, a.m.K, a.m.N, bn)))
        return cudaErrorInvalidValue;
    TcArgs p{};
    p.swap = swap ? 1 : 0;
    p.T = a.T;
    p.N = a.m.N;
    p.K = a.m.K;
    p.xsT = a.xsT;
    p.xs_stride = a.xs_stride > 0 ? a.xs_stride : G4_XST_STRIDE;
    p.wsT = a.m.sT;
    p.epi = a.epi;
    p.out = a.out;
    p.out_stride = a.out_stride;
    p.ple_u = a.ple_u;
    p.u_stride = a.u_stride;
    p.gelu = a.gelu;
    p.err = a.err;
    if (fuse_q) {
        p.qout = a.qout;
        p.qs = a.qs;
        p.qsT = a.qsT;
    }
    if (bn == 128) return launch_bn<128>(ma, mb, p, sms, st, pdl);
    if (bn == 64) return launch_bn<64>(ma, mb, p, sms, st, pdl);
    return launch_bn<32>(ma, mb, p, sms, st, pdl);
}
