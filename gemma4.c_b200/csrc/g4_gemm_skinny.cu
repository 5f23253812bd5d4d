// g4_gemm_skinny.cu — int8 GEMM over a few token rows (T <= 64): the
// multi-sequence decode step (one row per sequence) and short chunks.
//
// Reference: matmul_int8 (gemma4.c:192-262) per token row, with the exact
// arithmetic of every other path: the int32 dot of each 64-wide group, then
// the fp32 chain acc = fma((float)dot_g, ws[n][g] * xs[t][g], acc) over g
// ascending, so the outputs are bit-identical to the GEMV, SIMT and tcgen05
// paths.
//
// With T <= 64 rows the GEMM does 2T operations per weight byte and is bound
// by the weight stream; what limits a 128-row tensor-core tile here is that a
// CTA walks all K groups in sequence (the chain must run g ascending), so the
// weight stream only covers the SMs if a CTA owns few output rows. Here the
// work unit is a block of 16 x WM consecutive output rows (one contiguous byte
// run of W) x every token row; persistent CTAs walk blocks blockIdx.x,
// + gridDim.x, ... with one ring whose phases run on from block to block:
//   - one producer lane, per stage of GS = 8 groups (4 when K % 512 != 0):
//     the block's weight tile (16 WM rows x 64 GS bytes; the int8 matrix is
//     viewed as 16-bit elements so that one box row, i.e. one TMA row
//     request, carries 512 bytes: 64-byte rows made the copy engine the
//     limiter), the activation tile (Tp token rows x 64 GS bytes; rows >= T
//     are zero-filled by the tensor map), and the groups' weight and
//     activation scales (fp32, group-major). The weight boxes of the first
//     stages are issued before waiting for the previous kernel (programmatic
//     dependent launch): they do not depend on it.
//   - consumer warp (rb, tg): output rows 16 rb .. 16 rb + 15 of the block x
//     token rows 8 NT tg ..; per group and 8-token tile two mma.sync
//     m16n8k32 (s8 x s8 -> s32) give the exact group dots in registers, and
//     the lane advances its four fp32 chains right away (packed f32x2, each
//     lane of the pair rounds like fmaf). The legacy mma.sync path runs at
//     ~60-80 cycles per m16n8k32 per scheduler on sm_100a, which is what
//     bounds this kernel (measured per stage); for wide N the tcgen05 GEMM
//     with transposed roles takes over (g4_gemm_skinny_preferred).
// Fragment order: the int32 dot does not depend on the order of its 64
// products, so a lane loads 16 contiguous bytes of its weight row (bytes
// 16 q .. 16 q + 15 of the group, q = lane % 4) and of its token row and
// feeds words 0-1 to the first MMA and words 2-3 to the second. A and B see
// the same byte for every k slot (the slot's k depends only on lane % 4 in
// both fragment layouts), so each MMA pair sums exactly the group's products.
#include <cuda.h>

#include "../../include/g4cuda.h"
#include "g4_common.cuh"
#include "g4_internal.h"

namespace {

constexpr int kMaxGS = 8;         // groups per stage (a box row of up to 512 bytes)
constexpr int kMaxWarps = 15;     // consumer warps per CTA (+ the producer: 4 warps per scheduler)
constexpr int kStageBudget = 160 * 1024;
constexpr int kSmemMax = 200 * 1024;   // opt-in size (launches use less; the ring depth varies per shape)

struct SkArgs {
    int T, N, K;
    int tp;                 // token rows staged per group (multiple of 8)
    int wm, wt;             // consumer warps along output rows / token rows
    int stages;
    int gs;                 // groups per stage (8, or 4 when K % 512 != 0)
    uint32_t stage_bytes, off_x, off_ws, off_xs;
    int epi;
    float *out;
    int out_stride;
    const float *ple_u;
    int u_stride;
    const float *gelu;
    int *err;
};

G4_DEV void tma2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
G4_DEV void tma2d_hint(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
        "%3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// d += A (16 x 32, s8, row) * B (32 x 8, s8, col), int32 accumulate.
G4_DEV void mma_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

G4_DEV void emit(const SkArgs &p, int t, int n, float v) {
    if (p.epi == EPI_PLE)
        v = geglu_one(v, p.ple_u[(size_t)t * p.u_stride + n], p.gelu, 4096, -8.0f, 8.0f, 4095.0f / 16.0f);
    p.out[(size_t)t * p.out_stride + n] = v;
}

template <int NT>
__global__ void __launch_bounds__(32 * (kMaxWarps + 1), 1)
    k_gemm_skinny(const __grid_constant__ CUtensorMap mw, const __grid_constant__ CUtensorMap mx,
                  const __grid_constant__ CUtensorMap mws, const __grid_constant__ CUtensorMap mxs, const SkArgs p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 127) & ~(uintptr_t)127);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nc = p.wm * p.wt, RB = 16 * p.wm;
    const int GS = p.gs, RW = 64 * GS;   // a staged row: GS groups of 64 bytes
    constexpr int kUnroll = NT == 4 ? 2 : 4;
    const int nst = p.K / RW, S = p.stages;
    // persistent: row blocks blockIdx.x, + gridDim.x, ...; the ring and its
    // barrier phases run on across blocks (global stage counter c)
    const int nblk = p.N / RB;
    const int my_blocks = (nblk - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
    const int total = my_blocks * nst;
    uint64_t *full = (uint64_t *)(smem + (size_t)S * p.stage_bytes);
    uint64_t *empty = full + S;
    if (tid == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], nc);
        }
        mbar_fence_init();
    }
    __syncthreads();
    griddep_launch();

    if (warp == nc) {
        // ---------------- producer ----------------
        if (lane == 0) {
            const uint64_t pol = l2_policy_evict_first();
            const int pre = total < S ? total : S;
            int issued = 0;
            auto weights = [&](int c) {
                const int s = c % S, st = c % nst, r0 = ((int)blockIdx.x + (c / nst) * (int)gridDim.x) * RB;
                uint8_t *b = smem + (size_t)s * p.stage_bytes;
                mbar_arrive_expect_tx(&full[s], p.stage_bytes);
                // the int8 rows are viewed as 16-bit elements: x counts byte pairs
                tma2d_hint(b, &mw, st * RW / 2, r0, &full[s], pol);
                tma2d(b + p.off_ws, &mws, r0, st * GS, &full[s]);
            };
            for (int c = 0; c < pre; c++) weights(c);
            griddep_wait();   // activations and their scales come from the previous kernel
            for (int c = 0; c < total; c++) {
                const int s = c % S, st = c % nst;
                if (c >= pre) {
                    if (!mbar_wait(&empty[s], ((c / S) - 1) & 1, p.err, G4D_TIMEOUT_EMPTY | ((c & 0xfff) << 8))) break;
                    weights(c);
                }
                uint8_t *b = smem + (size_t)s * p.stage_bytes;
                tma2d(b + p.off_x, &mx, st * RW / 2, 0, &full[s]);
                tma2d(b + p.off_xs, &mxs, 0, st * GS, &full[s]);
                issued = c + 1;
            }
            // Let every copy land before the CTA's shared memory goes away (after a
            // consumer timeout the consumers may have left early). Stages [0, pre) were
            // armed before the loop, so they count too; bounded by one deadline.
            const int armed = issued > pre ? issued : pre;
            const uint64_t t0 = g4_globaltimer();
            for (int k = armed > S ? armed - S : 0; k < armed; k++)
                while (!mbar_try_wait(&full[k % S], (k / S) & 1) && g4_globaltimer() - t0 < G4_WAIT_NS) {
                }
        }
        __syncwarp();
        return;
    }

    // ---------------- consumers ----------------
    const int rb = warp % p.wm, tg = warp / p.wm;
    const int gid = lane >> 2, q = lane & 3;
    griddep_wait();   // the previous kernel may still read what the epilogues overwrite
    for (int bi = 0, c = 0; bi < my_blocks; bi++) {
        uint64_t acc_lo[NT], acc_hi[NT];   // rows gid / gid + 8, token rows 2q and 2q + 1 of each tile
#pragma unroll
        for (int j = 0; j < NT; j++) acc_lo[j] = acc_hi[j] = pk(0.0f, 0.0f);
        for (int st = 0; st < nst; st++, c++) {
            const int s = c % S;
            const bool got = mbar_wait(&full[s], (c / S) & 1, p.err, G4D_TIMEOUT_FULL | ((c & 0xfff) << 8));
            if (!__all_sync(0xffffffffu, got)) return;
            const uint8_t *b = smem + (size_t)s * p.stage_bytes;
            const uint8_t *wb = b + (rb * 16 + gid) * RW + q * 16;
            const uint8_t *xb = b + p.off_x + (tg * 8 * NT + gid) * RW + q * 16;
            const float *wsb = (const float *)(b + p.off_ws) + rb * 16 + gid;
            const float *xsb = (const float *)(b + p.off_xs) + tg * 8 * NT + 2 * q;
#pragma unroll(kUnroll)
            for (int gi = 0; gi < GS; gi++) {
                const uint4 alo = *(const uint4 *)(wb + gi * 64);
                const uint4 ahi = *(const uint4 *)(wb + gi * 64 + 8 * RW);
                const float wlo = wsb[gi * RB], whi = wsb[gi * RB + 8];
#pragma unroll
                for (int j = 0; j < NT; j++) {
                    const uint4 bx = *(const uint4 *)(xb + gi * 64 + 8 * j * RW);
                    int d[4] = {0, 0, 0, 0};
                    mma_s8(d, alo.x, ahi.x, alo.y, ahi.y, bx.x, bx.y);
                    mma_s8(d, alo.z, ahi.z, alo.w, ahi.w, bx.z, bx.w);
                    const float2 xv = *(const float2 *)(xsb + gi * p.tp + 8 * j);
                    const uint64_t x2 = pk(xv.x, xv.y);
                    acc_lo[j] =
                        fma2(pk(__int2float_rn(d[0]), __int2float_rn(d[1])), mul2(pk(wlo, wlo), x2), acc_lo[j]);
                    acc_hi[j] =
                        fma2(pk(__int2float_rn(d[2]), __int2float_rn(d[3])), mul2(pk(whi, whi), x2), acc_hi[j]);
                }
            }
            __syncwarp();   // this warp's reads of the stage are done
            if (lane == 0) mbar_arrive(&empty[s]);
        }

        // ---------------- epilogue of the block ----------------
        const int n_lo = ((int)blockIdx.x + bi * (int)gridDim.x) * RB + rb * 16 + gid;
#pragma unroll
        for (int j = 0; j < NT; j++) {
            const int t0 = tg * 8 * NT + 8 * j + 2 * q;
            const float2 lo = upk(acc_lo[j]), hi = upk(acc_hi[j]);
            if (p.epi == EPI_GEGLU_PAIR) {
                // interleaved rows: gate n (even gid) and up n + 1 live four lanes apart
                const float ulo0 = __shfl_down_sync(0xffffffffu, lo.x, 4);
                const float ulo1 = __shfl_down_sync(0xffffffffu, lo.y, 4);
                const float uhi0 = __shfl_down_sync(0xffffffffu, hi.x, 4);
                const float uhi1 = __shfl_down_sync(0xffffffffu, hi.y, 4);
                if (gid & 1) continue;
                const float *tab = p.gelu;
                const int h_lo = n_lo >> 1, h_hi = (n_lo + 8) >> 1;
                if (t0 < p.T) {
                    p.out[(size_t)t0 * p.out_stride + h_lo] =
                        geglu_one(lo.x, ulo0, tab, 4096, -8.0f, 8.0f, 4095.0f / 16.0f);
                    p.out[(size_t)t0 * p.out_stride + h_hi] =
                        geglu_one(hi.x, uhi0, tab, 4096, -8.0f, 8.0f, 4095.0f / 16.0f);
                }
                if (t0 + 1 < p.T) {
                    p.out[(size_t)(t0 + 1) * p.out_stride + h_lo] =
                        geglu_one(lo.y, ulo1, tab, 4096, -8.0f, 8.0f, 4095.0f / 16.0f);
                    p.out[(size_t)(t0 + 1) * p.out_stride + h_hi] =
                        geglu_one(hi.y, uhi1, tab, 4096, -8.0f, 8.0f, 4095.0f / 16.0f);
                }
            } else {
                if (t0 < p.T) {
                    emit(p, t0, n_lo, lo.x);
                    emit(p, t0, n_lo + 8, hi.x);
                }
                if (t0 + 1 < p.T) {
                    emit(p, t0 + 1, n_lo, lo.y);
                    emit(p, t0 + 1, n_lo + 8, hi.y);
                }
            }
        }
    }
}

// ---- host side ----------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// Row-major [rows][cols] of `esize`-byte elements (row stride `stride` bytes),
// boxes of box_rows x box_cols, no swizzle; out-of-range rows read as zero.
bool make_map2d(CUtensorMap *m, CUtensorMapDataType type, const void *base, int cols, int rows, size_t stride,
                int box_cols, int box_rows) {
    EncodeTiledFn fn = (EncodeTiledFn)g4_tmap_encoder();
    if (!fn || ((uintptr_t)base & 15) || (stride & 15)) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)stride};
    const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, type, 2, (void *)base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Tiling for an N-output GEMM over T token rows (sweeps on the B200): the
// widest row block (16 wm rows; fewer re-reads of the activation tile per
// weight byte) that still leaves about half an SM's worth of blocks per SM
// pair, i.e. >= sms / 2 blocks; then the fewest 8-token tiles per warp (nt)
// that keep the CTA at 4 consumer warps (one row block wide) or 8.
void pick_tiling(int N, int T, int sms, int *wm_out, int *nt_out) {
    int wm = 1;
    for (int w = 8; w > 1; w >>= 1)
        if (N % (16 * w) == 0 && N / (16 * w) >= sms / 2) {
            wm = w;
            break;
        }
    const int cap = wm <= 2 ? 4 : 8;
    int nt = 1;
    while (nt < 4 && wm * ((T + 8 * nt - 1) / (8 * nt)) > cap) nt <<= 1;
    while (wm > 1 && wm * ((T + 8 * nt - 1) / (8 * nt)) > kMaxWarps) wm >>= 1;
    *wm_out = wm;
    *nt_out = nt;
}

// Launch geometry of an N x K GEMM over T token rows (wm, nt: 0 = chosen from
// the shape): tiling, staged layout and ring depth into p, threads per CTA,
// dynamic shared memory. False when the combination does not fit.
bool plan(int N, int K, int T, int sms, int wm, int nt, SkArgs &p, int &threads, int &smem) {
    if (T < 1 || T > G4_SKINNY_MAX_T || K % 256 || N % 16) return false;
    if (wm <= 0 || nt <= 0) {
        int w, n;
        pick_tiling(N, T, sms, &w, &n);
        if (wm <= 0) wm = w;
        if (nt <= 0) nt = n;
    }
    if (nt != 1 && nt != 2 && nt != 4) return false;
    const int wt = (T + 8 * nt - 1) / (8 * nt);
    if (wm * wt > kMaxWarps || N % (16 * wm)) return false;
    p.T = T;
    p.N = N;
    p.K = K;
    p.tp = wt * 8 * nt;
    p.wm = wm;
    p.wt = wt;
    const int RB = 16 * wm;
    p.gs = K % (64 * kMaxGS) == 0 ? kMaxGS : 4;
    const int RW = 64 * p.gs;
    p.off_x = (uint32_t)(RB * RW);
    p.off_ws = p.off_x + (uint32_t)(p.tp * RW);
    p.off_xs = p.off_ws + (uint32_t)(p.gs * RB * 4);
    p.stage_bytes = p.off_xs + (uint32_t)(p.gs * p.tp * 4);
    const int stages = kStageBudget / (int)p.stage_bytes;
    p.stages = stages < 2 ? 2 : stages > 8 ? 8 : stages;
    threads = 32 * (p.wm * p.wt + 1);
    smem = p.stages * (int)p.stage_bytes + 2 * p.stages * 8 + 128;
    return smem <= kSmemMax;
}

template <int NT>
cudaError_t launch_nt(const CUtensorMap (&maps)[4], const SkArgs &p, int blocks, cudaStream_t st, bool pdl) {
    const int threads = 32 * (p.wm * p.wt + 1);
    const int smem = p.stages * (int)p.stage_bytes + 2 * p.stages * 8 + 128;
    if (smem > kSmemMax) return cudaErrorInvalidValue;
    cudaError_t e = g4_smem_optin((const void *)k_gemm_skinny<NT>, kSmemMax);
    if (e != cudaSuccess) return e;
    // persistent CTAs: as many as fit on the SMs (two when the ring and the
    // register file allow)
    const int per_sm = smem <= 110 * 1024 && threads <= 256 ? 2 : 1, cap = per_sm * g4_device_sms();
    return g4_launch(k_gemm_skinny<NT>, dim3(blocks < cap ? blocks : cap), dim3(threads), (size_t)smem, st, pdl,
                     maps[0], maps[1], maps[2], maps[3], p);
}

}  // namespace

bool g4_gemm_skinny_supported(const GemmArgs &a) {
    return a.T >= 1 && a.T <= G4_SKINNY_MAX_T && a.m.sT != nullptr && a.xsT != nullptr && a.m.K % 256 == 0 &&
           a.m.N % 16 == 0 && (a.epi == EPI_STORE || a.epi == EPI_GEGLU_PAIR || a.epi == EPI_PLE) &&
           a.dots_out == nullptr && g4_tmap_encoder() != nullptr;
}

bool g4_gemm_skinny_preferred(const GemmArgs &a) {
    // measured against the tcgen05 GEMM with transposed roles (128 weight rows x
    // the token rows): faster on every shape with N < 8192 and on all shapes up
    // to 8 token rows; the lm_head, the gate/up and the per-layer model
    // projection (N >= 8192) at 9-64 rows go to the tensor cores
    return g4_gemm_skinny_supported(a) && (a.T <= 8 || a.m.N < 8192);
}

cudaError_t g4_launch_gemm_skinny(const GemmArgs &a, cudaStream_t st, bool pdl, int wm, int nt) {
    if (!g4_gemm_skinny_supported(a)) return cudaErrorNotSupported;
    SkArgs p{};
    int threads = 0, smem = 0;
    if (!plan(a.m.N, a.m.K, a.T, g4_device_sms(), wm, nt, p, threads, smem)) return cudaErrorInvalidValue;
    nt = p.tp / (8 * p.wt);
    const int RB = 16 * p.wm, G = a.m.K / 64, RW = 64 * p.gs;
    p.epi = a.epi;
    p.out = a.out;
    p.out_stride = a.out_stride;
    p.ple_u = a.ple_u;
    p.u_stride = a.u_stride;
    p.gelu = a.gelu;
    p.err = a.err;
    CUtensorMap maps[4];
    // the int8 matrices as 16-bit elements, so that one box row carries 512 bytes
    if (!make_map2d(&maps[0], CU_TENSOR_MAP_DATA_TYPE_UINT16, a.m.w, a.m.K / 2, a.m.N, (size_t)a.m.K, RW / 2, RB) ||
        !make_map2d(&maps[1], CU_TENSOR_MAP_DATA_TYPE_UINT16, a.xq, a.m.K / 2, a.T, (size_t)a.m.K, RW / 2, p.tp) ||
        !make_map2d(&maps[2], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.m.sT, a.m.N, G, (size_t)a.m.N * 4, RB, p.gs) ||
        !make_map2d(&maps[3], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.xsT, G4_XST_STRIDE, G, (size_t)G4_XST_STRIDE * 4,
                    p.tp, p.gs))
        return cudaErrorInvalidValue;
    const int blocks = a.m.N / RB;
    switch (nt) {
    case 4: return launch_nt<4>(maps, p, blocks, st, pdl);
    case 2: return launch_nt<2>(maps, p, blocks, st, pdl);
    default: return launch_nt<1>(maps, p, blocks, st, pdl);
    }
}

// Launch geometry of the small-batch GEMM for an N x K matrix over T token rows
// as the engine would run it (host only: no CUDA call beyond the SM count).
extern "C" int g4_skinny_plan(int N, int K, int T, int *wm, int *nt, int *stages, int *threads, int *smem_bytes) {
    SkArgs p{};
    int th = 0, sm = 0;
    if (!plan(N, K, T, g4_device_sms(), 0, 0, p, th, sm)) return G4_ERR_INVALID;
    if (wm) *wm = p.wm;
    if (nt) *nt = p.tp / (8 * p.wt);
    if (stages) *stages = p.stages;
    if (threads) *threads = th;
    if (smem_bytes) *smem_bytes = sm;
    return G4_OK;
}
