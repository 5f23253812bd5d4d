// g4_gemv.cu — decode-path int8 GEMV (T <= 4 token rows) with fused prologues
// and epilogues.
//
// Reference: matmul_int8 / matmul_block (gemma4.c:192-262) and the ops around
// each call site in forward/attention/logits (gemma4.c:411-522).
//
// Design (one producer warp + 8 consumer warps per CTA, one CTA per SM):
//   - Each CTA owns a contiguous range of output rows, which in the row-major
//     device layout is one contiguous byte range. The producer streams it
//     through a ring of ~16 KB stages with 1-D bulk async copies (the TMA
//     engine; large copies are what reach full HBM bandwidth on B200, ~6.8 TB/s
//     measured, where per-thread 16-byte loads stay latency-bound). A stage is
//     R whole rows plus their FP16 scales; an mbarrier counts the bytes.
//   - The producer starts at kernel entry, before griddepcontrol.wait: with
//     programmatic dependent launch the weight stream overlaps the tail of the
//     previous kernel. Only the consumers wait for the previous kernel.
//   - Consumers build the int8 activation (fused RMSNorm / residual /
//     embedding + dynamic quantisation, gemma4.c:265-279) in shared memory,
//     then each warp takes row pairs (lanes 0-15 row A, 16-31 row B, 256 bytes
//     per row per step): a 16-byte dp4a partial per lane, a quad reduction to
//     the exact int32 dot of each 64-group, and the row's fp32 chain advanced in
//     order, acc = fma((float)dot_g, ws_g * xs_g, acc) with g ascending — the
//     reference's rounding sequence (gemma4.c:218), so outputs are bit-exact
//     given the same activation. A warp releases a stage by arriving on the
//     stage's "consumed" mbarrier; there are no CTA-wide barriers in the loop.
//   - Epilogues fuse GeGLU of interleaved gate/up rows, the PLE GeGLU, and the
//     logits soft-cap with a grid-wide argmax (last-CTA ticket).
#include "g4_gemv_dev.cuh"

namespace {

constexpr int kThreads = kConsumers + 32;   // + producer warp
constexpr int kMaxT = 4;
constexpr int kRingBytes = 88 * 1024;
constexpr int kMaxStages = 8;     // ring slots
constexpr int kMaxChunks = 256;    // stages one CTA may stream (one single-use mbarrier each)

__host__ __device__ inline int round_up(int v, int a) { return (v + a - 1) / a * a; }

__host__ __device__ inline int num_stages(int K) {
    int s = kRingBytes / (stage_rows(K) * K);
    return s > kMaxStages ? kMaxStages : (s < 2 ? 2 : s);
}

struct Layout {
    int R, S, slot, sslot;
    int off_ring, off_sring, off_bars, off_xq, off_xs, off_vec, off_red, total;
};

__host__ __device__ inline Layout make_layout(int K, int T, int pro) {
    Layout L;
    const int G = K / 64;
    L.R = stage_rows(K);
    L.S = num_stages(K);
    L.slot = round_up(L.R * K, 128);
    L.sslot = round_up(L.R * G * 2, 16);
    int o = 0;
    L.off_ring = o;
    o += L.S * L.slot;
    L.off_sring = o;
    o += L.S * L.sslot;
    L.off_bars = round_up(o, 16);
    o = L.off_bars + (kMaxChunks + kMaxStages) * 8;
    L.off_xq = o;
    o += round_up(T * K, 16);
    L.off_xs = o;
    o += round_up(T * G * 4, 16);
    L.off_vec = o;
    o += (pro == PRO_NORM_QUANT || pro == PRO_RES_NORM_QUANT || pro == PRO_RES_QUANT || pro == PRO_EMBED_QUANT)
             ? G4_HIDDEN * 4
             : 0;
    L.off_red = round_up(o, 16);
    o = L.off_red + 128 * 4;
    L.total = o;
    return L;
}

template <int T, int PRO, int EPI>
__global__ void __launch_bounds__(kThreads, 2) k_gemv(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int K = a.m.K, N = a.m.N, G = K >> 6;
    const Layout L = make_layout(K, T, PRO);
    const int R = L.R, S = L.S, PPS = L.R / 2;   // pairs per stage
    uint8_t *ring = smem + L.off_ring;
    uint8_t *sring = smem + L.off_sring;
    // full[c]: stage c landed (one barrier per stage, used once, so a warp that
    // runs ahead can never observe an earlier use of the same ring slot);
    // empty[slot]: all pairs of the slot's current stage consumed (only the
    // producer waits on it, strictly in order).
    uint64_t *full = (uint64_t *)(smem + L.off_bars);
    uint64_t *empty = full + kMaxChunks;
    int8_t *xq = (int8_t *)(smem + L.off_xq);
    float *xs = (float *)(smem + L.off_xs);
    float *vec = (float *)(smem + L.off_vec);
    float *red = (float *)(smem + L.off_red);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int npairs = N >> 1;
    const int c0 = (int)((long long)blockIdx.x * npairs / gridDim.x);
    const int c1 = (int)((long long)(blockIdx.x + 1) * npairs / gridDim.x);
    const int n0 = 2 * c0, rows = 2 * (c1 - c0);
    const int nstages = (rows + R - 1) / R;

    if (nstages > kMaxChunks) {   // host sizes grids so this cannot happen
        if (tid == 0) g4_set_error(a.err, G4D_BAD_SHAPE);
        return;
    }
    __shared__ int fail, issued;   // a wait ran out; stages the producer issued
    if (tid == 0) {
        for (int i = 0; i < nstages; i++) mbar_init(&full[i], 1);
        for (int i = 0; i < S; i++) mbar_init(&empty[i], PPS);
        mbar_fence_init();
        fail = 0;
        issued = 0;
    }
    __syncthreads();
    griddep_launch();

    if (warp == kWarps) {
        // ---------------- producer ----------------
        if (lane == 0) {
            const uint64_t pol = l2_policy_evict_first();
            int c = 0;
            for (; c < nstages; c++) {
                const int slot = c % S, use = c / S;
                if (use > 0 && !mbar_wait(&empty[slot], (use - 1) & 1, a.err,
                                          G4D_TIMEOUT_EMPTY | (c << 8) | ((int)blockIdx.x << 20))) {
                    fail = 1;
                    break;
                }
                const int r0 = n0 + c * R, nr = min(R, n0 + rows - r0);
                mbar_arrive_expect_tx(&full[c], (uint32_t)(nr * K + nr * G * 2));
                bulk_g2s(ring + slot * L.slot, a.m.w + (size_t)r0 * K, (uint32_t)(nr * K), &full[c], pol);
                bulk_g2s(sring + slot * L.sslot, a.m.s + (size_t)r0 * G, (uint32_t)(nr * G * 2), &full[c], pol);
            }
            issued = c;
        }
        __syncwarp();
        bar_sync(2, kThreads);   // join the consumers (see the end of the kernel)
        if (lane == 0 && fail) drain_stages(full, issued);
        return;
    }

    // ---------------- consumers ----------------
    const int half = lane >> 4, q = lane & 15;
    griddep_wait();
    prologue<T, PRO>(a, xq, xs, vec, red);
    csync();

    float best_v = -INFINITY;
    int best_i = 0x7fffffff;
    for (int pr = warp; pr < rows / 2; pr += kWarps) {
        const int c = pr / PPS, slot = c % S;
        const int lr = 2 * (pr - c * PPS) + half;         // row within the stage
        const int n = n0 + c * R + lr;
        // a wait that runs out ends the row loop for the whole warp, which still
        // takes the consumer barriers below (no CTA deadlock on the error path)
        const bool got = mbar_wait(&full[c], 0, a.err, G4D_TIMEOUT_FULL | (c << 8) | ((int)blockIdx.x << 20));
        if (!__all_sync(0xffffffffu, got)) {
            if (lane == 0) fail = 1;
            break;
        }
        const uint8_t *wrow = ring + slot * L.slot + lr * K + q * 16;
        const uint16_t *srow = (const uint16_t *)(sring + slot * L.sslot) + lr * G;
        float acc[T];
        pair_dot<T>(wrow, srow, xq, xs, K, acc, a.dots_out ? a.dots_out + (size_t)n * G : nullptr, (size_t)N * G);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        // lanes 0-15 hold row n (even), lanes 16-31 row n (odd)
#pragma unroll
        for (int t = 0; t < T; t++) {
            const float up = __shfl_sync(0xffffffffu, acc[t], 16);
            epilogue_row<EPI>(a, t, n, acc[t], up, q == 0, best_v, best_i);
        }
    }

    if (EPI == EPI_LOGITS) {
        // first strict maximum (gemma4.c:537-541): per warp half, per CTA, then last CTA
        float *cv = red;                 // [kWarps*2]
        int *ci = (int *)(red + 64);
        if (q == 0) {
            cv[warp * 2 + half] = best_v;
            ci[warp * 2 + half] = best_i;
        }
        csync();
        __shared__ unsigned last;
        if (tid == 0) {
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int k = 0; k < kWarps * 2; k++)
                if (cv[k] > bv || (cv[k] == bv && ci[k] < bi)) { bv = cv[k]; bi = ci[k]; }
            a.argmax_part[(size_t)blockIdx.x * 2] = bv;
            a.argmax_part[(size_t)blockIdx.x * 2 + 1] = __int_as_float(bi);
            __threadfence();
            last = atomicAdd(a.ticket, 1u) == gridDim.x - 1;
        }
        csync();
        if (last && tid == 0) {
            __threadfence();
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int k = 0; k < (int)gridDim.x; k++) {
                const float v = __ldcg(&a.argmax_part[(size_t)k * 2]);
                const int ix = __float_as_int(__ldcg(&a.argmax_part[(size_t)k * 2 + 1]));
                if (v > bv || (v == bv && ix < bi)) { bv = v; bi = ix; }
            }
            a.argmax_out[0] = bi;
            *a.ticket = 0u;
        }
    }
    // all 288 threads: after it the producer lane drains in-flight copies if a wait failed
    bar_sync(2, kThreads);
}

template <int T, int PRO, int EPI>
cudaError_t launch_t(const GemvArgs &a, int grid, cudaStream_t st, bool pdl) {
    const Layout L = make_layout(a.m.K, T, PRO);
    auto kern = k_gemv<T, PRO, EPI>;
    {
        cudaError_t e = g4_smem_optin((const void *)kern, 200 * 1024);
        if (e != cudaSuccess) return e;
    }
    if (L.total > 200 * 1024) return cudaErrorInvalidValue;
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
#undef G4_CASE
    return cudaErrorInvalidValue;
}

}  // namespace

void g4_gemv_plan(GemvArgs &a, int grid) {
    (void)grid;
    a.kc = a.m.K;
    a.row_gran = 2;
    a.rb = stage_rows(a.m.K);
}

int g4_gemv_smem_bytes(const GemvArgs &a, int pro) {
    const int T = a.T <= 1 ? 1 : (a.T <= 2 ? 2 : 4);
    return make_layout(a.m.K, T, pro).total;
}

cudaError_t g4_launch_gemv(const GemvArgs &a, int pro, int epi, int grid, cudaStream_t st, bool pdl) {
    if (a.T < 1 || a.T > kMaxT || a.m.K % 256 != 0 || a.m.N % 2 != 0 || grid < 1) return cudaErrorInvalidValue;
    const int max_rows = 2 * ((a.m.N / 2 + grid - 1) / grid);
    if ((max_rows + stage_rows(a.m.K) - 1) / stage_rows(a.m.K) > kMaxChunks) return cudaErrorInvalidValue;
    if (epi == EPI_LOGITS && a.T != 1) return cudaErrorInvalidValue;
    // bulk-copy sizes and addresses must be 16-byte multiples: scale slices of
    // odd row offsets need G even or K >= 512
    if ((a.m.K / 64) * 2 % 16 != 0 && stage_rows(a.m.K) % 8 != 0) return cudaErrorInvalidValue;
    switch (a.T) {
    case 1: return launch_pe<1>(a, pro, epi, grid, st, pdl);
    case 2: return launch_pe<2>(a, pro, epi, grid, st, pdl);
    case 3: return launch_pe<3>(a, pro, epi, grid, st, pdl);
    default: return launch_pe<4>(a, pro, epi, grid, st, pdl);
    }
}
