// g4_gemm_simt.cu — prefill int8 GEMM, portable SIMT version (dp4a).
//
// Reference: matmul_int8 (gemma4.c:192-262) over T token rows. Same exact
// arithmetic as the decode GEMV: int32 dot per (token, row, 64-group), then an
// fp32 chain acc = fma((float)dot_g, ws_g * xs_g, acc) with g ascending.
//
// Tile: 64 tokens x 64 output rows, one 64-wide K group per step, cp.async
// double buffering, 256 threads each owning 4 tokens x 4 rows. This kernel is
// the correctness baseline and the fallback for shapes the tensor-core GEMM
// does not cover.
#include "g4_common.cuh"
#include "g4_internal.h"

namespace {

constexpr int BM = 64, BN = 64, LDA = 80;  // padded row stride (bytes): conflict-free int4 reads

G4_DEV void cp_async16(void *dst, const void *src, bool pred) {
    uint32_t d = smem_u32(dst);
    int n = pred ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
}
G4_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
G4_DEV void cp_async_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__global__ void __launch_bounds__(256) k_gemm_simt(const GemmArgs a) {
    __shared__ __align__(16) uint8_t As[2][BM * LDA];
    __shared__ __align__(16) uint8_t Bs[2][BN * LDA];
    __shared__ float xs_s[2][BM];
    __shared__ float ws_s[2][BN];

    const int K = a.m.K, N = a.m.N, G = K / 64, T = a.T;
    const int n_base = blockIdx.x * BN, t_base = blockIdx.y * BM;
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;

    griddep_launch();
    griddep_wait();

    // loader mapping: thread -> (row = tid / 4, 16-byte quarter = tid % 4)
    const int lr = tid >> 2, lq = tid & 3;
    auto load = [&](int buf, int g) {
        const int t = t_base + lr;
        const bool tv = t < T;
        cp_async16(&As[buf][lr * LDA + lq * 16], a.xq + (size_t)(tv ? t : 0) * K + g * 64 + lq * 16, tv);
        cp_async16(&Bs[buf][lr * LDA + lq * 16], a.m.w + (size_t)(n_base + lr) * K + g * 64 + lq * 16, true);
        cp_async_commit();
        if (tid < BM) {
            int tt = t_base + tid;
            xs_s[buf][tid] = tt < T ? a.xs[(size_t)tt * G + g] : 0.0f;
        } else if (tid < BM + BN) {
            int r = tid - BM;
            ws_s[buf][r] = h2f(a.m.s[(size_t)(n_base + r) * G + g]);
        }
    };

    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int jj = 0; jj < 4; jj++) acc[i][jj] = 0.0f;

    load(0, 0);
    for (int g = 0; g < G; g++) {
        const int buf = g & 1;
        cp_async_wait0();
        __syncthreads();
        if (g + 1 < G) load(buf ^ 1, g + 1);

        int d[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int jj = 0; jj < 4; jj++) d[i][jj] = 0;
#pragma unroll
        for (int k = 0; k < 64; k += 16) {
            int4 xa[4], wb[4];
#pragma unroll
            for (int i = 0; i < 4; i++) xa[i] = *(const int4 *)&As[buf][(ty * 4 + i) * LDA + k];
#pragma unroll
            for (int jj = 0; jj < 4; jj++) wb[jj] = *(const int4 *)&Bs[buf][(tx + 16 * jj) * LDA + k];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int jj = 0; jj < 4; jj++) {
                    int v = d[i][jj];
                    v = dp4a((uint32_t)xa[i].x, (uint32_t)wb[jj].x, v);
                    v = dp4a((uint32_t)xa[i].y, (uint32_t)wb[jj].y, v);
                    v = dp4a((uint32_t)xa[i].z, (uint32_t)wb[jj].z, v);
                    v = dp4a((uint32_t)xa[i].w, (uint32_t)wb[jj].w, v);
                    d[i][jj] = v;
                }
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float xsv = xs_s[buf][ty * 4 + i];
#pragma unroll
            for (int jj = 0; jj < 4; jj++) {
                const float scale = __fmul_rn(ws_s[buf][tx + 16 * jj], xsv);
                acc[i][jj] = __fmaf_rn(__int2float_rn(d[i][jj]), scale, acc[i][jj]);
            }
        }
        if (a.dots_out) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int t = t_base + ty * 4 + i;
                if (t < T)
#pragma unroll
                    for (int jj = 0; jj < 4; jj++)
                        a.dots_out[((size_t)t * N + n_base + tx + 16 * jj) * G + g] = d[i][jj];
            }
        }
    }

    // epilogue
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int t = t_base + ty * 4 + i;
#pragma unroll
        for (int jj = 0; jj < 4; jj++) {
            const int n = n_base + tx + 16 * jj;
            const float v = acc[i][jj];
            if (a.epi == EPI_GEGLU_PAIR) {
                // row n+1 (the up row) lives in the neighbouring lane
                float up = __shfl_down_sync(0xffffffffu, v, 1);
                if (t < T && (n & 1) == 0)
                    a.out[(size_t)t * a.out_stride + (n >> 1)] =
                        geglu_one(v, up, a.gelu, 4096, -8.0f, 8.0f, 4095.0f / 16.0f);
            } else if (t < T) {
                if (a.epi == EPI_PLE)
                    a.out[(size_t)t * a.out_stride + n] =
                        geglu_one(v, a.ple_u[(size_t)t * a.u_stride + n], a.gelu, 4096, -8.0f, 8.0f, 4095.0f / 16.0f);
                else
                    a.out[(size_t)t * a.out_stride + n] = v;
            }
        }
    }
}

}  // namespace

cudaError_t g4_launch_gemm_simt(const GemmArgs &a, cudaStream_t st, bool pdl) {
    if (a.m.N % BN != 0 || a.m.K % 64 != 0 || a.T < 1) return cudaErrorInvalidValue;
    dim3 grid(a.m.N / BN, (a.T + BM - 1) / BM);
    return g4_launch(k_gemm_simt, grid, dim3(256), 0, st, pdl, a);
}

cudaError_t g4_launch_gemm(const GemmArgs &a, cudaStream_t st, bool pdl) { return g4_launch_gemm_simt(a, st, pdl); }
