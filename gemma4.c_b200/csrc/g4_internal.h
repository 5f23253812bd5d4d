// g4_internal.h — structures shared by the g4cuda kernels and the host engine.
//
// Device weight layout (repacked once at load from the file's 16-row-block
// layout, exporter.py:304-316):
//   - every int8 matrix is row-major W[N][K] (K contiguous), so a row is one
//     contiguous byte run for the decode GEMV's bulk copies and K-major tiles
//     for the prefill GEMM;
//   - its FP16 scales are row-major S[N][K/64];
//   - fused matrices: QKV rows are q | k | v concatenated (layers 0-14), and
//     gate/up rows are interleaved (row 2i = gate i, 2i+1 = up i) so one
//     GEMV/GEMM produces both halves of every GeGLU pair.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "g4_format.h"

// Device-side error codes written to the context's error word (reported by the
// host as G4_ERR_DEVICE). Wait timeouts also carry where they gave up:
// bits 8-19 the stage index, bits 20-31 the CTA.
enum : int {
    G4D_OK = 0,
    G4D_TIMEOUT_FULL = 1,   // consumer waited too long for a weight stage
    G4D_TIMEOUT_EMPTY = 2,  // producer waited too long for a free stage
    G4D_BAD_TOKEN = 3,      // token id outside the vocabulary
    G4D_BAD_SHAPE = 4,
};

struct DMat {
    const int8_t *w;     // [N][K]
    const uint16_t *s;   // [N][K/64] fp16 bits
    const float *sT;     // [K/64][N] the same scales as fp32, group-major (tensor-core GEMM), or NULL
    int N, K;
};

// ---- GEMV (decode, T <= 4 tokens) ------------------------------------------
enum GemvPro : int {
    PRO_QUANT = 0,          // x = src
    PRO_LOADQ = 1,          // xq/xs already quantised in global memory
    PRO_NORM_QUANT = 2,     // x = rmsnorm(src, w_pre)
    PRO_RES_NORM_QUANT = 3, // r' = (res_in + rmsnorm(src, w_post)) * scalar; x = rmsnorm(r', w_pre)
    PRO_RES_QUANT = 4,      // r' = res_in + rmsnorm(src, w_post); x = r'
    PRO_EMBED_QUANT = 5,    // x = embed(token) * sqrt(1536) (written to res_out); PLE rows gathered
};
enum GemvEpi : int {
    EPI_STORE = 0,      // out[t][n] = acc
    EPI_GEGLU_PAIR = 1, // interleaved gate/up rows: out[t][n/2] = geglu(gate, up)
    EPI_PLE = 2,        // out[t][n] = geglu(acc, u[t][n])
    EPI_LOGITS = 3,     // out[t][n] = 30 tanh(acc/30) and argmax over n
};

struct GemvArgs {
    DMat m;
    int T;
    int rb;                 // rows per batch (stage = rb rows x kc bytes)
    int kc;                 // K-chunk bytes per stage
    int row_gran;           // row split granularity (1 or 2)
    // prologue
    const float *src;       // [T][src_stride]
    int src_stride;
    const int8_t *xq_in;    // PRO_LOADQ: [T][K]
    const float *xs_in;     //            [T][K/64]
    const float *w_post;    // norm weights
    const float *w_pre;
    const float *res_in;    // [T][1536]
    float *res_out;         // written by block 0
    const float *scalar;    // layer_scalar (device), NULL = 1
    const int *tokens;      // PRO_EMBED_QUANT
    DMat embed;             //   token embedding table (row-major)
    DMat embed_ple;         //   per-layer embedding table
    float *ple_emb;         //   [T][8960] gathered, x16
    float embed_mult, ple_mult;
    float eps;
    // epilogue
    float *out;
    int out_stride;
    const float *ple_u;     // EPI_PLE: [T][u_stride]
    int u_stride;
    const float *gelu;      // 4096-entry table
    float *argmax_part;     // EPI_LOGITS: [grid][T][2] (value, index as float bits)
    int *argmax_out;        // [T]
    unsigned *ticket;
    int32_t *dots_out;      // optional debug: int32 per (t, n, g)
    int *err;
    int strict;             // reference-order (sequential) RMSNorm sums
};

// ---- GEMM (prefill, T > 4) -------------------------------------------------
constexpr int G4_XST_STRIDE = G4_BATCH;
// token rows of one tensor-core GEMM outside the engine (kernel tests and the
// prefill-GEMM sweep of benchmark config 3)
constexpr int G4_GEMM_MAX_T = 16384;
// one prefill-attention partial: rows x (hd outputs) + row max + row sum, for
// 64 rows at hd 256 (32 rows at hd 512 need less)
constexpr int G4_PRE_PART_SLOT = 64 * (256 + 2);   // row stride of group-major activation scales

struct GemmArgs {
    DMat m;
    int T;
    const int8_t *xq;       // [T][K]
    const float *xs;        // [T][K/64]
    const float *xsT;       // [K/64][xs_stride] the same scales group-major (tensor-core path), or NULL
    int xs_stride;          // row stride of xsT / qsT; 0 = G4_XST_STRIDE (the engine's 512-row chunks)
    int epi;                // GemvEpi subset: STORE, GEGLU_PAIR, PLE
    float *out;
    int out_stride;
    const float *ple_u;
    int u_stride;
    const float *gelu;
    int32_t *dots_out;      // optional debug
    int *err;
    // EPI_GEGLU_PAIR on the tensor-core path: quantise the GEGLU rows for the
    // next GEMM (quantize, gemma4.c:265-279) into qout [T][N/2], qs [T][N/128]
    // and qsT (group-major) instead of storing them as fp32; NULL = store
    int8_t *qout;
    float *qs, *qsT;
};

// Small-batch GEMM (g4_gemm_skinny.cu): T <= G4_SKINNY_MAX_T token rows.
constexpr int G4_SKINNY_MAX_T = 64;
bool g4_gemm_tc_swapped(const GemmArgs &a);   // the tcgen05 GEMM runs with transposed roles (T <= 64)
bool g4_gemm_skinny_supported(const GemmArgs &a);
bool g4_gemm_skinny_preferred(const GemmArgs &a);   // supported and faster than the tcgen05 GEMM
// wm: output rows per block / 16, nt: 8-token tiles per warp (0 = chosen from the shape)
cudaError_t g4_launch_gemm_skinny(const GemmArgs &a, cudaStream_t st, bool pdl, int wm = 0, int nt = 0);
// Peak of the int8 tensor pipe (back-to-back tcgen05 kind::i8 MMAs on every SM);
// *ops receives the int8 operations of the launch
cudaError_t g4_launch_mma_peak(int iters, int *err, cudaStream_t st, double *ops);
// cuTensorMapEncodeTiled from the driver (NULL if unavailable)
void *g4_tmap_encoder();

// ---- attention ---------------------------------------------------------------
struct AttnArgs {
    int hd;                 // 256 or 512
    int pairs;              // rotated pairs (128 sliding, 64 global)
    int window;             // 512 for sliding layers, 0 = global
    int mask;               // ring slots - 1
    int T;                  // tokens in the chunk
    int start_pos;          // host-side start (prefill) ...
    const int *pos_dev;     // ... or device-side position (decode graphs); used when non-NULL
    float *qkv;             // [T][qkv_stride]: q (heads*hd) [| k hd | v hd]
    int qkv_stride;
    int has_kv;             // this layer owns (writes) the cache
    const float *q_norm, *k_norm;
    const float *rope_cos, *rope_sin;   // [131072][pairs]
    float *kcache, *vcache;             // [ring][hd]
    float *part;            // decode split partials [splits][8][hd + 4]: m, l, pad, pad, o[hd]
    float *out;             // [T][8*hd]
    int8_t *xq;             // decode combine: quantised output [8*hd]
    float *xs;
    int *err;
    int strict;             // reference-order norms / softmax / value sums
    float *scores;          // strict: [T][8][score_stride] scratch
    int score_stride;
    // multi-sequence batches (g4_forward_batch): row t belongs to sequence
    // row_seq[t] at position row_pos[t]; sequence s's ring starts seq_stride
    // floats after sequence 0's. NULL row_seq: one sequence, positions start_pos + t.
    const int *row_seq, *row_pos;
    size_t seq_stride;
    // fast prefill: CTAs of the balanced key-tile schedule and their partial
    // slots (2 per CTA, G4_PRE_PART_SLOT floats each)
    float *pre_part;
    int pre_ctas;
    // fast prefill: also quantise the output rows for o_proj (gemma4.c:459)
    // into xq [T][8*hd], xs [T][8*hd/64] and, when set, xsT (group-major)
    int quant_out;
    float *xsT;
    // tensor-core prefill: the workspace already holds this chunk's K/V split
    // of the same cache (a layer that reads another layer's cache)
    int reuse_kv;
};

// ---- persistent decode step (g4_decode.cu) ---------------------------------
enum DecodeOpType : int {
    OP_GEMV = 0,       // GemvArgs g with (pro, epi)
    OP_ATTN = 1,       // split-KV attention, AttnArgs at (CTA c = split c)
    OP_COMBINE = 2,    // merge splits + quantise, CTA c = 256 output dims
    OP_PLE_PREP = 3,   // per-layer inputs: CTA c = layer c
    OP_FINISH = 4,     // last residual update (CTA 0)
};

struct alignas(16) DecodeOp {
    int type, pro, epi, barrier;   // barrier: grid-wide barrier after the op
    // GEMV row partition over the grid (host-computed): CTA b owns row pairs
    // [b q + min(b, r), +q + (b < r)); stages of srows rows, nst[0] / nst[1]
    // stages for q / q + 1 pairs
    int part_q, part_r, srows, nst[2];
    GemvArgs g;
    AttnArgs at;
    // OP_PLE_PREP
    const float *pli, *ple_emb, *ple_norm;
    float ple_eps, ple_scale;
    float *ple_u;
    // OP_FINISH: res_out = (res_in + rmsnorm(h, w)) * scalar
    const float *fin_h, *fin_w, *fin_res_in, *fin_scalar;
    float *fin_res_out;
};

struct DecodeParams {
    const DecodeOp *ops;             // 16-byte aligned
    int nops;
    const int *pos;                  // the step's position (device)
    int splits;                       // attention splits (= grid)
    unsigned long long *bar;          // grid-barrier arrival counter (monotonic)
    unsigned long long *bar_base;     // its value when this launch starts
    int *err;
    int starve;                       // test aid: the producer issues no weight copy, so the
                                      // consumers' bounded waits run out (G4D_TIMEOUT_FULL)
    // optional timeline (zeroed by the host): [0] latest CTA start, then per op o
    // at 1+6o: latest prologue end (GEMV), latest op end, latest barrier exit,
    // longest stage wait of a consumer warp (ns), latest issue of the op's
    // first stage, latest issue of its last stage; %globaltimer nanoseconds
    unsigned long long *trace;
};

size_t g4_decode_smem_bytes();
cudaError_t g4_launch_decode(const DecodeParams &p, int grid, cudaStream_t st);
// stages of every GEMV op this CTA streams (for sizing checks)
int g4_decode_max_stages(const DecodeOp *ops, int nops, int grid);
// the GEMV row partition fields of a decode op for a persistent grid of `grid` CTAs
void g4_decode_set_partition(DecodeOp &op, int grid);

// ---- launchers (g4_*.cu) ---------------------------------------------------
cudaError_t g4_launch_scales_t(const uint16_t *s, int N, int K, float *sT, cudaStream_t st);
cudaError_t g4_launch_softcap_argmax(float *logits, int rows, int n, int *argmax, cudaStream_t st);
int g4_gemv_smem_bytes(const GemvArgs &a, int stages);
// Fills the launch plan (rb = most rows one CTA owns) for a grid of `grid` CTAs.
void g4_gemv_plan(GemvArgs &a, int grid);
cudaError_t g4_launch_gemv(const GemvArgs &a, int pro, int epi, int grid, cudaStream_t st, bool pdl);
cudaError_t g4_launch_gemm(const GemmArgs &a, cudaStream_t st, bool pdl);
cudaError_t g4_launch_attn_decode(const AttnArgs &a, int splits, cudaStream_t st, bool pdl);
// one token per row, each row its own sequence and position (q/k/v already
// post-processed by g4_launch_qkv_post): split-KV partials then combine into a.out
cudaError_t g4_launch_attn_rows(const AttnArgs &a, int splits, cudaStream_t st, bool pdl);
cudaError_t g4_launch_attn_combine(const AttnArgs &a, int splits, cudaStream_t st, bool pdl);
// top-64 temperature sampling (gemma4.c:536-561) from a top-64 list; state: xorshift state
cudaError_t g4_launch_sample64(const float *vals, const int *ids, float temperature, unsigned long long *state,
                               int *token, cudaStream_t st);
// Raise a kernel's dynamic shared-memory limit to `bytes` once per device
// (the attribute lives in each device's context); thread-safe.
cudaError_t g4_smem_optin(const void *kernel, int bytes);
// Multiprocessor count of the current device.
int g4_device_sms();
cudaError_t g4_launch_qkv_post(const AttnArgs &a, cudaStream_t st, bool pdl);
cudaError_t g4_launch_attn_prefill(const AttnArgs &a, cudaStream_t st, bool pdl);
cudaError_t g4_launch_attn_strict(const AttnArgs &a, cudaStream_t st, bool pdl);
// Prefill attention on the tensor cores (g4_attn_tc.cu, tcgen05 GEMMs on fp16 hi/lo operand pairs):
// workspace bytes for the chunk `a` describes (0: the path cannot run it) and
// the launches into that workspace (256-byte aligned); q/k/v already post-processed.
size_t g4_attn_tc_ws_bytes(const AttnArgs &a);
cudaError_t g4_launch_attn_tc(const AttnArgs &a, void *ws, size_t ws_bytes, cudaStream_t st, bool pdl);

cudaError_t g4_launch_repack(const int8_t *packed_w, const uint16_t *packed_s, int N, int K, int8_t *w, uint16_t *s,
                             int row_offset, int row_stride_mul, cudaStream_t st);
// Load-time repacking of many matrices per launch (the model upload): one job
// per packed matrix piece (whole 16-row blocks) already in device memory.
struct RepackJob {
    const int8_t *src_w;      // packed [N/16][K/64][16][16][4]
    const uint16_t *src_s;    // packed [N/16][K/64][16]
    int8_t *dst_w;            // row-major destination matrix
    uint16_t *dst_s;
    int N, K, row_offset, row_mul;
};
struct ScalesJob {
    const uint16_t *s;        // [N][G] fp16
    float *sT;                // [G][N] fp32
    int N, G;
};
cudaError_t g4_launch_repack_jobs(const RepackJob *jobs_dev, int njobs, cudaStream_t st);
cudaError_t g4_launch_scales_t_jobs(const ScalesJob *jobs_dev, int njobs, cudaStream_t st);
cudaError_t g4_launch_rows_embed(const int *tokens, int T, DMat embed, DMat embed_ple, float mult, float ple_mult,
                                 float *res, float *ple_emb, int *err, cudaStream_t st, bool pdl);
// xsT (optional): the scales again, group-major [K/64][G4_XST_STRIDE] (tensor-core GEMM)
cudaError_t g4_launch_rows_quant(const float *src, int src_stride, int T, int K, int8_t *xq, float *xs,
                                 cudaStream_t st, bool pdl, float *xsT = nullptr);
// mode: 0 = norm+quant, 1 = res+norm+quant, 2 = res+quant, 3 = res finish (no quant)
cudaError_t g4_launch_rows_norm(int mode, const float *src, int T, const float *w_post, const float *res_in,
                                float *res_out, const float *scalar, const float *w_pre, float eps, int8_t *xq,
                                float *xs, cudaStream_t st, bool pdl, float *y_out = nullptr, int strict = 0,
                                float *xsT = nullptr);
cudaError_t g4_launch_ple_prep(const float *pli, const float *ple_emb, const float *w, float eps, float scale, int T,
                               float *u, cudaStream_t st, bool pdl, int strict = 0);

// Launch with (optional) programmatic dependent launch.
template <typename... Args>
cudaError_t g4_launch(void (*kern)(Args...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                      Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}
