// g4_engine.cu — context, model upload, forward/logits orchestration, C ABI.
//
// Replaces gemma4.c's forward (gemma4.c:463-509) and logits (:512-522) and
// the state they use (InferenceState, :157-167). The host side of this file
// only sequences kernels; all arithmetic runs on the device.
//
// Paths:
//   - T = 1 (decode): 8 kernels per layer, every int8 projection a GEMV with
//     its RMSNorm/residual/quantise producer fused into the prologue and its
//     GeGLU consumer fused into the epilogue; captured once into a CUDA graph
//     whose kernels read the token and position from device memory; PDL lets
//     each GEMV stream its weights while its predecessor drains.
//   - T = 2..4: same GEMVs, attention through the chunk kernels.
//   - T > 4 (prefill chunks): row kernels + GEMM + chunk attention.
#include <cuda_profiler_api.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <utility>
#include <vector>

#include "../../include/g4cuda.h"
#include "g4_format.h"
#include "g4_internal.h"

cudaError_t g4_launch_gemm_tc(const GemmArgs &a, cudaStream_t st, bool pdl);
cudaError_t g4_launch_gemm_simt(const GemmArgs &a, cudaStream_t st, bool pdl);
bool g4_gemm_tc_supported(const GemmArgs &a);
cudaError_t g4_launch_topk(const float *x, int n, int k, float *part_v, int *part_i, float *vals, int *ids,
                           cudaStream_t st);

namespace {

constexpr int kMaxT = G4_BATCH;
constexpr int kSplits = 148;   // decode attention splits (one CTA per SM)
constexpr int kQkvStride = G4_HEADS * G4_HD_GLOBAL + 2 * G4_HD_GLOBAL;   // 5120
constexpr int kMaxFfn = 12288;

struct Layer {
    DMat qkv, o, gu, down, pleg, plep;
    const float *in_norm, *post_attn, *pre_ffn, *post_ffn, *post_ple, *q_norm, *k_norm, *scalar;
    const float *rope_cos, *rope_sin;
    int hd, pairs, global, owner, has_kv, qw, ffn;
    float *kcache, *vcache;
    int ring;
};

}  // namespace

struct g4_ctx {
    int device = 0, num_sms = 148;
    cudaStream_t st = nullptr;
    uint8_t *arena = nullptr;
    size_t arena_bytes = 0, arena_used = 0;
    DMat embed{}, embed_ple{}, pmp{};
    const float *final_norm = nullptr, *ple_norm = nullptr, *gelu = nullptr;
    Layer L[G4_NUM_LAYERS];
    // activations / state
    uint8_t *state = nullptr;
    float *res[2] = {nullptr, nullptr};
    int cur = 0;
    int8_t *xq = nullptr;
    float *xsT = nullptr;            // group-major activation scales (tensor-core GEMM)
    // second activation set: the gate/up GEMM quantises its GEGLU rows into it
    // while its own input (xq, xs, xsT) is still being read
    int8_t *xq2 = nullptr;
    float *xs2 = nullptr, *xsT2 = nullptr;
    float *xs = nullptr, *qkv = nullptr, *attn = nullptr, *h = nullptr, *gu = nullptr, *pg = nullptr;
    float *pli = nullptr, *ple_emb = nullptr, *ple_u = nullptr, *logits = nullptr, *part = nullptr;
    float *pre_part = nullptr;       // prefill attention partial slots
    float *argmax_part = nullptr, *topk_v = nullptr;
    unsigned long long *rng_d = nullptr;   // sampling xorshift state (gemma4.c:527: starts at 42)
    int *sample_tok = nullptr;
    int *argmax_out = nullptr, *topk_i = nullptr;
    unsigned *ticket = nullptr;
    int *err = nullptr, *tokens_d = nullptr, *pos_d = nullptr;
    float *kv = nullptr;
    size_t kv_bytes = 0;
    // sequencing
    int last_T = 0;
    int logits_row_cached = -1;
    bool use_graph = true, use_pdl = true;
    int gemm_path = 0;
    int layers = G4_NUM_LAYERS;   // layers to run (testing aid)
    bool strict = false;          // reference-order reductions (bit-exact forward)
    float *scores = nullptr;      // strict attention scratch
    size_t scores_cap = 0;
    // tensor-core prefill attention: path option and its workspace (grown on
    // demand): the global layers' region, then the sliding layers' region
    int attn_path = 0;
    void *tc_ws = nullptr;
    size_t tc_ws_gcap = 0, tc_ws_scap = 0;
    cudaGraphExec_t g_decode = nullptr;
    int graph_cur = 0;
    bool decode_warm = false;
    // multi-sequence steps (one row per sequence): one graph per row count,
    // captured once that count has run kRowGraphAfter steps eagerly (a capture
    // costs ~10 ms of host time; serving shifts its batch size every few steps)
    std::vector<cudaGraphExec_t> g_rows;
    std::vector<int> rows_warm;
    int rows_cur = 0;
    cudaEvent_t events[16] = {};
    // persistent single-token decode (g4_decode.cu)
    bool persistent = true;          // G4_OPT_PERSISTENT
    void *scales_t = nullptr;        // group-major fp32 weight scales (tensor-core GEMM)
    size_t scales_t_bytes = 0;
    // multi-sequence serving (g4_seq_alloc / g4_forward_batch / g4_logits_batch)
    int max_seqs = 0;
    int batch_splits = 0;            // G4_OPT_BATCH_SPLITS: 0 = auto
    void *bkv = nullptr, *bbuf = nullptr;
    size_t bkv_bytes = 0;
    float *bk[G4_NUM_LAYERS] = {}, *bv[G4_NUM_LAYERS] = {};   // sequence 0's K and V of the ring a layer reads
    int bring[G4_NUM_LAYERS] = {};
    int *row_seq_d = nullptr, *row_pos_d = nullptr, *bargmax = nullptr;
    float *bpart = nullptr, *blogits = nullptr, *bres = nullptr, *embed_st = nullptr;
    // logits of many rows (g4_logits_rows): two chunks of kDumpRows rows, their
    // copy stream and events; own group-major lm_head scales when no batch state
    void *dump_buf = nullptr;
    float *dump_log[2] = {nullptr, nullptr};
    int *dump_arg = nullptr;
    float *dump_st_scales = nullptr;
    cudaStream_t dump_st = nullptr;
    cudaEvent_t dump_done[2] = {nullptr, nullptr}, dump_copied[2] = {nullptr, nullptr};
    std::vector<int> blast;          // last row of each sequence of the last batch
    bool pending = false;            // a single-token forward waiting to be launched
    bool starve_next = false;        // g4_test_starve_next_step
    DecodeOp *dec_fwd = nullptr, *dec_fwdlog = nullptr;
    int n_fwd = 0, n_fwdlog = 0, dec_cur = 0, dec_layers = 0;
    unsigned long long *bar = nullptr, *bar_base = nullptr;
    std::vector<DecodeOp> dec_host;          // host copy of the forward+logits op list
    unsigned long long *trace = nullptr;     // timeline buffer (g4_trace_decode)
    char msg[512] = {0};
};

namespace {

int fail(g4_ctx *c, int code, const char *fmt, ...) {
    if (c) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(c->msg, sizeof(c->msg), fmt, ap);
        va_end(ap);
    }
    return code;
}

#define CK(call)                                                                                     \
    do {                                                                                             \
        cudaError_t e_ = (call);                                                                     \
        if (e_ != cudaSuccess)                                                                       \
            return fail(c, e_ == cudaErrorMemoryAllocation ? G4_ERR_NOMEM : G4_ERR_CUDA, "%s: %s (%s:%d)", \
                        #call, cudaGetErrorString(e_), __FILE__, __LINE__);                          \
    } while (0)

uint8_t *arena_take(g4_ctx *c, size_t bytes) {
    size_t off = (c->arena_used + 255) & ~(size_t)255;
    if (off + bytes > c->arena_bytes) return nullptr;
    c->arena_used = off + bytes;
    return c->arena + off;
}

struct Rec {
    uint64_t data, scales;
    int32_t shape[4];
};

// Resolve a record field (file offset, or a pointer into the same mapping after
// gemma4.c:681-685's fix-up) to a host pointer inside the image.
const uint8_t *resolve(const uint8_t *base, uint64_t bytes, uint64_t v, uint64_t need) {
    if (!v) return nullptr;
    uint64_t off = v;
    if (v >= bytes) {
        uintptr_t b = (uintptr_t)base;
        if (v < b || v - b >= bytes) return nullptr;
        off = v - b;
    }
    if (off + need > bytes) return nullptr;
    return base + off;
}

struct HostMat {
    const int8_t *w;
    const uint16_t *s;
    int N, K;
};

int get_mat(g4_ctx *c, const uint8_t *img, uint64_t bytes, const Rec *r, int idx, int N, int K, HostMat *out) {
    const Rec &x = r[idx];
    if (x.shape[0] != N || x.shape[1] != K)
        return fail(c, G4_ERR_FORMAT, "record %d: shape %dx%d, expected %dx%d", idx, x.shape[0], x.shape[1], N, K);
    out->w = (const int8_t *)resolve(img, bytes, x.data, (uint64_t)N * K);
    out->s = (const uint16_t *)resolve(img, bytes, x.scales, (uint64_t)N * (K / 64) * 2);
    out->N = N;
    out->K = K;
    if (!out->w || !out->s) return fail(c, G4_ERR_FORMAT, "record %d: data/scales outside the image", idx);
    return G4_OK;
}

int get_vec(g4_ctx *c, const uint8_t *img, uint64_t bytes, const Rec *r, int idx, int n, const float **out) {
    const Rec &x = r[idx];
    if (x.shape[0] != n) return fail(c, G4_ERR_FORMAT, "record %d: length %d, expected %d", idx, x.shape[0], n);
    *out = (const float *)resolve(img, bytes, x.data, (uint64_t)n * 4);
    if (!*out) return fail(c, G4_ERR_FORMAT, "record %d: data outside the image", idx);
    return G4_OK;
}

// Load-time repacking: packed matrix pieces (whole 16-row blocks) are gathered
// into one staging buffer (host images), or used where they lie (device
// images), and every fill is repacked by ONE launch of k_repack_jobs.
struct Uploader {
    static constexpr int kMaxJobs = 512;
    g4_ctx *c = nullptr;
    bool device_src = false;
    uint8_t *stage = nullptr;
    size_t stage_bytes = 0, used = 0;
    RepackJob *jobs_dev = nullptr;
    std::vector<RepackJob> jobs;

    ~Uploader() {
        if (stage) cudaFree(stage);
        if (jobs_dev) cudaFree(jobs_dev);
    }
    int flush() {
        if (jobs.empty()) return G4_OK;
        CK(cudaMemcpyAsync(jobs_dev, jobs.data(), jobs.size() * sizeof(RepackJob), cudaMemcpyHostToDevice, c->st));
        CK(g4_launch_repack_jobs(jobs_dev, (int)jobs.size(), c->st));
        CK(cudaStreamSynchronize(c->st));   // the staging buffer and the job list are reused
        jobs.clear();
        used = 0;
        return G4_OK;
    }
    int add(const HostMat &hm, DMat dst, int row_offset, int row_mul) {
        const int K = hm.K, G = K / 64;
        const size_t per_row = (size_t)K + (size_t)G * 2;
        for (int r0 = 0; r0 < hm.N;) {
            int nr = hm.N - r0;
            RepackJob j{};
            if (device_src) {
                j.src_w = hm.w + (size_t)r0 * K;
                j.src_s = hm.s + (size_t)r0 * G;
            } else {
                int fit = (int)((stage_bytes - used) / (per_row + 1)) / 16 * 16 - 16;
                if (fit < 16 || (fit < nr && used > 0)) {
                    if (int rc = flush()) return rc;
                    fit = (int)(stage_bytes / (per_row + 1)) / 16 * 16 - 16;
                    if (fit < 16) return fail(c, G4_ERR_INVALID, "staging buffer too small");
                }
                nr = nr < fit ? nr : fit;
                uint8_t *w = stage + used;
                const size_t wb = ((size_t)nr * K + 255) & ~(size_t)255;
                uint8_t *sc = w + wb;
                CK(cudaMemcpyAsync(w, hm.w + (size_t)r0 * K, (size_t)nr * K, cudaMemcpyDefault, c->st));
                CK(cudaMemcpyAsync(sc, hm.s + (size_t)r0 * G, (size_t)nr * G * 2, cudaMemcpyDefault, c->st));
                used += wb + (((size_t)nr * G * 2 + 255) & ~(size_t)255);
                j.src_w = (const int8_t *)w;
                j.src_s = (const uint16_t *)sc;
            }
            j.dst_w = (int8_t *)dst.w;
            j.dst_s = (uint16_t *)dst.s;
            j.N = nr;
            j.K = K;
            j.row_offset = row_offset + r0 * row_mul;
            j.row_mul = row_mul;
            jobs.push_back(j);
            r0 += nr;
            if ((int)jobs.size() >= kMaxJobs)
                if (int rc = flush()) return rc;
        }
        return G4_OK;
    }
};

DMat alloc_mat(g4_ctx *c, int N, int K) {
    DMat m{};
    m.N = N;
    m.K = K;
    m.w = (const int8_t *)arena_take(c, (size_t)N * K);
    m.s = (const uint16_t *)arena_take(c, (size_t)N * (K / 64) * 2);
    return m;
}

const float *upload_vec(g4_ctx *c, const float *h, size_t n, int *rc) {
    float *d = (float *)arena_take(c, n * 4);
    if (!d) { *rc = G4_ERR_NOMEM; return nullptr; }
    cudaError_t e = cudaMemcpyAsync(d, h, n * 4, cudaMemcpyDefault, c->st);   // host or device image
    if (e != cudaSuccess) *rc = G4_ERR_CUDA;
    return d;
}

size_t mat_bytes(int N, int K) { return (((size_t)N * K + 255) & ~(size_t)255) + (((size_t)N * (K / 64) * 2 + 255) & ~(size_t)255); }

// img: the model image (host memory, or device memory when hdr is given);
// hdr: a host copy of the image's first G4_WEIGHTS_OFFSET + record-table bytes
// (magic and records are parsed on the host), or NULL when img is host memory.
int open_impl(g4_ctx *c, const uint8_t *img, uint64_t bytes, const uint8_t *hdr = nullptr) {
    const uint8_t *h = hdr ? hdr : img;
    if (bytes < G4_WEIGHTS_OFFSET + (uint64_t)G4_NUM_RECORDS * G4_RECORD_BYTES || memcmp(h, "MOG", 4) != 0)
        return fail(c, G4_ERR_FORMAT, "not a gemma4.c model image (magic \"MOG\")");
    const Rec *r = (const Rec *)(h + G4_WEIGHTS_OFFSET);

    CK(cudaSetDevice(c->device));
    CK(cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, c->device));
    CK(cudaStreamCreateWithFlags(&c->st, cudaStreamNonBlocking));

    // ---- collect host views + validate geometry ----
    HostMat embed, eple, pmp;
    int rc;
    if ((rc = get_mat(c, img, bytes, r, G4_R_EMBED, G4_VOCAB, G4_HIDDEN, &embed))) return rc;
    if ((rc = get_mat(c, img, bytes, r, G4_R_EMBED_PER_LAYER, G4_VOCAB, G4_NUM_LAYERS * G4_PLE, &eple))) return rc;
    if ((rc = get_mat(c, img, bytes, r, G4_R_PLE_MODEL_PROJ, G4_NUM_LAYERS * G4_PLE, G4_HIDDEN, &pmp))) return rc;
    struct HL {
        HostMat q, k, v, o, gate, up, down, pleg, plep;
        const float *vec[8];
        const float *cosv, *sinv;
        int pairs;
    } hl[G4_NUM_LAYERS];
    size_t total = mat_bytes(G4_VOCAB, G4_HIDDEN) + mat_bytes(G4_VOCAB, G4_NUM_LAYERS * G4_PLE) +
                   mat_bytes(G4_NUM_LAYERS * G4_PLE, G4_HIDDEN);
    for (int l = 0; l < G4_NUM_LAYERS; l++) {
        const int global = g4_layer_is_global(l), hd = global ? G4_HD_GLOBAL : G4_HD_SLIDING;
        const int kv = l < G4_NUM_KV_LAYERS, ffn = kv ? 6144 : 12288, qw = G4_HEADS * hd;
        HL &x = hl[l];
        if ((rc = get_mat(c, img, bytes, r, G4_R_LAYER(l, G4_L_Q_PROJ), qw, G4_HIDDEN, &x.q))) return rc;
        if (kv) {
            if ((rc = get_mat(c, img, bytes, r, G4_R_LAYER(l, G4_L_K_PROJ), hd, G4_HIDDEN, &x.k))) return rc;
            if ((rc = get_mat(c, img, bytes, r, G4_R_LAYER(l, G4_L_V_PROJ), hd, G4_HIDDEN, &x.v))) return rc;
        } else if (r[G4_R_LAYER(l, G4_L_K_PROJ)].data || r[G4_R_LAYER(l, G4_L_V_PROJ)].data) {
            return fail(c, G4_ERR_FORMAT, "layer %d: unexpected K/V weights on a shared-cache layer", l);
        }
        if ((rc = get_mat(c, img, bytes, r, G4_R_LAYER(l, G4_L_O_PROJ), G4_HIDDEN, qw, &x.o))) return rc;
        if ((rc = get_mat(c, img, bytes, r, G4_R_LAYER(l, G4_L_GATE), ffn, G4_HIDDEN, &x.gate))) return rc;
        if ((rc = get_mat(c, img, bytes, r, G4_R_LAYER(l, G4_L_UP), ffn, G4_HIDDEN, &x.up))) return rc;
        if ((rc = get_mat(c, img, bytes, r, G4_R_LAYER(l, G4_L_DOWN), G4_HIDDEN, ffn, &x.down))) return rc;
        if ((rc = get_mat(c, img, bytes, r, G4_R_LAYER(l, G4_L_PLE_GATE), G4_PLE, G4_HIDDEN, &x.pleg))) return rc;
        if ((rc = get_mat(c, img, bytes, r, G4_R_LAYER(l, G4_L_PLE_PROJ), G4_HIDDEN, G4_PLE, &x.plep))) return rc;
        const int vidx[8] = {G4_L_INPUT_NORM, G4_L_POST_ATTN_NORM, G4_L_PRE_FFN_NORM, G4_L_POST_FFN_NORM,
                             G4_L_POST_PLE_NORM, G4_L_Q_NORM, G4_L_K_NORM, G4_L_LAYER_SCALAR};
        const int vlen[8] = {G4_HIDDEN, G4_HIDDEN, G4_HIDDEN, G4_HIDDEN, G4_HIDDEN, hd, hd, 1};
        for (int i = 0; i < 8; i++) {
            x.vec[i] = nullptr;
            if (i == 6 && !kv) continue;
            if ((rc = get_vec(c, img, bytes, r, G4_R_LAYER(l, vidx[i]), vlen[i], &x.vec[i]))) return rc;
        }
        const Rec &rcos = r[G4_R_LAYER(l, G4_L_ROPE_COS)], &rsin = r[G4_R_LAYER(l, G4_L_ROPE_SIN)];
        x.pairs = rcos.shape[1];
        const int want_pairs = global ? 64 : 128;
        if (rcos.shape[0] != G4_MAX_CONTEXT || x.pairs != want_pairs || rsin.shape[1] != x.pairs ||
            rsin.shape[0] != G4_MAX_CONTEXT)
            return fail(c, G4_ERR_FORMAT, "layer %d: rope table shape", l);
        x.cosv = (const float *)resolve(img, bytes, rcos.data, (uint64_t)G4_MAX_CONTEXT * x.pairs * 4);
        x.sinv = (const float *)resolve(img, bytes, rsin.data, (uint64_t)G4_MAX_CONTEXT * x.pairs * 4);
        if (!x.cosv || !x.sinv) return fail(c, G4_ERR_FORMAT, "layer %d: rope tables outside the image", l);
        total += mat_bytes(qw + (kv ? 2 * hd : 0), G4_HIDDEN) + mat_bytes(G4_HIDDEN, qw) + mat_bytes(2 * ffn, G4_HIDDEN) +
                 mat_bytes(G4_HIDDEN, ffn) + mat_bytes(G4_PLE, G4_HIDDEN) + mat_bytes(G4_HIDDEN, G4_PLE) +
                 8 * 4 * 1024 + 2 * 256;
    }
    const float *final_norm, *ple_norm, *gelu;
    if ((rc = get_vec(c, img, bytes, r, G4_R_NORM, G4_HIDDEN, &final_norm))) return rc;
    if ((rc = get_vec(c, img, bytes, r, G4_R_PLE_PROJ_NORM, G4_PLE, &ple_norm))) return rc;
    const Rec &rg = r[G4_R_GELU];
    if (rg.shape[0] != 4096 || rg.shape[1] != -8 || rg.shape[2] != 8)
        return fail(c, G4_ERR_FORMAT, "gelu table shape (%d,%d,%d)", rg.shape[0], rg.shape[1], rg.shape[2]);
    gelu = (const float *)resolve(img, bytes, rg.data, 4096 * 4);
    if (!gelu) return fail(c, G4_ERR_FORMAT, "gelu table outside the image");
    total += 2 * (size_t)G4_MAX_CONTEXT * (128 + 64) * 4 + 64 * 1024;

    // ---- device allocation ----
    c->arena_bytes = total + (1 << 20);
    CK(cudaMalloc(&c->arena, c->arena_bytes));
    c->embed = alloc_mat(c, G4_VOCAB, G4_HIDDEN);
    c->embed_ple = alloc_mat(c, G4_VOCAB, G4_NUM_LAYERS * G4_PLE);
    c->pmp = alloc_mat(c, G4_NUM_LAYERS * G4_PLE, G4_HIDDEN);
    for (int l = 0; l < G4_NUM_LAYERS; l++) {
        Layer &Y = c->L[l];
        HL &x = hl[l];
        Y.global = g4_layer_is_global(l);
        Y.hd = Y.global ? G4_HD_GLOBAL : G4_HD_SLIDING;
        Y.has_kv = l < G4_NUM_KV_LAYERS;
        Y.owner = g4_cache_owner(l);
        Y.ffn = x.gate.N;
        Y.qw = G4_HEADS * Y.hd;
        Y.pairs = x.pairs;
        Y.qkv = alloc_mat(c, Y.qw + (Y.has_kv ? 2 * Y.hd : 0), G4_HIDDEN);
        Y.o = alloc_mat(c, G4_HIDDEN, Y.qw);
        Y.gu = alloc_mat(c, 2 * Y.ffn, G4_HIDDEN);
        Y.down = alloc_mat(c, G4_HIDDEN, Y.ffn);
        Y.pleg = alloc_mat(c, G4_PLE, G4_HIDDEN);
        Y.plep = alloc_mat(c, G4_HIDDEN, G4_PLE);
    }
    if (!c->embed.w || !c->L[G4_NUM_LAYERS - 1].plep.s) return fail(c, G4_ERR_NOMEM, "weight arena too small");

    // ---- upload + repack ----
    Uploader upl;
    upl.c = c;
    upl.device_src = hdr != nullptr;   // the image is already in device memory (g4_open_file)
    upl.stage_bytes = upl.device_src ? 0 : (size_t)256 << 20;
    if (upl.stage_bytes) CK(cudaMalloc(&upl.stage, upl.stage_bytes));
    CK(cudaMalloc(&upl.jobs_dev, Uploader::kMaxJobs * sizeof(RepackJob)));
    rc = upl.add(embed, c->embed, 0, 1);
    if (!rc) rc = upl.add(eple, c->embed_ple, 0, 1);
    if (!rc) rc = upl.add(pmp, c->pmp, 0, 1);
    for (int l = 0; l < G4_NUM_LAYERS && !rc; l++) {
        Layer &Y = c->L[l];
        HL &x = hl[l];
        rc = upl.add(x.q, Y.qkv, 0, 1);
        if (!rc && Y.has_kv) rc = upl.add(x.k, Y.qkv, Y.qw, 1);
        if (!rc && Y.has_kv) rc = upl.add(x.v, Y.qkv, Y.qw + Y.hd, 1);
        if (!rc) rc = upl.add(x.o, Y.o, 0, 1);
        if (!rc) rc = upl.add(x.gate, Y.gu, 0, 2);
        if (!rc) rc = upl.add(x.up, Y.gu, 1, 2);
        if (!rc) rc = upl.add(x.down, Y.down, 0, 1);
        if (!rc) rc = upl.add(x.pleg, Y.pleg, 0, 1);
        if (!rc) rc = upl.add(x.plep, Y.plep, 0, 1);
    }
    if (!rc) rc = upl.flush();
    if (rc) return rc;
    // group-major fp32 copies of the layer and per-layer-projection scales
    // (tensor-core GEMM), all in one launch
    {
        std::vector<DMat *> mats;
        mats.push_back(&c->pmp);
        for (int l = 0; l < G4_NUM_LAYERS; l++) {
            Layer &Y = c->L[l];
            for (DMat *m : {&Y.qkv, &Y.o, &Y.gu, &Y.down, &Y.pleg, &Y.plep}) mats.push_back(m);
        }
        size_t bytes = 0;
        for (DMat *m : mats) bytes += ((size_t)m->N * (m->K / 64) * 4 + 255) & ~(size_t)255;
        CK(cudaMalloc(&c->scales_t, bytes));
        std::vector<ScalesJob> sj;
        size_t off = 0;
        for (DMat *m : mats) {
            float *d = (float *)((uint8_t *)c->scales_t + off);
            sj.push_back(ScalesJob{m->s, d, m->N, m->K / 64});
            m->sT = d;
            off += ((size_t)m->N * (m->K / 64) * 4 + 255) & ~(size_t)255;
        }
        static_assert(sizeof(ScalesJob) <= sizeof(RepackJob), "scale jobs reuse the repack job buffer");
        if (sj.size() > (size_t)Uploader::kMaxJobs) return fail(c, G4_ERR_INVALID, "too many scale jobs");
        CK(cudaMemcpyAsync(upl.jobs_dev, sj.data(), sj.size() * sizeof(ScalesJob), cudaMemcpyHostToDevice, c->st));
        CK(g4_launch_scales_t_jobs((const ScalesJob *)upl.jobs_dev, (int)sj.size(), c->st));
        CK(cudaStreamSynchronize(c->st));
        c->scales_t_bytes = bytes;
    }
    int vr = G4_OK;
    const float *rope_dev[4] = {nullptr, nullptr, nullptr, nullptr};
    for (int l = 0; l < G4_NUM_LAYERS; l++) {
        Layer &Y = c->L[l];
        HL &x = hl[l];
        Y.in_norm = upload_vec(c, x.vec[0], G4_HIDDEN, &vr);
        Y.post_attn = upload_vec(c, x.vec[1], G4_HIDDEN, &vr);
        Y.pre_ffn = upload_vec(c, x.vec[2], G4_HIDDEN, &vr);
        Y.post_ffn = upload_vec(c, x.vec[3], G4_HIDDEN, &vr);
        Y.post_ple = upload_vec(c, x.vec[4], G4_HIDDEN, &vr);
        Y.q_norm = upload_vec(c, x.vec[5], Y.hd, &vr);
        Y.k_norm = Y.has_kv ? upload_vec(c, x.vec[6], Y.hd, &vr) : nullptr;
        Y.scalar = upload_vec(c, x.vec[7], 1, &vr);
        const int ti = Y.global ? 2 : 0;
        if (!rope_dev[ti]) {
            rope_dev[ti] = upload_vec(c, x.cosv, (size_t)G4_MAX_CONTEXT * x.pairs, &vr);
            rope_dev[ti + 1] = upload_vec(c, x.sinv, (size_t)G4_MAX_CONTEXT * x.pairs, &vr);
        }
        Y.rope_cos = rope_dev[ti];
        Y.rope_sin = rope_dev[ti + 1];
    }
    c->final_norm = upload_vec(c, final_norm, G4_HIDDEN, &vr);
    c->ple_norm = upload_vec(c, ple_norm, G4_PLE, &vr);
    c->gelu = upload_vec(c, gelu, 4096, &vr);
    if (vr) return fail(c, vr, "uploading vectors failed");
    CK(cudaStreamSynchronize(c->st));

    // ---- state ----
    struct { void **p; size_t bytes; } bufs[] = {
        {(void **)&c->res[0], (size_t)kMaxT * G4_HIDDEN * 4},
        {(void **)&c->res[1], (size_t)kMaxT * G4_HIDDEN * 4},
        {(void **)&c->xq, (size_t)kMaxT * kMaxFfn},
        {(void **)&c->xs, (size_t)kMaxT * kMaxFfn / 64 * 4},
        {(void **)&c->xsT, (size_t)G4_XST_STRIDE * kMaxFfn / 64 * 4},
        {(void **)&c->xq2, (size_t)kMaxT * kMaxFfn},
        {(void **)&c->xs2, (size_t)kMaxT * kMaxFfn / 64 * 4},
        {(void **)&c->xsT2, (size_t)G4_XST_STRIDE * kMaxFfn / 64 * 4},
        {(void **)&c->qkv, (size_t)kMaxT * kQkvStride * 4},
        {(void **)&c->attn, (size_t)kMaxT * G4_HEADS * G4_HD_GLOBAL * 4},
        {(void **)&c->h, (size_t)kMaxT * G4_HIDDEN * 4},
        {(void **)&c->gu, (size_t)kMaxT * kMaxFfn * 4},
        {(void **)&c->pg, (size_t)kMaxT * G4_PLE * 4},
        {(void **)&c->pli, (size_t)kMaxT * G4_NUM_LAYERS * G4_PLE * 4},
        {(void **)&c->ple_emb, (size_t)kMaxT * G4_NUM_LAYERS * G4_PLE * 4},
        {(void **)&c->ple_u, (size_t)kMaxT * G4_NUM_LAYERS * G4_PLE * 4},
        {(void **)&c->logits, (size_t)G4_VOCAB * 4},
        {(void **)&c->part, (size_t)kSplits * G4_HEADS * (G4_HD_GLOBAL + 4) * 4},
        {(void **)&c->pre_part, (size_t)2 * c->num_sms * G4_PRE_PART_SLOT * 4},
        {(void **)&c->argmax_part, (size_t)1024 * 4 * 2 * 4},
        {(void **)&c->rng_d, 8},
        {(void **)&c->sample_tok, 4},
        {(void **)&c->topk_v, (size_t)1024 * 64 * 4},
        {(void **)&c->topk_i, (size_t)1024 * 64 * 4},
        {(void **)&c->argmax_out, 64},
        {(void **)&c->ticket, 64},
        {(void **)&c->err, 64},
        {(void **)&c->tokens_d, (size_t)kMaxT * 4},
        {(void **)&c->pos_d, 64},
        {(void **)&c->bar, 64},
    };
    size_t st_total = 0;
    for (auto &b : bufs) st_total += (b.bytes + 255) & ~(size_t)255;
    CK(cudaMalloc(&c->state, st_total));
    CK(cudaMemset(c->state, 0, st_total));
    size_t off = 0;
    for (auto &b : bufs) {
        *b.p = c->state + off;
        off += (b.bytes + 255) & ~(size_t)255;
    }
    {
        const unsigned long long seed = 42;
        CK(cudaMemcpy(c->rng_d, &seed, 8, cudaMemcpyHostToDevice));
    }
    // KV rings: 12 sliding (owners 0-3, 5-8, 10-13) + 3 global (owners 4, 9, 14)
    const size_t sl = (size_t)2 * G4_SLIDING_RING * G4_HD_SLIDING * 4, gl = (size_t)2 * G4_MAX_CONTEXT * G4_HD_GLOBAL * 4;
    c->kv_bytes = 12 * sl + 3 * gl;
    CK(cudaMalloc(&c->kv, c->kv_bytes));
    CK(cudaMemset(c->kv, 0, c->kv_bytes));
    for (int l = 0; l < G4_NUM_LAYERS; l++) {
        Layer &Y = c->L[l];
        const int o = Y.owner;
        if (Y.global) {
            Y.ring = G4_MAX_CONTEXT;
            Y.kcache = (float *)((uint8_t *)c->kv + 12 * sl + (size_t)(o / 5) * gl);
        } else {
            Y.ring = G4_SLIDING_RING;
            Y.kcache = (float *)((uint8_t *)c->kv + (size_t)((o / 5) * 4 + o % 5) * sl);
        }
        Y.vcache = Y.kcache + (size_t)Y.ring * Y.hd;
    }
    c->bar_base = c->bar + 1;
    CK(cudaStreamSynchronize(c->st));
    return G4_OK;
}

// ---------------------------------------------------------------------------
// launch sequences

// Per-kernel profile of one launch sequence: an event after every launch; with
// launches serialised (no PDL), kernel i took ev[i] - ev[i-1].
struct Prof {
    static constexpr int kMax = 512;
    cudaEvent_t ev[kMax + 1];
    int cls[kMax];
    double bytes[kMax];
    int n = 0;
};

struct Seq {
    g4_ctx *c;
    bool pdl;
    cudaError_t e = cudaSuccess;
    Prof *prof = nullptr;
    std::vector<DecodeOp> *rec = nullptr;   // record the sequence as persistent-decode ops
    int next_cls = 2;          // 0 int8 weight GEMV, 1 attention, 2 other
    double next_bytes = 0;
    void tag(int cls, double bytes) { next_cls = cls; next_bytes = bytes; }
    void ck(cudaError_t x) {
        if (e == cudaSuccess && x != cudaSuccess) e = x;
        if (prof && prof->n < Prof::kMax) {
            cudaEventRecord(prof->ev[prof->n + 1], c->st);
            prof->cls[prof->n] = next_cls;
            prof->bytes[prof->n] = next_bytes;
            prof->n++;
        }
        next_cls = 2;
        next_bytes = 0;
    }
};

GemvArgs gemv_base(g4_ctx *c, const DMat &m, int T) {
    GemvArgs a{};
    a.m = m;
    a.T = T;
    a.eps = G4_RMS_EPS;
    a.gelu = c->gelu;
    a.err = c->err;
    a.strict = c->strict;
    g4_gemv_plan(a, c->num_sms);
    return a;
}

void gemv(Seq &q, GemvArgs &a, int pro, int epi) {
    if (q.rec) {
        DecodeOp op{};
        op.type = OP_GEMV;
        op.pro = pro;
        op.epi = epi;
        op.barrier = 1;
        op.g = a;
        q.rec->push_back(op);
        return;
    }
    q.tag(0, (double)a.m.N * a.m.K + (double)a.m.N * (a.m.K / 64) * 2);
    const int pairs = a.m.N / 2;
    const int grid = pairs < q.c->num_sms ? pairs : q.c->num_sms;
    g4_gemv_plan(a, grid);
    q.ck(g4_launch_gemv(a, pro, epi, grid, q.c->st, q.pdl));
}

// Returns true when the tensor-core path also quantised its GEGLU rows into
// xq / xs / xsT (fuse_quant and EPI_GEGLU_PAIR); then `out` is not written.
bool gemm(Seq &q, const DMat &m, int T, int epi, float *out, int out_stride, const float *u, int u_stride,
          bool fuse_quant = false) {
    g4_ctx *c = q.c;
    GemmArgs a{};
    a.m = m;
    a.T = T;
    a.xq = c->xq;
    a.xs = c->xs;
    a.xsT = c->xsT;
    a.epi = epi;
    a.out = out;
    a.out_stride = out_stride;
    a.ple_u = u;
    a.u_stride = u_stride;
    a.gelu = c->gelu;
    a.err = c->err;
    if (c->gemm_path == 1 || !g4_gemm_tc_supported(a) || c->gemm_path == -1) {
        q.ck(g4_launch_gemm_simt(a, c->st, q.pdl));
        return false;
    }
    // a few token rows (multi-sequence decode): the weight-streaming mma GEMM
    if ((c->gemm_path == 3 && g4_gemm_skinny_supported(a)) || (c->gemm_path == 0 && g4_gemm_skinny_preferred(a))) {
        q.ck(g4_launch_gemm_skinny(a, c->st, q.pdl));
        return false;
    }
    // (the transposed-role tiles of a few token rows do not quantise: rows_quant follows)
    const bool fuse = fuse_quant && epi == EPI_GEGLU_PAIR && m.N % 128 == 0 && !g4_gemm_tc_swapped(a);
    if (fuse) {   // into the second set: this GEMM still reads xq / xs / xsT
        a.qout = c->xq2;
        a.qs = c->xs2;
        a.qsT = c->xsT2;
    }
    q.ck(g4_launch_gemm_tc(a, c->st, q.pdl));
    return fuse;
}

AttnArgs attn_base(g4_ctx *c, const Layer &Y, int T, int start_pos, const int *pos_dev) {
    AttnArgs a{};
    a.hd = Y.hd;
    a.pairs = Y.pairs;
    a.window = Y.global ? 0 : G4_SLIDING_WINDOW;
    a.mask = Y.ring - 1;
    a.T = T;
    a.start_pos = start_pos;
    a.pos_dev = pos_dev;
    a.qkv = c->qkv;
    a.qkv_stride = kQkvStride;
    a.has_kv = Y.has_kv;
    a.q_norm = Y.q_norm;
    a.k_norm = Y.k_norm;
    a.rope_cos = Y.rope_cos;
    a.rope_sin = Y.rope_sin;
    a.kcache = Y.kcache;
    a.vcache = Y.vcache;
    a.part = c->part;
    a.pre_part = c->pre_part;
    a.pre_ctas = c->num_sms;
    a.out = c->attn;
    a.xq = c->xq;
    a.xs = c->xs;
    a.err = c->err;
    a.strict = c->strict;
    a.scores = c->scores;
    a.score_stride = start_pos + T;
    return a;
}

// Decode path, T <= 4 tokens. pos_dev != NULL: positions and tokens come from
// device memory (graph replay); otherwise from start_pos / tokens_d.
cudaError_t enqueue_small(g4_ctx *c, int T, int start_pos, const int *pos_dev, Prof *prof = nullptr,
                          std::vector<DecodeOp> *rec = nullptr) {
    Seq q{c, c->use_pdl && !prof};
    q.prof = prof;
    q.rec = rec;
    int cur = 0;
    const float emb_mult = sqrtf((float)G4_HIDDEN), ple_mult = sqrtf((float)G4_PLE);
    {
        GemvArgs a = gemv_base(c, c->pmp, T);
        a.tokens = c->tokens_d;
        a.embed = c->embed;
        a.embed_ple = c->embed_ple;
        a.ple_emb = c->ple_emb;
        a.embed_mult = emb_mult;
        a.ple_mult = ple_mult;
        a.res_out = c->res[0];
        a.out = c->pli;
        a.out_stride = G4_NUM_LAYERS * G4_PLE;
        gemv(q, a, PRO_EMBED_QUANT, EPI_STORE);
        if (rec) {
            DecodeOp op{};
            op.type = OP_PLE_PREP;
            op.barrier = 0;   // ple_u is first read by layer 0's per-layer gate, several barriers later
            op.pli = c->pli;
            op.ple_emb = c->ple_emb;
            op.ple_norm = c->ple_norm;
            op.ple_eps = 1e-6f * G4_HIDDEN;
            op.ple_scale = 1.0f / sqrtf(2.0f);
            op.ple_u = c->ple_u;
            rec->push_back(op);
        } else {
            q.ck(g4_launch_ple_prep(c->pli, c->ple_emb, c->ple_norm, 1e-6f * G4_HIDDEN, 1.0f / sqrtf(2.0f), T,
                                    c->ple_u, c->st, q.pdl, c->strict));
        }
    }
    for (int l = 0; l < c->layers; l++) {
        const Layer &Y = c->L[l];
        // K1: q|k|v with the input norm (and the previous layer's PLE residual update)
        {
            GemvArgs a = gemv_base(c, Y.qkv, T);
            a.out = c->qkv;
            a.out_stride = kQkvStride;
            a.w_pre = Y.in_norm;
            if (l == 0) {
                a.src = c->res[cur];
                a.src_stride = G4_HIDDEN;
                gemv(q, a, PRO_NORM_QUANT, EPI_STORE);
            } else {
                const Layer &P = c->L[l - 1];
                a.src = c->h;
                a.src_stride = G4_HIDDEN;
                a.w_post = P.post_ple;
                a.scalar = P.scalar;
                a.res_in = c->res[cur];
                a.res_out = c->res[cur ^ 1];
                cur ^= 1;
                gemv(q, a, PRO_RES_NORM_QUANT, EPI_STORE);
            }
        }
        // attention
        AttnArgs at = attn_base(c, Y, T, start_pos, pos_dev);
        const bool fused_decode = T == 1 && !c->strict;
        if (fused_decode && rec) {
            DecodeOp op{};
            op.type = OP_ATTN;
            op.barrier = 1;
            op.at = at;
            rec->push_back(op);
            op.type = OP_COMBINE;
            rec->push_back(op);
        } else if (fused_decode) {
            const int p = start_pos, kf = Y.global ? 0 : (p + 1 > G4_SLIDING_WINDOW ? p + 1 - G4_SLIDING_WINDOW : 0);
            q.tag(1, (double)(p + 1 - kf) * Y.hd * 8);
            q.ck(g4_launch_attn_decode(at, kSplits, c->st, q.pdl));
            q.tag(1, 0);
            q.ck(g4_launch_attn_combine(at, kSplits, c->st, q.pdl));
        } else {
            q.ck(g4_launch_qkv_post(at, c->st, q.pdl));
            q.ck(c->strict ? g4_launch_attn_strict(at, c->st, q.pdl) : g4_launch_attn_prefill(at, c->st, q.pdl));
        }
        // o_proj
        {
            GemvArgs a = gemv_base(c, Y.o, T);
            a.out = c->h;
            a.out_stride = G4_HIDDEN;
            if (fused_decode) {
                a.xq_in = c->xq;
                a.xs_in = c->xs;
                gemv(q, a, PRO_LOADQ, EPI_STORE);
            } else {
                a.src = c->attn;
                a.src_stride = Y.qw;
                gemv(q, a, PRO_QUANT, EPI_STORE);
            }
        }
        // gate|up with post-attn norm + residual + pre-ffn norm
        {
            GemvArgs a = gemv_base(c, Y.gu, T);
            a.row_gran = 2;
            a.src = c->h;
            a.src_stride = G4_HIDDEN;
            a.w_post = Y.post_attn;
            a.res_in = c->res[cur];
            a.res_out = c->res[cur ^ 1];
            cur ^= 1;
            a.w_pre = Y.pre_ffn;
            a.out = c->gu;
            a.out_stride = Y.ffn;
            gemv(q, a, PRO_RES_NORM_QUANT, EPI_GEGLU_PAIR);
        }
        // down
        {
            GemvArgs a = gemv_base(c, Y.down, T);
            a.src = c->gu;
            a.src_stride = Y.ffn;
            a.out = c->h;
            a.out_stride = G4_HIDDEN;
            gemv(q, a, PRO_QUANT, EPI_STORE);
        }
        // per-layer input gate with post-ffn norm + residual
        {
            GemvArgs a = gemv_base(c, Y.pleg, T);
            a.src = c->h;
            a.src_stride = G4_HIDDEN;
            a.w_post = Y.post_ffn;
            a.res_in = c->res[cur];
            a.res_out = c->res[cur ^ 1];
            cur ^= 1;
            a.out = c->pg;
            a.out_stride = G4_PLE;
            a.ple_u = c->ple_u + l * G4_PLE;
            a.u_stride = G4_NUM_LAYERS * G4_PLE;
            gemv(q, a, PRO_RES_QUANT, EPI_PLE);
        }
        // per-layer projection
        {
            GemvArgs a = gemv_base(c, Y.plep, T);
            a.src = c->pg;
            a.src_stride = G4_PLE;
            a.out = c->h;
            a.out_stride = G4_HIDDEN;
            gemv(q, a, PRO_QUANT, EPI_STORE);
        }
    }
    const Layer &Z = c->L[c->layers - 1];
    if (rec) {
        DecodeOp op{};
        op.type = OP_FINISH;
        op.fin_h = c->h;
        op.fin_w = Z.post_ple;
        op.fin_res_in = c->res[cur];
        op.fin_res_out = c->res[cur ^ 1];
        op.fin_scalar = Z.scalar;
        rec->push_back(op);
    } else {
        q.ck(g4_launch_rows_norm(3, c->h, T, Z.post_ple, c->res[cur], c->res[cur ^ 1], Z.scalar, nullptr, G4_RMS_EPS,
                                 nullptr, nullptr, c->st, q.pdl, nullptr, c->strict));
    }
    cur ^= 1;
    c->cur = cur;
    return q.e;
}

// Multi-sequence batch: rows carry their own (sequence, position) (single-token
// rows of several sequences), or all rows are one sequence `seq` from start_pos.
constexpr int kRowGraphAfter = 32;   // eager steps of a row count before its graph is captured

struct BatchPlan {
    bool rows;
    int seq;
};

// Prefill attention on the tensor cores for this layer kind and chunk
// (G4_OPT_ATTN_PATH); the CUDA-core kernel otherwise. Auto: by the chunk's
// work W = sum over its tokens of the keys each sees. The tensor path has a
// fixed cost of ~33 us (four or five launches, TMEM and pipeline set-up) and
// then ~0.06 ns per unit of W, the CUDA-core kernel ~0.8 ns (global,
// 512-wide heads) or ~0.38 ns (sliding) per unit (B200). Measured: a
// 512-token chunk at position 0 (W = 131k) takes 52 vs 107 us (global) and
// 49 vs 52 us (sliding) on the tensor cores; 128 tokens at position 100
// (W = 21k) 43 vs 39 us (global).
constexpr long long kTcMinWorkGlobal = 64 * 1024, kTcMinWorkSliding = 128 * 1024;
bool attn_on_tensor_cores(const g4_ctx *c, bool global, int T, int start_pos) {
    if (c->strict || c->attn_path == 1) return false;
    if (c->attn_path == 2) return true;
    long long w = 0;
    for (int t = 0; t < T; t++) {
        const int p = start_pos + t;
        w += global || p + 1 <= G4_SLIDING_WINDOW ? p + 1 : G4_SLIDING_WINDOW;
    }
    return w >= (global ? kTcMinWorkGlobal : kTcMinWorkSliding);
}

// Tensor-core attention workspace bytes of one layer kind for a chunk of T
// tokens at start_pos; 0 if that kind does not take the path.
size_t tc_ws_need(const g4_ctx *c, bool global, int T, int start_pos, int ring_global, bool *bad) {
    if (!attn_on_tensor_cores(c, global, T, start_pos)) return 0;
    AttnArgs a{};
    a.hd = global ? 512 : 256;
    a.window = global ? 0 : G4_SLIDING_WINDOW;
    a.mask = (global ? ring_global : 1024) - 1;
    a.T = T;
    a.start_pos = start_pos;
    a.qkv = a.kcache = a.vcache = a.out = (float *)c;   // non-null placeholders: only the size is asked
    const size_t b = g4_attn_tc_ws_bytes(a);
    if (!b) *bad = true;
    return b;
}

// Grow the tensor-core attention workspace for a chunk of T tokens at
// start_pos (before any launch of the chunk: freeing waits for the stream).
// The global and the sliding layers get separate regions, so that a layer that
// reads another layer's cache can reuse that layer's K/V split of the chunk.
// A growth costs a stream drain and a large allocation (~15 ms), so it
// provisions ahead: the global region for the last chunk of the whole context
// range when the device has four times that much memory free (2.7 GB at
// 131072 positions), else for twice the need; the sliding region for its
// largest chunk (the window bounds it).
int ensure_tc_ws(g4_ctx *c, int T, int start_pos, int ring_global) {
    bool bad = false;
    const size_t ng = tc_ws_need(c, true, T, start_pos, ring_global, &bad);
    const size_t ns = tc_ws_need(c, false, T, start_pos, ring_global, &bad);
    if (bad) return fail(c, G4_ERR_INVALID, "tensor-core attention cannot run T %d at %d", T, start_pos);
    if (ng <= c->tc_ws_gcap && ns <= c->tc_ws_scap) return G4_OK;
    CK(cudaStreamSynchronize(c->st));
    if (c->tc_ws) cudaFree(c->tc_ws);
    c->tc_ws = nullptr;
    size_t wg = c->tc_ws_gcap, ws = c->tc_ws_scap;
    c->tc_ws_gcap = c->tc_ws_scap = 0;
    if (ng > wg) {
        bool bad_full = false;
        const size_t full = tc_ws_need(c, true, G4_BATCH, ring_global - G4_BATCH, ring_global, &bad_full);
        size_t free_b = 0, total_b = 0;
        wg = 2 * ng;
        if (!bad_full && full >= ng && cudaMemGetInfo(&free_b, &total_b) == cudaSuccess && free_b / 4 > full) wg = full;
    }
    {   // the sliding region at its largest with the first growth of either
        bool bad_s = false;
        const size_t smax = tc_ws_need(c, false, G4_BATCH, 4 * G4_SLIDING_WINDOW, ring_global, &bad_s);
        ws = !bad_s && smax > ws ? smax : ws;
        ws = ns > ws ? ns : ws;
    }
    wg = (wg + 1023) / 1024 * 1024;
    if (cudaMalloc(&c->tc_ws, wg + ws) != cudaSuccess) {
        cudaGetLastError();   // not sticky: retry at the exact needs
        wg = (ng + 1023) / 1024 * 1024;
        ws = ns;
        CK(cudaMalloc(&c->tc_ws, wg + ws));
    }
    c->tc_ws_gcap = wg;
    c->tc_ws_scap = ws;
    return G4_OK;
}

cudaError_t enqueue_prefill(g4_ctx *c, int T, int start_pos, const BatchPlan *bp = nullptr) {
    Seq q{c, c->use_pdl};
    int cur = 0;
    // per layer kind (sliding, global): the cache whose K/V split of this chunk
    // the tensor-core workspace region holds
    const float *tc_split_of[2] = {nullptr, nullptr};
    q.ck(g4_launch_rows_embed(c->tokens_d, T, c->embed, c->embed_ple, sqrtf((float)G4_HIDDEN), sqrtf((float)G4_PLE),
                              c->res[0], c->ple_emb, c->err, c->st, q.pdl));
    q.ck(g4_launch_rows_quant(c->res[0], G4_HIDDEN, T, G4_HIDDEN, c->xq, c->xs, c->st, q.pdl, c->xsT));
    gemm(q, c->pmp, T, EPI_STORE, c->pli, G4_NUM_LAYERS * G4_PLE, nullptr, 0);
    q.ck(g4_launch_ple_prep(c->pli, c->ple_emb, c->ple_norm, 1e-6f * G4_HIDDEN, 1.0f / sqrtf(2.0f), T, c->ple_u, c->st,
                            q.pdl, c->strict));
    for (int l = 0; l < c->layers; l++) {
        const Layer &Y = c->L[l];
        if (l == 0) {
            q.ck(g4_launch_rows_norm(0, c->res[cur], T, nullptr, nullptr, nullptr, nullptr, Y.in_norm, G4_RMS_EPS, c->xq,
                                     c->xs, c->st, q.pdl, nullptr, c->strict, c->xsT));
        } else {
            const Layer &P = c->L[l - 1];
            q.ck(g4_launch_rows_norm(1, c->h, T, P.post_ple, c->res[cur], c->res[cur ^ 1], P.scalar, Y.in_norm,
                                     G4_RMS_EPS, c->xq, c->xs, c->st, q.pdl, nullptr, c->strict, c->xsT));
            cur ^= 1;
        }
        gemm(q, Y.qkv, T, EPI_STORE, c->qkv, kQkvStride, nullptr, 0);
        AttnArgs at = attn_base(c, Y, T, start_pos, nullptr);
        if (bp) {   // the batch rings: [sequence][K ring | V ring]
            const size_t stride = (size_t)2 * c->bring[l] * Y.hd;
            at.mask = c->bring[l] - 1;
            at.kcache = c->bk[l];
            at.vcache = c->bv[l];
            if (bp->rows) {
                at.row_seq = c->row_seq_d;
                at.row_pos = c->row_pos_d;
                at.seq_stride = stride;
                at.part = c->bpart;
            } else {
                at.kcache += (size_t)bp->seq * stride;
                at.vcache += (size_t)bp->seq * stride;
            }
        }
        q.ck(g4_launch_qkv_post(at, c->st, q.pdl));
        if (bp && bp->rows) {
            // key splits per row: about four CTAs per SM over the batch but at least 16
            // (each split's tile loop is latency-bound), or a fixed count
            int sp = c->batch_splits ? c->batch_splits : (4 * c->num_sms + T - 1) / T;
            sp = sp < 16 ? 16 : sp > kSplits ? kSplits : sp;
            // the combine also quantises the rows for o_proj
            at.quant_out = 1;
            at.xq = c->xq;
            at.xs = c->xs;
            at.xsT = c->xsT;
            q.ck(g4_launch_attn_rows(at, sp, c->st, q.pdl));
        }
        else if (!c->strict) {
            // the tiled kernels also quantise their output rows for o_proj
            at.quant_out = 1;
            at.xsT = c->xsT;
            if (attn_on_tensor_cores(c, Y.global, T, start_pos)) {
                const int kind = Y.global ? 1 : 0;
                at.reuse_kv = !Y.has_kv && tc_split_of[kind] == at.kcache;
                uint8_t *ws = (uint8_t *)c->tc_ws + (kind ? 0 : c->tc_ws_gcap);
                q.ck(g4_launch_attn_tc(at, ws, kind ? c->tc_ws_gcap : c->tc_ws_scap, c->st, q.pdl));
                tc_split_of[kind] = at.kcache;
            } else
                q.ck(g4_launch_attn_prefill(at, c->st, q.pdl));
        } else
            q.ck(g4_launch_attn_strict(at, c->st, q.pdl));
        if (!at.quant_out) q.ck(g4_launch_rows_quant(c->attn, Y.qw, T, Y.qw, c->xq, c->xs, c->st, q.pdl, c->xsT));
        gemm(q, Y.o, T, EPI_STORE, c->h, G4_HIDDEN, nullptr, 0);
        q.ck(g4_launch_rows_norm(1, c->h, T, Y.post_attn, c->res[cur], c->res[cur ^ 1], nullptr, Y.pre_ffn, G4_RMS_EPS,
                                 c->xq, c->xs, c->st, q.pdl, nullptr, c->strict, c->xsT));
        cur ^= 1;
        if (gemm(q, Y.gu, T, EPI_GEGLU_PAIR, c->gu, Y.ffn, nullptr, 0, true)) {
            // down_proj reads the second set the fused epilogue wrote
            std::swap(c->xq, c->xq2);
            std::swap(c->xs, c->xs2);
            std::swap(c->xsT, c->xsT2);
            gemm(q, Y.down, T, EPI_STORE, c->h, G4_HIDDEN, nullptr, 0);
            std::swap(c->xq, c->xq2);
            std::swap(c->xs, c->xs2);
            std::swap(c->xsT, c->xsT2);
        } else {
            q.ck(g4_launch_rows_quant(c->gu, Y.ffn, T, Y.ffn, c->xq, c->xs, c->st, q.pdl, c->xsT));
            gemm(q, Y.down, T, EPI_STORE, c->h, G4_HIDDEN, nullptr, 0);
        }
        q.ck(g4_launch_rows_norm(2, c->h, T, Y.post_ffn, c->res[cur], c->res[cur ^ 1], nullptr, nullptr, G4_RMS_EPS,
                                 c->xq, c->xs, c->st, q.pdl, nullptr, c->strict, c->xsT));
        cur ^= 1;
        gemm(q, Y.pleg, T, EPI_PLE, c->pg, G4_PLE, c->ple_u + l * G4_PLE, G4_NUM_LAYERS * G4_PLE);
        q.ck(g4_launch_rows_quant(c->pg, G4_PLE, T, G4_PLE, c->xq, c->xs, c->st, q.pdl, c->xsT));
        gemm(q, Y.plep, T, EPI_STORE, c->h, G4_HIDDEN, nullptr, 0);
    }
    const Layer &Z = c->L[c->layers - 1];
    q.ck(g4_launch_rows_norm(3, c->h, T, Z.post_ple, c->res[cur], c->res[cur ^ 1], Z.scalar, nullptr, G4_RMS_EPS,
                             nullptr, nullptr, c->st, q.pdl, nullptr, c->strict));
    cur ^= 1;
    c->cur = cur;
    return q.e;
}

// Record the single-token step as persistent-decode op lists (forward only, and
// forward + logits of row 0) and upload them; called once the context exists.
void drop_row_graphs(g4_ctx *c) {
    for (cudaGraphExec_t &g : c->g_rows)
        if (g) cudaGraphExecDestroy(g);
    c->g_rows.clear();
    c->rows_warm.clear();
}

void free_decode(g4_ctx *c) {
    if (c->dec_fwd) cudaFree(c->dec_fwd);
    if (c->dec_fwdlog) cudaFree(c->dec_fwdlog);
    c->dec_fwd = c->dec_fwdlog = nullptr;
    c->n_fwd = c->n_fwdlog = 0;
    c->dec_layers = 0;
    c->dec_host.clear();
    if (c->trace) cudaFree(c->trace);
    c->trace = nullptr;
}

int build_decode(g4_ctx *c) {
    if (c->dec_fwd && c->dec_layers == c->layers) return G4_OK;
    free_decode(c);
    std::vector<DecodeOp> ops;
    const int cur_save = c->cur;
    cudaError_t e = enqueue_small(c, 1, 0, c->pos_d, nullptr, &ops);
    c->dec_cur = c->cur;
    c->cur = cur_save;
    if (e) return fail(c, G4_ERR_CUDA, "decode op list: %s", cudaGetErrorString(e));
    ops.back().barrier = 0;
    for (DecodeOp &op : ops)
        if (op.type == OP_GEMV) g4_decode_set_partition(op, c->num_sms);
    std::vector<DecodeOp> withlog(ops);
    // replace the last residual update by the lm_head GEMV whose prologue performs it
    const DecodeOp fin = withlog.back();
    DecodeOp lm{};
    lm.type = OP_GEMV;
    lm.pro = PRO_RES_NORM_QUANT;
    lm.epi = EPI_LOGITS;
    lm.g = gemv_base(c, c->embed, 1);
    lm.g.src = fin.fin_h;
    lm.g.src_stride = G4_HIDDEN;
    lm.g.w_post = fin.fin_w;
    lm.g.scalar = fin.fin_scalar;
    lm.g.res_in = fin.fin_res_in;
    lm.g.res_out = fin.fin_res_out;
    lm.g.w_pre = c->final_norm;
    lm.g.out = c->logits;
    lm.g.out_stride = G4_VOCAB;
    lm.g.argmax_part = c->argmax_part;
    lm.g.argmax_out = c->argmax_out;
    lm.g.ticket = c->ticket;
    g4_decode_set_partition(lm, c->num_sms);
    withlog.back() = lm;
    if (g4_decode_max_stages(ops.data(), (int)ops.size(), c->num_sms) > (1 << 20) ||
        g4_decode_max_stages(withlog.data(), (int)withlog.size(), c->num_sms) > (1 << 20) || c->num_sms < kSplits) {
        c->persistent = false;   // geometry outside the persistent kernel's limits: keep the graph path
        return G4_OK;
    }
    CK(cudaMalloc(&c->dec_fwd, ops.size() * sizeof(DecodeOp)));
    CK(cudaMalloc(&c->dec_fwdlog, withlog.size() * sizeof(DecodeOp)));
    CK(cudaMemcpy(c->dec_fwd, ops.data(), ops.size() * sizeof(DecodeOp), cudaMemcpyHostToDevice));
    CK(cudaMemcpy(c->dec_fwdlog, withlog.data(), withlog.size() * sizeof(DecodeOp), cudaMemcpyHostToDevice));
    c->n_fwd = (int)ops.size();
    c->n_fwdlog = (int)withlog.size();
    c->dec_layers = c->layers;
    c->dec_host = withlog;
    return G4_OK;
}

cudaError_t launch_decode(g4_ctx *c, bool with_logits, unsigned long long *trace = nullptr) {
    DecodeParams p{};
    p.trace = trace;
    p.ops = with_logits ? c->dec_fwdlog : c->dec_fwd;
    p.nops = with_logits ? c->n_fwdlog : c->n_fwd;
    p.splits = kSplits;
    p.pos = c->pos_d;
    p.bar = c->bar;
    p.bar_base = c->bar_base;
    p.err = c->err;
    p.starve = c->starve_next ? 1 : 0;
    c->starve_next = false;
    return g4_launch_decode(p, c->num_sms, c->st);
}

// Launch a deferred single-token forward on its own (without logits).
int flush_pending(g4_ctx *c) {
    if (!c->pending) return G4_OK;
    c->pending = false;
    cudaError_t e = launch_decode(c, false);
    if (e) return fail(c, G4_ERR_CUDA, "decode launch: %s", cudaGetErrorString(e));
    return G4_OK;
}

int check_device_error(g4_ctx *c) {
    int e = 0;
    cudaError_t ce = cudaMemcpyAsync(&e, c->err, 4, cudaMemcpyDeviceToHost, c->st);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(c->st);
    if (ce != cudaSuccess) return fail(c, G4_ERR_CUDA, "device: %s", cudaGetErrorString(ce));
    if (e) {
        cudaMemsetAsync(c->err, 0, 4, c->st);
        if (c->bar) cudaMemsetAsync(c->bar, 0, 16, c->st);   // a failed persistent step leaves them uneven
        cudaStreamSynchronize(c->st);
        const int code = e & 0xff;
        const char *what = code == G4D_BAD_TOKEN ? "token id outside the vocabulary"
                           : code == G4D_TIMEOUT_FULL || code == G4D_TIMEOUT_EMPTY ? "kernel wait timed out"
                                                                                    : "kernel error";
        return fail(c, G4_ERR_DEVICE, "device reported error %d (stage %d, block %d): %s", code, (e >> 8) & 0xfff,
                    (unsigned)e >> 20, what);
    }
    return G4_OK;
}

}  // namespace

// ---------------------------------------------------------------------------
// C ABI

cudaError_t g4_smem_optin(const void *kernel, int bytes) {
    static std::mutex mu;
    static std::vector<std::pair<int, const void *>> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    for (const auto &d : done)
        if (d.first == dev && d.second == kernel) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done.emplace_back(dev, kernel);
    return e;
}

int g4_device_sms() {
    int dev = 0, n = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

extern "C" {

const char *g4_strerror(int code) {
    switch (code) {
    case G4_OK: return "ok";
    case G4_ERR_INVALID: return "invalid argument";
    case G4_ERR_FORMAT: return "bad model image";
    case G4_ERR_CUDA: return "CUDA error";
    case G4_ERR_NOMEM: return "out of memory";
    case G4_ERR_DEVICE: return "device-side error";
    case G4_ERR_STATE: return "call out of sequence";
    default: return "unknown error";
    }
}

const char *g4_last_error(g4_ctx *c) { return c ? c->msg : "no context"; }

static char g_open_msg[512];

int g4_open(const void *image, uint64_t bytes, int device, g4_ctx **out) {
    if (!out) return G4_ERR_INVALID;
    *out = nullptr;
    if (!image || device < 0) return G4_ERR_INVALID;
    g4_ctx *c = new g4_ctx();
    c->device = device;
    int rc = open_impl(c, (const uint8_t *)image, bytes);
    if (rc) {
        snprintf(g_open_msg, sizeof(g_open_msg), "%s", c->msg);
        g4_close(c);
        return rc;
    }
    *out = c;
    return G4_OK;
}

const char *g4_open_error(void) { return g_open_msg; }

// The .bin straight to the device: the file is read in 64 MB pieces into two
// page-locked buffers, each piece copied to a device-resident image while the
// next one is read; the repacking then reads that image (device to device).
// Only the header and record table are parsed from a host copy.
int g4_open_file(const char *path, int device, g4_ctx **out) {
    if (!path || !out || device < 0) return G4_ERR_INVALID;
    *out = nullptr;
    FILE *f = fopen(path, "rb");
    if (!f) return G4_ERR_INVALID;
    fseek(f, 0, SEEK_END);
    const long long n = ftell(f);
    fseek(f, 0, SEEK_SET);
    const size_t hdr_bytes = (size_t)G4_WEIGHTS_OFFSET + (size_t)G4_NUM_RECORDS * G4_RECORD_BYTES;
    if (n < (long long)hdr_bytes) {
        fclose(f);
        return G4_ERR_FORMAT;
    }
    constexpr size_t kPiece = 64ull << 20;
    int rc = G4_OK;
    uint8_t *hdr = (uint8_t *)malloc(hdr_bytes);
    uint8_t *pin[2] = {nullptr, nullptr};
    uint8_t *dimg = nullptr;
    cudaStream_t st = nullptr;
    cudaEvent_t ev[2] = {nullptr, nullptr};
    if (!hdr || cudaSetDevice(device) != cudaSuccess || cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) ||
        cudaMalloc(&dimg, (size_t)n) != cudaSuccess || cudaHostAlloc(&pin[0], kPiece, 0) != cudaSuccess ||
        cudaHostAlloc(&pin[1], kPiece, 0) != cudaSuccess || cudaEventCreate(&ev[0]) || cudaEventCreate(&ev[1])) {
        rc = G4_ERR_NOMEM;
    }
    for (size_t off = 0, i = 0; rc == G4_OK && off < (size_t)n; off += kPiece, i++) {
        const size_t len = (size_t)n - off < kPiece ? (size_t)n - off : kPiece;
        uint8_t *b = pin[i & 1];
        if (i >= 2 && cudaEventSynchronize(ev[i & 1]) != cudaSuccess) rc = G4_ERR_CUDA;   // its last copy is done
        if (rc == G4_OK && fread(b, 1, len, f) != len) rc = G4_ERR_FORMAT;
        if (rc == G4_OK && off < hdr_bytes)
            memcpy(hdr + off, b, hdr_bytes - off < len ? hdr_bytes - off : len);
        if (rc == G4_OK && (cudaMemcpyAsync(dimg + off, b, len, cudaMemcpyHostToDevice, st) != cudaSuccess ||
                            cudaEventRecord(ev[i & 1], st) != cudaSuccess))
            rc = G4_ERR_CUDA;
    }
    fclose(f);
    if (st && cudaStreamSynchronize(st) != cudaSuccess && rc == G4_OK) rc = G4_ERR_CUDA;
    if (rc == G4_OK) {
        g4_ctx *c = new g4_ctx();
        c->device = device;
        rc = open_impl(c, dimg, (uint64_t)n, hdr);
        if (rc != G4_OK) {
            snprintf(g_open_msg, sizeof(g_open_msg), "%s", c->msg);
            g4_close(c);
        } else {
            *out = c;
        }
    }
    for (int i = 0; i < 2; i++) {
        if (pin[i]) cudaFreeHost(pin[i]);
        if (ev[i]) cudaEventDestroy(ev[i]);
    }
    if (st) cudaStreamDestroy(st);
    if (dimg) cudaFree(dimg);
    free(hdr);
    return rc;
}

int g4_close(g4_ctx *c) {
    if (!c) return G4_ERR_INVALID;
    flush_pending(c);
    if (c->st) cudaStreamSynchronize(c->st);
    free_decode(c);
    drop_row_graphs(c);
    if (c->g_decode) cudaGraphExecDestroy(c->g_decode);
    for (int i = 0; i < 16; i++)
        if (c->events[i]) cudaEventDestroy(c->events[i]);
    if (c->arena) cudaFree(c->arena);
    if (c->scales_t) cudaFree(c->scales_t);
    if (c->dump_st) cudaStreamSynchronize(c->dump_st);
    for (int i = 0; i < 2; i++) {
        if (c->dump_done[i]) cudaEventDestroy(c->dump_done[i]);
        if (c->dump_copied[i]) cudaEventDestroy(c->dump_copied[i]);
    }
    if (c->dump_st) cudaStreamDestroy(c->dump_st);
    if (c->dump_buf) cudaFree(c->dump_buf);
    if (c->bkv) cudaFree(c->bkv);
    if (c->bbuf) cudaFree(c->bbuf);
    if (c->state) cudaFree(c->state);
    if (c->kv) cudaFree(c->kv);
    if (c->scores) cudaFree(c->scores);
    if (c->tc_ws) cudaFree(c->tc_ws);
    if (c->st) cudaStreamDestroy(c->st);
    delete c;
    return G4_OK;
}

int g4_set_option(g4_ctx *c, int option, int value) {
    if (!c) return G4_ERR_INVALID;
    int rc = flush_pending(c);
    if (rc) return rc;
    drop_row_graphs(c);   // every option can change what a multi-sequence step launches
    switch (option) {
    case G4_OPT_PERSISTENT: c->persistent = value != 0; break;
    case G4_OPT_BATCH_SPLITS:
        if (value < 0 || value > kSplits) return fail(c, G4_ERR_INVALID, "batch splits %d out of range", value);
        c->batch_splits = value;
        break;
    case G4_OPT_GRAPHS: c->use_graph = value != 0; break;
    case G4_OPT_PDL:
        c->use_pdl = value != 0;
        if (c->g_decode) { cudaGraphExecDestroy(c->g_decode); c->g_decode = nullptr; }
        break;
    case G4_OPT_GEMM_PATH: c->gemm_path = value; break;
    case G4_OPT_ATTN_PATH:
        if (value < 0 || value > 2) return fail(c, G4_ERR_INVALID, "attention path %d out of range", value);
        c->attn_path = value;
        break;
    case G4_OPT_STRICT: c->strict = value != 0; break;
    case G4_OPT_LAYERS:
        if (value < 1 || value > G4_NUM_LAYERS) return fail(c, G4_ERR_INVALID, "layers %d out of range", value);
        c->layers = value;
        if (c->g_decode) { cudaGraphExecDestroy(c->g_decode); c->g_decode = nullptr; }
        CK(cudaStreamSynchronize(c->st));
        free_decode(c);
        break;
    default: return fail(c, G4_ERR_INVALID, "unknown option %d", option);
    }
    return G4_OK;
}

int g4_forward(g4_ctx *c, const int *tokens, size_t count, int start_pos) {
    if (!c) return G4_ERR_INVALID;
    if (!tokens || count < 1 || count > (size_t)kMaxT || start_pos < 0 ||
        (long long)start_pos + (long long)count > G4_MAX_CONTEXT)
        return fail(c, G4_ERR_INVALID, "forward: count %zu start_pos %d out of range", count, start_pos);
    for (size_t i = 0; i < count; i++)
        if (tokens[i] < 0 || tokens[i] >= G4_VOCAB) return fail(c, G4_ERR_INVALID, "forward: token %d out of range", tokens[i]);
    cudaSetDevice(c->device);
    int rc = flush_pending(c);
    if (rc) return rc;
    const int T = (int)count;
    if (T == 1 && c->persistent && !c->strict) {
        rc = build_decode(c);
        if (rc) return rc;
    }
    if (c->strict) {
        const size_t need = (size_t)T * G4_HEADS * ((size_t)start_pos + T) * 4;
        if (need > c->scores_cap) {
            CK(cudaStreamSynchronize(c->st));
            if (c->scores) cudaFree(c->scores);
            c->scores = nullptr;
            c->scores_cap = 0;
            CK(cudaMalloc(&c->scores, need));
            c->scores_cap = need;
        }
    }
    CK(cudaMemcpyAsync(c->tokens_d, tokens, count * 4, cudaMemcpyHostToDevice, c->st));
    cudaError_t e;
    if (T == 1 && c->persistent && !c->strict) {
        // deferred: launched by the next call, fused with the lm_head when that call is g4_logits
        CK(cudaMemcpyAsync(c->pos_d, &start_pos, 4, cudaMemcpyHostToDevice, c->st));
        c->pending = true;
        c->cur = c->dec_cur;
    } else if (T == 1 && c->use_graph && !c->strict) {
        CK(cudaMemcpyAsync(c->pos_d, &start_pos, 4, cudaMemcpyHostToDevice, c->st));
        if (!c->g_decode) {
            if (!c->decode_warm) {
                // first call runs eagerly (sets kernel attributes), later calls replay the graph
                e = enqueue_small(c, 1, start_pos, c->pos_d);
                if (e) return fail(c, G4_ERR_CUDA, "decode launch: %s", cudaGetErrorString(e));
                c->decode_warm = true;
                c->graph_cur = c->cur;
                c->last_T = T;
                return G4_OK;
            }
            cudaGraph_t g = nullptr;
            CK(cudaStreamBeginCapture(c->st, cudaStreamCaptureModeThreadLocal));
            e = enqueue_small(c, 1, start_pos, c->pos_d);
            cudaError_t e2 = cudaStreamEndCapture(c->st, &g);
            if (e || e2) {
                if (g) cudaGraphDestroy(g);
                return fail(c, G4_ERR_CUDA, "decode capture: %s", cudaGetErrorString(e ? e : e2));
            }
            e = cudaGraphInstantiate(&c->g_decode, g, 0);
            cudaGraphDestroy(g);
            if (e) return fail(c, G4_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(e));
            c->graph_cur = c->cur;
        }
        CK(cudaGraphLaunch(c->g_decode, c->st));
        c->cur = c->graph_cur;
    } else if (T <= 4) {
        e = enqueue_small(c, T, start_pos, nullptr);
        if (e) return fail(c, G4_ERR_CUDA, "decode launch: %s", cudaGetErrorString(e));
    } else {
        rc = ensure_tc_ws(c, T, start_pos, G4_MAX_CONTEXT);
        if (rc) return rc;
        e = enqueue_prefill(c, T, start_pos);
        if (e) return fail(c, G4_ERR_CUDA, "prefill launch: %s", cudaGetErrorString(e));
    }
    c->last_T = T;
    return G4_OK;
}

static cudaError_t enqueue_logits(g4_ctx *c, size_t row, Prof *prof = nullptr) {
    GemvArgs a = gemv_base(c, c->embed, 1);
    a.src = c->res[c->cur] + row * G4_HIDDEN;
    a.src_stride = G4_HIDDEN;
    a.w_pre = c->final_norm;
    a.out = c->logits;
    a.out_stride = G4_VOCAB;
    a.argmax_part = c->argmax_part;
    a.argmax_out = c->argmax_out;
    a.ticket = c->ticket;
    Seq q{c, c->use_pdl && !prof};
    q.prof = prof;
    gemv(q, a, PRO_NORM_QUANT, EPI_LOGITS);
    return q.e;
}

int g4_logits(g4_ctx *c, size_t row, float *out, int *argmax) {
    if (!c) return G4_ERR_INVALID;
    if (c->last_T == 0 || row >= (size_t)c->last_T)
        return fail(c, G4_ERR_STATE, "logits: row %zu not computed by the last forward (%d rows)", row, c->last_T);
    cudaSetDevice(c->device);
    if (c->pending) {
        // one persistent launch: the deferred single-token forward and its logits
        c->pending = false;
        cudaError_t e = launch_decode(c, true);
        if (e) return fail(c, G4_ERR_CUDA, "decode launch: %s", cudaGetErrorString(e));
        if (!out && !argmax) return G4_OK;
        if (out) CK(cudaMemcpyAsync(out, c->logits, (size_t)G4_VOCAB * 4, cudaMemcpyDeviceToHost, c->st));
        if (argmax) CK(cudaMemcpyAsync(argmax, c->argmax_out, 4, cudaMemcpyDeviceToHost, c->st));
        return check_device_error(c);
    }
    if (!out && !argmax) {
        // nothing to return: enqueue only (the reference benchmark discards logits, gemma4.c:641)
        cudaError_t e = enqueue_logits(c, row);
        if (e) return fail(c, G4_ERR_CUDA, "logits launch: %s", cudaGetErrorString(e));
        return G4_OK;
    }
    GemvArgs a = gemv_base(c, c->embed, 1);
    a.src = c->res[c->cur] + row * G4_HIDDEN;
    a.src_stride = G4_HIDDEN;
    a.w_pre = c->final_norm;
    a.out = c->logits;
    a.out_stride = G4_VOCAB;
    a.argmax_part = c->argmax_part;
    a.argmax_out = c->argmax_out;
    a.ticket = c->ticket;
    Seq q{c, c->use_pdl};
    gemv(q, a, PRO_NORM_QUANT, EPI_LOGITS);
    if (q.e) return fail(c, G4_ERR_CUDA, "logits launch: %s", cudaGetErrorString(q.e));
    if (out) CK(cudaMemcpyAsync(out, c->logits, (size_t)G4_VOCAB * 4, cudaMemcpyDeviceToHost, c->st));
    if (argmax) CK(cudaMemcpyAsync(argmax, c->argmax_out, 4, cudaMemcpyDeviceToHost, c->st));
    return check_device_error(c);
}

int g4_topk(g4_ctx *c, size_t row, int k, float *values, int *ids) {
    if (!c || !values || !ids || k < 1 || k > 64) return G4_ERR_INVALID;
    int rc = g4_logits(c, row, nullptr, nullptr);
    if (rc) return rc;
    CK(g4_launch_topk(c->logits, G4_VOCAB, k, c->topk_v, c->topk_i, c->topk_v + 1024 * 32, c->topk_i + 1024 * 32,
                      c->st));
    CK(cudaMemcpyAsync(values, c->topk_v + 1024 * 32, (size_t)k * 4, cudaMemcpyDeviceToHost, c->st));
    CK(cudaMemcpyAsync(ids, c->topk_i + 1024 * 32, (size_t)k * 4, cudaMemcpyDeviceToHost, c->st));
    return check_device_error(c);
}

int g4_set_seed(g4_ctx *c, uint64_t seed) {
    if (!c) return G4_ERR_INVALID;
    cudaSetDevice(c->device);
    int rc = flush_pending(c);
    if (rc) return rc;
    const unsigned long long v = seed;
    CK(cudaMemcpyAsync(c->rng_d, &v, 8, cudaMemcpyHostToDevice, c->st));
    CK(cudaStreamSynchronize(c->st));
    return G4_OK;
}

int g4_sample(g4_ctx *c, size_t row, float temperature, int *token) {
    if (!c || !token) return G4_ERR_INVALID;
    if (!(temperature > 0.0f)) return g4_logits(c, row, nullptr, token);   // greedy: the first maximum
    int rc = g4_logits(c, row, nullptr, nullptr);
    if (rc) return rc;
    CK(g4_launch_topk(c->logits, G4_VOCAB, 64, c->topk_v, c->topk_i, c->topk_v + 1024 * 32, c->topk_i + 1024 * 32,
                      c->st));
    CK(g4_launch_sample64(c->topk_v + 1024 * 32, c->topk_i + 1024 * 32, temperature, c->rng_d, c->sample_tok,
                          c->st));
    CK(cudaMemcpyAsync(token, c->sample_tok, 4, cudaMemcpyDeviceToHost, c->st));
    return check_device_error(c);
}

int g4_sync(g4_ctx *c) {
    if (!c) return G4_ERR_INVALID;
    cudaSetDevice(c->device);
    int rc = flush_pending(c);
    if (rc) return rc;
    return check_device_error(c);
}

int g4_read_residual(g4_ctx *c, size_t rows, float *out) {
    if (!c || !out || rows > (size_t)kMaxT) return G4_ERR_INVALID;
    cudaSetDevice(c->device);
    int rc = flush_pending(c);
    if (rc) return rc;
    CK(cudaMemcpyAsync(out, c->res[c->cur], rows * G4_HIDDEN * 4, cudaMemcpyDeviceToHost, c->st));
    return check_device_error(c);
}

int g4_read_cache(g4_ctx *c, int layer, int which, int slot0, int nslots, float *out) {
    if (!c || !out || layer < 0 || layer >= G4_NUM_LAYERS || nslots < 0) return G4_ERR_INVALID;
    const Layer &Y = c->L[layer];
    if (slot0 < 0 || slot0 + nslots > Y.ring) return G4_ERR_INVALID;
    cudaSetDevice(c->device);
    int rc = flush_pending(c);
    if (rc) return rc;
    const float *src = (which ? Y.vcache : Y.kcache) + (size_t)slot0 * Y.hd;
    CK(cudaMemcpyAsync(out, src, (size_t)nslots * Y.hd * 4, cudaMemcpyDeviceToHost, c->st));
    return check_device_error(c);
}

int g4_read_ple(g4_ctx *c, size_t rows, float *out) {
    if (!c || !out || rows > (size_t)kMaxT) return G4_ERR_INVALID;
    cudaSetDevice(c->device);
    int rc = flush_pending(c);
    if (rc) return rc;
    CK(cudaMemcpyAsync(out, c->ple_u, rows * G4_NUM_LAYERS * G4_PLE * 4, cudaMemcpyDeviceToHost, c->st));
    return check_device_error(c);
}

int g4_read_seq_cache(g4_ctx *c, int seq, int layer, int which, int slot0, int nslots, float *out) {
    if (!c || !out || layer < 0 || layer >= G4_NUM_LAYERS || nslots < 0 || seq < 0 || seq >= c->max_seqs)
        return G4_ERR_INVALID;
    const int ring = c->bring[layer], hd = c->L[layer].hd;
    if (slot0 < 0 || slot0 + nslots > ring) return G4_ERR_INVALID;
    cudaSetDevice(c->device);
    int rc = flush_pending(c);
    if (rc) return rc;
    const size_t stride = (size_t)2 * ring * hd;   // one sequence's K ring then V ring
    const float *src = (which ? c->bv[layer] : c->bk[layer]) + (size_t)seq * stride + (size_t)slot0 * hd;
    CK(cudaMemcpyAsync(out, src, (size_t)nslots * hd * 4, cudaMemcpyDeviceToHost, c->st));
    return check_device_error(c);
}

void *g4_stream(g4_ctx *c) {
    if (!c) return nullptr;
    flush_pending(c);   // work the caller enqueues next must follow the last forward
    return (void *)c->st;
}

int g4_mark(g4_ctx *c, int slot) {
    if (!c || slot < 0 || slot >= 16) return G4_ERR_INVALID;
    int rc = flush_pending(c);
    if (rc) return rc;
    if (!c->events[slot]) CK(cudaEventCreate(&c->events[slot]));
    CK(cudaEventRecord(c->events[slot], c->st));
    return G4_OK;
}

int g4_elapsed(g4_ctx *c, int a, int b, float *ms) {
    if (!c || !ms || a < 0 || b < 0 || a >= 16 || b >= 16 || !c->events[a] || !c->events[b]) return G4_ERR_INVALID;
    CK(cudaEventSynchronize(c->events[b]));
    CK(cudaEventElapsedTime(ms, c->events[a], c->events[b]));
    return G4_OK;
}

// Algorithmic bytes of one persistent-decode op at position pos.
static double op_bytes(const g4_ctx *c, const DecodeOp &op, int pos) {
    if (op.type == OP_GEMV) return (double)op.g.m.N * op.g.m.K + (double)op.g.m.N * (op.g.m.K / 64) * 2;
    if (op.type == OP_ATTN) {
        const int kf = op.at.window && pos + 1 > op.at.window ? pos + 1 - op.at.window : 0;
        return (double)(pos + 1 - kf) * op.at.hd * 8;
    }
    (void)c;
    return 0.0;
}

int g4_trace_decode(g4_ctx *c, int token, int pos, int cap, int *types, double *t_ns, int *nops) {
    if (!c || !nops || token < 0 || token >= G4_VOCAB || pos < 0 || pos >= G4_MAX_CONTEXT || cap < 0 ||
        (cap > 0 && (!types || !t_ns)))
        return G4_ERR_INVALID;
    cudaSetDevice(c->device);
    if (int rc = flush_pending(c)) return rc;
    if (!c->persistent || c->strict) return fail(c, G4_ERR_STATE, "trace: persistent decode is off");
    if (int rc = build_decode(c)) return rc;
    if (!c->persistent) return fail(c, G4_ERR_STATE, "trace: persistent decode unavailable on this device");
    const int n = c->n_fwdlog;
    const size_t tb = (size_t)(1 + 6 * n) * sizeof(unsigned long long);
    if (!c->trace) CK(cudaMalloc(&c->trace, tb));
    std::vector<unsigned long long> h(1 + 6 * n);
    CK(cudaMemcpyAsync(c->tokens_d, &token, 4, cudaMemcpyHostToDevice, c->st));
    CK(cudaMemcpyAsync(c->pos_d, &pos, 4, cudaMemcpyHostToDevice, c->st));
    CK(cudaMemsetAsync(c->trace, 0, tb, c->st));
    cudaError_t e = launch_decode(c, true, c->trace);
    if (e) return fail(c, G4_ERR_CUDA, "decode launch: %s", cudaGetErrorString(e));
    c->last_T = 1;
    c->cur = c->dec_cur;
    CK(cudaMemcpyAsync(h.data(), c->trace, tb, cudaMemcpyDeviceToHost, c->st));
    if (int rc = check_device_error(c)) return rc;
    *nops = n;
    for (int i = 0; i < n && i < cap; i++) {
        types[i] = c->dec_host[i].type;
        for (int k = 0; k < 6; k++) {
            const unsigned long long t = h[1 + 6 * i + k];
            if (k == 3) t_ns[6 * i + k] = (double)t;                     // a duration
            else t_ns[6 * i + k] = t ? (double)t - (double)h[0] : -1.0;   // producer may start first
        }
    }
    return G4_OK;
}

int g4_profile_decode(g4_ctx *c, int token, int pos, float ms[3], double bytes[3], int launches[3]) {
    if (!c || !ms || !bytes || !launches || token < 0 || token >= G4_VOCAB || pos < 0 || pos >= G4_MAX_CONTEXT)
        return G4_ERR_INVALID;
    cudaSetDevice(c->device);
    if (int rc0 = flush_pending(c)) return rc0;
    if (c->persistent && !c->strict) {
        // one traced persistent step: an op's time runs from the previous barrier exit to its own
        if (int rc0 = build_decode(c)) return rc0;
    }
    if (c->persistent && !c->strict) {
        std::vector<int> types(c->n_fwdlog);
        std::vector<double> t(6 * (size_t)c->n_fwdlog);
        int n = 0;
        if (int rc0 = g4_trace_decode(c, token, pos, (int)types.size(), types.data(), t.data(), &n)) return rc0;
        for (int k = 0; k < 3; k++) { ms[k] = 0; bytes[k] = 0; launches[k] = 0; }
        double prev = 0.0;
        for (int i = 0; i < n; i++) {
            const int cls = types[i] == OP_GEMV ? 0 : (types[i] == OP_ATTN || types[i] == OP_COMBINE) ? 1 : 2;
            const double end = t[6 * i + 2];
            ms[cls] += (float)((end - prev) * 1e-6);
            bytes[cls] += op_bytes(c, c->dec_host[i], pos);
            launches[cls]++;
            prev = end;
        }
        return G4_OK;
    }
    Prof *pr = new Prof();
    for (int i = 0; i <= Prof::kMax; i++) cudaEventCreate(&pr->ev[i]);
    int rc = G4_OK;
    cudaError_t e = cudaMemcpyAsync(c->tokens_d, &token, 4, cudaMemcpyHostToDevice, c->st);
    if (!e) e = cudaMemcpyAsync(c->pos_d, &pos, 4, cudaMemcpyHostToDevice, c->st);
    if (!e) e = cudaEventRecord(pr->ev[0], c->st);
    if (!e) e = enqueue_small(c, 1, pos, nullptr, pr);
    c->last_T = 1;
    if (!e) e = enqueue_logits(c, 0, pr);
    if (!e) e = cudaStreamSynchronize(c->st);
    for (int k = 0; k < 3; k++) { ms[k] = 0; bytes[k] = 0; launches[k] = 0; }
    if (e) rc = fail(c, G4_ERR_CUDA, "profile: %s", cudaGetErrorString(e));
    else {
        for (int i = 0; i < pr->n; i++) {
            float t = 0;
            cudaEventElapsedTime(&t, pr->ev[i], pr->ev[i + 1]);
            ms[pr->cls[i]] += t;
            bytes[pr->cls[i]] += pr->bytes[i];
            launches[pr->cls[i]]++;
        }
    }
    for (int i = 0; i <= Prof::kMax; i++) cudaEventDestroy(pr->ev[i]);
    delete pr;
    return rc ? rc : check_device_error(c);
}

int g4_test_starve_next_step(g4_ctx *c) {
    if (!c) return G4_ERR_INVALID;
    if (!c->persistent || c->strict) return fail(c, G4_ERR_STATE, "starve: persistent decode is off");
    c->starve_next = true;
    return G4_OK;
}

int g4_launches_per_token(g4_ctx *c, int *n) {
    if (!c || !n) return G4_ERR_INVALID;
    // embed/PLE GEMV + PLE prep, 7 kernels per layer (qkv, attention, combine,
    // o, gate|up, down, ple gate, ple proj => 8), final residual, logits
    *n = (c->persistent && !c->strict) ? 1 : 2 + 8 * c->layers + 1 + 1;
    return G4_OK;
}

int g4_profiler_range(int on) {
    cudaError_t e = on ? cudaProfilerStart() : cudaProfilerStop();
    return e == cudaSuccess ? G4_OK : G4_ERR_CUDA;
}

int g4_device_bytes(g4_ctx *c, uint64_t *weights, uint64_t *total) {
    if (!c) return G4_ERR_INVALID;
    if (weights) *weights = c->arena_used;
    if (total) *total = c->arena_bytes + c->kv_bytes + c->bkv_bytes;
    return G4_OK;
}

// ---- multi-sequence serving ------------------------------------------------

int g4_seq_alloc(g4_ctx *c, int max_seqs, int max_context) {
    if (!c || max_seqs < 1 || max_seqs > G4_MAX_SEQS || max_context < 1 || max_context > G4_MAX_CONTEXT)
        return G4_ERR_INVALID;
    cudaSetDevice(c->device);
    if (int rc = flush_pending(c)) return rc;
    CK(cudaStreamSynchronize(c->st));
    drop_row_graphs(c);   // the graphs hold the old rings' addresses
    if (c->bkv) cudaFree(c->bkv);
    if (c->bbuf) cudaFree(c->bbuf);
    c->bkv = c->bbuf = nullptr;
    c->max_seqs = 0;
    c->blast.clear();
    int gring = 1024;
    while (gring < max_context) gring <<= 1;
    // per sequence: the 12 sliding owner rings (1024 slots) and the 3 global owner rings (gring slots)
    const size_t sl = (size_t)2 * G4_SLIDING_RING * G4_HD_SLIDING * 4, gl = (size_t)2 * gring * G4_HD_GLOBAL * 4;
    c->bkv_bytes = (size_t)max_seqs * (12 * sl + 3 * gl);
    if (cudaMalloc(&c->bkv, c->bkv_bytes) != cudaSuccess) {
        c->bkv = nullptr;
        c->bkv_bytes = 0;
        return fail(c, G4_ERR_NOMEM, "sequence KV: %zu bytes", (size_t)max_seqs * (12 * sl + 3 * gl));
    }
    for (int l = 0; l < G4_NUM_LAYERS; l++) {
        const Layer &Y = c->L[l];
        const int o = Y.owner;
        uint8_t *base = (uint8_t *)c->bkv;
        if (Y.global) {
            c->bring[l] = gring;
            c->bk[l] = (float *)(base + (size_t)max_seqs * 12 * sl + (size_t)(o / 5) * max_seqs * gl);
        } else {
            c->bring[l] = G4_SLIDING_RING;
            c->bk[l] = (float *)(base + (size_t)((o / 5) * 4 + o % 5) * max_seqs * sl);
        }
        c->bv[l] = c->bk[l] + (size_t)c->bring[l] * Y.hd;
    }
    // rows, split partials (one row per sequence), logits, gathered residual rows, lm_head scales
    const size_t part = (size_t)max_seqs * kSplits * G4_HEADS * (G4_HD_GLOBAL + 4) * 4;
    const size_t logits = (size_t)max_seqs * G4_VOCAB * 4;
    const size_t est = (size_t)G4_VOCAB * (G4_HIDDEN / 64) * 4;
    size_t off[8], tot = 0;
    const size_t sz[8] = {(size_t)G4_BATCH * 4, (size_t)G4_BATCH * 4, (size_t)max_seqs * 4, part, logits,
                          (size_t)max_seqs * G4_HIDDEN * 4, est, 0};
    for (int i = 0; i < 7; i++) {
        off[i] = tot;
        tot += (sz[i] + 255) & ~(size_t)255;
    }
    if (cudaMalloc(&c->bbuf, tot) != cudaSuccess) {
        c->bbuf = nullptr;
        return fail(c, G4_ERR_NOMEM, "sequence buffers: %zu bytes", tot);
    }
    uint8_t *b = (uint8_t *)c->bbuf;
    c->row_seq_d = (int *)(b + off[0]);
    c->row_pos_d = (int *)(b + off[1]);
    c->bargmax = (int *)(b + off[2]);
    c->bpart = (float *)(b + off[3]);
    c->blogits = (float *)(b + off[4]);
    c->bres = (float *)(b + off[5]);
    c->embed_st = (float *)(b + off[6]);
    CK(g4_launch_scales_t(c->embed.s, G4_VOCAB, G4_HIDDEN, c->embed_st, c->st));
    CK(cudaStreamSynchronize(c->st));
    c->max_seqs = max_seqs;
    return G4_OK;
}

int g4_forward_batch(g4_ctx *c, int n, const int *seq_ids, const int *tokens, const int *offsets,
                     const int *start_pos) {
    if (!c) return G4_ERR_INVALID;
    if (!c->max_seqs) return fail(c, G4_ERR_STATE, "forward_batch: call g4_seq_alloc first");
    if (c->strict) return fail(c, G4_ERR_STATE, "forward_batch: not available in strict mode");
    if (n < 1 || n > c->max_seqs || !seq_ids || !tokens || !offsets || !start_pos || offsets[0] != 0)
        return fail(c, G4_ERR_INVALID, "forward_batch: bad arguments (n %d)", n);
    const int T = offsets[n];
    if (T < 1 || T > G4_BATCH) return fail(c, G4_ERR_INVALID, "forward_batch: %d rows (1..%d)", T, G4_BATCH);
    std::vector<int> rs(T), rp(T);
    for (int i = 0; i < n; i++) {
        const int cnt = offsets[i + 1] - offsets[i];
        if (cnt < 1 || (n > 1 && cnt != 1))
            return fail(c, G4_ERR_INVALID, "forward_batch: sequence %d has %d tokens (several sequences: 1 each)", i,
                        cnt);
        if (seq_ids[i] < 0 || seq_ids[i] >= c->max_seqs)
            return fail(c, G4_ERR_INVALID, "forward_batch: sequence id %d out of range", seq_ids[i]);
        for (int j = 0; j < i; j++)
            if (seq_ids[j] == seq_ids[i]) return fail(c, G4_ERR_INVALID, "forward_batch: sequence %d twice", seq_ids[i]);
        const long long last = (long long)start_pos[i] + cnt - 1;
        if (start_pos[i] < 0 || last >= c->bring[4] || last >= G4_MAX_CONTEXT)
            return fail(c, G4_ERR_INVALID, "forward_batch: positions %d..%lld beyond the sequence capacity %d",
                        start_pos[i], last, c->bring[4]);
        for (int k = 0; k < cnt; k++) {
            const int tk = tokens[offsets[i] + k];
            if (tk < 0 || tk >= G4_VOCAB) return fail(c, G4_ERR_INVALID, "forward_batch: token %d out of range", tk);
            rs[offsets[i] + k] = seq_ids[i];
            rp[offsets[i] + k] = start_pos[i] + k;
        }
    }
    cudaSetDevice(c->device);
    if (int rc = flush_pending(c)) return rc;
    CK(cudaMemcpyAsync(c->tokens_d, tokens, (size_t)T * 4, cudaMemcpyHostToDevice, c->st));
    CK(cudaMemcpyAsync(c->row_seq_d, rs.data(), (size_t)T * 4, cudaMemcpyHostToDevice, c->st));
    CK(cudaMemcpyAsync(c->row_pos_d, rp.data(), (size_t)T * 4, cudaMemcpyHostToDevice, c->st));
    // one sequence with several tokens: the prefill attention over its ring; else one row per sequence
    // (single-token rows use the same split attention as single-sequence decode)
    BatchPlan bp{T == n, seq_ids[0]};
    if (bp.rows && c->use_graph) {
        // rows read their sequence and position from the device arrays above, so
        // one graph per row count replays any step of that many sequences
        if ((int)c->g_rows.size() <= T) {
            c->g_rows.resize(T + 1, nullptr);
            c->rows_warm.resize(T + 1, 0);
        }
        if (!c->g_rows[T] && c->rows_warm[T] >= kRowGraphAfter) {
            cudaGraph_t g = nullptr;
            CK(cudaStreamBeginCapture(c->st, cudaStreamCaptureModeThreadLocal));
            cudaError_t e = enqueue_prefill(c, T, start_pos[0], &bp);
            cudaError_t e2 = cudaStreamEndCapture(c->st, &g);
            if (e || e2) {
                if (g) cudaGraphDestroy(g);
                return fail(c, G4_ERR_CUDA, "forward_batch capture: %s", cudaGetErrorString(e ? e : e2));
            }
            e = cudaGraphInstantiate(&c->g_rows[T], g, 0);
            cudaGraphDestroy(g);
            if (e) {
                c->g_rows[T] = nullptr;
                return fail(c, G4_ERR_CUDA, "forward_batch graph: %s", cudaGetErrorString(e));
            }
            c->rows_cur = c->cur;
        }
        if (c->g_rows[T]) {
            CK(cudaGraphLaunch(c->g_rows[T], c->st));
            c->cur = c->rows_cur;
        } else {
            cudaError_t e = enqueue_prefill(c, T, start_pos[0], &bp);
            if (e) return fail(c, G4_ERR_CUDA, "forward_batch launch: %s", cudaGetErrorString(e));
            c->rows_warm[T]++;
        }
    } else {
        // layer 4 is the first global layer (gemma4.c:417-419): its batch ring
        const int rc = ensure_tc_ws(c, T, start_pos[0], c->bring[4]);
        if (rc) return rc;
        cudaError_t e = enqueue_prefill(c, T, start_pos[0], &bp);
        if (e) return fail(c, G4_ERR_CUDA, "forward_batch launch: %s", cudaGetErrorString(e));
    }
    c->last_T = 0;   // the single-sequence rows are gone
    c->blast.resize(n);
    for (int i = 0; i < n; i++) c->blast[i] = offsets[i + 1] - 1;
    // the host vectors above are pageable: the copies completed before the calls returned
    return G4_OK;
}

// Logits of rows [row0, row0 + n) of the last forward into out[n][262144]
// (the reference's --dump-logits loop, gemma4.c:567-570): chunks of kDumpRows
// rows, each the final norm + one tensor-core lm_head GEMM + soft-cap on the
// library stream, copied to the host on a second stream while the next chunk
// computes. Bit-identical to g4_logits row by row.
constexpr int kDumpRows = 64;
int g4_logits_rows(g4_ctx *c, size_t row0, size_t n, float *out) {
    if (!c || !out || n == 0) return G4_ERR_INVALID;
    if (c->last_T == 0 || row0 + n > (size_t)c->last_T)
        return fail(c, G4_ERR_STATE, "logits_rows: rows %zu..%zu not computed by the last forward (%d rows)", row0,
                    row0 + n, c->last_T);
    cudaSetDevice(c->device);
    int rc = flush_pending(c);
    if (rc) return rc;
    if (!c->dump_buf) {
        const size_t lb = (size_t)kDumpRows * G4_VOCAB * 4, sb = (size_t)G4_VOCAB * (G4_HIDDEN / 64) * 4;
        CK(cudaMalloc(&c->dump_buf, 2 * lb + sb + kDumpRows * 4));
        uint8_t *b = (uint8_t *)c->dump_buf;
        c->dump_log[0] = (float *)b;
        c->dump_log[1] = (float *)(b + lb);
        c->dump_st_scales = (float *)(b + 2 * lb);
        c->dump_arg = (int *)(b + 2 * lb + sb);
        CK(g4_launch_scales_t(c->embed.s, G4_VOCAB, G4_HIDDEN, c->dump_st_scales, c->st));
        CK(cudaStreamCreateWithFlags(&c->dump_st, cudaStreamNonBlocking));
        for (int i = 0; i < 2; i++) {
            CK(cudaEventCreateWithFlags(&c->dump_done[i], cudaEventDisableTiming));
            CK(cudaEventCreateWithFlags(&c->dump_copied[i], cudaEventDisableTiming));
            CK(cudaEventRecord(c->dump_copied[i], c->dump_st));
        }
    }
    DMat em = c->embed;
    em.sT = c->dump_st_scales;
    for (size_t r = 0, ch = 0; r < n; r += kDumpRows, ch++) {
        const int m = (int)(n - r < (size_t)kDumpRows ? n - r : kDumpRows), b = (int)(ch & 1);
        Seq q{c, c->use_pdl};
        CK(cudaStreamWaitEvent(c->st, c->dump_copied[b], 0));   // this buffer's previous copy is done
        q.ck(g4_launch_rows_norm(0, c->res[c->cur] + (row0 + r) * G4_HIDDEN, m, nullptr, nullptr, nullptr, nullptr,
                                 c->final_norm, G4_RMS_EPS, c->xq, c->xs, c->st, q.pdl, nullptr, 0, c->xsT));
        gemm(q, em, m, EPI_STORE, c->dump_log[b], G4_VOCAB, nullptr, 0);
        q.ck(g4_launch_softcap_argmax(c->dump_log[b], m, G4_VOCAB, c->dump_arg, c->st));
        if (q.e) return fail(c, G4_ERR_CUDA, "logits_rows launch: %s", cudaGetErrorString(q.e));
        CK(cudaEventRecord(c->dump_done[b], c->st));
        CK(cudaStreamWaitEvent(c->dump_st, c->dump_done[b], 0));
        CK(cudaMemcpyAsync(out + r * G4_VOCAB, c->dump_log[b], (size_t)m * G4_VOCAB * 4,
                           cudaMemcpyDeviceToHost, c->dump_st));
        CK(cudaEventRecord(c->dump_copied[b], c->dump_st));
    }
    CK(cudaStreamSynchronize(c->dump_st));
    return check_device_error(c);
}

int g4_logits_batch(g4_ctx *c, int *argmax, float *logits) {
    if (!c) return G4_ERR_INVALID;
    if (c->blast.empty()) return fail(c, G4_ERR_STATE, "logits_batch: no batch forward to read");
    cudaSetDevice(c->device);
    const int n = (int)c->blast.size();
    for (int i = 0; i < n; i++)
        CK(cudaMemcpyAsync(c->bres + (size_t)i * G4_HIDDEN, c->res[c->cur] + (size_t)c->blast[i] * G4_HIDDEN,
                           G4_HIDDEN * 4, cudaMemcpyDeviceToDevice, c->st));
    Seq q{c, c->use_pdl};
    q.ck(g4_launch_rows_norm(0, c->bres, n, nullptr, nullptr, nullptr, nullptr, c->final_norm, G4_RMS_EPS, c->xq,
                             c->xs, c->st, q.pdl, nullptr, 0, c->xsT));
    DMat em = c->embed;
    em.sT = c->embed_st;
    gemm(q, em, n, EPI_STORE, c->blogits, G4_VOCAB, nullptr, 0);
    q.ck(g4_launch_softcap_argmax(c->blogits, n, G4_VOCAB, c->bargmax, c->st));
    if (q.e) return fail(c, G4_ERR_CUDA, "logits_batch launch: %s", cudaGetErrorString(q.e));
    if (argmax) CK(cudaMemcpyAsync(argmax, c->bargmax, (size_t)n * 4, cudaMemcpyDeviceToHost, c->st));
    if (logits) CK(cudaMemcpyAsync(logits, c->blogits, (size_t)n * G4_VOCAB * 4, cudaMemcpyDeviceToHost, c->st));
    return check_device_error(c);
}

}  // extern "C"
