/*
 * g4cuda.h — C ABI of libg4cuda.so, the B200 (sm_100a) implementation of
 * gemma4.c's transformer forward path.
 *
 * The library replaces the two hot-path functions a gemma4.c host calls:
 *
 *   void   forward(Model*, InferenceState*, const int *tokens, size_t n, int start_pos)
 *            (gemma4.c:463)  ->  g4_forward
 *   float *logits(Model*, InferenceState*, size_t token_row)
 *            (gemma4.c:512)  ->  g4_logits (+ g4_topk for the sampling loop,
 *                                gemma4.c:536-561)
 *
 * The model stays in gemma4.c's .bin layout (exporter.py); g4_open takes the
 * mapped file (records holding file offsets, or already fixed-up pointers into
 * the same mapping, gemma4.c:681-685) and builds the device copy and the
 * device-resident FP32 KV caches, which replace InferenceState.
 *
 * Conventions: plain C types only; every function returns G4_OK (0) or a
 * negative G4_ERR_* code and never aborts. Calls on one context must come from
 * one host thread at a time. g4_forward is asynchronous (stream ordered);
 * device-side failures surface at the next synchronising call (g4_logits,
 * g4_topk, g4_sync, reads).
 */
#ifndef G4CUDA_H
#define G4CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define G4_OK 0
#define G4_ERR_INVALID (-1)  /* bad argument (null pointer, range, token id) */
#define G4_ERR_FORMAT (-2)   /* model image rejected (magic, record, shape) */
#define G4_ERR_CUDA (-3)     /* CUDA runtime error */
#define G4_ERR_NOMEM (-4)    /* device or pinned allocation failed */
#define G4_ERR_DEVICE (-5)   /* a kernel reported an error (wait timeout, bad token) */
#define G4_ERR_STATE (-6)    /* call out of sequence (e.g. logits of a row not computed) */

typedef struct g4_ctx g4_ctx;

/* Upload a model image (the whole .bin mapping, `bytes` long) to `device`.
 * Replaces main's mmap + pointer fix-up + calloc(InferenceState)
 * (gemma4.c:673-686). The image is only read during the call. */
int g4_open(const void *image, uint64_t bytes, int device, g4_ctx **out);
/* Same, reading the .bin at `path` straight to the device: 64 MB pieces through
 * two page-locked buffers, each copied while the next is read, then the
 * one-time repacking from that device image (it needs the file's size in free
 * device memory during the call). */
int g4_open_file(const char *path, int device, g4_ctx **out);
int g4_close(g4_ctx *ctx);
/* Message for the last failed g4_open / g4_open_file in this process. */
const char *g4_open_error(void);

/* forward (gemma4.c:463-509): run `count` tokens (1..512, the reference's
 * BATCH_SIZE) at positions start_pos..start_pos+count-1, updating the KV caches
 * and the per-row residual stream. Position semantics are the reference's:
 * chunks must be called in order and start_pos + count <= 131072. */
int g4_forward(g4_ctx *ctx, const int *tokens, size_t count, int start_pos);

/* logits (gemma4.c:512-522) of residual row `row` (< count of the last
 * forward): final RMSNorm, int8 lm_head over the tied embedding, 30*tanh(x/30).
 * `out` (262144 floats, may be NULL) receives the logits and `argmax` (may be
 * NULL) the greedy token (first maximum, gemma4.c:537-541). Synchronises,
 * except when both are NULL: then the call only enqueues (the reference's
 * benchmark computes logits it never reads, gemma4.c:641). */
int g4_logits(g4_ctx *ctx, size_t row, float *out, int *argmax);

/* The logits of rows [row0, row0 + n) of the last forward into out[n][262144]
 * (the reference's --dump-logits loop over logits(), gemma4.c:567-570): the
 * lm_head of 64 rows at a time on the tensor cores, each chunk copied to the
 * host while the next computes (page-locked `out` copies fastest). Identical
 * bits to g4_logits row by row. Synchronises. */
int g4_logits_rows(g4_ctx *ctx, size_t row0, size_t n, float *out);

/* Top-k (k <= 64) of the logits of `row`, descending, ties to the lower id:
 * the candidate list of gemma4.c:544-551. Synchronises. */
int g4_topk(g4_ctx *ctx, size_t row, int k, float *values, int *ids);

/* sample (gemma4.c:536-561) on the device: temperature > 0 draws from the
 * smallest prefix of the top 64 holding 95 % of their probability mass with the
 * reference's xorshift generator (random_uniform, gemma4.c:527-534), whose state
 * lives in the context (42 after g4_open, like the reference); temperature <= 0
 * is the greedy argmax. Only the token (4 bytes) is read back. */
int g4_sample(g4_ctx *ctx, size_t row, float temperature, int *token);
/* Set the sampling generator's state (the reference's rng_state). */
int g4_set_seed(g4_ctx *ctx, uint64_t seed);

/* Top-k (k <= 64) of n <= 262144 floats already in device memory, written to
 * caller-provided device buffers `values`/`ids` on `stream` (a cudaStream_t;
 * NULL = the default stream): the same selection as g4_topk (descending,
 * ties to the lower index), but this entry point allocates nothing. It is for
 * hosts that cannot call cudaMalloc on their decode path — frameworks that
 * own every byte of device memory through their own pool, hosts that capture
 * the decode loop into CUDA graphs (allocation is not allowed while a stream
 * is being captured), and latency-critical loops that must not block in the
 * allocator. It has no counterpart in the reference (which samples on the
 * CPU).
 * Its one piece of scratch is a fixed 32 KB array in the library's device
 * image, which every GPU that loads the library keeps until exit; n above
 * 262144 or k above 64 is rejected with G4_ERR_INVALID. The first call on a
 * device looks up that array's device address, so make it before capturing a
 * stream. The looked-up address is kept for the life of the process: after
 * cudaDeviceReset on a device, restart the process before calling this again.
 * All calls share the array: calls whose kernels overlap on the GPU
 * (different streams, no ordering between them) race on it. Asynchronous: no
 * synchronisation, results valid once the stream reaches them; a launch error
 * of its own two kernels is returned as G4_ERR_CUDA. */
int g4_topk_noalloc(const float *logits, int n, int k, float *values, int *ids, void *stream);

/* Wait for queued work; returns any device-side error. */
int g4_sync(g4_ctx *ctx);

/* Message for the last error on this context (never NULL). */
const char *g4_last_error(g4_ctx *ctx);
const char *g4_strerror(int code);

/* Options (g4_set_option): */
#define G4_OPT_GRAPHS 1      /* capture single-token decode in a CUDA graph (default 1) */
#define G4_OPT_PDL 2         /* programmatic dependent launch between kernels (default 1) */
#define G4_OPT_GEMM_PATH 3   /* prefill GEMM: 0 auto (small-batch mma for T <= 64 rows when
                                N < 8192 or T <= 8; else tcgen05, with transposed roles
                                up to 64 rows), 1 SIMT dp4a, 2 tcgen05, 3 small-batch mma
                                wherever it applies (T <= 64) */
#define G4_OPT_LAYERS 4      /* run only the first N layers (testing aid; default 35) */
/* Reference-order arithmetic (default 0): RMSNorm sums of squares, attention
 * scores, softmax and value sums are evaluated in gemma4.c's sequential order
 * with the host C library's expf, so the whole forward reproduces the
 * reference bit for bit (logits up to tanhf). Much slower; for verification. */
#define G4_OPT_STRICT 5
/* Single-token decode as ONE persistent cooperative kernel per step (default
 * 1): g4_forward with one token is deferred; the next g4_logits launches the
 * forward and the lm_head together, any other call launches the forward alone
 * first. Same bits as the multi-kernel path. Not used in strict mode. */
#define G4_OPT_PERSISTENT 6
/* Key splits per row of a multi-sequence decode step (g4_forward_batch):
 * 0 (default) = about four CTAs per SM over the batch, at least 16 per row;
 * 148 = the partition
 * single-sequence decode uses, which makes every batch row bit-identical to
 * decoding that sequence alone (other values change only the attention's
 * floating-point summation order). */
#define G4_OPT_BATCH_SPLITS 7
/* Prefill attention of a chunk (g4_forward / one-sequence g4_forward_batch):
 * 0 (default) auto = tensor cores (tcgen05 GEMMs for Q K^T and P V on fp16
 * hi/lo operand pairs, fp32 accumulation) where the chunk's work (the keys its
 * tokens see, summed) is at least 64k on a global layer or 128k on a sliding
 * one, CUDA cores below; 1 CUDA cores everywhere; 2 tensor cores everywhere.
 * The paths differ in floating-point order only (outputs agree to fp32
 * rounding: a relative error near 2^-21 per product). Not used in strict
 * mode. The tensor-core path's device workspace is allocated at the first
 * chunk that takes it: for the whole context range (about 2.7 GB for global
 * layers at 131072 positions, plus ~50 MB for sliding ones) when the device
 * has four times that free, else twice the chunk's need, grown on demand;
 * g4_close frees it. */
#define G4_OPT_ATTN_PATH 8
int g4_set_option(g4_ctx *ctx, int option, int value);

/* ---- multi-sequence serving (ragged batches of independent sequences) ----
 * No reference counterpart in gemma4.c (one sequence per process); the
 * single-sequence calls above are unaffected and keep their own KV cache.
 *
 * g4_seq_alloc: device KV rings for `max_seqs` sequences (<= G4_MAX_SEQS)
 * holding positions 0 .. max_context - 1 each (global rings rounded up to a
 * power of two >= 1024; sliding rings 1024). Re-allocating drops all sequences.
 *
 * g4_forward_batch: `n` sequences; sequence seq_ids[i] (distinct, < max_seqs)
 * consumes tokens[offsets[i] .. offsets[i+1]) at positions start_pos[i] ...,
 * offsets[0] == 0 and offsets[n] <= 512 rows in total. Either one sequence
 * with up to 512 tokens (a prefill chunk, in order as for g4_forward) or
 * several sequences with exactly one token each (a decode step). With
 * G4_OPT_BATCH_SPLITS 148 a batch row computes the same bits as the same token
 * through g4_forward on a context holding only that sequence. Not available in
 * strict mode.
 *
 * g4_logits_batch: for each sequence of the last g4_forward_batch, the
 * soft-capped logits of its last token (logits: [n][262144] or NULL) and the
 * greedy argmax (argmax: [n] or NULL). */
#define G4_MAX_SEQS 256
int g4_seq_alloc(g4_ctx *ctx, int max_seqs, int max_context);
int g4_forward_batch(g4_ctx *ctx, int n, const int *seq_ids, const int *tokens, const int *offsets,
                     const int *start_pos);
int g4_logits_batch(g4_ctx *ctx, int *argmax, float *logits);

/* ---- introspection (tests, benchmarks) ---- */
int g4_read_residual(g4_ctx *ctx, size_t rows, float *out);          /* [rows][1536] */
/* `nslots` ring slots of the K (which=0) or V (which=1) cache `layer` reads. */
int g4_read_cache(g4_ctx *ctx, int layer, int which, int slot0, int nslots, float *out);
/* The per-layer inputs of the last forward's rows ([rows][35][256]: the
 * token-conditioned input each layer's gate multiplies, gemma4.c:468-477). */
int g4_read_ple(g4_ctx *ctx, size_t rows, float *out);
/* Ring slots of sequence `seq`'s K (which=0) / V (which=1) cache that `layer`
 * reads (multi-sequence serving, after g4_seq_alloc). */
int g4_read_seq_cache(g4_ctx *ctx, int seq, int layer, int which, int slot0, int nslots, float *out);
/* The context's cudaStream_t. Copies, events and ordinary launches a host
 * adds to it are ordered after the library's work as usual. The library's
 * kernels let programmatic dependents start early, so a kernel launched here
 * with cudaLaunchAttributeProgrammaticStreamSerialization must call
 * cudaGridDependencySynchronize() (griddepcontrol.wait) before it touches
 * anything the library wrote. */
void *g4_stream(g4_ctx *ctx);
/* Open (1) / close (0) the profiler capture range (ncu --profile-from-start off). */
int g4_profiler_range(int on);
int g4_device_bytes(g4_ctx *ctx, uint64_t *weights, uint64_t *total);
/* CUDA-event timing on the context's stream: record slot (0..15), then the
 * elapsed milliseconds between two recorded slots (waits for the later one). */
int g4_mark(g4_ctx *ctx, int slot);
int g4_elapsed(g4_ctx *ctx, int slot_a, int slot_b, float *ms);
/* One single-token decode step at `pos` plus its logits, launched eagerly with
 * an event after every kernel: per-class device time, algorithmic bytes and
 * launch counts. Class 0: int8 weight GEMVs; 1: attention (+ combine); 2: rest.
 * Advances the KV cache like g4_forward. */
int g4_profile_decode(g4_ctx *ctx, int token, int pos, float ms[3], double bytes[3], int launches[3]);
/* One single-token step at `pos` (forward + logits) as the persistent kernel,
 * with a device timeline: for op i (in launch order) types[i] is 0 int8 GEMV,
 * 1 split attention, 2 split combine, 3 per-layer-input prep, 4 last residual
 * update; t_ns[6i..6i+5] are, in nanoseconds from the latest CTA start, when
 * the latest CTA finished the op's prologue (GEMV only, else -1), the op, and
 * the grid barrier after it; then the longest time one consumer warp waited
 * for the op's weights to land (a duration); then when the latest producer
 * issued the op's first and its last weight stage (GEMV only, else -1). Advances the KV cache like g4_forward. *nops gets the
 * op count; at most `cap` ops are written. G4_ERR_STATE if persistent decode
 * is off (G4_OPT_PERSISTENT 0 or strict mode). With G4_OPT_PERSISTENT on,
 * g4_profile_decode reports this timeline by class (ops, not kernels). */
int g4_trace_decode(g4_ctx *ctx, int token, int pos, int cap, int *types, double *t_ns, int *nops);
/* Kernels one single-token decode step (forward + logits) launches. */
int g4_launches_per_token(g4_ctx *ctx, int *n);
/* Failure-path test aid (no reference counterpart): the next persistent
 * single-token step's weight producers issue no copies, so every consumer's
 * bounded wait (2 s) runs out; the step then reports G4_ERR_DEVICE at the next
 * synchronising call, the context resets its error word and barrier counters,
 * and later steps run normally. G4_ERR_STATE when persistent decode is off. */
int g4_test_starve_next_step(g4_ctx *ctx);

/* ---- synthetic model images (benchmarks and parity tests) ----
 * A seeded random-init Gemma 4 E2B in the exact .bin layout gemma4.c reads. */
uint64_t g4synth_image_bytes(void);
int g4synth_fill(uint8_t *image, uint64_t bytes, uint64_t seed, unsigned flags);
int g4synth_write_file(const char *path, uint64_t seed, unsigned flags);

/* ---- single-kernel entry points (host buffers in and out; each call
 * allocates and frees its own device buffers on the current device) ---- */
/* quantize (gemma4.c:265-279): x[rows][width] -> q[rows][width], s[rows][width/64] */
int g4k_quantize(const float *x, int rows, int width, int8_t *q, float *s);
/* matmul_int8 (gemma4.c:257-262) on a packed matrix (exporter.py:304-316 layout):
 * out[T][N]; `dots` (may be NULL) receives the int32 of every (t, n, 64-group)
 * as [T][N][K/64]. path: 0 auto, 1 decode GEMV (T <= 4), 2 SIMT GEMM,
 * 3 tcgen05 GEMM, 4 small-batch mma GEMM (T <= 64); paths 3 and 4 do not
 * return dots. T <= 512 (the reference's chunk), except path 3: T <= 16384. */
int g4k_linear(const int8_t *w_packed, const uint16_t *s_packed, int N, int K, const int8_t *xq, const float *xs,
               int T, int path, float *out, int32_t *dots);
/* Average duration of the decode GEMV on an N x K int8 matrix over `iters`
 * launches (weights cycled through enough copies to exceed L2), and the
 * algorithmic bytes (int8 weights + FP16 scales) one launch streams. */
int g4_bench_gemv(int N, int K, int T, int iters, int pdl, float *ms_per_launch, double *bytes_per_launch);
/* Prefill GEMM timing (path 2 SIMT dp4a with T <= 512, 3 tcgen05 with
 * T <= 16384, 4 small-batch mma with T <= 64) on T x N x K: average
 * launch duration and int8 operations (2 T N K) per launch. */
int g4_bench_gemm(int N, int K, int T, int path, int iters, float *ms_per_launch, double *ops_per_launch);
/* Launch geometry the small-batch GEMM (T <= 64 token rows) would use for an
 * N x K matrix (no reference counterpart; host-side planning, no kernel runs):
 * output rows per unit / 16 (wm), 8-token tiles per warp (nt), ring stages,
 * threads per CTA and dynamic shared memory. G4_ERR_INVALID when the shape is
 * not supported or does not fit. */
int g4_skinny_plan(int N, int K, int T, int *wm, int *nt, int *stages, int *threads, int *smem_bytes);
/* Measured int8 tensor-core peak of this GPU (no reference counterpart: the
 * denominator of the prefill GEMM's roofline): `iters` back-to-back tcgen05
 * kind::i8 MMAs (M 128, N 256, K 32) on every SM; duration of one launch and
 * its int8 operations. */
int g4_bench_mma_i8(int iters, float *ms_per_launch, double *ops_per_launch);
/* One attention sub-layer (attention, gemma4.c:411-461) over an FP32 KV ring:
 * hd 256 = sliding layer (window 512, 128 rope pairs), hd 512 = global layer
 * (no window, 64 pairs). qkv[T][10*hd] holds each token's raw q (8 heads) | k | v;
 * q_norm / k_norm [hd] (NULL = weight 1); rope_cos / rope_sin
 * [start_pos + T][pairs]; kring / vring [ring][hd] (ring a power of two >= 1024)
 * are read and receive the chunk's keys and values; out[T][8*hd].
 * mode 0: prefill fast path (q/k/v post-processing + tiled kernel); 1: strict
 * (the reference's floating-point order); 2: single-token decode (split-KV
 * over `splits` CTAs + combine, T == 1); 3: batched-row decode path (one row
 * per token at start_pos + t, `splits` key splits); 4: prefill on the tensor
 * cores (tcgen05 GEMMs on fp16 hi/lo operand pairs for Q K^T and P V). iters > 0: the attention
 * kernels (without post-processing) are then repeated `iters` times and the
 * average duration per call is written to ms_per_call. xq / xs (mode 0 or 4, both
 * or neither): the output rows as the kernel quantises them for o_proj
 * (quantize, gemma4.c:265-279): xq[T][8*hd], xs[T][8*hd/64]. */
int g4k_attention(int hd, int ring, int T, int start_pos, int mode, int splits, const float *qkv,
                  const float *q_norm, const float *k_norm, const float *rope_cos, const float *rope_sin,
                  float *kring, float *vring, float *out, int8_t *xq, float *xs, int iters, float *ms_per_call);
/* The tensor-core prefill attention's schedule for a chunk of T tokens at
 * start_pos on a GPU with `sms` SMs, checked on the host (no GPU needed): S
 * tiles inside the workspace, every P V stage covered exactly once by the
 * per-CTA runs, partial slots distinct, the combine's CTA ranges exact.
 * Returns 0 (or the number of the first failed check); outputs the S units,
 * the P V stages, the P V CTAs and the workspace bytes. */
int g4k_attn_tc_plan(int hd, int T, int start_pos, int sms, int *units_s, int *stages_o, int *ctas_o,
                     unsigned long long *ws_bytes);
/* sample (gemma4.c:536-561) of one logits row[n] on the device (top-64 and the
 * draw); *state: the xorshift state before the call, the state after it on return */
int g4k_sample(const float *logits, int n, float temperature, unsigned long long *state, int *token);
/* rmsnorm (gemma4.c:360-373) of hidden-width rows followed by quantize */
int g4k_rmsnorm_quant(const float *x, int rows, const float *w, float eps, float *y, int8_t *q, float *s);

#ifdef __cplusplus
}
#endif
#endif
