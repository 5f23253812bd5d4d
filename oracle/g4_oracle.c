/*
 * g4_oracle.c — CPU restatement of gemma4.c's transformer forward path.
 *
 * TEST INFRASTRUCTURE, NOT PRODUCT: this file is the parity checker for the
 * CUDA library. It is built into oracle/liboracle.so and only the tests, the
 * smoke check and the benchmark's CPU-baseline leg load it.
 *
 * Every function restates the arithmetic of the reference function it cites
 * (file:line in qmog-ai/gemma4.c) in portable C, with the same rounding steps:
 *   - the file is compiled with -ffp-contract=off, as the reference's
 *     -std=c11 build is, so a*b+c rounds twice unless fmaf() is written;
 *   - fmaf() appears exactly where the reference uses an FMA intrinsic (the
 *     per-group dequant chain, attention scores, the weighted value sum).
 * With the same libm (expf, tanhf, sqrtf) the whole forward is then bit-for-bit
 * the reference's: tests/test_oracle_golden.py checks it against golden vectors
 * that the reference itself produced (tests/golden/make_golden.py).
 *
 * OpenMP parallelises over independent outputs only, so results do not depend
 * on the thread count.
 */
#include "g4_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define NL 35
#define HID 1536
#define VOCAB 262144
#define MAXCTX 131072
#define WINDOW 512
#define CHUNK 512
#define RING 1024
#define PLEW 256
#define NREC 671

int or_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

float or_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t mant = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0x1Fu) bits = sign | 0x7F800000u | (mant << 13);
    else if (exp != 0) bits = sign | ((exp + 112u) << 23) | (mant << 13);
    else if (mant == 0) bits = sign;
    else { /* subnormal: value = mant * 2^-24 */
        int e = -1;
        do { mant <<= 1; e++; } while (!(mant & 0x400u));
        bits = sign | ((uint32_t)(112 - e) << 23) | ((mant & 0x3FFu) << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* gemma4.c:265-279 quantize: per 64-value group, scale = max|x| / 127,
 * q = rintf(x * (1/scale)), zero groups give scale 0 and q = 0. */
void or_quantize(int8_t *q, float *scales, const float *x, size_t rows, size_t width) {
    size_t groups = rows * (width / 64);
    #pragma omp parallel for schedule(static)
    for (size_t gi = 0; gi < groups; gi++) {
        const float *src = x + gi * 64;
        float amax = 0.0f;
        for (int j = 0; j < 64; j++) {
            float a = fabsf(src[j]);
            if (a > amax) amax = a;
        }
        float s = amax / 127.0f;
        float inv = s > 0.0f ? 1.0f / s : 0.0f;
        for (int j = 0; j < 64; j++) q[gi * 64 + j] = (int8_t)rintf(src[j] * inv);
        scales[gi] = s;
    }
}

/* Packed weight byte of (row n, column k): exporter.py:304-316 lays a matrix
 * out as [n/16][k/64][(k%64)/4][n%16][k%4]. */
static inline int8_t packed_at(const int8_t *w, int K, int n, int k) {
    size_t blk = (size_t)(n / 16), g = (size_t)(k / 64);
    size_t off = ((blk * (size_t)(K / 64) + g) * 16 + (size_t)((k % 64) / 4)) * 64 + (size_t)(n % 16) * 4 + (size_t)(k % 4);
    return w[off];
}

/* FP16 scale of (row n, group g): exporter.py:310 lays scales as [n/16][g][n%16]. */
static inline float packed_scale(const uint16_t *s, int K, int n, int g) {
    return or_f16_to_f32(s[((size_t)(n / 16) * (size_t)(K / 64) + (size_t)g) * 16 + (size_t)(n % 16)]);
}

/* Exact int32 dot of one 64-group (gemma4.c:206-215 VNNI, 237-245 AVX2: both
 * produce the exact integer sum since |q| <= 127 never saturates). */
static inline int32_t group_dot(const int8_t *x64, const int8_t *w, int K, int n, int g) {
    /* the 64 bytes of (n, g) sit at 16 chunks of 4, 64 bytes apart */
    const int8_t *base = w + (((size_t)(n / 16) * (size_t)(K / 64) + (size_t)g) * 16) * 64 + (size_t)(n % 16) * 4;
    int32_t acc = 0;
    for (int c = 0; c < 16; c++)
        for (int b = 0; b < 4; b++) acc += (int32_t)x64[c * 4 + b] * (int32_t)base[c * 64 + b];
    return acc;
}

void or_linear_dots(int32_t *dots, const int8_t *xq, size_t tokens, const int8_t *w, int N, int K) {
    int G = K / 64;
    #pragma omp parallel for schedule(static)
    for (int n = 0; n < N; n++)
        for (size_t t = 0; t < tokens; t++)
            for (int g = 0; g < G; g++)
                dots[((size_t)t * N + n) * G + g] = group_dot(xq + t * (size_t)K + (size_t)g * 64, w, K, n, g);
}

/* gemma4.c:192-262 matmul_int8: for each output, acc = 0 then for g ascending
 * acc = fma((float)dot_g, w_scale_g * x_scale_g, acc) — the product of the two
 * scales is rounded first (gemma4.c:218 / :248). */
void or_linear(float *out, const int8_t *xq, const float *xs, size_t tokens,
               const int8_t *w, const uint16_t *s, int N, int K) {
    int G = K / 64;
    #pragma omp parallel for schedule(static)
    for (int n = 0; n < N; n++) {
        for (size_t t = 0; t < tokens; t++) {
            float acc = 0.0f;
            for (int g = 0; g < G; g++) {
                int32_t d = group_dot(xq + t * (size_t)K + (size_t)g * 64, w, K, n, g);
                float scale = packed_scale(s, K, n, g) * xs[t * (size_t)G + (size_t)g];
                acc = fmaf((float)d, scale, acc);
            }
            out[t * (size_t)N + (size_t)n] = acc;
        }
    }
}

/* gemma4.c:360-373 rmsnorm: sequential sum of squares, then
 * w * ((1/sqrtf(ss/n + eps)) * x); a NULL weight means 1. In-place is allowed. */
void or_rmsnorm(float *out, const float *in, const float *weight, int width, float eps, size_t rows) {
    #pragma omp parallel for schedule(static)
    for (size_t r = 0; r < rows; r++) {
        const float *x = in + r * (size_t)width;
        float *y = out + r * (size_t)width;
        float ss = 0.0f;
        for (int i = 0; i < width; i++) ss += x[i] * x[i];
        float inv = 1.0f / sqrtf(ss / (float)width + eps);
        for (int i = 0; i < width; i++) y[i] = (weight ? weight[i] : 1.0f) * (inv * x[i]);
    }
}

/* gemma4.c:375-378 add_and_scale */
void or_add_scale(float *out, const float *addend, size_t count, float scale) {
    #pragma omp parallel for schedule(static)
    for (size_t i = 0; i < count; i++) out[i] = (out[i] + addend[i]) * scale;
}

/* gemma4.c:381-398 apply_rope: rotates (j, j + head_dim/2) for j < pairs with
 * the table row of position start_pos + token. */
void or_rope(float *v, const float *cos_table, const float *sin_table, int pairs,
             int heads, int head_dim, int start_pos, size_t tokens) {
    #pragma omp parallel for schedule(static)
    for (size_t t = 0; t < tokens; t++) {
        const float *c = cos_table + ((size_t)start_pos + t) * (size_t)pairs;
        const float *sn = sin_table + ((size_t)start_pos + t) * (size_t)pairs;
        for (int h = 0; h < heads; h++) {
            float *x = v + (t * (size_t)heads + (size_t)h) * (size_t)head_dim;
            int half = head_dim / 2;
            for (int j = 0; j < pairs; j++) {
                float a = x[j], b = x[j + half];
                x[j] = a * c[j] - b * sn[j];
                x[j + half] = b * c[j] + a * sn[j];
            }
        }
    }
}

/* gemma4.c:310-331 geglu: table lookup with linear interpolation on
 * [lower, upper); x <= lower -> table[0], x >= upper -> x. The last interval
 * uses index size-1 with fraction 0 (the reference then reads one entry past
 * the table and multiplies it by 0, so the value is table[size-1]). */
void or_geglu(float *gate, const float *up, int rows, int width, int up_stride,
              const float *table, int table_size, int lower, int upper) {
    const float lo = (float)lower, hi = (float)upper;
    const float scale = (float)(table_size - 1) / (hi - lo);
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++)
        for (int i = 0; i < width; i++) {
            float x = gate[(size_t)r * width + i];
            if (x <= lo) x = table[0];
            else if (!(x >= hi)) {
                float pos = (x - lo) * scale;
                int idx = (int)pos;
                float frac = pos - (float)idx;
                float next = idx + 1 < table_size ? table[idx + 1] : table[idx];
                x = table[idx] + frac * (next - table[idx]);
            }
            gate[(size_t)r * width + i] = x * up[(size_t)r * up_stride + i];
        }
}

/* gemma4.c:337-358 embedding: dequantise packed rows, scale = fp16 * multiplier. */
void or_embedding(float *out, const int8_t *w, const uint16_t *s, int width,
                  const int *tokens, size_t count, float multiplier) {
    int G = width / 64;
    #pragma omp parallel for schedule(static)
    for (size_t t = 0; t < count; t++) {
        int n = tokens[t];
        for (int g = 0; g < G; g++) {
            float scale = packed_scale(s, width, n, g) * multiplier;
            for (int j = 0; j < 64; j++)
                out[t * (size_t)width + (size_t)g * 64 + j] = (float)packed_at(w, width, n, g * 64 + j) * scale;
        }
    }
}

/* gemma4.c:281-294 attention_scores for one key: 16 FMA lanes over the
 * dimension (lanes i and 8+i of each 16-wide step), then the same reduction
 * tree as the reference's horizontal sum. */
float or_score(const float *q, const float *k, int head_dim) {
    float s0[8] = {0}, s1[8] = {0};
    for (int j = 0; j < head_dim; j += 16)
        for (int i = 0; i < 8; i++) {
            s0[i] = fmaf(q[j + i], k[j + i], s0[i]);
            s1[i] = fmaf(q[j + 8 + i], k[j + 8 + i], s1[i]);
        }
    float s8[8], s4[4];
    for (int i = 0; i < 8; i++) s8[i] = s0[i] + s1[i];
    for (int i = 0; i < 4; i++) s4[i] = s8[i] + s8[i + 4];
    float a = s4[0] + s4[2], b = s4[1] + s4[3];
    return a + b;
}

/* gemma4.c:400-408 softmax: running max with rescaled sum, then normalise. */
void or_softmax(float *v, int n) {
    float mx = v[0], sum = 1.0f;
    for (int i = 1; i < n; i++) {
        if (v[i] > mx) { sum = sum * expf(mx - v[i]) + 1.0f; mx = v[i]; }
        else sum += expf(v[i] - mx);
    }
    for (int i = 0; i < n; i++) v[i] = expf(v[i] - mx) / sum;
}

/* gemma4.c:281-307 for one (head, query): scores, softmax, then each output
 * dimension is an FMA chain over the keys in order (weighted_value_sum). */
void or_attend(float *out, const float *q, const float *kc, const float *vc,
               int first, int n, int mask, int head_dim, float *scores) {
    for (int i = 0; i < n; i++) scores[i] = or_score(q, kc + (size_t)((first + i) & mask) * head_dim, head_dim);
    or_softmax(scores, n);
    for (int d = 0; d < head_dim; d++) {
        float acc = 0.0f;
        for (int i = 0; i < n; i++) acc = fmaf(scores[i], vc[(size_t)((first + i) & mask) * head_dim + d], acc);
        out[d] = acc;
    }
}

/* gemma4.c:519 */
void or_softcap(float *x, size_t n) {
    #pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; i++) x[i] = 30.0f * tanhf(x[i] / 30.0f);
}

/* gemma4.c:537-541: first strict maximum. */
int or_argmax(const float *x, int n) {
    int best = 0;
    for (int i = 1; i < n; i++) if (x[i] > x[best]) best = i;
    return best;
}

/* gemma4.c:544-551: insertion into a descending top list; equal values keep
 * the earlier (lower) id ahead. */
void or_topk(const float *x, int n, int k, float *vals, int *ids) {
    for (int i = 0; i < k; i++) { vals[i] = -INFINITY; ids[i] = -1; }
    for (int t = 0; t < n; t++) {
        if (x[t] <= vals[k - 1]) continue;
        int i = k - 1;
        while (i > 0 && x[t] > vals[i - 1]) { vals[i] = vals[i - 1]; ids[i] = ids[i - 1]; i--; }
        vals[i] = x[t];
        ids[i] = t;
    }
}

/* gemma4.c:529-534 random_uniform: xorshift64 step, top 24 bits of the
 * multiplied state over 2^24. */
float or_random_uniform(unsigned long long *state) {
    unsigned long long x = *state;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *state = x;
    return (float)((x * 0x2545F4914F6CDD1DULL) >> 40) / 16777216.0f;
}

/* gemma4.c:536-561 sample: greedy argmax at temperature <= 0; otherwise the
 * top-64 list (or_topk order), exp(score / T - top / T) with a running sum, the
 * smallest prefix holding 95 % of the sum, one uniform draw scaled by that
 * prefix mass and a walk down the prefix. */
int or_sample(const float *logits, int n, float temperature, unsigned long long *state) {
    if (temperature <= 0.0f) return or_argmax(logits, n);
    float vals[64];
    int ids[64];
    or_topk(logits, n, 64, vals, ids);
    float sum = 0.0f, mx = vals[0] / temperature;
    for (int i = 0; i < 64; i++) {
        vals[i] = expf(vals[i] / temperature - mx);
        sum += vals[i];
    }
    float mass = 0.0f;
    int count = 0;
    while (mass < 0.95f * sum) mass += vals[count++];
    float th = or_random_uniform(state) * mass;
    for (int i = 0; i < count; i++)
        if ((th -= vals[i]) <= 0.0f) return ids[i];
    return ids[count - 1];
}

/* ------------------------------------------------------------------------ */
/* Whole model                                                               */

typedef struct { uint64_t data, scales; int32_t shape[4]; } rec;
typedef struct { const void *data; const uint16_t *scales; int shape[4]; } tens;

struct or_model {
    tens t[NREC];
};

#define L_(l, s) (2 + (l) * 19 + (s))

or_model *or_model_open(const uint8_t *image, uint64_t bytes) {
    if (!image || bytes < 33429936ull + NREC * 32ull || memcmp(image, "MOG", 4) != 0) return NULL;
    or_model *m = (or_model *)calloc(1, sizeof(or_model));
    const rec *r = (const rec *)(image + 33429936ull);
    for (int i = 0; i < NREC; i++) {
        m->t[i].data = r[i].data ? (const void *)(image + r[i].data) : NULL;
        m->t[i].scales = r[i].scales ? (const uint16_t *)(image + r[i].scales) : NULL;
        memcpy(m->t[i].shape, r[i].shape, sizeof(r[i].shape));
    }
    return m;
}

void or_model_close(or_model *m) { free(m); }

struct or_state {
    float *residual;   /* [CHUNK][HID] */
    float *hidden;     /* [CHUNK][8*HID] */
    float *aux;        /* [CHUNK][8*HID] */
    int8_t *q;         /* [CHUNK][8*HID] */
    float *qs;         /* [CHUNK][8*HID/64] */
    float *ple;        /* [CHUNK][NL][PLEW] */
    float *sliding[3][4]; /* [2][RING][256] */
    float *full[3];       /* [2][MAXCTX][512] */
};

or_state *or_state_new(void) {
    or_state *s = (or_state *)calloc(1, sizeof(or_state));
    s->residual = calloc((size_t)CHUNK * HID, 4);
    s->hidden = calloc((size_t)CHUNK * 8 * HID, 4);
    s->aux = calloc((size_t)CHUNK * 8 * HID, 4);
    s->q = calloc((size_t)CHUNK * 8 * HID, 1);
    s->qs = calloc((size_t)CHUNK * 8 * HID / 64, 4);
    s->ple = calloc((size_t)CHUNK * NL * PLEW, 4);
    for (int a = 0; a < 3; a++) {
        for (int b = 0; b < 4; b++) s->sliding[a][b] = calloc((size_t)2 * RING * 256, 4);
        s->full[a] = calloc((size_t)2 * MAXCTX * 512, 4);
    }
    return s;
}

void or_state_free(or_state *s) {
    if (!s) return;
    free(s->residual); free(s->hidden); free(s->aux); free(s->q); free(s->qs); free(s->ple);
    for (int a = 0; a < 3; a++) {
        for (int b = 0; b < 4; b++) free(s->sliding[a][b]);
        free(s->full[a]);
    }
    free(s);
}

float *or_state_residual(or_state *s) { return s->residual; }

static int owner_of(int layer) { /* gemma4.c:419-420 */
    int global = layer % 5 == 4, o = layer;
    while (o >= 15 || (o % 5 == 4) != global) o--;
    return o;
}

float *or_state_cache(or_state *s, int layer, int which) {
    int o = owner_of(layer);
    int global = layer % 5 == 4;
    float *k = global ? s->full[o / 5] : s->sliding[o / 5][o % 5];
    int hd = global ? 512 : 256, len = global ? MAXCTX : RING;
    return which ? k + (size_t)len * hd : k;
}

static void lin(float *out, const or_state *s, const tens *w, size_t T) {
    or_linear(out, s->q, s->qs, T, (const int8_t *)w->data, w->scales, w->shape[0], w->shape[1]);
}

/* gemma4.c:411-461 attention */
static void attention_layer(const or_model *m, or_state *s, int layer, int start_pos, size_t T) {
    const tens *L = &m->t[L_(layer, 0)];
    int global = layer % 5 == 4;
    int len = global ? MAXCTX : RING, mask = len - 1;
    int hd = L[8].shape[0];             /* q_norm */
    int qw = L[10].shape[0];            /* q_proj rows */
    int heads = qw / hd;
    float *kc = or_state_cache(s, layer, 0), *vc = or_state_cache(s, layer, 1);
    const float *cosv = (const float *)L[17].data, *sinv = (const float *)L[18].data;
    int pairs = L[17].shape[1];

    or_quantize(s->q, s->qs, s->hidden, T, (size_t)L[10].shape[1]);
    lin(s->aux, s, &L[10], T);
    or_rmsnorm(s->aux, s->aux, (const float *)L[8].data, hd, 1e-6f, T * (size_t)heads);
    or_rope(s->aux, cosv, sinv, pairs, heads, hd, start_pos, T);

    if (L[11].data) {
        /* K and V land in ring slots (start_pos + t) & mask; the reference writes
         * the T rows contiguously from start_pos & mask, which is the same slot
         * set whenever the chunk does not cross the ring end. */
        float *k = (float *)malloc((size_t)T * hd * 4), *v = (float *)malloc((size_t)T * hd * 4);
        lin(k, s, &L[11], T);
        lin(v, s, &L[12], T);
        or_rmsnorm(k, k, (const float *)L[9].data, hd, 1e-6f, T);
        or_rmsnorm(v, v, NULL, hd, 1e-6f, T);
        or_rope(k, cosv, sinv, pairs, 1, hd, start_pos, T);
        for (size_t t = 0; t < T; t++) {
            size_t slot = (size_t)((start_pos + (int)t) & mask);
            memcpy(kc + slot * hd, k + t * hd, (size_t)hd * 4);
            memcpy(vc + slot * hd, v + t * hd, (size_t)hd * 4);
        }
        free(k);
        free(v);
    }

    #pragma omp parallel
    {
        float *scores = (float *)malloc(((size_t)start_pos + T) * 4);
        #pragma omp for collapse(2) schedule(dynamic, 1)
        for (int h = 0; h < heads; h++)
            for (size_t t = 0; t < T; t++) {
                int p = start_pos + (int)t;
                int first = (!global && p + 1 > WINDOW) ? p + 1 - WINDOW : 0;
                or_attend(s->hidden + t * qw + (size_t)h * hd, s->aux + t * qw + (size_t)h * hd,
                          kc, vc, first, p + 1 - first, mask, hd, scores);
            }
        free(scores);
    }

    or_quantize(s->q, s->qs, s->hidden, T, (size_t)L[13].shape[1]);
    lin(s->hidden, s, &L[13], T);
}

/* gemma4.c:463-509 forward */
void or_forward(const or_model *m, or_state *s, const int *tokens, size_t T, int start_pos) {
    or_forward_layers(m, s, tokens, T, start_pos, NL);
}

/* The token-conditioned inputs of every layer (gemma4.c:468-477): the scaled
 * token embedding into the residual stream, and the per-layer inputs (model
 * projection of the embedding, RMSNorm, plus the per-layer embedding, times
 * 1/sqrt(2)). */
void or_prologue(const or_model *m, or_state *s, const int *tokens, size_t T) {
    const tens *E = &m->t[0], *EP = &m->t[1];
    const tens *norm_ple = &m->t[2 + NL * 19 + 2], *pmp = &m->t[2 + NL * 19 + 1];
    int plw = norm_ple->shape[0];

    or_embedding(s->residual, (const int8_t *)E->data, E->scales, E->shape[1], tokens, T, sqrtf((float)HID));
    or_quantize(s->q, s->qs, s->residual, T, HID);
    or_linear(s->ple, s->q, s->qs, T, (const int8_t *)pmp->data, pmp->scales, pmp->shape[0], pmp->shape[1]);
    or_rmsnorm(s->ple, s->ple, (const float *)norm_ple->data, plw, 1e-6f * HID, T * NL);
    or_embedding(s->hidden, (const int8_t *)EP->data, EP->scales, EP->shape[1], tokens, T, sqrtf((float)plw));
    or_add_scale(s->ple, s->hidden, T * NL * (size_t)plw, 1.0f / sqrtf(2.0f));
}

/* One decoder layer (the loop body of gemma4.c:479-507) on the T residual rows
 * in the state, at positions start_pos.., with the per-layer inputs in the
 * state: attention (writing this layer's K/V when it owns a cache), the
 * feed-forward block and the per-layer-input gate, each added back onto the
 * residual stream. */
void or_layer(const or_model *m, or_state *s, int l, int start_pos, size_t T) {
    const tens *gelu = &m->t[2 + NL * 19 + 3];
    const float *gt = (const float *)gelu->data;
    const int plw = m->t[2 + NL * 19 + 2].shape[0];
    const tens *L = &m->t[L_(l, 0)];
    or_rmsnorm(s->hidden, s->residual, (const float *)L[0].data, HID, 1e-6f, T);
    attention_layer(m, s, l, start_pos, T);
    or_rmsnorm(s->hidden, s->hidden, (const float *)L[3].data, HID, 1e-6f, T);
    or_add_scale(s->residual, s->hidden, T * HID, 1.0f);

    or_rmsnorm(s->hidden, s->residual, (const float *)L[2].data, HID, 1e-6f, T);
    or_quantize(s->q, s->qs, s->hidden, T, (size_t)L[14].shape[1]);
    lin(s->hidden, s, &L[14], T);
    lin(s->aux, s, &L[15], T);
    or_geglu(s->hidden, s->aux, (int)T, L[14].shape[0], L[14].shape[0], gt, gelu->shape[0], gelu->shape[1], gelu->shape[2]);
    or_quantize(s->q, s->qs, s->hidden, T, (size_t)L[16].shape[1]);
    lin(s->hidden, s, &L[16], T);
    or_rmsnorm(s->hidden, s->hidden, (const float *)L[4].data, HID, 1e-6f, T);
    or_add_scale(s->residual, s->hidden, T * HID, 1.0f);

    or_quantize(s->q, s->qs, s->residual, T, HID);
    lin(s->hidden, s, &L[6], T);
    or_geglu(s->hidden, s->ple + (size_t)l * plw, (int)T, plw, NL * plw, gt, gelu->shape[0], gelu->shape[1], gelu->shape[2]);
    or_quantize(s->q, s->qs, s->hidden, T, (size_t)L[7].shape[1]);
    lin(s->hidden, s, &L[7], T);
    or_rmsnorm(s->hidden, s->hidden, (const float *)L[5].data, HID, 1e-6f, T);
    or_add_scale(s->residual, s->hidden, T * HID, ((const float *)L[1].data)[0]);
}

/* forward restricted to the first `layers` layers (a testing aid for
 * bisecting mismatches; layers = 35 is the reference's forward). */
void or_forward_layers(const or_model *m, or_state *s, const int *tokens, size_t T, int start_pos, int layers) {
    or_prologue(m, s, tokens, T);
    for (int l = 0; l < layers; l++) or_layer(m, s, l, start_pos, T);
}

float *or_state_ple(or_state *s) { return s->ple; }

/* logits() (gemma4.c:512-522) of the first `rows` (<= 512) residual rows at
 * once, into out[rows][262144]: the same per-row arithmetic as or_logits, with
 * the lm_head matrix read once for all rows. */
void or_logits_rows(const or_model *m, or_state *s, size_t rows, float *out) {
    const tens *E = &m->t[0], *norm = &m->t[2 + NL * 19];
    or_rmsnorm(s->hidden, s->residual, (const float *)norm->data, HID, 1e-6f, rows);
    or_quantize(s->q, s->qs, s->hidden, rows, HID);
    or_linear(out, s->q, s->qs, rows, (const int8_t *)E->data, E->scales, E->shape[0], E->shape[1]);
    or_softcap(out, rows * (size_t)E->shape[0]);
}

/* gemma4.c:512-522 logits: final norm of one residual row, quantise, tied
 * embedding GEMV, soft-cap. Returns a pointer valid until the next call. */
float *or_logits(const or_model *m, or_state *s, size_t row) {
    const tens *E = &m->t[0], *norm = &m->t[2 + NL * 19];
    or_rmsnorm(s->hidden, s->residual + row * HID, (const float *)norm->data, HID, 1e-6f, 1);
    or_quantize(s->q, s->qs, s->hidden, 1, HID);
    or_linear(s->hidden, s->q, s->qs, 1, (const int8_t *)E->data, E->scales, E->shape[0], E->shape[1]);
    or_softcap(s->hidden, (size_t)E->shape[0]);
    return s->hidden;
}
