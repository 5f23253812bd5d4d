/*
 * g4synth.c — seeded synthetic Gemma 4 E2B model images in the gemma4.c .bin
 * layout.
 *
 * The real checkpoint is not available, so benchmarks and parity tests run on a
 * random-init model with the exact geometry gemma4.c reads. The layout rules
 * are the exporter's:
 *   - tensors are allocated in the order exporter.py:104-149 visits them
 *     (embeddings, then per layer the 19 slots with the shared RoPE tables
 *     allocated on first use, then the GELU table, final norm,
 *     per_layer_model_projection, per_layer_projection_norm);
 *   - each allocation advances a 64-byte-aligned cursor by count bytes (int8)
 *     or 4*count bytes (fp32), and quantised tensors follow their data with
 *     count/64 FP16 scales (exporter.py:51-70);
 *   - records of layers >= 15 for k_norm/k_proj/v_proj are all zero
 *     (exporter.py:121-124,347).
 *
 * Values: int8 weights uniform over [-127, 127]; one FP16
 * scale per row, base 0.02/73.61 (std of the int8 distribution) times a
 * per-row factor in [0.75, 1.25], so dequantised weights have std ~0.02; norm
 * weights and layer scalars 1.0. Flags add per-(row, group) scale jitter and
 * random norm weights, which tests use to catch indexing mistakes.
 *
 * All randomness is counter-based (splitmix64 of seed, tensor, index), so the
 * image is identical for any thread count and on any machine.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../csrc/g4_format.h"
#include "g4synth.h"

static uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

static uint64_t mix3(uint64_t seed, uint64_t a, uint64_t b) {
    return splitmix64(splitmix64(seed ^ 0x5851F42D4C957F2Dull) ^ splitmix64(a * 0x2545F4914F6CDD1Dull + b));
}

/* uniform in [0, 1) from 24 random bits */
static float unit_float(uint64_t r) { return (float)(r >> 40) * (1.0f / 16777216.0f); }

/* fp32 -> fp16 bits, round to nearest even (normal and subnormal range). */
uint16_t g4synth_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7FFFFFFFu;
    if (absx >= 0x7F800000u) return (uint16_t)(sign | (absx > 0x7F800000u ? 0x7E00u : 0x7C00u));
    if (absx >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* rounds to inf */
    int exp = (int)(absx >> 23) - 127;
    uint32_t mant = (absx & 0x7FFFFFu) | 0x800000u;
    if (exp < -24) return (uint16_t)sign;
    int shift = exp >= -14 ? 13 : 13 + (-14 - exp);
    uint32_t half_exp = exp >= -14 ? (uint32_t)(exp + 15) : 0u;
    uint32_t m = exp >= -14 ? (absx & 0x7FFFFFu) : mant;
    uint32_t q = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t halfway = 1u << (shift - 1);
    uint32_t out = (half_exp << 10) + q;
    if (rem > halfway || (rem == halfway && (q & 1u))) out++;
    return (uint16_t)(sign | out);
}

typedef struct {
    int kind;       /* 0 = int8 matrix, 1 = fp32 vector/table */
    int rows, cols; /* cols = 0 for 1-D */
    int record;     /* record index, -1 for a shared table already recorded */
    int tag;        /* what to fill: see fill_tensor */
    int layer;
} alloc_item;

enum { TAG_MATRIX, TAG_NORM, TAG_SCALAR, TAG_ROPE_COS_S, TAG_ROPE_SIN_S, TAG_ROPE_COS_G, TAG_ROPE_SIN_G, TAG_GELU };

#define MAX_ITEMS 700

static int build_items(alloc_item *items) {
    int n = 0;
#define ADD(kind_, rows_, cols_, rec_, tag_, layer_) \
    items[n++] = (alloc_item){(kind_), (rows_), (cols_), (rec_), (tag_), (layer_)}
    ADD(0, G4_VOCAB, G4_HIDDEN, G4_R_EMBED, TAG_MATRIX, -1);
    ADD(0, G4_VOCAB, G4_NUM_LAYERS * G4_PLE, G4_R_EMBED_PER_LAYER, TAG_MATRIX, -1);
    int rope_s_done = 0, rope_g_done = 0;
    for (int l = 0; l < G4_NUM_LAYERS; l++) {
        int global = g4_layer_is_global(l);
        int kv = l < G4_NUM_KV_LAYERS;
        int hd = global ? G4_HD_GLOBAL : G4_HD_SLIDING;
        int ffn = l < G4_NUM_KV_LAYERS ? 6144 : 12288;
        ADD(1, G4_HIDDEN, 0, G4_R_LAYER(l, G4_L_INPUT_NORM), TAG_NORM, l);
        ADD(1, 1, 0, G4_R_LAYER(l, G4_L_LAYER_SCALAR), TAG_SCALAR, l);
        ADD(1, G4_HIDDEN, 0, G4_R_LAYER(l, G4_L_PRE_FFN_NORM), TAG_NORM, l);
        ADD(1, G4_HIDDEN, 0, G4_R_LAYER(l, G4_L_POST_ATTN_NORM), TAG_NORM, l);
        ADD(1, G4_HIDDEN, 0, G4_R_LAYER(l, G4_L_POST_FFN_NORM), TAG_NORM, l);
        ADD(1, G4_HIDDEN, 0, G4_R_LAYER(l, G4_L_POST_PLE_NORM), TAG_NORM, l);
        ADD(0, G4_PLE, G4_HIDDEN, G4_R_LAYER(l, G4_L_PLE_GATE), TAG_MATRIX, l);
        ADD(0, G4_HIDDEN, G4_PLE, G4_R_LAYER(l, G4_L_PLE_PROJ), TAG_MATRIX, l);
        ADD(1, hd, 0, G4_R_LAYER(l, G4_L_Q_NORM), TAG_NORM, l);
        if (kv) ADD(1, hd, 0, G4_R_LAYER(l, G4_L_K_NORM), TAG_NORM, l);
        ADD(0, G4_HEADS * hd, G4_HIDDEN, G4_R_LAYER(l, G4_L_Q_PROJ), TAG_MATRIX, l);
        if (kv) ADD(0, hd, G4_HIDDEN, G4_R_LAYER(l, G4_L_K_PROJ), TAG_MATRIX, l);
        if (kv) ADD(0, hd, G4_HIDDEN, G4_R_LAYER(l, G4_L_V_PROJ), TAG_MATRIX, l);
        ADD(0, G4_HIDDEN, G4_HEADS * hd, G4_R_LAYER(l, G4_L_O_PROJ), TAG_MATRIX, l);
        ADD(0, ffn, G4_HIDDEN, G4_R_LAYER(l, G4_L_GATE), TAG_MATRIX, l);
        ADD(0, ffn, G4_HIDDEN, G4_R_LAYER(l, G4_L_UP), TAG_MATRIX, l);
        ADD(0, G4_HIDDEN, ffn, G4_R_LAYER(l, G4_L_DOWN), TAG_MATRIX, l);
        /* shared RoPE tables: allocated the first time a layer of that type uses them */
        if (!global && !rope_s_done) {
            ADD(1, G4_MAX_CONTEXT, 128, -2, TAG_ROPE_COS_S, l);
            ADD(1, G4_MAX_CONTEXT, 128, -3, TAG_ROPE_SIN_S, l);
            rope_s_done = 1;
        }
        if (global && !rope_g_done) {
            ADD(1, G4_MAX_CONTEXT, 64, -4, TAG_ROPE_COS_G, l);
            ADD(1, G4_MAX_CONTEXT, 64, -5, TAG_ROPE_SIN_G, l);
            rope_g_done = 1;
        }
    }
    ADD(1, 4096, 0, G4_R_GELU, TAG_GELU, -1);
    ADD(1, G4_HIDDEN, 0, G4_R_NORM, TAG_NORM, -1);
    ADD(0, G4_NUM_LAYERS * G4_PLE, G4_HIDDEN, G4_R_PLE_MODEL_PROJ, TAG_MATRIX, -1);
    ADD(1, G4_PLE, 0, G4_R_PLE_PROJ_NORM, TAG_NORM, -1);
#undef ADD
    return n;
}

/* Computes every record; returns the image size in bytes. */
uint64_t g4synth_layout(g4_record *records /* G4_NUM_RECORDS entries, may be NULL */) {
    static alloc_item items[MAX_ITEMS];
    int n = build_items(items);
    g4_record recs[G4_NUM_RECORDS];
    memset(recs, 0, sizeof(recs));
    g4_record rope[4];
    memset(rope, 0, sizeof(rope));
    uint64_t cursor = g4_align64(4 + G4_TOKENIZER_SPAN + G4_TEXT_TENSOR_SPAN);
    for (int i = 0; i < n; i++) {
        alloc_item *it = &items[i];
        g4_record r;
        memset(&r, 0, sizeof(r));
        uint64_t count = (uint64_t)it->rows * (uint64_t)(it->cols ? it->cols : 1);
        r.data = cursor;
        cursor = g4_align64(cursor + count * (it->kind == 0 ? 1 : 4));
        if (it->kind == 0) {
            r.scales = cursor;
            cursor = g4_align64(cursor + count / G4_GROUP * 2);
        }
        r.shape[0] = it->rows;
        r.shape[1] = it->cols;
        if (it->tag == TAG_GELU) { r.shape[0] = 4096; r.shape[1] = -8; r.shape[2] = 8; }
        if (it->record >= 0) recs[it->record] = r;
        else rope[-it->record - 2] = r;
    }
    /* every layer points at the shared table of its type (exporter.py:99-102,129) */
    for (int l = 0; l < G4_NUM_LAYERS; l++) {
        int g = g4_layer_is_global(l) ? 2 : 0;
        recs[G4_R_LAYER(l, G4_L_ROPE_COS)] = rope[g];
        recs[G4_R_LAYER(l, G4_L_ROPE_SIN)] = rope[g + 1];
    }
    if (records) memcpy(records, recs, sizeof(recs));
    return cursor;
}

uint64_t g4synth_image_bytes(void) { return g4synth_layout(NULL); }

static void fill_matrix(uint8_t *image, const g4_record *r, uint64_t seed, uint64_t tid, unsigned flags) {
    int rows = r->shape[0], cols = r->shape[1];
    int groups = cols / G4_GROUP;
    int8_t *data = (int8_t *)(image + r->data);
    uint16_t *scales = (uint16_t *)(image + r->scales);
    uint64_t count = (uint64_t)rows * (uint64_t)cols;
    uint64_t words = count / 4;
    uint64_t key = mix3(seed, tid, 0x1234567ull);
    #pragma omp parallel for schedule(static)
    for (int64_t w = 0; w < (int64_t)words; w++) {
        uint64_t x = splitmix64(key + (uint64_t)w * 0x9E3779B97F4A7C15ull);
        for (int j = 0; j < 4; j++) {
            uint32_t h = (uint32_t)((x >> (16 * j)) & 0xFFFFu);
            data[(uint64_t)w * 4 + j] = (int8_t)((int)((h * 255u) >> 16) - 127);
        }
    }
    const float base = 0.02f / 73.6122f;
    #pragma omp parallel for schedule(static)
    for (int n = 0; n < rows; n++) {
        float row_factor = 0.75f + 0.5f * unit_float(mix3(seed, tid | (1ull << 62), (uint64_t)n));
        for (int g = 0; g < groups; g++) {
            float f = row_factor;
            if (flags & G4SYN_GROUP_SCALES)
                f = 0.5f + unit_float(mix3(seed, tid | (1ull << 61), (uint64_t)n * 4096u + (uint64_t)g));
            uint64_t at = ((uint64_t)(n / G4_BLOCK_ROWS) * (uint64_t)groups + (uint64_t)g) * G4_BLOCK_ROWS + (uint64_t)(n % G4_BLOCK_ROWS);
            scales[at] = g4synth_f32_to_f16(base * f);
        }
    }
}

static void fill_rope(uint8_t *image, const g4_record *r, int is_sin, int head_dim, float theta) {
    int positions = r->shape[0], pairs = r->shape[1];
    float *out = (float *)(image + r->data);
    float freq[256];
    for (int j = 0; j < pairs; j++) {
        float exponent = (float)(2 * j) / (float)head_dim;      /* exporter.py:81 */
        freq[j] = 1.0f / powf(theta, exponent);                  /* exporter.py:82 */
    }
    #pragma omp parallel for schedule(static)
    for (int p = 0; p < positions; p++)
        for (int j = 0; j < pairs; j++) {
            float angle = (float)p * freq[j];                    /* exporter.py:83 */
            out[(uint64_t)p * pairs + j] = is_sin ? (float)sin((double)angle) : (float)cos((double)angle);
        }
}

static void fill_gelu(uint8_t *image, const g4_record *r) {
    float *out = (float *)(image + r->data);
    const int n = 4096;
    for (int i = 0; i < n; i++) {
        /* np.linspace(-8, 8, 4096, dtype=float32) evaluates in double then rounds */
        float x = (float)(-8.0 + (double)i * (16.0 / (double)(n - 1)));
        if (i == n - 1) x = 8.0f;
        float inner = 0.7978845608f * (x + 0.044715f * x * x * x);
        out[i] = 0.5f * x * (1.0f + tanhf(inner));                /* exporter.py:73-75 */
    }
}

int g4synth_fill(uint8_t *image, uint64_t bytes, uint64_t seed, unsigned flags) {
    g4_record recs[G4_NUM_RECORDS];
    uint64_t need = g4synth_layout(recs);
    if (!image || bytes < need) return -1;
    /* header + tokenizer (zero counts: --bench never tokenises) + records */
    memset(image, 0, (size_t)recs[G4_R_EMBED].data);
    memcpy(image, "MOG", 4);
    memcpy(image + G4_WEIGHTS_OFFSET, recs, sizeof(recs));

    static alloc_item items[MAX_ITEMS];
    int n = build_items(items);
    g4_record rope[4];
    int rope_seen = 0;
    for (int i = 0; i < n; i++) {
        alloc_item *it = &items[i];
        const g4_record *r;
        if (it->record >= 0) r = &recs[it->record];
        else {
            int which = -it->record - 2;
            int l = it->layer;
            rope[which] = recs[G4_R_LAYER(l, (which & 1) ? G4_L_ROPE_SIN : G4_L_ROPE_COS)];
            r = &rope[which];
            rope_seen++;
        }
        uint64_t tid = (uint64_t)i + 1;
        /* zero the alignment padding behind this tensor */
        uint64_t count = (uint64_t)r->shape[0] * (uint64_t)(it->cols ? it->cols : 1);
        if (it->tag == TAG_GELU) count = 4096;
        uint64_t end = r->data + count * (it->kind == 0 ? 1 : 4);
        if (it->kind == 0) {
            memset(image + end, 0, (size_t)(r->scales - end));
            uint64_t send = r->scales + count / G4_GROUP * 2;
            memset(image + send, 0, (size_t)(g4_align64(send) - send));
        } else {
            memset(image + end, 0, (size_t)(g4_align64(end) - end));
        }
        switch (it->tag) {
        case TAG_MATRIX: fill_matrix(image, r, seed, tid, flags); break;
        case TAG_NORM: {
            float *w = (float *)(image + r->data);
            for (int j = 0; j < r->shape[0]; j++)
                w[j] = (flags & G4SYN_RANDOM_NORMS) ? 0.5f + unit_float(mix3(seed, tid, (uint64_t)j)) : 1.0f;
            break;
        }
        case TAG_SCALAR: {
            float *w = (float *)(image + r->data);
            w[0] = (flags & G4SYN_RANDOM_NORMS) ? 0.5f + unit_float(mix3(seed, tid, 0)) : 1.0f;
            break;
        }
        case TAG_ROPE_COS_S: fill_rope(image, r, 0, G4_HD_SLIDING, 10000.0f); break;
        case TAG_ROPE_SIN_S: fill_rope(image, r, 1, G4_HD_SLIDING, 10000.0f); break;
        case TAG_ROPE_COS_G: fill_rope(image, r, 0, G4_HD_GLOBAL, 1000000.0f); break;
        case TAG_ROPE_SIN_G: fill_rope(image, r, 1, G4_HD_GLOBAL, 1000000.0f); break;
        case TAG_GELU: fill_gelu(image, r); break;
        default: return -2;
        }
    }
    return rope_seen == 4 ? 0 : -3;
}

int g4synth_write_file(const char *path, uint64_t seed, unsigned flags) {
    uint64_t bytes = g4synth_image_bytes();
    uint8_t *image = (uint8_t *)malloc((size_t)bytes);
    if (!image) return -1;
    int rc = g4synth_fill(image, bytes, seed, flags);
    if (rc == 0) {
        FILE *f = fopen(path, "wb");
        if (!f) rc = -4;
        else {
            if (fwrite(image, 1, (size_t)bytes, f) != (size_t)bytes) rc = -5;
            if (fclose(f)) rc = -5;
        }
    }
    free(image);
    return rc;
}
