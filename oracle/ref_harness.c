/*
 * ref_harness.c — TEST INFRASTRUCTURE. Builds the unmodified reference
 * gemma4.c (included from its own source tree, never copied) into a shared
 * library with its `main` renamed, and adds a few accessors so tests and the
 * benchmark's CPU-baseline leg can call the reference's own forward/logits and
 * kernels on seeded inputs. Built by oracle/Makefile into oracle/_ref/ only.
 */
#define main gemma4_ref_main
#include "gemma4.c"
#undef main

size_t g4ref_state_bytes(void) { return sizeof(InferenceState); }
InferenceState *g4ref_state_new(void) { return (InferenceState *)calloc(1, sizeof(InferenceState)); }
void g4ref_state_free(InferenceState *s) { free(s); }
float *g4ref_state_residual(InferenceState *s) { return s->residual; }
float *g4ref_state_hidden(InferenceState *s) { return s->hidden; }
int g4ref_threads(void) { return thread_count(); }

/* Model view over an image whose records hold file offsets: copies the header
 * and records into a separate Model and turns offsets into pointers the way
 * gemma4.c:681-685 does, leaving the image itself untouched. */
Model *g4ref_model_view(uint8_t *image) {
    Model *m = (Model *)malloc(sizeof(Model));
    if (!m) return NULL;
    memcpy(m->magic, image, 4);
    memcpy(&m->weights, image + offsetof(Model, weights), sizeof(m->weights));
    Tensor *t = (Tensor *)&m->weights;
    for (size_t i = 0; i < sizeof(m->weights) / sizeof(*t); i++) {
        t[i].data = t[i].data ? (void *)(image + (uintptr_t)t[i].data) : NULL;
        t[i].scales = t[i].scales ? (uint16_t *)(image + (uintptr_t)t[i].scales) : NULL;
    }
    return m;
}
void g4ref_model_free(Model *m) { free(m); }

/* A Tensor for a standalone packed matrix (kernel-level golden vectors). */
void g4ref_matmul(float *out, const int8_t *xq, const float *xs, void *w, uint16_t *s, int N, int K, size_t rows) {
    Tensor t;
    memset(&t, 0, sizeof(t));
    t.data = w;
    t.scales = s;
    t.shape[0] = N;
    t.shape[1] = K;
    matmul_int8(out, xq, xs, &t, rows);
}
void g4ref_rmsnorm(float *out, const float *in, float *w, int width, float eps, size_t rows) {
    Tensor t;
    memset(&t, 0, sizeof(t));
    t.data = w;
    t.shape[0] = width;
    rmsnorm(out, in, w ? &t : NULL, width, eps, rows);
}
void g4ref_geglu(float *gate, const float *up, int rows, int width, int up_stride, float *table) {
    Tensor t;
    memset(&t, 0, sizeof(t));
    t.data = table;
    t.shape[0] = 4096;
    t.shape[1] = -8;
    t.shape[2] = 8;
    geglu(gate, up, rows, width, up_stride, &t);
}
void g4ref_rope(float *cosv, float *sinv, int pairs, float *v, int heads, int head_dim, int start_pos, size_t tokens) {
    Tensor c, s;
    memset(&c, 0, sizeof(c));
    memset(&s, 0, sizeof(s));
    c.data = cosv;
    s.data = sinv;
    c.shape[0] = s.shape[0] = MAX_CONTEXT;
    c.shape[1] = s.shape[1] = pairs;
    apply_rope(&c, &s, v, heads, head_dim, start_pos, tokens);
}
void g4ref_embedding(float *out, void *w, uint16_t *s, int width, const int *tokens, size_t count, float mult) {
    Tensor t;
    memset(&t, 0, sizeof(t));
    t.data = w;
    t.scales = s;
    t.shape[0] = VOCAB_SIZE;
    t.shape[1] = width;
    embedding(out, &t, tokens, count, mult);
}
