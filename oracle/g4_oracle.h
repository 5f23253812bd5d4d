/*
 * g4_oracle.h — CPU restatement of gemma4.c's forward path. TEST
 * INFRASTRUCTURE ONLY: the parity checker for the CUDA library. Nothing in the
 * product links or calls it; tests, the smoke check and the CPU-baseline leg of
 * the benchmark do.
 */
#ifndef G4_ORACLE_H
#define G4_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- kernels (each cites the reference function it restates) ---- */
void or_quantize(int8_t *q, float *scales, const float *x, size_t rows, size_t width);
/* int32 dot of every (token, output row, 64-group): dots[(t*N + n)*G + g] */
void or_linear_dots(int32_t *dots, const int8_t *xq, size_t tokens, const int8_t *w_packed, int N, int K);
void or_linear(float *out, const int8_t *xq, const float *xs, size_t tokens,
               const int8_t *w_packed, const uint16_t *s_packed, int N, int K);
void or_rmsnorm(float *out, const float *in, const float *weight, int width, float eps, size_t rows);
void or_add_scale(float *out, const float *addend, size_t count, float scale);
void or_rope(float *v, const float *cos_table, const float *sin_table, int pairs,
             int heads, int head_dim, int start_pos, size_t tokens);
void or_geglu(float *gate, const float *up, int rows, int width, int up_stride,
              const float *table, int table_size, int lower, int upper);
void or_embedding(float *out, const int8_t *w_packed, const uint16_t *s_packed, int width,
                  const int *tokens, size_t count, float multiplier);
float or_f16_to_f32(uint16_t h);
float or_score(const float *q, const float *k, int head_dim);
void or_softmax(float *v, int n);
void or_softcap(float *x, size_t n);
int or_argmax(const float *x, int n);
/* Top-k in the reference's sampling order (descending, ties keep the lower id). */
void or_topk(const float *x, int n, int k, float *vals, int *ids);
/* One attention head for one query over ring positions [first, first+n). */
void or_attend(float *out, const float *q, const float *kcache, const float *vcache,
               int first, int n, int mask, int head_dim, float *scratch);

/* ---- whole model ---- */
typedef struct or_model or_model;
typedef struct or_state or_state;
/* `image` is a .bin image whose tensor records hold file offsets. */
or_model *or_model_open(const uint8_t *image, uint64_t bytes);
void or_model_close(or_model *m);
or_state *or_state_new(void);
void or_state_free(or_state *s);
void or_forward(const or_model *m, or_state *s, const int *tokens, size_t count, int start_pos);
void or_forward_layers(const or_model *m, or_state *s, const int *tokens, size_t count, int start_pos, int layers);
float *or_logits(const or_model *m, or_state *s, size_t row);
/* Teacher-forced pieces of forward: the per-layer inputs of T tokens, and one
 * layer applied to the residual rows (and per-layer inputs) in the state. */
void or_prologue(const or_model *m, or_state *s, const int *tokens, size_t T);
void or_layer(const or_model *m, or_state *s, int layer, int start_pos, size_t T);
float *or_state_residual(or_state *s);
/* Per-layer inputs [512 rows][35][256]. */
float *or_state_ple(or_state *s);
/* logits of residual rows [0, rows) into out[rows][262144]. */
void or_logits_rows(const or_model *m, or_state *s, size_t rows, float *out);
/* Key (which=0) or value (which=1) cache that `layer` reads. */
float *or_state_cache(or_state *s, int layer, int which);
int or_num_threads(void);

#ifdef __cplusplus
}
#endif
float or_random_uniform(unsigned long long *state);
int or_sample(const float *logits, int n, float temperature, unsigned long long *state);

#endif
