/*
 * g4_format.h — the gemma4.c ".bin" model-file layout, as the host sees it.
 *
 * The file is the contract between the reference exporter and any runtime, so
 * every constant here must agree with it:
 *   - header "MOG\0" (4 B), then the tokenizer section (33,429,932 B), then 671
 *     tensor records of 32 B each (gemma4.c:119-155 `Tensor`/`ModelWeights`,
 *     exporter.py:31 `TENSOR_RECORD = "<QQ4i"`), then 64-byte-aligned data from
 *     offset align64(4 + 33,429,932 + 55,008) (exporter.py:29-34,333).
 *   - 2-D weights are int8 packed as [row_block(16)][group(K/64)][chunk(16)]
 *     [row(16)][4 bytes] with one FP16 scale per (row, 64-group) stored as
 *     [row_block][group][16] (exporter.py:304-316).
 *   - 1-D tensors, RoPE tables and the GELU table are little-endian fp32.
 *
 * Record indices follow the C struct order of `ModelWeights`/`LayerWeights`
 * (gemma4.c:125-155): embed, embed_per_layer, 35 x 19 layer slots, norm,
 * per_layer_model_projection, per_layer_projection_norm, gelu_table.
 *
 * This header is plain C so the C host, the synthetic-model writer and the
 * CUDA library (C++) share one definition.
 */
#ifndef G4_FORMAT_H
#define G4_FORMAT_H

#include <stddef.h>
#include <stdint.h>

#define G4_NUM_LAYERS 35
#define G4_NUM_KV_LAYERS 15          /* exporter.py:18 — layers 15..34 share caches */
#define G4_HIDDEN 1536
#define G4_VOCAB 262144
#define G4_MAX_CONTEXT 131072
#define G4_SLIDING_WINDOW 512
#define G4_BATCH 512                 /* reference prefill chunk (gemma4.c:31) */
#define G4_SLIDING_RING 1024         /* SLIDING_WINDOW + BATCH_SIZE (gemma4.c:415) */
#define G4_PLE 256                   /* per-layer-input width (gemma4.c:163) */
#define G4_HEADS 8
#define G4_HD_SLIDING 256
#define G4_HD_GLOBAL 512
#define G4_GROUP 64                  /* quantisation group (exporter.py:25) */
#define G4_BLOCK_ROWS 16             /* packed row block (exporter.py:26) */
#define G4_SOFTCAP 30.0f             /* gemma4.c:519 */
#define G4_RMS_EPS 1e-6f

#define G4_TOKENIZER_SPAN 33429932ull /* exporter.py:29, sizeof(Tokenizer) gemma4.c:176 */
#define G4_WEIGHTS_OFFSET 33429936ull /* offsetof(Model, weights) gemma4.c:176 */
#define G4_TEXT_TENSOR_SPAN 55008ull  /* exporter.py:33 */
#define G4_LAYER_SLOTS 19
#define G4_NUM_RECORDS (2 + G4_NUM_LAYERS * G4_LAYER_SLOTS + 4) /* 671 */
#define G4_RECORD_BYTES 32

/* Layer slot order inside one LayerWeights (gemma4.c:125-145). */
enum g4_layer_slot {
    G4_L_INPUT_NORM = 0,
    G4_L_LAYER_SCALAR,
    G4_L_PRE_FFN_NORM,
    G4_L_POST_ATTN_NORM,
    G4_L_POST_FFN_NORM,
    G4_L_POST_PLE_NORM,
    G4_L_PLE_GATE,
    G4_L_PLE_PROJ,
    G4_L_Q_NORM,
    G4_L_K_NORM,
    G4_L_Q_PROJ,
    G4_L_K_PROJ,
    G4_L_V_PROJ,
    G4_L_O_PROJ,
    G4_L_GATE,
    G4_L_UP,
    G4_L_DOWN,
    G4_L_ROPE_COS,
    G4_L_ROPE_SIN
};

/* Whole-model record indices (gemma4.c:147-155). */
#define G4_R_EMBED 0
#define G4_R_EMBED_PER_LAYER 1
#define G4_R_LAYER(l, slot) (2 + (l) * G4_LAYER_SLOTS + (slot))
#define G4_R_NORM (2 + G4_NUM_LAYERS * G4_LAYER_SLOTS + 0)
#define G4_R_PLE_MODEL_PROJ (2 + G4_NUM_LAYERS * G4_LAYER_SLOTS + 1)
#define G4_R_PLE_PROJ_NORM (2 + G4_NUM_LAYERS * G4_LAYER_SLOTS + 2)
#define G4_R_GELU (2 + G4_NUM_LAYERS * G4_LAYER_SLOTS + 3)

/* One 32-byte tensor record as stored in the file: data and scales are byte
 * offsets from the start of the file (0 = absent) until a loader fixes them up
 * to pointers (gemma4.c:681-685). */
typedef struct {
    uint64_t data;
    uint64_t scales;
    int32_t shape[4];
} g4_record;

static inline int g4_layer_is_global(int layer) { return layer % 5 == 4; } /* gemma4.c:414 */

/* Layer whose KV cache `layer` reads: itself for layers < 15, otherwise the
 * latest earlier layer of the same attention type that owns K/V weights
 * (gemma4.c:419-420). */
static inline int g4_cache_owner(int layer) {
    int owner = layer;
    while (owner >= G4_NUM_KV_LAYERS || g4_layer_is_global(owner) != g4_layer_is_global(layer)) owner--;
    return owner;
}

static inline uint64_t g4_align64(uint64_t v) { return (v + 63) & ~(uint64_t)63; }

#endif
