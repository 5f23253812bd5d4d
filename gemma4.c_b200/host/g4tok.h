/*
 * g4tok.h — the prompt tokenizer and token text of a gemma4.c model file, for
 * the C host (run.c). Restates tokenize / apply_bpe_merges / token_text
 * (gemma4.c:61-113) over the tokenizer section the exporter writes into the
 * .bin, which sits right after the 4-byte magic (gemma4.c:34-54, 169-172).
 */
#ifndef G4TOK_H
#define G4TOK_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Section layout of the file (the contract between exporter and runtime). */
#define G4TOK_VOCAB 262144
#define G4TOK_TEXT 94            /* bytes per decoded token text, NUL included */
#define G4TOK_SPECIALS 256
#define G4TOK_ENCODE 32768
#define G4TOK_MERGES 514906
#define G4TOK_BYTES 33429932ull  /* the whole section */

typedef struct {
    char key[8];   /* a UTF-8 piece (NUL padded) or two int32 token ids */
    int32_t result, rank;
} g4tok_lookup;

typedef struct {
    char text[G4TOK_TEXT];
    int32_t id;   /* at offset 96 (two bytes of padding before it) */
} g4tok_special;

typedef struct {
    int32_t merge_count, encode_count, special_count;
    char texts[G4TOK_VOCAB][G4TOK_TEXT];
    g4tok_special specials[G4TOK_SPECIALS];
    g4tok_lookup encode[G4TOK_ENCODE];
    g4tok_lookup merges[G4TOK_MERGES];
} g4tok_table;

/* The tokenizer section of a mapped model file (4 bytes in), or NULL when the
 * mapping is too short. */
const g4tok_table *g4tok_from_image(const void *image, size_t bytes);

/* Token ids of the concatenation of three segments, <bos> (id 2) first:
 * special tokens matched at '<', then one piece per UTF-8 character (a space
 * is U+2581), byte tokens (238 + byte) for pieces outside the direct vocabulary,
 * then BPE merges in rank order. Returns the count, or -1 when more than
 * `capacity` ids would be needed. */
int g4tok_encode(const g4tok_table *tok, const char *segments[3], int *ids, int capacity);

/* The text of token `id` ("" outside the vocabulary). */
const char *g4tok_text(const g4tok_table *tok, int id);

#ifdef __cplusplus
}
#endif
#endif
