/*
 * g4tok.c — prompt tokenizer of a gemma4.c model file (see g4tok.h).
 *
 * The arithmetic of tokenisation is the reference's (gemma4.c:61-113), since
 * the same prompt must give the same ids: greedy special-token matching at
 * '<', one lookup per UTF-8 character, byte tokens for misses, then the
 * lowest-rank adjacent merge applied until none matches (the leftmost of equal
 * ranks). Lookups are binary searches over the exporter's sorted 8-byte keys.
 */
#define _POSIX_C_SOURCE 200809L
#include "g4tok.h"

#include <string.h>

_Static_assert(sizeof(g4tok_lookup) == 16, "lookup entry layout");
_Static_assert(sizeof(g4tok_special) == 100 && offsetof(g4tok_special, id) == 96, "special entry layout");
_Static_assert(sizeof(g4tok_table) == G4TOK_BYTES, "tokenizer section layout");

const g4tok_table *g4tok_from_image(const void *image, size_t bytes) {
    if (!image || bytes < 4 + G4TOK_BYTES) return NULL;
    return (const g4tok_table *)((const char *)image + 4);
}

/* Entry whose key equals `key` in entries[0, n) sorted by memcmp, or NULL. */
static const g4tok_lookup *find_key(const g4tok_lookup *entries, int n, const void *key) {
    int lo = 0, hi = n - 1;
    while (lo <= hi) {
        const int mid = lo + (hi - lo) / 2;
        const int c = memcmp(key, entries[mid].key, 8);
        if (c == 0) return &entries[mid];
        if (c < 0) hi = mid - 1;
        else lo = mid + 1;
    }
    return NULL;
}

/* Apply merges to ids[0, n) in place; returns the new count. */
static int merge_pairs(const g4tok_table *tok, int *ids, int n) {
    const int nm = tok->merge_count < 0 ? 0 : tok->merge_count > G4TOK_MERGES ? G4TOK_MERGES : tok->merge_count;
    for (;;) {
        const g4tok_lookup *best = NULL;
        int at = -1;
        for (int i = 0; i + 1 < n; i++) {
            int32_t pair[2] = {ids[i], ids[i + 1]};
            const g4tok_lookup *m = find_key(tok->merges, nm, pair);
            if (m && (!best || m->rank < best->rank)) {
                best = m;
                at = i;
            }
        }
        if (!best) return n;
        ids[at] = best->result;
        memmove(ids + at + 1, ids + at + 2, (size_t)(n - at - 2) * sizeof(*ids));
        n--;
    }
}

int g4tok_encode(const g4tok_table *tok, const char *segments[3], int *ids, int capacity) {
    const int ns = tok->special_count < 0 ? 0 : tok->special_count > G4TOK_SPECIALS ? G4TOK_SPECIALS
                                                                                     : tok->special_count;
    const int ne = tok->encode_count < 0 ? 0 : tok->encode_count > G4TOK_ENCODE ? G4TOK_ENCODE : tok->encode_count;
    int n = 1;   /* ids[0] is <bos> */
    if (capacity < 1) return -1;
    for (int sgi = 0; sgi < 3; sgi++) {
        const char *p = segments[sgi];
        while (*p) {
            if (n >= capacity) return -1;
            if (*p == '<') {
                int hit = -1;
                for (int i = 0; i < ns && hit < 0; i++) {
                    const size_t len = strnlen(tok->specials[i].text, G4TOK_TEXT);
                    if (strncmp(p, tok->specials[i].text, len) == 0) {
                        hit = tok->specials[i].id;
                        p += len;
                    }
                }
                if (hit >= 0) {
                    ids[n++] = hit;
                    continue;
                }
            }
            char piece[8] = {0};
            if (*p == ' ') {   /* SentencePiece's word boundary U+2581 */
                piece[0] = (char)0xE2;
                piece[1] = (char)0x96;
                piece[2] = (char)0x81;
                p++;
            } else {
                piece[0] = *p++;
                if (((unsigned char)piece[0] & 0xC0) == 0xC0)
                    for (int k = 1; k < 4 && ((unsigned char)*p & 0xC0) == 0x80; k++) piece[k] = *p++;
            }
            const g4tok_lookup *e = find_key(tok->encode, ne, piece);
            if (e) {
                ids[n++] = e->result;
                continue;
            }
            for (const unsigned char *b = (const unsigned char *)piece; *b; b++) {
                if (n >= capacity) return -1;
                ids[n++] = 238 + *b;   /* byte tokens: ids 238 .. 493 */
            }
        }
    }
    n = 1 + merge_pairs(tok, ids + 1, n - 1);
    ids[0] = 2;
    return n;
}

const char *g4tok_text(const g4tok_table *tok, int id) {
    return id >= 0 && id < G4TOK_VOCAB ? tok->texts[id] : "";
}
