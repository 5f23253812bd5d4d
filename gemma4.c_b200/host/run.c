/*
 * run.c — command-line host of libg4cuda.so with gemma4.c's interface
 * (gemma4.c:647-694):
 *
 *   run [-m model.bin] [-t temperature] [-n max_new_tokens]
 *       [--bench prefill_tokens generated_tokens] [--dump-logits] [prompt]
 *
 * The model file is mapped read-only; its tokenizer section drives the prompt
 * encoding and token text (g4tok.c), and the weights go to the GPU through
 * g4_open. Every forward and logits call of the reference's host loops —
 * prefill / --dump-logits (gemma4.c:563-572), generate (:574-608) and
 * benchmark (:627-645) — is the C ABI's g4_forward / g4_logits_rows / g4_sample
 * / g4_logits instead; sampling runs on the device with the reference's
 * xorshift generator, seeded from the clock as gemma4.c:688 does.
 */
#define _POSIX_C_SOURCE 200809L
#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

#include "../../include/g4cuda.h"
#include "g4tok.h"

#define CHUNK 512            /* tokens per forward call (the reference's BATCH_SIZE) */
#define MAX_CONTEXT 131072
#define VOCAB 262144

static double now_s(void) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return (double)t.tv_sec + (double)t.tv_nsec / 1e9;
}

static void die_rc(g4_ctx *ctx, const char *what, int rc) {
    fprintf(stderr, "%s failed: %s (%s)\n", what, g4_strerror(rc), ctx ? g4_last_error(ctx) : g4_open_error());
    exit(1);
}

#define CALL(ctx, what, expr)                 \
    do {                                      \
        int rc_ = (expr);                     \
        if (rc_ != G4_OK) die_rc(ctx, what, rc_); \
    } while (0)

/* Forward the prompt in chunks; with dump_logits write every position's
 * logits (262144 fp32) to stdout (gemma4.c:563-572). */
static void prefill(g4_ctx *ctx, const int *ids, int n, int dump_logits, float *dump) {
    for (int pos = 0; pos < n; pos += CHUNK) {
        const int m = n - pos < CHUNK ? n - pos : CHUNK;
        CALL(ctx, "g4_forward", g4_forward(ctx, ids + pos, (size_t)m, pos));
        if (dump_logits) {
            CALL(ctx, "g4_logits_rows", g4_logits_rows(ctx, 0, (size_t)m, dump));
            if (fwrite(dump, sizeof(float) * VOCAB, (size_t)m, stdout) != (size_t)m) {
                perror("stdout");
                exit(1);
            }
        }
    }
}

static void benchmark(g4_ctx *ctx, int prefill_tokens, int generated_tokens) {
    static int ids[MAX_CONTEXT];
    if (prefill_tokens > MAX_CONTEXT) prefill_tokens = MAX_CONTEXT;
    if (prefill_tokens > 0) {
        for (int i = 0; i < prefill_tokens; i++) ids[i] = 2 + i % 1000;   /* gemma4.c:630 */
        const double t0 = now_s();
        prefill(ctx, ids, prefill_tokens, 0, NULL);
        CALL(ctx, "g4_logits", g4_logits(ctx, (size_t)((prefill_tokens - 1) % CHUNK), NULL, NULL));
        CALL(ctx, "g4_sync", g4_sync(ctx));
        printf("pp%d %.2f tok/s\n", prefill_tokens, (double)prefill_tokens / (now_s() - t0));
        fflush(stdout);
    }
    if (generated_tokens > 0) {
        const int token = 2;
        const double t0 = now_s();
        for (int pos = prefill_tokens; pos < prefill_tokens + generated_tokens; pos++) {
            CALL(ctx, "g4_forward", g4_forward(ctx, &token, 1, pos));
            CALL(ctx, "g4_logits", g4_logits(ctx, 0, NULL, NULL));   /* computed, not read (gemma4.c:641) */
        }
        CALL(ctx, "g4_sync", g4_sync(ctx));
        printf("tg%d@d%d %.2f tok/s\n", generated_tokens, prefill_tokens,
               (double)generated_tokens / (now_s() - t0));
        fflush(stdout);
    }
}

static void generate(g4_ctx *ctx, const g4tok_table *tok, const char *prompt, int max_new_tokens,
                     float temperature, int dump_logits) {
    static int ids[MAX_CONTEXT];
    const int styled = !dump_logits && isatty(STDOUT_FILENO);
    if (max_new_tokens < 0) {
        fprintf(stderr, "-n must be non-negative\n");
        exit(1);
    }
    const char *segments[3] = {dump_logits ? "" : "<|turn>user\n", prompt,
                               dump_logits ? "" : "<turn|>\n<|turn>model\n"};
    const int n = g4tok_encode(tok, segments, ids, MAX_CONTEXT);
    if (n < 0) {
        fprintf(stderr, "prompt exceeds the %d-token context limit\n", MAX_CONTEXT);
        exit(1);
    }
    if (styled) {
        fputs("\n\033[2;36m────────────────────────────────\033[0m\n", stdout);
        fflush(stdout);
    }
    float *dump = NULL;
    if (dump_logits) {
        dump = (float *)malloc(sizeof(float) * VOCAB * (size_t)CHUNK);
        if (!dump) {
            fprintf(stderr, "out of memory\n");
            exit(1);
        }
    }
    prefill(ctx, ids, n, dump_logits, dump);
    free(dump);
    if (dump_logits) return;

    int end = n + max_new_tokens;
    if (end > MAX_CONTEXT || end < n) end = MAX_CONTEXT;
    for (int pos = n; pos < end; pos++) {
        int next = 0;
        const size_t row = pos == n ? (size_t)((n - 1) % CHUNK) : 0;
        CALL(ctx, "g4_sample", g4_sample(ctx, row, temperature, &next));
        if (next == 1 || next == 106) break;   /* <eos>, <turn|> */
        fputs(g4tok_text(tok, next), stdout);
        fflush(stdout);
        CALL(ctx, "g4_forward", g4_forward(ctx, &next, 1, pos));
    }
    putchar('\n');
}

int main(int argc, char **argv) {
    const char *model_path = "gemma4-E2B-int8.bin";
    const char *prompt = "Why is the sky blue?";
    float temperature = 1.0f;
    int max_new_tokens = 1024;
    int bench = 0, dump_logits = 0, prefill_tokens = 0, generated_tokens = 256;
    for (int i = 1; i < argc; i++) {
        if (!strcmp(argv[i], "-m") && i + 1 < argc) model_path = argv[++i];
        else if (!strcmp(argv[i], "-t") && i + 1 < argc) temperature = (float)atof(argv[++i]);
        else if (!strcmp(argv[i], "-n") && i + 1 < argc) max_new_tokens = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--bench")) {
            bench = 1;
            if (i + 1 < argc) prefill_tokens = atoi(argv[++i]);
            if (i + 1 < argc) generated_tokens = atoi(argv[++i]);
        } else if (!strcmp(argv[i], "--dump-logits")) dump_logits = 1;
        else prompt = argv[i];
    }
    const int fd = open(model_path, O_RDONLY);
    struct stat st;
    if (fd < 0 || fstat(fd, &st)) {
        perror(model_path);
        return 1;
    }
    void *image = mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (image == MAP_FAILED) {
        perror("mmap");
        return 1;
    }
    if ((size_t)st.st_size < 4 || memcmp(image, "MOG", 4) != 0) {
        fprintf(stderr, "bad model file\n");
        return 1;
    }
    const g4tok_table *tok = g4tok_from_image(image, (size_t)st.st_size);
    if (!tok) {
        fprintf(stderr, "bad model file\n");
        return 1;
    }
    g4_ctx *ctx = NULL;
    CALL(NULL, "g4_open", g4_open(image, (uint64_t)st.st_size, 0, &ctx));
    CALL(ctx, "g4_set_seed", g4_set_seed(ctx, (uint64_t)(now_s() * 1e9)));
    if (bench) benchmark(ctx, prefill_tokens, generated_tokens);
    else generate(ctx, tok, prompt, max_new_tokens, temperature, dump_logits);
    g4_close(ctx);
    munmap(image, (size_t)st.st_size);
    return 0;
}
