// g4_decode.cu — single-token decode as one persistent kernel per step.
//
// Reference: forward (gemma4.c:463-509) for one token, optionally followed by
// logits (gemma4.c:512-522), i.e. one step of benchmark()/generate()
// (gemma4.c:599-606, 637-642).
//
// One cooperative launch, one CTA per SM (8 consumer warps + 1 producer warp).
// The host builds the step as a list of ops (every int8 GEMV with its fused
// prologue/epilogue, split-KV attention, split combine, PLE prep, last
// residual update) that run in order, separated by grid-wide barriers where an
// op reads what the previous one wrote.
//
// Weight streaming. The producer warp streams this CTA's weight slices of
// EVERY GEMV of the step, in op order, with TMA bulk copies into one byte ring
// of shared memory (160 KB). It only waits for ring space, never for grid
// barriers, so HBM keeps streaming while the consumers sit in a barrier, a
// prologue or attention. A stage is a run of whole row pairs (weights then
// their fp16 scales, contiguous) placed at the next ring offset, or at offset 0
// when it would not fit before the end; producer and consumers derive the same
// offsets from the same stage sizes. Each stage has a single-use mbarrier for
// "landed"; consumers count finished row pairs per stage (mod 64) and the
// producer frees ring space in stage order.
//
// The arithmetic is the standalone kernels' (g4_gemv_dev.cuh,
// g4_attn_dev.cuh): same exact int32 dots, same ordered dequant chains, same
// reductions and attention tiles, so both paths give the same bits.
#include "g4_attn_dev.cuh"
#include "g4_gemv_dev.cuh"

namespace {

constexpr int kThreads = kConsumers + 32;
constexpr unsigned kRingBytes = 160 * 1024;
constexpr unsigned kStageMaxW = 64 * 1024;  // weight bytes of one stage at most
constexpr int kFifo = 64;                  // stages in flight at most
constexpr int kMaxStages = 1152;           // single-use stage barriers per step
constexpr int kMaxK = 12288;
constexpr int kKT256 = DecodeKT<256>::value, kKT512 = DecodeKT<512>::value;

__host__ __device__ constexpr int cmax(int a, int b) { return a > b ? a : b; }
constexpr int kAttnBytes = cmax(decode_smem_floats(256, kKT256), decode_smem_floats(512, kKT512)) * 4;
constexpr int kGemvScratch = kMaxK + (kMaxK / 64) * 4 + G4_HIDDEN * 4;   // xq + xs + vec bytes
constexpr int kDotsBytes = 32 * (kMaxK / 64) * 4;   // group-parallel dots: [G][32 rows] int32
constexpr int kScratchBytes = cmax(cmax(kAttnBytes, kGemvScratch + kDotsBytes), (512 + 16) * 4);
// the GELU table's copy sits in the group-parallel dots region past the dots of
// K <= 1536 ([24 groups][32 rows] int32); GEGLU GEMVs have K = 1536
constexpr int kGeluOff = 8192;
static_assert(kGeluOff >= 32 * (1536 / 64) * 4 && kGeluOff + 4096 * 4 <= kDotsBytes, "GELU table copy");

constexpr int kOffRing = 0;
constexpr int kOffFull = kOffRing + (int)kRingBytes;
constexpr int kOffDone = kOffFull + kMaxStages * 8;
constexpr int kOffFifo = kOffDone + kFifo * 4;       // per in-flight stage: ring end, pairs
constexpr int kOffScratch = (kOffFifo + kFifo * 8 + 127) / 128 * 128;
constexpr int kOffRed = kOffScratch + kScratchBytes;
constexpr int kOffOps = kOffRed + 512 * 4;           // two op descriptors (current, next)
constexpr int kOpWords = (int)(sizeof(DecodeOp) / 16);
constexpr int kSmemBytes = kOffOps + 2 * (int)sizeof(DecodeOp);
static_assert(sizeof(DecodeOp) % 16 == 0 && kOpWords <= kConsumers, "op descriptor copy");
static_assert(kSmemBytes + 256 <= 227 * 1024, "shared memory budget");

G4_DEV unsigned long long ld_acquire_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
G4_DEV void red_release_add(unsigned long long *p, unsigned long long v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Grid-wide barrier among the consumer warps of all CTAs (bounded wait). A CTA
// whose op failed (fail != 0: a stage that never arrived) does not arrive; the
// others then give up after the bounded wait. Returns the same value to every
// consumer thread of the CTA. The arrival is a gpu-scope release (it orders the
// CTA's earlier writes, seen by thread 0 through the CTA barrier) and the
// polling load an acquire.
// tr (tracing only): [1] <- latest time a CTA finished the op, [2] <- latest barrier exit.
G4_DEV bool grid_barrier(const DecodeParams &P, unsigned long long target, const volatile int *fail,
                         unsigned long long *tr) {
    csync();
    __shared__ int ok;
    if (threadIdx.x == 0) {
        if (tr) atomicMax(tr + 1, (unsigned long long)g4_globaltimer());
        ok = *fail == 0;
        if (ok) {
            red_release_add(P.bar, 1ull);
            if (ld_acquire_u64(P.bar) < target) {
                const uint64_t t0 = g4_globaltimer();
                while (ld_acquire_u64(P.bar) < target) {
                    if (g4_globaltimer() - t0 > G4_WAIT_NS) {
                        g4_set_error(P.err, G4D_TIMEOUT_FULL | (0xfff << 8) | ((int)blockIdx.x << 20));
                        ok = 0;
                        break;
                    }
                }
            }
            if (tr) atomicMax(tr + 2, (unsigned long long)g4_globaltimer());
        }
    }
    csync();
    return ok != 0;
}

// Rows per weight stage: at most 32 (one per lane) and 64 KB of weights,
// an even number when more than one (GEGLU row pairs stay in one stage).
__host__ __device__ constexpr int dstage_rows(int K) {
    return (int)(kStageMaxW / (unsigned)K) >= 32 ? 32 : ((int)(kStageMaxW / (unsigned)K) & ~1) < 2 ? 1
                                                       : ((int)(kStageMaxW / (unsigned)K) & ~1);
}

// This CTA's rows of a GEMV: whole row pairs, split evenly over the grid with
// the op's precomputed partition (no integer division in the kernel).
struct CtaRows {
    int n0, rows, R, nst;
};
__host__ __device__ inline CtaRows cta_rows_of(const DecodeOp &op, int b) {
    CtaRows c;
    const int more = b < op.part_r;
    c.n0 = 2 * (b * op.part_q + (more ? b : op.part_r));
    c.rows = 2 * (op.part_q + more);
    c.R = op.srows;
    c.nst = op.nst[more];
    return c;
}
G4_DEV CtaRows cta_rows(const DecodeOp &op) { return cta_rows_of(op, blockIdx.x); }
// Fill the partition fields of a GEMV op for a grid of `grid` CTAs.
void set_partition(DecodeOp &op, int grid) {
    const int npairs = op.g.m.N / 2, R = dstage_rows(op.g.m.K);
    op.part_q = npairs / grid;
    op.part_r = npairs % grid;
    op.srows = R;
    op.nst[0] = (2 * op.part_q + R - 1) / R;
    op.nst[1] = (2 * op.part_q + 2 + R - 1) / R;
}
// Row-parallel schedule (a warp per stage) for CTAs with more than 32 rows,
// else group-parallel (all warps on each stage, one chain pass at the end).
__host__ __device__ inline bool row_parallel(const CtaRows &cr) { return cr.rows > 32; }
// Consumer releases a stage needs before its ring space is reused.
__host__ __device__ inline unsigned stage_releases(const CtaRows &cr) { return row_parallel(cr) ? 1u : 8u; }
G4_DEV int stage_nr(const CtaRows &cr, int j) { return min(cr.R, cr.rows - j * cr.R); }
// bytes of stage j: nr rows of K int8 weights, then nr * K/64 fp16 scales
G4_DEV unsigned stage_bytes(const CtaRows &cr, int j, int K) {
    const unsigned nr = (unsigned)stage_nr(cr, j);
    return nr * (unsigned)K + nr * (unsigned)(K >> 6) * 2u;
}
// Next ring position (monotonic byte count) for a stage of sz bytes: skip the
// tail of the ring when the stage would not fit before its end.
G4_DEV unsigned ring_take(unsigned &head, unsigned sz) {
    const unsigned off = head % kRingBytes;
    if (off + sz > kRingBytes) head += kRingBytes - off;
    const unsigned start = head;
    head += sz;
    return start;
}

// The kernel runs every op of the step once per layer, so its instruction
// footprint is what the SM's instruction caches must hold: the GEMV is one
// function with run-time prologue/epilogue selection (one copy of the row
// loop), and each prologue variant exists once.
G4_DEV __noinline__ void decode_prologue(const GemvArgs &a, int pro, int8_t *xq, float *xs, float *vec, float *red) {
    switch (pro) {
    case PRO_EMBED_QUANT: prologue<1, PRO_EMBED_QUANT>(a, xq, xs, vec, red); break;
    case PRO_NORM_QUANT: prologue<1, PRO_NORM_QUANT>(a, xq, xs, vec, red); break;
    case PRO_RES_NORM_QUANT: prologue<1, PRO_RES_NORM_QUANT>(a, xq, xs, vec, red); break;
    case PRO_LOADQ: prologue<1, PRO_LOADQ>(a, xq, xs, vec, red); break;
    case PRO_QUANT: prologue<1, PRO_QUANT>(a, xq, xs, vec, red); break;
    default: prologue<1, PRO_RES_QUANT>(a, xq, xs, vec, red); break;
    }
}

// Exact int32 dot of one 64-byte group of a row with the quantised input: four
// 16-byte chunks, visited in an order rotated by `rot` so that lanes reading
// different rows at the same offset spread over the shared-memory banks.
G4_DEV int group_dot(const uint8_t *w, const int8_t *x, int rot) {
    int d0 = 0, d1 = 0;
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const int cc = (c + rot) & 3;
        const uint4 w4 = *(const uint4 *)(w + cc * 16);
        const int4 x4 = *(const int4 *)(x + cc * 16);
        d0 = dp4a(w4.x, (uint32_t)x4.x, d0);
        d1 = dp4a(w4.y, (uint32_t)x4.y, d1);
        d0 = dp4a(w4.z, (uint32_t)x4.z, d0);
        d1 = dp4a(w4.w, (uint32_t)x4.w, d1);
    }
    return d0 + d1;
}

// One row's ordered dequantisation chain from its group dots (gemma4.c:245-259):
// acc = fma((float)dot_g, ws_g * xs_g, acc), g ascending. The four scales of
// groups g..g+3 are one 8-byte load.
G4_DEV float chain_step(float acc, int d, float ws, float xsg) {
    return __fmaf_rn(__int2float_rn(d), __fmul_rn(ws, xsg), acc);
}
G4_DEV float scale_at(uint2 s4, int k) {
    const uint32_t w = (k & 2) ? s4.y : s4.x;
    return h2f((uint16_t)((k & 1) ? (w >> 16) : (w & 0xFFFFu)));
}

// Per-row epilogue of a finished row (lane = row within the stage). GEGLU
// pairs are lanes (2i, 2i + 1) of the same warp, so every lane of the warp
// must call it. gelu: the GELU table (shared memory); u: the row's per-layer
// input (EPI_PLE), loaded before the row's dots so its latency is hidden.
G4_DEV void row_epilogue(const GemvArgs &a, int epi, int n, float acc, bool active, const float *gelu, float u,
                         float &best_v, int &best_i) {
    const float up = __shfl_down_sync(0xffffffffu, acc, 1);
    if (!active) return;
    if (epi == EPI_STORE) {
        a.out[n] = acc;
    } else if (epi == EPI_GEGLU_PAIR) {
        if ((n & 1) == 0) a.out[n >> 1] = geglu_one(acc, up, gelu, 4096, -8.0f, 8.0f, 4095.0f / 16.0f);
    } else if (epi == EPI_PLE) {
        a.out[n] = geglu_one(acc, u, gelu, 4096, -8.0f, 8.0f, 4095.0f / 16.0f);
    } else {
        const float sv = __fmul_rn(30.0f, tanhf(__fdiv_rn(acc, 30.0f)));   // gemma4.c:519
        a.out[n] = sv;
        if (sv > best_v || (sv == best_v && n < best_i)) { best_v = sv; best_i = n; }
    }
}

// One GEMV op, consumer side. cs: this op's first stage index; head: ring
// position of its first stage (advanced past the op on return).
//
// A stage holds up to 32 whole rows (lane = row). Two schedules:
//  - row-parallel (8 or more stages): warp w takes stages w, w + 8, ... and
//    runs each row's dots and chain in its lane;
//  - group-parallel (fewer stages): all warps take one stage at a time, warp w
//    computes the dots of groups [w G / 8, (w + 1) G / 8) of every row into
//    shared memory, then warp 0 runs the rows' chains.
// A warp whose stage wait runs out leaves as a whole warp and sets *fail; it
// still takes every consumer barrier below, so the CTA never deadlocks.
G4_DEV __noinline__ void gemv_op(const GemvArgs &a, const CtaRows cr, int pro, int epi, int cs, unsigned &head,
                                 uint8_t *smem, volatile int *fail, unsigned long long *tr) {
    const int K = a.m.K, G = K >> 6;
    uint8_t *ring = smem + kOffRing;
    uint64_t *full = (uint64_t *)(smem + kOffFull);
    int *done = (int *)(smem + kOffDone);
    int8_t *xq = (int8_t *)(smem + kOffScratch);
    float *xs = (float *)(smem + kOffScratch + kMaxK);
    float *vec = (float *)(smem + kOffScratch + kMaxK + (kMaxK / 64) * 4);
    float *red = (float *)(smem + kOffRed);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // GEGLU epilogues look their GELU values up in a shared-memory copy of the
    // table, copied in while the prologue runs (past the group dots of K <= 1536)
    float *gelu_s = (float *)(smem + kOffScratch + kGemvScratch + kGeluOff);
    const bool geglu = epi == EPI_GEGLU_PAIR || epi == EPI_PLE;
    if (geglu) {
        for (int i = tid; i < 4096 / 4; i += kConsumers) cp_async16(gelu_s + 4 * i, a.gelu + 4 * i);
        cp_async_commit();
    }
    // the per-layer input of warp 0's rows (group-parallel EPI_PLE), early
    float u0 = 0.0f;
    if (epi == EPI_PLE && warp == 0 && lane < cr.rows) u0 = a.ple_u[cr.n0 + lane];

    decode_prologue(a, pro, xq, xs, vec, red);
    if (geglu) cp_async_wait<0>();
    csync();
    if (tr && tid == 0) atomicMax(tr, (unsigned long long)g4_globaltimer());
    float best_v = -INFINITY;
    int best_i = 0x7fffffff;
    unsigned h = head, st = 0;
    unsigned long long wait_ns = 0;   // tracing: time this warp waited for stages to land
    int jc = -1;                      // stage whose ring position st holds
    auto seek = [&](int j) {
        while (jc < j) {
            jc++;
            st = ring_take(h, stage_bytes(cr, jc, K));
        }
    };
    auto land = [&](int c) -> bool {   // warp-uniform wait for stage c
        unsigned long long tw = 0;
        if (tr && !mbar_try_wait(full + c, 0)) tw = g4_globaltimer();
        const bool got = c < kMaxStages &&
                         mbar_wait(full + c, 0, a.err, G4D_TIMEOUT_FULL | ((c & 0xfff) << 8) | ((int)blockIdx.x << 20));
        if (tw) wait_ns += g4_globaltimer() - tw;
        return __all_sync(0xffffffffu, got);
    };

    if (row_parallel(cr)) {
        // ---- row-parallel: warp w takes stages w, w + 8, ...; lane = row ----
        for (int j = warp; j < cr.nst; j += kWarps) {
            seek(j);
            if (!land(cs + j)) {
                if (lane == 0) *fail = 1;
                break;
            }
            const int nr = stage_nr(cr, j);
            const int r = lane < nr ? lane : nr - 1;   // idle lanes re-read the last row
            const float u = epi == EPI_PLE ? a.ple_u[cr.n0 + j * cr.R + r] : 0.0f;
            const uint8_t *sb = ring + st % kRingBytes;
            const uint8_t *wr = sb + (size_t)r * K;
            const uint16_t *sr = (const uint16_t *)(sb + (size_t)nr * K) + r * G;
            float acc = 0.0f;
            for (int g0 = 0; g0 < G; g0 += 4) {
                const uint2 s4 = *(const uint2 *)(sr + g0);
                const float4 x4 = *(const float4 *)(xs + g0);
                int d[4];
#pragma unroll
                for (int k = 0; k < 4; k++) d[k] = group_dot(wr + (g0 + k) * 64, xq + (g0 + k) * 64, lane);
                acc = chain_step(acc, d[0], scale_at(s4, 0), x4.x);
                acc = chain_step(acc, d[1], scale_at(s4, 1), x4.y);
                acc = chain_step(acc, d[2], scale_at(s4, 2), x4.z);
                acc = chain_step(acc, d[3], scale_at(s4, 3), x4.w);
            }
            __syncwarp();
            if (lane == 0) atomicAdd(&done[(cs + j) % kFifo], 1);   // the stage is no longer read
            row_epilogue(a, epi, cr.n0 + j * cr.R + lane, acc, lane < nr, gelu_s, u, best_v, best_i);
        }
    } else {
        // ---- group-parallel: (row, group) dots of every stage spread over all
        // consumer threads into D[g][row]; each warp releases a stage when its
        // share is done; then warp 0 runs the 32-or-fewer rows' chains ----
        int *D = (int *)(smem + kOffScratch + kGemvScratch);
        uint16_t *S = (uint16_t *)vec;   // [rows][G] fp16 scales kept for the chain
        for (int j = 0; j < cr.nst; j++) {
            seek(j);
            const bool ok = land(cs + j);
            if (!ok) {
                if (lane == 0) *fail = 1;
                continue;
            }
            const int nr = stage_nr(cr, j), items = nr * G;
            const uint8_t *sb = ring + st % kRingBytes;
            for (int i = tid; i < items; i += 2 * kConsumers) {
                const int i2 = i + kConsumers;
                const int r1 = i % nr, g1 = i / nr;
                const int r2 = i2 < items ? i2 % nr : r1, g2 = i2 < items ? i2 / nr : g1;
                const int d1 = group_dot(sb + (size_t)r1 * K + g1 * 64, xq + g1 * 64, tid);
                const int d2 = group_dot(sb + (size_t)r2 * K + g2 * 64, xq + g2 * 64, tid);
                D[g1 * 32 + j * cr.R + r1] = d1;
                if (i2 < items) D[g2 * 32 + j * cr.R + r2] = d2;
            }
            const uint16_t *ss = (const uint16_t *)(sb + (size_t)nr * K);
            for (int i = tid; i < items; i += kConsumers) S[j * cr.R * G + i] = ss[i];
            __syncwarp();
            if (lane == 0) atomicAdd(&done[(cs + j) % kFifo], 1);   // this warp no longer reads the stage
        }
        csync();
        if (warp == 0 && cr.rows > 0) {
            const int r = lane < cr.rows ? lane : cr.rows - 1;
            const uint16_t *sr = S + r * G;
            float acc = 0.0f;
            // unrolled so that later groups' loads issue while the chain runs
            // (the chain order itself is unchanged)
#pragma unroll 4
            for (int g = 0; g < G; g += 4) {
                const uint2 s4 = *(const uint2 *)(sr + g);
                const float4 x4 = *(const float4 *)(xs + g);
                acc = chain_step(acc, D[g * 32 + r], scale_at(s4, 0), x4.x);
                acc = chain_step(acc, D[(g + 1) * 32 + r], scale_at(s4, 1), x4.y);
                acc = chain_step(acc, D[(g + 2) * 32 + r], scale_at(s4, 2), x4.z);
                acc = chain_step(acc, D[(g + 3) * 32 + r], scale_at(s4, 3), x4.w);
            }
            row_epilogue(a, epi, cr.n0 + lane, acc, lane < cr.rows, gelu_s, u0, best_v, best_i);
        }
    }
    // every warp leaves with the ring position after the op's last stage
    seek(cr.nst - 1);
    head = h;
    if (tr && lane == 0) atomicMax(tr + 3, wait_ns);
    if (epi == EPI_LOGITS) {
        // first strict maximum (gemma4.c:537-541): per lane, per warp, per CTA, then last CTA
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
            if (ov > best_v || (ov == best_v && oi < best_i)) { best_v = ov; best_i = oi; }
        }
        float *cv = red;
        int *ci = (int *)(red + 64);
        if (lane == 0) {
            cv[warp] = best_v;
            ci[warp] = best_i;
        }
        csync();
        __shared__ unsigned last;
        if (tid == 0) {
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int k = 0; k < kWarps; k++)
                if (cv[k] > bv || (cv[k] == bv && ci[k] < bi)) { bv = cv[k]; bi = ci[k]; }
            a.argmax_part[(size_t)blockIdx.x * 2] = bv;
            a.argmax_part[(size_t)blockIdx.x * 2 + 1] = __int_as_float(bi);
            __threadfence();
            last = atomicAdd(a.ticket, 1u) == gridDim.x - 1;
        }
        csync();
        if (last && tid == 0) {
            __threadfence();
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int k = 0; k < (int)gridDim.x; k++) {
                const float v = __ldcg(&a.argmax_part[(size_t)k * 2]);
                const int ix = __float_as_int(__ldcg(&a.argmax_part[(size_t)k * 2 + 1]));
                if (v > bv || (v == bv && ix < bi)) { bv = v; bi = ix; }
            }
            a.argmax_out[0] = bi;
            *a.ticket = 0u;
        }
    }
}

G4_DEV void run_gemv(const DecodeOp &op, int cs, unsigned &head, uint8_t *smem, volatile int *fail,
                     unsigned long long *tr) {
    const GemvArgs &a = op.g;
    const bool pro_ok = op.pro == PRO_EMBED_QUANT || op.pro == PRO_NORM_QUANT || op.pro == PRO_RES_NORM_QUANT ||
                        op.pro == PRO_LOADQ || op.pro == PRO_QUANT || op.pro == PRO_RES_QUANT;
    const bool epi_ok = op.epi == EPI_STORE || op.epi == EPI_GEGLU_PAIR || op.epi == EPI_PLE || op.epi == EPI_LOGITS;
    if (pro_ok && epi_ok) return gemv_op(a, cta_rows(op), op.pro, op.epi, cs, head, smem, fail, tr);
    g4_set_error(a.err, G4D_BAD_SHAPE);
    if (threadIdx.x == 0) *fail = 1;
}

// u[l][:] = (rmsnorm(pli[l][:], w, eps) + ple_emb[l][:]) * scale, CTA l (gemma4.c:474-477)
G4_DEV void ple_prep_op(const DecodeOp &op, float *red) {
    const int l = blockIdx.x;
    if (l >= G4_NUM_LAYERS) return;
    const int i = threadIdx.x;   // 256 consumers = 256 values
    const float x = op.pli[l * G4_PLE + i];
    const float ss = block_sum(__fmul_rn(x, x), red);
    const float y = rms_apply(x, rms_inv(ss, (float)G4_PLE, op.ple_eps), op.ple_norm[i]);
    op.ple_u[l * G4_PLE + i] = __fmul_rn(__fadd_rn(y, op.ple_emb[l * G4_PLE + i]), op.ple_scale);
}

// res_out = (res_in + rmsnorm(h, w)) * scalar for the one token row (CTA 0; gemma4.c:505-506)
G4_DEV void finish_op(const DecodeOp &op, float *red) {
    if (blockIdx.x != 0) return;
    constexpr int PER = G4_HIDDEN / kConsumers;
    const int tid = threadIdx.x;
    float v[PER];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < PER; i++) {
        v[i] = op.fin_h[tid + i * kConsumers];
        ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
    }
    ss = block_sum(ss, red);
    const float inv = rms_inv(ss, (float)G4_HIDDEN, G4_RMS_EPS);
    const float sc = op.fin_scalar ? *op.fin_scalar : 1.0f;
#pragma unroll
    for (int i = 0; i < PER; i++) {
        const int e = tid + i * kConsumers;
        float r = __fadd_rn(op.fin_res_in[e], rms_apply(v[i], inv, op.fin_w[e]));
        if (op.fin_scalar) r = __fmul_rn(r, sc);
        op.fin_res_out[e] = r;
    }
}

// Producer lane: every GEMV stage of the step, in op order.
G4_DEV void produce(const DecodeParams &P, uint8_t *smem, volatile int *fail, int *issued) {
    constexpr int TW = 6;
    uint8_t *ring = smem + kOffRing;
    uint64_t *full = (uint64_t *)(smem + kOffFull);
    volatile int *done = (volatile int *)(smem + kOffDone);
    uint2 *fifo = (uint2 *)(smem + kOffFifo);   // stage c % kFifo: (ring end, pairs)
    const uint64_t pol = l2_policy_evict_first();
    unsigned head = 0, tail = 0;   // monotonic ring positions: next free byte, end of released space
    int cs = 0, oldest = 0;        // next stage to issue, oldest stage not yet released
    if (P.starve) {                // test aid: nothing is issued, every stage wait runs out
        *issued = 0;
        return;
    }
    for (int o = 0; o < P.nops && !*fail; o++) {
        const DecodeOp &op = P.ops[o];
        if (op.type != OP_GEMV) continue;
        const DMat &m = op.g.m;
        const int K = m.K, G = K >> 6;
        const CtaRows cr = cta_rows(op);
        for (int j = 0; j < cr.nst; j++, cs++) {
            if (cs >= kMaxStages) {
                g4_set_error(P.err, G4D_BAD_SHAPE);
                *fail = 1;
                *issued = cs;
                return;
            }
            const unsigned sz = stage_bytes(cr, j, K);
            const unsigned start = ring_take(head, sz);
            // free space in stage order until [start, start + sz) is released
            while (head - tail > kRingBytes || cs - oldest >= kFifo) {
                const uint2 f = fifo[oldest % kFifo];
                volatile int *d = done + oldest % kFifo;
                if (*d != (int)f.y) {
                    const uint64_t t0 = g4_globaltimer();
                    while (*d != (int)f.y) {
                        if (g4_globaltimer() - t0 > G4_WAIT_NS) {
                            g4_set_error(P.err, G4D_TIMEOUT_EMPTY | ((cs & 0xfff) << 8) | ((int)blockIdx.x << 20));
                            *fail = 1;
                            *issued = cs;
                            return;
                        }
                    }
                }
                *d = 0;
                tail = f.x;
                oldest++;
            }
            const int nr = stage_nr(cr, j), r0 = cr.n0 + j * cr.R;
            fifo[cs % kFifo] = make_uint2(head, stage_releases(cr));
            uint8_t *dst = ring + start % kRingBytes;
            mbar_arrive_expect_tx(&full[cs], sz);
            bulk_g2s(dst, m.w + (size_t)r0 * K, (uint32_t)(nr * K), &full[cs], pol);
            bulk_g2s(dst + nr * K, m.s + (size_t)r0 * G, (uint32_t)(nr * G * 2), &full[cs], pol);
            if (P.trace && (j == 0 || j == cr.nst - 1))
                atomicMax(P.trace + 1 + TW * o + (j == 0 ? 4 : 5), (unsigned long long)g4_globaltimer());
        }
    }
    *issued = cs;
}

__global__ void __launch_bounds__(kThreads, 1) k_decode(const DecodeParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = (uint64_t *)(smem + kOffFull);
    int *done = (int *)(smem + kOffDone);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // a step queued behind a failed one does nothing (its barrier counters are
    // stale until the host reads the error and resets them)
    if (*(volatile int *)P.err) return;

    // The host sizes the step to at most kMaxStages stages per CTA
    // (g4_decode_max_stages); producer and consumers check it again per stage.
    __shared__ int fail, issued;   // a wait ran out; stages the producer issued
    for (int i = tid; i < kMaxStages; i += kThreads) mbar_init(&full[i], 1);
    if (tid < kFifo) done[tid] = 0;
    if (tid == 0) {
        fail = 0;
        issued = 0;
    }
    mbar_fence_init();
    __syncthreads();

    if (warp == kWarps) {
        // ---------------- producer ----------------
        if (lane == 0) produce(P, smem, &fail, &issued);
        __syncwarp();
        bar_sync(2, kThreads);   // join the consumers (end of the kernel)
        if (lane == 0 && fail) drain_stages(full, issued);
        return;
    }

    // ---------------- consumers ----------------
    // Op descriptors are read from shared memory: the next op's is copied in
    // (cp.async) while the current op runs, so no op starts with a memory
    // round trip for its own arguments. The position is read once.
    const unsigned long long base = *P.bar_base;
    const int pos = *P.pos;
    unsigned long long target = base;
    float *scratch = (float *)(smem + kOffScratch);
    float *red = (float *)(smem + kOffRed);
    DecodeOp *opbuf = (DecodeOp *)(smem + kOffOps);
    auto fetch_op = [&](int o) {
        if (tid < kOpWords)
            cp_async16((uint8_t *)&opbuf[o & 1] + tid * 16, (const uint8_t *)&P.ops[o] + tid * 16);
        cp_async_commit();
    };
    fetch_op(0);
    cp_async_wait<0>();
    csync();
    bool ok = true;
    int cs = 0;
    unsigned head = 0;
    if (P.trace && tid == 0) atomicMax(P.trace, (unsigned long long)g4_globaltimer());
    for (int o = 0; o < P.nops && ok; o++) {
        // op o's descriptor is in place (waited for before the barrier that ended
        // op o - 1); op o - 1's buffer is free for op o + 1's
        if (o + 1 < P.nops) fetch_op(o + 1);
        const DecodeOp &op = opbuf[o & 1];
        unsigned long long *tr = P.trace ? P.trace + 1 + 6 * o : nullptr;
        switch (op.type) {
        case OP_GEMV:
            run_gemv(op, cs, head, smem, &fail, tr);
            cs += cta_rows(op).nst;
            break;
        case OP_ATTN:
            if ((int)blockIdx.x < P.splits) {
                if (op.at.hd == 256) attn_decode_split<256, kKT256>(op.at, pos, blockIdx.x, P.splits, scratch);
                else attn_decode_split<512, kKT512>(op.at, pos, blockIdx.x, P.splits, scratch);
            }
            break;
        case OP_COMBINE:
            if ((int)blockIdx.x < kHeads * op.at.hd / kCombineDims) {
                if (op.at.hd == 256)
                    attn_combine_part<256>(op.at, pos, blockIdx.x, P.splits, scratch, op.at.part, op.at.out, op.at.xq,
                                           op.at.xs);
                else
                    attn_combine_part<512>(op.at, pos, blockIdx.x, P.splits, scratch, op.at.part, op.at.out, op.at.xq,
                                           op.at.xs);
            }
            break;
        case OP_PLE_PREP: ple_prep_op(op, red); break;
        case OP_FINISH: finish_op(op, red); break;
        default:
            if (tid == 0) fail = 1;   // unknown op type (uniform: every thread reads the same op)
        }
        cp_async_wait<0>();   // this thread's share of op o + 1's descriptor landed
        if (op.barrier) {
            target += gridDim.x;
            ok = grid_barrier(P, target, &fail, tr);
        } else {
            csync();
            if (tr && tid == 0) {
                const unsigned long long t = g4_globaltimer();
                atomicMax(tr + 1, t);
                atomicMax(tr + 2, t);
            }
        }
    }
    csync();
    ok = ok && !fail;
    // the next launch starts from the final count
    if (ok && blockIdx.x == 0 && tid == 0) *P.bar_base = target;
    bar_sync(2, kThreads);   // all 288 threads: then the producer lane drains in-flight copies on failure
}

}  // namespace

size_t g4_decode_smem_bytes() { return (size_t)kSmemBytes; }

void g4_decode_set_partition(DecodeOp &op, int grid) { set_partition(op, grid); }

int g4_decode_max_stages(const DecodeOp *ops, int nops, int grid) {
    int worst = 0;
    for (int b = 0; b < grid; b++) {
        int total = 0;
        for (int o = 0; o < nops; o++) {
            if (ops[o].type != OP_GEMV) continue;
            const DMat &m = ops[o].g.m;
            DecodeOp pop = ops[o];
            set_partition(pop, grid);
            const CtaRows cr = cta_rows_of(pop, b);
            // group-parallel CTAs keep all their rows' scales ([rows][G] fp16) in 6 KB
            if ((size_t)cr.R * m.K + (size_t)cr.R * (m.K / 64) * 2 > kRingBytes / 2 || m.K > kMaxK ||
                (!row_parallel(cr) && (size_t)cr.rows * (m.K / 64) * 2 > (size_t)G4_HIDDEN * 4))
                return 1 << 30;
            total += cr.nst;
        }
        worst = total > worst ? total : worst;
    }
    return worst <= kMaxStages ? worst : 1 << 30;
}

cudaError_t g4_launch_decode(const DecodeParams &p, int grid, cudaStream_t st) {
    {
        cudaError_t e = g4_smem_optin((const void *)k_decode, kSmemBytes);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_decode, p);
}
