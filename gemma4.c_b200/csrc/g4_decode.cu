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
// op reads what the previous one wrote. The producer warp streams this CTA's
// weight slices of EVERY GEMV of the step, in op order, through one ring of
// TMA bulk-copy stages; it only waits for free ring slots, never for barriers,
// so the HBM stream runs on while consumers sit in barriers, attention or
// prologues. Each stage has its own single-use mbarrier; a slot is released
// when the consumers have finished every row pair of its stage.
//
// The arithmetic is the standalone kernels' (g4_gemv_dev.cuh,
// g4_attn_dev.cuh): same exact int32 dots, same ordered dequant chains.
#include "g4_attn_dev.cuh"
#include "g4_gemv_dev.cuh"

namespace {

constexpr int kThreads = kConsumers + 32;
constexpr int kSlots = 4;
constexpr int kSlotBytes = 24576;          // largest stage: 2 rows x 12288
constexpr int kSSlotBytes = 1024;          // largest stage's scales
constexpr int kMaxStages = 1536;           // single-use stage barriers per step
constexpr int kMaxK = 12288;
constexpr int kKT256 = DecodeKT<256>::value, kKT512 = DecodeKT<512>::value;

__host__ __device__ constexpr int cmax(int a, int b) { return a > b ? a : b; }
constexpr int kAttnFloats = cmax(decode_smem_floats(256, kKT256), decode_smem_floats(512, kKT512));
constexpr int kGemvScratch = kMaxK + (kMaxK / 64) * 4 + G4_HIDDEN * 4;   // xq + xs + vec bytes
constexpr int kScratchBytes = cmax(kAttnFloats * 4, kGemvScratch);

constexpr int kOffRing = 0;
constexpr int kOffSRing = kOffRing + kSlots * kSlotBytes;
constexpr int kOffFull = kOffSRing + kSlots * kSSlotBytes;
constexpr int kOffEmpty = kOffFull + kMaxStages * 8;
constexpr int kOffDone = kOffEmpty + kSlots * 8;
constexpr int kOffScratch = (kOffDone + kSlots * 4 + 127) / 128 * 128;
constexpr int kOffRed = kOffScratch + kScratchBytes;
constexpr int kSmemBytes = kOffRed + 512 * 4;

G4_DEV unsigned long long ld_acquire_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Grid-wide barrier among the consumer warps of all CTAs (bounded wait). A CTA
// whose op failed (fail != 0: a stage that never arrived) does not arrive; the
// others then give up after the bounded wait. Returns the same value to every
// consumer thread of the CTA.
// tr (tracing only): [1] <- latest time a CTA finished the op, [2] <- latest barrier exit.
G4_DEV bool grid_barrier(const DecodeParams &P, unsigned long long target, const volatile int *fail,
                         unsigned long long *tr) {
    csync();
    __shared__ int ok;
    if (threadIdx.x == 0 && tr) atomicMax(tr + 1, (unsigned long long)g4_globaltimer());
    if (threadIdx.x == 0 && *fail) ok = 0;
    if (threadIdx.x == 0 && !*fail) {
        ok = 1;
        __threadfence();
        atomicAdd(P.bar, 1ull);
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
        __threadfence();
        if (tr) atomicMax(tr + 2, (unsigned long long)g4_globaltimer());
    }
    csync();
    return ok != 0;
}

struct CtaRows {
    int n0, rows, R, nst;
};
G4_DEV CtaRows cta_rows(const DMat &m) {
    CtaRows c;
    const int npairs = m.N >> 1;
    const int c0 = (int)((long long)blockIdx.x * npairs / gridDim.x);
    const int c1 = (int)((long long)(blockIdx.x + 1) * npairs / gridDim.x);
    c.n0 = 2 * c0;
    c.rows = 2 * (c1 - c0);
    c.R = stage_rows(m.K);
    c.nst = (c.rows + c.R - 1) / c.R;
    return c;
}

// One GEMV op, consumer side. cs: this op's first stage index. A warp whose
// stage wait runs out leaves the row loop as a whole warp and sets *fail; it
// still takes every consumer barrier below, so the CTA never deadlocks.
template <int PRO, int EPI>
G4_DEV void gemv_op(const GemvArgs &a, int cs, uint8_t *smem, volatile int *fail, unsigned long long *tr) {
    const int K = a.m.K, G = K >> 6;
    uint8_t *ring = smem + kOffRing;
    uint8_t *sring = smem + kOffSRing;
    uint64_t *full = (uint64_t *)(smem + kOffFull);
    uint64_t *empty = (uint64_t *)(smem + kOffEmpty);
    int *done = (int *)(smem + kOffDone);
    int8_t *xq = (int8_t *)(smem + kOffScratch);
    float *xs = (float *)(smem + kOffScratch + kMaxK);
    float *vec = (float *)(smem + kOffScratch + kMaxK + (kMaxK / 64) * 4);
    float *red = (float *)(smem + kOffRed);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, half = lane >> 4, q = lane & 15;

    prologue<1, PRO>(a, xq, xs, vec, red);
    csync();
    if (tr && tid == 0) atomicMax(tr, (unsigned long long)g4_globaltimer());
    const CtaRows cr = cta_rows(a.m);
    const int PPS = cr.R / 2;
    float best_v = -INFINITY;
    int best_i = 0x7fffffff;
    for (int pr = warp; pr < cr.rows / 2; pr += kWarps) {
        const int j = pr / PPS, c = cs + j, slot = c % kSlots;
        const int lr = 2 * (pr - j * PPS) + half;
        const int n = cr.n0 + j * cr.R + lr;
        const bool got = mbar_wait(full + c, 0, a.err, G4D_TIMEOUT_FULL | ((c & 0xfff) << 8) | ((int)blockIdx.x << 20));
        if (!__all_sync(0xffffffffu, got)) {
            if (lane == 0) *fail = 1;
            break;
        }
        float acc[1];
        pair_dot<1>(ring + slot * kSlotBytes + lr * K + q * 16, (const uint16_t *)(sring + slot * kSSlotBytes) + lr * G,
                    xq, xs, K, acc, nullptr, 0);
        __syncwarp();
        if (lane == 0) {
            const int pairs = min(cr.R, cr.rows - j * cr.R) / 2;
            if (atomicAdd(&done[slot], 1) + 1 == pairs) {
                done[slot] = 0;
                mbar_arrive(&empty[slot]);
            }
        }
        const float up = __shfl_sync(0xffffffffu, acc[0], 16);
        epilogue_row<EPI>(a, 0, n, acc[0], up, q == 0, best_v, best_i);
    }
    if (EPI == EPI_LOGITS) {
        float *cv = red;
        int *ci = (int *)(red + 64);
        if (q == 0) {
            cv[warp * 2 + half] = best_v;
            ci[warp * 2 + half] = best_i;
        }
        csync();
        __shared__ unsigned last;
        if (tid == 0) {
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int k = 0; k < kWarps * 2; k++)
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

G4_DEV void run_gemv(const DecodeOp &op, int cs, uint8_t *smem, volatile int *fail, unsigned long long *tr) {
    const GemvArgs &a = op.g;
#define G4_OP(P, E) \
    if (op.pro == P && op.epi == E) return gemv_op<P, E>(a, cs, smem, fail, tr);
    G4_OP(PRO_EMBED_QUANT, EPI_STORE)
    G4_OP(PRO_NORM_QUANT, EPI_STORE)
    G4_OP(PRO_RES_NORM_QUANT, EPI_STORE)
    G4_OP(PRO_LOADQ, EPI_STORE)
    G4_OP(PRO_RES_NORM_QUANT, EPI_GEGLU_PAIR)
    G4_OP(PRO_QUANT, EPI_STORE)
    G4_OP(PRO_RES_QUANT, EPI_PLE)
    G4_OP(PRO_RES_NORM_QUANT, EPI_LOGITS)
#undef G4_OP
    g4_set_error(a.err, G4D_BAD_SHAPE);
    *fail = 1;
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

__global__ void __launch_bounds__(kThreads, 1) k_decode(const DecodeParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = (uint64_t *)(smem + kOffFull);
    uint64_t *empty = (uint64_t *)(smem + kOffEmpty);
    int *done = (int *)(smem + kOffDone);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // a step queued behind a failed one does nothing (its barrier counters are
    // stale until the host reads the error and resets them)
    if (*(volatile int *)P.err) return;

    // stages this CTA streams in the whole step
    int total = 0;
    for (int o = 0; o < P.nops; o++)
        if (P.ops[o].type == OP_GEMV) total += cta_rows(P.ops[o].g.m).nst;
    if (total > kMaxStages) {
        if (tid == 0) g4_set_error(P.err, G4D_BAD_SHAPE);
        return;
    }
    __shared__ int fail, issued;   // a wait ran out; stages the producer issued
    for (int i = tid; i < total; i += kThreads) mbar_init(&full[i], 1);
    if (tid < kSlots) {
        mbar_init(&empty[tid], 1);
        done[tid] = 0;
    }
    if (tid == 0) {
        fail = 0;
        issued = 0;
    }
    mbar_fence_init();
    __syncthreads();

    if (warp == kWarps) {
        // ---------------- producer: every GEMV slice of the step, in op order ----------------
        if (lane == 0) {
            const uint64_t pol = l2_policy_evict_first();
            int cs = 0;
            for (int o = 0; o < P.nops && !*(volatile int *)&fail; o++) {
                const DecodeOp &op = P.ops[o];
                if (op.type != OP_GEMV) continue;
                const DMat &m = op.g.m;
                const int K = m.K, G = K >> 6;
                const CtaRows cr = cta_rows(m);
                for (int j = 0; j < cr.nst; j++, cs++) {
                    const int slot = cs % kSlots, use = cs / kSlots;
                    if (use > 0 && !mbar_wait(&empty[slot], (use - 1) & 1, P.err,
                                              G4D_TIMEOUT_EMPTY | ((cs & 0xfff) << 8) | ((int)blockIdx.x << 20))) {
                        fail = 1;
                        break;
                    }
                    const int r0 = cr.n0 + j * cr.R, nr = min(cr.R, cr.rows - j * cr.R);
                    mbar_arrive_expect_tx(&full[cs], (uint32_t)(nr * K + nr * G * 2));
                    bulk_g2s(smem + kOffRing + slot * kSlotBytes, m.w + (size_t)r0 * K, (uint32_t)(nr * K), &full[cs],
                             pol);
                    bulk_g2s(smem + kOffSRing + slot * kSSlotBytes, m.s + (size_t)r0 * G, (uint32_t)(nr * G * 2),
                             &full[cs], pol);
                }
            }
            issued = cs;   // stages whose copies were issued
        }
        __syncwarp();
        bar_sync(2, kThreads);   // join the consumers (end of the kernel)
        if (lane == 0 && fail) drain_stages(full, issued);
        return;
    }

    // ---------------- consumers ----------------
    const unsigned long long base = *P.bar_base;
    unsigned long long target = base;
    float *scratch = (float *)(smem + kOffScratch);
    float *red = (float *)(smem + kOffRed);
    bool ok = true;
    int cs = 0;
    if (P.trace && tid == 0) atomicMax(P.trace, (unsigned long long)g4_globaltimer());
    for (int o = 0; o < P.nops && ok; o++) {
        const DecodeOp &op = P.ops[o];
        unsigned long long *tr = P.trace ? P.trace + 1 + 3 * o : nullptr;
        switch (op.type) {
        case OP_GEMV:
            run_gemv(op, cs, smem, &fail, tr);
            cs += cta_rows(op.g.m).nst;
            break;
        case OP_ATTN:
            if ((int)blockIdx.x < P.splits) {
                if (op.at.hd == 256) attn_decode_split<256, kKT256>(op.at, blockIdx.x, P.splits, scratch);
                else attn_decode_split<512, kKT512>(op.at, blockIdx.x, P.splits, scratch);
            }
            break;
        case OP_COMBINE:
            if ((int)blockIdx.x < kHeads * op.at.hd / 256) {
                if (op.at.hd == 256) attn_combine_part<256>(op.at, blockIdx.x, P.splits, scratch);
                else attn_combine_part<512>(op.at, blockIdx.x, P.splits, scratch);
            }
            break;
        case OP_PLE_PREP: ple_prep_op(op, red); break;
        case OP_FINISH: finish_op(op, red); break;
        default:
            if (tid == 0) fail = 1;   // unknown op type (uniform: every thread reads the same op)
        }
        if (op.barrier) {
            target += gridDim.x;
            ok = grid_barrier(P, target, &fail, tr);
        } else if (tr) {
            csync();
            if (tid == 0) {
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

int g4_decode_max_stages(const DecodeOp *ops, int nops, int grid) {
    int worst = 0;
    for (int b = 0; b < grid; b++) {
        int total = 0;
        for (int o = 0; o < nops; o++) {
            if (ops[o].type != OP_GEMV) continue;
            const DMat &m = ops[o].g.m;
            const int npairs = m.N / 2;
            const int c0 = (int)((long long)b * npairs / grid), c1 = (int)((long long)(b + 1) * npairs / grid);
            const int rows = 2 * (c1 - c0), R = stage_rows(m.K);
            if (R * m.K > kSlotBytes || R * (m.K / 64) * 2 > kSSlotBytes || m.K > kMaxK) return 1 << 30;
            total += (rows + R - 1) / R;
        }
        worst = total > worst ? total : worst;
    }
    return worst <= kMaxStages ? worst : 1 << 30;
}

cudaError_t g4_launch_decode(const DecodeParams &p, int grid, cudaStream_t st) {
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(k_decode, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        if (e != cudaSuccess) return e;
        configured = true;
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
