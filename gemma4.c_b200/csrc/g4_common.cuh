// g4_common.cuh — device helpers shared by every g4cuda kernel (sm_100a only).
//
// Conventions:
//   - Bit-exactness: the reference is built -std=c11, so no a*b+c contraction;
//     every place whose rounding must match uses the explicit __f*_rn
//     intrinsics, and FMAs appear only where the reference uses FMA intrinsics.
//   - Every spin (mbarrier waits, tickets) is bounded by a %globaltimer budget;
//     on expiry the kernel records an error code in the context's device error
//     word and returns, leaving the CUDA context usable.
//   - Kernels are launched with programmatic dependent launch: anything that
//     reads the previous kernel's output sits after griddep_wait().
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#ifndef __CUDACC__
#error "g4_common.cuh is CUDA-only"
#endif

#define G4_DEV __device__ __forceinline__


// ~2 s wall budget for any single wait.
#define G4_WAIT_NS 2000000000ull

G4_DEV uint64_t g4_globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

G4_DEV void g4_set_error(int *err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// ---- programmatic dependent launch --------------------------------------
G4_DEV void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
G4_DEV void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- mbarrier + bulk async copy (TMA engine, 1-D) ------------------------
G4_DEV uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

G4_DEV void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
G4_DEV void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

G4_DEV void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
G4_DEV void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
G4_DEV bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait on phase `parity`; returns false (and records `code`) on timeout.
G4_DEV bool mbar_wait(uint64_t *bar, uint32_t parity, int *err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = g4_globaltimer();
    while (!mbar_try_wait(bar, parity)) {
        if (g4_globaltimer() - t0 > G4_WAIT_NS) {
            g4_set_error(err, code);
            return false;
        }
    }
    return true;
}

// After a failed wait: give the bulk copies this CTA issued (stages
// [0, issued), one single-use barrier each) time to land, bounded by one
// overall deadline, so that none still writes shared memory when the CTA exits.
G4_DEV void drain_stages(uint64_t *full, int issued) {
    const uint64_t t0 = g4_globaltimer();
    for (int c = 0; c < issued; c++)
        while (!mbar_try_wait(&full[c], 0))
            if (g4_globaltimer() - t0 > G4_WAIT_NS) return;
}

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes, 16-B multiples,
// both addresses 16-B aligned). Weights are streamed once per token, so they are
// marked evict-first in L2.
G4_DEV void bulk_g2s(void *dst_smem, const void *src_gmem, uint32_t bytes, uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
G4_DEV uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
G4_DEV uint64_t l2_policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Named barrier among the first `threads` threads (consumer warps only).
G4_DEV void bar_sync(int id, int threads) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory"); }

// ---- exact integer / float helpers --------------------------------------
G4_DEV int dp4a(uint32_t a, uint32_t b, int c) { return __dp4a((int)a, (int)b, c); }

G4_DEV float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// gemma4.c:265-279: scale = max|x| / 127 (IEEE divide), inv = 1/scale,
// q = rintf(x * inv) (round-half-even), zero group -> scale 0, q 0.
G4_DEV float quant_scale(float amax) { return __fdiv_rn(amax, 127.0f); }
G4_DEV float quant_inv(float scale) { return scale > 0.0f ? __frcp_rn(scale) : 0.0f; }
G4_DEV int quant_one(float x, float inv) { return __float2int_rn(__fmul_rn(x, inv)); }

// gemma4.c:360-373 rmsnorm tail: inv_rms = 1 / sqrtf(ss / n + eps);
// out = w * (inv_rms * x). The sum of squares itself is reduced in parallel,
// so only this tail is bit-exact.
G4_DEV float rms_inv(float ss, float width, float eps) {
    return __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(ss, width), eps)));
}
G4_DEV float rms_apply(float x, float inv, float w) { return __fmul_rn(w, __fmul_rn(inv, x)); }

// gemma4.c:310-331 geglu element: LUT GELU with linear interpolation, times up.
G4_DEV float geglu_one(float x, float up, const float *__restrict__ table, int size, float lo, float hi, float scale) {
    if (x <= lo) {
        x = table[0];
    } else if (!(x >= hi)) {
        float pos = __fmul_rn(__fsub_rn(x, lo), scale);
        int idx = (int)pos;
        float frac = __fsub_rn(pos, (float)idx);
        float t0 = table[idx];
        float t1 = idx + 1 < size ? table[idx + 1] : t0;
        x = __fadd_rn(t0, __fmul_rn(frac, __fsub_rn(t1, t0)));
    }
    return __fmul_rn(x, up);
}

// ---- strict (reference-order) arithmetic ----------------------------------
// The reference sums squares sequentially (gemma4.c:367-368: product rounded,
// then added). Strict mode reproduces that order with one thread.
G4_DEV float seq_sumsq(const float *x, int n) {
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
    return ss;
}

// expf with the results of the host C library the reference links (glibc
// 2.39): the published table-driven method (x * 32/ln2 split into k + r,
// 2^(k/32) from a 32-entry table of doubles, degree-3 polynomial in r, one
// rounding to float), evaluated in IEEE double with no contraction. Checked
// exhaustively against the host expf over every float in [-104, 88.7]; the two
// inputs where the host returns the other neighbour of the exact value are
// listed explicitly.
__device__ __constant__ uint64_t g4_exp2_tab[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull,
};

G4_DEV float expf_host(float x) {
    const uint32_t ux = __float_as_uint(x);
    const uint32_t abstop = (ux >> 20) & 0x7ffu;
    if (abstop >= 0x42bu) {                                   // |x| >= 88 or not finite
        if (ux == 0xff800000u) return 0.0f;                   // -inf
        if (abstop >= 0x7f8u) return x + x;                   // nan, +inf
        if (x > 0x1.62e42ep6f) return __int_as_float(0x7f800000);   // overflow
        if (x < -0x1.9fe368p6f) return 0.0f;                  // underflow
    }
    if (ux == 0xc27c65d9u) return 0x1.f45326p-92f;             // x = -0x1.f8cbb2p+5
    if (ux == 0x4202422fu) return 0x1.f93e38p+46f;             // x =  0x1.04845ep+5
    const double inv_ln2_n = 0x1.71547652b82fep+0 * 32.0;
    const double shift = 0x1.8p+52;
    const double c0 = 0x1.c6af84b912394p-5 / 32.0 / 32.0 / 32.0;
    const double c1 = 0x1.ebfce50fac4f3p-3 / 32.0 / 32.0;
    const double c2 = 0x1.62e42ff0c52d6p-1 / 32.0;
    const double z = __dmul_rn(inv_ln2_n, (double)x);
    double kd = __dadd_rn(z, shift);
    const uint64_t ki = (uint64_t)__double_as_longlong(kd);
    kd = __dsub_rn(kd, shift);
    const double r = __dsub_rn(z, kd);
    const uint64_t t = g4_exp2_tab[ki & 31u] + (ki << 47);
    const double s = __longlong_as_double((long long)t);
    const double zz = __dadd_rn(__dmul_rn(c0, r), c1);
    const double r2 = __dmul_rn(r, r);
    double y = __dadd_rn(__dmul_rn(c2, r), 1.0);
    y = __dadd_rn(__dmul_rn(zz, r2), y);
    y = __dmul_rn(y, s);
    return __double2float_rn(y);
}

// Packed pairs of fp32 (two independent IEEE round-to-nearest operations per
// instruction, so each lane of the pair rounds exactly like fmul/fmaf).
G4_DEV uint64_t pk(float x, float y) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(x), "f"(y));
    return r;
}
G4_DEV float2 upk(uint64_t v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
G4_DEV uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
G4_DEV uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
// ---- reductions -----------------------------------------------------------
G4_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
G4_DEV float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
