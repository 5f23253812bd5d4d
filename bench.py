#!/usr/bin/env python3
"""Benchmark of the gemma4.c forward path on B200 (libg4cuda.so).

Headline (one JSON line on rank 0): decode tok/s at context 512, the
reference's `./run --bench 512 128` decode figure (the reference's README.md:76) — one step is
one token: forward(1 token) + logits, on the synthetic Gemma 4 E2B model of
benchmark config 1 (random-init weights in gemma4.c's .bin layout, seed 0; the
real checkpoint is not available). Alongside: prefill tok/s at 512 and 16384,
decode tok/s at 16384, the HBM roofline of the decode step kernel, the int8
tensor-core roofline of the prefill GEMM, and the reference CPU path timed on
this host.

  python bench.py [--gpus N] [--steps K] [--warmup W]        # our CUDA path
  python bench.py --impl reference [...]                     # the reference's CPU path
  torchrun --nproc-per-node N bench.py --gpus N ...          # N replicas (weak scaling)

value: device-resident decode — the step's token is already in device memory
(g4_forward copies 8 bytes per step; the same fixed token id the reference
benchmark feeds, gemma4.c:637-641) and logits are enqueued without readback;
K steps timed with CUDA events on the library's stream between barriers, max
over ranks. e2e: the greedy generation loop through the public C ABI — token
id host->device, forward, logits with argmax device->host, next token from the
argmax — every step.
"""
import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "gemma4.c_b200"))

PUBLISHED_DECODE_512 = 25.16   # the reference's README.md:76: tg128 @ d512, Ryzen 7 7700, 8 threads
INT8_DENSE_TOPS = 4500.0       # B200 datasheet dense int8 (reported beside the measured peak)
# prefill GEMM shapes of one token through the model: (N, K, count) over the 35 layers
# + per_layer_model_projection; lm_head is not part of a prefill chunk
PREFILL_SHAPES = ((2560, 1536, 12), (5120, 1536, 3), (2048, 1536, 16), (4096, 1536, 4),
                  (1536, 2048, 28), (1536, 4096, 7), (12288, 1536, 15), (24576, 1536, 20),
                  (1536, 6144, 15), (1536, 12288, 20), (256, 1536, 35), (1536, 256, 35), (8960, 1536, 1))
# benchmark config 2: every projection shape of one layer (both head widths and
# MLP widths), the fused shapes the engine streams, and the lm_head
GEMV_SHAPES = (("q_sliding", 2048, 1536), ("q_global", 4096, 1536), ("kv_sliding", 256, 1536),
               ("kv_global", 512, 1536), ("qkv_fused_sliding", 2560, 1536), ("o_sliding", 1536, 2048),
               ("o_global", 1536, 4096), ("gate_up_6144", 6144, 1536), ("gate_up_12288", 12288, 1536),
               ("gate_up_fused_24576", 24576, 1536), ("down_6144", 1536, 6144), ("down_12288", 1536, 12288),
               ("ple_gate", 256, 1536), ("ple_proj", 1536, 256), ("per_layer_model_proj", 8960, 1536),
               ("lm_head", 262144, 1536))
# benchmark config 3: the projection shapes of one layer on the tensor cores
GEMM_SHAPES = (("qkv_sliding", 2560, 1536), ("q_global", 4096, 1536), ("o_sliding", 1536, 2048),
               ("gate_up_12288", 12288, 1536), ("gate_up_24576", 24576, 1536), ("down_6144", 1536, 6144),
               ("down_12288", 1536, 12288), ("ple_gate", 256, 1536), ("ple_proj", 1536, 256))
PREFILL = 512
CTX_LONG = 16384
# nominal FP32 FMA peak: 148 SMs x 128 lanes x 2 FLOP x 1.965 GHz (no measured figure on this pool)
FP32_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12
ATTN_CTX = (512, 2048, 8192, 16384)


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


class Dist:
    """Process-group plumbing for N replicas: barrier and max over ranks."""

    def __init__(self):
        self.rank, self.world, self.local = env_int("RANK", 0), env_int("WORLD_SIZE", 1), env_int("LOCAL_RANK", 0)
        self.pg = None
        if self.world > 1:
            import datetime

            import torch
            import torch.distributed as dist
            self.torch, self.dist = torch, dist
            backend = "nccl" if torch.cuda.is_available() else "gloo"
            if backend == "nccl":
                torch.cuda.set_device(self.local)
            kw = {"device_id": torch.device("cuda", self.local)} if backend == "nccl" else {}
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120), **kw)
            self.backend = backend
            self.pg = True

    def barrier(self):
        if self.pg:
            self.dist.barrier()

    def max(self, v):
        if not self.pg:
            return v
        t = self.torch.tensor([float(v)], dtype=self.torch.float64,
                              device="cuda" if self.backend == "nccl" else "cpu")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def gather(self, v):
        """[v of rank 0, v of rank 1, ...] on every rank."""
        if not self.pg:
            return [float(v)]
        t = self.torch.zeros(self.world, dtype=self.torch.float64,
                             device="cuda" if self.backend == "nccl" else "cpu")
        t[self.rank] = float(v)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM)
        return [float(x) for x in t.tolist()]

    def close(self):
        if self.pg:
            self.dist.barrier()
            self.dist.destroy_process_group()


class Clocks:
    """nvidia-smi clock / throttle sampling over the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device, self.proc, self.path = device, None, None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        try:
            for line in open(self.path):
                f = [x.strip() for x in line.split(",")]
                if len(f) < 9:
                    continue
                try:
                    sm.append(float(f[1]))
                    mx = max(mx, float(f[2]))
                except ValueError:
                    continue
                for n, v in zip(names, f[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
            os.unlink(self.path)
        except OSError:
            return None
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def workload_config(world):
    """The `config` both arms print (the driver compares them)."""
    return {"workload": "decode after a 512-token prefill (gemma4.c --bench 512 K); one step = "
                        "forward(1 token) + logits",
            "model": "gemma4-E2B random-init (.bin layout, seed 0)", "global_batch": world,
            "seq_len": PREFILL, "parallelism": f"replicas x{world}",
            "l2": "weights streamed per step (2.35 GB) exceed L2 (126 MB)"}


def prompt_ids(n, seed=0):
    return np.random.default_rng(seed).integers(0, 262144, size=n).astype(np.int32)


def cpu_reference_decode(img, max_seconds=10.0, max_steps=256, prompt=PREFILL):
    """The unmodified reference (oracle/_ref) on this host: prefill `prompt`
    tokens, then decode until max_seconds or max_steps. Returns a dict."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracle import Reference
    Reference.use_all_cores()
    ref = Reference()
    m = ref.open_model(img)
    try:
        ids = prompt_ids(prompt)
        t0 = time.perf_counter()
        for s in range(0, prompt, 512):
            m.forward(ids[s:s + 512], s)
        m.logits((prompt - 1) % 512)
        t_pref = time.perf_counter() - t0
        tok = np.array([2], np.int32)
        steps, t0 = 0, time.perf_counter()
        while steps < max_steps and time.perf_counter() - t0 < max_seconds:
            m.forward(tok, prompt + steps)
            m.logits(0)
            steps += 1
        dt = time.perf_counter() - t0
        return {"prefill_tok_s": prompt / t_pref, "decode_tok_s": steps / dt, "steps": steps, "seconds": dt,
                "cores": ref.threads(), "variant": ref.variant}
    finally:
        m.close()


def run_reference_arm(args, dist):
    """--impl reference: the reference's own CPU implementation of the path on
    this host's cores (rank 0 only), same metric and workload. Only the
    reference library (oracle/_ref, which also carries the synthetic-model
    writer) is loaded; its OpenMP team is the reference's default, one thread
    per physical core (gemma4.c:182-188), whatever OMP_NUM_THREADS a launcher
    exported."""
    if dist.rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracle import Reference
    Reference.use_all_cores()
    ref = Reference()
    img = ref.synth_image(seed=0, flags=0)
    m = ref.open_model(img)
    ids = prompt_ids(PREFILL)
    m.forward(ids, 0)
    m.logits(PREFILL - 1)
    tok = np.array([2], np.int32)
    pos = PREFILL
    for _ in range(args.warmup):
        m.forward(tok, pos)
        m.logits(0)
        pos += 1
    t0 = time.perf_counter()
    for _ in range(args.steps):
        m.forward(tok, pos)
        m.logits(0)
        pos += 1
    dt = time.perf_counter() - t0
    v = args.steps / dt
    line = {
        "impl": "reference", "metric": "decode tok/s @ctx 512", "value": v, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": v / PUBLISHED_DECODE_512, "dtype": "int8", "data": "synthetic",
        "config": workload_config(dist.world),
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": ref.threads(), "kind": "reference",
                         "sample": f"{args.steps} decode steps after a {PREFILL}-token prefill ({ref.variant} build, "
                                   f"{ref.threads()} OpenMP threads: the reference's default of one per core)"},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    m.close()
    print(json.dumps(line), flush=True)


def decode_timed(m, start, steps, warmup, dist, clocks=None, profile_range=False):
    tok = np.array([2], np.int32)
    pos = start
    for _ in range(warmup):
        m.forward(tok, pos)
        m.logits_async(0)
        pos += 1
    m.sync()
    dist.barrier()
    if clocks:
        clocks.start()
    if profile_range:
        m.L.g4_profiler_range(1)
    m.mark(0)
    for _ in range(steps):
        m.forward(tok, pos)
        m.logits_async(0)
        pos += 1
    m.mark(1)
    if profile_range:
        m.sync()
        m.L.g4_profiler_range(0)
    ms = m.elapsed(0, 1)
    m.sync()
    c = clocks.stop() if clocks else None
    dist.barrier()
    return dist.max(ms), pos, c


def prefill_timed(m, n, reps, dist):
    ids = prompt_ids(n)
    times = []
    for r in range(reps + 1):
        m.sync()
        dist.barrier()
        m.mark(2)
        for s in range(0, n, 512):
            m.forward(ids[s:s + 512], s)
        m.logits_async((n - 1) % 512)
        m.mark(3)
        ms = dist.max(m.elapsed(2, 3))
        if r > 0 or reps == 0:
            times.append(ms)
    return n / (np.mean(times) / 1e3), float(np.mean(times))


def pack_sequences(plen, world, per_gpu):
    """Bin-pack sequences over `world` replicas, `per_gpu` each: longest prompt
    first onto the replica with the fewest prompt tokens so far (prefill time
    follows prompt tokens; every replica then finishes together)."""
    load, members = [0] * world, [[] for _ in range(world)]
    for i in np.argsort(-plen, kind="stable"):
        r = min((r for r in range(world) if len(members[r]) < per_gpu), key=lambda r: load[r])
        members[r].append(int(i))
        load[r] += int(plen[i])
    return [sorted(mb) for mb in members]


def batched_serving(m, dist, seqs=64, profile_step=None):
    """Benchmark config 5 (multi-sequence serving): one ragged batch of 64 x N
    independent sequences (prompts log-uniform in [128, 8192], decode lengths
    uniform in [32, 512], ids uniform, seed 2), bin-packed by prompt length
    onto the N replicas, 64 sequences each (N = 1: all 64 in draw order). Each
    prompt is prefilled (512-token chunks) and its first token sampled; then
    all unfinished sequences of a replica decode together, one token per
    sequence per step, greedy, through g4_forward_batch / g4_logits_batch
    (argmax read back every step). Times: CUDA events on the library stream,
    max over ranks."""
    import g4cuda as g4
    rng = np.random.default_rng(2)
    total = seqs * dist.world
    plen_all = np.exp(rng.uniform(np.log(128), np.log(8192), total)).astype(np.int64)
    dlen_all = rng.integers(32, 513, total)
    mine = pack_sequences(plen_all, dist.world, seqs)[dist.rank]
    plen, dlen = plen_all[mine], dlen_all[mine]
    prompts_all = [rng.integers(0, g4.VOCAB, size=int(n)).astype(np.int32) for n in plen_all]
    prompts = [prompts_all[i] for i in mine]
    m.seq_alloc(seqs, int(plen.max() + dlen.max()))
    m.sync()
    dist.barrier()
    m.mark(6)
    nxt = np.zeros(seqs, np.int32)
    for i, p in enumerate(prompts):
        for s0 in range(0, len(p), 512):
            m.forward_batch([i], [p[s0:s0 + 512]], [s0])
        _, am = m.logits_batch()
        nxt[i] = am[0]
    m.mark(7)
    pos = plen.copy()
    left = dlen - 1                      # the first token came with the prefill
    steps = generated = 0
    kv_bytes = 0.0
    while True:
        act = np.nonzero(left > 0)[0]
        if act.size == 0:
            break
        if steps == profile_step:
            m.sync()
            m.L.g4_profiler_range(1)
        m.forward_batch(act.astype(np.int32), [[int(nxt[i])] for i in act], pos[act].astype(np.int32))
        _, am = m.logits_batch()
        nxt[act] = am
        if steps == profile_step:
            m.sync()
            m.L.g4_profiler_range(0)
        # KV read this step: sliding layers min(ctx, 512) keys, global layers all keys, fp32 K + V
        ctx = pos[act] + 1
        kv_bytes += float((28 * np.minimum(ctx, 512) * 256 * 8 + 7 * ctx * 512 * 8).sum())
        pos[act] += 1
        left[act] -= 1
        steps += 1
        generated += act.size
    m.mark(8)
    pre_ms_r, dec_ms_r = m.elapsed(6, 7), m.elapsed(7, 8)
    weights = 2350706688.0
    # whole-job aggregates: every rank's own tokens, over the slowest rank's time
    prompts_r = dist.gather(int(plen.sum()))
    gen_r = dist.gather(generated)
    newtok_r = dist.gather(int(dlen.sum()))
    pre_r, dec_r = dist.gather(pre_ms_r), dist.gather(dec_ms_r)
    steps_r = dist.gather(steps)
    hbm_r = dist.gather((steps * weights + kv_bytes) / (dec_ms_r / 1e3) / 1e9)
    pre_ms, dec_ms = max(pre_r), max(dec_r)
    return {
        "workload": f"{seqs} x {dist.world} sequences (seed 2), prompts log-uniform [128, 8192], decode lengths "
                    f"U[32, 512], greedy; bin-packed by prompt length, {seqs} per GPU",
        "prefill_tok_s": sum(prompts_r) / (pre_ms / 1e3),
        "decode_tok_s": sum(gen_r) / (dec_ms / 1e3),
        "total_tok_s": (sum(prompts_r) + sum(newtok_r)) / ((pre_ms + dec_ms) / 1e3),
        "decode_hbm_gbs_per_gpu": hbm_r,
        "prefill_s": pre_ms / 1e3, "decode_s": dec_ms / 1e3,
        "per_rank": {"prompt_tokens": [int(x) for x in prompts_r], "new_tokens": [int(x) for x in newtok_r],
                     "decode_steps": [int(x) for x in steps_r],
                     "prefill_s": [x / 1e3 for x in pre_r], "decode_s": [x / 1e3 for x in dec_r]},
    }


def attention_bench(g4, hbm_peak, prefill_iters=10, decode_iters=50):
    """Attention over the FP32 KV ring at contexts 512..16384 (benchmark config 4):
    per layer kind, the last 512-token prefill chunk of a context (causal over
    the chunk, start = ctx - 512) and one decode token at position ctx - 1, each
    timed with CUDA events over repeated launches (post-processed q, filled
    ring). Q/K/V are N(0, 1) from seed 1, q/k RMS-normalised (weight 1) and
    rotated; the ring's earlier keys are normalised random vectors (a rotation
    of a Gaussian vector is Gaussian). The model mix is 28 sliding + 7 global
    layers."""
    res = {}
    for ctx in ATTN_CTX:
        row = {}
        for hd, kind, n_layers in ((256, "sliding", 28), (512, "global", 7)):
            window = 512 if hd == 256 else 0
            ring = 1024 if hd == 256 else max(1024, 1 << (ctx - 1).bit_length())
            rng = np.random.default_rng(1)
            qkv = rng.standard_normal((PREFILL, 10 * hd)).astype(np.float32)
            k = rng.standard_normal((ring, hd)).astype(np.float32)
            v = rng.standard_normal((ring, hd)).astype(np.float32)
            k /= np.sqrt((k * k).mean(axis=1, keepdims=True))
            v /= np.sqrt((v * v).mean(axis=1, keepdims=True))
            pairs, theta = (128, 1e4) if hd == 256 else (64, 1e6)
            ang = np.arange(ctx, dtype=np.float64)[:, None] * theta ** (-np.arange(pairs) * 2.0 / hd)[None, :]
            cos_t, sin_t = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
            start = ctx - PREFILL
            keys = np.array([min(p + 1, window) if window else p + 1 for p in range(start, ctx)], np.float64)
            flops = float(keys.sum()) * 8 * hd * 4            # q.k and p.v, 2 FLOP per multiply-add
            _, ms_c = g4.attention(qkv, hd, k.copy(), v.copy(), start, cos_t, sin_t, mode=g4.ATTN_PREFILL,
                                   iters=prefill_iters)
            _, ms_t = g4.attention(qkv, hd, k.copy(), v.copy(), start, cos_t, sin_t, mode=g4.ATTN_PREFILL_TC,
                                   iters=prefill_iters)
            # the path the engine takes for this chunk (G4_OPT_ATTN_PATH 0: by the keys its tokens see)
            on_tc = float(keys.sum()) >= (64 * 1024 if hd == 512 else 128 * 1024)
            ms_p = ms_t if on_tc else ms_c
            _, ms_d = g4.attention(qkv[:1], hd, k, v, ctx - 1, cos_t, sin_t, mode=g4.ATTN_DECODE, splits=148,
                                   iters=decode_iters)
            dbytes = float(keys[-1]) * hd * 8                 # fp32 K and V rows read by one decode token
            tfl = flops / (ms_p / 1e3) / 1e12
            gbs = dbytes / (ms_d / 1e3) / 1e9
            row[kind] = {"prefill_chunk_us": ms_p * 1e3, "prefill_tflops": tfl,
                         "prefill_path": "tensor cores" if on_tc else "cuda cores",
                         "prefill_cuda_core_us": ms_c * 1e3, "prefill_tensor_core_us": ms_t * 1e3,
                         "prefill_cuda_core_frac_fp32_peak": flops / (ms_c / 1e3) / 1e12 / FP32_TFLOPS,
                         "decode_us": ms_d * 1e3,
                         "decode_kv_gbs": gbs, "decode_frac_hbm": gbs / hbm_peak, "layers": n_layers}
        row["model_prefill_chunk_ms"] = sum(row[k]["prefill_chunk_us"] * row[k]["layers"]
                                            for k in ("sliding", "global")) / 1e3
        row["model_decode_us"] = sum(row[k]["decode_us"] * row[k]["layers"] for k in ("sliding", "global"))
        res[f"ctx{ctx}"] = row
    res["note"] = ("prefill: the engine's path for a 512-token chunk (tensor cores: tcgen05 GEMMs on fp16 hi/lo "
                   "operands, k_tc_*, where the chunk's key work is >= 64k global / 128k sliding; else CUDA cores: "
                   "k_attn_prefill + merge), both timed; "
                   "TFLOP/s count the attention's own FLOPs (q.k and p.v), the CUDA-core frac is of the nominal "
                   f"FP32 FMA peak {FP32_TFLOPS:.1f} TFLOP/s; decode: split-KV kernel + combine standalone (inside k_decode "
                   "the same code runs as one phase), frac of the measured HBM copy bandwidth")
    return res


def run_ours(args, dist):
    import g4cuda as g4
    hbm_peak, peak_kind = peaks()
    img = g4.synth_image(seed=0, flags=0)
    m = g4.Model(img, device=dist.local)

    # prefill @512 (also fills the cache for the decode run)
    pre512, pre512_ms = prefill_timed(m, PREFILL, 2, dist)
    # decode @512: the headline
    clocks = Clocks(dist.local)
    ms, pos, clk = decode_timed(m, PREFILL, args.steps, args.warmup, dist, clocks, args.profile_range)
    value = dist.world * args.steps / (ms / 1e3)
    per_step = ms / args.steps

    # end to end through the C ABI: host token in, argmax out, greedy loop
    tok = 2
    m.sync()
    dist.barrier()
    t0 = time.perf_counter()
    m.mark(4)
    for _ in range(args.steps):
        m.forward(np.array([tok], np.int32), pos)
        _, tok = m.logits(0, want_logits=False)
        pos += 1
    m.mark(5)
    wall = time.perf_counter() - t0
    e2e_ms = dist.max(max(m.elapsed(4, 5), wall * 1e3))
    e2e = dist.world * args.steps / (e2e_ms / 1e3)

    # device timeline of one decode step (per op class) and its algorithmic bytes:
    # int8 weights + fp16 scales of every GEMV incl. lm_head, plus the KV read
    prof_ms, prof_bytes, prof_n = m.profile_decode(2, pos)
    pos += 1
    step_bytes = prof_bytes[0] + prof_bytes[1]
    # the decode step is ONE kernel (k_decode): its roofline is the step's bytes
    # over the step time measured above with CUDA events
    dec_gbs = step_bytes / (per_step / 1e3) / 1e9
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "decode_step_traffic.json")) as f:
            traffic = float(json.load(f)["dram_bytes_per_launch"])
    except (OSError, KeyError, ValueError):
        traffic = None

    # prefill GEMM on the tensor cores at T = 512 over the model's shapes
    gemm_ops = gemm_ms = 0.0
    for N, K, cnt in PREFILL_SHAPES:
        if cnt:
            ms_g, ops_g = g4.bench_gemm(N, K, PREFILL, 3, iters=10)
            gemm_ms += cnt * ms_g
            gemm_ops += cnt * ops_g
    gemm_tops = gemm_ops / (gemm_ms / 1e3) / 1e12 if gemm_ms else 0.0
    # benchmark config 3: M in {512, 2048, 8192, 16384} over one layer's projection shapes
    gemm_sweep = None
    if not args.short:
        gemm_sweep = {}
        for M in (512, 2048, 8192, 16384):
            row, ops_m, ms_m = {}, 0.0, 0.0
            for name, N, K in GEMM_SHAPES:
                ms_g, ops_g = g4.bench_gemm(N, K, M, 3, iters=3 if M > 2048 else 10)
                row[name] = ops_g / (ms_g / 1e3) / 1e12
                ops_m += ops_g
                ms_m += ms_g
            row["all_tops"] = ops_m / (ms_m / 1e3) / 1e12
            gemm_sweep[f"M{M}"] = row
    # measured int8 tensor peak of this GPU (back-to-back tcgen05 kind::i8 MMAs on every SM)
    try:
        ms_p, ops_p = g4.bench_mma_i8(20000)
        int8_peak, int8_kind = ops_p / (ms_p / 1e3) / 1e12, "measured (k_mma_peak: tcgen05 kind::i8 back to back)"
    except Exception as e:  # noqa: BLE001 - report the datasheet figure instead
        int8_peak, int8_kind = INT8_DENSE_TOPS, f"nominal dense int8 (datasheet); measurement failed: {e}"

    batched = batched_serving(m, dist, profile_step=20 if args.profile_range else None) if not args.no_batched else None
    attention = attention_bench(g4, hbm_peak) if not args.no_attention else None

    # the other contexts of the reference's README table (pp / tg128 @ d2048, 8192, 16384)
    long = {}
    if not args.short:
        for ctx in (2048, 8192, CTX_LONG):
            pre_c, _ = prefill_timed(m, ctx, 0, dist)
            n_dec = max(8, args.steps // 4)
            ms_c, _, _ = decode_timed(m, ctx, n_dec, 3, dist)
            long[f"prefill_tok_s_{ctx}"] = dist.world * pre_c
            long[f"decode_tok_s_{ctx}"] = dist.world * n_dec / (ms_c / 1e3)
            kv = 28 * min(ctx, 512) * 256 * 8 + 7 * ctx * 512 * 8
            long[f"decode_frac_hbm_{ctx}"] = (2350706688.0 + kv) / (ms_c / n_dec / 1e3) / 1e9 / hbm_peak

    # strict mode (reference-order reductions: the bit-exact configuration), decode at ctx 512
    strict = None
    if not args.short:
        pre_s, _ = prefill_timed(m, PREFILL, 0, dist)
        m.set_option(5, 1)   # G4_OPT_STRICT
        n_s = 8
        ms_s, _, _ = decode_timed(m, PREFILL, n_s, 3, dist)
        m.set_option(5, 0)
        strict = {"decode_tok_s_512": dist.world * n_s / (ms_s / 1e3), "ms_per_step": ms_s / n_s,
                  "note": "G4_OPT_STRICT: RMSNorm sums, attention scores, softmax and value sums in gemma4.c's "
                          "sequential order with the host libm's expf; bit-identical residual stream"}

    # benchmark config 2: the decode GEMV (M = 1) on every projection shape and the lm_head
    gemv_sweep = None
    if not args.short:
        gemv_sweep = {}
        for name, N, K in GEMV_SHAPES:
            ms_v, by = g4.bench_gemv(N, K, 1, iters=50)
            gemv_sweep[name] = {"N": N, "K": K, "us": ms_v * 1e3, "gbs": by / (ms_v / 1e3) / 1e9,
                                "frac_hbm": by / (ms_v / 1e3) / 1e9 / hbm_peak}

    line = {
        "metric": "decode tok/s @ctx 512", "value": value, "unit": "tok/s", "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": value / PUBLISHED_DECODE_512,
        "dtype": "int8", "data": "synthetic",
        "config": workload_config(dist.world),
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 4},
        "gpu_launches": args.steps * m.launches_per_token(),
        "roofline": {"bound": "hbm", "achieved": dec_gbs, "peak": hbm_peak, "unit": "GB/s",
                     "frac": dec_gbs / hbm_peak, "traffic": traffic, "algorithmic_bytes": step_bytes,
                     "kernel": "k_decode: persistent single-token step (all int8 GEMVs incl. lm_head, "
                               "attention, norms) = the only launch per step", "peak_kind": peak_kind},
        "profile_ms": {"gemv": prof_ms[0], "attention": prof_ms[1], "other": prof_ms[2],
                       "ops": prof_n, "source": "device timeline of one traced k_decode launch (op end minus "
                                                "the previous barrier exit, %globaltimer); the tracing itself "
                                                "lengthens that launch, so the classes sum to more than "
                                                "ms_per_step"},
        "prefill_roofline": {"bound": "tensor", "achieved": gemm_tops, "peak": int8_peak,
                             "unit": "TOP/s", "frac": gemm_tops / int8_peak,
                             "peak_nominal": INT8_DENSE_TOPS, "frac_nominal": gemm_tops / INT8_DENSE_TOPS,
                             "kernel": "k_gemm_tc (tcgen05 kind::i8, exact per-group fp32 chain) at T=512 over "
                                       "the model's projection shapes",
                             "peak_kind": int8_kind},
        "prefill_tok_s_512": dist.world * pre512,
    }
    line.update(long)
    if strict:
        line["strict"] = strict
    if gemv_sweep:
        line["decode_gemv_sweep"] = gemv_sweep
    if gemm_sweep:
        line["prefill_gemm_sweep"] = gemm_sweep
    if batched:
        line["batched"] = batched
    if attention:
        line["attention"] = attention
    if clk:
        line["clocks"] = clk
    m.close()
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        cb = cpu_reference_decode(img)
        line["cpu_baseline"] = {"value": cb["decode_tok_s"], "unit": "tok/s", "cores": cb["cores"],
                                "kind": "reference",
                                "sample": f"{cb['steps']} decode steps ({cb['seconds']:.1f} s) after a "
                                          f"{PREFILL}-token prefill, {cb['variant']} build",
                                "prefill_tok_s_512": cb["prefill_tok_s"]}
    if dist.rank == 0:
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--short", action="store_true", help="skip the 16384-context runs")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batched", action="store_true", help="skip the 64-sequence serving run (config 5)")
    ap.add_argument("--no-attention", action="store_true", help="skip the attention sweep (config 4)")
    ap.add_argument("--profile-range", action="store_true",
                    help="open the profiler capture range around the timed decode steps and one "
                         "64-sequence serving step (step 20) only (for ncu --profile-from-start off)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        # the reference arm runs on rank 0's host cores only; other ranks exit at once
        dist = Dist.__new__(Dist)
        dist.rank, dist.world, dist.local, dist.pg = env_int("RANK", 0), env_int("WORLD_SIZE", 1), 0, None
        run_reference_arm(args, dist)
        return
    dist = Dist()
    try:
        run_ours(args, dist)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
