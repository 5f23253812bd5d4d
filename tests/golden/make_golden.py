"""Generate the golden vectors from the reference itself.

Runs the unmodified reference gemma4.c (compiled from its own sources into
oracle/_ref by `make -C oracle ref`) on seeded inputs and stores inputs and
outputs as small .npz fixtures:

  kernels.npz — quantize, matmul_int8 (two shapes), rmsnorm (with and without
                weight), apply_rope (sliding and partial global), geglu
                (including the table edges), embedding, softmax;
  sample.npz  — sample() (top-64, temperature, 95 % prefix, xorshift draw) on
                48 seeded logits rows of 1024 values at several temperatures,
                with the generator state chained from 42 through the rows;
  model.npz   — whole-model forward/logits on the seed-0 synthetic E2B image
                (per-group scales, random norms): a 6-token prefill and one
                decode step; stores the top-32 of the logits, float64 checksums
                of the full logits, and the residual rows.

The reference has no tests or fixtures of its own (it ships 11 source/text
files), so these vectors are the pin for the oracle restatement. Regenerate
with `python tests/golden/make_golden.py` in a container that has the
reference sources.
"""
import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "gemma4.c_b200"))

from oracle import Reference  # noqa: E402


def pack(w, s):
    N, K = w.shape
    G = K // 64
    wp = w.reshape(N // 16, 16, G, 16, 4).transpose(0, 2, 3, 1, 4).reshape(-1)
    sp = s.reshape(N // 16, 16, G).transpose(0, 2, 1).reshape(-1)
    return np.ascontiguousarray(wp, np.int8), np.ascontiguousarray(sp, np.uint16)


def kernels(ref):
    rng = np.random.default_rng(1234)
    out = {}
    # quantize: random rows with an outlier row, a zero group, exact halves
    x = rng.standard_normal((4, 1536)).astype(np.float32)
    x[1] *= 50.0
    x[2, :64] = 0.0
    x[3, :64] = np.linspace(-127, 127, 64).astype(np.float32)
    x[3, 0] = -127.0
    x[3, 1:7] = [2.5, 3.5, -2.5, -3.5, 0.5, -0.5]
    q, s = ref.quantize(x)
    out.update(quant_x=x, quant_q=q, quant_s=s)
    # matmul_int8 on two shapes
    for tag, (N, K, T) in {"mm_a": (32, 256, 3), "mm_b": (16, 1536, 1)}.items():
        w = rng.integers(-127, 128, size=(N, K)).astype(np.int8)
        sc = rng.uniform(1e-4, 1e-2, size=(N, K // 64)).astype(np.float16).view(np.uint16)
        wp, sp = pack(w, sc)
        xq, xs = ref.quantize(rng.standard_normal((T, K)).astype(np.float32))
        y = ref.linear(xq, xs, wp, sp, N, K)
        out.update({f"{tag}_wp": wp, f"{tag}_sp": sp, f"{tag}_xq": xq, f"{tag}_xs": xs, f"{tag}_out": y,
                    f"{tag}_shape": np.array([N, K, T], np.int32)})
    # rmsnorm
    x = rng.standard_normal((3, 1536)).astype(np.float32)
    w = rng.uniform(0.5, 1.5, 1536).astype(np.float32)
    out.update(rms_x=x, rms_w=w, rms_y=ref.rmsnorm(x, w, 1e-6))
    x2 = rng.standard_normal((2, 256)).astype(np.float32)
    out.update(rms2_x=x2, rms2_y=ref.rmsnorm(x2, None, 1e-6))
    # rope: tables for positions 0..1002, sliding (256, 128 pairs) and global (512, 64 pairs)
    for tag, (hd, pairs, theta) in {"rope_s": (256, 128, 1e4), "rope_g": (512, 64, 1e6)}.items():
        P = 1003
        freq = (np.float32(1) / np.power(np.float32(theta), 2 * np.arange(pairs, dtype=np.float32) / np.float32(hd)))
        ang = np.arange(P, dtype=np.float32)[:, None] * freq
        ct, st = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
        v = rng.standard_normal((2, 8 * hd)).astype(np.float32)
        y = ref.rope(v, ct, st, 8, hd, 1001)   # rows 1001, 1002 of the tables
        out.update({f"{tag}_cos": ct[1001:], f"{tag}_sin": st[1001:], f"{tag}_v": v, f"{tag}_y": y,
                    f"{tag}_cfg": np.array([hd, pairs], np.int32)})
    # geglu with the table edges
    xs_ = np.linspace(-8, 8, 4096, dtype=np.float32)
    table = (0.5 * xs_ * (1.0 + np.tanh(0.7978845608 * (xs_ + 0.044715 * xs_ * xs_ * xs_)))).astype(np.float32)
    gate = rng.standard_normal((2, 256)).astype(np.float32) * 4
    gate[0, :8] = [-8.0, -8.000001, np.nextafter(np.float32(8), np.float32(0)), 8.0, 100.0, -100.0, 1e-3, 0.0]
    up = rng.standard_normal((2, 512)).astype(np.float32)
    out.update(geglu_gate=gate, geglu_up=up, geglu_table=table,
               geglu_y=ref.geglu(gate, up, 256, 512, table))
    # embedding from a 64-row packed table
    w = rng.integers(-127, 128, size=(64, 1536)).astype(np.int8)
    sc = rng.uniform(1e-4, 1e-2, size=(64, 24)).astype(np.float16).view(np.uint16)
    wp, sp = pack(w, sc)
    toks = np.array([0, 17, 63, 5], np.int32)
    out.update(emb_wp=wp, emb_sp=sp, emb_tokens=toks, emb_y=ref.embedding(wp, sp, 1536, toks, np.float32(np.sqrt(np.float32(1536)))))
    # softmax
    sm = rng.standard_normal(777).astype(np.float32) * 16
    smo = sm.copy()
    ref.lib.softmax(smo, smo.size)
    out.update(softmax_x=sm, softmax_y=smo)
    return out


def model(ref):
    import g4cuda
    img = g4cuda.synth_image(seed=0, flags=g4cuda.SYN_GROUP_SCALES | g4cuda.SYN_RANDOM_NORMS)
    m = ref.open_model(img)
    rng = np.random.default_rng(77)
    toks = rng.integers(0, 262144, size=7).astype(np.int32)
    out = {"tokens": toks}
    m.forward(toks[:6], 0)
    out["prefill_residual"] = m.residual(6)
    for tag, row in (("prefill_row5", 5), ("prefill_row0", 0)):
        lg = m.logits(row)
        top = np.argsort(-lg, kind="stable")[:32]
        out[f"{tag}_top_ids"] = top.astype(np.int32)
        out[f"{tag}_top_vals"] = lg[top]
        out[f"{tag}_sum"] = np.array([lg.astype(np.float64).sum(), (lg.astype(np.float64) ** 2).sum()])
    m.forward(toks[6:7], 6)
    out["decode_residual"] = m.residual(1)
    lg = m.logits(0)
    top = np.argsort(-lg, kind="stable")[:32]
    out["decode_top_ids"] = top.astype(np.int32)
    out["decode_top_vals"] = lg[top]
    out["decode_sum"] = np.array([lg.astype(np.float64).sum(), (lg.astype(np.float64) ** 2).sum()])
    m.close()
    return out


def samples(ref):
    rng = np.random.default_rng(11)
    rows, temps, toks, states = [], [], [], []
    state = 42
    for i in range(48):
        lg = (rng.standard_normal(1024) * rng.uniform(0.5, 6.0)).astype(np.float32)
        if i % 6 == 0:                      # ties at the top
            lg[rng.integers(0, 1024, 20)] = lg.max()
        t = (0.0, 0.25, 0.7, 1.0, 1.6, 3.0)[i % 6]
        tok, state = ref.sample(lg, t, state)
        rows.append(lg)
        temps.append(t)
        toks.append(tok)
        states.append(state)
    return {"logits": np.stack(rows), "temperature": np.array(temps, np.float32),
            "token": np.array(toks, np.int32), "state": np.array(states, np.uint64)}


def main():
    ref = Reference()
    np.savez_compressed(os.path.join(HERE, "sample.npz"), **samples(ref))
    np.savez_compressed(os.path.join(HERE, "kernels.npz"), **kernels(ref))
    np.savez_compressed(os.path.join(HERE, "model.npz"), **model(ref))
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    main()
