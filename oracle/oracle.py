"""ctypes bindings for the parity checker — TEST INFRASTRUCTURE ONLY.

`Oracle` wraps liboracle.so, our C restatement of gemma4.c's forward path
(oracle/g4_oracle.c). `Reference` wraps oracle/_ref/libg4ref_*.so, the
unmodified reference gemma4.c compiled from its own sources with accessor
functions (oracle/ref_harness.c). Only tests, the smoke check and the
benchmark's CPU-baseline leg import this module; the product never does.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")


def _ptr(a):
    return a.ctypes.data_as(C.c_void_p)


def aligned(a, align=64):
    """Copy of `a` at an `align`-byte boundary: the reference's AVX-512 path uses
    aligned loads on weight tensors, which a mapped model file guarantees."""
    a = np.ascontiguousarray(a)
    raw = np.empty(a.nbytes + align, np.uint8)
    off = (-raw.ctypes.data) % align
    out = raw[off:off + a.nbytes].view(a.dtype).reshape(a.shape)
    out[...] = a
    return out


def cpu_flags():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    return set(line.split(":", 1)[1].split())
    except OSError:
        pass
    return set()


class Oracle:
    """Our C restatement (oracle/g4_oracle.c)."""

    def __init__(self, path=None):
        path = path or os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle`")
        L = self.lib = C.CDLL(path)
        L.or_quantize.argtypes = [_i8p, _f32p, _f32p, C.c_size_t, C.c_size_t]
        L.or_linear_dots.argtypes = [_i32p, _i8p, C.c_size_t, _i8p, C.c_int, C.c_int]
        L.or_linear.argtypes = [_f32p, _i8p, _f32p, C.c_size_t, _i8p, _u16p, C.c_int, C.c_int]
        L.or_rmsnorm.argtypes = [_f32p, _f32p, C.c_void_p, C.c_int, C.c_float, C.c_size_t]
        L.or_rope.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_size_t]
        L.or_geglu.argtypes = [_f32p, _f32p, C.c_int, C.c_int, C.c_int, _f32p, C.c_int, C.c_int, C.c_int]
        L.or_embedding.argtypes = [_f32p, C.c_void_p, C.c_void_p, C.c_int, _i32p, C.c_size_t, C.c_float]
        L.or_softcap.argtypes = [_f32p, C.c_size_t]
        L.or_argmax.argtypes = [_f32p, C.c_int]
        L.or_argmax.restype = C.c_int
        L.or_topk.argtypes = [_f32p, C.c_int, C.c_int, _f32p, _i32p]
        L.or_sample.argtypes = [_f32p, C.c_int, C.c_float, C.POINTER(C.c_ulonglong)]
        L.or_sample.restype = C.c_int
        L.or_attend.argtypes = [_f32p, _f32p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, _f32p]
        L.or_model_open.argtypes = [C.c_void_p, C.c_uint64]
        L.or_model_open.restype = C.c_void_p
        L.or_model_close.argtypes = [C.c_void_p]
        L.or_state_new.restype = C.c_void_p
        L.or_state_free.argtypes = [C.c_void_p]
        L.or_forward.argtypes = [C.c_void_p, C.c_void_p, _i32p, C.c_size_t, C.c_int]
        L.or_logits.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t]
        L.or_logits.restype = C.POINTER(C.c_float)
        L.or_state_residual.argtypes = [C.c_void_p]
        L.or_state_residual.restype = C.POINTER(C.c_float)
        L.or_state_cache.argtypes = [C.c_void_p, C.c_int, C.c_int]
        L.or_state_cache.restype = C.POINTER(C.c_float)
        L.or_state_ple.argtypes = [C.c_void_p]
        L.or_state_ple.restype = C.POINTER(C.c_float)
        L.or_prologue.argtypes = [C.c_void_p, C.c_void_p, _i32p, C.c_size_t]
        L.or_layer.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_size_t]
        L.or_logits_rows.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, _f32p]
        L.or_num_threads.restype = C.c_int

    # kernels ---------------------------------------------------------------
    def quantize(self, x):
        x = np.ascontiguousarray(x, np.float32)
        rows, width = x.shape
        q = np.empty((rows, width), np.int8)
        s = np.empty((rows, width // 64), np.float32)
        self.lib.or_quantize(q, s, x, rows, width)
        return q, s

    def linear_dots(self, xq, w_packed, N, K):
        T = xq.shape[0]
        d = np.empty((T, N, K // 64), np.int32)
        self.lib.or_linear_dots(d, np.ascontiguousarray(xq), T, w_packed, N, K)
        return d

    def linear(self, xq, xs, w_packed, s_packed, N, K):
        T = xq.shape[0]
        out = np.empty((T, N), np.float32)
        self.lib.or_linear(out, np.ascontiguousarray(xq), np.ascontiguousarray(xs, np.float32), T,
                           w_packed, s_packed, N, K)
        return out

    def rmsnorm(self, x, w, eps=1e-6):
        x = np.ascontiguousarray(x, np.float32)
        rows, width = x.shape
        out = np.empty_like(x)
        wp = None if w is None else np.ascontiguousarray(w, np.float32)
        self.lib.or_rmsnorm(out, x, None if wp is None else _ptr(wp), width, eps, rows)
        return out

    def rope(self, v, cos_t, sin_t, heads, head_dim, start_pos):
        v = np.array(v, np.float32, copy=True, order="C")
        T = v.shape[0]
        self.lib.or_rope(v, np.ascontiguousarray(cos_t), np.ascontiguousarray(sin_t), cos_t.shape[1],
                         heads, head_dim, start_pos, T)
        return v

    def sample(self, logits, temperature, state):
        """gemma4.c:536-561 on one row; returns (token, state after the draw)."""
        st = C.c_ulonglong(state)
        tok = self.lib.or_sample(np.ascontiguousarray(logits, np.float32), logits.size, temperature, C.byref(st))
        return tok, st.value

    def attention(self, qkv, hd, kring, vring, start_pos, cos_t, sin_t, q_norm=None, k_norm=None):
        """One attention sub-layer as attention_layer restates gemma4.c:411-461,
        from raw per-token q (8 heads) | k | v rows: q/k RMSNorm (k, q with
        weights), v RMSNorm without weight, RoPE, ring write at (start_pos + t)
        & (ring - 1), then or_attend per (token, head). hd 256 is a sliding
        layer (window 512), hd 512 a global one. kring / vring are updated in
        place; returns out[T][8*hd]."""
        qkv = np.ascontiguousarray(qkv, np.float32)
        T = qkv.shape[0]
        ring = kring.shape[0]
        mask, window = ring - 1, (512 if hd == 256 else 0)
        q = qkv[:, :8 * hd].reshape(T * 8, hd)
        k = qkv[:, 8 * hd:9 * hd]
        v = qkv[:, 9 * hd:10 * hd]
        q = self.rope(self.rmsnorm(q, q_norm if q_norm is not None else np.ones(hd, np.float32)).reshape(T, 8 * hd),
                      cos_t, sin_t, 8, hd, start_pos)
        k = self.rope(self.rmsnorm(k, k_norm if k_norm is not None else np.ones(hd, np.float32)),
                      cos_t, sin_t, 1, hd, start_pos)
        v = self.rmsnorm(v, None)
        for t in range(T):
            kring[(start_pos + t) & mask] = k[t]
            vring[(start_pos + t) & mask] = v[t]
        out = np.empty((T, 8 * hd), np.float32)
        scores = np.empty(start_pos + T, np.float32)
        kp, vp = _ptr(kring), _ptr(vring)
        row = np.empty(hd, np.float32)
        for t in range(T):
            p = start_pos + t
            first = p + 1 - window if window and p + 1 > window else 0
            for h in range(8):
                qh = np.ascontiguousarray(q[t, h * hd:(h + 1) * hd])
                self.lib.or_attend(row, qh, kp, vp, first, p + 1 - first, mask, hd, scores)
                out[t, h * hd:(h + 1) * hd] = row
        return out

    def geglu(self, gate, up, width, up_stride, table):
        gate = np.array(gate, np.float32, copy=True, order="C")
        rows = gate.shape[0]
        self.lib.or_geglu(gate, np.ascontiguousarray(up, np.float32), rows, width, up_stride,
                          np.ascontiguousarray(table, np.float32), 4096, -8, 8)
        return gate

    def embedding(self, w_packed, s_packed, width, tokens, mult):
        tokens = np.ascontiguousarray(tokens, np.int32)
        out = np.empty((len(tokens), width), np.float32)
        self.lib.or_embedding(out, _ptr(w_packed), _ptr(s_packed), width, tokens, len(tokens), mult)
        return out

    def softcap(self, x):
        x = np.array(x, np.float32, copy=True, order="C")
        self.lib.or_softcap(x, x.size)
        return x

    def topk(self, x, k):
        x = np.ascontiguousarray(x, np.float32)
        vals = np.empty(k, np.float32)
        ids = np.empty(k, np.int32)
        self.lib.or_topk(x, x.size, k, vals, ids)
        return vals, ids

    # whole model -------------------------------------------------------------
    def open_model(self, image):
        h = self.lib.or_model_open(_ptr(image), image.nbytes)
        if not h:
            raise ValueError("oracle rejected the model image")
        return OracleModel(self, image, h)


class OracleModel:
    def __init__(self, oracle, image, handle):
        self.o, self.image, self.h = oracle, image, handle
        self.state = oracle.lib.or_state_new()

    def forward(self, tokens, start_pos):
        tokens = np.ascontiguousarray(tokens, np.int32)
        self.o.lib.or_forward(self.h, self.state, tokens, len(tokens), start_pos)

    def logits(self, row):
        p = self.o.lib.or_logits(self.h, self.state, row)
        return np.ctypeslib.as_array(p, shape=(262144,)).copy()

    def residual(self, rows):
        p = self.o.lib.or_state_residual(self.state)
        return np.ctypeslib.as_array(p, shape=(rows, 1536)).copy()

    def cache(self, layer, which, slots, head_dim):
        p = self.o.lib.or_state_cache(self.state, layer, which)
        return np.ctypeslib.as_array(p, shape=(slots, head_dim)).copy()

    # teacher forcing: state views the tests write into, and one layer at a time
    def residual_view(self, rows):
        """Writable view of the first `rows` residual rows of the state."""
        p = self.o.lib.or_state_residual(self.state)
        return np.ctypeslib.as_array(p, shape=(rows, 1536))

    def ple_view(self, rows):
        """Writable view of the per-layer inputs [rows][35][256] of the state."""
        p = self.o.lib.or_state_ple(self.state)
        return np.ctypeslib.as_array(p, shape=(rows, 35, 256))

    def cache_view(self, layer, which, slots, head_dim):
        """Writable view of the K (0) / V (1) ring that `layer` reads."""
        p = self.o.lib.or_state_cache(self.state, layer, which)
        return np.ctypeslib.as_array(p, shape=(slots, head_dim))

    def prologue(self, tokens):
        tokens = np.ascontiguousarray(tokens, np.int32)
        self.o.lib.or_prologue(self.h, self.state, tokens, len(tokens))

    def layer(self, layer, start_pos, rows):
        self.o.lib.or_layer(self.h, self.state, layer, start_pos, rows)

    def logits_rows(self, rows):
        """logits() of residual rows [0, rows) of the state, [rows][262144]."""
        out = np.empty((rows, 262144), np.float32)
        self.o.lib.or_logits_rows(self.h, self.state, rows, out)
        return out

    def close(self):
        if self.state:
            self.o.lib.or_state_free(self.state)
            self.o.lib.or_model_close(self.h)
            self.state = None


class Reference:
    """The unmodified reference gemma4.c (oracle/_ref), VNNI build when the host
    supports it, else the AVX2 build (both give identical results)."""

    def __init__(self, variant=None):
        flags = cpu_flags()
        if variant is None:
            need = {"avx512f", "avx512bw", "avx512vl", "avx512dq", "avx512cd", "avx512_vnni"}
            variant = "vnni" if need <= flags else "avx2"
        path = os.path.join(HERE, "_ref", f"libg4ref_{variant}.so")
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: build the reference with `make -C oracle ref`")
        self.variant = variant
        L = self.lib = C.CDLL(path)
        L.g4ref_state_new.restype = C.c_void_p
        L.g4ref_state_free.argtypes = [C.c_void_p]
        L.g4ref_state_residual.argtypes = [C.c_void_p]
        L.g4ref_state_residual.restype = C.POINTER(C.c_float)
        L.g4ref_threads.restype = C.c_int
        L.g4ref_model_view.argtypes = [C.c_void_p]
        L.g4ref_model_view.restype = C.c_void_p
        L.g4ref_model_free.argtypes = [C.c_void_p]
        L.forward.argtypes = [C.c_void_p, C.c_void_p, _i32p, C.c_size_t, C.c_int]
        L.logits.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t]
        L.logits.restype = C.POINTER(C.c_float)
        L.quantize.argtypes = [_i8p, _f32p, _f32p, C.c_size_t, C.c_size_t]
        L.g4ref_matmul.argtypes = [_f32p, _i8p, _f32p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_size_t]
        L.g4ref_rmsnorm.argtypes = [_f32p, _f32p, C.c_void_p, C.c_int, C.c_float, C.c_size_t]
        L.g4ref_geglu.argtypes = [_f32p, _f32p, C.c_int, C.c_int, C.c_int, _f32p]
        L.g4ref_rope.argtypes = [_f32p, _f32p, C.c_int, _f32p, C.c_int, C.c_int, C.c_int, C.c_size_t]
        L.g4ref_embedding.argtypes = [_f32p, C.c_void_p, C.c_void_p, C.c_int, _i32p, C.c_size_t, C.c_float]
        L.softmax.argtypes = [_f32p, C.c_int]
        L.sample.argtypes = [_f32p, C.c_int, C.c_float]
        L.sample.restype = C.c_int
        L.g4synth_image_bytes.restype = C.c_uint64
        L.g4synth_fill.argtypes = [C.c_void_p, C.c_uint64, C.c_uint64, C.c_uint]
        L.g4synth_fill.restype = C.c_int

    def synth_image(self, seed=0, flags=0):
        """The seeded synthetic model image (the same bytes as g4cuda.synth_image),
        written by the copy of the synthetic-model writer linked into this
        library, so the reference leg loads no other shared object."""
        n = self.lib.g4synth_image_bytes()
        raw = np.empty(n + 4096, np.uint8)
        off = (-raw.ctypes.data) % 4096
        img = raw[off:off + n]
        if self.lib.g4synth_fill(img.ctypes.data, n, seed, flags) != 0:
            raise RuntimeError("g4synth_fill failed")
        return img

    @staticmethod
    def use_all_cores():
        """The reference sizes its OpenMP team from OMP_NUM_THREADS when that is
        set, else one thread per physical core (gemma4.c:182-188). Launchers such
        as torchrun export OMP_NUM_THREADS=1; dropping it restores the
        reference's own default. Returns the value removed (or None)."""
        return os.environ.pop("OMP_NUM_THREADS", None)

    def threads(self):
        return self.lib.g4ref_threads()

    def sample(self, logits, temperature, state):
        """The reference's own sample() with its global rng_state set to `state`;
        returns (token, rng_state after the call)."""
        rs = C.c_ulonglong.in_dll(self.lib, "rng_state")
        rs.value = state
        tok = self.lib.sample(np.array(logits, np.float32, copy=True), logits.size, temperature)
        return tok, rs.value

    def quantize(self, x):
        x = np.ascontiguousarray(x, np.float32)
        rows, width = x.shape
        q = np.empty((rows, width), np.int8)
        s = np.empty((rows, width // 64), np.float32)
        self.lib.quantize(q, s, x, rows, width)
        return q, s

    def linear(self, xq, xs, w_packed, s_packed, N, K):
        T = xq.shape[0]
        out = np.empty((T, N), np.float32)
        w_packed, s_packed = aligned(w_packed), aligned(s_packed)
        self.lib.g4ref_matmul(out, np.ascontiguousarray(xq), np.ascontiguousarray(xs, np.float32),
                              _ptr(w_packed), _ptr(s_packed), N, K, T)
        return out

    def rmsnorm(self, x, w, eps=1e-6):
        x = np.ascontiguousarray(x, np.float32)
        rows, width = x.shape
        out = np.empty_like(x)
        wp = None if w is None else np.ascontiguousarray(w, np.float32)
        self.lib.g4ref_rmsnorm(out, x, None if wp is None else _ptr(wp), width, eps, rows)
        return out

    def rope(self, v, cos_t, sin_t, heads, head_dim, start_pos):
        v = np.array(v, np.float32, copy=True, order="C")
        self.lib.g4ref_rope(np.ascontiguousarray(cos_t), np.ascontiguousarray(sin_t), cos_t.shape[1], v,
                            heads, head_dim, start_pos, v.shape[0])
        return v

    def geglu(self, gate, up, width, up_stride, table):
        gate = np.array(gate, np.float32, copy=True, order="C")
        self.lib.g4ref_geglu(gate, np.ascontiguousarray(up, np.float32), gate.shape[0], width, up_stride,
                             np.ascontiguousarray(table, np.float32))
        return gate

    def embedding(self, w_packed, s_packed, width, tokens, mult):
        tokens = np.ascontiguousarray(tokens, np.int32)
        out = np.empty((len(tokens), width), np.float32)
        w_packed, s_packed = aligned(w_packed), aligned(s_packed)
        self.lib.g4ref_embedding(out, _ptr(w_packed), _ptr(s_packed), width, tokens, len(tokens), mult)
        return out

    def open_model(self, image):
        view = self.lib.g4ref_model_view(_ptr(image))
        return ReferenceModel(self, image, view)


class ReferenceModel:
    def __init__(self, ref, image, view):
        self.r, self.image, self.view = ref, image, view
        self.state = ref.lib.g4ref_state_new()
        if not self.state:
            raise MemoryError("reference InferenceState allocation failed")

    def forward(self, tokens, start_pos):
        tokens = np.ascontiguousarray(tokens, np.int32)
        self.r.lib.forward(self.view, self.state, tokens, len(tokens), start_pos)

    def logits(self, row):
        p = self.r.lib.logits(self.view, self.state, row)
        return np.ctypeslib.as_array(p, shape=(262144,)).copy()

    def residual(self, rows):
        p = self.r.lib.g4ref_state_residual(self.state)
        return np.ctypeslib.as_array(p, shape=(rows, 1536)).copy()

    def close(self):
        if self.state:
            self.r.lib.g4ref_state_free(self.state)
            self.r.lib.g4ref_model_free(self.view)
            self.state = None
