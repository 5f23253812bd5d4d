"""Python binding of libg4cuda.so (include/g4cuda.h) via ctypes.

Mirrors the reference's hot-path interface — `forward(tokens, start_pos)` and
`logits(row)` of gemma4.c:463 and gemma4.c:512 — on a device context, plus the
single-kernel entry points the parity tests drive. No torch: device memory,
streams and kernels all live inside the C library.

Importing this module never falls back to a CPU path: if the shared library
is missing, `load()` raises.
"""
import ctypes as C
import os
import re

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "libg4cuda.so")
HEADER = os.path.join(ROOT, "include", "g4cuda.h")

VOCAB = 262144
HIDDEN = 1536
NUM_LAYERS = 35
MAX_CONTEXT = 131072
G4_OK = 0
ERRORS = {-1: "G4_ERR_INVALID", -2: "G4_ERR_FORMAT", -3: "G4_ERR_CUDA", -4: "G4_ERR_NOMEM",
          -5: "G4_ERR_DEVICE", -6: "G4_ERR_STATE"}
OPT_GRAPHS, OPT_PDL, OPT_GEMM_PATH, OPT_LAYERS, OPT_STRICT, OPT_PERSISTENT, OPT_BATCH_SPLITS = 1, 2, 3, 4, 5, 6, 7
SYN_GROUP_SCALES, SYN_RANDOM_NORMS = 1, 2

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")


class G4Error(RuntimeError):
    def __init__(self, code, msg=""):
        self.code = code
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")


_lib = None


def load(path=LIB_PATH):
    """Load libg4cuda.so once; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} not built: run `make -C gemma4.c_b200` or __graft_entry__.build()")
    L = C.CDLL(path)
    vp = C.c_void_p
    L.g4_open.argtypes = [vp, C.c_uint64, C.c_int, C.POINTER(vp)]
    L.g4_open_file.argtypes = [C.c_char_p, C.c_int, C.POINTER(vp)]
    L.g4_open_error.restype = C.c_char_p
    L.g4_close.argtypes = [vp]
    L.g4_forward.argtypes = [vp, _i32p, C.c_size_t, C.c_int]
    L.g4_logits.argtypes = [vp, C.c_size_t, vp, vp]
    L.g4_topk.argtypes = [vp, C.c_size_t, C.c_int, _f32p, _i32p]
    L.g4_sync.argtypes = [vp]
    L.g4_last_error.argtypes = [vp]
    L.g4_last_error.restype = C.c_char_p
    L.g4_strerror.restype = C.c_char_p
    L.g4_set_option.argtypes = [vp, C.c_int, C.c_int]
    L.g4_read_residual.argtypes = [vp, C.c_size_t, _f32p]
    L.g4_read_cache.argtypes = [vp, C.c_int, C.c_int, C.c_int, C.c_int, _f32p]
    L.g4_test_starve_next_step.argtypes = [vp]
    L.g4_read_ple.argtypes = [vp, C.c_size_t, _f32p]
    L.g4_read_seq_cache.argtypes = [vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _f32p]
    L.g4_stream.argtypes = [vp]
    L.g4_stream.restype = vp
    L.g4_device_bytes.argtypes = [vp, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]
    L.g4synth_image_bytes.restype = C.c_uint64
    L.g4synth_fill.argtypes = [vp, C.c_uint64, C.c_uint64, C.c_uint]
    L.g4synth_write_file.argtypes = [C.c_char_p, C.c_uint64, C.c_uint]
    L.g4k_quantize.argtypes = [_f32p, C.c_int, C.c_int, _i8p, _f32p]
    L.g4k_linear.argtypes = [_i8p, _u16p, C.c_int, C.c_int, _i8p, _f32p, C.c_int, C.c_int, _f32p, vp]
    L.g4k_rmsnorm_quant.argtypes = [_f32p, C.c_int, _f32p, C.c_float, vp, _i8p, _f32p]
    L.g4_bench_gemm.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_float),
                                C.POINTER(C.c_double)]
    L.g4_bench_mma_i8.argtypes = [C.c_int, C.POINTER(C.c_float), C.POINTER(C.c_double)]
    L.g4_skinny_plan.argtypes = [C.c_int] * 3 + [C.POINTER(C.c_int)] * 5
    L.g4_bench_gemv.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_float),
                                C.POINTER(C.c_double)]
    L.g4k_attention.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _f32p, vp, vp, _f32p,
                                _f32p, _f32p, _f32p, _f32p, vp, vp, C.c_int, C.POINTER(C.c_float)]
    L.g4k_sample.argtypes = [_f32p, C.c_int, C.c_float, C.POINTER(C.c_ulonglong), C.POINTER(C.c_int)]
    L.g4_sample.argtypes = [vp, C.c_size_t, C.c_float, C.POINTER(C.c_int)]
    L.g4_set_seed.argtypes = [vp, C.c_uint64]
    L.g4_logits_rows.argtypes = [vp, C.c_size_t, C.c_size_t, vp]
    L.g4_profiler_range.argtypes = [C.c_int]
    L.g4_mark.argtypes = [vp, C.c_int]
    L.g4_elapsed.argtypes = [vp, C.c_int, C.c_int, C.POINTER(C.c_float)]
    L.g4_profile_decode.argtypes = [vp, C.c_int, C.c_int, C.POINTER(C.c_float), C.POINTER(C.c_double),
                                    C.POINTER(C.c_int)]
    L.g4_launches_per_token.argtypes = [vp, C.POINTER(C.c_int)]
    L.g4_trace_decode.argtypes = [vp, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_double),
                                  C.POINTER(C.c_int)]
    L.g4_topk_noalloc.argtypes = [vp, C.c_int, C.c_int, vp, vp, vp]
    L.g4_seq_alloc.argtypes = [vp, C.c_int, C.c_int]
    L.g4_forward_batch.argtypes = [vp, C.c_int, _i32p, _i32p, _i32p, _i32p]
    L.g4_logits_batch.argtypes = [vp, vp, vp]
    _lib = L
    return L


def header_symbols(header=HEADER):
    """Function names declared in include/g4cuda.h."""
    text = open(header).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(g4[a-z0-9_]*)\s*\(", text)))


def _check(code, ctx=None):
    if code != G4_OK:
        L = load()
        msg = L.g4_last_error(ctx).decode() if ctx else L.g4_strerror(code).decode()
        raise G4Error(code, msg)


# ---------------------------------------------------------------------------
# synthetic model images

def aligned_empty(nbytes, align=4096):
    """Page-aligned uint8 buffer (the reference's AVX-512 path needs 64-byte
    aligned tensors, which a mapped file gives and a plain numpy array may not)."""
    raw = np.empty(nbytes + align, np.uint8)
    off = (-raw.ctypes.data) % align
    return raw[off:off + nbytes]


def synth_image(seed=0, flags=0):
    """A seeded random-init Gemma 4 E2B image in the gemma4.c .bin layout."""
    L = load()
    n = L.g4synth_image_bytes()
    img = aligned_empty(n)
    _check(L.g4synth_fill(img.ctypes.data, n, seed, flags))
    return img


# ---------------------------------------------------------------------------
# the model context

class Model:
    """A device context: forward/logits exactly as gemma4.c's hot path."""

    def __init__(self, image=None, path=None, device=0):
        L = self.L = load()
        h = C.c_void_p()
        if path is not None:
            rc = L.g4_open_file(path.encode(), device, C.byref(h))
        else:
            rc = L.g4_open(image.ctypes.data, image.nbytes, device, C.byref(h))
        if rc != G4_OK:
            raise G4Error(rc, L.g4_open_error().decode())
        self.h = h

    def set_option(self, option, value):
        _check(self.L.g4_set_option(self.h, option, int(value)), self.h)

    def forward(self, tokens, start_pos):
        tokens = np.ascontiguousarray(tokens, np.int32)
        _check(self.L.g4_forward(self.h, tokens, tokens.size, int(start_pos)), self.h)

    def logits(self, row=0, want_logits=True):
        out = np.empty(VOCAB, np.float32) if want_logits else None
        am = C.c_int(-1)
        _check(self.L.g4_logits(self.h, row, out.ctypes.data if out is not None else None, C.byref(am)), self.h)
        return out, am.value

    def logits_rows(self, row0, n, out=None):
        """Logits of n rows of the last forward (g4_logits_rows), [n][VOCAB]."""
        if out is None:
            out = np.empty((n, VOCAB), np.float32)
        _check(self.L.g4_logits_rows(self.h, row0, n, out.ctypes.data), self.h)
        return out

    def sample(self, row, temperature):
        """Next token drawn on the device (g4_sample) from logits row `row`."""
        tok = C.c_int(0)
        _check(self.L.g4_sample(self.h, row, temperature, C.byref(tok)), self.h)
        return tok.value

    def set_seed(self, seed):
        _check(self.L.g4_set_seed(self.h, seed), self.h)

    def topk(self, row, k):
        v = np.empty(k, np.float32)
        i = np.empty(k, np.int32)
        _check(self.L.g4_topk(self.h, row, k, v, i), self.h)
        return v, i

    def sync(self):
        _check(self.L.g4_sync(self.h), self.h)

    def residual(self, rows):
        out = np.empty((rows, HIDDEN), np.float32)
        _check(self.L.g4_read_residual(self.h, rows, out), self.h)
        return out

    def cache(self, layer, which, slot0, nslots, head_dim):
        out = np.empty((nslots, head_dim), np.float32)
        _check(self.L.g4_read_cache(self.h, layer, which, slot0, nslots, out), self.h)
        return out

    def ple(self, rows):
        """Per-layer inputs of the last forward's rows, [rows][35][256]."""
        out = np.empty((rows, NUM_LAYERS, 256), np.float32)
        _check(self.L.g4_read_ple(self.h, rows, out), self.h)
        return out

    def seq_cache(self, seq, layer, which, slot0, nslots, head_dim):
        out = np.empty((nslots, head_dim), np.float32)
        _check(self.L.g4_read_seq_cache(self.h, seq, layer, which, slot0, nslots, out), self.h)
        return out

    def stream(self):
        return self.L.g4_stream(self.h)

    def logits_async(self, row=0):
        """Enqueue logits without reading them back (no synchronisation)."""
        _check(self.L.g4_logits(self.h, row, None, None), self.h)

    def mark(self, slot):
        _check(self.L.g4_mark(self.h, slot), self.h)

    def elapsed(self, a, b):
        ms = C.c_float()
        _check(self.L.g4_elapsed(self.h, a, b, C.byref(ms)), self.h)
        return ms.value

    def profile_decode(self, token, pos):
        ms = (C.c_float * 3)()
        by = (C.c_double * 3)()
        n = (C.c_int * 3)()
        _check(self.L.g4_profile_decode(self.h, token, pos, ms, by, n), self.h)
        return list(ms), list(by), list(n)

    def trace_decode(self, token, pos, cap=512):
        """Persistent decode step with a device timeline: (types[n], t_ns[n, 6])."""
        types = (C.c_int * cap)()
        t = (C.c_double * (6 * cap))()
        n = C.c_int()
        _check(self.L.g4_trace_decode(self.h, token, pos, cap, types, t, C.byref(n)), self.h)
        k = min(n.value, cap)
        return np.array(types[:k], np.int32), np.array(t[:6 * k], np.float64).reshape(k, 6)

    # ---- multi-sequence serving ----
    def seq_alloc(self, max_seqs, max_context):
        _check(self.L.g4_seq_alloc(self.h, max_seqs, max_context), self.h)

    def forward_batch(self, seq_ids, token_lists, start_pos):
        """token_lists[i] (list/array of ids) for sequence seq_ids[i] from start_pos[i]."""
        seq_ids = np.ascontiguousarray(seq_ids, np.int32)
        lens = [len(t) for t in token_lists]
        offsets = np.zeros(len(lens) + 1, np.int32)
        offsets[1:] = np.cumsum(lens)
        toks = np.ascontiguousarray(np.concatenate([np.asarray(t, np.int32) for t in token_lists]), np.int32)
        _check(self.L.g4_forward_batch(self.h, len(lens), seq_ids, toks, offsets,
                                       np.ascontiguousarray(start_pos, np.int32)), self.h)
        self._batch_n = len(lens)

    def logits_batch(self, want_logits=False):
        """(logits [n][vocab] or None, argmax [n]) of the last forward_batch."""
        n = self._batch_n
        am = np.zeros(n, np.int32)
        lg = np.zeros((n, VOCAB), np.float32) if want_logits else None
        _check(self.L.g4_logits_batch(self.h, am.ctypes.data, lg.ctypes.data if lg is not None else None), self.h)
        return lg, am

    def launches_per_token(self):
        n = C.c_int()
        _check(self.L.g4_launches_per_token(self.h, C.byref(n)), self.h)
        return n.value

    def device_bytes(self):
        w, t = C.c_uint64(), C.c_uint64()
        _check(self.L.g4_device_bytes(self.h, C.byref(w), C.byref(t)), self.h)
        return w.value, t.value

    def close(self):
        if self.h:
            self.L.g4_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


# ---------------------------------------------------------------------------
# single-kernel entry points

def pack_matrix(w, s):
    """Row-major int8 [N][K] + scales [N][K/64] (fp16 bits) -> the .bin packed
    layout (exporter.py:304-316): [N/16][K/64][16 chunks][16 rows][4]."""
    N, K = w.shape
    G = K // 64
    wp = w.reshape(N // 16, 16, G, 16, 4).transpose(0, 2, 3, 1, 4).reshape(-1)
    sp = s.reshape(N // 16, 16, G).transpose(0, 2, 1).reshape(-1)
    return np.ascontiguousarray(wp, np.int8), np.ascontiguousarray(sp, np.uint16)


def quantize(x):
    L = load()
    x = np.ascontiguousarray(x, np.float32)
    rows, width = x.shape
    q = np.empty((rows, width), np.int8)
    s = np.empty((rows, width // 64), np.float32)
    _check(L.g4k_quantize(x, rows, width, q, s))
    return q, s


def linear(w_packed, s_packed, N, K, xq, xs, path=0, want_dots=False):
    L = load()
    xq = np.ascontiguousarray(xq, np.int8)
    xs = np.ascontiguousarray(xs, np.float32)
    T = xq.shape[0]
    out = np.empty((T, N), np.float32)
    dots = np.empty((T, N, K // 64), np.int32) if want_dots else None
    _check(L.g4k_linear(w_packed, s_packed, N, K, xq, xs, T, path, out,
                        dots.ctypes.data if dots is not None else None))
    return out, dots


def bench_gemm(N, K, T, path=3, iters=20):
    """(ms per launch, int8 ops per launch) of the prefill GEMM."""
    L = load()
    ms, ops = C.c_float(), C.c_double()
    _check(L.g4_bench_gemm(N, K, T, path, iters, C.byref(ms), C.byref(ops)))
    return ms.value, ops.value


def skinny_plan(N, K, T):
    """Launch geometry of the small-batch GEMM: dict(wm, nt, stages, threads, smem)."""
    L = load()
    v = [C.c_int() for _ in range(5)]
    _check(L.g4_skinny_plan(N, K, T, *[C.byref(x) for x in v]))
    return dict(zip(("wm", "nt", "stages", "threads", "smem"), (x.value for x in v)))


def bench_mma_i8(iters=20000):
    """(ms, int8 ops) of one launch of back-to-back tcgen05 kind::i8 MMAs on every SM."""
    L = load()
    ms, ops = C.c_float(), C.c_double()
    _check(L.g4_bench_mma_i8(iters, C.byref(ms), C.byref(ops)))
    return ms.value, ops.value


def bench_gemv(N, K, T=1, iters=200, pdl=True):
    """(ms per launch, algorithmic bytes per launch) of the decode GEMV."""
    L = load()
    ms, by = C.c_float(), C.c_double()
    _check(L.g4_bench_gemv(N, K, T, iters, int(pdl), C.byref(ms), C.byref(by)))
    return ms.value, by.value


ATTN_PREFILL, ATTN_STRICT, ATTN_DECODE, ATTN_ROWS, ATTN_PREFILL_TC = 0, 1, 2, 3, 4


def attention(qkv, hd, kring, vring, start_pos, cos_t, sin_t, mode=ATTN_PREFILL, splits=148, q_norm=None,
              k_norm=None, iters=0, quant=False):
    """One attention sub-layer on the GPU (g4k_attention). qkv[T][10*hd] raw
    q | k | v; kring / vring [ring][hd] are updated in place with the chunk's
    keys and values. Returns (out[T][8*hd], ms per call or None), and with
    quant=True (prefill modes) also the kernel's quantised rows (xq, xs)."""
    L = load()
    qkv = np.ascontiguousarray(qkv, np.float32)
    T = qkv.shape[0]
    out = np.empty((T, 8 * hd), np.float32)
    qn = None if q_norm is None else np.ascontiguousarray(q_norm, np.float32)
    kn = None if k_norm is None else np.ascontiguousarray(k_norm, np.float32)
    ms = C.c_float(0.0)
    xq = np.empty((T, 8 * hd), np.int8) if quant else None
    xs = np.empty((T, 8 * hd // 64), np.float32) if quant else None
    _check(L.g4k_attention(hd, kring.shape[0], T, start_pos, mode, splits, qkv,
                           None if qn is None else qn.ctypes.data, None if kn is None else kn.ctypes.data,
                           np.ascontiguousarray(cos_t, np.float32), np.ascontiguousarray(sin_t, np.float32),
                           kring, vring, out, None if xq is None else xq.ctypes.data,
                           None if xs is None else xs.ctypes.data, iters, C.byref(ms)))
    if quant:
        return out, (ms.value if iters else None), xq, xs
    return out, (ms.value if iters else None)


def attn_tc_plan(hd, T, start_pos, sms=148):
    """Host check of the tensor-core attention schedule (g4k_attn_tc_plan, no
    GPU work): returns (rc, S units, P V stages, P V CTAs, workspace bytes),
    rc 0 when every check holds."""
    L = load()
    f = L.g4k_attn_tc_plan
    f.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
    us, so, g1, wb = C.c_int(), C.c_int(), C.c_int(), C.c_ulonglong()
    rc = f(hd, T, start_pos, sms, C.byref(us), C.byref(so), C.byref(g1), C.byref(wb))
    return rc, us.value, so.value, g1.value, wb.value


def sample(logits, temperature, state):
    """Device sample() (g4k_sample) of one logits row; returns (token, state after)."""
    L = load()
    st, tok = C.c_ulonglong(state), C.c_int(0)
    _check(L.g4k_sample(np.ascontiguousarray(logits, np.float32), logits.size, temperature, C.byref(st),
                        C.byref(tok)))
    return tok.value, st.value


def rmsnorm_quant(x, w, eps=1e-6):
    L = load()
    x = np.ascontiguousarray(x, np.float32)
    rows = x.shape[0]
    y = np.empty_like(x)
    q = np.empty((rows, HIDDEN), np.int8)
    s = np.empty((rows, HIDDEN // 64), np.float32)
    _check(L.g4k_rmsnorm_quant(x, rows, np.ascontiguousarray(w, np.float32), eps, y.ctypes.data, q, s))
    return y, q, s
