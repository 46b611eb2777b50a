"""ctypes access to the two CPU oracles. TEST INFRASTRUCTURE ONLY.

* ``Restatement`` loads ``oracle/_build/liboracle.so``: my C restatement of the reference's hot-path arithmetic
  (``oracle/neko_oracle.c``), pinned to the reference by ``tests/golden`` and by the live comparison tests.
* ``Reference`` loads ``oracle/_ref/libneko_ref.so``: the reference's own C++ CPU engine compiled from its
  sources (``oracle/Makefile``), through the extern "C" shim in ``oracle/ref_shim.cpp``.

Only tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import this module: it is
the checker, never the thing measured or shipped.

Both expose the same op API, so a test can run either one:
``quantize``, ``dequantize``, ``matmul``, ``layer_norm``, ``rms_norm``, ``rope``, ``silu_mul``, ``gelu``,
``store_kv``, ``attention``, plus ``softmax_rows``/``rope_table``/``embed`` on the restatement.
Weight formats: 0 = F16, 1 = FP8 (E4M3 blocks), 2 = FP4 (E2M1 blocks) (quant.h:19).
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
F16, FP8, FP4 = 0, 1, 2
GELU, ACCUMULATE = 1, 2

_f = C.POINTER(C.c_float)
_u8 = C.POINTER(C.c_uint8)
_u16 = C.POINTER(C.c_uint16)
_i32 = C.POINTER(C.c_int)


def _p(a, t):
    return None if a is None else a.ctypes.data_as(t)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


class _Ops:
    prefix = ""

    def _fn(self, name, res, *args):
        f = getattr(self.lib, self.prefix + name)
        f.restype = res
        f.argtypes = list(args)
        return f

    def row_bytes(self, fmt, cols):
        raise NotImplementedError

    def quantize(self, fmt, w):
        """[rows][cols] f32 -> [rows][row_bytes] uint8 in the engine's row format (quant.cpp:255-279)."""
        w = _c(w, np.float32)
        rows, cols = w.shape
        out = np.zeros((rows, self.row_bytes(fmt, cols)), np.uint8)
        self._quantize(fmt, rows, cols, w, out)
        return out

    def dequantize(self, fmt, q, cols):
        q = _c(q, np.uint8)
        rows = q.shape[0]
        out = np.zeros((rows, cols), np.float32)
        self._dequantize(fmt, rows, cols, q, out)
        return out

    def matmul(self, fmt, x, q, K, bias=None, y=None, y_stride=None, flags=0, n_off=0):
        """y[t][n_off + n] (+)= act(x[t] . W[n] + bias[n]) (cpu_ops.h:17-23)."""
        x = _c(x, np.float32).reshape(-1, K)
        q = _c(q, np.uint8)
        rows = q.shape[0]
        T = x.shape[0]
        y_stride = rows if y_stride is None else y_stride
        if y is None:
            y = np.zeros((T, y_stride), np.float32)
        assert y.dtype == np.float32 and y.flags.c_contiguous
        b = None if bias is None else _c(bias, np.float32)
        flat = y.reshape(-1)
        view = flat[n_off:]
        self._matmul(fmt, x, T, K, q, rows, b, view, y_stride, flags)
        return y


class Restatement(_Ops):
    prefix = "no_"

    def __init__(self, path=None):
        path = path or os.path.join(HERE, "_build", "liboracle.so")
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is missing: run `make -C oracle oracle` (or __graft_entry__.build())")
        self.lib = C.CDLL(path)
        self._rb = self._fn("row_bytes", C.c_size_t, C.c_int, C.c_int)
        self._q = self._fn("quantize_rows", None, C.c_int, C.c_int, C.c_int, _f, _u8)
        self._dq = self._fn("dequantize_rows", None, C.c_int, C.c_int, C.c_int, _u8, _f)
        self._mm = self._fn("matmul", None, C.c_int, _f, C.c_int, C.c_int, _u8, C.c_int, _f, _f, C.c_int, C.c_int)
        self._ln = self._fn("layer_norm", None, _f, _f, _f, _f, C.c_int, C.c_int, C.c_float)
        self._rms = self._fn("rms_norm", None, _f, _f, _f, C.c_int, C.c_int, C.c_float)
        self._rope = self._fn("rope", None, _f, C.c_int, C.c_int, _f)
        self._silu = self._fn("silu_mul", None, _f, _f, C.c_int, C.c_int)
        self._gelu = self._fn("gelu", C.c_float, C.c_float)
        self._kv = self._fn("store_kv", None, _f, _f, C.c_int, _u16, _u16, C.c_int, C.c_int, C.c_int)
        self._att = self._fn("attention", None, _f, C.c_int, _u16, _u16, _f, C.c_int, C.c_int, C.c_int, C.c_int,
                             C.c_int)
        self._sm = self._fn("softmax_rows", None, _f, _f, C.c_int, C.c_int)
        self._rt = self._fn("rope_table", None, C.c_int, C.c_int, C.c_double, _f)
        self._emb = self._fn("embed", None, C.c_int, _u8, C.c_int, _i32, C.c_int, _f, C.c_int, _f)
        self._am = self._fn("argmax", C.c_int, _f, C.c_int)
        self._h = self._fn("f32_to_f16", C.c_uint16, C.c_float)
        self._hf = self._fn("f16_to_f32", C.c_float, C.c_uint16)

    def row_bytes(self, fmt, cols):
        return int(self._rb(fmt, cols))

    def _quantize(self, fmt, rows, cols, w, out):
        self._q(fmt, rows, cols, _p(w, _f), _p(out, _u8))

    def _dequantize(self, fmt, rows, cols, q, out):
        self._dq(fmt, rows, cols, _p(q, _u8), _p(out, _f))

    def _matmul(self, fmt, x, T, K, q, rows, b, view, y_stride, flags):
        self._mm(fmt, _p(x, _f), T, K, _p(q, _u8), rows, _p(b, _f), _p(view, _f), y_stride, flags)

    def layer_norm(self, x, g, b, eps):
        x = _c(x, np.float32)
        C_ = x.shape[-1]
        y = np.empty_like(x)
        self._ln(_p(x, _f), _p(y, _f), _p(_c(g, np.float32), _f), _p(_c(b, np.float32), _f), x.size // C_, C_, eps)
        return y

    def rms_norm(self, x, w, eps):
        x = _c(x, np.float32)
        C_ = x.shape[-1]
        y = np.empty_like(x)
        self._rms(_p(x, _f), _p(y, _f), _p(_c(w, np.float32), _f), x.size // C_, C_, eps)
        return y

    def rope(self, x, n_heads, hd, cs_row):
        """In place on n_heads consecutive heads of x (a 1-D float32 view); cs_row = hd/2 (cos, sin) pairs."""
        cs = _c(cs_row, np.float32)
        self._rope(_p(x, _f), n_heads, hd, _p(cs, _f))

    def silu_mul(self, h, I):
        h = _c(h, np.float32).reshape(-1, 2 * I)
        out = np.empty((h.shape[0], I), np.float32)
        self._silu(_p(h, _f), _p(out, _f), h.shape[0], I)
        return out

    def gelu(self, v):
        return float(self._gelu(float(v)))

    def store_kv(self, k, v, src_stride, kc, vc, width, T, pos0):
        self._kv(_p(k, _f), _p(v, _f), src_stride, _p(kc, _u16), _p(vc, _u16), width, T, pos0)

    def attention(self, q, q_stride, kc, vc, T, n_head, n_kv, hd, pos0):
        out = np.empty((T, n_head * hd), np.float32)
        self._att(_p(_c(q, np.float32), _f), q_stride, _p(kc, _u16), _p(vc, _u16), _p(out, _f), T, n_head, n_kv, hd,
                  pos0)
        return out

    def softmax_rows(self, x):
        x = _c(x, np.float32)
        y = np.empty_like(x)
        self._sm(_p(x, _f), _p(y, _f), x.size // x.shape[-1], x.shape[-1])
        return y

    def rope_table(self, ctx, hd, theta):
        out = np.empty((ctx, hd), np.float32)
        self._rt(ctx, hd, float(theta), _p(out, _f))
        return out

    def embed(self, fmt, table, cols, tokens, wpe=None, pos0=0):
        tokens = _c(tokens, np.int32)
        x = np.empty((len(tokens), cols), np.float32)
        w = None if wpe is None else _c(wpe, np.float32)
        self._emb(fmt, _p(_c(table, np.uint8), _u8), cols, _p(tokens, _i32), len(tokens), _p(w, _f), pos0, _p(x, _f))
        return x

    def argmax(self, x):
        x = _c(x, np.float32)
        return int(self._am(_p(x, _f), x.size))

    def f32_to_f16(self, a):
        a = _c(a, np.float32).reshape(-1)
        return np.array([self._h(float(v)) for v in a], np.uint16)


def host_isa_level():
    """The x86-64 ISA level of this host's CPU from /proc/cpuinfo: 4 (AVX-512 F/BW/CD/DQ/VL), 3 (AVX2 + FMA +
    BMI2), else 1."""
    try:
        with open("/proc/cpuinfo") as f:
            flags = next((ln.split(":", 1)[1].split() for ln in f if ln.startswith("flags")), [])
    except OSError:
        return 1
    fl = set(flags)
    if {"avx2", "fma", "bmi2", "movbe"} <= fl:
        if {"avx512f", "avx512bw", "avx512cd", "avx512dq", "avx512vl"} <= fl:
            return 4
        return 3
    return 1


def native_build():
    """(library name, description) of the reference CPU engine built for timing on this host: the x86-64-v4 or
    -v3 build of oracle/Makefile's ref_native target, or the portable checker build when neither fits."""
    lvl = host_isa_level()
    for v in (4, 3):
        name = f"libneko_ref_native_v{v}.so"
        if lvl >= v and os.path.exists(os.path.join(HERE, "_ref", name)):
            return name, f"-O3 -march=x86-64-v{v} (FMA contraction on)"
    return "libneko_ref.so", "-O3, no -march, -ffp-contract=off (portable checker build)"


class Reference(_Ops):
    """The reference engine compiled from its own sources (oracle/_ref). cuda=True loads the variant whose
    first GPU backend slot is the B200 backend (needs nekochat_b200/libneko_cuda.so and a GPU)."""

    prefix = "ref_"

    def __init__(self, cuda=False, path=None, native=False):
        """native=True loads the timing build for this host's ISA level (native_build()) instead of the
        deterministic checker; use it only to time the reference, never to check results."""
        name = "libneko_ref_cuda.so" if cuda else "libneko_ref.so"
        if native and not cuda and path is None:
            name = native_build()[0]
        self.build = name
        path = path or os.path.join(HERE, "_ref", name)
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is missing: build it with `make -C oracle` where the reference exists")
        self.lib = C.CDLL(path)
        self.cuda = cuda
        self._err = self._fn("last_error", C.c_char_p)
        self._rb = self._fn("quant_row_bytes", C.c_long, C.c_int, C.c_int)
        self._q = self._fn("quantize_matrix", C.c_int, C.c_int, C.c_int, C.c_int, _f, _u8, C.c_int)
        self._dq = self._fn("dequantize_rows", C.c_int, C.c_int, C.c_int, C.c_int, _u8, _f)
        self._mm = self._fn("matmul", C.c_int, C.c_int, _f, C.c_int, C.c_int, _u8, C.c_int, _f, _f, C.c_int, C.c_int,
                            C.c_int)
        self._ln = self._fn("layer_norm", None, _f, _f, _f, _f, C.c_int, C.c_int, C.c_float)
        self._rms = self._fn("rms_norm", None, _f, _f, _f, C.c_int, C.c_int, C.c_float)
        self._rope = self._fn("rope", None, _f, C.c_int, C.c_int, _f)
        self._silu = self._fn("silu_mul", None, _f, _f, C.c_int, C.c_int)
        self._gelu = self._fn("gelu", C.c_float, C.c_float)
        self._kv = self._fn("store_kv", None, _f, _f, C.c_int, _u16, _u16, C.c_int, C.c_int, C.c_int)
        self._att = self._fn("attention", None, _f, C.c_int, _u16, _u16, _f, C.c_int, C.c_int, C.c_int, C.c_int,
                             C.c_int, C.c_int)
        self._h = self._fn("f32_to_f16", C.c_uint16, C.c_float)
        self._load = self._fn("model_load", C.c_void_p, C.c_char_p, C.c_int, C.c_int, C.c_int)
        self._free = self._fn("model_free", None, C.c_void_p)
        self._fwd = self._fn("model_forward", C.c_int, C.c_void_p, _i32, C.c_int, C.c_int, _f)
        self._dbg = self._fn("model_set_debug", None, C.c_void_p, C.c_int, C.c_int)
        self._vocab = self._fn("model_vocab", C.c_int, C.c_void_p)
        self._ctx = self._fn("model_context", C.c_int, C.c_void_p)
        self._be = self._fn("model_backend", C.c_int, C.c_void_p, C.c_char_p, C.c_int)
        self._hw = self._fn("hardware_threads", C.c_int)
        if cuda:
            self._st = self._fn("selftest_cuda", C.c_int, C.c_char_p, C.c_int)
        self.threads = 1

    def error(self):
        return self._err().decode()

    def _check(self, rc):
        if rc != 0:
            raise RuntimeError(self.error())

    def row_bytes(self, fmt, cols):
        return int(self._rb(fmt, cols))

    def _quantize(self, fmt, rows, cols, w, out):
        self._check(self._q(fmt, rows, cols, _p(w, _f), _p(out, _u8), 0))

    def _dequantize(self, fmt, rows, cols, q, out):
        self._check(self._dq(fmt, rows, cols, _p(q, _u8), _p(out, _f)))

    def _matmul(self, fmt, x, T, K, q, rows, b, view, y_stride, flags):
        self._check(self._mm(fmt, _p(x, _f), T, K, _p(q, _u8), rows, _p(b, _f), _p(view, _f), y_stride, flags,
                             self.threads))

    layer_norm = Restatement.layer_norm
    rms_norm = Restatement.rms_norm
    rope = Restatement.rope
    silu_mul = Restatement.silu_mul
    gelu = Restatement.gelu
    store_kv = Restatement.store_kv
    f32_to_f16 = Restatement.f32_to_f16

    def attention(self, q, q_stride, kc, vc, T, n_head, n_kv, hd, pos0):
        out = np.empty((T, n_head * hd), np.float32)
        self._att(_p(_c(q, np.float32), _f), q_stride, _p(kc, _u16), _p(vc, _u16), _p(out, _f), T, n_head, n_kv, hd,
                  pos0, self.threads)
        return out

    def hardware_threads(self):
        return int(self._hw())

    def selftest_cuda(self):
        buf = C.create_string_buffer(4096)
        rc = self._st(buf, 4096)
        return rc, buf.value.decode()

    def load_model(self, model_dir, fmt, threads=0, backend=3):
        """loadModel(readModelType(dir), dir, {backend, threads, weights=fmt}) (model.cpp:175-193).
        backend: 0 = Auto (GPU first), 3 = CPU."""
        h = self._load(model_dir.encode(), backend, fmt, threads)
        if not h:
            raise RuntimeError(self.error())
        return RefModel(self, h)

    def sample(self, logits, history, temperature, top_k, top_p, repeat_penalty, repeat_last_n, seed):
        """Sampler::sample with a fixed seed; returns (token, the logits after the repetition penalty)."""
        x = np.ascontiguousarray(logits, dtype=np.float32).copy()
        h = np.ascontiguousarray(history, dtype=np.int32)
        f = self._fn("sample", C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_float, C.c_int, C.c_float,
                     C.c_float, C.c_int, C.c_ulonglong)
        t = f(x.ctypes.data, len(x), h.ctypes.data, len(h), temperature, top_k, top_p, repeat_penalty,
              repeat_last_n, seed)
        return int(t), x

    def tensor_f32(self, path, name, count):
        """TensorStore::toF32 of one tensor of a safetensors file (FP8 weights dequantized with their scales)."""
        out = np.empty(count, np.float32)
        f = self._fn("tensor_f32", C.c_long, C.c_char_p, C.c_char_p, C.c_void_p, C.c_long)
        n = f(path.encode(), name.encode(), out.ctypes.data, count)
        if n < 0:
            raise RuntimeError(self.error())
        return out[:n]

    def sampler_draw(self, seed):
        """The uniform value behind the first draw of a Sampler seeded with `seed`."""
        return float(self._fn("sampler_draw", C.c_double, C.c_ulonglong)(seed))

class RefModel:
    def __init__(self, ref, h):
        self.ref, self.h = ref, h
        self.vocab = int(ref._vocab(h))
        self.context = int(ref._ctx(h))

    def forward(self, tokens, pos0, out_width=None):
        """Model::forward(tokens, T, pos0, logits) (model.h:72): the last token's logits, or the debug dump."""
        tokens = _c(tokens, np.int32)
        n = out_width if out_width is not None else self.vocab
        out = np.zeros(max(n, self.vocab), np.float32)
        self.ref._check(self.ref._fwd(self.h, _p(tokens, _i32), len(tokens), pos0, _p(out, _f)))
        return out[:n]

    def set_debug(self, layers, stage=0):
        self.ref._dbg(self.h, layers, stage)

    def backend(self):
        buf = C.create_string_buffer(4096)
        self.ref._be(self.h, buf, 4096)
        return buf.value.decode()

    def close(self):
        if self.h:
            self.ref._free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
