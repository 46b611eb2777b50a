"""The native GPT-2 / Qwen3 runner (``neko_model_*`` of include/neko_cuda.h).

``Model.forward`` has the semantics of the engine's ``Model::forward(tokens, T, pos0, logits)``
(app/architecture/shared/cpp/model.h:72) for one sequence slot; ``decode`` is the batched step the engine
cannot express; ``stage`` + ``step`` run greedy decoding entirely on the device (the bench's inner loop).
"""
import ctypes as C
import weakref

import numpy as np

from . import ARCH_GPT2, ARCH_QWEN3, ModelConfig, NekoError, lib
from . import workload


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _current_device():
    try:
        import torch
        return torch.cuda.current_device() if torch.cuda.is_available() else 0
    except ImportError:
        return 0


class Model:
    def __init__(self, shape, fmt, context, max_seqs=1, max_rows=64, device=None):
        """device: CUDA device index of the runner (default: torch's current device, else 0)."""
        if device is None:
            device = _current_device()
        self.device = device
        s = dict(shape)
        self.shape = s
        cfg = ModelConfig()
        cfg.arch = ARCH_QWEN3 if s["arch"] == "qwen3" else ARCH_GPT2
        cfg.vocab, cfg.embd, cfg.layers, cfg.heads = s["vocab"], s["embd"], s["layers"], s["heads"]
        cfg.kv_heads, cfg.head_dim, cfg.ff, cfg.max_pos = s["kv_heads"], s["head_dim"], s["ff"], s["max_pos"]
        cfg.eps, cfg.rope_theta, cfg.weight_format = s["eps"], s["rope_theta"], fmt
        cfg.context, cfg.max_seqs, cfg.max_rows = context, max_seqs, max_rows
        self.cfg = cfg
        self.vocab = s["vocab"]
        self.fmt = fmt
        self.context = context
        err = C.create_string_buffer(1024)
        self._views = []  # weak references to the host_logits views handed out
        self.h = lib().neko_model_create(device, C.byref(cfg), err, 1024)
        if not self.h:
            raise NekoError("neko_model_create: " + err.value.decode())

    def _check(self, rc, what):
        if rc != 0:
            raise NekoError(f"{what}: status {rc}: {lib().neko_model_last_error(self.h).decode()}")

    def set_tensor(self, name, array):
        a = np.ascontiguousarray(array, dtype=np.float32)
        rows, cols = (a.shape[0], int(np.prod(a.shape[1:]))) if a.ndim > 1 else (1, a.shape[0])
        self._check(lib().neko_model_set_tensor(self.h, name.encode(), _p(a), rows, cols), f"set_tensor {name}")

    def set_tensor_fp8(self, name, codes, scales):
        """An FP8 (E4M3) checkpoint weight: codes uint8 [rows][cols] and its block scales [sR][sC] (any float
        dtype, widened to f32; a 0-d or 1-element scale is per tensor), dequantized and quantized on the GPU."""
        q = np.ascontiguousarray(codes, dtype=np.uint8)
        sc = np.ascontiguousarray(scales, dtype=np.float32)
        s2 = sc.reshape(sc.shape[0] if sc.ndim else 1, -1)
        self._check(lib().neko_model_set_tensor_fp8(self.h, name.encode(), _p(q), q.shape[0], q.shape[1], _p(s2),
                                                    s2.shape[0], s2.shape[1]), f"set_tensor_fp8 {name}")

    def set_tensor_device(self, name, t):
        """t: a contiguous float32 CUDA tensor on the model's device."""
        if t.device.type != "cuda" or t.device.index != self.device:
            raise NekoError(f"set_tensor_device {name}: tensor on {t.device}, model on cuda:{self.device}")
        rows, cols = (t.shape[0], t.numel() // t.shape[0]) if t.dim() > 1 else (1, t.shape[0])
        self._check(lib().neko_model_set_tensor_device(self.h, name.encode(), C.c_void_p(t.data_ptr()), rows, cols),
                    f"set_tensor_device {name}")

    def load_random_device(self, seed=0, host_copy=None, f16_exact=False):
        """Random-init weights generated on the GPU (torch, seeded): N(0, 0.02) matrices, unit norm gains, zero
        biases, in workload.tensor_specs order. host_copy(name, f16 numpy array) receives each tensor for a CPU
        baseline checkpoint when given. f16_exact rounds every tensor through f16 before it is loaded, so the
        runner's weights equal the f16 checkpoint written from host_copy (parity runs against the reference)."""
        import torch
        dev = torch.device("cuda", self.device)
        g = torch.Generator(device=dev).manual_seed(seed)
        for name, shp, kind in workload.tensor_specs(self.shape):
            if kind == "w":
                t = torch.randn(shp, generator=g, device=dev, dtype=torch.float32).mul_(0.02)
            elif kind == "g":
                t = torch.ones(shp, device=dev, dtype=torch.float32)
            else:
                t = torch.zeros(shp, device=dev, dtype=torch.float32)
            if f16_exact:
                t = t.half().float()
            self.set_tensor_device(name, t)
            if host_copy is not None:
                host_copy(name, t.half().cpu().numpy())
            del t
        self._check(lib().neko_model_finalize(self.h), "finalize")
        return self

    def load(self, tensors):
        """tensors: iterable of (name, float32 array), e.g. workload.weights(shape), or (name, uint8 codes,
        scales) for an FP8 (E4M3) checkpoint weight with its block scales."""
        for item in tensors:
            if len(item) == 3:
                self.set_tensor_fp8(*item)
            else:
                self.set_tensor(*item)
        self._check(lib().neko_model_finalize(self.h), "finalize")
        return self

    def forward(self, tokens, pos0, slot=0):
        """Model::forward: last token's logits (vocab floats)."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty(self.vocab, np.float32)
        self._check(lib().neko_model_forward(self.h, slot, _p(t), len(t), pos0, _p(out)), "forward")
        return out

    def prefill(self, tokens, slot=0, pos0=0, chunk=None):
        """Runs a prompt in chunks of <= chunk tokens (Engine::generate's prefill loop, engine.cpp:98-112; at most
        max_rows, 64 like Model::kMaxBatch by default) and returns the last token's logits."""
        chunk = min(chunk or 64, self.cfg.max_rows)
        tokens = np.asarray(tokens, np.int32)
        logits = None
        for i in range(0, len(tokens), chunk):
            logits = self.forward(tokens[i:i + chunk], pos0 + i, slot)
        return logits

    def decode(self, slots, tokens, pos, want_logits=True, out=None):
        """One decode step for n sequences. Returns (logits [n][vocab] or None, argmax [n]). `out`: a float32
        C-contiguous array of at least n * vocab floats to receive the logits, reused across steps the way the
        engine reuses its logits vector (engine.cpp:56)."""
        if not self.h:
            raise NekoError("decode: the model is closed")
        slots = np.ascontiguousarray(slots, dtype=np.int32)
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        pos = np.ascontiguousarray(pos, dtype=np.int32)
        n = len(slots)
        if out is not None and want_logits:
            if out.dtype != np.float32 or not out.flags.c_contiguous or out.size < n * self.vocab:
                raise NekoError("decode: out must be a C-contiguous float32 array of n * vocab floats")
            logits = out.reshape(-1)[:n * self.vocab].reshape(n, self.vocab)
        else:
            logits = np.empty((n, self.vocab), np.float32) if want_logits else None
        am = np.empty(n, np.int32)
        self._check(lib().neko_model_decode(self.h, n, _p(slots), _p(tokens), _p(pos), _p(logits), _p(am)),
                    "decode")
        return logits, am

    def stage(self, slots, tokens, pos):
        slots = np.ascontiguousarray(slots, dtype=np.int32)
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        pos = np.ascontiguousarray(pos, dtype=np.int32)
        self._check(lib().neko_model_stage(self.h, len(slots), _p(slots), _p(tokens), _p(pos)), "stage")

    def step(self, n, max_pos, stream=None):
        """Enqueues one greedy decode step of the n staged sequences on `stream` (a cudaStream_t handle)."""
        self._check(lib().neko_model_step(self.h, n, max_pos, C.c_void_p(stream) if stream else None), "step")

    def tokens(self, n):
        t = np.empty(n, np.int32)
        p = np.empty(n, np.int32)
        self._check(lib().neko_model_tokens(self.h, n, _p(t), _p(p)), "tokens")
        return t, p

    def host_logits(self, rows):
        """A [rows][vocab] float32 view of the runner's pinned logits buffer: as decode's `out` it takes the
        logits with no second host copy, and the next call overwrites it. The buffer belongs to the runner: after
        close() the model no longer runs, and the runner (with this buffer) is destroyed only once every view
        handed out here has been released, so a view never points at freed memory."""
        if not self.h:
            raise NekoError("host_logits: the model is closed")
        n = C.c_size_t(0)
        ptr = lib().neko_model_host_logits(self.h, C.byref(n))
        if not ptr or rows * self.vocab > n.value:
            raise NekoError("host_logits: buffer unavailable or too small")
        view = np.ctypeslib.as_array(C.cast(ptr, C.POINTER(C.c_float)), shape=(rows, self.vocab)).view(np.ndarray)
        self._views.append(weakref.ref(view))
        return view

    def set_stop(self, stop_ids, max_new):
        """Stop ids and token budget for the device greedy loop (Engine::generate's loop on the device);
        max_new = 0 turns it off."""
        ids = np.ascontiguousarray(stop_ids, dtype=np.int32)
        self._check(lib().neko_model_set_stop(self.h, _p(ids) if len(ids) else None, len(ids), max_new), "set_stop")
        self._max_new = max_new

    def generated(self, n):
        """(list of n int32 arrays of generated tokens, reasons: 0 max_new, 1 stop id, -1 running)."""
        L = getattr(self, "_max_new", 0)
        t = np.empty((n, L), np.int32)
        c = np.empty(n, np.int32)
        r = np.empty(n, np.int32)
        self._check(lib().neko_model_generated(self.h, n, _p(t), _p(c), _p(r)), "generated")
        return [t[i, :c[i]].copy() for i in range(n)], r

    def set_debug(self, layers, stage=0):
        """Model::setDebugLayers(n, stage) (model.h:101): forward() then returns the hidden states after n layers
        (stage 0) or the intermediate after `stage` inside layer n; n < 0 restores logits."""
        self._check(lib().neko_model_set_debug(self.h, layers, stage), "set_debug")

    def hidden(self, tokens, pos0, slot=0, width=None):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        width = width or self.shape["embd"]
        out = np.empty(max(self.vocab, len(t) * width), np.float32)
        self._check(lib().neko_model_forward(self.h, slot, _p(t), len(t), pos0, _p(out)), "forward")
        return out[:len(t) * width].reshape(len(t), width)

    def memory(self):
        w, kv, ws = C.c_int64(), C.c_int64(), C.c_int64()
        self._check(lib().neko_model_memory(self.h, C.byref(w), C.byref(kv), C.byref(ws)), "memory")
        return dict(weights=w.value, kv=kv.value, workspace=ws.value)

    def step_launches(self, n):
        return int(lib().neko_model_step_launches(self.h, n))

    def graph_kernels(self):
        """Kernel nodes of the most recently captured step graph."""
        return int(lib().neko_model_graph_kernels(self.h))

    def set_decode_kernel(self, enable):
        """Run decode steps of 1..4 sequences as one persistent kernel (True, the default) or as the per-operator
        kernel chain (False); 2 makes the kernel's next steps hit a wait that runs out (timeout test). Returns
        whether the single-kernel path is available for this model."""
        rc = int(lib().neko_model_set_decode_kernel(self.h, int(enable)))
        self._check(min(rc, 0), "set_decode_kernel")
        return rc == 1

    def matrix(self, which):
        """(device pointer, rows, cols, format) of one packed matrix: 'layers.L.wqkv|wo|wgu|wdown' or 'head'."""
        p, r, c = C.c_void_p(), C.c_int(), C.c_int()
        fmt = lib().neko_model_matrix(self.h, which.encode(), C.byref(p), C.byref(r), C.byref(c))
        if fmt < 0:
            raise NekoError(f"matrix {which}: {lib().neko_model_last_error(self.h).decode()}")
        return p.value, r.value, c.value, fmt

    def close(self):
        """Ends the model. The runner is destroyed now, or, while host_logits views are still referenced, when
        the last of them is released."""
        if not self.h:
            return
        h, self.h = self.h, None
        alive = [v for v in (r() for r in getattr(self, "_views", [])) if v is not None]
        self._views = []
        if not alive:
            lib().neko_model_destroy(h)
            return
        left = [len(alive)]

        def release():
            left[0] -= 1
            if left[0] == 0:
                lib().neko_model_destroy(h)
        for v in alive:
            weakref.finalize(v, release)

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def decode_kernel_launches(shape, fmt):
    """Kernel launches of a decode step on the single decode kernel: 1, or 2 when the LM head runs as its own
    launch (FP8 heads with a hidden size that is a multiple of 128: the decode kernel, then the head GEMV with the
    final norm, the greedy argmax and the token / position finalize)."""
    return 2 if fmt == 1 and shape["embd"] % 128 == 0 else 1


def build(shape_name, fmt, context, max_seqs=1, max_rows=64, seed=0, perturb=False, device=None):
    s = workload.shape(shape_name)
    m = Model(s, fmt, context, max_seqs, max_rows, device)
    return m.load(workload.weights(s, seed, perturb))
