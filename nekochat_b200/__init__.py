"""B200 (sm_100a) compute backend for NekoChat's inference engine.

The product is ``libneko_cuda.so`` (CUDA kernels + the C ABI of ``include/neko_cuda.h``); this package is a thin
ctypes layer over it so Python callers, the tests and ``bench.py`` go through exactly the entry points a C/C++
engine binds. It mirrors the engine's interfaces:

* :class:`ComputeBackend` - ``gpu::ComputeBackend`` (app/architecture/shared/cpp/gpu/compute.h:24-45): buffers,
  ``begin``/``dispatch``/``flush``/``submit_and_wait`` of the nine :class:`Kernel` ids with the shaders' parameter
  blocks.
* :mod:`nekochat_b200.ops` - single operators on torch CUDA tensors (device pointers).
* :class:`Model` - the native GPT-2 / Qwen3 runner (``Model::forward`` semantics plus batched decode).

There is no CPU fallback: importing works without a GPU, but every call needs the compiled library and a CUDA
device, and fails loudly otherwise.
"""
import ctypes as C
import enum
import os
import struct

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libneko_cuda.so")

_lib = None


class NekoError(RuntimeError):
    """A failed backend call (the engine's NekoError, app/architecture/shared/cpp/common.h:27-31)."""


class Kernel(enum.IntEnum):
    """gpu::Kernel (compute.h:17); the order is the engine's NEKO_KERNELS list."""
    Embed = 0
    LayerNorm = 1
    Matmul = 2
    KvStore = 3
    Attention = 4
    Rope = 5
    SiluMul = 6
    MatmulQ8 = 7
    MatmulQ4 = 8


F16, FP8, FP4 = 0, 1, 2
GELU, ACCUMULATE, BIAS = 1, 2, 4
ARCH_GPT2, ARCH_QWEN3 = 0, 1


def float_bits(f):
    """gpu::floatBits (compute.h:53-58): a float's bits as int32."""
    return struct.unpack("<i", struct.pack("<f", float(f)))[0]


class ModelConfig(C.Structure):
    """neko_model_config (include/neko_cuda.h)."""
    _fields_ = [("arch", C.c_int), ("vocab", C.c_int), ("embd", C.c_int), ("layers", C.c_int), ("heads", C.c_int),
                ("kv_heads", C.c_int), ("head_dim", C.c_int), ("ff", C.c_int), ("max_pos", C.c_int),
                ("eps", C.c_float), ("rope_theta", C.c_double), ("weight_format", C.c_int), ("context", C.c_int),
                ("max_seqs", C.c_int), ("max_rows", C.c_int)]


_vp, _i32p, _u8p, _f32p = C.c_void_p, C.POINTER(C.c_int32), C.POINTER(C.c_uint8), C.POINTER(C.c_float)

# name -> (restype, argtypes)
_SIGS = {
    "neko_last_error": (C.c_char_p, []),
    "neko_abi_version": (C.c_int, []),
    "neko_cuda_create": (_vp, [C.c_int, C.c_char_p, C.c_size_t]),
    "neko_cuda_destroy": (None, [_vp]),
    "neko_cuda_last_error": (C.c_char_p, [_vp]),
    "neko_cuda_name": (C.c_char_p, [_vp]),
    "neko_cuda_device_name": (C.c_int, [_vp, C.c_char_p, C.c_size_t]),
    "neko_cuda_max_buffer_bytes": (C.c_size_t, [_vp]),
    "neko_cuda_create_buffer": (_vp, [_vp, C.c_size_t, _vp, C.c_int]),
    "neko_cuda_upload": (C.c_int, [_vp, _vp, C.c_size_t, _vp, C.c_size_t]),
    "neko_cuda_download": (C.c_int, [_vp, _vp, C.c_size_t, _vp, C.c_size_t]),
    "neko_cuda_begin": (C.c_int, [_vp]),
    "neko_cuda_dispatch": (C.c_int, [_vp, C.c_int, C.POINTER(_vp), _i32p, C.c_uint32, C.c_uint32]),
    "neko_cuda_flush": (C.c_int, [_vp]),
    "neko_cuda_submit_and_wait": (C.c_int, [_vp]),
    "neko_cuda_buffer_size": (C.c_size_t, [_vp]),
    "neko_cuda_buffer_device_ptr": (_vp, [_vp]),
    "neko_row_bytes": (C.c_int64, [C.c_int, C.c_int]),
    "neko_op_quantize": (C.c_int, [C.c_int, _vp, C.c_int, C.c_int, C.c_int64, C.c_int, _vp, _vp]),
    "neko_op_dequantize": (C.c_int, [C.c_int, _vp, C.c_int, C.c_int, _vp, _vp]),
    "neko_op_matmul": (C.c_int, [C.c_int, _vp, C.c_int, C.c_int, _vp, C.c_int, _vp, _vp, C.c_int, C.c_int, C.c_int,
                                 _vp]),
    "neko_op_matmul_fused": (C.c_int, [C.c_int, _vp, C.c_int, C.c_int, _vp, C.c_int, C.c_int, _vp, _vp, C.c_float,
                                       C.c_int, _vp, _vp, C.c_int, C.c_int, C.c_int, _vp]),
    "neko_op_norm": (C.c_int, [_vp, _vp, _vp, _vp, C.c_int, C.c_int, C.c_float, _vp]),
    "neko_op_softmax": (C.c_int, [_vp, _vp, C.c_int, C.c_int, _vp]),
    "neko_op_attention": (C.c_int, [_vp, C.c_int, _vp, _vp, _vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _vp]),
    "neko_op_argmax": (C.c_int, [_vp, C.c_int, C.c_int, _vp, _vp]),
    "neko_op_sample": (C.c_int, [_vp, C.c_int, C.c_int, _vp, _vp, C.c_int, _vp, _vp, _vp, _vp]),
    "neko_op_fp8_block_dequant": (C.c_int, [_vp, C.c_int64, C.c_int64, _vp, C.c_int64, C.c_int64, _vp, _vp]),
    "neko_op_attention_noalloc": (C.c_int, [_vp, C.c_int, _vp, _vp, _vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                            _vp]),
    "neko_model_create": (_vp, [C.c_int, C.POINTER(ModelConfig), C.c_char_p, C.c_size_t]),
    "neko_model_destroy": (None, [_vp]),
    "neko_model_last_error": (C.c_char_p, [_vp]),
    "neko_model_set_tensor": (C.c_int, [_vp, C.c_char_p, _vp, C.c_int64, C.c_int64]),
    "neko_model_set_tensor_device": (C.c_int, [_vp, C.c_char_p, _vp, C.c_int64, C.c_int64]),
    "neko_model_set_tensor_fp8": (C.c_int, [_vp, C.c_char_p, _vp, C.c_int64, C.c_int64, _vp, C.c_int64,
                                            C.c_int64]),
    "neko_model_finalize": (C.c_int, [_vp]),
    "neko_model_set_stop": (C.c_int, [_vp, _vp, C.c_int, C.c_int]),
    "neko_model_host_logits": (_vp, [_vp, C.POINTER(C.c_size_t)]),
    "neko_model_generated": (C.c_int, [_vp, C.c_int, _vp, _vp, _vp]),
    "neko_model_forward": (C.c_int, [_vp, C.c_int, _vp, C.c_int, C.c_int, _vp]),
    "neko_model_decode": (C.c_int, [_vp, C.c_int, _vp, _vp, _vp, _vp, _vp]),
    "neko_model_stage": (C.c_int, [_vp, C.c_int, _vp, _vp, _vp]),
    "neko_model_step": (C.c_int, [_vp, C.c_int, C.c_int, _vp]),
    "neko_model_tokens": (C.c_int, [_vp, C.c_int, _vp, _vp]),
    "neko_model_memory": (C.c_int, [_vp, C.POINTER(C.c_int64), C.POINTER(C.c_int64), C.POINTER(C.c_int64)]),
    "neko_model_step_launches": (C.c_int, [_vp, C.c_int]),
    "neko_model_graph_kernels": (C.c_int, [_vp]),
    "neko_model_set_decode_kernel": (C.c_int, [_vp, C.c_int]),
    "neko_model_set_debug": (C.c_int, [_vp, C.c_int, C.c_int]),
    "neko_model_matrix": (C.c_int, [_vp, C.c_char_p, C.POINTER(C.c_void_p), C.POINTER(C.c_int),
                                    C.POINTER(C.c_int)]),
}


def lib():
    """The loaded libneko_cuda.so. Raises if it has not been built (there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise NekoError(f"{LIB_PATH} is missing: build it with `python nekochat_b200/build.py` "
                            "(or __graft_entry__.build())")
        l = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def exported_symbols():
    return sorted(_SIGS)


def check(rc, what="", ctx=None):
    if rc != 0:
        l = lib()
        msg = (l.neko_cuda_last_error(ctx) if ctx else l.neko_last_error()) or b""
        raise NekoError(f"{what}: status {rc}: {msg.decode(errors='replace')}")
    return rc


from .backend import Buffer, ComputeBackend  # noqa: E402
from .model import Model  # noqa: E402
from . import ops  # noqa: E402,F401


class Sampling(C.Structure):
    """neko_sampling (include/neko_cuda.h): SamplingParams without the seed."""
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int), ("top_p", C.c_float), ("repeat_penalty", C.c_float),
                ("repeat_last_n", C.c_int)]
