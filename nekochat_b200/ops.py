"""Single operators of the C ABI (``neko_op_*``) on torch CUDA tensors. torch is only the device allocator and
stream here; the arithmetic is the library's."""
import ctypes as C

from . import NekoError, check, lib


def _ptr(t):
    if t is None:
        return None
    if not t.is_cuda or not t.is_contiguous():
        raise NekoError("ops take contiguous CUDA tensors")
    return C.c_void_p(t.data_ptr())


def _stream():
    import torch
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def row_bytes(fmt, cols):
    """quantRowBytes (quant.cpp:199-208)."""
    return int(lib().neko_row_bytes(fmt, cols))


def quantize(fmt, w, transpose_f16=False):
    """quantizeMatrix (quant.cpp:255-279) on the GPU. w: [rows][cols] float32 CUDA tensor (or [cols][rows] with
    transpose_f16, the Conv1D layout). Returns [rows][row_bytes] uint8."""
    import torch
    if transpose_f16:
        cols, rows = w.shape
    else:
        rows, cols = w.shape
    out = torch.zeros((rows, row_bytes(fmt, cols)), dtype=torch.uint8, device=w.device)
    ld = w.shape[1]
    check(lib().neko_op_quantize(fmt, _ptr(w), rows, cols, ld, 1 if transpose_f16 else 0, _ptr(out), _stream()),
          "quantize")
    return out


def dequantize(fmt, q, cols):
    """QMatrix::dequantizeRow for every row (quant.cpp:230-253)."""
    import torch
    out = torch.empty((q.shape[0], cols), dtype=torch.float32, device=q.device)
    check(lib().neko_op_dequantize(fmt, _ptr(q), q.shape[0], cols, _ptr(out), _stream()), "dequantize")
    return out


def matmul(fmt, x, q, K, bias=None, y=None, y_stride=None, n_off=0, flags=0):
    """cpu::matmul semantics (cpu_ops.h:17-23): y[t][n_off + n] (+)= act(x[t] . W[n] + bias[n])."""
    import torch
    T = x.numel() // K
    rows = q.shape[0]
    y_stride = rows if y_stride is None else y_stride
    if y is None:
        y = torch.zeros((T, y_stride), dtype=torch.float32, device=x.device)
    if bias is not None:
        flags |= 4
    check(lib().neko_op_matmul(fmt, _ptr(x), T, K, _ptr(q), rows, _ptr(bias), _ptr(y), y_stride, n_off, flags,
                               _stream()), "matmul")
    return y


def matmul_fused(fmt, x, q, K, rows, norm=0, gamma=None, beta=None, eps=1e-6, swiglu=False, bias=None, y=None,
                 y_stride=None, n_off=0, flags=0):
    """Norm prologue (0 none, 1 RMSNorm, 2 LayerNorm) + matmul, or the SwiGLU pair (q holds 2 * rows rows)."""
    import torch
    T = x.numel() // K
    y_stride = rows if y_stride is None else y_stride
    if y is None:
        y = torch.zeros((T, y_stride), dtype=torch.float32, device=x.device)
    if bias is not None:
        flags |= 4
    check(lib().neko_op_matmul_fused(fmt, _ptr(x), T, K, _ptr(q), rows, norm, _ptr(gamma), _ptr(beta), eps,
                                     1 if swiglu else 0, _ptr(bias), _ptr(y), y_stride, n_off, flags, _stream()),
          "matmul_fused")
    return y


def norm(x, gamma, beta=None, eps=1e-6):
    """cpu::rmsNorm (beta None) / cpu::layerNorm over the last dimension."""
    import torch
    C_ = x.shape[-1]
    y = torch.empty_like(x)
    check(lib().neko_op_norm(_ptr(x), _ptr(y), _ptr(gamma), _ptr(beta), x.numel() // C_, C_, eps, _stream()), "norm")
    return y


def softmax(x):
    import torch
    C_ = x.shape[-1]
    y = torch.empty_like(x)
    check(lib().neko_op_softmax(_ptr(x), _ptr(y), x.numel() // C_, C_, _stream()), "softmax")
    return y


def argmax(x):
    import torch
    C_ = x.shape[-1]
    out = torch.empty(x.numel() // C_, dtype=torch.int32, device=x.device)
    check(lib().neko_op_argmax(_ptr(x), x.numel() // C_, C_, _ptr(out), _stream()), "argmax")
    return out


def sample(logits, u, temperature=0.8, top_k=40, top_p=0.95, repeat_penalty=1.1, repeat_last_n=64, history=None,
           hist_len=None):
    """Sampler::sample per row of logits [rows][V] (modified in place by the repetition penalty) with the uniform
    draws u [rows] (float64); history [rows][S] int32 with hist_len [rows] valid tokens. Returns int32 [rows]."""
    import torch
    from . import Sampling
    rows, V = logits.shape
    out = torch.empty(rows, dtype=torch.int32, device=logits.device)
    sp = Sampling(temperature, top_k, top_p, repeat_penalty, repeat_last_n)
    check(lib().neko_op_sample(_ptr(logits), rows, V, _ptr(history) if history is not None else None,
                               _ptr(hist_len) if hist_len is not None else None,
                               history.shape[1] if history is not None else 0,
                               _ptr(u) if u is not None else None, C.byref(sp), _ptr(out), _stream()), "sample")
    return out


def fp8_block_dequant(codes, scales):
    """An FP8 (E4M3) checkpoint weight as f32 (TensorStore::toF32, tensor_store.cpp:543-571, 578-590): codes
    uint8 [rows][cols], scales float32 [sR][sC] (the "_scale_inv" / "_scale" tensor; 1 x 1 per tensor), both CUDA
    tensors. Returns float32 [rows][cols]."""
    import torch
    rows, cols = codes.shape
    s2 = scales.reshape(scales.shape[0] if scales.dim() else 1, -1)
    out = torch.empty((rows, cols), dtype=torch.float32, device=codes.device)
    check(lib().neko_op_fp8_block_dequant(_ptr(codes), rows, cols, _ptr(scales), s2.shape[0], s2.shape[1], _ptr(out),
                                          _stream()), "fp8_block_dequant")
    return out


def attention(q, q_stride, k_cache, v_cache, T, n_head, n_kv, hd, pos0):
    """cpu::attention (cpu_ops.cpp:544-575) over engine-layout caches [ctx][n_kv * hd] (int16/uint16 f16 bits)."""
    import torch
    out = torch.empty((T, n_head * hd), dtype=torch.float32, device=q.device)
    check(lib().neko_op_attention(_ptr(q), q_stride, _ptr(k_cache), _ptr(v_cache), _ptr(out), T, n_head, n_kv, hd,
                                  pos0, _stream()), "attention")
    return out
