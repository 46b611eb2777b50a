"""Python mirror of the engine's ``gpu::ComputeBackend`` (app/architecture/shared/cpp/gpu/compute.h:24-45) over the
C ABI ``neko_cuda_*``. Same methods, argument meaning and error behaviour (a failure raises :class:`NekoError`,
the engine's ``fail()``), so tests read like the engine's own ``gpu::selfTest`` (gpu/compute.cpp:32-290)."""
import ctypes as C

import numpy as np

from . import NekoError, check, lib


class Buffer:
    """gpu::Buffer (compute.h:19-22): owned by the backend, alive until the backend is destroyed."""

    def __init__(self, backend, handle, size):
        self.backend, self.handle, self.size = backend, handle, size

    @property
    def device_ptr(self):
        return lib().neko_cuda_buffer_device_ptr(self.handle)


class ComputeBackend:
    """createVulkan / createGles (compute.h:47-48), here on CUDA device ``device``."""

    def __init__(self, device=0):
        err = C.create_string_buffer(1024)
        self.ctx = lib().neko_cuda_create(device, err, 1024)
        if not self.ctx:
            raise NekoError(f"CUDA backend unavailable: {err.value.decode()}")
        self._keep = []

    def name(self):
        return lib().neko_cuda_name(self.ctx).decode()

    def device_name(self):
        buf = C.create_string_buffer(256)
        lib().neko_cuda_device_name(self.ctx, buf, 256)
        return buf.value.decode()

    def max_buffer_bytes(self):
        return int(lib().neko_cuda_max_buffer_bytes(self.ctx))

    def create(self, nbytes, init=None, readback=False):
        """create(bytes, init, readback) (compute.h:34). init: a numpy array (its bytes are copied)."""
        src = None
        if init is not None:
            init = np.ascontiguousarray(init)
            src = init.ctypes.data_as(C.c_void_p)
        h = lib().neko_cuda_create_buffer(self.ctx, nbytes, src, 1 if readback else 0)
        if not h:
            raise NekoError("create: " + lib().neko_cuda_last_error(self.ctx).decode())
        return Buffer(self, h, nbytes)

    def create_from(self, array, readback=False):
        array = np.ascontiguousarray(array)
        return self.create(array.nbytes, array, readback)

    def upload(self, buf, offset, array):
        array = np.ascontiguousarray(array)
        check(lib().neko_cuda_upload(self.ctx, buf.handle, offset, array.ctypes.data_as(C.c_void_p), array.nbytes),
              "upload", self.ctx)

    def download(self, buf, offset, nbytes, dtype=np.float32):
        out = np.empty(nbytes // np.dtype(dtype).itemsize, dtype)
        check(lib().neko_cuda_download(self.ctx, buf.handle, offset, out.ctypes.data_as(C.c_void_p), out.nbytes),
              "download", self.ctx)
        return out

    def begin(self):
        check(lib().neko_cuda_begin(self.ctx), "begin", self.ctx)

    def dispatch(self, kernel, bindings, params, gx, gy):
        """dispatch(Kernel, Buffer* const[4], const int32_t[8], gx, gy) (compute.h:40)."""
        b = (C.c_void_p * 4)(*[(x.handle if x is not None else None) for x in (list(bindings) + [None] * 4)[:4]])
        p = (C.c_int32 * 8)(*(list(params) + [0] * 8)[:8])
        check(lib().neko_cuda_dispatch(self.ctx, int(kernel), b, p, gx, gy), f"dispatch {kernel!r}", self.ctx)

    def flush(self):
        check(lib().neko_cuda_flush(self.ctx), "flush", self.ctx)

    def submit_and_wait(self):
        check(lib().neko_cuda_submit_and_wait(self.ctx), "submitAndWait", self.ctx)

    def close(self):
        if self.ctx:
            lib().neko_cuda_destroy(self.ctx)
            self.ctx = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
