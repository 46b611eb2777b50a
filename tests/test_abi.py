"""The C-ABI library builds for sm_100a, loads without a GPU and exports every entry point include/neko_cuda.h
declares. No compute call is made here."""
import ctypes as C
import os
import re

import pytest

import nekochat_b200 as nb
from nekochat_b200 import workload

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "neko_cuda.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(neko_\w+)\s*\(", text)))


def test_library_present_and_loads():
    assert os.path.exists(nb.LIB_PATH), "libneko_cuda.so not built"
    nb.lib()


def test_exports_every_declared_symbol():
    decl = declared_functions()
    assert len(decl) >= 30
    lib = C.CDLL(nb.LIB_PATH)
    missing = [n for n in decl if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"
    # the Python binding covers the whole ABI
    assert sorted(nb.exported_symbols()) == decl


def test_abi_version_and_row_bytes_without_gpu():
    l = nb.lib()
    assert l.neko_abi_version() == 1
    for fmt in (0, 1, 2):
        for cols in (64, 96, 768, 1024, 2560, 3072, 9728):
            assert l.neko_row_bytes(fmt, cols) == workload.row_bytes(fmt, cols)


def test_create_fails_cleanly_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(nb.NekoError):
        nb.ComputeBackend(0)


def test_kernel_ids_match_engine_enum():
    # gpu::Kernel order (compute.h:17) == NEKO_KERNELS (CMakeLists.txt:23)
    names = ["Embed", "LayerNorm", "Matmul", "KvStore", "Attention", "Rope", "SiluMul", "MatmulQ8", "MatmulQ4"]
    assert [k.name for k in nb.Kernel] == names
    assert [k.value for k in nb.Kernel] == list(range(9))
    assert nb.float_bits(1.0) == 0x3F800000
