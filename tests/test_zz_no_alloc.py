"""neko_op_attention_noalloc: attention that takes its split-KV scratch from a fixed array inside the library
instead of allocating it, for callers that cannot let a library allocate device memory (engines that account
for every device byte they hold, callers that must not hit an out-of-memory failure mid-reply, hosts that
forbid allocator calls once decoding has started).

Checked through the C ABI against the allocating entry point neko_op_attention, on two calls in a row (the
second must not be affected by what the first left in the shared scratch), with the tolerance the other
attention tests use, and against the C restatement of the reference's cpu::attention (cpu_ops.cpp:544-575). This
file is collected last so a failure here cannot hide another test's result."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
TOL = 2e-3


def _oracle(q, kc, vc, H, KV, hd, T, pos0):
    from oracle.oracle import Restatement
    return Restatement().attention(q, q.shape[1], kc.view(np.uint16), vc.view(np.uint16), T, H, KV, hd, pos0)


def _case(rng, H, KV, hd, T, pos0):
    ctx = pos0 + T
    q = rng.uniform(-1, 1, (T, (H + 2 * KV) * hd)).astype(np.float32)
    kc = rng.uniform(-1, 1, (ctx, KV * hd)).astype(np.float16).view(np.int16)
    vc = rng.uniform(-1, 1, (ctx, KV * hd)).astype(np.float16).view(np.int16)
    return q, kc, vc


def _run(entry, torch, q, kc, vc, H, KV, hd, T, pos0):
    import nekochat_b200 as nb
    tq, tk, tv = (torch.from_numpy(a).cuda() for a in (q, kc, vc))
    out = torch.full((T, H * hd), float("nan"), device="cuda")
    rc = getattr(nb.lib(), entry)(C.c_void_p(tq.data_ptr()), q.shape[1], C.c_void_p(tk.data_ptr()),
                                  C.c_void_p(tv.data_ptr()), C.c_void_p(out.data_ptr()), T, H, KV, hd, pos0,
                                  C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, nb.lib().neko_last_error().decode()
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("H,KV,hd,T,pos0", [(16, 8, 128, 1, 700), (32, 8, 128, 1, 4000), (4, 2, 64, 3, 1030)])
def test_noalloc_matches_allocating_attention_twice(H, KV, hd, T, pos0):
    import torch
    assert torch.cuda.is_available()
    rng = np.random.default_rng(pos0 * 7 + T)
    for call in range(2):  # two calls in a row, different inputs
        q, kc, vc = _case(rng, H, KV, hd, T, pos0 + 37 * call)
        want = _run("neko_op_attention", torch, q, kc, vc, H, KV, hd, T, pos0 + 37 * call)
        got = _run("neko_op_attention_noalloc", torch, q, kc, vc, H, KV, hd, T, pos0 + 37 * call)
        assert np.all(np.isfinite(got))
        d = np.abs(got - want)
        assert np.all(d <= TOL * (1 + np.abs(want))), f"call {call}: max err {d.max()}"
        ref = _oracle(q, kc, vc, H, KV, hd, T, pos0 + 37 * call)
        d = np.abs(got - ref)
        assert np.all(d <= TOL * (1 + np.abs(ref))), f"call {call}: max err vs oracle {d.max()}"


def test_noalloc_single_split_needs_no_scratch():
    """Many rows x KV heads (more than the fixed ticket count) in a single-split plan: no scratch is used, so the
    call runs, and matches the allocating entry point and the oracle."""
    import torch
    H, KV, hd, T, pos0 = 16, 8, 128, 1025, 0
    q, kc, vc = _case(np.random.default_rng(3), H, KV, hd, T, pos0)
    want = _run("neko_op_attention", torch, q, kc, vc, H, KV, hd, T, pos0)
    got = _run("neko_op_attention_noalloc", torch, q, kc, vc, H, KV, hd, T, pos0)
    d = np.abs(got - want)
    assert np.all(d <= TOL * (1 + np.abs(want))), f"max err {d.max()}"
    for r in (0, 1, 511, 1024):  # the oracle is a scalar loop: row r alone is query r at position r
        ref = _oracle(q[r:r + 1], kc, vc, H, KV, hd, 1, r)[0]
        d = np.abs(got[r] - ref)
        assert np.all(d <= TOL * (1 + np.abs(ref))), f"row {r}: max err vs oracle {d.max()}"


def test_noalloc_rejects_unsupported_group_as_bad_argument():
    """Sixteen query heads per KV head is beyond the kernels: a bad argument, reported before any work."""
    import torch
    import nekochat_b200 as nb
    tiny = torch.zeros(16, device="cuda")
    rc = nb.lib().neko_op_attention_noalloc(C.c_void_p(tiny.data_ptr()), 18 * 64, C.c_void_p(tiny.data_ptr()),
                                            C.c_void_p(tiny.data_ptr()), C.c_void_p(tiny.data_ptr()), 1, 16, 1, 64,
                                            0, None)
    assert rc == -1  # NEKO_ERR_ARG


def test_noalloc_rejects_shapes_beyond_its_scratch():
    """A shape whose split-KV state exceeds the fixed scratch fails with a clear error and launches nothing."""
    import torch
    import nekochat_b200 as nb
    T, H, KV, hd, pos0 = 295, 8, 1, 256, 600  # a valid shape: 2 splits x 295 rows x 8 heads x 258 floats > 4 MiB
    tiny = torch.zeros(16, device="cuda")
    rc = nb.lib().neko_op_attention_noalloc(C.c_void_p(tiny.data_ptr()), (H + 2 * KV) * hd, C.c_void_p(tiny.data_ptr()),
                                            C.c_void_p(tiny.data_ptr()), C.c_void_p(tiny.data_ptr()), T, H, KV, hd,
                                            pos0, None)
    assert rc == -6  # NEKO_ERR_UNSUPPORTED
    assert "fixed scratch holds" in nb.lib().neko_last_error().decode()
