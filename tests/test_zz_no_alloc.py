"""The allocation-free split-K GEMM entry point, called through its exported C symbol.

Some callers of this library cannot allocate device memory where they call it
(a fixed memory budget set by the host program, a plugin inside another
runtime's allocator, a path where cudaMalloc/cudaFree and the synchronisation
they imply are not allowed).  `rkt_gemm_bf16_splitk_noalloc` serves them with
a static device scratch array; this test checks it against the regular
split-K entry point (which takes a caller-provided workspace) on two calls in a
row, and that an oversized request is refused without launching anything.
This file is collected last on purpose.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _sym():
    import rocket_b200._C as C
    lib = ctypes.CDLL(C.__file__)
    f = lib.rkt_gemm_bf16_splitk_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                  ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    return f


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def test_noalloc_splitk_matches_regular_entry_point_twice():
    from rocket_b200 import ops
    f = _sym()
    stream = torch.cuda.current_stream().cuda_stream
    status = torch.zeros(1, dtype=torch.int32, device="cuda")  # device-side error bits
    for call, (m, n, k, s) in enumerate([(64, 1024, 4096, 8), (37, 512, 2048, 4)]):
        g = torch.Generator(device="cuda").manual_seed(100 + call)
        x = torch.randn(m, k, device="cuda", generator=g).bfloat16()
        w = (torch.randn(n, k, device="cuda", generator=g) * 0.02).bfloat16()
        out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
        rc = f(w.data_ptr(), x.data_ptr(), out.data_ptr(), n, k, m, s, status.data_ptr(), stream)
        assert rc == 0, rc
        regular = ops.linear_bf16(x, w, splits=s)
        torch.cuda.synchronize()
        assert int(status.item()) == 0  # no wait gave up
        ref = x.float() @ w.float().t()
        assert _rel(out, regular) < 1e-2
        assert _rel(out, ref) < 1e-2


def test_noalloc_rejects_oversized_request():
    f = _sym()
    stream = torch.cuda.current_stream().cuda_stream
    m, n, k, s = 256, 8192, 4096, 8  # 8 * 256 * 8192 floats > 4 MiB of scratch
    x = torch.zeros(m, k, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(n, k, dtype=torch.bfloat16, device="cuda")
    out = torch.full((m, n), 7.0, dtype=torch.bfloat16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert f(w.data_ptr(), x.data_ptr(), out.data_ptr(), n, k, m, s, status.data_ptr(), stream) == -5
    assert f(w.data_ptr(), x.data_ptr(), out.data_ptr(), n, k, m, s, None, stream) == -2
    torch.cuda.synchronize()
    assert torch.all(out == 7.0)  # nothing was launched
