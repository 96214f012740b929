"""GPU checks of kt_qmatmul_noalloc (the matmul whose split-K workspace is a
static array in the library image) against kt_qmatmul.  The file name sorts
last so that these run after every other test as well as alone."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

TOL_FP32 = 1e-3


def rel_err(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))


def call(lib, fn, qt, x, y, m, accumulate=False, alpha=1.0):
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return getattr(lib, fn)(qt._ctx.handle, qt.handle, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()),
                            m, int(accumulate), float(alpha), None, stream)


@pytest.mark.parametrize("k,n,m", [(4096, 14336, 1), (2048, 5632, 4), (14336, 4096, 2), (768, 32000, 1),
                                   (2048, 2048, 8)])
def test_noalloc_matches_qmatmul_on_two_calls_in_a_row(kt, k, n, m):
    from kotensor_b200 import _lib
    lib = kt.load_library()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(k * 7 + n + m)
    w = torch.randn((k, n), generator=gen, device="cuda") * 0.02
    qt = kt.QuantizedTensor.quantize(w, kt.Quantization(4, 64))
    x = torch.randn((m, k), generator=gen, device="cuda")
    c0 = torch.randn((m, n), generator=gen, device="cuda")
    ref = c0.clone()
    _lib.check(call(lib, "kt_qmatmul", qt, x, ref, m, accumulate=True, alpha=0.5))
    for _ in range(2):
        y = c0.clone()
        _lib.check(call(lib, "kt_qmatmul_noalloc", qt, x, y, m, accumulate=True, alpha=0.5))
        torch.cuda.synchronize()
        assert rel_err(y.cpu().numpy(), ref.cpu().numpy()) <= TOL_FP32
    assert kt.Context.get().take_error() == 0


def test_noalloc_rejects_a_workspace_beyond_its_array(kt):
    """K = 65536 at m = 4 needs 64 K-splits of 16 column tiles (4 MiB of partial
    tiles plus the counters): rejected; m = 1 fits and runs."""
    from kotensor_b200 import _lib
    lib = kt.load_library()
    k, n, g = 65536, 4096, 64
    q = torch.zeros((k, n // 2), dtype=torch.uint8, device="cuda")
    s = torch.zeros((k // g, n), dtype=torch.float32, device="cuda")
    z = torch.zeros((k // g, n), dtype=torch.uint8, device="cuda")
    ctx = kt.Context.get()
    out = ctypes.c_void_p()
    _lib.check(lib.kt_qweight_from_device(ctx.handle, 4, g, k, n, ctypes.c_void_p(q.data_ptr()),
                                          ctypes.c_void_p(s.data_ptr()), ctypes.c_void_p(z.data_ptr()),
                                          None, ctypes.byref(out)))
    torch.cuda.synchronize()
    qt = kt.QuantizedTensor(out, ctx)
    x = torch.randn((4, k), device="cuda")
    y = torch.ones((4, n), device="cuda")
    st = call(lib, "kt_qmatmul_noalloc", qt, x, y, 4)
    assert st == _lib.KT_ERR_INVALID_ARGUMENT
    assert b"static workspace" in lib.kt_last_error()
    _lib.check(call(lib, "kt_qmatmul_noalloc", qt, x, y, 1))
    torch.cuda.synchronize()
    assert not torch.any(y[0]).item()  # zero weights, accumulate = 0
    assert kt.Context.get().take_error() == 0
