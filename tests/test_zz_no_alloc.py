"""GPU checks of kt_qmatmul_noalloc, the matmul whose scratch memory is a static
array in the library image, for callers that cannot let the library allocate
device memory at call time (a decode loop on a fixed memory budget, a host
runtime that accounts for every device byte).  It runs the kernels kt_qmatmul
chooses, so its results must equal kt_qmatmul's bit for bit, on two calls in a
row (the array keeps the previous call's contents), and match the oracle
within the tolerance of the kernel that ran.  The file name sorts last so that
these run after every other test as well as alone."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

TOL_FP32 = 1e-3
TOL_BF16 = 2e-2
KT_PATH_TENSOR_CORE = 2


def rel_err(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))


def call(lib, fn, qt, x, y, m, accumulate=False, alpha=1.0):
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return getattr(lib, fn)(qt._ctx.handle, qt.handle, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()),
                            m, int(accumulate), float(alpha), None, stream)


# (bits, K, N, m): every kernel family kt_qmatmul routes to -- the m = 1 integer
# tensor-core GEMV (split-K in clusters and through the array), m = 2..8 on the
# fp16 tensor-core GEMV (m = 5..8 as two token groups in one launch), the fp32
# streaming GEMV (INT8 at m = 2..8), the tcgen05 GEMM at m >= 9 (INT4 and INT8,
# with and without split-K), the generic kernel (ragged N)
CASES = [(4, 4096, 14336, 1), (4, 14336, 4096, 1), (4, 768, 32000, 1), (4, 2048, 5632, 4), (4, 14336, 4096, 2),
         (4, 4096, 14336, 6), (4, 2048, 5632, 7), (8, 2048, 2048, 1), (8, 2048, 2048, 4), (8, 2048, 2048, 64),
         (4, 4096, 14336, 16),
         (4, 4096, 14336, 64), (4, 2048, 5632, 96), (8, 2048, 2048, 9), (4, 512, 1000, 12)]


@pytest.mark.parametrize("bits,k,n,m", CASES)
def test_noalloc_equals_qmatmul_on_two_calls_in_a_row(kt, oracle, bits, k, n, m):
    from kotensor_b200 import _lib
    lib = kt.load_library()
    rng = np.random.default_rng(k * 7 + n + m + bits)
    w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
    ref_q = oracle.quantize(w, bits, 64)
    qt = kt.QuantizedTensor.from_arrays(ref_q.qdata, ref_q.scales, ref_q.zeros, (k, n), bits, 64)
    xh = rng.standard_normal((m, k), dtype=np.float32)
    c0h = rng.standard_normal((m, n), dtype=np.float32)
    x = torch.from_numpy(xh).cuda()
    c0 = torch.from_numpy(c0h).cuda()
    ref = c0.clone()
    _lib.check(call(lib, "kt_qmatmul", qt, x, ref, m, accumulate=True, alpha=0.5))
    for _ in range(2):
        y = c0.clone()
        _lib.check(call(lib, "kt_qmatmul_noalloc", qt, x, y, m, accumulate=True, alpha=0.5))
        torch.cuda.synchronize()
        assert torch.equal(y, ref)  # the same kernels: the same bits
    path = ctypes.c_int32()
    _lib.check(lib.kt_qmatmul_path(qt.handle, m, ctypes.byref(path)))
    tol = TOL_BF16 if path.value == KT_PATH_TENSOR_CORE else TOL_FP32
    if k * n * m <= 2048 * 5632 * 128:  # the oracle finishes in seconds
        expect = c0h + np.float32(0.5) * oracle.multiply_quantized(xh, ref_q)
        assert rel_err(y.cpu().numpy(), expect) <= tol
    assert kt.Context.get().take_error() == 0


def test_noalloc_rejects_scratch_beyond_its_array(kt):
    """The tcgen05 GEMM at m = 512 on K = 16384 keeps 16 MiB of bf16
    activations alone: rejected with a message naming the static workspace;
    m = 1 fits and runs."""
    from kotensor_b200 import _lib
    lib = kt.load_library()
    k, n, g = 16384, 4096, 64
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
    x = torch.randn((512, k), device="cuda")
    y = torch.ones((512, n), device="cuda")
    st = call(lib, "kt_qmatmul_noalloc", qt, x, y, 512)
    assert st == _lib.KT_ERR_INVALID_ARGUMENT
    assert b"static workspace" in lib.kt_last_error()
    _lib.check(call(lib, "kt_qmatmul_noalloc", qt, x, y, 1))
    torch.cuda.synchronize()
    assert not torch.any(y[0]).item()  # zero weights, accumulate = 0
    assert torch.all(y[1:] == 1.0).item()  # the rejected call wrote nothing
    assert kt.Context.get().take_error() == 0
