"""QLoRA on the GPU: LoRALinear over a quantized base (kt_lora_qmatmul with the
low-rank term in the matmul epilogue, kt_lora_backward) and fusedCrossEntropyLoss
with a quantized head (kt_fused_cross_entropy), against the CPU restatement
(oracle/qlora_oracle.py).

Reference behaviour ported (Engine/kotensor/src/test/kotlin/):
  TrainingTest.testFusedLossWithQuantizedHeadAndFrozenWeights  (loss and hidden gradient)
  TrainingTest fused loss tests: masked rows get no gradient, large vocabularies stream in chunks
  QuantizationTest LoRA-on-quantized tests: a fresh adapter (B = 0) leaves the base output unchanged
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from oracle import qlora_oracle as QO  # noqa: E402


def _tensor_core(layer, m):
    """Whether kt_qmatmul takes the bf16 tcgen05 GEMM for this weight and m (2e-2 tolerance)."""
    from kotensor_b200 import _lib
    return layer.weight.matmul_path(m) == _lib.KT_PATH_TENSOR_CORE


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def _layer(kt, oracle, k, n, bits, seed, group=64):
    from kotensor_b200 import QuantizedLinear, Quantization
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((k, n)) * 0.05).astype(np.float32)
    q = oracle.quantize(w, bits, group)
    layer = QuantizedLinear(k, n, Quantization(bits, group))
    layer.weight = kt.QuantizedTensor.from_arrays(q.qdata, q.scales, q.zeros, (k, n), bits, group)
    layer.bias.copy_(torch.from_numpy((rng.standard_normal(n) * 0.1).astype(np.float32)).reshape(1, n))
    return layer, q


def _adapter(layer, rank, seed, alpha=2.0):
    from kotensor_b200.lora import LoRALinear
    g = torch.Generator().manual_seed(seed)
    lora = LoRALinear(layer, rank=rank, alpha=alpha, generator=g)
    lora.lora_b.copy_(torch.randn(lora.lora_b.shape, generator=g) * 0.3)
    return lora


# (bits, K, N, m): m covers the INT4 tensor-core GEMV (m <= 4), the fp32 GEMV
# (m <= 8), the tcgen05 GEMM (m >= 9) and the generic kernel (m >= 9 on shapes
# without TMA descriptors, e.g. N = 333).
CASES = [(4, 256, 333, 1), (4, 512, 1024, 3), (8, 256, 333, 1), (8, 384, 640, 6), (4, 256, 512, 7),
         (4, 512, 1024, 16), (4, 1024, 2048, 64), (8, 256, 333, 20), (8, 512, 640, 24)]


@pytest.mark.parametrize("bits,k,n,m", CASES)
@pytest.mark.parametrize("rank", [1, 4, 12, 64])
def test_lora_forward_matches_oracle(kt, oracle, bits, k, n, m, rank):
    layer, q = _layer(kt, oracle, k, n, bits, seed=k + n + m)
    lora = _adapter(layer, rank, seed=rank)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(k * m + rank)).cuda()
    out = lora(x)
    base = layer(x)
    torch.cuda.synchronize()
    ref, ref_p = QO.lora_forward(x.cpu().numpy(), q, layer.bias.cpu().numpy(), lora.lora_a.cpu().numpy(),
                                 lora.lora_b.cpu().numpy(), lora.scaling)
    # fp32 sums in another order: bounded relative to sum |x_k A_kr| (a projection
    # that cancels to a small value is not held to 1e-5 of itself)
    scale_p = np.abs(x.cpu().numpy()).astype(np.float64) @ np.abs(lora.lora_a.cpu().numpy()).astype(np.float64)
    assert np.abs(lora._projected[:m].cpu().numpy() - ref_p).max() <= 1e-5 * scale_p.max()
    tensor_core = _tensor_core(layer, m)
    assert _rel(out.cpu().numpy(), ref) <= (2e-2 if tensor_core else 1e-3)
    # the epilogue's low-rank term alone, against float64 (isolates it from the base path's rounding)
    low = (out - base).double().cpu().numpy()
    want = (ref_p.astype(np.float64) @ lora.lora_b.double().cpu().numpy()) * lora.scaling
    assert np.abs(low - want).max() <= 1e-4 * max(np.abs(want).max(), np.abs(base.cpu().numpy()).max())
    assert kt.Context.get().take_error() == 0


def test_fresh_adapter_leaves_the_base_output_unchanged(kt, oracle):
    from kotensor_b200.lora import LoRALinear
    layer, _ = _layer(kt, oracle, 512, 768, 4, seed=3)
    lora = LoRALinear(layer, rank=8, alpha=16.0)
    for m in (1, 4, 16):
        x = torch.randn(m, 512, device="cuda")
        assert torch.equal(lora(x), layer(x))
    assert torch.count_nonzero(lora.delta_weights()) == 0


@pytest.mark.parametrize("bits,k,n,m", [(4, 256, 333, 1), (8, 384, 640, 5), (4, 512, 1024, 32), (4, 2048, 4096, 3)])
@pytest.mark.parametrize("rank", [4, 16])
def test_lora_backward_matches_oracle(kt, oracle, bits, k, n, m, rank):
    layer, q = _layer(kt, oracle, k, n, bits, seed=k * m)
    lora = _adapter(layer, rank, seed=7)
    g_in = torch.Generator().manual_seed(k + n * m + rank)
    x = torch.randn(m, k, generator=g_in).cuda()
    dy = torch.randn(m, n, generator=g_in).cuda()
    lora(x)
    dx = torch.full((m, k), 0.5, device="cuda")
    lora.backward(x, dy, dx, accumulate_dx=True)
    torch.cuda.synchronize()
    ref_dx, ref_ga, ref_gb = QO.lora_backward(x.cpu().numpy(), dy.cpu().numpy(), q, lora.lora_a.cpu().numpy(),
                                              lora.lora_b.cpu().numpy(), lora.scaling,
                                              lora._projected[:m].cpu().numpy())
    from kotensor_b200 import _lib
    # kt_qmatmul_t takes the bf16 tcgen05 kernel for INT4 at m >= 16 (tolerance 2e-2)
    dx_tol = 2e-2 if layer.weight.transposed_path(m) == _lib.KT_PATH_TENSOR_CORE else 1e-3
    assert _rel(dx.cpu().numpy() - 0.5, ref_dx) <= dx_tol
    assert _rel(lora.grad_a.cpu().numpy(), ref_ga) <= 1e-4
    assert _rel(lora.grad_b.cpu().numpy(), ref_gb) <= 1e-4
    # gradients accumulate (Tensor.grad +=), bit-identically on a second pass
    ga, gb = lora.grad_a.clone(), lora.grad_b.clone()
    lora.backward(x, dy)
    assert torch.equal(lora.grad_a, 2 * ga) or _rel(lora.grad_a.cpu().numpy(), 2 * ga.cpu().numpy()) <= 1e-6
    assert _rel(lora.grad_b.cpu().numpy(), 2 * gb.cpu().numpy()) <= 1e-6
    # deterministic
    dx2 = torch.full((m, k), 0.5, device="cuda")
    lora.backward(x, dy, dx2, accumulate_dx=True)
    assert torch.equal(dx, dx2)
    assert kt.Context.get().take_error() == 0


def _head(kt, oracle, dim, vocab, bits, seed):
    return _layer(kt, oracle, dim, vocab, bits, seed, group=64)


@pytest.mark.parametrize("bits,dim,vocab,rows", [(4, 256, 5000, 13), (8, 128, 3001, 6), (4, 512, 32000, 40),
                                                 (8, 64, 1 << 20, 80)])
def test_fused_cross_entropy_matches_oracle(kt, oracle, bits, dim, vocab, rows):
    from kotensor_b200.loss import fused_cross_entropy_loss, IGNORE_INDEX
    head, q = _head(kt, oracle, dim, vocab, bits, seed=vocab)
    rng = np.random.default_rng(rows)
    targets = [int(t) for t in rng.integers(0, vocab, rows)]
    targets[1] = IGNORE_INDEX
    targets[rows - 2] = IGNORE_INDEX
    hidden = torch.from_numpy(rng.standard_normal((rows, dim)).astype(np.float32)).cuda()
    hidden_grad = torch.zeros_like(hidden)
    bias_grad = torch.zeros(vocab, device="cuda")
    loss = fused_cross_entropy_loss(hidden, head, targets, hidden_grad=hidden_grad, bias_grad=bias_grad)
    torch.cuda.synchronize()
    ref_loss, ref_hg, ref_bg = QO.fused_cross_entropy(hidden.cpu().numpy(), q, head.bias.cpu().numpy(), targets)
    active = rows - 2
    chunk = min(active, (1 << 26) // vocab)
    tensor_core = _tensor_core(head, chunk)
    tol = 2e-2 if tensor_core else 1e-3
    assert abs(float(loss.item()) - float(ref_loss)) <= tol * max(1.0, abs(float(ref_loss)))
    # the hidden gradient also goes through kt_qmatmul_t (bf16 tensor cores at m >= 16)
    from kotensor_b200 import _lib
    hg_bf16 = tensor_core or head.weight.transposed_path(chunk) == _lib.KT_PATH_TENSOR_CORE
    assert _rel(hidden_grad.cpu().numpy(), ref_hg) <= (5e-2 if hg_bf16 else 2e-3)
    assert _rel(bias_grad.cpu().numpy(), ref_bg) <= (5e-2 if tensor_core else 2e-3)
    hg = hidden_grad.cpu().numpy()
    assert not hg[1].any() and not hg[rows - 2].any()  # masked rows get no gradient
    assert kt.Context.get().take_error() == 0


def test_fused_cross_entropy_on_the_devices_own_logits(kt, oracle):
    """Given the logits the device's matmul produces, the loss and the logit
    gradients follow the reference's formulas to float32 rounding."""
    from kotensor_b200.loss import fused_cross_entropy_loss
    head, q = _head(kt, oracle, 256, 7000, 4, seed=11)
    rng = np.random.default_rng(2)
    rows = 24
    targets = [int(t) for t in rng.integers(0, 7000, rows)]
    hidden = torch.from_numpy(rng.standard_normal((rows, 256)).astype(np.float32)).cuda()
    bias_grad = torch.zeros(7000, device="cuda")
    loss = fused_cross_entropy_loss(hidden, head, targets, bias_grad=bias_grad)
    logits = head(hidden).double().cpu().numpy()  # same m, same matmul path
    mx = logits.max(axis=1, keepdims=True)
    e = np.exp(logits - mx)
    s = e.sum(axis=1, keepdims=True)
    want = np.mean(mx[:, 0] + np.log(s[:, 0]) - logits[np.arange(rows), targets])
    assert abs(float(loss.item()) - want) <= 1e-5 * max(1.0, abs(want))
    g = e / s
    g[np.arange(rows), targets] -= 1.0
    assert _rel(bias_grad.cpu().numpy(), (g / rows).sum(axis=0)) <= 1e-4


def test_fused_cross_entropy_edge_cases(kt, oracle):
    from kotensor_b200.loss import fused_cross_entropy_loss, IGNORE_INDEX
    head, _ = _head(kt, oracle, 64, 100, 8, seed=5)
    hidden = torch.randn(3, 64, device="cuda")
    hg = torch.zeros_like(hidden)
    loss = fused_cross_entropy_loss(hidden, head, [IGNORE_INDEX] * 3, hidden_grad=hg)
    assert float(loss.item()) == 0.0 and not hg.any()
    with pytest.raises(ValueError, match="target 100 out of bounds 100"):
        fused_cross_entropy_loss(hidden, head, [0, 100, 1])
    with pytest.raises(ValueError, match="targets cannot be empty"):
        fused_cross_entropy_loss(hidden[:0], head, [])


def test_qlora_training_step_reduces_the_loss(kt, oracle):
    """A QLoRA step end to end on the device: LoRA projection over a quantized
    base, fused loss over a quantized head, gradients back through both, SGD on
    the adapter only; the loss goes down and the base weights stay as they were."""
    from kotensor_b200.loss import fused_cross_entropy_loss
    layer, _ = _layer(kt, oracle, 256, 256, 4, seed=21)
    head, _ = _head(kt, oracle, 256, 1000, 4, seed=22)
    lora = _adapter(layer, 8, seed=3, alpha=8.0)
    rng = np.random.default_rng(9)
    x = torch.from_numpy(rng.standard_normal((12, 256)).astype(np.float32)).cuda()
    targets = [int(t) for t in rng.integers(0, 1000, 12)]
    before = layer.weight.download()
    losses = []
    for _ in range(5):
        hidden = lora(x)
        hidden_grad = torch.zeros_like(hidden)
        loss = fused_cross_entropy_loss(hidden, head, targets, hidden_grad=hidden_grad)
        losses.append(float(loss.item()))
        lora.zero_grad()
        lora.backward(x, hidden_grad)
        with torch.no_grad():
            lora.lora_a -= 0.5 * lora.grad_a
            lora.lora_b -= 0.5 * lora.grad_b
    assert losses[-1] < losses[0], losses
    after = layer.weight.download()
    assert all(np.array_equal(a, b) for a, b in zip(before, after) if a is not None)
    assert kt.Context.get().take_error() == 0
