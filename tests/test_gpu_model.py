"""QuantLinear forward passes on the GPU against the oracle: the MMVQ result of the dequantised
GGUF weights and the Q8_1-quantised input, within the fp32 output tolerance of the kernel
tests; 1, 3 and 19 tokens (19 = three launches of up to 8 columns), leading batch dims,
bias, half-precision input, and a model rewritten by optimize()."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.nn as nn  # noqa: E402

from kernel_anvil.gguf import write_gguf  # noqa: E402
from kernel_anvil.model import QuantLinear, load_gguf_linears, optimize  # noqa: E402
from oracle import oracle  # noqa: E402

pytestmark = pytest.mark.gpu
Y_TOL = 1e-3


def _oracle(q: QuantLinear, x: torch.Tensor) -> np.ndarray:
    x2 = x.detach().float().reshape(-1, q.in_features).cpu().numpy()
    W = q.weight_blocks.cpu().numpy()
    y = oracle.mmvq(q.quant, W, oracle.quantize_q8_1(x2), q.out_features, q.in_features, x2.shape[0])
    y = y.reshape(x2.shape[0], q.out_features)
    if q.bias is not None:
        y = y + q.bias.detach().cpu().numpy()
    return y


@pytest.mark.parametrize("shape", [(1, 4096), (3, 4096), (2, 19, 4096)])
@pytest.mark.parametrize("qt", ["Q4_K", "Q6_K", "Q8_0"])
def test_forward_matches_oracle(tmp_path, shape, qt):
    K = shape[-1]
    path = write_gguf(tmp_path / "m.gguf", [("w", qt, 640, K)], seed=3)
    q = QuantLinear.from_gguf(path, "w")
    x = torch.randn(*shape, device="cuda")
    y = q(x)
    assert y.shape == (*shape[:-1], 640)
    ref = _oracle(q, x)
    assert oracle.max_rel_err(y.reshape(-1, 640).cpu().numpy(), ref) <= Y_TOL


def test_bias_and_half_input():
    torch.manual_seed(1)
    lin = nn.Linear(1024, 300, bias=True).cuda()
    q = QuantLinear.from_linear(lin, "Q8_0")
    x = torch.randn(5, 1024, device="cuda").half()
    y = q(x)
    assert y.dtype == torch.float16
    ref = _oracle(q, x.float())
    assert oracle.max_rel_err(y.float().cpu().numpy(), ref) <= 2e-3  # fp16 output rounding
    # the quantized linear tracks the fp32 linear to the Q8_0/Q8_1 quantisation error
    fp = lin(x.float()).detach()
    assert float((y.float() - fp).abs().max() / fp.abs().max()) < 0.05


def test_optimize_model_runs_on_mmvq():
    torch.manual_seed(2)
    model = nn.Sequential(nn.Linear(512, 1024), nn.GELU(), nn.Linear(1024, 256)).cuda()
    x = torch.randn(1, 512, device="cuda")
    ref = model(x).detach()
    optimize(model, "Q8_0", verbose=False)
    assert all(type(m) is not nn.Linear for m in model.modules())
    y = model(x).detach()
    assert float((y - ref).abs().max() / ref.abs().max()) < 0.05


def test_load_gguf_linears_on_gpu(tmp_path):
    path = write_gguf(tmp_path / "m.gguf", [("a", "Q4_K", 256, 1024), ("b", "Q5_K", 128, 512)], seed=4)
    mods = load_gguf_linears(path)
    for name, K in (("a", 1024), ("b", 512)):
        q = mods[name]
        x = torch.randn(2, K, device="cuda")
        assert oracle.max_rel_err(q(x).cpu().numpy(), _oracle(q, x)) <= Y_TOL
