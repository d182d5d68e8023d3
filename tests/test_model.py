"""QuantLinear and optimize() on CPU: construction, quantisation against gguf-py, module
replacement, GGUF loading, and the absence of a CPU compute path (the reference's
SmithyLinear / optimize() tests, tests/test_model.py there, restated for quantized weights).
The forward pass itself is covered on the GPU by tests/test_gpu_model.py."""
import numpy as np
import pytest
import torch
import torch.nn as nn

from kernel_anvil._native import AnvilError
from kernel_anvil.gguf import write_gguf
from kernel_anvil.model import QuantLinear, load_gguf_linears, optimize
from kernel_anvil.quants import resolve_type


def test_from_linear_matches_gguf_quantiser():
    from gguf import GGMLQuantizationType, quants

    torch.manual_seed(0)
    lin = nn.Linear(256, 48, bias=True)
    q = QuantLinear.from_linear(lin, "Q8_0")
    want = quants.quantize(lin.weight.detach().numpy(), GGMLQuantizationType.Q8_0)
    assert np.array_equal(q.weight_blocks.numpy(), want)
    assert (q.in_features, q.out_features, q.quant) == (256, 48, "Q8_0")
    assert torch.equal(q.bias, lin.bias.detach())
    assert "quant=Q8_0" in repr(q)


def test_k_quants_come_from_gguf_files():
    with pytest.raises(AnvilError, match="GGUF"):
        QuantLinear.from_linear(nn.Linear(256, 8), "Q4_K")


def test_block_shape_checked():
    with pytest.raises(AnvilError, match="bytes"):
        QuantLinear(torch.zeros((4, 100), dtype=torch.uint8), "Q4_K", 256)


def test_no_cpu_forward():
    q = QuantLinear.from_linear(nn.Linear(64, 8), "Q8_0")
    with pytest.raises(AnvilError, match="CUDA"):
        q(torch.randn(2, 64))


def test_optimize_replaces_eligible_linears():
    model = nn.Sequential(nn.Linear(64, 32), nn.ReLU(), nn.Sequential(nn.Linear(32, 96)),
                          nn.Linear(96, 7), nn.Linear(10, 4))
    optimize(model, "Q8_0", verbose=False)
    kinds = [type(m).__name__ for m in model.modules() if isinstance(m, (nn.Linear, QuantLinear))]
    assert kinds == ["QuantLinear", "QuantLinear", "QuantLinear", "Linear"]  # 10 % 32 != 0 stays


def test_load_gguf_linears(tmp_path):
    path = write_gguf(tmp_path / "m.gguf", [("a.weight", "Q4_K", 16, 512), ("b.weight", "Q6_K", 8, 256),
                                            ("norm", "F32", 1, 64), ("c.weight", "Q8_0", 5, 64)])
    mods = load_gguf_linears(path, device="cpu")
    assert sorted(mods) == ["a.weight", "b.weight", "c.weight"]
    a = mods["a.weight"]
    assert (a.quant, a.out_features, a.in_features) == ("Q4_K", 16, 512)
    assert a.weight_blocks.shape == (16, resolve_type("Q4_K").row_bytes(512))
