"""GPU parity of the gate/up (SwiGLU) epilogue against the CPU oracle, through the C ABI.

Bars: max|y - y_ref| / max|y_ref| <= 1e-3 against silu(W_gate . x) * (W_up . x) evaluated in
float64 by the oracle from the same Q8_1 activation (the MMVQ tolerance), and
|y - silu(g) * u| <= 1e-5 max|y| against the kernel's own separate gate and up GEMVs.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from kernel_anvil import mmvq as ops  # noqa: E402
from kernel_anvil._native import AnvilError  # noqa: E402
from kernel_anvil.quants import make_activation, make_weights  # noqa: E402
from oracle import oracle  # noqa: E402

pytestmark = pytest.mark.gpu

TYPES = ["Q4_K", "Q5_K", "Q6_K", "Q8_0", "Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q2_K", "Q3_K", "IQ4_NL",
         "IQ4_XS"]
Y_TOL = 1e-3


def dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def check_glu(qt, nrows, K, nwarps=0, rpb=0, seed=0):
    Wg = make_weights(qt, nrows, K, seed=seed)
    Wu = make_weights(qt, nrows, K, seed=seed + 100)
    x = make_activation(K, seed=seed + 1)
    xq_ref = oracle.quantize_q8_1(x)
    Wgd, Wud = dev(Wg), dev(Wu)
    xq = ops.quantize_q8_1(dev(x))
    y = ops.mmvq_glu(Wgd, Wud, qt, xq, nwarps=nwarps, rows_per_block=rpb)
    g = ops.mmvq(Wgd, qt, xq)
    u = ops.mmvq(Wud, qt, xq)
    own = torch.nn.functional.silu(g) * u
    torch.cuda.synchronize()
    y_ref = oracle.mmvq_glu(qt, Wg, Wu, xq_ref, nrows, K)
    err = oracle.max_rel_err(y.cpu().numpy(), y_ref)
    assert err <= Y_TOL, f"{qt} {nrows}x{K} nw={nwarps} rpb={rpb}: err {err:.3e}"
    y64 = y.double()
    assert float((y64 - own.double()).abs().max()) <= 1e-5 * float(y64.abs().max()) + 1e-30
    return y


@pytest.mark.parametrize("qt", TYPES)
@pytest.mark.parametrize("rpb", [0, 2, 4, 8])
def test_glu_matches_oracle(qt, rpb):
    check_glu(qt, 1000, 4096, rpb=rpb, seed=rpb)


@pytest.mark.parametrize("qt", ["Q4_K", "Q6_K", "Q8_0", "Q5_1"])
@pytest.mark.parametrize("nwarps", [1, 2, 8])
@pytest.mark.parametrize("nrows", [1, 3, 37])
def test_glu_small_and_ragged(qt, nwarps, nrows):
    check_glu(qt, nrows, 2048, nwarps=nwarps, rpb=4, seed=nrows)


@pytest.mark.parametrize("qt,nrows,K", [("Q4_K", 12288, 4096), ("Q6_K", 12288, 4096),
                                         ("Q8_0", 256, 256), ("Q4_0", 4864, 14336)])
def test_glu_shapes(qt, nrows, K):
    check_glu(qt, nrows, K, seed=7)


def test_glu_f32_equals_quantise_then_glu():
    qt, n, K = "Q4_K", 3000, 4096
    Wg, Wu = dev(make_weights(qt, n, K, seed=1)), dev(make_weights(qt, n, K, seed=2))
    x = dev(make_activation(K, seed=3)).reshape(-1)
    a = ops.mmvq_glu_f32(Wg, Wu, qt, x)
    b = ops.mmvq_glu(Wg, Wu, qt, ops.quantize_q8_1(x))
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_glu_chain_graph_matches_eager():
    """quantise -> gate/up -> down as a CUDA graph with PDL equals the eager launches."""
    K, F = 2048, 5120
    Wg, Wu = dev(make_weights("Q4_K", F, K, seed=4)), dev(make_weights("Q4_K", F, K, seed=5))
    Wd = dev(make_weights("Q6_K", K, F, seed=6))
    x = torch.randn(1, K, device="cuda")
    xq = torch.empty(ops.q8_1_bytes(K), dtype=torch.uint8, device="cuda")
    h = torch.empty(1, F, device="cuda")
    hq = torch.empty(ops.q8_1_bytes(F), dtype=torch.uint8, device="cuda")
    y = torch.empty(1, K, device="cuda")
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        ch = ops.Chain()
        ch.add_quantize(x, xq)
        ch.add_mmvq_glu(Wg, Wu, "Q4_K", xq, h)
        ch.add_quantize(h, hq)
        ch.add_mmvq(Wd, "Q6_K", hq, y)
        assert ch.num_steps == 4 and ch.n_launches == 4 and ch.n_mmvq == 3
        ch.instantiate(pdl=True)
        for _ in range(3):
            ch.launch()
    stream.synchronize()
    h_ref = ops.mmvq_glu(Wg, Wu, "Q4_K", ops.quantize_q8_1(x))
    y_ref = ops.mmvq(Wd, "Q6_K", ops.quantize_q8_1(h_ref))
    torch.cuda.synchronize()
    assert torch.equal(h, h_ref) and torch.equal(y, y_ref)
    ch.close()


def test_glu_argument_errors():
    from kernel_anvil import _native
    K = 96  # three Q8_0 blocks: 102-byte rows, not a multiple of 16
    Wg, Wu = dev(make_weights("Q8_0", 4, K)), dev(make_weights("Q8_0", 4, K, seed=1))
    xq = ops.quantize_q8_1(dev(make_activation(K)))
    with pytest.raises(AnvilError, match="multiple of 16 bytes"):
        ops.mmvq_glu(Wg, Wu, "Q8_0", xq)
    K = 1024
    Wg, Wu = dev(make_weights("Q4_K", 8, K)), dev(make_weights("Q4_K", 6, K))
    xq = ops.quantize_q8_1(dev(make_activation(K)))
    with pytest.raises(AnvilError, match="same number of rows"):
        ops.mmvq_glu(Wg, Wu, "Q4_K", xq)
    flat = torch.empty(Wg.numel() + 16, dtype=torch.uint8, device="cuda")
    rc = _native.lib().anvil_mmvq_glu(12, flat.data_ptr() + 1, Wg.data_ptr(), xq.data_ptr(),
                                      flat.data_ptr(), 8, K, 0, 0, 0, None)
    assert rc == _native.ANVIL_ERR_ALIGN
    rc = _native.lib().anvil_mmvq_glu(12, Wg.data_ptr(), Wg.data_ptr(), xq.data_ptr(), None, 8, K, 0, 0,
                                      0, None)
    assert rc == _native.ANVIL_ERR_INVALID
    assert ops.take_device_status() == 0
