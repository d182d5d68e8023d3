"""GPU parity of the sm_100a kernels against the CPU oracle, through the C ABI.

Bars (stated here, checked below):
  * Q8_1 quantisation: bit-exact.
  * MMVQ integer block sums (the production kernel run in its probe mode): bit-exact.
  * MMVQ fp32 y: max|y - y_ref| / max|y_ref| <= 1e-3 against dequant(W) . dequant(Q8_1(x))
    evaluated in float64 by the oracle (the tolerance the north-star states).
"""
import json

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from kernel_anvil import mmvq as ops  # noqa: E402
from kernel_anvil._native import AnvilError  # noqa: E402
from kernel_anvil.quants import make_activation, make_weights  # noqa: E402
from oracle import oracle  # noqa: E402

pytestmark = pytest.mark.gpu

TYPES = ["Q4_K", "Q5_K", "Q6_K", "Q8_0", "Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q2_K", "Q3_K", "IQ4_NL",
         "IQ4_XS", "IQ2_XXS", "IQ2_XS", "IQ2_S", "IQ3_XXS", "IQ3_S", "IQ1_S", "IQ1_M"]
Y_TOL = 1e-3


def dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run_case(qt, nrows, K, ncols=1, nwarps=0, rpb=0, seed=0):
    W = make_weights(qt, nrows, K, seed=seed)
    x = make_activation(K, ncols=ncols, seed=seed + 1)
    xq_ref = oracle.quantize_q8_1(x)
    Wd, xd = dev(W), dev(x)
    xq = ops.quantize_q8_1(xd)
    y = ops.mmvq(Wd, qt, xq, ncols=ncols, nwarps=nwarps, rows_per_block=rpb)
    sums = ops.block_sums(Wd, qt, xq, ncols=ncols, nwarps=nwarps, rows_per_block=rpb)
    torch.cuda.synchronize()
    return W, xq_ref, xq.cpu().numpy(), y.cpu().numpy(), sums.cpu().numpy()


def check_case(qt, nrows, K, ncols=1, nwarps=0, rpb=0, seed=0):
    W, xq_ref, xq, y, sums = run_case(qt, nrows, K, ncols, nwarps, rpb, seed)
    np.testing.assert_array_equal(xq.reshape(-1), xq_ref.reshape(-1))
    np.testing.assert_array_equal(sums, oracle.block_sums(qt, W, xq_ref, nrows, K, ncols))
    y_ref = oracle.mmvq(qt, W, xq_ref, nrows, K, ncols)
    err = oracle.max_rel_err(y, y_ref)
    assert err <= Y_TOL, f"{qt} {nrows}x{K} ncols={ncols} nw={nwarps} rpb={rpb}: err {err:.3e}"
    return err


# ---- quantiser ---------------------------------------------------------------------

@pytest.mark.parametrize("K,ncols", [(32, 1), (1024, 3), (4096, 1), (12288, 2), (4096, 8)])
def test_quantize_q8_1_bit_exact(K, ncols):
    x = make_activation(K, ncols=ncols, seed=K + ncols)
    x[0, :32] = 0.0                          # all-zero block: d = 0, q = 0
    x[0, 32:64] *= 1e-30                     # tiny magnitudes (subnormal d)
    if K >= 128:
        x[0, 64:96] = np.linspace(-5, 5, 32)  # exact ties after division
        x[0, 96:128] = 3.0e4                  # large, equal values
    got = ops.quantize_q8_1(dev(x)).cpu().numpy()
    np.testing.assert_array_equal(got.reshape(-1), oracle.quantize_q8_1(x).reshape(-1))


# ---- MMVQ parity ---------------------------------------------------------------------

@pytest.mark.parametrize("qt", TYPES)
@pytest.mark.parametrize("nwarps", [1, 2, 4, 8])
@pytest.mark.parametrize("rpb", [1, 2, 4, 8])
def test_config_grid_bit_exact(qt, nwarps, rpb):
    """The autoforge grid (nwarps x rpb) on one shape with a ragged row count."""
    check_case(qt, 37, 2048, 1, nwarps, rpb, seed=3)


@pytest.mark.parametrize("qt", TYPES)
@pytest.mark.parametrize("ncols", range(1, 9))
def test_batched_columns(qt, ncols):
    check_case(qt, 70, 1024, ncols, 4, 2, seed=ncols)


@pytest.mark.parametrize("qt,nrows,K", [
    ("Q4_K", 1, 256), ("Q4_K", 3, 256), ("Q4_K", 4096, 4096),
    ("Q5_K", 5, 512), ("Q5_K", 1000, 10240),
    ("Q6_K", 1, 256), ("Q6_K", 33, 1024),      # 840-byte rows: not 16-byte multiples
    ("Q6_K", 17, 3072), ("Q6_K", 9, 5120),     # 2520 / 4200-byte rows
    ("Q6_K", 1024, 4096), ("Q6_K", 300, 12288),
    ("Q8_0", 1, 32), ("Q8_0", 13, 96),         # 102-byte rows
    ("Q4_0", 1, 32), ("Q4_0", 7, 96), ("Q4_0", 4096, 4096),   # 18- / 54-byte rows
    ("Q4_1", 5, 64), ("Q4_1", 2048, 4096),
    ("Q5_0", 3, 32), ("Q5_0", 11, 160), ("Q5_0", 1024, 14336),  # 22- / 110-byte rows
    ("Q5_1", 9, 224), ("Q5_1", 1024, 4096),
    ("Q8_0", 7, 1056), ("Q8_0", 3072, 1024), ("Q8_0", 1024, 3072),
    # lattice I-quants: one-block rows of 50..110 bytes (no 16-byte multiple), long rows
    ("IQ2_XXS", 3, 256), ("IQ2_XXS", 4096, 4096), ("IQ2_XS", 5, 768), ("IQ2_XS", 1024, 4096),
    ("IQ2_S", 7, 256), ("IQ2_S", 2048, 4096), ("IQ3_XXS", 9, 512), ("IQ3_XXS", 4096, 4096),
    ("IQ3_S", 1, 256), ("IQ3_S", 1024, 12288), ("IQ1_S", 11, 256), ("IQ1_S", 4096, 4096),
    ("IQ1_M", 3, 1280), ("IQ1_M", 2048, 8192),
])
def test_shapes(qt, nrows, K):
    check_case(qt, nrows, K, 1, 0, 0, seed=nrows)


def test_config0_full_size():
    """Q4_K 4096 x 4096, batch 1: the single-GEMV workload."""
    err = check_case("Q4_K", 4096, 4096, 1, 0, 0, seed=0)
    assert err < 1e-5


@pytest.mark.parametrize("qt,nrows,K", [("Q4_K", 12288, 4096), ("Q6_K", 4096, 12288),
                                        ("Q4_K", 28672, 8192), ("Q4_K", 8192, 28672)])
def test_large_shapes_y(qt, nrows, K):
    W = make_weights(qt, nrows, K, seed=1)
    x = make_activation(K, seed=2)
    xq_ref = oracle.quantize_q8_1(x)
    y = ops.mmvq(dev(W), qt, ops.quantize_q8_1(dev(x))).cpu().numpy()
    assert oracle.max_rel_err(y, oracle.mmvq(qt, W, xq_ref, nrows, K)) <= Y_TOL


@pytest.mark.parametrize("qt", TYPES)
def test_fused_f32_path_matches_two_step(qt):
    K = 2048
    W = dev(make_weights(qt, 300, K, seed=8))
    x = dev(make_activation(K, ncols=2, seed=9))
    y1 = ops.mmvq(W, qt, ops.quantize_q8_1(x), ncols=2)
    y2 = ops.mmvq_f32(W, qt, x)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)


@pytest.mark.parametrize("qt,ncols", [("Q4_K", 8), ("Q6_K", 7), ("Q8_0", 6), ("Q2_K", 8)])
def test_long_rows_many_columns_in_chunks(qt, ncols):
    """K = 28672 with 6-8 columns: the staged activation exceeds shared memory, so the launch
    runs in column chunks; y and the int32 block sums still meet the bars, and the fp32-input
    path equals quantise + MMVQ."""
    K = 28672
    check_case(qt, 300, K, ncols, seed=ncols)
    W = dev(make_weights(qt, 64, K, seed=1))
    x = dev(make_activation(K, ncols=ncols, seed=2))
    with ops.tensor_cores(0):  # the same dp4a kernel on both paths: the same bits
        y1 = ops.mmvq(W, qt, ops.quantize_q8_1(x), ncols=ncols)
    y2 = ops.mmvq_f32(W, qt, x)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    # Q4_K at 4+ columns takes the tensor-core kernel by default: other summation order
    y3 = ops.mmvq(W, qt, ops.quantize_q8_1(x), ncols=ncols)
    torch.cuda.synchronize()
    assert oracle.max_rel_err(y3.cpu().numpy(), y2.cpu().numpy()) <= 1e-5


def test_pdl_launch_same_result():
    K = 4096
    W = dev(make_weights("Q4_K", 512, K, seed=4))
    x = dev(make_activation(K, seed=5))
    y1 = ops.mmvq(W, "Q4_K", ops.quantize_q8_1(x))
    y2 = ops.mmvq(W, "Q4_K", ops.quantize_q8_1(x, pdl=True), pdl=True)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)


def test_chain_graph_matches_eager():
    """A small decode-shaped chain captured as a CUDA graph with PDL equals eager launches."""
    torch.manual_seed(0)
    shapes = [("Q4_K", 512, 1024, "a"), ("Q6_K", 256, 1024, "a"), ("Q4_K", 1024, 512, "b"),
              ("Q8_0", 768, 2048, "c"), ("Q5_K", 512, 2048, "c")]
    Ks = {"a": 1024, "b": 512, "c": 2048}
    xs = {k: torch.randn(1, K, device="cuda") for k, K in Ks.items()}
    xqs = {k: torch.empty(ops.q8_1_bytes(K), dtype=torch.uint8, device="cuda") for k, K in Ks.items()}
    Ws = [dev(make_weights(qt, n, K, seed=i)) for i, (qt, n, K, _) in enumerate(shapes)]
    ys = [torch.empty(1, n, device="cuda") for (_, n, _, _) in shapes]
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        ch = ops.Chain()
        seen = set()
        for (qt, n, K, a), W, y in zip(shapes, Ws, ys):
            if a not in seen:
                ch.add_quantize(xs[a], xqs[a])
                seen.add(a)
            ch.add_mmvq(W, qt, xqs[a], y)
        assert ch.num_steps == len(shapes) + len(Ks)
        ch.instantiate(pdl=True)
        for _ in range(3):
            ch.launch()
    stream.synchronize()
    for (qt, n, K, a), W, y in zip(shapes, Ws, ys):
        ref = ops.mmvq(W, qt, ops.quantize_q8_1(xs[a]))
        torch.cuda.synchronize()
        assert torch.equal(y, ref), qt
    ch.close()


def test_smithy_table_drives_plan(sandbox_home, monkeypatch, tmp_path):
    from kernel_anvil import _native

    cfg = {"configs": {"12": {"2,2": {"nwarps": 2, "rows_per_block": 4}}}}
    p = tmp_path / "c.json"
    p.write_text(json.dumps(cfg))
    monkeypatch.setenv("SMITHY_CONFIG", str(p))
    _native.lib().anvil_smithy_reset()
    try:
        pl = ops.plan("Q4_K", 4096, 4096)
        assert (pl["nwarps"], pl["rows_per_block"]) == (2, 4)
        pl = ops.plan("Q4_K", 4096, 4096, nwarps=8, rows_per_block=1)  # explicit wins
        assert (pl["nwarps"], pl["rows_per_block"]) == (8, 1)
    finally:
        _native.lib().anvil_smithy_reset()


# ---- argument errors (rejected on the host, nothing launched) -------------------------

def test_argument_errors():
    K = 1024
    W = dev(make_weights("Q4_K", 8, K))
    xq = ops.quantize_q8_1(dev(make_activation(K)))
    with pytest.raises(AnvilError, match="16-byte aligned"):
        flat = torch.empty(W.numel() + 16, dtype=torch.uint8, device="cuda")
        ops.mmvq(flat[1:1 + W.numel()], "Q4_K", xq, nrows=8, K=K)
    with pytest.raises(ValueError, match="divisible by 256"):
        ops.mmvq(W.view(-1), "Q4_K", xq, nrows=8, K=1000)
    from kernel_anvil import _native
    rc = _native.lib().anvil_mmvq(12, W.data_ptr(), xq.data_ptr(), xq.data_ptr(), 8, 1000, 1, 0, 0, None)
    assert rc == _native.ANVIL_ERR_INVALID and "multiple of the block size" in _native.last_error()
    with pytest.raises(AnvilError, match="ncols"):
        ops.mmvq(W, "Q4_K", torch.zeros(9 * ops.q8_1_bytes(K), dtype=torch.uint8, device="cuda"), ncols=9)
    with pytest.raises(AnvilError, match="CUDA tensor"):
        ops.mmvq(W.cpu(), "Q4_K", xq)
    with pytest.raises(ValueError, match="unsupported quant type"):
        ops.mmvq(W, "Q8_K", xq)  # ggml's dot-product intermediate type: no MMVQ kernel


def test_no_device_wait_gave_up():
    torch.cuda.synchronize()
    assert ops.take_device_status() == 0


# ---- grouped launches: several GEMVs on one input -------------------------------------

@pytest.mark.parametrize("qt,rows,K", [("Q4_K", (4096, 1024, 1024), 4096), ("Q6_K", (700, 129), 2048),
                                       ("Q8_0", (2048, 1024, 1024, 3), 1024), ("Q5_K", (512,), 4096)])
@pytest.mark.parametrize("ncols", [1, 3])
def test_grouped_matches_single(qt, rows, K, ncols):
    Ws = [dev(make_weights(qt, n, K, seed=40 + i)) for i, n in enumerate(rows)]
    x = dev(make_activation(K, ncols=ncols, seed=41))
    ys = ops.mmvq_grouped_f32(Ws, qt, x, nwarps=4, rows_per_block=4)
    for W, n, y in zip(Ws, rows, ys):
        ref = ops.mmvq_f32(W, qt, x, nwarps=4, rows_per_block=4)
        torch.cuda.synchronize()
        assert torch.equal(y, ref)  # same launch shape: the same arithmetic in the same order
    # the built-in launch shape, against the oracle
    ys = ops.mmvq_grouped_f32(Ws, qt, x)
    xq = oracle.quantize_q8_1(x.cpu().numpy())
    for W, n, y in zip(Ws, rows, ys):
        y_ref = oracle.mmvq(qt, W.cpu().numpy(), xq, n, K, ncols)
        assert oracle.max_rel_err(y.cpu().numpy(), y_ref) <= Y_TOL


def test_grouped_chain_equals_per_gemv_chain():
    from kernel_anvil.chains import DeviceChain, get_chain

    spec = get_chain("qwen3_8b").head(14)
    a = DeviceChain(spec, executor="graph")
    b = DeviceChain(spec, executor="graph", grouped=True)
    c = DeviceChain(spec, executor="graph", grouped=True, fused=True)
    assert c.launches_per_step < b.launches_per_step < a.launches_per_step
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for dc in (a, b, c):
            dc.instantiate()
            dc.launch()
    torch.cuda.synchronize()
    assert ops.take_device_status() == 0
    for ya, yb, yc in zip(a.outputs, b.outputs, c.outputs):
        torch.testing.assert_close(yb, ya, rtol=1e-5, atol=1e-5 * float(ya.abs().max()))
        torch.testing.assert_close(yc, ya, rtol=1e-5, atol=1e-5 * float(ya.abs().max()))
    for dc in (a, b, c):
        dc.close()


def test_grouped_argument_errors():
    W = dev(make_weights("Q4_K", 8, 1024))
    x = dev(make_activation(1024))
    with pytest.raises(AnvilError, match="1..4"):
        ops.mmvq_grouped_f32([W] * 5, "Q4_K", x)
    with pytest.raises(AnvilError, match="1..4"):
        ops.mmvq_grouped_f32([], "Q4_K", x)


# ---- tensor-core path (mma.sync m16n8k32 int8): Q4_K / Q5_K, 2..8 columns --------------

@pytest.mark.parametrize("qt", ["Q4_K", "Q5_K"])
@pytest.mark.parametrize("nrows,K,ncols", [(1, 256, 2), (17, 1280, 3), (1000, 4096, 8),
                                           (12288, 4096, 8), (300, 12288, 5), (64, 28672, 8),
                                           (4096, 1024, 2), (33, 768, 7)])
def test_tensor_core_path_matches_oracle(qt, nrows, K, ncols):
    """Block sums from the MMA tiles bit-exact, y within the tolerance, and the dp4a kernel's
    y within fp32 rounding of it; ragged tails (rows not a multiple of 16, K not a multiple
    of the 1024-weight chunk) included."""
    with ops.tensor_cores(2):
        W, xq_ref, xq, y, sums = run_case(qt, nrows, K, ncols, seed=nrows + K)
    np.testing.assert_array_equal(sums, oracle.block_sums(qt, W, xq_ref, nrows, K, ncols))
    y_ref = oracle.mmvq(qt, W, xq_ref, nrows, K, ncols)
    assert oracle.max_rel_err(y, y_ref) <= Y_TOL
    with ops.tensor_cores(0):
        _, _, _, y_dp4a, sums_dp4a = run_case(qt, nrows, K, ncols, seed=nrows + K)
    np.testing.assert_array_equal(sums_dp4a, sums)
    assert oracle.max_rel_err(y, y_dp4a) <= 1e-5


def test_tensor_core_switch_and_grouped():
    with pytest.raises(AnvilError):
        ops.set_tensor_core_min_cols(1)
    with pytest.raises(AnvilError):
        ops.set_tensor_core_min_cols(9)
    assert ops.tensor_core_min_cols() == 4
    # a grouped launch (three matrices on one activation) through the same tiles
    K, rows, ncols = 2048, [300, 17, 1024], 4
    Ws = [make_weights("Q4_K", r, K, seed=80 + i) for i, r in enumerate(rows)]
    x = make_activation(K, ncols=ncols, seed=90)
    xq = ops.quantize_q8_1(dev(x))
    ys = [torch.empty((ncols, r), dtype=torch.float32, device="cuda") for r in rows]
    ch = ops.Chain()
    ch.add_mmvq_grouped([dev(w) for w in Ws], "Q4_K", xq, ys, rows, K=K, ncols=ncols)
    with torch.cuda.stream(torch.cuda.Stream()):
        ch.instantiate()
        ch.launch()
    torch.cuda.synchronize()
    xq_ref = oracle.quantize_q8_1(x)
    for W, y, r in zip(Ws, ys, rows):
        assert oracle.max_rel_err(y.cpu().numpy(), oracle.mmvq("Q4_K", W, xq_ref, r, K, ncols)) <= Y_TOL
    ch.close()
