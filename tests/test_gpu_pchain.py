"""The persistent chain kernel (anvil_pchain_*) on one GPU.

Every GEMV of a persistent chain must equal what anvil_mmvq computes for the same rows:
bit for bit when the chain picked the same rows per tile and lanes per row as the
single-GEMV launch (same arithmetic, same reduction order), else within the fp32 output
tolerance against the oracle.  Also: repeated launches (the barrier epochs), groups
mixing weight types, the in-kernel quantisation against the quantiser, argument errors."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from kernel_anvil import mmvq as ops  # noqa: E402
from kernel_anvil._native import AnvilError  # noqa: E402
from kernel_anvil.chains import DeviceChain, get_chain  # noqa: E402
from kernel_anvil.mmvq import host_lanes_per_row  # noqa: E402
from kernel_anvil.pchain import PersistentChain, take_status  # noqa: E402
from kernel_anvil.quants import make_activation, make_weights, resolve_type  # noqa: E402
from oracle import oracle  # noqa: E402

pytestmark = pytest.mark.gpu
Y_TOL = 1e-3


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _single(W, qt, x, rpb):
    """anvil_mmvq on the quantiser's Q8_1 of x (the per-GEMV path)."""
    return ops.mmvq(W, qt, ops.quantize_q8_1(x), ncols=x.shape[0], rows_per_block=rpb)


def _check_against_single(pc, idx, W, qt, x, y, nrows, K):
    rpb, lb = pc.gemv_shape(idx)
    ref = _single(W, qt, x, rpb)
    torch.cuda.synchronize()
    info = resolve_type(qt)
    if lb == host_lanes_per_row(K // info.qk, rpb):
        assert torch.equal(y, ref), f"GEMV {idx} ({qt} {nrows}x{K}, rpb {rpb}, lb {lb}) not bit-exact"
    Wn = W.cpu().numpy()
    y_ref = oracle.mmvq(qt, Wn, oracle.quantize_q8_1(x.cpu().numpy()), nrows, K, x.shape[0])
    assert oracle.max_rel_err(y.cpu().numpy(), y_ref) <= Y_TOL


# groups: (K, [(qt, nrows, rows_per_block)]) sharing the group's input
CASES = {
    "one_q4k": [(4096, [("Q4_K", 4096, 0)])],
    "qkv_mixed": [(4096, [("Q4_K", 4096, 0), ("Q4_K", 1024, 0), ("Q6_K", 1024, 0)]),
                  (4096, [("Q4_K", 4096, 0)]),
                  (4096, [("Q4_K", 12288, 0), ("Q4_K", 12288, 0)]),
                  (12288, [("Q6_K", 4096, 0)])],
    "all_types_odd_rows": [(2048, [("Q5_K", 777, 2), ("Q8_0", 333, 4), ("Q4_K", 65, 1)]),
                           (1024, [("Q8_0", 1000, 8), ("Q6_K", 129, 4)])],
    "q80_draft": [(1024, [("Q8_0", 2048, 0), ("Q8_0", 1024, 0), ("Q8_0", 1024, 0)]),
                  (2048, [("Q8_0", 1024, 0)]), (1024, [("Q8_0", 3072, 0), ("Q8_0", 3072, 0)]),
                  (3072, [("Q8_0", 1024, 0)])],
}


@pytest.mark.parametrize("case", sorted(CASES))
@pytest.mark.parametrize("ncols", [1, 2])
def test_pchain_matches_single_gemv(case, ncols):
    pc = PersistentChain()
    items = []
    seed = 10
    for K, gemvs in CASES[case]:
        x = dev(make_activation(K, ncols=ncols, seed=seed))
        pc.add_group(x, wait=True)
        for qt, nrows, rpb in gemvs:
            seed += 1
            W = dev(make_weights(qt, nrows, K, seed=seed))
            y = torch.full((ncols, nrows), float("nan"), device="cuda")
            pc.add_gemv(W, qt, y, nrows=nrows, rows_per_block=rpb)
            items.append((W, qt, x, y, nrows, K))
    pc.instantiate()
    for _ in range(3):  # three launches: the barrier targets advance per launch
        pc.launch()
    torch.cuda.synchronize()
    assert take_status() == 0
    for i, (W, qt, x, y, nrows, K) in enumerate(items):
        assert not torch.isnan(y).any()
        _check_against_single(pc, i, W, qt, x, y, nrows, K)
    pc.close()


def test_pchain_repeated_launches_identical():
    K, nrows = 4096, 3000
    x = dev(make_activation(K, seed=3))
    W = dev(make_weights("Q4_K", nrows, K, seed=4))
    y = torch.empty((1, nrows), device="cuda")
    pc = PersistentChain()
    pc.add_group(x)
    pc.add_gemv(W, "Q4_K", y, nrows=nrows)
    pc.instantiate(nwarps=4, ctas_per_sm=2)
    pc.launch()
    torch.cuda.synchronize()
    first = y.clone()
    for _ in range(20):
        pc.launch()
    torch.cuda.synchronize()
    assert torch.equal(first, y)
    # new input values in the same buffer are picked up by the next launch
    x.mul_(-2.0)
    pc.launch()
    torch.cuda.synchronize()
    assert torch.equal(y, _single(W, "Q4_K", x, pc.gemv_shape(0)[0]))
    pc.close()


def test_device_chain_persistent_equals_graph():
    spec = get_chain("qwen3_8b").head(14)  # two decoder layers, both Q6_K mixes
    a = DeviceChain(spec, executor="graph")
    b = DeviceChain(spec, executor="persistent")
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        a.instantiate()
        a.launch()
        b.launch()
    torch.cuda.synchronize()
    assert take_status() == 0 and ops.take_device_status() == 0
    for ya, yb in zip(a.outputs, b.outputs):
        torch.testing.assert_close(yb, ya, rtol=1e-5, atol=1e-5 * float(ya.abs().max()))
    a.close()
    b.close()


def test_pchain_argument_errors():
    pc = PersistentChain()
    W = torch.zeros(144 * 16, dtype=torch.uint8, device="cuda")
    y = torch.zeros(16, device="cuda")
    with pytest.raises(AnvilError, match="add a group first"):
        pc.add_gemv(W, "Q4_K", y, nrows=1)
    with pytest.raises(AnvilError, match="ncols"):
        pc.add_group(torch.zeros((3, 256), device="cuda"))
    with pytest.raises(AnvilError, match="multiple of 32"):
        pc.add_group(torch.zeros(100, device="cuda"))
    pc.add_group(torch.zeros(512, device="cuda"))
    with pytest.raises(AnvilError, match="outside"):
        pc.add_gemv(W, "Q4_K", y, nrows=4, row0=2, nrows_full=5)
    with pytest.raises(AnvilError, match="empty|no GEMV"):
        pc.instantiate()
    pc.close()


def _half_integer_activation(K, seed):
    """Blocks whose values sit on or next to half-integer multiples of the block scale
    d = amax / 127, where q = roundf(x / d) depends on the last bit of the quotient."""
    rng = np.random.default_rng(seed)
    x = np.empty(K, dtype=np.float32)
    for b in range(K // 32):
        amax = np.float32(rng.choice([127.0, 1.0, 3.0e-3, rng.uniform(0.1, 50.0)]))
        d = np.float32(amax / np.float32(127.0))
        k = rng.integers(-126, 126, size=32).astype(np.float32)
        v = (k + np.float32(0.5)) * d
        nudge = rng.choice([0, 1, -1], size=32)
        v = np.where(nudge == 1, np.nextafter(v, np.float32(np.inf)), v)
        v = np.where(nudge == -1, np.nextafter(v, np.float32(-np.inf)), v).astype(np.float32)
        v[0] = amax  # the block's max sets d
        x[32 * b:32 * b + 32] = v
    return x


@pytest.mark.parametrize("qt", ["Q8_0", "Q4_K"])
def test_pchain_quantisation_at_half_integers(qt):
    K, nrows = 2048, 1024
    x = dev(_half_integer_activation(K, seed=21))
    W = dev(make_weights(qt, nrows, K, seed=22))
    y = torch.empty((1, nrows), device="cuda")
    pc = PersistentChain()
    pc.add_group(x)
    pc.add_gemv(W, qt, y, nrows=nrows)
    pc.instantiate()
    pc.launch()
    torch.cuda.synchronize()
    rpb, lb = pc.gemv_shape(0)
    assert lb == host_lanes_per_row(K // resolve_type(qt).qk, rpb)
    # the quantiser kernel divides every value; the persistent kernel must agree bit for bit
    assert torch.equal(y, _single(W, qt, x.view(1, -1), rpb))
    xq = ops.quantize_q8_1(x.view(1, -1)).cpu().numpy().reshape(-1)
    assert np.array_equal(xq, oracle.quantize_q8_1(x.cpu().numpy()).reshape(-1))
    pc.close()
