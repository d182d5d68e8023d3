"""anvil_mmvq_f32_noalloc through the C ABI: same output as anvil_mmvq_f32 (caller scratch),
call after call, and the size limit of its static Q8_1 buffer rejected on the host.

Collected last (file name) so it also runs after every other GPU test in one process."""
import pytest

torch = pytest.importorskip("torch")

from kernel_anvil import _native  # noqa: E402
from kernel_anvil.mmvq import q8_1_bytes  # noqa: E402
from kernel_anvil.quants import make_activation, make_weights, resolve_type  # noqa: E402

pytestmark = pytest.mark.gpu

# Both entry points quantise x identically.  anvil_mmvq_f32 then runs the dp4a kernel with the
# quantiser fused in; the no-alloc entry point quantises into its static buffer and runs the
# Q8_1 kernel, which for Q4_K / Q5_K from 4 columns on is the tensor-core kernel: the same
# block sums, added up in another order.  So the outputs agree to float rounding: the largest
# difference may be 1e-5 of the largest output (the bar of the tests comparing two kernels).
REL = 1e-5
STATIC_XQ_BYTES = 1 << 20


def _assert_close(a, b):
    diff = float((a - b).abs().max())
    scale = float(b.abs().max()) or 1.0
    assert diff <= REL * scale, f"max |a - b| = {diff:.3e} against max |b| = {scale:.3e}"


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _reference(qt, W, x, nrows, K, ncols):
    info = resolve_type(qt)
    xq = torch.empty(q8_1_bytes(K, ncols), dtype=torch.uint8, device="cuda")
    y = torch.empty((ncols, nrows), dtype=torch.float32, device="cuda")
    rc = _native.lib().anvil_mmvq_f32(info.ggml_type, W.data_ptr(), x.data_ptr(), xq.data_ptr(),
                                      y.data_ptr(), nrows, K, ncols, 0, 0, _stream())
    assert rc == 0, _native.last_error()
    return y


def _noalloc(qt, W, x, nrows, K, ncols, y=None):
    info = resolve_type(qt)
    y = torch.empty((ncols, nrows), dtype=torch.float32, device="cuda") if y is None else y
    rc = _native.lib().anvil_mmvq_f32_noalloc(info.ggml_type, W.data_ptr(), x.data_ptr(),
                                              y.data_ptr(), nrows, K, ncols, 0, 0, _stream())
    assert rc == 0, _native.last_error()
    return y


# The last two shapes use the static buffer the hardest: K = 28672 with 8 columns does not
# fit one launch's shared memory, so the GEMV runs as column chunks that read their Q8_1
# columns at offsets inside the buffer; K = 98304 with 8 columns fills 884,736 of its
# 1,048,576 bytes (one-column chunks, the last reading near the end of the buffer).
@pytest.mark.parametrize("qt,nrows,K,ncols", [("Q4_K", 1000, 4096, 1), ("Q5_K", 257, 2048, 2),
                                              ("Q6_K", 640, 3072, 1), ("Q8_0", 513, 1024, 3),
                                              ("Q4_K", 4096, 12288, 1), ("Q4_K", 256, 28672, 8),
                                              ("Q4_K", 64, 98304, 8)])
def test_noalloc_matches_caller_scratch_two_calls(qt, nrows, K, ncols):
    W = torch.from_numpy(make_weights(qt, nrows, K, seed=11)).cuda()
    xa = torch.from_numpy(make_activation(K, ncols=ncols, seed=12)).cuda()
    xb = torch.from_numpy(make_activation(K, ncols=ncols, seed=13)).cuda() * 3.0
    ya = _noalloc(qt, W, xa, nrows, K, ncols)   # first call: per-device set-up
    yb = _noalloc(qt, W, xb, nrows, K, ncols)   # second call reuses the same buffer
    ra = _reference(qt, W, xa, nrows, K, ncols)
    rb = _reference(qt, W, xb, nrows, K, ncols)
    torch.cuda.synchronize()
    _assert_close(ya, ra)
    _assert_close(yb, rb)
    # the same input again, into the same output buffer: same result
    _noalloc(qt, W, xa, nrows, K, ncols, y=yb)
    torch.cuda.synchronize()
    _assert_close(yb, ra)


def test_noalloc_rejects_oversize_activation():
    K, ncols = 116512, 8  # 8 * (K/32) * 36 = 1048608 bytes, just over the buffer
    assert ncols * (K // 32) * 36 > STATIC_XQ_BYTES
    x = torch.zeros(16, dtype=torch.float32, device="cuda")
    y = torch.zeros(16, dtype=torch.float32, device="cuda")
    W = torch.zeros(256, dtype=torch.uint8, device="cuda")
    rc = _native.lib().anvil_mmvq_f32_noalloc(resolve_type("Q8_0").ggml_type, W.data_ptr(),
                                              x.data_ptr(), y.data_ptr(), 4, K, ncols, 0, 0,
                                              _stream())
    assert rc == _native.ANVIL_ERR_INVALID
    assert "static buffer" in _native.last_error()
    torch.cuda.synchronize()
    assert torch.count_nonzero(y).item() == 0  # nothing was launched
