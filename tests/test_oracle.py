"""The CPU oracle against the reference's pinned semantics (no GPU needed).

Pins, in order of strength:
  1. per-weight dequantisation == gguf-py gguf.quants.dequantize (the reference's declared
     dependency), bit for bit, from committed fixtures and freshly generated blocks;
  2. Q8_1 quantisation == gguf-py's Q8_0 rule (d = amax/127, round half away from zero)
     up to the x/d vs x*(1/d) rounding difference, measured and bounded;
  3. integer block sums and y are self-consistent with dequant(W) . dequant(Q8_1(x)).
"""
import numpy as np
import pytest

from kernel_anvil.quants import QUANT_TYPES, make_activation, make_weights
from oracle import oracle

TYPES = ["Q4_K", "Q5_K", "Q6_K", "Q8_0", "Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q2_K", "Q3_K", "IQ4_NL",
         "IQ4_XS", "IQ2_XXS", "IQ2_XS", "IQ2_S", "IQ3_XXS", "IQ3_S", "IQ1_S", "IQ1_M"]


@pytest.mark.parametrize("qt", TYPES)
def test_dequant_matches_gguf_fixture(golden_dir, qt):
    f = np.load(golden_dir / f"dequant_{qt}.npz")
    got = oracle.dequantize(qt, f["W"], int(f["nrows"]), int(f["K"]))
    np.testing.assert_array_equal(got.view(np.uint32), f["dequant"].view(np.uint32))


@pytest.mark.parametrize("qt", TYPES)
@pytest.mark.parametrize("seed", [0, 3])
def test_dequant_matches_gguf_live(qt, seed):
    gguf = pytest.importorskip("gguf")
    n, k = 16, 1024
    W = make_weights(qt, n, k, seed=seed)
    ref = gguf.quants.dequantize(W, getattr(gguf.GGMLQuantizationType, qt)).astype(np.float32)
    got = oracle.dequantize(qt, W, n, k)
    np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_half_conversion_matches_numpy():
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * np.float32(10.0) ** rng.integers(-9, 5, 20000),
        np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e-8, 2.98e-8, 5.96e-8, 6.1e-5, 6.097e-5,
                  np.inf, -np.inf, 1.0009765625, 1.00048828125, 1.00146484375], dtype=np.float32),
    ])
    with np.errstate(over="ignore"):
        want = vals.astype(np.float16).view(np.uint16)
    got = np.array([oracle.float_to_half_bits(float(v)) for v in vals], dtype=np.uint16)
    np.testing.assert_array_equal(got, want)


def test_q8_1_against_gguf_q8_0_rule(golden_dir):
    f = np.load(golden_dir / "q8_0_gguf.npz")
    x, q80 = f["x"], f["q8_0"]
    xq = oracle.quantize_q8_1(x)
    ncols, K = x.shape
    b1 = xq.reshape(-1, 36)
    b0 = q80.reshape(-1, 34)
    # d: identical rule and rounding (fp32 amax/127 -> fp16)
    np.testing.assert_array_equal(b1[:, 0:2], b0[:, 0:2])
    # quants: x/d (llama.cpp CUDA) vs x*(1/d) (gguf-py) may differ by one ulp of rounding
    diff = b1[:, 4:].view(np.int8).astype(int) - b0[:, 2:].view(np.int8).astype(int)
    assert np.abs(diff).max() <= 1
    assert np.count_nonzero(diff) <= 0.001 * diff.size
    # the all-zero block (first block of column 1) quantises to d = 0, s = 0, q = 0
    assert not b1[K // 32, :].any()


def test_q8_1_sum_field_is_fp16_of_block_sum():
    x = make_activation(4096, ncols=3, seed=9)
    xq = oracle.quantize_q8_1(x).reshape(-1, 36)
    s = xq[:, 2:4].copy().view(np.float16).astype(np.float64).ravel()
    exact = x.reshape(-1, 32).astype(np.float64).sum(axis=1)
    assert np.allclose(s, exact, rtol=2e-3, atol=1e-3)


def test_q8_1_round_half_away_and_range():
    # values that land exactly on .5 after division must round away from zero
    x = np.zeros((1, 32), dtype=np.float32)
    x[0, 0] = 127.0
    x[0, 1] = 2.5
    x[0, 2] = -2.5
    x[0, 3] = -127.0
    q = oracle.quantize_q8_1(x)[0, 4:].view(np.int8)
    assert q[0] == 127 and q[3] == -127
    assert q[1] == 3 and q[2] == -3


@pytest.mark.parametrize("qt", TYPES)
@pytest.mark.parametrize("ncols", [1, 3])
def test_mmvq_equals_dequant_dot(qt, ncols):
    n, k = 24, 1024
    W = make_weights(qt, n, k, seed=2)
    x = make_activation(k, ncols=ncols, seed=4)
    xq = oracle.quantize_q8_1(x)
    y = oracle.mmvq(qt, W, xq, n, k, ncols)
    wd = oracle.dequantize(qt, W, n, k).astype(np.float64)
    xd = oracle.dequantize_q8_1(xq, k).astype(np.float64)
    ref = xd @ wd.T
    assert oracle.max_rel_err(y, ref) < 1e-6  # fp32 rounding of the dequantised weights


@pytest.mark.parametrize("qt", TYPES)
def test_block_sums_reconstruct_y(qt):
    """sum over sub-blocks of (scale terms x exact int sums) == oracle y."""
    n, k = 6, 512
    W = make_weights(qt, n, k, seed=5)
    xq = oracle.quantize_q8_1(make_activation(k, seed=6))
    sums = oracle.block_sums(qt, W, xq, n, k)[0].astype(np.float64)
    xb = xq.reshape(-1, 36)
    d8 = xb[:, 0:2].copy().view(np.float16).astype(np.float64).ravel()
    qsum = xb[:, 4:].view(np.int8).astype(np.int64).sum(axis=1)
    info = QUANT_TYPES[qt]
    blocks = W.reshape(n, k // info.qk, info.block_size)
    y = np.zeros(n)
    for r in range(n):
        for b in range(k // info.qk):
            blk = blocks[r, b]
            if qt == "Q8_0" or qt in ("Q4_0", "Q5_0"):
                d = blk[0:2].copy().view(np.float16).astype(np.float64)[0]
                y[r] += d * d8[b] * sums[r, b]
            elif qt in ("Q4_1", "Q5_1"):  # unsigned quants; the min m times d8 * sum(q8)
                d, m = blk[0:4].copy().view(np.float16).astype(np.float64)
                y[r] += d * d8[b] * sums[r, b] + m * d8[b] * qsum[b]
            elif qt == "IQ4_NL":
                d = blk[0:2].copy().view(np.float16).astype(np.float64)[0]
                y[r] += d * d8[b] * sums[r, b]
            elif qt.startswith(("IQ1", "IQ2", "IQ3")):
                # w = d * F * (2 ls + 1 | 1 + 2 ls) * level per scale group of 16 or 32
                # (gguf-py IQ*.dequantize_blocks scale rules); IQ1_M's d is in the scale words
                if qt == "IQ1_M":
                    sw = blk[48:56].copy().view(np.uint16).astype(np.int64)
                    bits = sum(((int(sw[i]) >> 12) & 15) << (4 * i) for i in range(4))
                    d = float(np.array([bits], dtype=np.uint16).view(np.float16)[0])
                else:
                    d = float(blk[0:2].copy().view(np.float16)[0])
                g16 = qt in ("IQ2_XS", "IQ2_S", "IQ1_M")
                F = {"IQ3_XXS": 0.25, "IQ3_S": 1.0}.get(qt, 0.125)
                for g in range(16 if g16 else 8):
                    if qt == "IQ2_XXS":
                        ls = int(blk[2 + 8 * g + 7]) >> 4
                    elif qt in ("IQ2_XS", "IQ2_S"):
                        ls = (int(blk[(66 if qt == "IQ2_XS" else 74) + g // 2]) >> (4 * (g % 2))) & 15
                    elif qt == "IQ3_XXS":
                        ls = int(blk[66 + 4 * g + 3]) >> 4
                    elif qt == "IQ3_S":
                        ls = (int(blk[106 + g // 2]) >> (4 * (g % 2))) & 15
                    elif qt == "IQ1_S":
                        ls = (int(blk[34 + 2 * g]) | (int(blk[35 + 2 * g]) << 8)) >> 12 & 7
                    else:
                        ls = ((int(blk[48 + 2 * (g // 4)]) | (int(blk[49 + 2 * (g // 4)]) << 8))
                              >> (3 * (g % 4))) & 7
                    kb = 8 * b + (g // 2 if g16 else g)
                    y[r] += d * F * (2 * ls + 1) * d8[kb] * sums[r, (16 if g16 else 8) * b + g]
            elif qt == "IQ4_XS":
                d = blk[0:2].copy().view(np.float16).astype(np.float64)[0]
                sh = int(blk[2]) | (int(blk[3]) << 8)
                for j in range(8):
                    ls = ((int(blk[4 + j // 2]) >> (4 * (j % 2))) & 15) | (((sh >> (2 * j)) & 3) << 4)
                    y[r] += d * (ls - 32) * d8[8 * b + j] * sums[r, 8 * b + j]
            elif qt in ("Q2_K", "Q3_K"):
                # 16 groups of 16 weights; Q2_K: nibble scale and min, Q3_K: 6-bit scale - 32
                xq16 = xb[:, 4:].view(np.int8).astype(np.int64).reshape(-1, 2, 16).sum(axis=2)
                for g in range(16):
                    kb = 8 * b + g // 2
                    if qt == "Q2_K":
                        d, dmin = blk[80:84].copy().view(np.float16).astype(np.float64)
                        sc, m = int(blk[g]) & 15, int(blk[g]) >> 4
                        y[r] += d * sc * d8[kb] * sums[r, 16 * b + g] - dmin * m * d8[kb] * xq16[kb, g % 2]
                    else:
                        d = blk[108:110].copy().view(np.float16).astype(np.float64)[0]
                        s = blk[96:108].astype(int)
                        lo = s[g] & 15 if g < 8 else s[g - 8] >> 4
                        sc = (lo | (((s[8 + g % 4] >> (2 * (g // 4))) & 3) << 4)) - 32
                        y[r] += d * sc * d8[kb] * sums[r, 16 * b + g]
            elif qt == "Q6_K":
                d = blk[208:210].copy().view(np.float16).astype(np.float64)[0]
                sc = blk[192:208].view(np.int8).astype(np.float64)
                for g in range(16):
                    y[r] += d * sc[g] * d8[8 * b + g // 2] * sums[r, 16 * b + g]
            else:
                d, dmin = blk[0:4].copy().view(np.float16).astype(np.float64)
                s = blk[4:16].astype(int)
                for j in range(8):
                    if j < 4:
                        sc, m = s[j] & 63, s[j + 4] & 63
                    else:
                        sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4)
                        m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4)
                    kb = 8 * b + j
                    y[r] += d * sc * d8[kb] * sums[r, kb] - dmin * m * d8[kb] * qsum[kb]
    ref = oracle.mmvq(qt, W, xq, n, k)[0]
    assert oracle.max_rel_err(y, ref) < 1e-12


def test_oracle_threads_reported():
    assert oracle.num_threads() >= 1


def test_division_free_quantiser_arithmetic():
    """The kernels compute the quantiser's two IEEE quotients without a division:
    d = RN32(amax/127) as fp32(fp64(amax) * RN64(1/127)), and q = roundf(RN32(x/d)) as
    roundf(x * RN32(1/d)) except within 1e-4 of a half-integer, where RN32(fp64(x) * RN64(1/d))
    is used.  Restated here in numpy and checked against the correctly rounded quotients (fp64
    division then fp32 rounding, exact since 53 >= 2 * 24 + 2)."""
    c = np.float64(1.0) / np.float64(127.0)
    m = np.arange(1 << 23, dtype=np.uint32)
    for am in (((127 << 23) | m).view(np.float32), m[1:].view(np.float32),
               ((254 << 23) | m).view(np.float32)):
        got = (am.astype(np.float64) * c).astype(np.float32)
        ref = (am.astype(np.float64) / np.float64(127.0)).astype(np.float32)
        assert np.array_equal(got, ref)

    rng = np.random.default_rng(7)
    n = 2_000_000
    amax = np.abs(rng.standard_normal(n)).astype(np.float32) * np.float32(10.0) ** rng.integers(-30, 30, n)
    amax = amax.astype(np.float32)
    d = (amax.astype(np.float64) * c).astype(np.float32)
    d = np.where(d == 0, np.float32(1.0), d).astype(np.float32)
    k = rng.integers(-127, 127, n).astype(np.float32)
    x = ((k + np.float32(0.5)) * d).astype(np.float32)  # on or next to half-integer multiples of d
    nudge = rng.integers(-2, 3, n)
    for s in (1, 2):
        x = np.where(nudge >= s, np.nextafter(x, np.float32(np.inf)), x)
        x = np.where(nudge <= -s, np.nextafter(x, np.float32(-np.inf)), x)
    x = np.concatenate([x, (rng.standard_normal(n) * 64 * d).astype(np.float32)])
    d = np.concatenate([d, d])
    rd64 = np.float64(1.0) / d.astype(np.float64)
    rd = rd64.astype(np.float32)
    t = (x * rd).astype(np.float32)
    f = np.abs(t) - np.floor(np.abs(t))
    exact = (x.astype(np.float64) * rd64).astype(np.float32)
    t_used = np.where(np.abs(f - np.float32(0.5)) > np.float32(1e-4), t, exact)
    ref = (x.astype(np.float64) / d.astype(np.float64)).astype(np.float32)
    # roundf: round half away from zero
    rnd = lambda v: np.sign(v) * np.floor(np.abs(v) + np.float32(0.5))  # noqa: E731
    assert np.array_equal(rnd(t_used.astype(np.float64)), rnd(ref.astype(np.float64)))
    assert np.array_equal(exact, ref)  # the fp64 route alone is exact for every sample


@pytest.mark.parametrize("qt", ["Q4_K", "Q5_K", "Q2_K", "Q4_1", "Q5_1", "Q6_K", "Q8_0"])
def test_device_weights_are_centred(qt):
    """The chains' synthetic weights have mean ~0 (no offset shared by every output row)."""
    pytest.importorskip("torch")
    from kernel_anvil.quants import make_weights_device

    nrows, K = 256, 4096
    W = make_weights_device(qt, nrows, K, seed=5, device="cpu").numpy()
    w = oracle.dequantize(qt, W, nrows, K).astype(np.float64)
    assert abs(w.mean()) < 0.02 * w.std(), (w.mean(), w.std())


def test_iq_sign_table_is_even_parity():
    """The sign bytes of the I-quants (gguf-py IQ2_XXS.ksigns): bit 7 makes the count of set
    bits even, so 7 stored bits carry 8 signs."""
    gguf = pytest.importorskip("gguf")
    ks = np.frombuffer(gguf.quants.IQ2_XXS.ksigns, dtype=np.uint8)
    want = [i | ((bin(i).count("1") & 1) << 7) for i in range(128)]
    assert ks.tolist() == want


def test_type_ids_match_ggml():
    """Every ggml type id this build uses (kernels, smithy JSON keys) is gguf-py's."""
    gguf = pytest.importorskip("gguf")
    from kernel_anvil.codegen import GGML_TYPE_MAP

    for name, info in QUANT_TYPES.items():
        assert info.ggml_type == int(getattr(gguf.GGMLQuantizationType, name)), name
        assert GGML_TYPE_MAP[name] == info.ggml_type, name
        assert oracle.TYPE_IDS[name] == info.ggml_type, name
