"""The persistent chain kernel (anvil_pchain_*) on one GPU.

Fixed-input GEMVs must equal what anvil_mmvq computes for the same rows: bit for bit when
the chain picked the same rows per tile and lanes per row as the single-GEMV launch, else
within the fp32 output tolerance against the oracle.  Chained groups (inputs computed from
earlier outputs inside the kernel) are checked against the oracle GEMV by GEMV, and their
in-kernel quantisation (quants and fp32 d8) bit for bit against the oracle's chained-input
rule.  Also: repeated
launches (epochs and the two output parities), gate/up pairs, a wait that runs out, and
argument errors."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from chain_oracle import Y_TOL, check_chain  # noqa: E402
from kernel_anvil import mmvq as ops  # noqa: E402
from kernel_anvil._native import ANVIL_ERR_TIMEOUT, AnvilError  # noqa: E402
from kernel_anvil.chains import DeviceChain, get_chain  # noqa: E402
from kernel_anvil.mmvq import host_lanes_per_row  # noqa: E402
from kernel_anvil.pchain import (PersistentChain, output_words_bytes, raise_on_status,  # noqa: E402
                                 set_wait_limit_ns, take_status, trace_summary)
from kernel_anvil.quants import make_activation, make_weights, resolve_type  # noqa: E402
from oracle import oracle  # noqa: E402

pytestmark = pytest.mark.gpu


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


# groups: (K, [(qt, nrows, rows_per_block)]) sharing the group's fixed input
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
def test_pchain_fixed_inputs_match_single_gemv(case, ncols):
    pc = PersistentChain()
    items = []
    seed = 10
    for K, gemvs in CASES[case]:
        x = dev(make_activation(K, ncols=ncols, seed=seed))
        pc.add_group(x)
        for qt, nrows, rpb in gemvs:
            seed += 1
            W = dev(make_weights(qt, nrows, K, seed=seed))
            idx = pc.add_gemv(W, qt, nrows=nrows, rows_per_block=rpb)
            items.append((idx, W, qt, x, nrows, K))
    pc.instantiate()
    for _ in range(3):  # three launches: epochs 1..3, both output parities
        pc.launch()
    torch.cuda.synchronize()
    assert take_status() == 0
    assert pc.epoch == 3
    for idx, W, qt, x, nrows, K in items:
        y = pc.output(idx)
        assert not torch.isnan(y).any()
        _check_against_single(pc, idx, W, qt, x, y, nrows, K)
    pc.close()


def test_pchain_repeated_launches_identical():
    K, nrows = 4096, 3000
    x = dev(make_activation(K, seed=3))
    W = dev(make_weights("Q4_K", nrows, K, seed=4))
    pc = PersistentChain()
    pc.add_group(x)
    pc.add_gemv(W, "Q4_K", nrows=nrows)
    pc.instantiate(nwarps=4, ctas_per_sm=2)
    pc.launch()
    first = pc.output(0)
    for _ in range(21):  # ends on the other parity
        pc.launch()
    torch.cuda.synchronize()
    assert torch.equal(first, pc.output(0))
    # new input values in the same buffer are picked up by the next launch
    x.mul_(-2.0)
    pc.launch()
    torch.cuda.synchronize()
    assert torch.equal(pc.output(0), _single(W, "Q4_K", x.view(1, -1), pc.gemv_shape(0)[0]))
    pc.close()


def _decoder(pc, K=1024, inter=3072, seed=40, types=("Q4_K", "Q6_K", "Q8_0")):
    """A two-layer decoder-shaped chain with every chained input kind: q/k/v on a fixed x,
    o on q's output, a gate/up pair on o's, down on silu(gate)*up, and the next layer's
    q on down's output.  Returns the GEMV descriptions for the oracle."""
    qa, qb, qc = types
    rng_seed = [seed]

    def w(qt, n, k):
        rng_seed[0] += 1
        return dev(make_weights(qt, n, k, seed=rng_seed[0]))

    desc = []
    x = dev(make_activation(K, seed=seed))
    g0 = pc.add_group(x)
    Wq, Wk, Wv = w(qa, K, K), w(qa, 256, K), w(qb, 256, K)
    iq = pc.add_gemv(Wq, qa, nrows=K)
    desc += [(iq, "plain", qa, Wq, None, K, K, ("fixed", x))]
    desc += [(pc.add_gemv(Wk, qa, nrows=256), "plain", qa, Wk, None, 256, K, ("fixed", x))]
    desc += [(pc.add_gemv(Wv, qb, nrows=256), "plain", qb, Wv, None, 256, K, ("fixed", x))]
    g1 = pc.add_group_chained(iq)
    Wo = w(qa, K, K)
    io = pc.add_gemv(Wo, qa, nrows=K)
    desc += [(io, "plain", qa, Wo, None, K, K, ("chained", iq))]
    g2 = pc.add_group_chained(io)
    Wg, Wu = w(qa, inter, K), w(qa, inter, K)
    iglu = pc.add_glu(Wg, Wu, qa, nrows=inter)
    desc += [(iglu, "glu", qa, Wg, Wu, inter, K, ("chained", io))]
    g3 = pc.add_group_chained(iglu)
    Wd = w(qb, K, inter)
    idn = pc.add_gemv(Wd, qb, nrows=K)
    desc += [(idn, "plain", qb, Wd, None, K, inter, ("chained", iglu))]
    g4 = pc.add_group_chained(idn)
    Wq2 = w(qc, K, K)
    desc += [(pc.add_gemv(Wq2, qc, nrows=K), "plain", qc, Wq2, None, K, K, ("chained", idn))]
    return desc, (g0, g1, g2, g3, g4)


def _oracle_check(pc, desc):
    outs = {d[0]: pc.output(d[0]).cpu().numpy() for d in desc}
    for idx, kind, qt, W, W2, n, K, (how, src) in desc:
        assert not np.isnan(outs[idx]).any(), f"GEMV {idx}: values missing"
        if how == "fixed":
            xq, scale = oracle.quantize_q8_1(src.cpu().numpy()), None
        else:
            xq, scale = oracle.quantize_q8_1_chained(outs[src])
        if kind == "glu":
            W2n = W2.cpu().numpy()
            ref = (oracle.mmvq_glu(qt, W.cpu().numpy(), W2n, xq, n, K) if scale is None else
                   oracle.mmvq_glu_chained(qt, W.cpu().numpy(), W2n, xq, scale, n, K))
        else:
            ref = (oracle.mmvq(qt, W.cpu().numpy(), xq, n, K) if scale is None else
                   oracle.mmvq_chained(qt, W.cpu().numpy(), xq, scale, n, K))
        err = oracle.max_rel_err(outs[idx], ref)
        assert err <= Y_TOL, f"GEMV {idx} ({kind} {qt} {n}x{K}): error {err}"
    return outs


@pytest.mark.parametrize("types,K,inter", [(("Q4_K", "Q6_K", "Q8_0"), 1024, 3072),
                                           (("Q5_K", "Q8_0", "Q4_K"), 1024, 3072),
                                           (("Q4_K", "Q6_K", "Q8_0"), 8192, 1024)])
def test_pchain_chained_groups_match_oracle(types, K, inter):
    """Every chained input kind and the gate/up tiles of 1, 2 and 4 rows per matrix (K = 8192
    with 1024 gate/up rows takes one row of each per tile)."""
    pc = PersistentChain()
    desc, groups = _decoder(pc, K=K, inter=inter, types=types)
    # the chained groups' staged Q8_1, written out by the kernel, against the oracle's rule
    dumps = {g: torch.zeros(K // 32 * 36 if g != groups[3] else inter // 32 * 36, dtype=torch.uint8,
                            device="cuda") for g in groups[1:]}
    for g, buf in dumps.items():
        pc.set_group_dump(g, buf)
    pc.instantiate()
    for _ in range(3):
        pc.launch()
    torch.cuda.synchronize()
    assert take_status() == 0
    outs = _oracle_check(pc, desc)
    src_of = {groups[1]: desc[0][0], groups[2]: desc[3][0], groups[3]: desc[4][0], groups[4]: desc[5][0]}
    for g, buf in dumps.items():
        want = oracle.quantize_q8_1_chained(outs[src_of[g]])[0].reshape(-1)
        assert np.array_equal(buf.cpu().numpy(), want), f"group {g}: staged Q8_1 differs from the oracle"
    pc.close()


def test_pchain_chain_trace_and_epochs():
    pc = PersistentChain()
    desc, groups = _decoder(pc)
    pc.instantiate()
    trace = pc.enable_trace()
    for _ in range(4):
        pc.launch()
    torch.cuda.synchronize()
    assert take_status() == 0 and pc.epoch == 4
    _oracle_check(pc, desc)
    summ = trace_summary(trace)
    assert len(summ) == len(groups)
    for g, s in enumerate(summ):
        assert s["stage_start"][0] <= s["stage_end"][1] <= s["staged"][1] <= s["tiles_done"][1]
        if g:  # a group's staging barrier comes after the previous group's staging barrier
            assert s["staged"][0] >= summ[g - 1]["staged"][0]
    pc.close()


@pytest.mark.parametrize("name,n", [("qwen3_8b", 14), ("llama3_70b", 8)])
def test_device_chain_dataflow_matches_oracle(name, n):
    spec = get_chain(name).head(n)  # Qwen3-8B: two decoder layers, both Q6_K mixes
    dc = DeviceChain(spec, executor="persistent")
    assert dc.dataflow and dc.external_inputs == ["attn_in.0"]
    for _ in range(2):
        dc.launch()
    torch.cuda.synchronize()
    assert take_status() == 0 and ops.take_device_status() == 0
    check_chain(dc)
    dc.close()


def test_device_chain_fixed_inputs_equal_graph():
    spec = get_chain("qwen3_8b").head(14)
    a = DeviceChain(spec, executor="graph")
    b = DeviceChain(spec, executor="persistent", dataflow=False)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        a.instantiate()
        a.launch()
        b.launch()
    torch.cuda.synchronize()
    assert take_status() == 0 and ops.take_device_status() == 0
    for i, gm in enumerate(spec.gemvs):
        if b._items[b.pidx[i]] != [i]:
            continue  # gate/up pairs: silu(gate) * up, checked by check_chain
        torch.testing.assert_close(b.output(i), a.outputs[i], rtol=1e-5,
                                   atol=1e-5 * float(a.outputs[i].abs().max()))
    check_chain(b)
    a.close()
    b.close()


def test_pchain_input_wait_times_out_and_recovers():
    """A chained group whose producer rows never arrive: a two-rank chain built on one GPU
    whose "peer" output buffers are local zeroed buffers that no other rank writes.  Rank 0
    writes its rows; the chained group waits for rank 1's rows, gives up after the 10 ms
    bound, and the host reads the flag as ANVIL_ERR_TIMEOUT.  A rebuilt one-rank chain then
    matches the oracle."""
    K, n = 1024, 1024
    x = dev(make_activation(K, seed=5))
    Wq = dev(make_weights("Q4_K", n, K, seed=6))
    Wo = dev(make_weights("Q4_K", n, K, seed=7))
    bufs = [torch.zeros(output_words_bytes(n) // 8, dtype=torch.int64, device="cuda") for _ in range(4)]
    set_wait_limit_ns(10_000_000)
    try:
        pc = PersistentChain(world=2, rank=0)
        pc.add_group(x)
        iq = pc.add_gemv(Wq[: n // 2], "Q4_K", nrows=n // 2, row0=0, nrows_full=n,
                         y_ptrs=[bufs[0].data_ptr(), bufs[1].data_ptr()])
        pc.add_group_chained(iq)
        pc.add_gemv(Wo[: n // 2], "Q4_K", nrows=n // 2, row0=0, nrows_full=n,
                    y_ptrs=[bufs[2].data_ptr(), bufs[3].data_ptr()])
        pc.instantiate()
        pc.launch()
        torch.cuda.synchronize()  # the launch ends: every wait is bounded
        status = take_status()
        assert status & 2, f"status {status}: the input wait did not report"
        with pytest.raises(AnvilError) as e:
            raise_on_status(status)
        assert e.value.status == ANVIL_ERR_TIMEOUT
        pc.close()
    finally:
        set_wait_limit_ns(0)
    assert take_status() == 0
    # the context is still usable: a one-rank chain of the same GEMVs matches the oracle
    pc = PersistentChain()
    pc.add_group(x)
    iq = pc.add_gemv(Wq, "Q4_K", nrows=n)
    pc.add_group_chained(iq)
    io = pc.add_gemv(Wo, "Q4_K", nrows=n)
    pc.instantiate()
    pc.launch()
    torch.cuda.synchronize()
    assert take_status() == 0
    yq = pc.output(iq).cpu().numpy()
    ref_q = oracle.mmvq("Q4_K", Wq.cpu().numpy(), oracle.quantize_q8_1(x.cpu().numpy()), n, K)
    assert oracle.max_rel_err(yq, ref_q) <= Y_TOL
    xo, so = oracle.quantize_q8_1_chained(yq)
    ref_o = oracle.mmvq_chained("Q4_K", Wo.cpu().numpy(), xo, so, n, K)
    assert oracle.max_rel_err(pc.output(io).cpu().numpy(), ref_o) <= Y_TOL
    pc.close()


def test_pchain_argument_errors():
    pc = PersistentChain()
    W = torch.zeros(144 * 16, dtype=torch.uint8, device="cuda")
    with pytest.raises(AnvilError, match="add a group first"):
        pc.add_gemv(W, "Q4_K", nrows=1)
    with pytest.raises(AnvilError, match="ncols"):
        pc.add_group(torch.zeros((3, 256), device="cuda"))
    with pytest.raises(AnvilError, match="multiple of 32"):
        pc.add_group(torch.zeros(100, device="cuda"))
    with pytest.raises(AnvilError, match="earlier GEMV"):
        pc.add_group_chained(0)
    pc.add_group(torch.zeros(512, device="cuda"))
    with pytest.raises(AnvilError, match="outside"):
        pc.add_gemv(W, "Q4_K", nrows=4, row0=2, nrows_full=5)
    with pytest.raises(AnvilError, match="multiple of 16 bytes"):
        pc.add_glu(torch.zeros(210 * 4, dtype=torch.uint8, device="cuda"),
                   torch.zeros(210 * 4, dtype=torch.uint8, device="cuda"), "Q6_K", nrows=2)
    with pytest.raises(AnvilError, match="empty|no GEMV"):
        pc.instantiate()
    pc.close()
    pc = PersistentChain(world=2, rank=1)
    pc.add_group(torch.zeros(512, device="cuda"))
    with pytest.raises(AnvilError, match="every rank's output"):
        pc.add_gemv(W, "Q4_K", nrows=1)
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
    pc = PersistentChain()
    pc.add_group(x)
    pc.add_gemv(W, qt, nrows=nrows)
    pc.instantiate()
    pc.launch()
    torch.cuda.synchronize()
    rpb, lb = pc.gemv_shape(0)
    assert lb == host_lanes_per_row(K // resolve_type(qt).qk, rpb)
    # the quantiser kernel divides every value; the persistent kernel must agree bit for bit
    assert torch.equal(pc.output(0), _single(W, qt, x.view(1, -1), rpb))
    xq = ops.quantize_q8_1(x.view(1, -1)).cpu().numpy().reshape(-1)
    assert np.array_equal(xq, oracle.quantize_q8_1(x.cpu().numpy()).reshape(-1))
    pc.close()


@pytest.mark.parametrize("qt,K", [("Q4_K", 2048), ("Q4_K", 4096), ("Q8_0", 1024), ("Q6_K", 8192)])
def test_pchain_rank_stores_reach_every_rank(qt, K):
    """A two-rank chain built on one GPU, its second rank's buffers local stand-ins: rank 0's
    rows must be written, with the same values and epoch, into both ranks' buffers whatever
    the lanes per row of the tile shape (32, 16 or 8), and no other row may be touched."""
    n = 1024
    x = dev(make_activation(K, seed=31))
    W = dev(make_weights(qt, n, K, seed=32))
    shapes = (1, 2, 4, 8)
    bufs = {r: [torch.zeros(output_words_bytes(n) // 8, dtype=torch.int64, device="cuda") for _ in range(2)]
            for r in shapes}
    pc = PersistentChain(world=2, rank=0)
    pc.add_group(x)
    for rpb in shapes:
        pc.add_gemv(W[: n // 2], qt, nrows=n // 2, row0=0, nrows_full=n,
                    y_ptrs=[b.data_ptr() for b in bufs[rpb]], rows_per_block=rpb)
    pc.instantiate()
    lbs = {pc.gemv_shape(i)[1] for i in range(len(shapes))}
    pc.launch()  # epoch 1: parity 1, words [n, 2n) of each buffer
    torch.cuda.synchronize()
    assert take_status() == 0
    for i, rpb in enumerate(shapes):
        words = [b.view(2, n).cpu().numpy() for b in bufs[rpb]]
        for w in words:
            assert (w[1, : n // 2] >> 32 == 1).all(), f"rows per tile {rpb}: a row of this rank is missing"
            assert (w[1, n // 2:] == 0).all() and (w[0] == 0).all(), "a row outside this rank was written"
        assert np.array_equal(words[0], words[1])
        ref = _single(W[: n // 2], qt, x.view(1, -1), pc.gemv_shape(i)[0]).cpu().numpy().reshape(-1)
        vals = (words[0][1, : n // 2] & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
        assert oracle.max_rel_err(vals, ref) <= Y_TOL
    assert len(lbs) >= 1
    pc.close()


@pytest.mark.parametrize("n,K,rpb", [(1024, 8192, 0), (8192, 8192, 0), (28672, 8192, 0), (28672, 8192, 1),
                                     (28672, 8192, 2), (12288, 4096, 0)])
def test_pchain_gate_up_matches_oracle(n, K, rpb):
    """A gate/up pair on a fixed input against the oracle's silu(g) * u, over row counts and
    rows per tile (0 = the built-in choice)."""
    x = dev(make_activation(K, seed=51))
    Wg = dev(make_weights("Q4_K", n, K, seed=52))
    Wu = dev(make_weights("Q4_K", n, K, seed=53))
    pc = PersistentChain()
    pc.add_group(x)
    i = pc.add_glu(Wg, Wu, "Q4_K", nrows=n, rows_per_block=rpb)
    pc.instantiate()
    pc.launch()
    torch.cuda.synchronize()
    assert take_status() == 0
    got = pc.output(i).cpu().numpy()
    ref = oracle.mmvq_glu("Q4_K", Wg.cpu().numpy(), Wu.cpu().numpy(), oracle.quantize_q8_1(x.cpu().numpy()), n, K)
    err = oracle.max_rel_err(got, ref)
    assert err <= Y_TOL, f"shape {pc.gemv_shape(i)}: error {err}"
    pc.close()


@pytest.mark.parametrize("n", [1024, 4096, 8192, 16384, 28672])
def test_pchain_chained_gate_up_matches_oracle(n):
    """A gate/up pair whose input is the chained output of an 8192 x 8192 GEMV."""
    K = 8192
    x = dev(make_activation(K, seed=61))
    Wo = dev(make_weights("Q4_K", K, K, seed=62))
    Wg = dev(make_weights("Q4_K", n, K, seed=63))
    Wu = dev(make_weights("Q4_K", n, K, seed=64))
    pc = PersistentChain()
    pc.add_group(x)
    io = pc.add_gemv(Wo, "Q4_K", nrows=K)
    pc.add_group_chained(io)
    ig = pc.add_glu(Wg, Wu, "Q4_K", nrows=n)
    pc.instantiate()
    pc.launch()
    torch.cuda.synchronize()
    assert take_status() == 0
    yo = pc.output(io).cpu().numpy()
    got = pc.output(ig).cpu().numpy()
    xq, sc = oracle.quantize_q8_1_chained(yo)
    ref = oracle.mmvq_glu_chained("Q4_K", Wg.cpu().numpy(), Wu.cpu().numpy(), xq, sc, n, K)
    err = oracle.max_rel_err(got, ref)
    assert err <= Y_TOL, f"n={n} shape {pc.gemv_shape(ig)}: error {err}, got max {np.abs(got).max()}, ref max {np.abs(ref).max()}"
    pc.close()


@pytest.mark.parametrize("share", [0, 40, 100])
def test_pchain_static_share_does_not_change_outputs(share):
    """Tiles dealt round-robin or claimed at run time: bit-identical outputs, token after token
    (the counters of both epoch parities are reused), and the oracle agrees."""
    pc_ref, pc = PersistentChain(), PersistentChain()
    desc_ref, _ = _decoder(pc_ref, K=2048, inter=4096, seed=70)
    desc, _ = _decoder(pc, K=2048, inter=4096, seed=70)
    pc.set_static_share(share)
    pc_ref.instantiate()
    pc.instantiate()
    for _ in range(3):
        pc_ref.launch()
        pc.launch()
    torch.cuda.synchronize()
    assert take_status() == 0
    for d in desc:
        a, b = pc_ref.output(d[0]), pc.output(d[0])
        assert torch.equal(a, b), f"GEMV {d[0]} differs with a {share}% static share"
    _oracle_check(pc, desc)
    pc_ref.close()
    pc.close()


def test_pchain_static_share_argument_errors():
    pc = PersistentChain()
    pc.add_group(dev(make_activation(256, seed=1)))
    pc.add_gemv(dev(make_weights("Q4_K", 64, 256, seed=2)), "Q4_K", nrows=64)
    with pytest.raises(AnvilError):
        pc.set_static_share(101)
    with pytest.raises(AnvilError):
        pc.set_static_share(-1)
    pc.instantiate()
    with pytest.raises(AnvilError):
        pc.set_static_share(50)
    pc.close()
