"""Per-token GEMV chains of decode-shaped models, and their device-side builder.

A chain is the sequence of quantized GEMVs one decode token runs (the MMVQ launches of
llama.cpp's decode, docs/decode-pipeline-breakdown.md:20-21), each preceded by the Q8_1
quantisation of its input when that input is new.  Attention, norms and activations are
not part of the path: every distinct GEMV input is a fixed synthetic fp32 vector that
is quantised inside the chain, so the chain carries exactly the quantize + MMVQ work.

Shapes are (nrows N, ncols_x K) = (output features, input features).

The decoder chains also record their data flow (``ChainSpec.sources``): which GEMV output
each activation is computed from, with the ops between GEMVs that are not part of this path
reduced to what keeps the dependency: the attention output stands in as attn_q's output
(a vector of the same length), the ffn input as attn_output's, ffn_down's input as
silu(ffn_gate) * ffn_up, the next layer's attention input as ffn_down's output, and the
lm_head input as the last ffn_down's.  The persistent executor runs that flow (each group
reads its producer's output, scaled by a power of two); the graph executor keeps every
input a fixed synthetic vector.

  qwen3_8b      36 layers: q 4096x4096, k/v 1024x4096, o 4096x4096, gate/up 12288x4096,
                down 4096x12288; Q4_K except Q6_K on attn_v and ffn_down in even layers;
                lm_head 151936x4096 Q4_K.  253 GEMVs, 145 quantisations per token.
  qwen3_0_6b    28 layers, all Q8_0: q 2048x1024, k/v 1024x1024, o 1024x2048,
                gate/up 3072x1024, down 1024x3072 (speculative-decoding draft).
  llama3_70b    80 layers, all Q4_K: q/o 8192x8192, k/v 1024x8192, gate/up 28672x8192,
                down 8192x28672.
  qwen35_27b    tuned-shape set: Q4_K 5120x6144 x48, Q5_K 5120x10240 x48,
                Q4_K 6144x5120 x64, Q4_K 5120x1024 x22 (shapes as given, N x K).
"""
from __future__ import annotations

from collections import Counter
from dataclasses import dataclass, field

from kernel_anvil.quants import gemv_bytes, resolve_type


@dataclass(frozen=True)
class Gemv:
    name: str
    qt: str
    nrows: int
    K: int
    input: str  # id of the activation vector it consumes


@dataclass
class ChainSpec:
    name: str
    gemvs: list[Gemv]
    inputs: dict[str, int] = field(default_factory=dict)  # activation id -> K (in first-use order)
    # activation id -> ("copy", gemv name) or ("glu", gate name, up name): the GEMV output(s)
    # it is computed from; activations absent here are fixed inputs
    sources: dict[str, tuple] = field(default_factory=dict)

    def unique_shapes(self) -> dict[tuple[str, int, int], int]:
        """{(quant, N, K): count} over the chain's GEMVs."""
        return dict(Counter((g.qt, g.nrows, g.K) for g in self.gemvs))

    def algorithmic_bytes(self, ncols: int = 1) -> int:
        return sum(gemv_bytes(g.qt, g.nrows, g.K, ncols) for g in self.gemvs)

    def glu_algorithmic_bytes(self, ncols: int = 1) -> int:
        """Algorithmic bytes when every gate/up pair is one gate/up GEMV: both weight streams,
        one activation read and one output vector per pair."""
        total, i = 0, 0
        while i < len(self.gemvs):
            g = self.gemvs[i]
            if is_gate_up(self.gemvs[i:i + 2]):
                total += (2 * gemv_bytes(g.qt, g.nrows, g.K, ncols) - 4 * g.nrows * ncols
                          - gemv_bytes(g.qt, 0, g.K, ncols))
                i += 2
            else:
                total += gemv_bytes(g.qt, g.nrows, g.K, ncols)
                i += 1
        return total

    def weight_bytes(self) -> int:
        return sum(g.nrows * resolve_type(g.qt).row_bytes(g.K) for g in self.gemvs)

    def head(self, n: int, name: str | None = None) -> "ChainSpec":
        """The chain's first n GEMVs (with their inputs): a smaller case of the same shapes."""
        gemvs = self.gemvs[:n]
        used = {g.input for g in gemvs}
        names = {g.name for g in gemvs}
        sources = {a: src for a, src in self.sources.items()
                   if a in used and all(nm in names for nm in src[1:])}
        return ChainSpec(name or f"{self.name}[:{n}]", list(gemvs),
                         {a: k for a, k in self.inputs.items() if a in used}, sources)

    def fixed_inputs(self) -> list[str]:
        """Activations not computed from an earlier GEMV (in first-use order)."""
        return [a for a in self.inputs if a not in self.sources]


def _layered(name: str, n_layers: int, per_layer, tail=()) -> ChainSpec:
    spec = ChainSpec(name, [])
    for layer in range(n_layers):
        for gname, qt, n, k, inp in per_layer(layer):
            act = f"{inp}.{layer}"
            spec.inputs.setdefault(act, k)
            spec.gemvs.append(Gemv(f"blk.{layer}.{gname}", qt, n, k, act))
        blk = f"blk.{layer}"
        spec.sources[f"attn_out.{layer}"] = ("copy", f"{blk}.attn_q")
        spec.sources[f"ffn_in.{layer}"] = ("copy", f"{blk}.attn_output")
        spec.sources[f"ffn_act.{layer}"] = ("glu", f"{blk}.ffn_gate", f"{blk}.ffn_up")
        if layer > 0:
            spec.sources[f"attn_in.{layer}"] = ("copy", f"blk.{layer - 1}.ffn_down")
    for gname, qt, n, k, inp in tail:
        spec.inputs.setdefault(inp, k)
        spec.gemvs.append(Gemv(gname, qt, n, k, inp))
        spec.sources[inp] = ("copy", f"blk.{n_layers - 1}.ffn_down")
    _check_sources(spec)
    return spec


def _check_sources(spec: ChainSpec) -> None:
    """Every chained activation has its producer's length and a producer that comes first."""
    rows = {g.name: (i, g.nrows) for i, g in enumerate(spec.gemvs)}
    first_use = {}
    for i, g in enumerate(spec.gemvs):
        first_use.setdefault(g.input, i)
    for act, src in spec.sources.items():
        for nm in src[1:]:
            i, n = rows[nm]
            if n != spec.inputs[act] or i >= first_use[act]:
                raise ValueError(f"{spec.name}: {act} cannot be computed from {nm}")


def qwen3_8b() -> ChainSpec:
    h, kv, inter = 4096, 1024, 12288

    def layer(i):
        mix = "Q6_K" if i % 2 == 0 else "Q4_K"
        return [("attn_q", "Q4_K", h, h, "attn_in"), ("attn_k", "Q4_K", kv, h, "attn_in"),
                ("attn_v", mix, kv, h, "attn_in"), ("attn_output", "Q4_K", h, h, "attn_out"),
                ("ffn_gate", "Q4_K", inter, h, "ffn_in"), ("ffn_up", "Q4_K", inter, h, "ffn_in"),
                ("ffn_down", mix, h, inter, "ffn_act")]

    return _layered("qwen3_8b", 36, layer, tail=[("output", "Q4_K", 151936, h, "final")])


def qwen3_0_6b() -> ChainSpec:
    h, q, kv, inter = 1024, 2048, 1024, 3072

    def layer(i):
        return [("attn_q", "Q8_0", q, h, "attn_in"), ("attn_k", "Q8_0", kv, h, "attn_in"),
                ("attn_v", "Q8_0", kv, h, "attn_in"), ("attn_output", "Q8_0", h, q, "attn_out"),
                ("ffn_gate", "Q8_0", inter, h, "ffn_in"), ("ffn_up", "Q8_0", inter, h, "ffn_in"),
                ("ffn_down", "Q8_0", h, inter, "ffn_act")]

    return _layered("qwen3_0_6b", 28, layer)


def llama3_70b() -> ChainSpec:
    h, kv, inter = 8192, 1024, 28672

    def layer(i):
        return [("attn_q", "Q4_K", h, h, "attn_in"), ("attn_k", "Q4_K", kv, h, "attn_in"),
                ("attn_v", "Q4_K", kv, h, "attn_in"), ("attn_output", "Q4_K", h, h, "attn_out"),
                ("ffn_gate", "Q4_K", inter, h, "ffn_in"), ("ffn_up", "Q4_K", inter, h, "ffn_in"),
                ("ffn_down", "Q4_K", h, inter, "ffn_act")]

    return _layered("llama3_70b", 80, layer)


def qwen35_27b() -> ChainSpec:
    spec = ChainSpec("qwen35_27b", [])
    for qt, n, k, count in (("Q4_K", 5120, 6144, 48), ("Q5_K", 5120, 10240, 48),
                            ("Q4_K", 6144, 5120, 64), ("Q4_K", 5120, 1024, 22)):
        for i in range(count):
            act = f"in{k}.{i}"
            spec.inputs[act] = k
            spec.gemvs.append(Gemv(f"{qt}.{n}x{k}.{i}", qt, n, k, act))
    return spec


CHAINS = {"qwen3_8b": qwen3_8b, "qwen3_0_6b": qwen3_0_6b, "llama3_70b": llama3_70b,
          "qwen35_27b": qwen35_27b}


def get_chain(name: str) -> ChainSpec:
    try:
        return CHAINS[name]()
    except KeyError:
        raise ValueError(f"unknown chain {name!r}; have {sorted(CHAINS)}") from None


def is_gate_up(run: list) -> bool:
    """A run of GEMVs that is one FFN's gate and up projection (same type and shape)."""
    return (len(run) == 2 and run[0].name.endswith("ffn_gate") and run[1].name.endswith("ffn_up")
            and (run[0].qt, run[0].nrows, run[0].K) == (run[1].qt, run[1].nrows, run[1].K)
            and resolve_type(run[0].qt).row_bytes(run[0].K) % 16 == 0)


def spec_index(spec: ChainSpec, name: str) -> int:
    for i, g in enumerate(spec.gemvs):
        if g.name == name:
            return i
    raise KeyError(name)


def shard_rows(nrows: int, rank: int, world: int) -> tuple[int, int]:
    """Row range [start, stop) of `rank` when nrows rows are split over `world` ranks.

    Rows are independent in a GEMV and a GGUF block never spans two rows, so any split
    on row boundaries is exact; ranks get contiguous, near-equal slices."""
    base, extra = divmod(nrows, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


class DeviceChain:
    """Weights, activations and outputs of a ChainSpec on one GPU, plus its executor.

    With world > 1 every matrix holds only this rank's row shard (shard_rows).  Weights
    are drawn on the device (quants.make_weights_device).

    executor="graph": the anvil Chain (a CUDA graph of quantize + MMVQ launches with
    programmatic dependent launch); outputs are this rank's slices, (ncols, rows).  With
    grouped=True, consecutive GEMVs of one quant type on the same input (q/k, gate/up) are
    one launch (anvil_mmvq_grouped; with fused=True the launch quantises the fp32 input
    itself, anvil_mmvq_grouped_f32).  With glu=True (grouped, one column, separate
    quantisation) each ffn_gate/ffn_up pair is one gate/up launch (anvil_mmvq_glu) whose
    silu(gate) * up vector goes to the gate's output; the up output is left unwritten.
    executor="persistent": one persistent kernel per token (pchain.PersistentChain).
    GEMVs sharing an input form a group; each ffn_gate/ffn_up pair is one gate/up GEMV
    (silu(gate) * up).  With dataflow=True (and a spec that records it) every chained
    activation is its producer's output, read inside the kernel as it arrives; only the
    first input is a fixed vector.  Outputs are full (ncols, nrows) vectors read with
    output(i); with world > 1 every rank writes its rows into every rank's buffer, which
    lives in CUDA-IPC memory (needs `dist`).
    """

    def __init__(self, spec: ChainSpec, ncols: int = 1, seed: int = 0, device="cuda",
                 rank: int = 0, world: int = 1, nwarps: int = 0, rows_per_block: int = 0,
                 configs: dict | None = None, fused: bool = False, coresident: int = 1,
                 executor: str = "graph", dist=None, ctas_per_sm: int = 0, grouped: bool = False,
                 glu: bool = False, dataflow: bool = True, static_share: int | None = None):
        import torch

        from kernel_anvil.mmvq import Chain, q8_1_bytes
        from kernel_anvil.quants import make_weights_device

        if executor not in ("graph", "persistent"):
            raise ValueError(f"executor must be 'graph' or 'persistent', not {executor!r}")
        self.spec = spec
        self.ncols = ncols
        self.rank, self.world = rank, world
        self.executor = executor
        self.grouped = grouped and executor == "graph"
        self.glu = glu and self.grouped and ncols == 1 and not fused
        g = torch.Generator(device=device)
        g.manual_seed(seed + 7919)
        # All fp32 inputs live in one buffer so a step's inputs arrive with one copy.
        total = sum(k * ncols for k in spec.inputs.values())
        self.x_all = torch.randn(total, generator=g, device=device, dtype=torch.float32)
        self.x, off = {}, 0
        for a, k in spec.inputs.items():
            self.x[a] = self.x_all[off:off + k * ncols].view(ncols, k)
            off += k * ncols
        self.weights, self.outputs, self.rows, self.launch_cfg = [], [], [], []
        for i, gm in enumerate(spec.gemvs):
            r0, r1 = shard_rows(gm.nrows, rank, world)
            self.weights.append(make_weights_device(gm.qt, r1 - r0, gm.K,
                                                    seed=seed * 100003 + i * 31 + rank, device=device))
            self.rows.append((r0, r1))
            nw, rpb = nwarps, rows_per_block
            if configs and (gm.qt, gm.nrows, gm.K) in configs:
                c = configs[(gm.qt, gm.nrows, gm.K)]
                nw, rpb = c["nwarps"], c["rows_per_block"]
            self.launch_cfg.append((nw, rpb))
        self.chain = None
        self.pchain = None
        self.arena = None
        self.pidx: list[int | None] = []   # persistent: chain GEMV index of each spec GEMV
        self.dataflow = False
        if executor == "graph":
            self.xq = {a: torch.empty(q8_1_bytes(k, ncols), dtype=torch.uint8, device=device)
                       for a, k in spec.inputs.items()}
            self.chain = Chain()
            if coresident != 1:
                self.chain.set_coresident(coresident)
            quantized: set[str] = set()
            if grouped:
                self.outputs = [torch.empty((ncols, r1 - r0), dtype=torch.float32, device=device)
                                for r0, r1 in self.rows]
                i = 0
                while i < len(spec.gemvs):
                    j = i + 1
                    while (j < len(spec.gemvs) and j - i < 4 and spec.gemvs[j].input == spec.gemvs[i].input
                           and spec.gemvs[j].qt == spec.gemvs[i].qt):
                        j += 1
                    gm = spec.gemvs[i]
                    nw, rpb = self.launch_cfg[i]
                    rows = [r1 - r0 for r0, r1 in self.rows[i:j]]
                    if self.glu and is_gate_up(spec.gemvs[i:j]):
                        if gm.input not in quantized:
                            self.chain.add_quantize(self.x[gm.input], self.xq[gm.input])
                            quantized.add(gm.input)
                        self.chain.add_mmvq_glu(self.weights[i], self.weights[i + 1], gm.qt,
                                                self.xq[gm.input], self.outputs[i])
                    elif fused:
                        self.chain.add_mmvq_grouped_f32(
                            self.weights[i:j], gm.qt, self.x[gm.input], self.xq[gm.input],
                            self.outputs[i:j], rows, K=gm.K, ncols=ncols, nwarps=nw,
                            rows_per_block=rpb)
                    else:
                        if gm.input not in quantized:
                            self.chain.add_quantize(self.x[gm.input], self.xq[gm.input])
                            quantized.add(gm.input)
                        self.chain.add_mmvq_grouped(self.weights[i:j], gm.qt, self.xq[gm.input],
                                                    self.outputs[i:j], rows, K=gm.K, ncols=ncols,
                                                    nwarps=nw, rows_per_block=rpb)
                    i = j
            for gm, W, (r0, r1), (nw, rpb) in zip(spec.gemvs, self.weights, self.rows, self.launch_cfg):
                if grouped:
                    break
                n = r1 - r0
                y = torch.empty((ncols, n), dtype=torch.float32, device=device)
                if fused:
                    # each GEMV quantises its fp32 input in its own prologue
                    self.chain.add_mmvq_f32(W, gm.qt, self.x[gm.input], self.xq[gm.input], y, nrows=n,
                                            K=gm.K, ncols=ncols, nwarps=nw, rows_per_block=rpb)
                else:
                    if gm.input not in quantized:
                        self.chain.add_quantize(self.x[gm.input], self.xq[gm.input])
                        quantized.add(gm.input)
                    self.chain.add_mmvq(W, gm.qt, self.xq[gm.input], y, nrows=n, K=gm.K, ncols=ncols,
                                        nwarps=nw, rows_per_block=rpb)
                self.outputs.append(y)
        else:
            self._build_persistent(device, nwarps, ctas_per_sm, dist, dataflow, static_share)

    def _build_persistent(self, device, nwarps: int, ctas_per_sm: int, dist, dataflow: bool,
                          static_share: int | None) -> None:
        from kernel_anvil.pchain import PeerArena, PersistentChain, output_words_bytes

        spec, ncols = self.spec, self.ncols
        sources = spec.sources if dataflow else {}
        self.dataflow = bool(sources)
        # chain GEMVs in order: a gate/up pair is one gate/up GEMV, every other GEMV its own
        items: list[list[int]] = []
        i = 0
        while i < len(spec.gemvs):
            if is_gate_up(spec.gemvs[i:i + 2]):
                items.append([i, i + 1])
                i += 2
            else:
                items.append([i])
                i += 1
        if self.world > 1:
            if dist is None:
                raise ValueError("a sharded persistent chain needs the process group (dist)")
            layout = [(f"y{j}", output_words_bytes(spec.gemvs[it[0]].nrows, ncols))
                      for j, it in enumerate(items)]
            self.arena = PeerArena(layout, dist)
        pc = PersistentChain(self.world, self.rank)
        self.pidx = [None] * len(spec.gemvs)
        prev = None
        for j, it in enumerate(items):
            gm = spec.gemvs[it[0]]
            if gm.input != prev:
                src = sources.get(gm.input)
                if src is None:
                    pc.add_group(self.x[gm.input])
                else:
                    producer = self.pidx[spec_index(spec, src[1])]
                    if producer is None or (src[0] == "glu" and len(items[producer]) != 2):
                        raise ValueError(f"{gm.input}: its producer is not a chain GEMV")
                    pc.add_group_chained(producer)
                prev = gm.input
            (r0, r1), (_, rpb) = self.rows[it[0]], self.launch_cfg[it[0]]
            ys = self.arena.ptrs(f"y{j}") if self.arena else None
            if len(it) == 2:
                idx = pc.add_glu(self.weights[it[0]], self.weights[it[1]], gm.qt, nrows=r1 - r0, row0=r0,
                                 nrows_full=gm.nrows, y_ptrs=ys, rows_per_block=rpb)
            else:
                idx = pc.add_gemv(self.weights[it[0]], gm.qt, nrows=r1 - r0, row0=r0, nrows_full=gm.nrows,
                                  y_ptrs=ys, rows_per_block=rpb)
            assert idx == j
            for k in it:
                self.pidx[k] = j
        if static_share is not None:
            pc.set_static_share(static_share)
        pc.instantiate(nwarps=nwarps, ctas_per_sm=ctas_per_sm)
        self.pchain = pc
        self._items = items
        self.outputs = [None] * len(spec.gemvs)

    def output(self, i: int):
        """Spec GEMV i's output: (ncols, rows) for the graph executor (this rank's rows), the
        full (ncols, nrows) vector for the persistent one (for a gate/up pair, the
        silu(gate) * up vector, under either GEMV's index)."""
        if self.chain:
            return self.outputs[i]
        return self.pchain.output(self.pidx[i])

    @property
    def external_inputs(self) -> list[str]:
        """Activations the step takes from outside the chain (copied in every step)."""
        return self.spec.fixed_inputs() if self.dataflow else list(self.spec.inputs)

    @property
    def algorithmic_bytes(self) -> int:
        return self.chain.algorithmic_bytes if self.chain else self.pchain.algorithmic_bytes

    @property
    def launches_per_step(self) -> int:
        return self.chain.n_launches if self.chain else 1

    def instantiate(self, pdl: bool = True) -> None:
        if self.chain:
            self.chain.instantiate(pdl=pdl)

    def launch(self) -> None:
        if self.chain:
            self.chain.launch()
        else:
            self.pchain.launch()

    def close(self) -> None:
        if self.chain:
            self.chain.close()
        if self.pchain:
            self.pchain.close()
        if self.arena:
            self.arena.close()
            self.arena = None
