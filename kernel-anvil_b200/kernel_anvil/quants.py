"""GGUF quant-type metadata and seeded synthetic weight/activation generators.

``QUANT_TYPES`` mirrors the reference's per-type table (kernel_anvil/hip_codegen.py:46-102:
ggml type id, values per block ``qk``, ``block_size`` bytes) for the types this build has
sm_100a kernels for; ``qi``/``vdr`` are kept for callers that print them.

The generators write blocks directly in GGUF layout with the value distributions the
workloads are specified with:

* Q4_K (144 B): fp16 d and dmin from |N(0,1)|*1e-3, 12 bytes of packed 6-bit
  scales/mins uniform, 128 bytes of 4-bit quants uniform.
* Q5_K (176 B): as Q4_K plus 32 uniform high-bit bytes.  The specification's "all
  uniform random" cannot mean uniform fp16 bit patterns for d/dmin (those include NaN
  and Inf), so d/dmin follow the Q4_K rule.
* Q6_K (210 B): 128 B low nibbles and 64 B high 2-bit fields uniform, 16 int8 scales
  uniform in [-32, 31], fp16 d from |N(0,1)|*1e-3.
* Q8_0 (34 B): fp16 d from |N(0,1)|*1e-2, 32 int8 quants uniform in [-127, 127].
* activations: fp32 N(0,1).

``make_weights`` (numpy, seeded ``default_rng``) is bit-reproducible and used for parity
tests; ``make_weights_device`` draws on the GPU with a seeded torch generator for the
multi-GB chain workloads.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

QK_K = 256
Q8_1_BLOCK_SIZE = 36  # GPU block_q8_1: half2 {d, s} + int8[32] (hip_codegen.py:101-102)


@dataclass(frozen=True)
class QuantTypeInfo:
    name: str
    ggml_type: int
    qk: int
    qi: int
    vdr: int
    block_size: int

    @property
    def bytes_per_weight(self) -> float:
        return self.block_size / self.qk

    def row_bytes(self, K: int) -> int:
        if K % self.qk:
            raise ValueError(f"K must be divisible by {self.qk} ({self.name} block size), got K={K}")
        return K // self.qk * self.block_size


QUANT_TYPES: dict[str, QuantTypeInfo] = {
    "Q4_0": QuantTypeInfo("Q4_0", 2, 32, 4, 2, 18),
    "Q4_1": QuantTypeInfo("Q4_1", 3, 32, 4, 2, 20),
    "Q5_0": QuantTypeInfo("Q5_0", 6, 32, 4, 2, 22),
    "Q5_1": QuantTypeInfo("Q5_1", 7, 32, 4, 2, 24),
    "Q8_0": QuantTypeInfo("Q8_0", 8, 32, 8, 2, 34),
    "Q2_K": QuantTypeInfo("Q2_K", 10, 256, 16, 1, 84),
    "Q3_K": QuantTypeInfo("Q3_K", 11, 256, 16, 1, 110),
    "Q4_K": QuantTypeInfo("Q4_K", 12, 256, 32, 2, 144),
    "Q5_K": QuantTypeInfo("Q5_K", 13, 256, 32, 2, 176),
    "Q6_K": QuantTypeInfo("Q6_K", 14, 256, 32, 1, 210),
    "IQ2_XXS": QuantTypeInfo("IQ2_XXS", 16, 256, 16, 2, 66),
    "IQ2_XS": QuantTypeInfo("IQ2_XS", 17, 256, 16, 2, 74),
    "IQ2_S": QuantTypeInfo("IQ2_S", 22, 256, 16, 2, 82),
    "IQ3_XXS": QuantTypeInfo("IQ3_XXS", 18, 256, 16, 2, 98),
    "IQ3_S": QuantTypeInfo("IQ3_S", 21, 256, 16, 2, 110),
    "IQ1_S": QuantTypeInfo("IQ1_S", 19, 256, 8, 1, 50),
    # ggml's id of IQ1_M is 29 (gguf-py GGMLQuantizationType.IQ1_M); the reference's table
    # says 24, which ggml assigns to I8
    "IQ1_M": QuantTypeInfo("IQ1_M", 29, 256, 8, 1, 56),
    "IQ4_NL": QuantTypeInfo("IQ4_NL", 20, 32, 4, 2, 18),
    "IQ4_XS": QuantTypeInfo("IQ4_XS", 23, 256, 32, 4, 136),
}
# The I-quants whose fp16 d sits in bytes 0-1 (IQ1_M spreads it over its scale words).
_IQ_D_AT_0 = ("IQ2_XXS", "IQ2_XS", "IQ2_S", "IQ3_XXS", "IQ3_S", "IQ1_S")


def _iq1m_set_d(blocks: np.ndarray, d_bits: np.ndarray) -> None:
    """IQ1_M: fp16 d bits -> the top nibbles of the four scale words at bytes 48..55
    (bits 12-15 of word i hold bits 4i..4i+3 of d); the 3-bit scales below are kept."""
    sc = blocks[:, 48:56].copy().view(np.uint16).reshape(-1, 4)
    for i in range(4):
        sc[:, i] = (sc[:, i] & np.uint16(0x0FFF)) | (((d_bits >> np.uint16(4 * i)) & np.uint16(15)) << np.uint16(12))
    blocks[:, 48:56] = sc.view(np.uint8).reshape(-1, 8)
TYPE_BY_ID = {q.ggml_type: q for q in QUANT_TYPES.values()}


def get_quant_info(quant_type: str) -> QuantTypeInfo | None:
    """Look up a type by name; GGUF file-level suffixes (``Q4_K_M``) map to the block type.

    Same resolution order as the reference (kernel_anvil/hip_codegen.py:105-127): exact
    name first, then the name with a trailing ``_M``/``_S`` removed.
    """
    if quant_type in QUANT_TYPES:
        return QUANT_TYPES[quant_type]
    if quant_type.endswith(("_M", "_S")):
        return QUANT_TYPES.get(quant_type.rsplit("_", 1)[0])
    return None


def resolve_type(qt) -> QuantTypeInfo:
    """Accept a name, a ggml type id or a QuantTypeInfo."""
    if isinstance(qt, QuantTypeInfo):
        return qt
    if isinstance(qt, (int, np.integer)):
        info = TYPE_BY_ID.get(int(qt))
    else:
        info = get_quant_info(str(qt))
    if info is None:
        raise ValueError(f"unsupported quant type {qt!r}; have {sorted(QUANT_TYPES)}")
    return info


def gemv_bytes(qt, nrows: int, K: int, ncols: int = 1) -> int:
    """Algorithmic bytes of one GEMV: weights + Q8_1 activations read + fp32 outputs written."""
    info = resolve_type(qt)
    return nrows * info.row_bytes(K) + ncols * (K // 32) * Q8_1_BLOCK_SIZE + ncols * nrows * 4


def _fp16_abs_normal(rng: np.random.Generator, n: int, scale: float) -> np.ndarray:
    return (np.abs(rng.standard_normal(n)) * scale).astype(np.float16).view(np.uint8).reshape(n, 2)


def make_weights(qt, nrows: int, K: int, seed: int = 0) -> np.ndarray:
    """Seeded synthetic weight matrix in GGUF block layout, shape (nrows, row_bytes) uint8."""
    info = resolve_type(qt)
    row_bytes = info.row_bytes(K)  # validates K
    rng = np.random.default_rng(seed)
    nb = nrows * (K // info.qk)
    blocks = np.empty((nb, info.block_size), dtype=np.uint8)
    if info.name in ("Q4_K", "Q5_K"):
        blocks[:, 0:2] = _fp16_abs_normal(rng, nb, 1e-3)
        blocks[:, 2:4] = _fp16_abs_normal(rng, nb, 1e-3)
        blocks[:, 4:] = rng.integers(0, 256, size=(nb, info.block_size - 4), dtype=np.uint8)
    elif info.name == "Q6_K":
        blocks[:, 0:192] = rng.integers(0, 256, size=(nb, 192), dtype=np.uint8)
        blocks[:, 192:208] = rng.integers(-32, 32, size=(nb, 16), dtype=np.int8).view(np.uint8)
        blocks[:, 208:210] = _fp16_abs_normal(rng, nb, 1e-3)
    elif info.name == "Q8_0":
        blocks[:, 0:2] = _fp16_abs_normal(rng, nb, 1e-2)
        blocks[:, 2:34] = rng.integers(-127, 128, size=(nb, 32), dtype=np.int8).view(np.uint8)
    elif info.name == "Q2_K":
        # scales/mins nibbles, quants uniform; d, dmin from |N(0,1)| * 1e-2
        blocks[:, 0:80] = rng.integers(0, 256, size=(nb, 80), dtype=np.uint8)
        blocks[:, 80:82] = _fp16_abs_normal(rng, nb, 1e-2)
        blocks[:, 82:84] = _fp16_abs_normal(rng, nb, 1e-2)
    elif info.name == "Q3_K":
        blocks[:, 0:108] = rng.integers(0, 256, size=(nb, 108), dtype=np.uint8)
        blocks[:, 108:110] = _fp16_abs_normal(rng, nb, 1e-2)
    elif info.name in ("IQ4_NL", "IQ4_XS"):
        # d from |N(0,1)| * 1e-3 (levels reach +-127); scales and level indices uniform
        blocks[:, 2:] = rng.integers(0, 256, size=(nb, info.block_size - 2), dtype=np.uint8)
        blocks[:, 0:2] = _fp16_abs_normal(rng, nb, 1e-3)
    elif info.name in ("Q4_0", "Q4_1", "Q5_0", "Q5_1"):
        # d from |N(0,1)| * 1e-2; the _1 types' m (the block minimum) from -|N(0,1)| * 1e-1;
        # high bits (qh) and nibbles uniform
        blocks[:, 2:] = rng.integers(0, 256, size=(nb, info.block_size - 2), dtype=np.uint8)
        blocks[:, 0:2] = _fp16_abs_normal(rng, nb, 1e-2)
        if info.name.endswith("_1"):
            m = (-np.abs(rng.standard_normal(nb)) * 1e-1).astype(np.float16)
            blocks[:, 2:4] = m.view(np.uint8).reshape(nb, 2)
    elif info.name in _IQ_D_AT_0 or info.name == "IQ1_M":
        # lattice indices, sign bits, scales and delta bits uniform; d from |N(0,1)| * 1e-3
        blocks[:] = rng.integers(0, 256, size=(nb, info.block_size), dtype=np.uint8)
        d = _fp16_abs_normal(rng, nb, 1e-3)
        if info.name == "IQ1_M":
            _iq1m_set_d(blocks, d.copy().view(np.uint16).reshape(nb))
        else:
            blocks[:, 0:2] = d
    else:  # pragma: no cover - resolve_type rejects other types
        raise ValueError(info.name)
    return blocks.reshape(nrows, row_bytes)


def make_activation(K: int, ncols: int = 1, seed: int = 1) -> np.ndarray:
    """fp32 N(0,1) activations, shape (ncols, K)."""
    rng = np.random.default_rng(seed)
    return rng.standard_normal((ncols, K)).astype(np.float32)


def make_weights_device(qt, nrows: int, K: int, seed: int = 0, device="cuda"):
    """Synthetic weights drawn on the GPU, shape (nrows, row_bytes) uint8.

    The distributions are make_weights' with one change: the types with a block minimum
    (Q4_K, Q5_K, Q2_K, Q4_1, Q5_1) draw it so that a weight's expected value is zero, as it
    is for real quantised weights.  With make_weights' minima the weights have a positive
    mean (Q4_K: E[d*sc*q - dmin*m] = 31.5 * 1e-3 * E|N| * (7.5 - 1)), every output of a GEMV
    carries the same offset, and along a chain of GEMVs that offset grows until all rows
    of a gate projection share one sign.  The chains and the bench use these weights."""
    import torch

    info = resolve_type(qt)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    row_bytes = info.row_bytes(K)  # validates K
    nb = nrows * (K // info.qk)
    blocks = torch.randint(0, 256, (nb, info.block_size), dtype=torch.uint8, device=device, generator=g)

    def fp16_abs_normal(scale):
        v = torch.randn(nb, device=device, generator=g).abs_().mul_(scale).to(torch.float16)
        return v.view(torch.uint8).view(nb, 2)

    # mean quant of the types with a minimum: q uniform over 0..15 (Q4_K, Q4_1), 0..31 (Q5_K,
    # Q5_1), 0..3 (Q2_K); scale and min indices are uniform over the same range, so
    # E[dmin] = mean quant * E[d] centres the weights
    if info.name in ("Q4_K", "Q5_K"):
        blocks[:, 0:2] = fp16_abs_normal(1e-3)
        blocks[:, 2:4] = fp16_abs_normal(1e-3 * (7.5 if info.name == "Q4_K" else 15.5))
    elif info.name == "Q6_K":
        sc = torch.randint(-32, 32, (nb, 16), dtype=torch.int8, device=device, generator=g)
        blocks[:, 192:208] = sc.view(torch.uint8)
        blocks[:, 208:210] = fp16_abs_normal(1e-3)
    elif info.name == "Q8_0":
        blocks[:, 0:2] = fp16_abs_normal(1e-2)
        q = torch.randint(-127, 128, (nb, 32), dtype=torch.int8, device=device, generator=g)
        blocks[:, 2:34] = q.view(torch.uint8)
    elif info.name == "Q2_K":
        blocks[:, 80:82] = fp16_abs_normal(1e-2)
        blocks[:, 82:84] = fp16_abs_normal(1.5e-2)
    elif info.name == "Q3_K":
        blocks[:, 108:110] = fp16_abs_normal(1e-2)
    elif info.name in ("IQ4_NL", "IQ4_XS"):
        blocks[:, 0:2] = fp16_abs_normal(1e-3)
    elif info.name in _IQ_D_AT_0:
        blocks[:, 0:2] = fp16_abs_normal(1e-3)
    elif info.name == "IQ1_M":
        d = torch.randn(nb, device=device, generator=g).abs_().mul_(1e-3).to(torch.float16)
        dbits = d.view(torch.int16).to(torch.int32) & 0xFFFF
        sc = blocks[:, 48:56].contiguous().view(torch.int16).to(torch.int32) & 0xFFFF
        for i in range(4):
            sc[:, i] = (sc[:, i] & 0x0FFF) | (((dbits >> (4 * i)) & 15) << 12)
        blocks[:, 48:56] = sc.to(torch.int16).view(torch.uint8).view(nb, 8)
    elif info.name in ("Q4_0", "Q4_1", "Q5_0", "Q5_1"):
        blocks[:, 0:2] = fp16_abs_normal(1e-2)
        if info.name.endswith("_1"):
            mq = 7.5e-2 if info.name == "Q4_1" else 15.5e-2
            m = (torch.randn(nb, device=device, generator=g).abs_().mul_(-mq)).to(torch.float16)
            blocks[:, 2:4] = m.view(torch.uint8).view(nb, 2)
    return blocks.view(nrows, row_bytes)
