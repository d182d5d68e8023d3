"""Model-level drop-in: nn.Linear replaced by QuantLinear, which runs the B200 MMVQ kernels.

B200 counterpart of the reference's SmithyLinear / optimize() (kernel_anvil/model.py:30-86,
260-370).  The reference keeps FP16 weights and runs a tuned Triton GEMV for one token; here
the weights are GGUF quantized blocks on the GPU and every forward pass is the production
MMVQ path (Q8_1 activation quantisation + block dots), the same arithmetic llama.cpp's decode
runs.  Up to 8 tokens go through one launch (the batched speculative-decoding variant);
longer inputs are processed 8 columns at a time.  There is no CPU path: a forward pass on a
CPU tensor raises AnvilError.

  QuantLinear(blocks, quant, in_features, bias=None)      GGUF blocks (out_features, row_bytes)
  QuantLinear.from_linear(linear, quant="Q8_0")           quantises an fp weight (gguf-py Q8_0)
  QuantLinear.from_gguf(path, tensor_name)                 a tensor of a GGUF file, as stored
  load_gguf_linears(path)                                  every supported 2-D tensor of a file
  optimize(model, quant="Q8_0")                            replaces nn.Linear layers in place
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn as nn

from kernel_anvil import mmvq as ops
from kernel_anvil._native import ANVIL_ERR_INVALID, AnvilError
from kernel_anvil.quants import QUANT_TYPES, resolve_type

MAX_COLS = ops.MAX_COLS


class QuantLinear(nn.Module):
    """y = x W^T (+ bias) with W held as GGUF quantized blocks (one row per output feature).

    x: (..., in_features) on the GPU, any float dtype; the result has x's dtype.  The
    computation is MMVQ's: x quantised to Q8_1 per 32 values, integer block dots, fp32
    accumulation.  nwarps / rows_per_block: launch shape (0 = smithy table, then built-in).
    """

    def __init__(self, blocks: torch.Tensor, quant, in_features: int, bias: torch.Tensor | None = None,
                 nwarps: int = 0, rows_per_block: int = 0):
        super().__init__()
        info = resolve_type(quant)
        if blocks.dtype != torch.uint8 or blocks.dim() != 2:
            raise AnvilError(ANVIL_ERR_INVALID, "blocks must be a 2-D uint8 tensor (out_features, row_bytes)")
        if blocks.shape[1] != info.row_bytes(in_features):
            raise AnvilError(ANVIL_ERR_INVALID,
                             f"{info.name} rows of {in_features} values take {info.row_bytes(in_features)} "
                             f"bytes, got {blocks.shape[1]}")
        self.quant = info.name
        self.in_features = int(in_features)
        self.out_features = int(blocks.shape[0])
        self.nwarps, self.rows_per_block = nwarps, rows_per_block
        self.register_buffer("weight_blocks", blocks.contiguous())
        if bias is not None:
            self.bias = nn.Parameter(bias.detach().to(torch.float32).clone(), requires_grad=False)
        else:
            self.bias = None

    @staticmethod
    def _total_tokens(x: torch.Tensor) -> int:
        n = 1
        for d in x.shape[:-1]:
            n *= int(d)
        return n

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[-1] != self.in_features:
            raise AnvilError(ANVIL_ERR_INVALID, f"expected {self.in_features} input features, got {x.shape[-1]}")
        T = self._total_tokens(x)
        x2 = x.reshape(T, self.in_features).to(torch.float32).contiguous()
        out = torch.empty((T, self.out_features), dtype=torch.float32, device=x.device)
        W = self.weight_blocks
        for c0 in range(0, T, MAX_COLS):
            c1 = min(T, c0 + MAX_COLS)
            ops.mmvq_f32(W, self.quant, x2[c0:c1], nwarps=self.nwarps,
                         rows_per_block=self.rows_per_block, out=out[c0:c1])
        if self.bias is not None:
            out += self.bias
        return out.to(x.dtype).reshape(*x.shape[:-1], self.out_features)

    @classmethod
    def from_linear(cls, linear: nn.Linear, quant="Q8_0", **launch) -> "QuantLinear":
        """Quantise an nn.Linear's weight to GGUF blocks (gguf-py's quantiser; it implements
        Q8_0, so the K-quants come from GGUF files: from_gguf)."""
        from gguf import GGMLQuantizationType, quants

        info = resolve_type(quant)
        w = linear.weight.detach().to(torch.float32).cpu().numpy()
        try:
            blocks = quants.quantize(np.ascontiguousarray(w), getattr(GGMLQuantizationType, info.name))
        except NotImplementedError:
            raise AnvilError(ANVIL_ERR_INVALID,
                             f"{info.name} weights are read from GGUF files (from_gguf); only Q8_0 "
                             "is quantised here") from None
        dev = linear.weight.device
        return cls(torch.from_numpy(np.ascontiguousarray(blocks)).to(dev), info, linear.in_features,
                   linear.bias, **launch)

    @classmethod
    def from_gguf(cls, path, tensor_name: str, bias: torch.Tensor | None = None, device="cuda",
                  **launch) -> "QuantLinear":
        """The GGUF tensor `tensor_name` as stored (no requantisation)."""
        from kernel_anvil.gguf import read_tensor_blocks

        qt, nrows, K, blocks = read_tensor_blocks(path, tensor_name)
        t = torch.from_numpy(np.ascontiguousarray(blocks).reshape(nrows, -1)).to(device)
        return cls(t, qt, K, bias, **launch)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"quant={self.quant}, bias={self.bias is not None}, nwarps={self.nwarps}, "
                f"rows_per_block={self.rows_per_block}")


def load_gguf_linears(path, device="cuda") -> dict[str, QuantLinear]:
    """Every 2-D tensor of a GGUF file whose type has an MMVQ kernel, as QuantLinear modules
    keyed by tensor name (tensor data read from the file as stored)."""
    from gguf import GGUFReader

    out = {}
    for t in GGUFReader(str(path)).tensors:  # one parse of the file for every tensor
        qt = t.tensor_type.name
        if len(t.shape) != 2 or qt not in QUANT_TYPES:
            continue
        K, nrows = int(t.shape[0]), int(t.shape[1])
        if K % resolve_type(qt).qk:
            continue
        blocks = torch.from_numpy(np.ascontiguousarray(t.data).reshape(nrows, -1)).to(device)
        out[t.name] = QuantLinear(blocks, qt, K, None)
    return out


def _replace(model: nn.Module, name: str, module: nn.Module) -> None:
    parts = name.split(".")
    parent = model
    for part in parts[:-1]:
        parent = getattr(parent, part)
    setattr(parent, parts[-1], module)


def optimize(model: nn.Module, quant="Q8_0", verbose: bool = True, **launch) -> nn.Module:
    """Replace every nn.Linear whose in_features is a multiple of the block size with a
    QuantLinear holding its weight quantised to `quant` (in place; returns the model)."""
    info = resolve_type(quant)
    linears = [(n, m) for n, m in model.named_modules() if type(m) is nn.Linear]
    replaced = 0
    for name, mod in linears:
        if mod.in_features % info.qk:
            continue
        _replace(model, name, QuantLinear.from_linear(mod, info, **launch))
        replaced += 1
    if verbose:
        print(f"[kernel-anvil] Replaced {replaced} of {len(linears)} nn.Linear layers with "
              f"QuantLinear ({info.name})")
    return model
