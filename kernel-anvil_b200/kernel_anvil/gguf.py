"""GGUF model parsing: tensor shapes, quant types, unique GEMV workloads, tensor data.

``parse_gguf`` / ``ModelProfile`` / ``TensorInfo`` / ``print_model_summary`` keep the
reference's interface (kernel_anvil/gguf.py:14-111) and parse results, including its key
convention: ``unique_shapes`` is keyed ``(quant, ne0, ne1)``, the GGUF dims order, which is
(columns, rows) of the weight matrix (gguf-py gguf_reader.py keeps ``shape = dims`` with
ne0 first).  ``ModelProfile.gemv_shapes()`` gives the same counts keyed by the true GEMV
shape ``(quant, N rows, K cols)``, which is what the MMVQ launch and the smithy lookup
``[bucket(nrows)][bucket(ncols)]`` (patches/smithy-config.h:319-331) use.

``read_tensor_blocks`` returns a quantized tensor's raw GGUF blocks as a (rows, row_bytes)
uint8 array ready to copy to the GPU; ``write_gguf`` writes synthetic models for tests.
"""
from __future__ import annotations

from collections import Counter
from dataclasses import dataclass, field
from pathlib import Path


@dataclass
class TensorInfo:
    name: str
    shape: tuple[int, ...]  # GGUF dims order: (ne0, ne1, ...) = (cols, rows, ...) for 2-D
    quant_type: str
    size_bytes: int


@dataclass
class ModelProfile:
    name: str
    architecture: str
    tensors: list[TensorInfo]
    unique_shapes: dict[tuple[str, int, int], int] = field(default_factory=dict)
    # (quant_type, ne0, ne1) -> count over 2-D tensors (reference convention)

    def gemv_shapes(self) -> dict[tuple[str, int, int], int]:
        """{(quant, N rows, K cols): count}: the unique GEMVs decode runs."""
        out: Counter = Counter()
        for (qt, ne0, ne1), c in self.unique_shapes.items():
            out[(qt, ne1, ne0)] += c
        return dict(out)


def _metadata_str(reader, key: str) -> str | None:
    """A string-valued metadata field, decoded by gguf-py itself (ReaderField.contents()),
    or None when the key is absent or holds something else."""
    field = reader.fields.get(key)
    if field is None:
        return None
    try:
        value = field.contents()
    except (IndexError, ValueError, TypeError):
        return None
    return value if isinstance(value, str) else None


def parse_gguf(path: str | Path) -> ModelProfile:
    """Read tensor metadata of a GGUF file (gguf-py GGUFReader; tensor data is memory-mapped,
    not read).  Raises FileNotFoundError for a missing file."""
    path = Path(path)
    if not path.exists():
        raise FileNotFoundError(f"GGUF file not found: {path}")
    from gguf import GGUFReader

    reader = GGUFReader(str(path))
    name = _metadata_str(reader, "general.name") or path.stem
    arch = _metadata_str(reader, "general.architecture") or "unknown"
    tensors, shapes = [], Counter()
    for t in reader.tensors:
        shape = tuple(int(x) for x in t.shape)
        qt = t.tensor_type.name
        tensors.append(TensorInfo(t.name, shape, qt, int(t.n_bytes)))
        if len(shape) == 2:
            shapes[(qt, shape[0], shape[1])] += 1
    return ModelProfile(name=name, architecture=arch, tensors=tensors, unique_shapes=dict(shapes))


def print_model_summary(profile: ModelProfile) -> None:
    """Human-readable overview: totals, then one line per unique GEMV workload with its true
    shape (rows x cols) and the GGUF dims key the tuner's JSON uses."""
    mats = [t for t in profile.tensors if len(t.shape) == 2]
    gib = sum(t.size_bytes for t in profile.tensors) / 2**30
    print(f"{profile.name} [{profile.architecture}]: {len(profile.tensors)} tensors, "
          f"{len(mats)} matrices, {gib:.2f} GiB")
    if not profile.unique_shapes:
        print("no 2-D tensors")
        return
    width = max(len(qt) for qt, _, _ in profile.unique_shapes)
    print(f"{len(profile.unique_shapes)} GEMV workloads (rows x cols; GGUF ne0 x ne1 in brackets):")
    for (qt, ne0, ne1), count in sorted(profile.unique_shapes.items(),
                                        key=lambda kv: (kv[0][0], -kv[0][2] * kv[0][1])):
        print(f"  {qt.ljust(width)}  {ne1:>7} x {ne0:<7} [{ne0} x {ne1}]  x{count}")


def read_tensor_blocks(path: str | Path, name: str):
    """(quant_type, nrows, K, blocks) of one 2-D tensor; blocks is a (nrows, row_bytes)
    uint8 view of the file's GGUF block data."""
    from gguf import GGUFReader

    reader = GGUFReader(str(path))
    for t in reader.tensors:
        if t.name == name:
            if len(t.shape) != 2:
                raise ValueError(f"{name} is not 2-D")
            K, nrows = int(t.shape[0]), int(t.shape[1])
            return t.tensor_type.name, nrows, K, t.data
    raise KeyError(name)


def write_gguf(path: str | Path, tensors, name: str = "synthetic", arch: str = "llama",
               seed: int = 0) -> Path:
    """Write a GGUF file whose 2-D tensors are seeded synthetic quantized weights.

    tensors: iterable of (tensor_name, quant, N rows, K cols)."""
    import numpy as np
    from gguf import GGMLQuantizationType, GGUFWriter

    from kernel_anvil.quants import make_weights

    path = Path(path)
    w = GGUFWriter(str(path), arch)
    w.add_name(name)
    for i, (tname, qt, n, k) in enumerate(tensors):
        if qt in ("F32", "F16"):
            dt = np.float32 if qt == "F32" else np.float16
            w.add_tensor(tname, np.zeros((n, k) if n > 1 else (k,), dtype=dt))
        else:
            w.add_tensor(tname, make_weights(qt, n, k, seed=seed + i),
                         raw_dtype=getattr(GGMLQuantizationType, qt))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return path
