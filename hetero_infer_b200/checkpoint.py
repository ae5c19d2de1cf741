"""Stage weights from an MLX-format safetensors snapshot, for the device stage.

The reference's weight index (hetero/shard.py:63-158): the safetensors
headers are parsed without touching tensor data, every tensor is classified
to the stages that own it, byte counts feed the planner, and a stage reads
only its own tensors.  Here a stage's tensors are memory-mapped straight out
of the files (no intermediate copy) and uploaded by `cuda_model.Stage`;
`stage_from_snapshot` does both.

The ownership rules and the dtype size table are the reference's (they
define the checkpoint format and the planner's accounting, so the results
are kept alike; here each tensor is classified once into a part of the
model and the byte counts are sums over parts); the reading is this
module's own.
"""
from __future__ import annotations

import glob
import json
import os
import struct
from typing import Dict, List, Tuple

import numpy as np

# bytes per element of each safetensors dtype (the format's table)
DTYPE_BYTES = {
    "BOOL": 1, "U8": 1, "I8": 1, "F8_E4M3": 1, "F8_E5M2": 1,
    "U16": 2, "I16": 2, "F16": 2, "BF16": 2,
    "U32": 4, "I32": 4, "F32": 4,
    "U64": 8, "I64": 8, "F64": 8,
}
# dtypes a stage can be built from (the packed weights are U32, scales and
# biases F16, norms F16/F32); BF16 has no NumPy type -- the reference's NumPy
# path cannot read it either
NUMPY_DTYPES = {
    "BOOL": np.bool_, "U8": np.uint8, "I8": np.int8, "U16": np.uint16, "I16": np.int16, "F16": np.float16,
    "U32": np.uint32, "I32": np.int32, "F32": np.float32, "U64": np.uint64, "I64": np.int64, "F64": np.float64,
}


def read_header(path: str) -> Tuple[Dict[str, dict], int]:
    """The tensor table of a safetensors file and the offset its data starts
    at (8-byte little-endian header length, then the JSON header)."""
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        head = json.loads(f.read(n))
    head.pop("__metadata__", None)
    return head, 8 + n


def _part(name: str):
    """The part of the model a tensor name belongs to: its decoder layer's
    index, "embed", "head", or None for a name outside the format."""
    if name.startswith("model.layers."):
        return int(name.split(".")[2])
    if name.startswith("model.embed_tokens"):
        return "embed"
    if name.startswith("lm_head") or name == "model.norm.weight":
        return "head"
    return None


class WeightIndex:
    """name -> (file, dtype, shape, bytes) across a snapshot directory, plus the
    snapshot's config.json (hetero/shard.py:72-158)."""

    def __init__(self, model_dir: str):
        self.dir = model_dir
        files = sorted(glob.glob(os.path.join(model_dir, "*.safetensors")))
        if not files:
            raise FileNotFoundError(f"no safetensors in {model_dir}")
        self.entries: Dict[str, Tuple[str, str, List[int], int]] = {}
        self._where: Dict[str, Tuple[int, int]] = {}  # name -> (absolute begin, end) in its file
        self._parts: Dict[str, object] = {}  # name -> layer index, "embed", "head" or None
        self._tot = None                     # part -> bytes, built on first use
        for path in files:
            head, data0 = read_header(path)
            for name, meta in head.items():
                shape = [int(s) for s in meta["shape"]]
                nb = DTYPE_BYTES[meta["dtype"]] * int(np.prod(shape, dtype=np.int64))
                b, e = meta["data_offsets"]
                if e - b != nb:
                    raise ValueError(f"{path}: {name} holds {e - b} bytes, its shape needs {nb}")
                self.entries[name] = (path, meta["dtype"], shape, nb)
                self._where[name] = (data0 + int(b), data0 + int(e))
                self._parts[name] = _part(name)
        with open(os.path.join(model_dir, "config.json")) as f:
            self.config = json.load(f)

    @property
    def tied(self) -> bool:
        """Tied embeddings: the head stage reuses the embedding matrix."""
        return bool(self.config.get("tie_word_embeddings", False))

    # Every tensor belongs to one part of the model: a decoder layer (its
    # index), the embedding table, or the head (lm_head and the final norm).
    # A stage owns its layers' range, the embedding when it embeds, the head
    # when it samples -- and, with tied embeddings, the head stage also holds
    # its own copy of the table.  Byte counts are sums over parts.
    def _part_of(self, name: str):
        part = self._parts.get(name, _part(name))
        if part is None:
            raise KeyError(f"unclassified tensor {name}")
        return part

    def _owns_part(self, part, spec) -> bool:
        if part == "embed":
            return spec.embed or (self.tied and spec.head)
        if part == "head":
            return spec.head
        return spec.start <= part < spec.end

    def owns(self, name: str, spec) -> bool:
        return self._owns_part(self._part_of(name), spec)

    def names(self) -> List[str]:
        return list(self.entries)

    def nbytes(self, name: str) -> int:
        return self.entries[name][3]

    def _part_bytes(self) -> Dict[object, int]:
        if self._tot is None:  # the index does not change after construction
            tot: Dict[object, int] = {}
            for name, (_, _, _, nb) in self.entries.items():
                part = self._parts[name]
                tot[part] = tot.get(part, 0) + nb
            self._tot = tot
        return self._tot

    def layer_bytes(self) -> List[int]:
        tot = self._part_bytes()
        return [tot.get(i, 0) for i in range(int(self.config["num_hidden_layers"]))]

    def embed_bytes(self) -> int:
        return self._part_bytes().get("embed", 0)

    def head_bytes(self) -> int:
        tot = self._part_bytes()
        return tot.get("head", 0) + (tot.get("embed", 0) if self.tied else 0)

    def total_bytes(self) -> int:
        return sum(nb for _, _, _, nb in self.entries.values())

    def shard_bytes(self, spec) -> int:
        tot = self._part_bytes()
        if None in tot:
            self._part_of(next(n for n, p in self._parts.items() if p is None))  # raises
        return sum(nb for part, nb in tot.items() if self._owns_part(part, spec))

    def load_shard(self, spec) -> Dict[str, np.ndarray]:
        """This stage's tensors only, as arrays mapped from the files."""
        out = {}
        maps = {}
        for name, (path, dt, shape, _) in self.entries.items():
            if not self.owns(name, spec):
                continue
            if dt not in NUMPY_DTYPES:
                raise TypeError(f"{name}: dtype {dt} is not supported")
            if path not in maps:
                maps[path] = np.memmap(path, dtype=np.uint8, mode="c")  # copy-on-write: nothing copied unless written
            b, e = self._where[name]
            out[name] = maps[path][b:e].view(NUMPY_DTYPES[dt]).reshape(shape)
        return out


def stage_from_snapshot(model_dir: str, spec, device="cuda", max_ctx: int = 2048):
    """The device stage owning `spec`, built from the snapshot's tensors."""
    from . import cuda_model
    idx = WeightIndex(model_dir)
    return cuda_model.Stage(idx.config, spec, idx.load_shard(spec), device=device, max_ctx=max_ctx)
