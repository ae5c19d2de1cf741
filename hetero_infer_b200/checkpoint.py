"""Stage weights from an MLX-format safetensors snapshot, for the device stage.

The reference's weight index (hetero/shard.py:63-158): the safetensors
headers are parsed without touching tensor data, every tensor is classified
to the stages that own it, byte counts feed the planner, and a stage reads
only its own tensors.  Here a stage's tensors are memory-mapped straight out
of the files (no intermediate copy) and uploaded by `cuda_model.Stage`;
`stage_from_snapshot` does both.

The ownership rules and the dtype size table are the reference's (they
define the checkpoint format and the planner's accounting, so they are kept
alike); the reading is this module's own.
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
        with open(os.path.join(model_dir, "config.json")) as f:
            self.config = json.load(f)

    @property
    def tied(self) -> bool:
        """Tied embeddings: the head stage reuses the embedding matrix."""
        return bool(self.config.get("tie_word_embeddings", False))

    def owns(self, name: str, spec) -> bool:
        if name.startswith("model.layers."):
            return spec.start <= int(name.split(".")[2]) < spec.end
        if name.startswith("model.embed_tokens"):
            return spec.embed or (self.tied and spec.head)  # a tied head keeps its own copy
        if name.startswith("lm_head") or name == "model.norm.weight":
            return spec.head
        raise KeyError(f"unclassified tensor {name}")

    def names(self) -> List[str]:
        return list(self.entries)

    def nbytes(self, name: str) -> int:
        return self.entries[name][3]

    def layer_bytes(self) -> List[int]:
        out = [0] * int(self.config["num_hidden_layers"])
        for name, (_, _, _, nb) in self.entries.items():
            if name.startswith("model.layers."):
                out[int(name.split(".")[2])] += nb
        return out

    def embed_bytes(self) -> int:
        return sum(nb for n, (_, _, _, nb) in self.entries.items() if n.startswith("model.embed_tokens"))

    def head_bytes(self) -> int:
        b = sum(nb for n, (_, _, _, nb) in self.entries.items()
                if n.startswith("lm_head") or n == "model.norm.weight")
        return b + (self.embed_bytes() if self.tied else 0)

    def total_bytes(self) -> int:
        return sum(nb for _, _, _, nb in self.entries.values())

    def shard_bytes(self, spec) -> int:
        return sum(nb for n, (_, _, _, nb) in self.entries.items() if self.owns(n, spec))

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
