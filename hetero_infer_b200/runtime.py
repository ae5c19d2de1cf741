"""The reference's stage runtime on the device: frames in, frames out.

The reference's pipeline runtime (hetero/engine.py) owns one stage shard,
its per-request KV caches and a loop that services frames: forward frames
carry token ids (first stage) or an encoded hidden state, and produce either
an encoded hidden state for the next stage or, on the stage with the head, a
sampled token (``StageRunner.run_frame``, engine.py:68-102); control frames
free a request, switch the codec, collect statistics, reset them or stop the
loop (``StageRunner.serve``, engine.py:104-147).  This module keeps that
contract -- the same constructor, the same frame headers and payload bytes --
with the stage on a B200:

* the wire codec (hetero/transport.py:198-225) runs on the device: the fp16
  frame is the hidden state cast on the device, the int8 frame comes from
  ``hq4_act_encode_i8_wire`` (fp16 rounding, then the codec, as the reference
  encodes ``backend.to_wire(y)``), and incoming frames are decoded on the
  device (``hq4_act_decode_i8``), so the only host traffic is the frame
  bytes themselves;
* the stage is ``cuda_model.Stage`` and the backend ``cuda_model.CudaBackend``
  (the reference's backend surface), so ``build_stage`` loads a shard from an
  MLX-format snapshot exactly as the reference's does (engine.py:162-173).

The transport is whatever object has ``send(header, payload=b"")`` and
``recv(timeout)``; ``LocalChannel`` is an in-process pair for running stages
in one process (the reference's TCP channel is out of scope: on one box the
GPUs exchange hidden states through ``pipeline.py`` over NCCL).
"""
from __future__ import annotations

import queue
import time
from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import numpy as np
import torch

from . import _lib, cuda_model


@dataclass
class StageStats:
    """Per-stage counters (hetero/engine.py:30-36)."""
    compute_s: float = 0.0
    frames: int = 0
    tokens: int = 0
    wait_s: float = 0.0
    bytes_out: int = 0


# -- the wire codec on the device (hetero/transport.py:198-225) ---------------

def encode(y: torch.Tensor, codec: str = "fp16") -> Tuple[dict, bytes]:
    """(header, payload) of the frame the reference's engine sends for the
    fp32 hidden state y: ``transport.encode(backend.to_wire(y), codec)``
    (engine.py:97).  fp16: the values cast to fp16.  int8: the fp16 values'
    per-row scale (max |x| / 127, 1 for a zero row) then the int8 rows."""
    if not (isinstance(y, torch.Tensor) and y.is_cuda):
        raise TypeError("encode takes the stage's device tensor")
    shape = [int(d) for d in y.shape]
    if codec == "fp16":
        return {"codec": "fp16", "shape": shape}, y.to(torch.float16).cpu().numpy().tobytes()
    if codec == "int8":
        from . import ops
        p = ops.act_encode_i8(y.float().contiguous().reshape(-1, shape[-1]), wire=True)
        return {"codec": "int8", "shape": shape}, p.cpu().numpy().tobytes()
    raise ValueError(f"unknown codec {codec}")


def decode(header: dict, payload: bytes, device) -> torch.Tensor:
    """The fp32 device tensor the reference's ``backend.from_wire(decode(...))``
    gives for a frame (transport.py:214-225, backends.py:103-104): the fp16
    values (int8: fp16(q * scale)) widened to fp32."""
    shape = tuple(int(d) for d in header["shape"])
    raw = torch.frombuffer(bytearray(payload), dtype=torch.uint8)
    if header["codec"] == "fp16":
        return raw.to(device).view(torch.float16).reshape(shape).float()
    if header["codec"] == "int8":
        from . import ops
        cols = shape[-1]
        rows = int(np.prod(shape[:-1]))
        if raw.numel() != rows * (4 + cols):
            raise ValueError(f"int8 frame of {raw.numel()} bytes for shape {shape}")
        return ops.act_decode_i8(raw.to(device), rows, cols, dtype=torch.float32).reshape(shape)
    raise ValueError(f"unknown codec {header['codec']}")


# -- the stage loop ---------------------------------------------------------------

class StageRunner:
    """Owns one shard on the device, its per-request caches, and the loop that
    services frames (hetero/engine.py:38-147, same constructor and frames)."""

    def __init__(self, stage, spec, n_layers_total: int, codec: str = "fp16",
                 sampler: Optional["Sampler"] = None, name: str = "stage", backend=None,
                 body_only: bool = False):
        self.name = name
        # a first stage that also owns the head applies it only when the
        # hidden state comes back around the ring (engine.py:44-46)
        self.body_only = body_only
        self.backend = backend or cuda_model.CudaBackend(stage.device, stage.max_ctx)
        self.stage = stage
        self.spec = spec
        self.n_layers_total = n_layers_total
        self.codec = codec
        self.sampler = sampler
        self.caches: Dict[str, cuda_model.DeviceKVCache] = {}
        self.stats = StageStats()

    def cache_for(self, req: str):
        c = self.caches.get(req)
        if c is None:
            c = self.backend.new_caches(len(self.stage.layers))
            self.caches[req] = c
        return c

    def free(self, req: str) -> None:
        self.caches.pop(req, None)

    def run_frame(self, header: dict, payload: bytes):
        """One forward frame -> (out_header, out_payload); (None, None) for an
        intermediate prefill chunk on the head stage (engine.py:68-102)."""
        req = header["req"]
        caches = self.cache_for(req)
        t0 = time.perf_counter()
        if self.spec.embed:
            x = self.backend.array(header["ids"])
        else:
            x = decode(header, payload, self.stage.device)
        want_tok = bool(header.get("logits", True)) and not self.body_only
        if self.body_only:
            y = self.stage.body(x, caches)
        else:
            y = self.stage(x, caches, apply_head=want_tok, last_only=True)
        if self.spec.head and not want_tok and not self.body_only:
            self.backend.eval(y)
            self.stats.compute_s += time.perf_counter() - t0
            self.stats.frames += 1
            return None, None
        if self.spec.head and not self.body_only:
            tok = self.sampler(y[:, -1, :], self.backend)
            self.stats.compute_s += time.perf_counter() - t0
            self.stats.frames += 1
            self.stats.tokens += 1
            return ({"t": "tok", "req": req, "tok": tok, "step": header.get("step", 0),
                     "last": header.get("last", True)}, b"")
        self.backend.eval(y)
        self.stats.compute_s += time.perf_counter() - t0
        self.stats.frames += 1
        h, p = encode(y, self.codec)
        h.update({"t": "fwd", "req": req, "step": header.get("step", 0), "last": header.get("last", True),
                  "logits": header.get("logits", True)})
        self.stats.bytes_out += len(p)
        return h, p

    def serve(self, inbound, outbound, stop_check=None) -> None:
        """Middle/last-stage loop: pull frames, compute, push onward; control
        frames as engine.py:104-147 handles them.  A transport error raised by
        ``inbound.recv`` (the reference surfaces a lost peer as
        ConnectionError) ends the loop by propagating."""
        while True:
            if stop_check is not None and stop_check():
                return
            t0 = time.perf_counter()
            header, payload = inbound.recv(timeout=None)
            self.stats.wait_s += time.perf_counter() - t0
            t = header.get("t")
            if t == "fwd":
                h, p = self.run_frame(header, payload)
                if h is not None:
                    outbound.send(h, p)
            elif t == "free":
                self.free(header["req"])
                if not self.spec.head:
                    outbound.send(header)
            elif t == "codec":
                self.codec = header["codec"]
                outbound.send(header)
            elif t == "shape":
                # link emulation settings travel on; there is no emulated link here
                outbound.send(header)
            elif t == "statq":
                link = outbound.stats() if hasattr(outbound, "stats") else {}
                header.setdefault("stats", []).append(
                    {"name": self.name, "compute_s": self.stats.compute_s, "frames": self.stats.frames,
                     "wait_s": self.stats.wait_s, "bytes_out": self.stats.bytes_out, "link": link})
                outbound.send(header)
            elif t == "reset":
                self.stats = StageStats()
                if not self.spec.head:
                    outbound.send(header)
            elif t in ("ping", "bw"):
                outbound.send({"t": "ack"})
            elif t == "stop":
                if not self.spec.head:
                    outbound.send(header)
                return


class Sampler:
    """Greedy or temperature/top-p sampling, delegated to the backend
    (hetero/engine.py:150-159)."""

    def __init__(self, temperature: float = 0.0, top_p: float = 1.0, seed: int = 0):
        self.temperature = temperature
        self.top_p = top_p
        self.rng = np.random.default_rng(seed)

    def __call__(self, logits, backend) -> int:
        return backend.sample(logits, self.temperature, self.top_p, self.rng)


def resident_bytes(index, spec, expansion: float = 1.0) -> int:
    """Bytes a shard occupies once loaded (engine.py:176-185): its layers
    times the backend's weight expansion (1 on the device: weights stay
    packed) plus everything else it owns."""
    lb = index.layer_bytes()
    layer = sum(lb[spec.start:spec.end])
    other = index.shard_bytes(spec) - layer
    return int(layer * expansion + other)


def build_stage(model_dir: str, spec, index=None, budget_bytes: int = 0, backend=None):
    """Load a shard onto the device, refusing to exceed the memory budget
    (engine.py:162-173): returns (stage, bytes, index)."""
    from . import checkpoint
    backend = backend or cuda_model.CudaBackend()
    index = index or checkpoint.WeightIndex(model_dir)
    need = resident_bytes(index, spec, backend.weight_expansion)
    if budget_bytes and need > budget_bytes:
        raise MemoryError(f"shard needs {need / 2**30:.2f} GiB on the {backend.name} backend but the "
                          f"budget is {budget_bytes / 2**30:.2f} GiB")
    stage, nbytes = backend.load_stage(model_dir, spec, index)
    return stage, nbytes, index


class LocalChannel:
    """One direction of an in-process frame link with the reference
    Channel's send/recv surface (transport.py:108-115); ``pair()`` gives two
    connected ends.  A ``close`` wakes a blocked reader with ConnectionError,
    as the reference's rx thread reports a lost peer."""

    def __init__(self, inq: "queue.Queue", outq: "queue.Queue"):
        self._in, self._out = inq, outq
        self.frames_sent = 0
        self.bytes_sent = 0

    @staticmethod
    def pair():
        a, b = queue.Queue(), queue.Queue()
        return LocalChannel(a, b), LocalChannel(b, a)

    def send(self, header: dict, payload: bytes = b"") -> None:
        self._out.put((header, payload))
        self.frames_sent += 1
        self.bytes_sent += len(payload)

    def recv(self, timeout: Optional[float] = None):
        try:
            item = self._in.get(timeout=timeout)
        except queue.Empty:
            raise TimeoutError("no frame within the timeout") from None
        if isinstance(item, Exception):
            raise item
        return item

    def close(self) -> None:
        self._out.put(ConnectionError("peer closed the channel"))

    def stats(self) -> dict:
        return {"bytes_sent": self.bytes_sent, "frames_sent": self.frames_sent}
