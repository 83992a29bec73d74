"""Streaming model and calibration input for the per-layer path.

The reference pipeline reads the whole model into host RAM with
``safetensors.torch.load_file`` and upcasts each weight to fp32 on the host
(pipeline.py:268, 524), and loads the whole calibration file, every layer's
Hessian included, before the first layer (pipeline.py:277; calibration_io.py).
For a 9B-parameter model with 16384-wide Hessians that is tens of GB of host
memory and a host-side fp32 copy per layer.

:class:`SafetensorsReader` reads one tensor at a time straight from the file
into the GPU in its stored dtype (fp16 stays fp16; the kernels upcast in their
loads): the header is parsed once, each tensor's byte range is read in chunks
into two pinned staging buffers that alternate, and each chunk is copied to the
device asynchronously on a copy stream while the next chunk is read.
:func:`load_calibration_lazy` opens a ``torch.save`` calibration file with
memory mapping, so a layer's Hessian is read from disk only when the pipeline
asks for that layer (the mapping keeps the reference's ``"hessians"`` /
``"amax_per_channel"`` / ``"metadata"`` layout, calibration_io.py:9-37).
"""

from __future__ import annotations

import json
import os
import struct
from collections.abc import Mapping

import torch

# safetensors dtype tags -> torch dtypes
_DTYPES = {
    "F64": torch.float64, "F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16,
    "I64": torch.int64, "I32": torch.int32, "I16": torch.int16, "I8": torch.int8, "U8": torch.uint8,
    "BOOL": torch.bool,
}


class SafetensorsReader(Mapping):
    """Read-only view of a .safetensors file: ``reader[name]`` (or
    ``reader.get(name, device)``) returns one tensor, read on demand."""

    def __init__(self, path: str, chunk_bytes: int = 64 << 20):
        self.path = path
        self.chunk = int(chunk_bytes)
        with open(path, "rb") as f:
            (n,) = struct.unpack("<Q", f.read(8))
            header = json.loads(f.read(n))
        self.metadata = header.pop("__metadata__", None) or {}
        self._base = 8 + n
        self._index = header
        self._fd = os.open(path, os.O_RDONLY)
        self._stage: list[torch.Tensor] = []
        self._stream: dict[int, torch.cuda.Stream] = {}

    def close(self) -> None:
        if self._fd >= 0:
            os.close(self._fd)
            self._fd = -1

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass

    def __iter__(self):
        return iter(self._index)

    def __len__(self) -> int:
        return len(self._index)

    def __getitem__(self, name: str) -> torch.Tensor:
        return self.get(name, "cpu")

    def info(self, name: str) -> tuple[torch.dtype, tuple[int, ...]]:
        e = self._index[name]
        return _DTYPES[e["dtype"]], tuple(e["shape"])

    def _read_into(self, buf: torch.Tensor, off: int, nbytes: int) -> None:
        view = memoryview(buf.numpy()).cast("B")[:nbytes]
        got = 0
        while got < nbytes:
            k = os.preadv(self._fd, [view[got:]], self._base + off + got)
            if k <= 0:
                raise OSError(f"{self.path}: short read at byte {self._base + off + got}")
            got += k

    def get(self, name: str, device="cpu") -> torch.Tensor:
        e = self._index[name]
        dtype = _DTYPES[e["dtype"]]
        shape = tuple(e["shape"])
        b0, b1 = e["data_offsets"]
        nbytes = b1 - b0
        dev = torch.device(device)
        if dev.type != "cuda":
            out = torch.empty(nbytes, dtype=torch.uint8)
            if nbytes:
                self._read_into(out, b0, nbytes)
            return out.view(dtype).reshape(shape)
        out = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        if not self._stage:
            self._stage = [torch.empty(self.chunk, dtype=torch.uint8).pin_memory() for _ in range(2)]
        idx = dev.index if dev.index is not None else torch.cuda.current_device()
        st = self._stream.get(idx)
        if st is None:
            st = self._stream[idx] = torch.cuda.Stream(dev)
        done = [None, None]
        pos, k = 0, 0
        while pos < nbytes:
            n = min(self.chunk, nbytes - pos)
            buf = self._stage[k & 1]
            if done[k & 1] is not None:
                done[k & 1].synchronize()  # the copy that last used this staging buffer
            self._read_into(buf, b0 + pos, n)
            with torch.cuda.stream(st):
                out[pos:pos + n].copy_(buf[:n], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(st)
            done[k & 1] = ev
            pos += n
            k += 1
        torch.cuda.current_stream(dev).wait_stream(st)
        out.record_stream(torch.cuda.current_stream(dev))
        return out.view(dtype).reshape(shape)


def load_calibration_lazy(path: str) -> dict:
    """A calibration file (``torch.save`` dict with ``"hessians"``,
    ``"amax_per_channel"``, ``"metadata"``, ...) opened with memory mapping:
    the returned dict has the reference's layout, and each tensor's bytes are
    read from disk only when it is used."""
    return torch.load(path, map_location="cpu", mmap=True, weights_only=True)
