"""Torch-backed stand-in for the `aie.iron` tensor API that the reference's host code allocates its NPU buffers with.

The reference's DiT host loop (redline/forward.py) creates every device buffer through `aie.iron` - `tensor`
(forward.py:84, 185-189, 202, 321, 406-409, 613), `zeros` (220-221, 298-299), `Tensor.numpy` (268, 339, 348),
`Tensor.subview` (307-308, 324-327, 393), `Tensor.mutate` (343, 354) and `Tensor.to` (355) - and passes them to
`npu.run(op, artifact, [tensors])`. This module offers the same calls over CUDA memory, so that module can stand in
for `aie.iron` and the reference's own block loops hand B200 buffers to `npu.Device.run`, which maps every artifact
onto this library's kernels. Buffers only: nothing here computes.

  tensor(array, dtype, device)   a device copy of a numpy array (the reference's V9 bfp16 blocks, bf16, ...)
  zeros(shape, dtype, device)    a zeroed device buffer
  Tensor.numpy()                 a host copy (stream-ordered: waits for the kernels queued before it)
  Tensor.subview(off, shape, dt) a view `off` BYTES into the buffer (the reference passes byte offsets of V9 tiles)
  Tensor.mutate()                a context manager: edit a host copy, written back on exit
  Tensor.torch()                 the torch view npu.Device works on (uint8 bytes for V9, bfloat16, float32, int32)

`device` ("npu" in the reference) selects the current CUDA device; set_device("cpu") keeps buffers in host memory
for host-only checks of a call sequence (no kernel accepts them).
"""

import contextlib

import numpy as np
import torch

_TORCH = {"bfloat16": torch.bfloat16, "float32": torch.float32, "float16": torch.float16, "int32": torch.int32,
          "uint16": torch.int16, "int16": torch.int16}
_device = None


def set_device(dev):
    """Where new buffers live: a torch device (or "cpu"); None = the current CUDA device."""
    global _device
    _device = None if dev is None else torch.device(dev)


def _where():
    return _device if _device is not None else torch.device("cuda", torch.cuda.current_device())


class Tensor:
    """A typed window of `shape` x `dtype` onto a flat byte buffer in device memory."""

    def __init__(self, buf, offset, shape, dtype):
        self._buf, self._off = buf, int(offset)
        self.shape = tuple(int(s) for s in (shape if isinstance(shape, (tuple, list)) else (shape,)))
        self.dtype = np.dtype(dtype)
        self.nbytes = int(np.prod(self.shape, dtype=np.int64)) * self.dtype.itemsize
        if self._off < 0 or self._off + self.nbytes > buf.numel():
            raise ValueError(f"view of {self.nbytes} bytes at {self._off} outside a {buf.numel()}-byte buffer")

    def bytes(self):
        """The view's bytes as a flat uint8 torch tensor (shares memory)."""
        return self._buf.narrow(0, self._off, self.nbytes)

    def torch(self):
        """The torch view npu.Device works on: bf16 / fp32 / int32 elements, or raw bytes for V9 blocks."""
        t = _TORCH.get(self.dtype.name)
        b = self.bytes()
        return b if t is None else b.view(t)

    def numpy(self):
        host = self.bytes().cpu().numpy()
        return np.frombuffer(host.tobytes(), self.dtype).reshape(self.shape)

    def subview(self, offset, shape, dtype=None):
        return Tensor(self._buf, self._off + int(offset), shape, self.dtype if dtype is None else dtype)

    @contextlib.contextmanager
    def mutate(self):
        arr = self.numpy().copy()
        yield arr
        src = np.ascontiguousarray(arr, self.dtype).view(np.uint8).reshape(-1)
        self.bytes().copy_(torch.from_numpy(src.copy()).to(self._buf.device))

    def to(self, device):
        """The reference moves a mutated host view back to the NPU; this buffer never left device memory."""
        return self

    def __repr__(self):
        return f"iron.Tensor(shape={self.shape}, dtype={self.dtype}, device={self._buf.device})"


def tensor(array, dtype=None, device="npu"):
    arr = np.ascontiguousarray(array if dtype is None else np.asarray(array).astype(dtype, copy=False))
    raw = torch.from_numpy(arr.reshape(-1).view(np.uint8).copy())
    return Tensor(raw.to(_where()), 0, arr.shape, arr.dtype)


def zeros(shape, dtype=np.float32, device="npu"):
    shape = tuple(shape) if isinstance(shape, (tuple, list)) else (int(shape),)
    nbytes = int(np.prod(shape, dtype=np.int64)) * np.dtype(dtype).itemsize
    return Tensor(torch.zeros(nbytes, dtype=torch.uint8, device=_where()), 0, shape, dtype)
