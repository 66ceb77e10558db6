"""Device buffers that other processes can map: cudaMalloc'd here (so one
CUDA IPC handle covers the whole buffer at offset 0), viewed as torch
tensors through ``__cuda_array_interface__`` (no copy), freed when the
last view is gone."""

from __future__ import annotations

import ctypes

import torch

from infera_b200.ops import _native

_TYPESTR = {torch.bfloat16: ("<i2", torch.int16), torch.float16: ("<f2", None), torch.float32: ("<f4", None),
            torch.int32: ("<i4", None), torch.uint8: ("|u1", None)}


class DeviceBuffer:
    def __init__(self, nbytes: int, device: torch.device):
        self.device = torch.device(device)
        self.nbytes = nbytes
        with torch.cuda.device(self.device):
            p = ctypes.c_void_p()
            _native.check(_native.kernels().ib_sym_alloc(nbytes, ctypes.byref(p)), "ib_sym_alloc")
        self.ptr = p.value

    def ipc_handle(self) -> bytes:
        h = (ctypes.c_char * 64)()
        with torch.cuda.device(self.device):
            _native.check(_native.kernels().ib_ipc_handle(ctypes.c_void_p(self.ptr), h), "ib_ipc_handle")
        return bytes(h)

    def __del__(self):
        try:
            if self.ptr:
                _native.kernels().ib_sym_free(ctypes.c_void_p(self.ptr))
                self.ptr = 0
        except Exception:
            pass


class _View:
    def __init__(self, buf: DeviceBuffer, shape, typestr: str):
        self._buf = buf
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (buf.ptr, False),
                                         "version": 3, "strides": None, "stream": None}


def device_tensor(shape, dtype: torch.dtype, device) -> tuple[torch.Tensor, DeviceBuffer]:
    """A zero-filled tensor over a fresh exportable allocation; keep the
    returned buffer alive as long as the tensor."""
    n = 1
    for d in shape:
        n *= int(d)
    elem = torch.empty((), dtype=dtype).element_size()
    buf = DeviceBuffer(n * elem, device)
    typestr, carrier = _TYPESTR[dtype]
    t = torch.as_tensor(_View(buf, shape, typestr), device=buf.device)
    if carrier is not None:
        t = t.view(dtype)
    t._ib_buffer = buf  # the tensor keeps its allocation alive
    return t, buf
