"""Zero-copy host I/O for decode: pinned host memory mapped into the device
address space (`hba_b200_host_alloc`).  The decode kernel reads the query
from it and writes out / LSE into it directly, so a serving step needs no
copy before or after the launch.

    buf = MappedHostBuffer(q_bytes + out_bytes + lse_bytes)
    q_h = buf.host_view(torch.bfloat16, (B, Hq, dh))          # host tensor: fill with the query
    out_h = buf.host_view(torch.bfloat16, (B, Hq, dh), offset=q_bytes)
    cache.decode_into(buf.device_view(0), buf.device_view(q_bytes), ...)
"""

import ctypes

import torch

from . import _lib


class DevicePointer:
    """A device address with the `data_ptr()` the library's wrappers read."""

    def __init__(self, addr):
        self.addr = int(addr)

    def data_ptr(self):
        return self.addr


class MappedHostBuffer:
    """`nbytes` of pinned, device-mapped host memory; `close()` frees it."""

    def __init__(self, nbytes):
        self.nbytes = int(nbytes)
        h, d = ctypes.c_void_p(), ctypes.c_void_p()
        _lib.check(_lib.load().hba_b200_host_alloc(self.nbytes, ctypes.byref(h), ctypes.byref(d)),
                   "hba_b200_host_alloc")
        self.host_ptr, self.dev_ptr = h.value, d.value
        self._bytes = torch.frombuffer((ctypes.c_uint8 * self.nbytes).from_address(self.host_ptr), dtype=torch.uint8)

    def host_view(self, dtype, shape, offset=0):
        """A CPU tensor over [offset, offset + numel * itemsize) of the buffer."""
        n = 1
        for s in shape:
            n *= int(s)
        size = n * torch.empty((), dtype=dtype).element_size()
        if offset < 0 or offset + size > self.nbytes or offset % 16:
            raise ValueError("host view out of the buffer or not 16-byte aligned")
        return self._bytes[offset: offset + size].view(dtype).view(*shape)

    def device_view(self, offset=0):
        """The device address of byte `offset` (for the library's pointer arguments)."""
        if offset < 0 or offset >= self.nbytes:
            raise ValueError("device view out of the buffer")
        return DevicePointer(self.dev_ptr + offset)

    def close(self):
        if self.host_ptr is not None:
            self._bytes = None
            _lib.load().hba_b200_host_free(ctypes.c_void_p(self.host_ptr))
            self.host_ptr = self.dev_ptr = None
