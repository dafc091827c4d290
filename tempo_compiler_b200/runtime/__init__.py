"""Drop-in replacement of the reference's board runtime (``board_package/runtime``) on a B200.

The reference's layer drivers import ``MemcpyKind``, ``minitpuSetDevice``, ``minitpuHostAlloc``, ``minitpuHostReset``,
``minitpuMalloc``, ``minitpuFree``, ``minitpuMemcpy`` and ``minitpuLaunchKernel`` from a module named ``runtime``
(board_package/gpt2_inference.py:49-58, board_checks.py:49-59). This module provides the same names with the same
argument meaning and error classes, backed by libtempo_b200.so: device memory is one arena addressed by 32-bit
kernel addresses from 0x80000000, copies and launches are synchronous, and a launch runs the B200 kernel the staged
image descriptor names. Installing it as ``sys.modules["runtime"]`` before importing the drivers swaps the backend,
exactly as the reference's emulator does (tools/emulators/emulate_board_checks.py:21-23).

Environment: ``TEMPO_DEVICE`` (default: ``LOCAL_RANK`` or 0) picks the GPU, ``TEMPO_ARENA_BYTES`` (default 1 GiB) the
arena, ``TEMPO_HOST_BYTES`` (default 64 MiB) the pinned host staging buffer, ``TEMPO_LAUNCH_TIMEOUT`` (default 10 s)
the bounded wait of every launch (the reference's completion poll, runtime/memcpy.py:49).
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import Sequence

import numpy as np

from tempo_compiler_b200 import lib as _lib

CDMA_ALIGN: int = 32
"""Byte alignment both copy operands require (runtime/memcpy.py:27)."""

_DEVICE_OPEN: list[bool] = [False]


class MemcpyKind:
    """The direction a copy takes (runtime/memcpy.py:65-75)."""

    HostToDevice = "HostToDevice"
    DeviceToHost = "DeviceToHost"


@dataclass(frozen=True)
class DeviceAddressSpace:
    """The arena's kernel-view map (runtime/address_space.py:8-135): one aperture, kernel and copy views identical."""

    kernel_base: int
    kernel_size: int
    reserved: int

    @property
    def copy_base(self) -> int:
        return self.kernel_base

    @property
    def copy_size(self) -> int:
        return self.kernel_size

    def contains_kernel(self, address: int, nbytes: int = 0) -> bool:
        return nbytes >= 0 and self.kernel_base <= address and address + nbytes <= self.kernel_base + self.kernel_size

    contains_copy = contains_kernel

    def to_copy(self, address: int, nbytes: int = 0) -> int:
        if not self.contains_kernel(address, nbytes):
            raise ValueError(f"Unable to translate a device range to a copy address. The range [0x{address:x}, "
                             f"0x{address + nbytes:x}) must lie inside the arena.")
        return address

    to_kernel = to_copy


class HostRegion:
    """One pinned host region carved from the staging buffer (runtime/backend.py HostRegion).

    Attributes:
        view: The region's contents as little-endian 32-bit words, writable in place.
        phys_addr: The region's host address, which the copy uses.
    """

    def __init__(self, buffer: np.ndarray, address: int, offset: int, words: int) -> None:
        self.view = buffer[offset // 4: offset // 4 + words]
        self.phys_addr = address + offset
        self.nbytes = words * 4

    def sync_to_device(self) -> None:
        """Pinned host memory is coherent: nothing to flush."""

    def sync_from_device(self) -> None:
        """Pinned host memory is coherent: nothing to invalidate."""


class _Staging:
    """The pinned host buffer host regions are bumped out of (runtime/device.py:84-146)."""

    def __init__(self) -> None:
        self.address = 0
        self.array: np.ndarray | None = None
        self.size = 0
        self.offset = 0

    def ensure(self) -> None:
        if self.array is not None:
            return
        _ensure_open()
        size = int(os.environ.get("TEMPO_HOST_BYTES", 64 << 20))
        pointer = ctypes.c_void_p()
        _lib.call("tempo_host_alloc", ctypes.byref(pointer), size)
        self.address = int(pointer.value)
        self.array = np.ctypeslib.as_array((ctypes.c_uint32 * (size // 4)).from_address(self.address))
        self.size = size
        self.offset = 0


_STAGING = _Staging()


def _round_up(value: int, align: int) -> int:
    return (value + align - 1) // align * align


def _device_index() -> int:
    return int(os.environ.get("TEMPO_DEVICE", os.environ.get("LOCAL_RANK", "0")))


def _ensure_open() -> None:
    if not _DEVICE_OPEN[0]:
        _lib.call("tempo_open", _device_index(), int(os.environ.get("TEMPO_ARENA_BYTES", 1 << 30)))
        _DEVICE_OPEN[0] = True


def open_device(uio_name: str = "minitpu", *, udmabuf_index: int = 0, address_space=None):
    """Opens the GPU and its arena (runtime/device.py:38-65); returns (address space, None)."""
    _ensure_open()
    return minitpuGetAddressSpace(), None


def minitpuSetDevice(uio_name: str) -> None:  # noqa: N802 -- the reference's name
    """Selects the device: opens the GPU and its arena on first use (runtime/device.py:68-81)."""
    _ensure_open()


def minitpuHostAlloc(nbytes: int, *, udmabuf_index: int | None = None) -> HostRegion:  # noqa: N802
    """Carves the next 32-byte-aligned pinned host region (runtime/device.py:84-125).

    Raises:
        RuntimeError: When the staging buffer is exhausted.
    """
    _STAGING.ensure()
    aligned = _round_up(int(nbytes), CDMA_ALIGN)
    if _STAGING.offset + aligned > _STAGING.size:
        raise RuntimeError(f"Unable to allocate host memory. The {_STAGING.size}-byte staging buffer is exhausted at "
                           f"offset {_STAGING.offset}, but got a request for {nbytes} bytes, {aligned} aligned.")
    region = HostRegion(_STAGING.array, _STAGING.address, _STAGING.offset, _round_up(int(nbytes), 4) // 4)
    _STAGING.offset += aligned
    return region


def minitpuHostReset() -> None:  # noqa: N802
    """Resets the host allocator; regions carved before are reused by later ones (runtime/device.py:128-134)."""
    _STAGING.offset = 0


def minitpuHostRewind() -> None:  # noqa: N802
    """Resets the host allocator's bump offset (runtime/device.py:137-145)."""
    _STAGING.offset = 0


def minitpuMalloc(nbytes: int) -> int:  # noqa: N802
    """First-fit device allocation, 32-byte aligned (runtime/device.py:148-175).

    Raises:
        ValueError: When the size is not positive.
        MemoryError: When no free span fits.
    """
    if nbytes <= 0:
        raise ValueError(f"Unable to allocate device memory. The requested size must be positive, but got {nbytes}.")
    _ensure_open()
    address = ctypes.c_uint32()
    _lib.call("tempo_malloc", ctypes.byref(address), int(nbytes))
    return int(address.value)


def minitpuFree(address: int) -> None:  # noqa: N802
    """Returns a device allocation (runtime/device.py:178-196). Raises KeyError for an unknown pointer."""
    _ensure_open()
    if not 0 <= int(address) <= 0xFFFFFFFF:
        raise KeyError(f"Unable to free device memory. The pointer 0x{int(address):x} was not returned by "
                       f"minitpuMalloc.")
    _lib.call("tempo_free", int(address))


def minitpuDeviceReset() -> None:  # noqa: N802
    """Forgets every device allocation (runtime/device.py:199-204)."""
    _ensure_open()
    _lib.call("tempo_device_reset")


def minitpuInAperture(address: int, nbytes: int = 0) -> bool:  # noqa: N802
    """Whether a range lies in the allocatable part of the arena (runtime/device.py:207-214)."""
    space = minitpuGetAddressSpace()
    return space.kernel_base + space.reserved <= address and address + max(0, nbytes) <= (
        space.kernel_base + space.kernel_size)


def minitpuGetAddressSpace() -> DeviceAddressSpace:  # noqa: N802
    """The arena's address map (runtime/address_space.py:180-192)."""
    _ensure_open()
    base, size, reserved = ctypes.c_uint32(), ctypes.c_uint64(), ctypes.c_uint32()
    _lib.call("tempo_address_space", ctypes.byref(base), ctypes.byref(size), ctypes.byref(reserved))
    return DeviceAddressSpace(kernel_base=int(base.value), kernel_size=int(size.value), reserved=int(reserved.value))


def minitpuConfigureAddressSpace(address_space) -> None:  # noqa: N802
    """The arena's map is fixed by the library; configuring another is refused (runtime/address_space.py:164-177)."""
    if not isinstance(address_space, DeviceAddressSpace):
        raise TypeError(f"Unable to configure the address space. The map must be a DeviceAddressSpace, but got "
                        f"{type(address_space).__name__}.")
    if address_space != minitpuGetAddressSpace():
        raise RuntimeError("Unable to change the device address space. The B200 arena's map is fixed at open.")


def _host_address(operand) -> int:
    return int(operand.phys_addr) if hasattr(operand, "phys_addr") else int(operand)


def minitpuMemcpy(dst, src, nbytes: int, kind: str) -> None:  # noqa: N802
    """Synchronous copy between a host region and the device (runtime/memcpy.py:93-161).

    Raises:
        ValueError: When the kind is unknown, the byte count is not positive, or an address is misaligned or
            outside the arena.
        TimeoutError: When the copy does not finish within the bounded wait.
    """
    if kind == MemcpyKind.HostToDevice:
        host, device = src, dst
    elif kind == MemcpyKind.DeviceToHost:
        host, device = dst, src
    else:
        raise ValueError(f"Unable to copy. The kind must be MemcpyKind.HostToDevice or MemcpyKind.DeviceToHost, but "
                         f"got {kind!r}.")
    if nbytes < 0:
        raise ValueError(f"Unable to copy. The byte count must be non-negative, but got {nbytes}.")
    if nbytes == 0:
        raise ValueError("Unable to copy. The byte count must be positive, but got a zero-length request.")
    _ensure_open()
    device = int(device)
    if not 0 <= device <= 0xFFFFFFFF:
        raise ValueError(f"Unable to copy. The device address 0x{device:x} must be a 32-bit kernel address.")
    if kind == MemcpyKind.HostToDevice:
        _lib.call("tempo_memcpy_h2d", device, _host_address(host), int(nbytes))
    else:
        _lib.call("tempo_memcpy_d2h", _host_address(host), device, int(nbytes))


def minitpuMemcpyAsync(dst, src, nbytes: int, kind: str, stream: None = None) -> None:  # noqa: N802
    """As :func:`minitpuMemcpy`; the only stream is None (runtime/memcpy.py:164-187)."""
    if stream is not None:
        raise ValueError(f"Unable to order a copy on a stream. The stream must be None, but got {stream!r}.")
    minitpuMemcpy(dst=dst, src=src, nbytes=nbytes, kind=kind)


def minitpuLaunchKernel(kbin_addr: int, kbin_size: int, *, args: Sequence[int] | None = None) -> None:  # noqa: N802
    """Launches the image staged at ``kbin_addr`` and waits for it (runtime/launch.py:44-141).

    Raises:
        ValueError: For a malformed launch: size not a positive multiple of 16 or past 65536 bytes, base negative,
            past 32 bits or not 32-byte aligned, more than four arguments, an argument outside [0, 0xFFFFFFFF], or an
            operand range outside the arena.
        RuntimeError: When the staged bytes are not an image descriptor of a known kind (the reference's launch error).
        TimeoutError: When the launch does not finish within the bounded wait.
    """
    if kbin_addr < 0:
        raise ValueError(f"Unable to launch a kernel. The binary base must be non-negative, but got {kbin_addr}.")
    _ensure_open()
    values = [int(a) for a in (args or [])]
    if len(values) > 4:
        raise ValueError(f"Unable to launch a kernel. At most 4 values fit the argument slots 0 to 3, but got "
                         f"{len(values)}.")
    array = (ctypes.c_int64 * max(1, len(values)))(*values)
    timeout = float(os.environ.get("TEMPO_LAUNCH_TIMEOUT", "10"))
    _lib.call("tempo_launch", int(kbin_addr), int(kbin_size), array, len(values), timeout)


def minitpuDrain(timeout: float = 2.0) -> bool:  # noqa: N802
    """Waits for outstanding work; True when the device is idle (runtime/memcpy.py:190-206)."""
    if not _DEVICE_OPEN[0]:
        return True
    try:
        _lib.call("tempo_sync", float(timeout))
    except TimeoutError:
        return False
    return True


def launches() -> int:
    """Launches run through this runtime so far."""
    count, used = ctypes.c_uint64(), ctypes.c_uint64()
    _lib.call("tempo_stats", ctypes.byref(count), ctypes.byref(used))
    return int(count.value)


__all__ = ["CDMA_ALIGN", "DeviceAddressSpace", "HostRegion", "MemcpyKind", "minitpuConfigureAddressSpace",
           "minitpuDeviceReset", "minitpuDrain", "minitpuFree", "minitpuGetAddressSpace", "minitpuHostAlloc",
           "minitpuHostReset", "minitpuHostRewind", "minitpuInAperture", "minitpuLaunchKernel", "minitpuMalloc",
           "minitpuMemcpy", "minitpuMemcpyAsync", "minitpuSetDevice", "open_device", "launches"]
