"""A host model of the drop-in runtime for CPU tests: the ``runtime`` module's calls over a byte array, each image kind
executed with the oracle's float64 arithmetic on the packed layouts.

It lets the block driver (``tempo_compiler_b200.dropin``) run its addressing, layouts and launch order without a GPU;
the numbers it produces are the oracle's, so a driver mistake (a wrong slot, offset, block stride or cache position)
shows up as a mismatch against the oracle's own chain. Argument binding follows the runtime's dispatcher
(``csrc/runtime.cu``) and its range checks.
"""

from __future__ import annotations

import struct

import numpy as np

from oracle import bf16 as ob
from oracle import references as orf

BASE = 0x8000_0000
RESERVED = 0x0010_0000
KINDS = {1: "gemm", 2: "gemm_bias", 3: "add", 4: "add_bias", 5: "layernorm", 6: "attention", 7: "decode_attention",
         8: "copy", 9: "halt"}


class MemcpyKind:
    HostToDevice = "HostToDevice"
    DeviceToHost = "DeviceToHost"


class _Region:
    def __init__(self, nbytes: int) -> None:
        self.view = np.zeros((nbytes + 3) // 4, np.uint32)
        self.phys_addr = id(self)

    def sync_to_device(self) -> None:
        pass

    def sync_from_device(self) -> None:
        pass


class _AddressSpace:
    kernel_base = BASE
    copy_base = BASE

    def __init__(self, size: int) -> None:
        self.kernel_size = self.copy_size = size
        self.reserved = RESERVED


class ImageModelRuntime:
    """Stands in for ``tempo_compiler_b200.runtime`` (the subset the block driver calls)."""

    MemcpyKind = MemcpyKind

    def __init__(self, arena_bytes: int = 256 << 20) -> None:
        self.memory = np.zeros(arena_bytes, np.uint8)
        self.next = RESERVED
        self.live: dict[int, int] = {}
        self.free_spans: list[tuple[int, int]] = []
        self.launches: list[str] = []

    # -- memory ---------------------------------------------------------------------------------------------------
    def minitpuSetDevice(self, name: str) -> None:  # noqa: N802
        pass

    def minitpuHostAlloc(self, nbytes: int, **_) -> _Region:  # noqa: N802
        return _Region(nbytes)

    def minitpuGetAddressSpace(self) -> _AddressSpace:  # noqa: N802
        return _AddressSpace(self.memory.size)

    def as_module(self):
        """A module object carrying the runtime's names, for ``sys.modules["runtime"]``."""
        import types
        module = types.ModuleType("runtime")
        module.MemcpyKind = MemcpyKind
        for name in dir(self):
            if name.startswith("minitpu"):
                setattr(module, name, getattr(self, name))
        return module

    def minitpuHostReset(self) -> None:  # noqa: N802
        pass

    def minitpuMalloc(self, nbytes: int) -> int:  # noqa: N802
        """First fit over freed spans, else the top of the arena (32-byte granules)."""
        if nbytes <= 0:
            raise ValueError("size must be positive")
        size = (nbytes + 31) // 32 * 32
        for index, (offset, span) in enumerate(self.free_spans):
            if span >= size:
                if span == size:
                    del self.free_spans[index]
                else:
                    self.free_spans[index] = (offset + size, span - size)
                break
        else:
            offset = self.next
            self.next += size
            if self.next > self.memory.size:
                raise MemoryError("arena exhausted")
        self.live[BASE + offset] = size
        return BASE + offset

    def minitpuFree(self, address: int) -> None:  # noqa: N802
        if address not in self.live:
            raise KeyError(hex(address))
        self.free_spans.append((address - BASE, self.live.pop(address)))

    def _span(self, address: int, nbytes: int) -> slice:
        offset = address - BASE
        if offset < 0 or offset + nbytes > self.memory.size:
            raise ValueError(f"range [0x{address:x}, +{nbytes}) outside the arena")
        return slice(offset, offset + nbytes)

    def minitpuMemcpy(self, dst, src, nbytes: int, kind: str) -> None:  # noqa: N802
        if nbytes <= 0:
            raise ValueError("byte count must be positive")
        if kind == MemcpyKind.HostToDevice:
            self.memory[self._span(dst, nbytes)] = src.view.view(np.uint8)[:nbytes]
        elif kind == MemcpyKind.DeviceToHost:
            dst.view.view(np.uint8)[:nbytes] = self.memory[self._span(src, nbytes)]
        else:
            raise ValueError(kind)

    # -- typed views of the arena -----------------------------------------------------------------------------------
    def words(self, address: int, count: int) -> np.ndarray:
        return self.memory[self._span(address, 2 * count)].view(np.uint16)

    def floats(self, address: int, count: int) -> np.ndarray:
        return ob.bf16_values(self.words(address, count))

    def store(self, address: int, values) -> None:
        self.words(address, np.asarray(values).size)[:] = ob.bf16_bits(np.asarray(values, np.float32).reshape(-1))

    def block(self, address: int, features: int) -> np.ndarray:
        """The [32, features] rows of one packed block operand."""
        return ob.unpack_activations(self.words(address, 32 * features), tokens=32, features=features)

    def put_block(self, address: int, rows) -> None:
        self.words(address, rows.size)[:] = ob.pack_activations(np.asarray(rows, np.float32))

    # -- launches ---------------------------------------------------------------------------------------------------
    def minitpuLaunchKernel(self, kbin_addr: int, kbin_size: int, *, args=None) -> None:  # noqa: N802
        head = self.memory[self._span(kbin_addr, 64)].tobytes()
        words = struct.unpack("<12I2f2I", head)
        if words[0] != 0x49324254:
            raise RuntimeError("not an image descriptor")
        kind, fields, scalars = KINDS[words[2]], words[4:12], words[12:14]
        args = list(args or []) + [0] * 4
        self.launches.append(kind)
        getattr(self, "_" + kind)(fields, scalars, *args[:4])

    def _halt(self, *_):
        pass

    def _gemm_bias(self, f, _s, a, w, drain, bias):
        depth, columns, activate = f[0], f[1], bool(f[2])
        x = self.block(a, depth)
        weights = ob.unpack_activations(self.words(w, depth * columns), tokens=depth, features=columns)
        b = self.floats(bias, columns * 4).reshape(-1, 4, 16)[:, 0, :].reshape(-1)
        if self.memory[self._span(drain, 512)].any():
            raise AssertionError("the drain's clearing tile is not zero")
        self.put_block(drain + 512, ob.bf16_grid(orf.gemm_f64(x, weights, bias=b, activate=activate)))

    _gemm = _gemm_bias

    def _add(self, f, _s, left, right, out, _unused=0):
        features = f[0]
        self.put_block(out, self.block(left, features) + self.block(right, features))

    def _add_bias(self, f, _s, left, bias, out, _unused=0):
        features = f[0]
        b = self.floats(bias, features * 4).reshape(-1, 4, 16)[:, 0, :].reshape(-1)
        self.put_block(out, self.block(left, features) + b)

    def _layernorm(self, f, _s, rows, constants, out, _unused=0):
        features = f[0]
        c = self.floats(constants, 2 * features)
        self.put_block(out, ob.bf16_grid(orf.layernorm_f64(self.block(rows, features), c[:features], c[features:])))

    def _fused_rows(self, address: int, tokens: int, width: int) -> np.ndarray:
        stride = 512 + 32 * 3 * width * 2
        return np.concatenate([self.block(address + b * stride, 3 * width) for b in range(tokens // 32)])

    def _attention(self, f, _s, _constants, _zero, fused, _unused=0):
        tokens, heads, head = f[0], f[1], f[2]
        width = heads * head
        rows = self._fused_rows(fused, tokens, width)
        out = np.concatenate([orf.causal_attention_f64(rows[:, h * head:(h + 1) * head],
                                                       rows[:, width + h * head:width + (h + 1) * head],
                                                       rows[:, 2 * width + h * head:2 * width + (h + 1) * head])
                              for h in range(heads)], axis=1)
        stride = 512 + 32 * 3 * width * 2
        for b in range(tokens // 32):
            block = self.block(fused + b * stride, 3 * width)
            block[:, :width] = ob.bf16_grid(out[b * 32:(b + 1) * 32])
            self.put_block(fused + b * stride, block)

    def _decode_attention(self, f, _s, constants, cache, fused, _unused=0):
        keys, heads, head, stated = f[0], f[1], f[2], f[3]
        width = heads * head
        masks = self.floats(constants + (2 + stated) * 512, keys * 16).reshape(keys // 16, 16, 16)
        key_mask = masks[:, :, 0].reshape(-1)    # keys on the tile rows: every query column alike
        stride = 512 + 32 * 2 * width * 2
        held = np.concatenate([self.block(cache + b * stride, 2 * width) for b in range(keys // 32)])
        block = self.block(fused, 3 * width)
        for h in range(heads):
            q = block[:16, h * head:(h + 1) * head]
            k = held[:, h * head:(h + 1) * head]
            v = held[:, width + h * head:width + (h + 1) * head]
            block[:16, h * head:(h + 1) * head] = ob.bf16_grid(
                orf.attention_f64(q, k, v, mask=np.broadcast_to(key_mask, (16, keys))))
        self.put_block(fused, block)

    def _copy(self, f, _s, source, _zero, destination, _unused=0):
        rows, stride = f[0], f[1]
        for r in range(rows):
            self.memory[self._span(destination + r * stride, 32)] = self.memory[self._span(source + r * stride, 32)]
