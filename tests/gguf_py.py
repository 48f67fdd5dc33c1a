"""A tiny independent GGUF reader for host-side tests (header, scalar metadata, tensor infos)."""
import struct

import numpy as np

_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}
TYPE_INFO = {0: (1, 4), 1: (1, 2), 8: (32, 34), 14: (256, 210), 30: (1, 2)}


class Reader:
    def __init__(self, path):
        self.buf = memoryview(open(path, "rb").read())
        self.p = 0
        magic, self.version, nt, nkv = struct.unpack_from("<IIQQ", self.buf, 0)
        assert magic == 0x46554747, "bad magic"
        self.p = 24
        self.meta = {}
        self.types = {}
        self.arrays = {}
        for _ in range(nkv):
            k = self._str()
            t = self._u32()
            if t == 9:
                at = self._u32()
                n = self._u64()
                vals = [self._val(at) for _ in range(n)]
                self.arrays[k] = vals
            else:
                self.meta[k] = self._val(t)
            self.types[k] = t
        self.tensors = {}
        for _ in range(nt):
            name = self._str()
            nd = self._u32()
            dims = [self._u64() for _ in range(nd)]
            ty = self._u32()
            off = self._u64()
            self.tensors[name] = (dims, ty, off)
        align = self.meta.get("general.alignment", 32)
        self.data_start = (self.p + align - 1) // align * align

    def _u32(self):
        v = struct.unpack_from("<I", self.buf, self.p)[0]
        self.p += 4
        return v

    def _u64(self):
        v = struct.unpack_from("<Q", self.buf, self.p)[0]
        self.p += 8
        return v

    def _str(self):
        n = self._u64()
        s = bytes(self.buf[self.p:self.p + n]).decode()
        self.p += n
        return s

    def _val(self, t):
        if t == 8:
            return self._str()
        fmt = _SCALAR[t]
        v = struct.unpack_from(fmt, self.buf, self.p)[0]
        self.p += struct.calcsize(fmt)
        return v

    def tensor_bytes(self, name):
        dims, ty, off = self.tensors[name]
        n = int(np.prod(dims))
        bs, ts = TYPE_INFO[ty]
        nb = (n + bs - 1) // bs * ts
        start = self.data_start + off
        return bytes(self.buf[start:start + nb])
