"""GGUF files through the library's reader (ef_gguf_*, csrc/gguf.cu): the
host side of the reference's js/gguf.js parseGGUF -- metadata, the tensor
table, and weights loaded from the file mapping into device tiles."""
from __future__ import annotations

import ctypes
import struct

from . import formats
from ._lib import EfError, check, lib

VALUE_FORMATS = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q",
                 12: "<d"}


class GGUFTensor:
    def __init__(self, index, name, type_id, dims, file_offset, nbytes):
        self.index, self.name, self.type_id, self.dims = index, name, type_id, dims
        self.file_offset, self.nbytes = file_offset, nbytes

    @property
    def k(self):
        return self.dims[0]

    @property
    def rows(self):
        r = 1
        for d in self.dims[1:]:
            r *= d
        return r


class GGUFFile:
    """An opened GGUF file (memory-mapped by the library)."""

    def __init__(self, path: str):
        L = lib()
        self.h = ctypes.c_void_p()
        err = ctypes.create_string_buffer(512)
        rc = L.ef_gguf_open(str(path).encode(), ctypes.byref(self.h), err, 512)
        if rc < 0:
            raise EfError(rc, err.value.decode(errors="replace"))
        v, a, ds = ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_uint64()
        nt, nm = ctypes.c_int64(), ctypes.c_int64()
        check(L.ef_gguf_header(self.h, ctypes.byref(v), ctypes.byref(a), ctypes.byref(ds), ctypes.byref(nt),
                               ctypes.byref(nm)))
        self.version, self.alignment, self.data_start = v.value, a.value, ds.value
        self.tensors = []
        for i in range(nt.value):
            name, ty, nd = ctypes.c_char_p(), ctypes.c_int(), ctypes.c_int()
            dims = (ctypes.c_int64 * 4)()
            off, nb = ctypes.c_uint64(), ctypes.c_uint64()
            check(L.ef_gguf_tensor(self.h, i, ctypes.byref(name), ctypes.byref(ty), ctypes.byref(nd), dims,
                                   ctypes.byref(off), ctypes.byref(nb)))
            self.tensors.append(GGUFTensor(i, name.value.decode(), ty.value, [dims[j] for j in range(max(nd.value, 1))],
                                           off.value, nb.value))
        self.by_name = {t.name: t for t in self.tensors}
        self.meta = {}
        for i in range(nm.value):
            key, ty, et, cnt, val = ctypes.c_char_p(), ctypes.c_int(), ctypes.c_int(), ctypes.c_uint64(), \
                ctypes.c_void_p()
            check(L.ef_gguf_meta(self.h, i, ctypes.byref(key), ctypes.byref(ty), ctypes.byref(et), ctypes.byref(cnt),
                                 ctypes.byref(val)))
            self.meta[key.value.decode()] = self._value(ty.value, et.value, cnt.value, val.value)

    @staticmethod
    def _value(ty, et, cnt, ptr):
        if ty == 8:
            return ctypes.string_at(ptr, cnt).decode(errors="replace")
        if ty == 9:
            if et == 8:
                return ("string[]", cnt)          # string arrays are not decoded
            fmt = VALUE_FORMATS[et]
            size = struct.calcsize(fmt)
            raw = ctypes.string_at(ptr, cnt * size)
            return [struct.unpack_from(fmt, raw, j * size)[0] for j in range(cnt)]
        return struct.unpack(VALUE_FORMATS[ty], ctypes.string_at(ptr, struct.calcsize(VALUE_FORMATS[ty])))[0]

    def tensor_bytes(self, name: str) -> bytes:
        t = self.by_name[name]
        return ctypes.string_at(lib().ef_gguf_tensor_data(self.h, t.index), t.nbytes)

    def load_weight(self, ops, name: str):
        """The tensor as a weight on ops' device (QuantOps.load_weight's Weight)."""
        from .ops import Weight
        t = self.by_name[name]
        h = ops.ctx.bind()
        w = ctypes.c_void_p()
        check(lib().ef_gguf_load_weight(h, self.h, name.encode(), ctypes.byref(w)), h)
        return Weight(ops.ctx, w, formats.type_name(t.type_id), t.rows, t.k, label=name)

    def close(self):
        if getattr(self, "h", None) is not None and self.h.value:
            lib().ef_gguf_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
