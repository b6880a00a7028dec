"""Host mirror of the reference's quantized operator API on the CUDA library.

`QuantOps` has the surface of `createQuantOps(device, {ctx, ...})`
(js/ops.js:748-1142): ``dequant``, ``matmul``, ``prepare``, ``upload``, ``ctx``,
``gemv.{matmul, gateUp, secciones, despachados, rechazados, conMarca}`` and
``gemm2.{plan, olvida, matmul, reproducible, cola}``, with the same argument
meaning, the same output layout (f32 ``[tokens][rows]``) and the same error
behaviour: an unsupported type, a bad ``k`` or a weight that does not match the
call raises; ``gemv``/``gemm2`` return ``None`` when their path does not apply
(js/ops.gemv.js:13-21, js/ops.gemm2.js:5-8).

Device memory and streams are torch's: activations and outputs are CUDA
tensors, and every launch goes on torch's current stream. The arithmetic is
the CUDA library's; nothing here computes on the host.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import formats
from ._lib import EF_NOT_APPLICABLE, EfError, check, lib

MAX_GEMV_TOKENS = 16


class Context:
    """A library context bound to one CUDA device (createContext, js/ops.js:134)."""

    def __init__(self, device: int = 0):
        self.device = int(device)
        h = ctypes.c_void_p()
        torch.cuda.init()
        rc = lib().ef_ctx_create(self.device, ctypes.byref(h))
        if rc < 0:
            raise EfError(rc, f"cannot create a context on cuda:{self.device}")
        self.h = h
        self._stream = None     # the stream last handed to the library (only bind() sets it)

    def bind(self):
        """Queue subsequent library work on torch's current stream of this device."""
        s = torch.cuda.current_stream(self.device).cuda_stream
        if s != self._stream:
            lib().ef_ctx_set_stream(self.h, ctypes.c_void_p(s))
            self._stream = s
        return self.h

    def sync(self):
        check(lib().ef_stream_sync(self.h), self.h)

    def close(self):
        if getattr(self, "h", None):
            lib().ef_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Weight:
    """A weight tensor repacked on the device (the loader's R buffer + mark,
    js/repack.js:241-306). ``size`` is the GGUF byte size, like GPUBuffer.size."""

    def __init__(self, ctx: Context, handle, type_name: str, rows: int, k: int, label: str = ""):
        self.ctx, self.h, self.type, self.rows, self.k, self.label = ctx, handle, type_name, rows, k, label
        self.size = formats.tensor_bytes(type_name, rows, k)

    def unpack(self) -> torch.Tensor:
        """The original GGUF bytes, rebuilt on the device (vuelveAlGGUF, js/repack.js:201-219)."""
        out = torch.empty(self.size, dtype=torch.uint8, device=f"cuda:{self.ctx.device}")
        h = self.ctx.bind()
        check(lib().ef_weight_unpack(h, self.h, ctypes.c_void_p(out.data_ptr())), h)
        return out

    def free(self):
        if self.h:
            lib().ef_weight_free(self.ctx.h, self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def _ptr(t: torch.Tensor):
    return ctypes.c_void_p(t.data_ptr())


class GemvOps:
    """quant.gemv (js/ops.gemv.js:44-221)."""

    def __init__(self, ops: "QuantOps"):
        self._ops = ops
        self._hechos = {"matmul": 0, "gateUp": 0, "secciones": 0}
        self.conMarca = True   # every weight carries its type and shape (the loader's mark)

    def _x(self, x, k, tokens):
        return self._ops._activations(x, k, tokens)

    def matmul(self, tipo, w, x, rows, k, tokens=1):
        if not (1 <= tokens <= MAX_GEMV_TOKENS):
            return None
        self._ops._check_weight(tipo, w, rows, k)
        xs = self._x(x, k, tokens)
        y = torch.empty((tokens, w.rows), dtype=torch.float32, device=xs.device)
        h = self._ops.ctx.bind()
        rc = check(lib().ef_gemv(h, w.h, _ptr(xs), tokens, _ptr(y)), h)
        if rc == EF_NOT_APPLICABLE:
            return None
        self._hechos["matmul"] += 1
        return y if rows == w.rows else y[:, :rows].contiguous()

    def gateUp(self, tipo, wg, wu, x, rows, k, tokens=1):
        if not (1 <= tokens <= MAX_GEMV_TOKENS):
            return None
        self._ops._check_weight(tipo, wg, rows, k)
        self._ops._check_weight(tipo, wu, rows, k)
        if wg.rows != wu.rows:
            return None
        xs = self._x(x, k, tokens)
        y = torch.empty((tokens, wg.rows), dtype=torch.float32, device=xs.device)
        h = self._ops.ctx.bind()
        rc = check(lib().ef_gemv_swiglu(h, wg.h, wu.h, _ptr(xs), tokens, _ptr(y)), h)
        if rc == EF_NOT_APPLICABLE:
            return None
        self._hechos["gateUp"] += 1
        return y if rows == wg.rows else y[:, :rows].contiguous()

    def secciones(self, tipo, ws, x, filas, k, tokens=1):
        n = len(ws)
        if n < 2 or n > 4 or len(filas) != n or not (1 <= tokens <= MAX_GEMV_TOKENS):
            return None
        for w, f in zip(ws, filas):
            self._ops._check_weight(tipo, w, f, k)
        xs = self._x(x, k, tokens)
        ys = [torch.empty((tokens, w.rows), dtype=torch.float32, device=xs.device) for w in ws]
        wh = (ctypes.c_void_p * n)(*[w.h.value for w in ws])
        yh = (ctypes.c_void_p * n)(*[y.data_ptr() for y in ys])
        h = self._ops.ctx.bind()
        rc = check(lib().ef_gemv_sections(h, wh, n, _ptr(xs), tokens, yh), h)
        if rc == EF_NOT_APPLICABLE:
            return None
        self._hechos["secciones"] += 1
        return [y if f == w.rows else y[:, :f].contiguous() for y, w, f in zip(ys, ws, filas)]

    def despachados(self):
        """Launches made per operation: proof that this path really ran."""
        return dict(self._hechos)

    def rechazados(self):
        """Kernel keys a compiler rejected (always empty: kernels are prebuilt)."""
        return []


class Gemm2Ops:
    """quant.gemm2 (js/ops.gemm2.js:143-304): prefill GEMM on the tensor cores."""

    def __init__(self, ops: "QuantOps"):
        self._ops = ops

    @staticmethod
    def plan(type, rows, k, tokens):
        """Pure planner (no device): the path a call would take, or None when
        the GEMV covers it (tokens <= 16) or the type has no kernel."""
        name = formats.type_name(type)
        if name not in formats.HOT_TYPES or tokens <= MAX_GEMV_TOKENS:
            return None
        be, _ = formats.block_info(name)
        if k % be:
            return None
        return {"via": "gemm", "type": name, "bpr": k // be, "tokens": tokens}

    def olvida(self):
        """The reference drops its x->f16 memo here; the library converts per call."""

    def matmul(self, type, w, x, rows, k, tokens, x_f16: bool = False):
        if self.plan(type, rows, k, tokens) is None:
            return None
        self._ops._check_weight(type, w, rows, k)
        if x_f16:
            xs = x.reshape(tokens, k).contiguous()
            assert xs.dtype == torch.float16
            xt = formats.type_id("F16")
        else:
            xs = self._ops._activations(x, k, tokens)
            xt = formats.type_id("F32")
        y = torch.empty((tokens, w.rows), dtype=torch.float32, device=xs.device)
        h = self._ops.ctx.bind()
        rc = check(lib().ef_gemm(h, w.h, _ptr(xs), xt, tokens, _ptr(y), 0), h)
        if rc == EF_NOT_APPLICABLE:
            return None
        return y if rows == w.rows else y[:, :rows].contiguous()

    def reproducible(self, type, rows, k, lote):
        return self.plan(type, rows, k, lote) is not None

    def status(self):
        """Synchronizes and raises EfError (EF_ERR_TIMEOUT) if a GEMM since the
        last check gave up on a bounded pipeline wait (its output is invalid)."""
        h = self._ops.ctx.bind()
        check(lib().ef_gemm_status(h), h)

    def cola(self, type, w, x1, rows, k, lote):
        """One token with the batch's kernel (js/ops.gemm2.js:294-302)."""
        if self.plan(type, rows, k, lote) is None:
            return None
        self._ops._check_weight(type, w, rows, k)
        xs = self._ops._activations(x1, k, 1)
        y = torch.empty((1, w.rows), dtype=torch.float32, device=xs.device)
        h = self._ops.ctx.bind()
        check(lib().ef_gemm(h, w.h, _ptr(xs), formats.type_id("F32"), 1, _ptr(y), 0), h)
        return y if rows == w.rows else y[:, :rows].contiguous()


class QuantOps:
    """createQuantOps (js/ops.js:748): quantized operators on one CUDA device."""

    def __init__(self, device: int = 0, ctx: Context | None = None):
        self.ctx = ctx or Context(device)
        self.device = torch.device(f"cuda:{self.ctx.device}")
        self.gemv = GemvOps(self)
        self.gemm2 = Gemm2Ops(self)

    # -- weights (the loader side: creaBufferR / writeBuffer, js/model.js:312-329)
    def load_weight(self, type, raw, rows: int, k: int, label: str = "") -> Weight:
        name = formats.type_name(type)
        if name not in formats.HOT_TYPES:
            raise EfError(-2, f"tipo de cuantización no soportado: «{name}»")
        need = formats.tensor_bytes(name, rows, k)
        h = ctypes.c_void_p()
        c = self.ctx.bind()
        if isinstance(raw, torch.Tensor) and raw.is_cuda:
            if raw.numel() * raw.element_size() < need:
                raise EfError(-7, f"{label or name}: {raw.numel()} bytes < {need}")
            check(lib().ef_weight_load_device(c, formats.type_id(name), _ptr(raw), rows, k, ctypes.byref(h)), c)
        else:
            a = np.ascontiguousarray(np.asarray(raw, dtype=np.uint8).reshape(-1))
            if a.size < need:
                raise EfError(-7, f"{label or name}: {a.size} bytes < {need}")
            check(lib().ef_weight_load(c, formats.type_id(name), a.ctypes.data_as(ctypes.c_void_p), rows, k,
                                       ctypes.byref(h)), c)
        return Weight(self.ctx, h, name, rows, k, label)

    def load_weight_slice(self, type, raw, rows, k, row0, nrows, k0, nk, label="") -> Weight:
        """The (row0:+nrows, k0:+nk) shard of a host tensor (one tensor-parallel rank)."""
        name = formats.type_name(type)
        a = np.ascontiguousarray(np.asarray(raw, dtype=np.uint8).reshape(-1))
        h = ctypes.c_void_p()
        c = self.ctx.bind()
        check(lib().ef_weight_load_slice(c, formats.type_id(name), a.ctypes.data_as(ctypes.c_void_p), rows, k,
                                         row0, nrows, k0, nk, ctypes.byref(h)), c)
        return Weight(self.ctx, h, name, nrows, nk, label)

    def load_weight_shard(self, type, raw, rows, k, axis, rank, nranks, label="") -> Weight:
        """Rank `rank` of `nranks`'s shard of a host tensor: axis 0 splits the output
        rows (column-parallel), axis 1 the input columns (row-parallel); even splits only."""
        name = formats.type_name(type)
        a = np.ascontiguousarray(np.asarray(raw, dtype=np.uint8).reshape(-1))
        h = ctypes.c_void_p()
        c = self.ctx.bind()
        check(lib().ef_weight_load_shard(c, formats.type_id(name), a.ctypes.data_as(ctypes.c_void_p), rows, k,
                                         axis, rank, nranks, ctypes.byref(h)), c)
        return Weight(self.ctx, h, name, rows // nranks if axis == 0 else rows, k // nranks if axis == 1 else k,
                      label)

    def _check_weight(self, tipo, w: Weight, rows, k):
        name = formats.type_name(tipo)
        if name not in formats.HOT_TYPES:
            raise EfError(-2, f"tipo de cuantización no soportado: «{name}»")
        be, _ = formats.block_info(name)
        if k % be:
            raise EfError(-3, f"matmul {name}: k={k} no es múltiplo de {be}")
        if not isinstance(w, Weight) or w.type != name or w.k != k or not (1 <= rows <= w.rows):
            got = f"{getattr(w, 'type', w.__class__.__name__)} {getattr(w, 'rows', '?')}x{getattr(w, 'k', '?')}"
            raise EfError(-6, f"{name}: the weight ({got}) does not serve rows={rows} k={k}")

    def _activations(self, x, k, tokens):
        n = tokens * k
        if (isinstance(x, torch.Tensor) and x.is_cuda and x.dtype == torch.float32 and x.numel() == n
                and x.is_contiguous()):
            return x.view(tokens, k)       # already the operand: no copy, no reshape chain
        if not isinstance(x, torch.Tensor):
            x = torch.as_tensor(np.asarray(x, np.float32))
        if x.dtype != torch.float32:
            raise EfError(-1, f"activations must be f32, got {x.dtype}")
        if x.numel() < tokens * k:
            raise EfError(-7, f"activations hold {x.numel()} values < tokens*k = {tokens * k}")
        x = x.reshape(-1)[: tokens * k].reshape(tokens, k)
        if not x.is_cuda:
            x = x.to(self.device)
        return x.contiguous()

    # -- the quant operator surface --------------------------------------
    def dequant(self, type, w: Weight, nBlocks: int) -> torch.Tensor:
        """Whole rows to f32, bit-exact (js/ops.js:813-823). nBlocks must cover whole rows."""
        name = formats.type_name(type)
        self._check_weight(name, w, w.rows, w.k)
        be, _ = formats.block_info(name)
        bpr = w.k // be
        if nBlocks % bpr or not (0 < nBlocks <= w.rows * bpr):
            raise EfError(-7, f"dequant: {nBlocks} blocks is not a whole number of rows of {bpr} blocks")
        nrows = nBlocks // bpr
        out = torch.empty(nBlocks * be, dtype=torch.float32, device=self.device)
        h = self.ctx.bind()
        check(lib().ef_dequant(h, w.h, 0, nrows, _ptr(out)), h)
        return out

    def gather(self, type, w: Weight, ids, dim: int, tokens: int) -> torch.Tensor:
        """Rows of a quantized table to f32, out[t] = dequant(W)[ids[t]] (js/ops.js:1104-1118, the
        embedding lookup): f32 [tokens][dim], bit-exact; an id outside the table's rows gives a
        zero row. dim must be the row length and a whole number of blocks, as in the reference."""
        name = formats.type_name(type)
        be, _ = formats.block_info(name)
        if dim % be:
            raise EfError(-3, f"gather {name}: dim={dim} is not a multiple of {be}")
        self._check_weight(name, w, w.rows, dim)
        if tokens < 1:
            raise EfError(-3, f"gather: tokens={tokens}")
        ids = torch.as_tensor(ids).reshape(-1)[:tokens].to(self.device, torch.int32).contiguous()
        if ids.numel() < tokens:
            raise EfError(-7, f"gather: {ids.numel()} ids < tokens = {tokens}")
        out = torch.empty((tokens, dim), dtype=torch.float32, device=self.device)
        h = self.ctx.bind()
        check(lib().ef_gather(h, w.h, _ptr(ids), tokens, _ptr(out)), h)
        return out

    def matmul(self, type, w: Weight, x, rows: int, k: int, tokens: int = 1) -> torch.Tensor:
        """Y[tokens][rows] = dequant(W) . X (js/ops.js:827-1101): GEMV up to 16 tokens,
        tensor-core GEMM above."""
        if tokens < 1:
            raise EfError(-3, f"matmul: tokens={tokens}")
        if tokens <= MAX_GEMV_TOKENS:
            y = self.gemv.matmul(type, w, x, rows, k, tokens)
        else:
            y = self.gemm2.matmul(type, w, x, rows, k, tokens)
        if y is None:   # not reachable for the hot-path types; kept for the contract
            raise EfError(-2, f"matmul {formats.type_name(type)}: no kernel for tokens={tokens}")
        return y

    def prepare(self, types):
        """Tables of the i-quants are compiled into the library: only validate."""
        for t in set(types):
            if formats.type_name(t) not in formats.HOT_TYPES:
                raise EfError(-2, f"tipo de cuantización no soportado: «{t}»")

    def upload(self, array, label="x") -> torch.Tensor:
        return torch.as_tensor(np.asarray(array)).to(self.device)

    def sync(self):
        self.ctx.sync()


def createQuantOps(device: int = 0, opts: dict | None = None) -> QuantOps:
    """Factory with the reference's name (js/ops.js:748)."""
    opts = opts or {}
    return QuantOps(device, ctx=opts.get("ctx"))
