"""The `B200` backend: the host-side mirror of furiosa-opt-std's `Backend` trait
(furiosa-opt-std/src/backend/mod.rs:41-248) over libfopt_b200.so.

`Cpu` delegates every op to `BufStorage` (furiosa-opt-std/src/backend/cpu.rs:18-158); `B200`
delegates to the CUDA kernels through the C ABI. The storage is the same packed byte image
(`Storage` below owns one device allocation), so `into_buf` / `from_buf` are plain copies and
equality is byte equality (storage/buf.rs:38-41). Method names, argument meaning and error
behaviour follow the trait: an ill-formed mapping raises `FoptError`, where the reference panics.

Closures become opcodes: `map` / `zip_with` / `zip3_with` / `reduce` take a program from `ops`
(or a reduce opcode) instead of a Rust closure.
"""
from __future__ import annotations

import ctypes as C
import os
import weakref
from typing import Optional, Sequence

import numpy as np

from . import _lib, dtypes, ops, rowfuse
from ._lib import check

REDUCE_OPS = _lib.REDUCE_OPS


class Mapping:
    """A parsed mapping expression (`furiosa_mapping::Mapping`). `axes` declares symbol sizes, e.g.
    Mapping("[A / 8, B % 4 # 16]", A=64, B=16)."""

    def __init__(self, expr: str, axes: Optional[dict] = None, **kw):
        decl = dict(axes or {})
        decl.update(kw)
        self.expr = expr
        self.axes = decl
        h = C.c_void_p()
        check(_lib.lib().fopt_mapping_parse(", ".join(f"{k}={v}" for k, v in decl.items()).encode(), expr.encode(),
                                            C.byref(h)))
        self._h = h

    @property
    def handle(self):
        return self._h

    @property
    def size(self) -> int:
        return int(_lib.lib().fopt_mapping_size(self._h))

    def eval(self, pos: int):
        """`M::map(pos)`: (status, {axis: coord}); status 0 live, 1 + PaddingKind padding, -1 OOB."""
        n = len(self.axes)
        buf = (C.c_int64 * max(n, 1))()
        st = _lib.lib().fopt_mapping_eval(self._h, pos, buf, n)
        return st, {k: int(buf[i]) for i, k in enumerate(self.axes)}

    def flat_shape(self) -> list:
        """The pair-split sizes (`flat_shape`, tensor/memory.rs:201-209) a loaded tensor must have."""
        dims, n = (C.c_int64 * 32)(), C.c_int32()
        check(_lib.lib().fopt_mapping_flat_shape(self.handle, dims, 32, C.byref(n)))
        return [dims[k] for k in range(min(n.value, 32))]

    def window_base(self, offset: dict) -> int:
        out = C.c_int64()
        check(_lib.lib().fopt_window_base(self._h, ", ".join(f"{k}:{v}" for k, v in offset.items()).encode(),
                                          C.byref(out)))
        return int(out.value)

    def __repr__(self):
        return f"m![{self.expr}]"

    def __del__(self):
        try:
            if self._h:
                _lib.lib().fopt_mapping_free(self._h)
        except Exception:
            pass


def m(expr: str, **axes) -> Mapping:
    return Mapping(expr, axes)


ST_DTYPES = {"BF16": "bf16", "F32": "f32", "I8": "i8", "I16": "i16", "I32": "i32", "F8_E4M3": "f8e4m3",
             "F8_E5M2": "f8e5m2"}


class SafeTensors:
    """An open safetensors file (header parsed natively; tensors stream to the device on demand)."""

    def __init__(self, path: str):
        h = C.c_void_p()
        check(_lib.lib().fopt_st_open(os.fsencode(path), C.byref(h)))
        self.handle = h
        self.path = path

    def __len__(self):
        return _lib.lib().fopt_st_count(self.handle)

    def info(self, index: int):
        name, dt, nd, nb = C.c_char_p(), C.c_char_p(), C.c_int32(), C.c_int64()
        shape = (C.c_int64 * 16)()
        check(_lib.lib().fopt_st_info(self.handle, index, C.byref(name), C.byref(dt), C.byref(nd), shape, 16,
                                      C.byref(nb)))
        return name.value.decode(), dt.value.decode(), [shape[k] for k in range(nd.value)], nb.value

    def names(self):
        return [self.info(k)[0] for k in range(len(self))]

    def index(self, name: str) -> int:
        i = C.c_int32()
        check(_lib.lib().fopt_st_find(self.handle, name.encode(), C.byref(i)))
        return i.value

    def close(self):
        if self.handle:
            _lib.lib().fopt_st_close(self.handle)
            self.handle = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Storage:
    """`B200::Storage<D>`: one owned device allocation holding the packed image of `n` elements.

    A storage made by `B200.relayout` as a plain broadcast (one value per row, or one row repeated)
    is lazy: it holds only the small source until something needs its bytes. Elementwise ops read
    the source directly with the broadcast index; any other use (its device pointer) writes the
    broadcast out first, so the observable image is always the relayout's."""

    def __init__(self, backend: "B200", dtype: str, n: int, zero: bool = True, lazy=None):
        self.backend = backend
        self.dtype = dtype
        self.n = n
        self.nbytes = dtypes.nbytes(dtype, n)
        self._ptr = C.c_void_p()
        # lazy: ("bcast", src Storage, Src Mapping, Dst Mapping, bcast code of fopt_elementwise_bcast)
        #    or ("ew", program, leaf inputs, origin): values not yet written (leaves may be lazy
        #       broadcasts; origin = (program, inputs) of the op that made it, before composition)
        #    or ("red", src Storage, op, identity bits, Src, Dst, rows, row length): a plain row
        #       reduction of a deferred elementwise value, not yet run
        self.lazy = lazy
        self._dependents = weakref.WeakSet()  # lazy storages that read this one
        if lazy is None:
            self._alloc(zero)
        else:
            for src in self._lazy_sources():
                src._dependents.add(self)

    def _lazy_sources(self):
        if self.lazy is None:
            return []
        return list(self.lazy[2]) if self.lazy[0] == "ew" else [self.lazy[1]]

    def _will_write(self) -> None:
        """Called before anything writes into this storage in place: lazy storages that read it
        take their values now."""
        for d in list(self._dependents):
            d.ptr  # noqa: B018 (materialises)
        self._dependents = weakref.WeakSet()

    def _alloc(self, zero: bool):
        p = C.c_void_p()
        alloc = _lib.lib().fopt_alloc if zero else _lib.lib().fopt_alloc_uninit
        check(alloc(self.backend.ctx, self.nbytes, C.byref(p)), self.backend.ctx)
        self._ptr = p
        # allocated while a step is being captured: the graph owns the memory once the capture ends
        self._capture = getattr(self.backend, "_capturing", None)

    @property
    def ptr(self) -> C.c_void_p:
        if self.lazy is not None:
            lazy, self.lazy = self.lazy, None
            if lazy[0] == "bcast":
                _, src, Src, Dst, _ = lazy
                self._alloc(True)
                check(_lib.lib().fopt_transpose(self.backend.ctx, self._ptr, src.ptr, _lib.DTYPES[src.dtype],
                                                Src.handle, Dst.handle, 0, 0, 1), self.backend.ctx)
            elif lazy[0] == "ew":
                _, prog, leaves, origin = lazy
                self._alloc(dtypes.BITS[self.dtype] == 4)
                self.backend._run_ew(prog, leaves, self, origin)
            else:
                _, src, op, bits, Src, Dst, _, _ = lazy
                self._alloc(False)
                self.backend._run_reduce(self, src, op, bits, Src, Dst)
        return self._ptr

    @property
    def addr(self) -> int:
        return self.ptr.value or 0

    def to_bytes(self) -> bytes:
        buf = (C.c_uint8 * self.nbytes)()
        check(_lib.lib().fopt_d2h(self.backend.ctx, buf, self.ptr, self.nbytes), self.backend.ctx)
        return bytes(buf)

    def to_numpy(self) -> np.ndarray:
        return dtypes.from_bytes(self.to_bytes(), self.dtype, self.n)

    def clone(self) -> "Storage":
        s = Storage(self.backend, self.dtype, self.n)
        check(_lib.lib().fopt_d2d(self.backend.ctx, s.ptr, self.ptr, self.nbytes), self.backend.ctx)
        return s

    def __eq__(self, other) -> bool:
        if not isinstance(other, Storage) or other.nbytes != self.nbytes:
            return False
        eq = C.c_int()
        check(_lib.lib().fopt_equal(self.backend.ctx, self.ptr, other.ptr, self.nbytes, C.byref(eq)), self.backend.ctx)
        return bool(eq.value)

    def __len__(self):
        return self.n

    __hash__ = object.__hash__  # identity: storages are tracked in sets of dependents

    def __del__(self):
        try:
            cap = getattr(self, "_capture", None)
            if cap is not None and getattr(self.backend, "_capturing", None) is not cap:
                return  # a graph's allocation (released by the graph)
            if self._ptr:
                _lib.lib().fopt_free(self.backend.ctx, self._ptr)
                self._ptr = C.c_void_p()
        except Exception:
            pass


class Graph:
    """A captured step (see `B200.capture`)."""

    def __init__(self, be: "B200", handle, outputs, token):
        self.be, self._h, self.outputs, self._token = be, handle, outputs, token

    def launch(self):
        check(_lib.lib().fopt_graph_launch(self.be.ctx, self._h), self.be.ctx)
        return self.outputs

    def close(self):
        if self._h:
            check(_lib.lib().fopt_graph_destroy(self.be.ctx, self._h), self.be.ctx)
            self._h = C.c_void_p()
            for o in (self.outputs if isinstance(self.outputs, tuple) else (self.outputs,)):
                o._ptr = C.c_void_p()  # released with the graph

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_COMPOSED = {}  # composition signature -> composed program (None: does not fit)


def _ep(kind=0, scale=None, axis=None, int_width=31, lo=-128, hi=127, row_scale=None, residual=None):
    e = _lib.Epilogue()
    e.row_scale = row_scale.addr if isinstance(row_scale, Storage) else (row_scale or 0)
    e.residual = residual.addr if isinstance(residual, Storage) else (residual or 0)
    e.kind = kind
    e.scale = scale.addr if isinstance(scale, Storage) else (scale or 0)
    e.scale_axis = axis.encode() if axis else None
    e.int_width, e.clip_lo, e.clip_hi = int_width, lo, hi
    return e


class B200:
    """The backend. One instance binds one GPU (`Backend::bind_device`, backend/mod.rs:246)."""

    def __init__(self, device: int = 0):
        ctx = C.c_void_p()
        check(_lib.lib().fopt_init(device, C.byref(ctx)))
        self.ctx = ctx
        self.device = device
        # write broadcasts out at relayout time instead of reading them lazily (for comparison)
        self.eager_broadcast = bool(os.environ.get("FOPT_EAGER_BROADCAST"))
        # engine-chain fusion of elementwise results (off: every op writes its result)
        self.fuse = not os.environ.get("FOPT_NO_FUSION")
        # row programs: a row reduction and the elementwise ops that read its broadcast result run as
        # one kernel per row (off: the reduction runs as its own kernel first)
        self.row_fusion = not os.environ.get("FOPT_NO_ROW_FUSION")
        self._capturing = None  # the open capture's token (see `capture`)

    # ---- CUDA graphs of whole steps ----
    def capture(self, fn) -> "Graph":
        """Records the device work of `fn()` (a step: a decoder block's forward, an MLP pass) into a
        CUDA graph instead of running it; `Graph.launch` replays it without the host work. `fn`
        returns a storage or a tuple of them: they are written inside the capture and hold each
        launch's results (same addresses every launch). Inputs are storages allocated before the
        capture: write new values into them between launches. Run `fn` once before capturing so
        its kernels are compiled and its workspaces sized."""
        if self._capturing is not None:
            raise RuntimeError("capture: a capture is already open")
        check(_lib.lib().fopt_capture_begin(self.ctx), self.ctx)
        token = object()
        self._capturing = token
        handle = C.c_void_p()
        try:
            outs = fn()
            for o in (outs if isinstance(outs, tuple) else (outs,)):
                o.ptr  # noqa: B018 (written inside the capture)
        finally:
            st = _lib.lib().fopt_capture_end(self.ctx, C.byref(handle))
            self._capturing = None
        check(st, self.ctx)
        return Graph(self, handle, outs, token)

    # ---- lifecycle (backend/mod.rs:45-90) ----
    def from_vec(self, mapping: Mapping, data, dtype: str) -> Storage:
        arr = np.asarray(data)
        if arr.size != mapping.size:
            raise ValueError(f"from_vec: {arr.size} values for a mapping of size {mapping.size}")
        return self.from_buf(mapping, dtypes.to_bytes(arr.reshape(-1), dtype), dtype)

    def from_buf(self, mapping: Mapping, buf: bytes, dtype: str) -> Storage:
        s = Storage(self, dtype, mapping.size)
        if len(buf) != s.nbytes:
            raise ValueError("from_buf: byte length does not match the mapping")
        host = (C.c_uint8 * len(buf)).from_buffer_copy(buf)
        check(_lib.lib().fopt_h2d(self.ctx, s.ptr, host, len(buf)), self.ctx)
        self.sync()
        return s

    def from_safetensors(self, st, name: str, mapping: Mapping, dtype: Optional[str] = None) -> Storage:
        """`HostTensor::from_safetensors(view).to_hbm()` (tensor/memory.rs:197-222) in one step: the
        tensor's shape must equal the mapping's pair-split sizes and its byte length the mapping's
        image; the bytes stream from the file into a new device storage."""
        own = isinstance(st, (str, bytes, os.PathLike))
        f = SafeTensors(st) if own else st
        try:
            i = f.index(name)
            _, st_dt, shape, nbytes = f.info(i)
            if st_dt not in ST_DTYPES:
                raise ValueError(f"from_safetensors: dtype {st_dt} is not a storage type")
            dt = ST_DTYPES[st_dt]
            if dtype is not None and dtype != dt:
                raise ValueError(f"from_safetensors: {name} is {dt}, not {dtype}")
            if shape != mapping.flat_shape():
                raise ValueError(f"from_safetensors: {name} has shape {shape}, the mapping {mapping.flat_shape()}")
            s = Storage(self, dt, mapping.size, zero=False)
            if nbytes != s.nbytes:
                raise ValueError(f"from_safetensors: {name} holds {nbytes} bytes, the mapping {s.nbytes}")
            check(_lib.lib().fopt_st_read(self.ctx, f.handle, i, s.ptr, nbytes), self.ctx)
            return s
        finally:
            if own:
                f.close()

    def zeroed(self, mapping: Mapping, dtype: str) -> Storage:
        return Storage(self, dtype, mapping.size)

    def into_vec(self, storage: Storage, mapping: Optional[Mapping] = None) -> np.ndarray:
        return storage.to_numpy()

    def into_buf(self, storage: Storage, mapping: Optional[Mapping] = None) -> bytes:
        return storage.to_bytes()

    def sync(self):
        check(_lib.lib().fopt_sync(self.ctx), self.ctx)

    def set_exact_fold(self, exact: bool):
        check(_lib.lib().fopt_set_exact_fold(self.ctx, int(exact)), self.ctx)
        self._exact_fold = bool(exact)

    @property
    def exact_fold(self) -> bool:
        """Whether f32 folds run in the reference's wire order (off by default)."""
        return getattr(self, "_exact_fold", False)

    @property
    def launches(self) -> int:
        return int(_lib.lib().fopt_launch_count(self.ctx))

    # ---- elementwise (backend/mod.rs:92-116) ----
    # Elementwise results of f32 / i32 type are deferred (engine-chain fusion): a deferred storage
    # keeps its program and leaf inputs; an elementwise consumer composes the program into its own,
    # a fused row reduction (`reduce`) folds the values without writing them, and any other use
    # writes them out first. Leaf inputs are ordinary storages or lazy broadcasts.
    DEFER = ("f32", "i32")
    MAX_LEAVES = 8

    @staticmethod
    def _leaf_args(leaves):
        """ctypes arrays (pointers, dtypes, bcast codes) for leaf inputs: a still-lazy broadcast is
        passed as its source with its code, anything else as itself."""
        srcs, codes = [], []
        for s in leaves:
            if s.lazy is not None and s.lazy[0] == "bcast":
                srcs.append(s.lazy[1])
                codes.append(s.lazy[4])
            else:
                srcs.append(s)
                codes.append(0)
        ptrs = (C.c_void_p * len(leaves))(*[s.addr for s in srcs])
        dts = (C.c_int * len(leaves))(*[_lib.DTYPES[s.dtype] for s in leaves])
        return ptrs, dts, (C.c_int64 * len(leaves))(*codes), any(codes)

    def _compose(self, prog, inputs: Sequence[Storage]):
        """Returns (program, leaves) with deferred elementwise inputs folded in, or None when the
        result would need more than 8 leaves, 32 instructions or 16 registers. More than 3 leaves
        run as a row program or through the origin (see `_run_ew`)."""
        leaves, keymap = [], {}

        def leaf_reg(st):
            if id(st) not in keymap:
                keymap[id(st)] = len(leaves)
                leaves.append(st)
            return keymap[id(st)]

        parts = []  # per consumer input: ("leaf", reg) or ("prog", program, [leaf regs])
        for s in inputs:
            if s.lazy is not None and s.lazy[0] == "ew":
                _, q, qleaves, _ = s.lazy
                parts.append(("prog", q, [leaf_reg(l) for l in qleaves]))
            else:
                parts.append(("leaf", leaf_reg(s)))
        if len(leaves) > self.MAX_LEAVES:
            return None
        # the composed program depends only on the programs and the leaf registers they read
        key = (bytes(prog), len(leaves),
               tuple((p[0], p[1]) if p[0] == "leaf" else (p[0], bytes(p[1]), tuple(p[2])) for p in parts))
        cache = _COMPOSED
        if key in cache:
            built = cache[key]
            return (built, leaves) if built is not None else None
        out = ops.Prog(len(leaves))
        regs = []
        try:
            for part in parts:
                regs.append(part[1] if part[0] == "leaf" else ops.inline(out, part[1], part[2]))
            built = out.build(ops.inline(out, prog, regs))
        except ValueError:
            built = None
        if len(cache) >= 4096:
            cache.clear()
        cache[key] = built
        return (built, leaves) if built is not None else None

    def _run_ew(self, prog, leaves, out: Storage, origin=None) -> None:
        if self.fuse and self.row_fusion and rowfuse.try_row_program(self, prog, leaves, out, origin):
            return
        if len(leaves) > 3:  # the generated kernels take 3 inputs: evaluate the deferred inputs first
            oprog, inputs = origin
            cprog, cleaves = self._compose(oprog, [self._force(s) if s.lazy is not None and s.lazy[0] == "ew" else s
                                                   for s in inputs])
            self._run_ew(cprog, cleaves, out)
            return
        ptrs, dts, codes, any_bcast = self._leaf_args(leaves)
        if any_bcast:
            st = _lib.lib().fopt_elementwise_bcast(self.ctx, C.byref(prog), len(leaves), ptrs, dts, codes, out._ptr,
                                                   _lib.DTYPES[out.dtype], out.n)
            if st == 0:
                return
            if st != _lib.FOPT_ERR_UNSUPPORTED:
                check(st, self.ctx)
            ptrs = (C.c_void_p * len(leaves))(*[s.addr for s in leaves])  # writes the broadcasts out
        check(_lib.lib().fopt_elementwise(self.ctx, C.byref(prog), len(leaves), ptrs, dts, out._ptr,
                                          _lib.DTYPES[out.dtype], out.n), self.ctx)

    def _ew(self, prog, inputs: Sequence[Storage], out_dtype: str) -> Storage:
        n = inputs[0].n
        for s in inputs:
            if s.n != n:
                raise ValueError("zip: operands must have the same element count")
        composed = self._compose(prog, inputs)
        if composed is None:  # evaluate the deferred inputs and run on their values
            composed = self._compose(prog, [self._force(s) if s.lazy is not None and s.lazy[0] == "ew" else s
                                            for s in inputs])
        cprog, leaves = composed
        origin = (prog, list(inputs))
        if self.fuse and out_dtype in self.DEFER:
            return Storage(self, out_dtype, n, lazy=("ew", cprog, leaves, origin))
        out = Storage(self, out_dtype, n, zero=dtypes.BITS[out_dtype] == 4)
        self._run_ew(cprog, leaves, out, origin)
        return out

    @staticmethod
    def _force(s: Storage) -> Storage:
        s.ptr  # noqa: B018 (materialises)
        return s

    def map(self, src: Storage, prog, out_dtype: str) -> Storage:
        return self._ew(prog, [src], out_dtype)

    def zip_with(self, a: Storage, b: Storage, prog, out_dtype: str) -> Storage:
        return self._ew(prog, [a, b], out_dtype)

    def zip3_with(self, a: Storage, b: Storage, c: Storage, prog, out_dtype: str) -> Storage:
        return self._ew(prog, [a, b, c], out_dtype)

    # ---- layout (backend/mod.rs:118-126, 208-218) ----
    def transpose(self, dst: Storage, src: Storage, Src: Mapping, Dst: Mapping, src_offset: Optional[dict] = None,
                  dst_offset: Optional[dict] = None, src_map: Optional[Mapping] = None,
                  dst_map: Optional[Mapping] = None, allow_broadcast: bool = False) -> None:
        if src.dtype != dst.dtype:
            raise ValueError("transpose: dtype mismatch")
        src_base = (src_map or Src).window_base(src_offset) if src_offset else 0
        dst_base = (dst_map or Dst).window_base(dst_offset) if dst_offset else 0
        dst._will_write()
        check(_lib.lib().fopt_transpose(self.ctx, dst.ptr, src.ptr, _lib.DTYPES[src.dtype], Src.handle, Dst.handle,
                                        src_base, dst_base, int(allow_broadcast)), self.ctx)

    def relayout(self, src: Storage, Src: Mapping, Dst: Mapping, allow_broadcast: bool = False) -> Storage:
        """A fresh Dst-laid-out copy (`Tensor::transpose(true)` on a zeroed destination). A plain
        broadcast of a byte-multiple type comes back lazy (see `Storage`)."""
        if allow_broadcast and dtypes.BITS[src.dtype] >= 8 and not self.eager_broadcast:
            kind, inner = C.c_int32(), C.c_int64()
            check(_lib.lib().fopt_broadcast_kind(Src.handle, Dst.handle, C.byref(kind), C.byref(inner)), None)
            if kind.value and inner.value % 8 == 0:
                code = inner.value if kind.value == 1 else -inner.value
                return Storage(self, src.dtype, Dst.size, lazy=("bcast", src, Src, Dst, code))
        dst = Storage(self, src.dtype, Dst.size)
        self.transpose(dst, src, Src, Dst, allow_broadcast=allow_broadcast)
        return dst

    def reshape(self, src: Storage, Src: Mapping, Dst: Mapping) -> Storage:
        if Src.size != Dst.size:
            raise ValueError("reshape: sizes differ")
        return src.clone()

    def transmute(self, storage: Storage, src_map: Mapping, dst_map: Mapping) -> Storage:
        if src_map.expr == dst_map.expr and src_map.axes == dst_map.axes:
            return storage
        out = Storage(self, storage.dtype, dst_map.size)
        check(_lib.lib().fopt_transmute(self.ctx, out.ptr, storage.ptr, _lib.DTYPES[storage.dtype], src_map.handle,
                                        dst_map.handle), self.ctx)
        return out

    def describe_relayout(self, Src: Mapping, Dst: Mapping, allow_broadcast: bool = False) -> str:
        buf = C.create_string_buffer(512)
        check(_lib.lib().fopt_describe_relayout(Src.handle, Dst.handle, int(allow_broadcast), buf, 512))
        return buf.value.decode()

    # ---- reduce (backend/mod.rs:128-133) ----
    def reduce(self, src: Storage, op: str, identity, Src: Mapping, Dst: Mapping,
               allow_broadcast: bool = False) -> Storage:
        """A row reduction of a deferred elementwise value comes back lazy when row programs are on:
        it runs when its value is needed, or inside the row program of a consumer of its broadcast."""
        if src.dtype == "i32":
            bits = int(np.int32(identity).view(np.uint32))
        elif src.dtype == "bf16":
            bits = int(np.uint32(dtypes.f32_to_bf16_bits(np.float32(identity))) << 16)
        else:
            bits = int(np.float32(identity).view(np.uint32))
        if (self.fuse and self.row_fusion and src.lazy is not None and src.lazy[0] == "ew" and not allow_broadcast
                and src.dtype in self.DEFER):
            rows, W = C.c_int64(), C.c_int64()
            st = _lib.lib().fopt_row_reduce_shape(self.ctx, Src.handle, Dst.handle, C.byref(rows), C.byref(W))
            if st == 0 and rows.value == Dst.size:
                return Storage(self, src.dtype, Dst.size,
                               lazy=("red", src, op, bits, Src, Dst, rows.value, W.value))
            if st not in (0, _lib.FOPT_ERR_UNSUPPORTED):
                check(st, self.ctx)
        out = Storage(self, src.dtype, Dst.size, zero=False)
        self._run_reduce(out, src, op, bits, Src, Dst, allow_broadcast)
        return out

    def _run_reduce(self, out: Storage, src: Storage, op: str, bits: int, Src: Mapping, Dst: Mapping,
                    allow_broadcast: bool = False) -> None:
        if src.lazy is not None and src.lazy[0] == "ew" and not allow_broadcast and len(src.lazy[2]) <= 3:
            _, prog, leaves, _ = src.lazy
            ptrs, dts, codes, _ = self._leaf_args(leaves)
            st = _lib.lib().fopt_reduce_map(self.ctx, out._ptr, C.byref(prog), len(leaves), ptrs, dts, codes,
                                            _lib.DTYPES[src.dtype], REDUCE_OPS[op], bits, Src.handle, Dst.handle)
            if st == 0:
                return
            if st != _lib.FOPT_ERR_UNSUPPORTED:
                check(st, self.ctx)
        check(_lib.lib().fopt_reduce(self.ctx, out._ptr, src.ptr, _lib.DTYPES[src.dtype], REDUCE_OPS[op], bits,
                                     Src.handle, Dst.handle, int(allow_broadcast)), self.ctx)

    # ---- contraction (backend/mod.rs:135-157) ----
    ACC = {"i8": "i32", "i4": "i32", "i5": "i32", "i9": "i32", "bf16": "f32", "f8e4m3": "f32", "f8e5m2": "f32"}

    def _contract(self, lhs, rhs, lhs_map, rhs_map, pre_reduce, out_map, out_dtype, ep=None, out=None) -> Storage:
        if lhs.dtype != rhs.dtype:
            raise ValueError("contraction: operand dtypes differ")
        if out is not None:
            out._will_write()
        if out is None:
            out = Storage(self, out_dtype, out_map.size, zero=False)
        elif out.dtype != out_dtype or out.n != out_map.size:
            raise ValueError("contraction: output storage does not match the output mapping")
        check(_lib.lib().fopt_contraction(self.ctx, out.ptr, _lib.DTYPES[out_dtype], lhs.ptr, rhs.ptr,
                                          _lib.DTYPES[lhs.dtype], lhs_map.handle, rhs_map.handle, pre_reduce.handle,
                                          out_map.handle, C.byref(ep) if ep is not None else None), self.ctx)
        return out

    def contraction(self, lhs, rhs, lhs_map, rhs_map, pre_reduce, out_map, out=None) -> Storage:
        """Accumulate wide, narrow once to the operand type (buf.rs:451-464). `out` optionally
        reuses an existing output storage."""
        return self._contract(lhs, rhs, lhs_map, rhs_map, pre_reduce, out_map, lhs.dtype, out=out)

    def contraction_prewidened(self, lhs, rhs, lhs_map, rhs_map, pre_reduce, out_map) -> Storage:
        """Operands already at accumulator width (i32 / f32) (buf.rs:468-481)."""
        if lhs.dtype not in ("i32", "f32"):
            raise ValueError("contraction_prewidened: operands must be i32 or f32")
        return self._contract(lhs, rhs, lhs_map, rhs_map, pre_reduce, out_map, lhs.dtype)

    def contraction_host(self, lhs, rhs, lhs_map, rhs_map, pre_reduce, out_map, in_dtype: str, out_dtype: str,
                         ep=None, out=None):
        """The contraction on host buffers (numpy arrays, or objects with `data_ptr()` such as pinned
        torch tensors): operands copied in, contracted and the result copied out in one pipelined
        call (`fopt_contraction_host`). Returns the result's bytes as a numpy uint8 array (or fills
        `out`). Asynchronous on the context's stream when `out` is given; synchronous otherwise."""
        def addr(x):
            return x.data_ptr() if hasattr(x, "data_ptr") else x.ctypes.data
        res = out if out is not None else np.empty(dtypes.nbytes(out_dtype, out_map.size), np.uint8)
        check(_lib.lib().fopt_contraction_host(self.ctx, addr(res), _lib.DTYPES[out_dtype], addr(lhs), addr(rhs),
                                               _lib.DTYPES[in_dtype], lhs_map.handle, rhs_map.handle,
                                               pre_reduce.handle, out_map.handle,
                                               C.byref(ep) if ep is not None else None), self.ctx)
        if out is None:
            self.sync()
        return res

    def contraction_wide(self, lhs, rhs, lhs_map, rhs_map, pre_reduce, out_map) -> Storage:
        """The engine's contract_outer widen + contract_lane fold in one op: narrow operands, wide
        (i32 / f32) output, without materialising the widened operand copies."""
        return self._contract(lhs, rhs, lhs_map, rhs_map, pre_reduce, out_map, self.ACC[lhs.dtype])

    def contraction_requant(self, lhs, rhs, lhs_map, rhs_map, pre_reduce, out_map, scale: Storage, scale_axis: str,
                            int_width: int = 31, lo: int = -128, hi: int = 127, out=None) -> Storage:
        """i8 x i8 -> i32 -> FxpToFp -> MulF(scale[axis]) -> FpToFxp -> Clip -> i8 commit, fused."""
        ep = _ep(1, scale, scale_axis, int_width, lo, hi)
        return self._contract(lhs, rhs, lhs_map, rhs_map, pre_reduce, out_map, "i8", ep, out=out)

    def contraction_dequant(self, lhs, rhs, lhs_map, rhs_map, pre_reduce, out_map, row_scale: Storage,
                            scale: Storage, scale_axis: str, out=None, residual: Optional[Storage] = None) -> Storage:
        """W8A8: i8 x i8 -> i32 -> FxpToFp -> MulF(row_scale[m]) -> MulF(scale[n]) -> bf16, fused.
        With `residual` (bf16, laid out as the output), the residual add that follows a projection
        is fused too: out = bf16(f32(residual) + f32(projection)), the projection rounded to bf16
        first, as the separate ops do."""
        if residual is not None and (residual.dtype != "bf16" or residual.n != out_map.size):
            raise ValueError("contraction_dequant: the residual must be bf16 laid out as the output")
        ep = _ep(5 if residual is not None else 3, scale, scale_axis, row_scale=row_scale, residual=residual)
        return self._contract(lhs, rhs, lhs_map, rhs_map, pre_reduce, out_map, "bf16", ep, out=out)

    def contraction_swiglu(self, lhs, rhs, lhs_map, rhs_map, pre_reduce, out_map, row_scale: Storage,
                           scale: Storage, scale_axis: str) -> Storage:
        """The gate and up projections of a SwiGLU and the activation, fused: rhs rows (and `scale`)
        interleave 128 gate and 128 up channels; each pair is dequantised to bf16 exactly as
        `contraction_dequant` does, and act = (g * sigmoid(g)) * u is computed in f32 as the
        elementwise program would. `out_map` names the interleaved [M, N] product; the result is the
        [M, N / 2] f32 activation. Raises FoptError (UNSUPPORTED) when the fused kernel does not
        apply (M or N not a multiple of 256)."""
        ep = _ep(4, scale, scale_axis, row_scale=row_scale)
        out = Storage(self, "f32", out_map.size // 2, zero=False)
        check(_lib.lib().fopt_contraction(self.ctx, out.ptr, _lib.DTYPES["f32"], lhs.ptr, rhs.ptr,
                                          _lib.DTYPES[lhs.dtype], lhs_map.handle, rhs_map.handle, pre_reduce.handle,
                                          out_map.handle, C.byref(ep)), self.ctx)
        return out

    # ---- gather / scatter (backend/mod.rs:159-206) ----
    def gather(self, src: Storage, dst: Storage, index: Storage, Src: Mapping, Dst: Mapping, payload: Mapping,
               axis: Mapping, Idx: Mapping, scaled: bool = False) -> None:
        dst._will_write()
        check(_lib.lib().fopt_gather(self.ctx, dst.ptr, src.ptr, index.ptr, _lib.DTYPES[src.dtype], Src.handle,
                                     Dst.handle, payload.handle, axis.handle, Idx.handle, int(scaled)), self.ctx)

    def scatter(self, src: Storage, dst: Storage, index: Storage, Src: Mapping, Dst: Mapping, payload: Mapping,
                key: Mapping, axis: Mapping, scaled: bool = False) -> None:
        dst._will_write()
        check(_lib.lib().fopt_scatter(self.ctx, dst.ptr, src.ptr, index.ptr, _lib.DTYPES[src.dtype], Src.handle,
                                      Dst.handle, payload.handle, key.handle, axis.handle, int(scaled)), self.ctx)

    # ---- fused attention ----
    def attention(self, q: Storage, k: Storage, v: Storage, batch: int, seq: int, hq: int, hkv: int,
                  head_dim: int = 128, scale: Optional[float] = None, causal: bool = True,
                  eps: float = 6.25e-8, out=None) -> Storage:
        o = out if out is not None else Storage(self, "bf16", q.n, zero=False)
        o._will_write()
        sc = scale if scale is not None else head_dim ** -0.5
        check(_lib.lib().fopt_attention(self.ctx, o.ptr, q.ptr, k.ptr, v.ptr, batch, seq, hq, hkv, head_dim,
                                        C.c_float(sc), int(causal), C.c_float(eps)), self.ctx)
        return o

    # ---- host transfers (backend/mod.rs:220-238) ----
    def to_hbm(self, host_values, Element: Mapping, dtype: str, Dst: Optional[Mapping] = None) -> Storage:
        """HostTensor -> HbmTensor: upload then relayout into the HBM mapping (`transpose(true)`)."""
        s = self.from_vec(Element, host_values, dtype)
        if Dst is None:
            return s
        return self.relayout(s, Element, Dst)

    def from_hbm(self, hbm: Storage, Element: Mapping, dtype: str, Dst: Optional[Mapping] = None) -> np.ndarray:
        s = hbm if Dst is None else self.relayout(hbm, Element, Dst)
        return s.to_numpy()

    def __del__(self):
        try:
            if self.ctx:
                _lib.lib().fopt_destroy(self.ctx)
                self.ctx = C.c_void_p()
        except Exception:
            pass
