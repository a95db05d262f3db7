"""ctypes binding of libfopt_b200.so (the C ABI in include/fopt_b200.h).

This is the Python stand-in for the Rust `extern "C"` block a `B200` backend crate would declare. The
library is required: there is no CPU fallback, and a missing or unbuilt library raises at import of
the op that needs it.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libfopt_b200.so")

# fopt_dtype
DTYPES = {"i8": 0, "i16": 1, "i32": 2, "bf16": 3, "f32": 4, "i4": 5, "f8e4m3": 6, "f8e5m2": 7, "f4e2m1": 8,
          "i5": 9, "i9": 10}
BITS = {"i8": 8, "i16": 16, "i32": 32, "bf16": 16, "f32": 32, "i4": 4, "f8e4m3": 8, "f8e5m2": 8, "f4e2m1": 4,
        "i5": 8, "i9": 16}

STATUS = {0: "OK", 1: "INVALID", 2: "CUDA", 3: "UNSUPPORTED", 4: "NCCL", 5: "TIMEOUT"}


class Insn(C.Structure):
    _fields_ = [("op", C.c_int32), ("dst", C.c_int32), ("a", C.c_int32), ("b", C.c_int32), ("c", C.c_int32),
                ("imm_i", C.c_int32)]


class Program(C.Structure):
    _fields_ = [("n_insn", C.c_int32), ("ret", C.c_int32), ("insn", Insn * 32)]


class RowSlot(C.Structure):
    """`fopt_row_slot`: one per-row scalar of a row program."""
    _fields_ = [("kind", C.c_int32), ("op", C.c_int32), ("identity_bits", C.c_uint32), ("dtype", C.c_int32),
                ("prog", C.POINTER(Program)), ("src", C.c_void_p), ("out", C.c_void_p)]


ROW_FOLD, ROW_SCALAR, ROW_LOAD = 0, 1, 2
REDUCE_OPS = {"Add": 0, "AddSat": 1, "Max": 2, "Min": 3, "Mul": 4}  # fopt_reduce_op
ROW_MAX_LEAVES = ROW_MAX_HELD = ROW_MAX_SLOTS = 8


class RowPlan(C.Structure):
    """`fopt_row_plan`: a row program (leaves, held values, per-row slots, final program)."""
    _fields_ = [("n_leaves", C.c_int32), ("n_held", C.c_int32), ("n_slots", C.c_int32),
                ("leaf", C.c_void_p * 8), ("leaf_dtype", C.c_int32 * 8), ("leaf_bcast", C.c_int64 * 8),
                ("held", C.POINTER(Program) * 8), ("slot", RowSlot * 8), ("final_prog", C.POINTER(Program)),
                ("out", C.c_void_p), ("out_dtype", C.c_int32), ("rows", C.c_int64), ("row_len", C.c_int64)]


class Epilogue(C.Structure):
    _fields_ = [("kind", C.c_int32), ("scale", C.c_void_p), ("scale_axis", C.c_char_p), ("int_width", C.c_int32),
                ("clip_lo", C.c_int32), ("clip_hi", C.c_int32), ("row_scale", C.c_void_p),
                ("residual", C.c_void_p)]


# (name, restype, argtypes) for every symbol the header declares.
_VP, _I32, _I64, _SZ, _CP = C.c_void_p, C.c_int32, C.c_int64, C.c_size_t, C.c_char_p
SIGNATURES = [
    ("fopt_init", _I32, [C.c_int, C.POINTER(_VP)]),
    ("fopt_destroy", _I32, [_VP]),
    ("fopt_last_error", _CP, [_VP]),
    ("fopt_sync", _I32, [_VP]),
    ("fopt_set_stream", _I32, [_VP, _VP]),
    ("fopt_get_stream", _VP, [_VP]),
    ("fopt_set_exact_fold", _I32, [_VP, C.c_int]),
    ("fopt_launch_count", _I64, [_VP]),
    ("fopt_alloc", _I32, [_VP, _SZ, C.POINTER(_VP)]),
    ("fopt_alloc_uninit", _I32, [_VP, _SZ, C.POINTER(_VP)]),
    ("fopt_free", _I32, [_VP, _VP]),
    ("fopt_h2d", _I32, [_VP, _VP, _VP, _SZ]),
    ("fopt_d2h", _I32, [_VP, _VP, _VP, _SZ]),
    ("fopt_d2d", _I32, [_VP, _VP, _VP, _SZ]),
    ("fopt_memset", _I32, [_VP, _VP, C.c_int, _SZ]),
    ("fopt_equal", _I32, [_VP, _VP, _VP, _SZ, C.POINTER(C.c_int)]),
    ("fopt_mapping_parse", _I32, [_CP, _CP, C.POINTER(_VP)]),
    ("fopt_mapping_free", _I32, [_VP]),
    ("fopt_mapping_size", _I64, [_VP]),
    ("fopt_mapping_eval", _I32, [_VP, _I64, C.POINTER(_I64), _I32]),
    ("fopt_window_base", _I32, [_VP, _CP, C.POINTER(_I64)]),
    ("fopt_describe_relayout", _I32, [_VP, _VP, C.c_int, C.c_char_p, _SZ]),
    ("fopt_transpose", _I32, [_VP, _VP, _VP, C.c_int, _VP, _VP, _I64, _I64, C.c_int]),
    ("fopt_transmute", _I32, [_VP, _VP, _VP, C.c_int, _VP, _VP]),
    ("fopt_gather", _I32, [_VP, _VP, _VP, _VP, C.c_int, _VP, _VP, _VP, _VP, _VP, C.c_int]),
    ("fopt_scatter", _I32, [_VP, _VP, _VP, _VP, C.c_int, _VP, _VP, _VP, _VP, _VP, C.c_int]),
    ("fopt_elementwise", _I32, [_VP, C.POINTER(Program), _I32, C.POINTER(_VP), C.POINTER(C.c_int), _VP, C.c_int,
                                _I64]),
    ("fopt_elementwise_source", _I32, [C.POINTER(Program), _I32, C.POINTER(C.c_int), C.c_int, C.c_char_p, _SZ,
                                       C.POINTER(_SZ)]),
    ("fopt_elementwise_jit_launches", C.c_int64, []),
    ("fopt_reduce_map_source", _I32, [C.POINTER(Program), _I32, C.POINTER(C.c_int), _I32, C.c_char_p, _SZ,
                                      C.POINTER(_SZ)]),
    ("fopt_elementwise_bcast", _I32, [C.c_void_p, C.POINTER(Program), _I32, C.POINTER(C.c_void_p), C.POINTER(C.c_int),
                                      C.POINTER(C.c_int64), C.c_void_p, C.c_int, C.c_int64]),
    ("fopt_reduce_map", _I32, [C.c_void_p, C.c_void_p, C.POINTER(Program), _I32, C.POINTER(C.c_void_p),
                               C.POINTER(C.c_int), C.POINTER(C.c_int64), C.c_int, C.c_int, C.c_uint32, C.c_void_p,
                               C.c_void_p]),
    ("fopt_struct_sizes", _I32, [C.POINTER(_SZ), _I32]),
    ("fopt_capture_begin", _I32, [C.c_void_p]),
    ("fopt_capture_end", _I32, [C.c_void_p, C.POINTER(C.c_void_p)]),
    ("fopt_graph_launch", _I32, [C.c_void_p, C.c_void_p]),
    ("fopt_graph_destroy", _I32, [C.c_void_p, C.c_void_p]),
    ("fopt_row_reduce_shape", _I32, [C.c_void_p, C.c_void_p, C.c_void_p, C.POINTER(C.c_int64), C.POINTER(C.c_int64)]),
    ("fopt_row_program", _I32, [C.c_void_p, C.POINTER(RowPlan)]),
    ("fopt_row_program_source", _I32, [C.POINTER(RowPlan), C.c_char_p, _SZ, C.POINTER(_SZ)]),
    ("fopt_st_open", _I32, [C.c_char_p, C.POINTER(C.c_void_p)]),
    ("fopt_st_close", _I32, [C.c_void_p]),
    ("fopt_st_count", _I32, [C.c_void_p]),
    ("fopt_st_info", _I32, [C.c_void_p, _I32, C.POINTER(C.c_char_p), C.POINTER(C.c_char_p), C.POINTER(C.c_int32),
                            C.POINTER(C.c_int64), _I32, C.POINTER(C.c_int64)]),
    ("fopt_st_find", _I32, [C.c_void_p, C.c_char_p, C.POINTER(C.c_int32)]),
    ("fopt_st_read", _I32, [C.c_void_p, C.c_void_p, _I32, C.c_void_p, _SZ]),
    ("fopt_mapping_flat_shape", _I32, [C.c_void_p, C.POINTER(C.c_int64), _I32, C.POINTER(C.c_int32)]),
    ("fopt_broadcast_kind", _I32, [C.c_void_p, C.c_void_p, C.POINTER(C.c_int32), C.POINTER(C.c_int64)]),
    ("fopt_reduce", _I32, [_VP, _VP, _VP, C.c_int, C.c_int, C.c_uint32, _VP, _VP, C.c_int]),
    ("fopt_reduce_noalloc", _I32, [_VP, _VP, _VP, C.c_int, C.c_int, C.c_uint32, _VP, _VP, C.c_int]),
    ("fopt_contraction", _I32, [_VP, _VP, C.c_int, _VP, _VP, C.c_int, _VP, _VP, _VP, _VP, C.POINTER(Epilogue)]),
    ("fopt_contraction_host", _I32, [_VP, _VP, C.c_int, _VP, _VP, C.c_int, _VP, _VP, _VP, _VP, C.POINTER(Epilogue)]),
    ("fopt_attention", _I32, [_VP, _VP, _VP, _VP, _VP, _I32, _I32, _I32, _I32, _I32, C.c_float, _I32, C.c_float]),
    ("fopt_comm_unique_id", _I32, [_VP]),
    ("fopt_comm_init", _I32, [_VP, _I32, _I32, _VP]),
    ("fopt_comm_destroy", _I32, [_VP]),
    ("fopt_allreduce_op", _I32, [_VP, _VP, _I64, C.c_int, C.c_int]),
    ("fopt_allreduce", _I32, [_VP, _VP, _I64, C.c_int]),
    ("fopt_chip_shuffle", _I32, [_VP, _VP, _VP, _SZ, C.POINTER(_I32), _I32]),
    ("fopt_chip_shuffle_plan", _I32, [C.POINTER(_I32), _I32, _I32, C.POINTER(_I32), C.POINTER(_I32),
                                      C.POINTER(_I32)]),
]

_lib = None


def lib() -> C.CDLL:
    """Loads the library (once). Raises if it has not been built: there is no fallback."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"libfopt_b200.so not built at {LIB_PATH}; run furiosa-opt_b200/build.py")
        l = C.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


class FoptError(RuntimeError):
    """A non-zero fopt_status, carrying fopt_last_error()'s message (the reference panics here)."""

    def __init__(self, status: int, msg: str):
        super().__init__(f"[{STATUS.get(status, status)}] {msg}")
        self.status = status


FOPT_ERR_UNSUPPORTED = 3  # fopt_status value the Python side branches on


def check(status: int, ctx=None) -> None:
    if status != 0:
        msg = lib().fopt_last_error(ctx)
        raise FoptError(status, msg.decode() if msg else "")
