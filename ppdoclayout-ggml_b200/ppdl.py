"""Python mirror of the B200 PP-DocLayoutV3 C ABIs (ctypes).

Two surfaces, both thin bindings of lib/libppdl_b200.so:

* the model API of include/ppdoclayout.h (ppdl_init / ppdl_infer /
  ppdl_infer_batch / ppdl_dump_raw / ppdl_free) — the reference's public C
  ABI (include/ppdoclayout.h:29-63 of caojiachen1/ppdoclayout-ggml) plus the
  additive batch and device-output entry points;
* the operator API of include/ppdl_ops.h (ppdl_op_launch) — the reference's
  tagged ggml custom-op hooks (patches/ggml-ppdl.patch:612-930), driven here
  with torch CUDA tensors as the device memory.

There is no CPU fallback: importing this module never loads anything else,
and every call fails loudly when the CUDA library is missing.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libppdl_b200.so")

PPDL_MAGIC = 0x5050444C
OP_MASKBOX, OP_MSDEF, OP_CONV, OP_CONVDIRECT, OP_BIASACT, OP_COPY = 1, 2, 3, 4, 5, 6
OP_WG_INPUT, OP_WG_OUTPUT, OP_WG_MADD = 7, 8, 9
OP_WG4_INPUT, OP_WG4_OUTPUT, OP_WG4_MADD, OP_TOPK = 10, 11, 12, 13

PPDL_OK, PPDL_ERR_UNSUPPORTED, PPDL_ERR_SHAPE, PPDL_ERR_CUDA = 0, 1, 2, 3

IMG_SIZE, NUM_DETS, DET_FIELDS, MASK_HW = 800, 300, 7, 200
BACKEND_CPU, BACKEND_CUDA = 0, 1


class Tensor(C.Structure):
    _fields_ = [("data", C.c_void_p), ("ne", C.c_int64 * 4)]


class OpDesc(C.Structure):
    _fields_ = [("dst", Tensor), ("src", Tensor * 4), ("op_params", C.c_int32 * 16)]


class Result(C.Structure):
    _fields_ = [("dets", C.POINTER(C.c_float)), ("num_dets", C.c_int32),
                ("masks", C.POINTER(C.c_int32)), ("infer_ms", C.c_double)]


_lib = None


def lib() -> C.CDLL:
    """The loaded product library; raises when it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `make -C {HERE}` "
                "(there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        L.ppdl_op_launch.argtypes = [C.POINTER(OpDesc), C.c_void_p]
        L.ppdl_op_launch.restype = C.c_int
        L.ppdl_op_supported.argtypes = [C.POINTER(OpDesc)]
        L.ppdl_op_supported.restype = C.c_int
        L.ppdl_op_last_error.restype = C.c_char_p
        if hasattr(L, "ppdl_init"):
            L.ppdl_init.argtypes = [C.c_char_p, C.c_int]
            L.ppdl_init.restype = C.c_void_p
            L.ppdl_init_ex.argtypes = [C.c_char_p, C.c_int, C.c_int]
            L.ppdl_init_ex.restype = C.c_void_p
            L.ppdl_infer.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.POINTER(Result)]
            L.ppdl_infer.restype = C.c_int
            L.ppdl_free.argtypes = [C.c_void_p]
            L.ppdl_free.restype = None
            L.ppdl_dump_raw.argtypes = [C.c_void_p, C.c_char_p]
            L.ppdl_dump_raw.restype = C.c_int
            L.ppdl_dump.argtypes = [C.c_void_p, C.c_char_p]
            L.ppdl_dump.restype = C.c_int
        _lib = L
    return _lib


def _tensor(t, ne=None) -> Tensor:
    """ppdl_tensor for a contiguous torch CUDA tensor; ne in ggml order
    (fastest first), defaulting to the reversed torch shape."""
    if t is None:
        return Tensor(None, (C.c_int64 * 4)(1, 1, 1, 1))
    assert t.is_cuda and t.is_contiguous(), "operator ABI takes contiguous CUDA tensors"
    if ne is None:
        ne = list(reversed(t.shape))
    ne = list(ne) + [1] * (4 - len(ne))
    return Tensor(C.c_void_p(t.data_ptr()), (C.c_int64 * 4)(*ne))


def make_desc(op_id, dst, srcs=(), params=(), dst_ne=None, src_ne=()) -> OpDesc:
    d = OpDesc()
    d.dst = _tensor(dst, dst_ne)
    for i in range(4):
        s = srcs[i] if i < len(srcs) else None
        ne = src_ne[i] if i < len(src_ne) else None
        d.src[i] = _tensor(s, ne)
    d.op_params[12] = PPDL_MAGIC - (1 << 32) if PPDL_MAGIC >= (1 << 31) else PPDL_MAGIC
    d.op_params[13] = op_id
    for i, v in enumerate(params):
        d.op_params[14 + i] = int(v)
    return d


def op_launch(op_id, dst, srcs=(), params=(), dst_ne=None, src_ne=(), stream=None) -> int:
    """ppdl_op_launch on torch tensors; returns the PPDL status code.
    `stream` is a torch.cuda.Stream or None for torch's current stream."""
    import torch
    d = make_desc(op_id, dst, srcs, params, dst_ne, src_ne)
    s = stream if stream is not None else torch.cuda.current_stream()
    return lib().ppdl_op_launch(C.byref(d), C.c_void_p(s.cuda_stream))


def op_supported(op_id, params=()) -> bool:
    d = OpDesc()
    d.op_params[12] = PPDL_MAGIC - (1 << 32)
    d.op_params[13] = op_id
    for i, v in enumerate(params):
        d.op_params[14 + i] = int(v)
    return bool(lib().ppdl_op_supported(C.byref(d)))


def last_error() -> str:
    return lib().ppdl_op_last_error().decode()


def check(status: int) -> None:
    if status != PPDL_OK:
        raise RuntimeError(f"ppdl_op_launch failed ({status}): {last_error()}")
