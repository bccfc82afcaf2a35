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


class ResultBits(C.Structure):
    """ppdl_result_bits: masks packed 1 bit per pixel (300 x 1250 words)."""
    _fields_ = [("dets", C.POINTER(C.c_float)), ("num_dets", C.c_int32),
                ("mask_bits", C.POINTER(C.c_uint32)), ("infer_ms", C.c_double)]


MASK_WORDS = 1250


def unpack_mask_bits(bits):
    """[..., 1250] uint32 words -> [..., 200, 200] uint8 masks (bit p & 31 of
    word p >> 5 is pixel p), the numpy form of ppdl_expand_mask_bits."""
    import numpy as np
    b = np.ascontiguousarray(bits, dtype=np.uint32)
    u8 = b.view(np.uint8).reshape(b.shape[:-1] + (MASK_WORDS * 4,))
    px = np.unpackbits(u8, axis=-1, bitorder="little")
    return px.reshape(b.shape[:-1] + (MASK_HW, MASK_HW))


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


STEP_KINDS = {0: "other", 1: "gemm_1x1", 2: "wg_madd", 3: "gemm_implicit", 4: "gemm_linear",
              5: "wg_input", 6: "wg_output", 7: "dwconv", 8: "msda", 9: "mask_box", 10: "topk",
              11: "postprocess", 12: "glue", 13: "im2col",
              14: "attention", 15: "conv_direct"}


class StepStat(C.Structure):
    _fields_ = [("name", C.c_char * 48), ("kind", C.c_int32), ("ms", C.c_float),
                ("flops", C.c_double), ("bytes", C.c_double)]


class Context:
    """One loaded model on one GPU (ppdl_ctx).  Mirrors the reference usage
    ppdl_init -> ppdl_infer (-> ppdl_dump_raw) -> ppdl_free."""

    def __init__(self, model_path: str, device: int = -1, max_batch: int = 1,
                 dumps: bool = False, backend: int = BACKEND_CUDA):
        L = lib()
        L.ppdl_init_dev.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_int]
        L.ppdl_init_dev.restype = C.c_void_p
        L.ppdl_infer_batch.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p,
                                       C.POINTER(Result)]
        L.ppdl_infer_batch.restype = C.c_int
        L.ppdl_infer_device.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]
        L.ppdl_infer_device.restype = C.c_int
        L.ppdl_device_outputs.argtypes = [C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p)]
        L.ppdl_device_outputs.restype = C.c_int
        L.ppdl_sync.argtypes = [C.c_void_p]
        L.ppdl_sync.restype = C.c_int
        self.lib = L
        self.max_batch = max_batch
        self.ctx = L.ppdl_init_dev(model_path.encode(), backend, device, max_batch, int(dumps))
        if not self.ctx:
            raise RuntimeError(f"ppdl_init failed for {model_path}")

    def infer(self, image, ori_h: int = IMG_SIZE, ori_w: int = IMG_SIZE):
        """One page (float32 [3,800,800]) -> (dets [300,7], masks [300,200,200])."""
        import numpy as np
        img = np.ascontiguousarray(image, dtype=np.float32)
        res = Result()
        rc = self.lib.ppdl_infer(self.ctx, img.ctypes.data, int(ori_h), int(ori_w), C.byref(res))
        if rc != 0:
            raise RuntimeError(f"ppdl_infer returned {rc}")
        dets = np.ctypeslib.as_array(res.dets, (NUM_DETS, DET_FIELDS)).copy()
        masks = np.ctypeslib.as_array(res.masks, (NUM_DETS, MASK_HW, MASK_HW)).copy()
        return dets, masks, res.infer_ms

    def infer_batch(self, images, ori_hw, copy=True):
        """n pages [n,3,800,800] -> list of (dets, masks).

        copy=True returns arrays the caller owns.  copy=False returns views
        of the context's pinned host buffers (what ppdl_infer_batch's
        ppdl_result points at), valid until the next inference on this
        context; it skips the 48 MB-per-page host copy of the masks.  Pages
        given in pinned host memory (e.g. a pinned torch tensor's .numpy())
        are copied to the device at full PCIe speed."""
        import numpy as np
        imgs = np.ascontiguousarray(images, dtype=np.float32)
        hw = np.ascontiguousarray(ori_hw, dtype=np.int32).reshape(-1, 2)
        n = imgs.shape[0]
        res = (Result * n)()
        rc = self.lib.ppdl_infer_batch(self.ctx, imgs.ctypes.data, n, hw.ctypes.data, res)
        if rc != 0:
            raise RuntimeError(f"ppdl_infer_batch returned {rc}")
        out = []
        for r in res:
            d = np.ctypeslib.as_array(r.dets, (NUM_DETS, DET_FIELDS))
            m = np.ctypeslib.as_array(r.masks, (NUM_DETS, MASK_HW, MASK_HW))
            out.append((d.copy(), m.copy()) if copy else (d, m))
        return out

    def infer_device(self, d_images_ptr: int, n: int, ori_hw) -> int:
        import numpy as np
        hw = np.ascontiguousarray(ori_hw, dtype=np.int32).reshape(-1, 2)
        self._hw = hw
        return self.lib.ppdl_infer_device(self.ctx, C.c_void_p(d_images_ptr), n, hw.ctypes.data)

    def device_outputs(self):
        d = C.c_void_p()
        m = C.c_void_p()
        rc = self.lib.ppdl_device_outputs(self.ctx, C.byref(d), C.byref(m))
        if rc != 0:
            raise RuntimeError("no device outputs")
        return d.value, m.value

    def sync(self) -> int:
        return self.lib.ppdl_sync(self.ctx)

    def infer_device_bits(self, d_images_ptr: int, n: int, ori_hw) -> int:
        """ppdl_infer_device with the masks left packed (no int32 expansion)."""
        import numpy as np
        L = self.lib
        L.ppdl_infer_device_bits.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]
        L.ppdl_infer_device_bits.restype = C.c_int
        hw = np.ascontiguousarray(ori_hw, dtype=np.int32).reshape(-1, 2)
        self._hw = hw
        return L.ppdl_infer_device_bits(self.ctx, C.c_void_p(d_images_ptr), n, hw.ctypes.data)

    def device_mask_bits(self) -> int:
        L = self.lib
        L.ppdl_device_mask_bits.argtypes = [C.c_void_p, C.POINTER(C.c_void_p)]
        L.ppdl_device_mask_bits.restype = C.c_int
        p = C.c_void_p()
        if L.ppdl_device_mask_bits(self.ctx, C.byref(p)) != 0:
            raise RuntimeError("no device outputs")
        return p.value

    def submit(self, images, ori_hw) -> int:
        """ppdl_submit_batch: enqueue n pages [n,3,800,800] (keep them alive
        and unchanged until wait() of the returned ticket; pinned memory lets
        the copy overlap the previous batch's forward)."""
        import numpy as np
        L = self.lib
        L.ppdl_submit_batch.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p,
                                        C.POINTER(C.c_int64)]
        L.ppdl_submit_batch.restype = C.c_int
        if not (isinstance(images, np.ndarray) and images.dtype == np.float32 and
                images.flags.c_contiguous):
            raise ValueError("submit() needs a C-contiguous float32 array that stays alive")
        hw = np.ascontiguousarray(ori_hw, dtype=np.int32).reshape(-1, 2)
        t = C.c_int64()
        rc = L.ppdl_submit_batch(self.ctx, images.ctypes.data, images.shape[0], hw.ctypes.data,
                                 C.byref(t))
        if rc != 0:
            raise RuntimeError(f"ppdl_submit_batch returned {rc}")
        return t.value

    def wait(self, ticket: int, n: int, copy=True):
        """ppdl_wait_batch: [(dets [300,7], mask_bits [300,1250] uint32)] of
        the n pages of ticket.  copy=False returns views of the context's
        pinned result slot, valid until ticket + 2 is submitted."""
        import numpy as np
        L = self.lib
        L.ppdl_wait_batch.argtypes = [C.c_void_p, C.c_int64, C.POINTER(ResultBits)]
        L.ppdl_wait_batch.restype = C.c_int
        res = (ResultBits * n)()
        rc = L.ppdl_wait_batch(self.ctx, ticket, res)
        if rc != 0:
            raise RuntimeError(f"ppdl_wait_batch returned {rc}")
        out = []
        for r in res:
            d = np.ctypeslib.as_array(r.dets, (NUM_DETS, DET_FIELDS))
            b = np.ctypeslib.as_array(r.mask_bits, (NUM_DETS, MASK_WORDS))
            out.append((d.copy(), b.copy()) if copy else (d, b))
        return out

    def stream_ptr(self) -> int:
        self.lib.ppdl_stream.argtypes = [C.c_void_p]
        self.lib.ppdl_stream.restype = C.c_void_p
        return self.lib.ppdl_stream(self.ctx) or 0

    def profile_steps(self, n: int):
        """[(name, kind, ms, flops_per_page, bytes_per_page)] of one eager
        forward of the last n pages, with a CUDA event after every step."""
        self.lib.ppdl_profile_steps.argtypes = [C.c_void_p, C.c_int, C.POINTER(StepStat), C.c_int]
        self.lib.ppdl_profile_steps.restype = C.c_int
        buf = (StepStat * 4096)()
        k = self.lib.ppdl_profile_steps(self.ctx, n, buf, 4096)
        if k < 0:
            raise RuntimeError("ppdl_profile_steps failed")
        return [(buf[i].name.decode(), STEP_KINDS.get(buf[i].kind, "other"), buf[i].ms,
                 buf[i].flops, buf[i].bytes) for i in range(k)]

    def profile_timeline(self, n: int):
        """[(end_ms, lane)] per step (the order of profile_steps): the end of
        each step from the start of the forward, with the lanes running
        concurrently as in the captured forward."""
        self.lib.ppdl_profile_timeline.argtypes = [C.c_void_p, C.c_int, C.POINTER(C.c_float),
                                                   C.POINTER(C.c_int32), C.c_int]
        self.lib.ppdl_profile_timeline.restype = C.c_int
        end = (C.c_float * 4096)()
        lane = (C.c_int32 * 4096)()
        k = self.lib.ppdl_profile_timeline(self.ctx, n, end, lane, 4096)
        if k < 0:
            raise RuntimeError("ppdl_profile_timeline failed")
        return [(end[i], lane[i]) for i in range(k)]

    def dump_raw(self, pfx: str) -> int:
        return self.lib.ppdl_dump_raw(self.ctx, pfx.encode())

    def dump(self, d: str) -> int:
        return self.lib.ppdl_dump(self.ctx, d.encode())

    def close(self):
        if self.ctx:
            self.lib.ppdl_free(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def last_error() -> str:
    return lib().ppdl_op_last_error().decode()


def check(status: int) -> None:
    if status != PPDL_OK:
        raise RuntimeError(f"ppdl_op_launch failed ({status}): {last_error()}")
