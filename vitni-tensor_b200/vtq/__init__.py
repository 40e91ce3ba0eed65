"""vtq -- Python host binding of the B200 k-quant linear backend (C ABI: include/vtq.h).

Mirrors vitni-tensor's quantized-linear interface: the same function names,
argument meaning (x [batch][in_feat] f32, row-major weight bytes, y_out
[batch][out_feat]) and error behaviour (``Internal`` for shape/length checks,
``NotImplemented`` for unsupported dtypes), as in src/ops/quant.rs and
src/model/forward_quantized.rs:663-785 of the reference.

All arithmetic runs in libvtq.so's sm_100a kernels. There is no CPU fallback:
importing works without a GPU, but any compute call raises if the library or a
device is missing.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from .formats import (F32, Q4_0, Q5_0, Q8_0, Q4_K, Q6_K, QuantTensor, row_bytes)  # noqa: F401

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("VTQ_LIBRARY") or os.path.join(_HERE, "libvtq.so")

PTR_HOST = 1
Q4K_FLOAT = 2

# Status codes (include/vtq.h).
OK, ERR_INTERNAL, ERR_NOT_IMPLEMENTED, ERR_GPU, ERR_OOM, ERR_TIMEOUT, ERR_INVALID_ARG = range(7)
ERR_MALFORMED, ERR_TRUNCATED = 7, 8

# Every symbol include/vtq.h declares.
EXPORTS = (
    "vtq_init", "vtq_destroy", "vtq_last_error", "vtq_set_stream", "vtq_synchronize",
    "vtq_weight_upload", "vtq_weight_free", "vtq_weight_info", "vtq_linear",
    "vtq_linear_dispatch", "vtq_linear_q4_k_integer", "vtq_linear_q6_k_integer",
    "vtq_linear_q4_k_fused", "vtq_linear_q4_0", "vtq_device_layout_bytes",
    "vtq_device_repack", "vtq_linear_device", "vtq_decode_open", "vtq_decode_last_error",
    "vtq_decode_config", "vtq_decode_run", "vtq_decode_close", "vtq_expf", "vtq_sinf",
    "vtq_cosf", "vtq_powf", "vtq_libm_sweep", "vtq_linear_host_noalloc",
    "vtq_gather_create", "vtq_gather_connect", "vtq_gather_y", "vtq_linear_gather",
    "vtq_gather_wait", "vtq_gather_destroy", "vtq_libm_sweep_device", "vtq_linear_gather_wait",
    "vtq_decode_timing", "vtq_decode_debug_buffer", "vtq_decode_step_kind",
    "vtq_exact_sum_host", "vtq_exact_sum_device", "vtq_decode_launches", "vtq_linear_list", "vtq_set_wait_limit",
    "vtq_linear_list_gather", "vtq_linear_device_workspace_bytes", "vtq_linear_device_ws",
)


class Error(Exception):
    """Base of the reference's error enum (src/error.rs:7-63)."""

    status = -1


class Internal(Error):
    status = ERR_INTERNAL


class NotImplementedOp(Error):
    status = ERR_NOT_IMPLEMENTED


class GpuError(Error):
    status = ERR_GPU


class OutOfMemory(Error):
    status = ERR_OOM


class Timeout(Error):
    status = ERR_TIMEOUT


class InvalidArg(Error):
    status = ERR_INVALID_ARG


class Malformed(Error):
    status = ERR_MALFORMED


class Truncated(Error):
    status = ERR_TRUNCATED


_ERRORS = {c.status: c for c in (Internal, NotImplementedOp, GpuError, OutOfMemory, Timeout,
                                 InvalidArg, Malformed, Truncated)}

_lib = None


class ListItem(ctypes.Structure):
    """vtq_list_item (include/vtq.h)."""
    _fields_ = [("w", ctypes.c_void_p), ("x", ctypes.c_void_p), ("y", ctypes.c_void_p),
                ("wait_for", ctypes.c_int32)]


LIST_MAX = 32
GATHER_DEFER = 4


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load libvtq.so (raises OSError if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise OSError(f"libvtq.so not built at {path}: run vitni-tensor_b200/build.py")
    lib = ctypes.CDLL(path)
    c_p, c_i32, c_i64, c_sz, c_u32 = (ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
                                       ctypes.c_size_t, ctypes.c_uint32)
    sig = {
        "vtq_init": (c_i32, [ctypes.c_int, ctypes.POINTER(c_p)]),
        "vtq_destroy": (c_i32, [c_p]),
        "vtq_last_error": (ctypes.c_char_p, [c_p]),
        "vtq_set_stream": (c_i32, [c_p, c_p]),
        "vtq_synchronize": (c_i32, [c_p]),
        "vtq_weight_upload": (c_i32, [c_p, c_i32, c_p, c_sz, c_i64, c_i64, c_i64, c_i64,
                                      ctypes.POINTER(c_p)]),
        "vtq_weight_free": (c_i32, [c_p]),
        "vtq_weight_info": (c_i32, [c_p, ctypes.POINTER(c_i32), ctypes.POINTER(c_i64),
                                    ctypes.POINTER(c_i64), ctypes.POINTER(c_sz)]),
        "vtq_linear": (c_i32, [c_p, c_p, c_p, c_p, c_i64, c_u32]),
        "vtq_linear_dispatch": (c_i32, [c_p, c_i32, c_p, c_p, c_sz, c_sz, c_sz, c_p, c_u32]),
        "vtq_linear_q4_k_integer": (c_i32, [c_p, c_p, c_p, c_sz, c_p, c_sz, c_sz, c_sz]),
        "vtq_linear_q6_k_integer": (c_i32, [c_p, c_p, c_p, c_sz, c_p, c_sz, c_sz, c_sz]),
        "vtq_linear_q4_k_fused": (c_i32, [c_p, c_p, c_p, c_sz, c_p, c_sz, c_sz, c_sz]),
        "vtq_linear_q4_0": (c_i32, [c_p, c_p, c_p, c_sz, c_p, c_sz, c_sz, c_sz]),
        "vtq_device_layout_bytes": (c_i64, [c_i32, c_i64, c_i64]),
        "vtq_device_repack": (c_i32, [c_i32, c_i64, c_i64, c_p, c_p, c_p]),
        "vtq_linear_device": (c_i32, [c_i32, c_p, c_i64, c_i64, c_p, c_i64, c_p, c_i64, c_i64,
                                      c_u32, c_p, c_p]),
        "vtq_decode_open": (c_i32, [c_p, ctypes.c_int, c_p, c_sz, ctypes.POINTER(c_p)]),
        "vtq_decode_last_error": (ctypes.c_char_p, [c_p]),
        "vtq_decode_config": (c_i32, [c_p, c_p]),
        "vtq_decode_run": (c_i32, [c_p, c_p, c_sz, c_sz, c_p, c_p]),
        "vtq_decode_close": (c_i32, [c_p]),
        "vtq_expf": (ctypes.c_float, [ctypes.c_float]),
        "vtq_sinf": (ctypes.c_float, [ctypes.c_float]),
        "vtq_cosf": (ctypes.c_float, [ctypes.c_float]),
        "vtq_powf": (ctypes.c_float, [ctypes.c_float, ctypes.c_float]),
        "vtq_libm_sweep": (None, [c_p, c_sz, c_p]),
        "vtq_decode_timing": (c_i32, [c_p, c_p]),
        "vtq_decode_step_kind": (c_i32, [c_p]),
        "vtq_decode_launches": (ctypes.c_ulonglong, [c_p]),
        "vtq_exact_sum_host": (ctypes.c_float, [c_p, c_sz, c_p]),
        "vtq_exact_sum_device": (c_i32, [c_p, c_i32, c_i32, c_i32, c_p]),
        "vtq_decode_debug_buffer": (c_i32, [c_p, ctypes.c_int, c_p, c_sz]),
        "vtq_linear_host_noalloc": (c_i32, [c_i32, c_p, c_i64, c_i64, c_p, c_p, c_i64, c_p]),
        "vtq_gather_create": (c_i32, [c_p, c_i32, c_i32, c_sz, ctypes.POINTER(c_p), c_p]),
        "vtq_gather_connect": (c_i32, [c_p, c_p]),
        "vtq_gather_y": (c_p, [c_p]),
        "vtq_linear_gather": (c_i32, [c_p, c_p, c_p, c_i64, c_p, c_i64, c_i64, c_i64, c_u32]),
        "vtq_gather_wait": (c_i32, [c_p, c_p, c_u32]),
        "vtq_gather_destroy": (c_i32, [c_p]),
        "vtq_libm_sweep_device": (c_i32, [c_p, c_sz, c_p]),
        "vtq_linear_list": (c_i32, [c_p, c_p, c_i32, c_u32]),
        "vtq_set_wait_limit": (c_i32, [c_p, ctypes.c_uint64]),
        "vtq_linear_device_workspace_bytes": (c_sz, [c_i32, c_i64, c_i64, c_u32]),
        "vtq_linear_device_ws": (c_i32, [c_i32, c_p, c_i64, c_i64, c_p, c_i64, c_p, c_i64, c_i64,
                                         c_u32, c_p, c_p, c_sz, c_p]),
        "vtq_linear_list_gather": (c_i32, [c_p, c_p, c_i32, c_p, c_u32, c_u32]),
        "vtq_linear_gather_wait": (c_i32, [c_p, c_p, c_p, c_i64, c_p, c_i64, c_i64, c_i64, c_u32,
                                           c_u32]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class Weight:
    """A device-resident weight matrix (rows [row_begin, row_end) of W)."""

    def __init__(self, ctx: "Context", handle: int, dtype: int, in_feat: int, rows: int,
                 row_begin: int):
        self.ctx, self.handle, self.dtype = ctx, handle, dtype
        self.in_feat, self.rows, self.row_begin = in_feat, rows, row_begin

    def device_bytes(self) -> int:
        sz = ctypes.c_size_t()
        self.ctx._check(self.ctx.lib.vtq_weight_info(self.handle, None, None, None,
                                                      ctypes.byref(sz)))
        return sz.value

    def free(self):
        if self.handle:
            self.ctx.lib.vtq_weight_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Context:
    """One CUDA device + stream (vtq_init)."""

    def __init__(self, device: int = 0):
        self.lib = load_library()
        h = ctypes.c_void_p()
        st = self.lib.vtq_init(device, ctypes.byref(h))
        if st != OK:
            raise _ERRORS.get(st, Error)(f"vtq_init({device}) failed with status {st}")
        self.handle = h.value
        self.device = device

    def _check(self, st: int):
        if st != OK:
            msg = self.lib.vtq_last_error(self.handle).decode()
            raise _ERRORS.get(st, Error)(msg)

    def close(self):
        if getattr(self, "handle", None):
            self.lib.vtq_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, stream_ptr: int | None):
        self._check(self.lib.vtq_set_stream(self.handle, stream_ptr))

    def synchronize(self):
        self._check(self.lib.vtq_synchronize(self.handle))

    def set_wait_limit(self, ns: int):
        """Bound of this context's device-side gather waits (default 2 s)."""
        self._check(self.lib.vtq_set_wait_limit(self.handle, int(ns)))

    # -- resident weights -------------------------------------------------
    def upload(self, dtype: int, data, in_feat: int, out_feat: int, row_begin: int = 0,
               row_end: int = -1) -> Weight:
        buf = np.frombuffer(bytes(data), np.uint8) if not isinstance(data, np.ndarray) else \
            np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        h = ctypes.c_void_p()
        self._check(self.lib.vtq_weight_upload(self.handle, dtype, _ptr(buf), buf.nbytes, in_feat,
                                               out_feat, row_begin, row_end, ctypes.byref(h)))
        re = out_feat if row_end < 0 else row_end
        return Weight(self, h.value, dtype, in_feat, re - row_begin, row_begin)

    def linear(self, w: Weight, x: np.ndarray, batch: int = 1, q4k_float: bool = False
               ) -> np.ndarray:
        """y = W x for host arrays (copies in/out inside the call)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.size != batch * w.in_feat:
            raise Internal("vtq_linear: x shape mismatch")
        y = np.empty(batch * w.rows, np.float32)
        flags = PTR_HOST | (Q4K_FLOAT if q4k_float else 0)
        self._check(self.lib.vtq_linear(self.handle, w.handle, _ptr(x), _ptr(y), batch, flags))
        return y

    def linear_ptr(self, w: Weight, x_ptr: int, y_ptr: int, batch: int = 1, host: bool = False,
                   q4k_float: bool = False):
        """vtq_linear on raw pointers (device pointers unless host=True)."""
        flags = (PTR_HOST if host else 0) | (Q4K_FLOAT if q4k_float else 0)
        self._check(self.lib.vtq_linear(self.handle, w.handle, x_ptr, y_ptr, batch, flags))

    def prepare_list(self, items, host: bool = False):
        """A reusable vtq_linear_list call: the item array is built once and the
        returned function makes the C call (for repeated calls on the same
        buffers, e.g. one decode step per call)."""
        arr = (ListItem * len(items))()
        for i, it in enumerate(items):
            w, xp, yp = it[:3]
            arr[i] = ListItem(w.handle, xp, yp, it[3] if len(it) > 3 else -1)
        fn, h, n, fl = self.lib.vtq_linear_list, self.handle, len(items), PTR_HOST if host else 0
        keep = [it[0] for it in items]  # the weights must outlive the call

        def call():
            st = fn(h, arr, n, fl)
            if st:
                self._check(st)
        call.keep = keep
        return call

    def linear_list(self, items, host: bool = False):
        """vtq_linear_list: items are (Weight, x_ptr, y_ptr[, wait_for]), device
        pointers (host pointers with host=True), run as one persistent launch in
        list order."""
        arr = (ListItem * len(items))()
        for i, it in enumerate(items):
            w, xp, yp = it[:3]
            arr[i] = ListItem(w.handle, xp, yp, it[3] if len(it) > 3 else -1)
        self._check(self.lib.vtq_linear_list(self.handle, arr, len(items), PTR_HOST if host else 0))


# -- reference-signature functions (host slices) ---------------------------------

def _as_f32(x) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32)


def _as_u8(w) -> np.ndarray:
    if isinstance(w, np.ndarray):
        return np.ascontiguousarray(w).view(np.uint8).reshape(-1)
    return np.frombuffer(bytes(w), np.uint8)


def _op(name: str):
    def fn(ctx: Context, x, w, y_out: np.ndarray, batch: int, in_feat: int, out_feat: int):
        xa, wa = _as_f32(x), _as_u8(w)
        if y_out.dtype != np.float32 or not y_out.flags.c_contiguous:
            raise Internal(f"{name}: y_out must be contiguous float32")
        if xa.size < batch * in_feat or y_out.size < batch * out_feat:
            raise Internal(f"{name}: x/y size mismatch")
        ctx._check(getattr(ctx.lib, "vtq_" + name)(ctx.handle, _ptr(xa), _ptr(wa), wa.nbytes,
                                                   _ptr(y_out), batch, in_feat, out_feat))
    fn.__name__ = name
    fn.__doc__ = f"Bit-identical GPU replacement of the reference's `{name}` (host slices)."
    return fn


linear_q4_k_integer = _op("linear_q4_k_integer")
linear_q6_k_integer = _op("linear_q6_k_integer")
linear_q4_k_fused = _op("linear_q4_k_fused")
linear_q4_0 = _op("linear_q4_0")


def linear_dispatch(ctx: Context, x, w: QuantTensor, in_feat: int, out_feat: int,
                    q4k_float: bool = False) -> np.ndarray:
    """linear_dispatch (src/model/forward_quantized.rs:663-785): batch 1, returns y."""
    xa, wa = _as_f32(x), _as_u8(w.bytes)
    if xa.size < in_feat:
        raise Internal("linear_dispatch: x shorter than in_feat")
    y = np.zeros(out_feat, np.float32)
    ctx._check(ctx.lib.vtq_linear_dispatch(ctx.handle, w.dtype, _ptr(xa), _ptr(wa), wa.nbytes,
                                           in_feat, out_feat, _ptr(y),
                                           Q4K_FLOAT if q4k_float else 0))
    return y


def _device_floats(ptr: int, n: int) -> np.ndarray:
    """Copy n floats from device address ptr to a new host array."""
    out = np.empty(n, np.float32)
    import torch

    class _A:
        __cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False),
                                    "version": 3}
    out[:] = torch.as_tensor(_A(), device="cuda").cpu().numpy()
    return out


class Gather:
    """Fused row-shard all-gather over NVLink (one per rank of a process group).

    Every rank owns a full-y buffer of `y_floats` floats; `linear` computes this
    rank's rows of a row-sharded weight and stores them into every rank's
    buffer, `wait` holds the stream until the expected ranks have arrived.
    The buffer handles are exchanged with torch.distributed (all_gather_object).
    """

    def __init__(self, ctx: "Context", y_floats: int, group=None):
        import torch.distributed as dist
        self.ctx, self.lib = ctx, ctx.lib
        single = not dist.is_available() or not dist.is_initialized()
        self.world, self.rank = (1, 0) if single else (dist.get_world_size(group),
                                                      dist.get_rank(group))
        h = ctypes.c_void_p()
        ipc = ctypes.create_string_buffer(64)
        ctx._check(self.lib.vtq_gather_create(ctx.handle, self.world, self.rank, y_floats,
                                              ctypes.byref(h), ipc))
        self.handle = h
        handles = [ipc.raw]
        if not single:
            handles = [None] * self.world
            dist.all_gather_object(handles, ipc.raw, group=group)
        blob = b"".join(handles)
        ctx._check(self.lib.vtq_gather_connect(self.handle, blob))
        self.y_ptr = self.lib.vtq_gather_y(self.handle)
        self.y_floats = y_floats

    def linear(self, w: "Weight", x_ptr: int, row0: int, ldy: int, y_offset: int = 0,
               batch: int = 1, wait_signals: int = 0, defer: bool = False):
        """wait_signals > 0: the launch ends only once that many rank arrivals
        (including this launch's) have reached this rank. defer: no arrival
        signal; the next signalling launch covers this one."""
        self.ctx._check(self.lib.vtq_linear_gather_wait(self.ctx.handle, w.handle, x_ptr, batch,
                                                        self.handle, y_offset, ldy, row0,
                                                        GATHER_DEFER if defer else 0,
                                                        wait_signals))

    def linear_list(self, items, wait_signals: int = 0):
        """vtq_linear_list_gather: items are (Weight, x_ptr, y_offset[, wait_for])
        with y at y_offset floats into this rank's gather buffer; one launch,
        one arrival signal to every rank."""
        arr = (ListItem * len(items))()
        for i, it in enumerate(items):
            w, xp, yo = it[:3]
            arr[i] = ListItem(w.handle, xp, self.y_ptr + 4 * yo, it[3] if len(it) > 3 else -1)
        self.ctx._check(self.lib.vtq_linear_list_gather(self.ctx.handle, arr, len(items),
                                                        self.handle, 0, wait_signals))

    def wait(self, signals: int):
        self.ctx._check(self.lib.vtq_gather_wait(self.ctx.handle, self.handle, signals))

    def close(self):
        if self.handle:
            self.lib.vtq_gather_destroy(self.handle)
            self.handle = None


class DecodeSession:
    """A GGUF Llama model resident on one GPU, decoded by run_quantized's loop
    (src/model/inference.rs:274-345) with every step on the device."""

    def __init__(self, gguf_blob: bytes, device: int = 0):
        self.lib = load_library()
        self._blob = np.frombuffer(bytes(gguf_blob), np.uint8)
        h = ctypes.c_void_p()
        st = self.lib.vtq_decode_open(None, device, _ptr(self._blob), self._blob.nbytes,
                                      ctypes.byref(h))
        self.handle = h.value
        if st != OK:
            msg = self.lib.vtq_decode_last_error(self.handle).decode() if self.handle else ""
            self.close()
            raise _ERRORS.get(st, Error)(msg)
        cfg = np.zeros(8, np.int64)
        self.lib.vtq_decode_config(self.handle, _ptr(cfg))
        keys = ("dim", "hidden", "layers", "heads", "kv_heads", "vocab", "seq_len", "shared")
        self.config = {k: int(v) for k, v in zip(keys, cfg)}
        # 0 per-op graph, 1 fused-op graph, 2 persistent kernel per step
        self.step_kind = int(self.lib.vtq_decode_step_kind(self.handle))

    def run(self, prompt, n_new: int, logits: bool = False):
        """Returns (generated token ids, per-step logits [n_prompt + n_new, vocab] or None)."""
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.zeros(max(1, n_new), np.uint32)
        lg = np.zeros((len(p) + n_new, self.config["vocab"]), np.float32) if logits else None
        st = self.lib.vtq_decode_run(self.handle, _ptr(p), len(p), n_new, _ptr(out),
                                     _ptr(lg) if lg is not None else None)
        if st != OK:
            raise _ERRORS.get(st, Error)(self.lib.vtq_decode_last_error(self.handle).decode())
        return out[:n_new].tolist(), lg

    def timing(self):
        """(ms of the decode steps, ms of the whole last run call), device time."""
        t = np.zeros(2, np.float32)
        self.lib.vtq_decode_timing(self.handle, _ptr(t))
        return float(t[0]), float(t[1])

    def launches(self) -> int:
        """Kernels launched for the last run's decode work (batched prompt + steps)."""
        return int(self.lib.vtq_decode_launches(self.handle))

    def close(self):
        if getattr(self, "handle", None):
            self.lib.vtq_decode_close(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def exact_sum_host(a) -> tuple:
    """(left-to-right fp32 sum of a, fell back to the plain loop) through the
    host evaluation of the run/crossing plan."""
    a = _as_f32(a)
    fb = ctypes.c_int(0)
    s = load_library().vtq_exact_sum_host(_ptr(a), a.size, ctypes.byref(fb))
    return np.float32(s), bool(fb.value)


def exact_sum_device(vecs, nthr: int = 256) -> np.ndarray:
    """Sums of the rows of vecs [nvec, n], one CTA of nthr threads per row."""
    v = np.ascontiguousarray(vecs, dtype=np.float32)
    out = np.zeros(v.shape[0], np.float32)
    st = load_library().vtq_exact_sum_device(_ptr(v), v.shape[0], v.shape[1], nthr, _ptr(out))
    if st != OK:
        raise _ERRORS.get(st, Error)(f"vtq_exact_sum_device: status {st}")
    return out


def device_layout_bytes(dtype: int, in_feat: int, rows: int) -> int:
    return load_library().vtq_device_layout_bytes(dtype, in_feat, rows)
