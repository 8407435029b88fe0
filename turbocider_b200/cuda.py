"""ctypes binding of libturbocider_cuda.so (include/turbocider_cuda.h).

This is the Python face of the C ABI, in the style of the reference's own
ctypes-driven op tests (tests/native/test_gguf_execution.py:67-85).  Device
buffers are torch tensors (PyTorch is used for device memory and streams
only); every computation runs in the CUDA library.  There is no CPU
fallback: loading fails loudly when the library is missing.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

# TURBOCIDER_CHECKED=1 loads the bounds-checked build (-DTC_BOUNDS_CHECK:
# out-of-range indices set STATUS_BOUNDS instead of faulting).
LIB_PATH = Path(__file__).resolve().parent / ("libturbocider_cuda_checked.so"
                                             if os.environ.get("TURBOCIDER_CHECKED") == "1"
                                             else "libturbocider_cuda.so")

Q4_K, Q5_K, Q6_K = 12, 13, 14
F32, F16, BF16 = 0, 1, 2
STAGE_BF16, STAGE_F16, STAGE_F16_X16 = 0, 1, 2
STATUS_NONFINITE_SCALE, STATUS_F16_OVERFLOW, STATUS_TIMEOUT, STATUS_GEOMETRY, STATUS_BF16_OVERFLOW = 1, 2, 4, 8, 16
STATUS_BOUNDS = 32
EPI_BIAS, EPI_GELU_TANH, EPI_GELU_ERF, EPI_SWIGLU, EPI_GATE_RESIDUAL = 1, 2, 4, 8, 16
BLOCK_BYTES = {Q4_K: 144, Q5_K: 176, Q6_K: 210}

_lib = None


class BackendError(RuntimeError):
    """A failed C-ABI call (status 1); the message is tc_cuda_last_error()."""


class DecodeError(BackendError):
    """Mirror of tc::gguf::DecodeError (reference native/core/gguf_decode.hpp:10-16)."""


class Cancelled(BackendError):
    """A call stopped by its cancel flag (status TC_CUDA_CANCELLED = 2; the
    reference's tc::Cancelled, native/core/common.hpp:19-21)."""


class CancelFlag:
    """A caller-owned cancel flag (int32, nonzero = cancel) for the calls that
    take one: tc_gguf_read, tc_relayout_host, tc_cuda_weight_load_gguf and
    LayerStream.  Thread-safe to set from another thread while a call runs
    (the reference's std::atomic<bool> cancel, gguf_decode.cpp:44-47)."""

    def __init__(self):
        self._v = C.c_int32(0)

    def set(self):
        self._v.value = 1

    def clear(self):
        self._v.value = 0

    @property
    def is_set(self) -> bool:
        return self._v.value != 0

    @property
    def pointer(self):
        return C.byref(self._v)


def _cancel_ptr(cancel):
    return cancel.pointer if cancel is not None else None


class LoadStats(C.Structure):
    """struct tc_gguf_load_stats."""
    _fields_ = [("bytes", C.c_uint64), ("chunks", C.c_uint64), ("seconds", C.c_double),
                ("read_seconds", C.c_double), ("wait_seconds", C.c_double)]


_vp, _u32, _u64, _i32 = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int32


class Epilogue(C.Structure):
    """struct tc_epilogue (include/turbocider_cuda.h)."""
    _fields_ = [("flags", _u32), ("n_gate_rows", _u32), ("bias", _vp), ("bias_up_offset", _u64), ("gate", _vp),
                ("ld_gate", _u64), ("seg_gate", C.POINTER(_i32)), ("residual", _vp), ("ld_residual", _u64)]


EXPORTS = {
    # name: (restype, argtypes)
    "tc_cuda_abi_version": (_u32, []),
    "tc_cuda_last_error": (C.c_char_p, []),
    "tc_cuda_init": (C.c_int, [C.c_int, C.POINTER(_vp)]),
    "tc_cuda_free": (None, [_vp]),
    "tc_cuda_status": (C.c_int, [_vp, C.POINTER(_u32), C.c_int]),
    "tc_cuda_weight_upload": (C.c_int, [_vp, _u32, _u64, _u64, _vp, _u64, _u64, _u64, C.POINTER(_vp)]),
    "tc_cuda_weight_create": (C.c_int, [_vp, _u32, _u64, _u64, C.POINTER(_vp)]),
    "tc_cuda_weight_fill_device": (C.c_int, [_vp, _vp, _vp, _u64, _vp]),
    "tc_cuda_weight_free": (None, [_vp]),
    "tc_cuda_weight_info": (C.c_int, [_vp, C.POINTER(_u32), C.POINTER(_u64), C.POINTER(_u64), C.POINTER(_u64)]),
    "tc_cuda_dequant": (C.c_int, [_vp, _vp, C.c_int, _vp, _u64, _vp]),
    "tc_cuda_decode": (C.c_int, [_vp, _u32, _vp, _u64, _u64, _u64, _u64, _u64, _u64, _u64, C.c_int, _vp, _u64,
                                 _u64, _u64, _vp]),
    "tc_cuda_decode_gather": (C.c_int, [_vp, _u32, _vp, _u64, _u64, _u64, _vp, _u64, _u64, _u64, C.c_int, _vp,
                                        _u64, _u64, _u64, _vp]),
    "tc_cuda_qlinear": (C.c_int, [_vp, C.POINTER(_vp), _u32, C.POINTER(_i32), C.POINTER(_i32), _u32, _vp, _vp,
                                  _u64, C.c_int, C.c_int, _vp]),
    "tc_cuda_qlinear_ex": (C.c_int, [_vp, C.POINTER(_vp), _u32, C.POINTER(_i32), C.POINTER(_i32), _u32, _vp, _vp,
                                     _u64, C.c_int, C.c_int, C.POINTER(Epilogue), _vp]),
    "tc_cuda_weight_upload_glu": (C.c_int, [_vp, _u32, _u64, _u64, _vp, _vp, _u64, _u64, _u64, C.POINTER(_vp)]),
    "tc_cuda_qlinear_gather": (C.c_int, [_vp, C.POINTER(_vp), _u32, C.POINTER(_i32), C.POINTER(_i32), _u32, _vp,
                                         _vp, _u64, C.c_int, C.c_int, C.POINTER(Epilogue), C.POINTER(_vp), _u32,
                                         _vp]),
    "tc_cuda_peer_alloc": (C.c_int, [_vp, _u64, C.POINTER(_vp), _vp]),
    "tc_cuda_peer_open": (C.c_int, [_vp, _vp, C.POINTER(_vp)]),
    "tc_cuda_peer_close": (C.c_int, [_vp, _vp]),
    "tc_cuda_peer_free": (C.c_int, [_vp, _vp]),
    "tc_cuda_peer_barrier": (C.c_int, [_vp, C.POINTER(_vp), _u32, _u32, _u32, _u32, _vp]),
    "tc_cuda_peer_push": (C.c_int, [_vp, _vp, C.POINTER(_vp), _u32, _u64, _u64, _u64, _u64, _vp]),
    "tc_cuda_set_push_fanout": (C.c_int, [_vp, C.c_int]),
    "tc_cuda_set_push_kernel": (C.c_int, [_vp, C.c_int]),
    "tc_cuda_set_path": (C.c_int, [_vp, C.c_int]),
    "tc_cuda_qlinear_batched": (C.c_int, [_vp, C.POINTER(_vp), _u32, _vp, _u32, C.POINTER(_vp), C.POINTER(_u64),
                                          C.c_int, _vp]),
    "tc_cuda_set_sm_limit": (C.c_int, [_vp, C.c_int]),
    "tc_cuda_qlinear_plan": (C.c_int, [_vp, _vp, _u32, C.c_int, C.POINTER(_u32), C.POINTER(_u32)]),
    "tc_quantize": (C.c_int, [_u32, _vp, _u64, _u64, _vp, _u64, C.c_int]),
    "tc_cuda_qlinear_small_static": (C.c_int, [_vp, _vp, _u32, _vp, _u64, C.c_int, _vp]),
    "tc_cuda_small_static_status": (C.c_int, [C.c_int, C.POINTER(_u32), C.c_int]),
    "tc_panel_bytes": (_u64, [_u32, _u64, _u64]),
    "tc_relayout_host": (C.c_int, [_u32, _vp, _u64, _u64, _u64, _u64, _u64, _vp, _u64, C.c_int, _vp]),
    "tc_cuda_weight_copy_panels": (C.c_int, [_vp, _vp, _vp, _u64, _vp]),
    "tc_gguf_open": (C.c_int, [C.c_char_p, C.c_char_p, C.POINTER(_vp)]),
    "tc_gguf_close": (None, [_vp]),
    "tc_gguf_info": (C.c_int, [_vp, C.POINTER(_u32), C.POINTER(_u32), C.POINTER(_u64), C.POINTER(_u64),
                               C.POINTER(_u64)]),
    "tc_gguf_tensor": (C.c_int, [_vp, _u64, C.c_char_p, _u64, C.POINTER(_u32), C.POINTER(_u32), C.POINTER(_u64),
                                 C.POINTER(_u64), C.POINTER(_u64)]),
    "tc_gguf_find": (C.c_int, [_vp, C.c_char_p, C.POINTER(_u64)]),
    "tc_gguf_meta": (C.c_int, [_vp, C.c_char_p, C.POINTER(_u32), C.POINTER(_u64), C.POINTER(C.c_int64),
                               C.POINTER(C.c_double), C.c_char_p, _u64, C.POINTER(_u64)]),
    "tc_gguf_read": (C.c_int, [_vp, _u64, _u64, _u64, _vp, _u64, _vp]),
    "tc_cuda_weight_load_gguf": (C.c_int, [_vp, _vp, _u64, _u64, _u64, _u64, _vp, C.POINTER(_vp),
                                           C.POINTER(LoadStats)]),
    "tc_gguf_validate_split": (C.c_int, [C.POINTER(_vp), _u32]),
}


def lib() -> C.CDLL:
    """Load the backend library (built in-tree by turbocider_b200.build)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing: run `python -m turbocider_b200.build` "
                              "(the CUDA backend has no CPU fallback)")
        handle = C.CDLL(str(LIB_PATH))
        for name, (res, args) in EXPORTS.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def _check(rc: int, cls=BackendError):
    if rc == 2:
        raise Cancelled(lib().tc_cuda_last_error().decode())
    if rc != 0:
        raise cls(lib().tc_cuda_last_error().decode())


def _stream_ptr(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return getattr(stream, "cuda_stream", stream)


def quantize(ggml_type: int, w: np.ndarray, threads: int | None = None) -> np.ndarray:
    """Quantise a fp32 [rows, cols] matrix to raw GGUF blocks (uint8 array)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    out = np.empty(rows * (cols // 256) * BLOCK_BYTES[ggml_type], dtype=np.uint8)
    rc = lib().tc_quantize(ggml_type, w.ctypes.data, rows, cols, out.ctypes.data, out.nbytes,
                           threads or os.cpu_count() or 1)
    if rc != 0:
        raise BackendError("tc_quantize rejected the input (type, shape or nonfinite values)")
    return out


def panel_bytes(ggml_type: int, n: int, k: int) -> int:
    """Bytes of the panel layout of an [n, k] weight (0 = unsupported)."""
    return int(lib().tc_panel_bytes(ggml_type, n, k))


def relayout_host(ggml_type: int, raw, n: int, k: int, n_begin: int = 0, n_count: int = 0, out=None,
                  threads: int | None = None, cancel: CancelFlag | None = None):
    """Panel layout of rows [n_begin, +n_count) of a raw GGUF matrix, built on
    the CPU (uint8 numpy array in, uint8 numpy array or pinned torch tensor
    out).  Raises Cancelled when `cancel` is set while it runs."""
    raw = np.ascontiguousarray(np.frombuffer(raw, dtype=np.uint8) if isinstance(raw, (bytes, bytearray))
                               else raw).view(np.uint8).reshape(-1)
    rows = n_count or (n - n_begin)
    size = panel_bytes(ggml_type, rows, k)
    if out is None:
        out = np.empty(size, dtype=np.uint8)
    ptr = out.data_ptr() if hasattr(out, "data_ptr") else out.ctypes.data
    cap = out.numel() if hasattr(out, "numel") else out.nbytes
    _check(lib().tc_relayout_host(ggml_type, raw.ctypes.data, raw.nbytes, n, k, n_begin, n_count, ptr, cap,
                                  threads or os.cpu_count() or 1, _cancel_ptr(cancel)), DecodeError)
    return out


class Context:
    """A device context: status word and workspace on one GPU."""

    def __init__(self, device: int = 0):
        self._h = _vp()
        _check(lib().tc_cuda_init(device, C.byref(self._h)))
        self.device = device

    @property
    def handle(self):
        return self._h

    def status(self, clear: bool = True) -> int:
        bits = _u32()
        _check(lib().tc_cuda_status(self._h, C.byref(bits), int(clear)))
        return bits.value

    def set_path(self, path: int):
        _check(lib().tc_cuda_set_path(self._h, path))

    def set_sm_limit(self, sms: int):
        """SMs the tensor-core GEMM may occupy (0 = all)."""
        _check(lib().tc_cuda_set_sm_limit(self._h, sms))

    def plan(self, weight, m: int, stage: int = STAGE_BF16) -> tuple[int, int]:
        """(kernel family, K splits) a one-segment call with m rows would use:
        kernel 1 GEMV, 2 2-CTA GEMM, 3 one-CTA GEMM, 4 dense."""
        kern, split = _u32(), _u32()
        _check(lib().tc_cuda_qlinear_plan(self._h, weight.handle, m, stage, C.byref(kern), C.byref(split)))
        return kern.value, split.value

    def set_push_fanout(self, streams: int):
        """Peer pushes spread over `streams` side streams (>= 2) or back to
        back on the caller's stream (0 / 1, the default)."""
        _check(lib().tc_cuda_set_push_fanout(self._h, int(streams)))

    def set_push_kernel(self, ctas: int):
        """Peer pushes by a kernel of `ctas` 128-thread blocks (the SMs store
        over NVLink) for 16-byte-aligned regions; 0 (the default): by the
        copy engines."""
        _check(lib().tc_cuda_set_push_kernel(self._h, int(ctas)))

    def close(self):
        if self._h:
            lib().tc_cuda_free(self._h)
            self._h = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Weight:
    """A K-quant weight resident in HBM (panel layout)."""

    def __init__(self, ctx: Context, handle, glu: bool = False):
        self.ctx, self._h = ctx, handle
        t, n, k, b = _u32(), _u64(), _u64(), _u64()
        _check(lib().tc_cuda_weight_info(handle, C.byref(t), C.byref(n), C.byref(k), C.byref(b)))
        self.ggml_type, self.n, self.k, self.device_bytes = t.value, n.value, k.value, b.value
        self.glu = glu
        self.n_out = n.value // 2 if glu else n.value   # output columns

    @classmethod
    def upload_glu(cls, ctx: Context, ggml_type: int, f: int, k: int, gate_raw, up_raw, col_begin: int = 0,
                   col_count: int = 0):
        """Gate and up halves of a SwiGLU projection ([f, k] raw GGUF rows each)
        as one interleaved weight for the fused SwiGLU epilogue."""
        def flat(r):
            return np.ascontiguousarray(np.frombuffer(r, dtype=np.uint8) if isinstance(r, (bytes, bytearray))
                                        else r).view(np.uint8).reshape(-1)
        g, u = flat(gate_raw), flat(up_raw)
        h = _vp()
        _check(lib().tc_cuda_weight_upload_glu(ctx.handle, ggml_type, f, k, g.ctypes.data, u.ctypes.data,
                                               min(g.nbytes, u.nbytes), col_begin, col_count, C.byref(h)),
               DecodeError)
        return cls(ctx, h, glu=True)

    @classmethod
    def upload(cls, ctx: Context, ggml_type: int, n: int, k: int, raw, n_begin: int = 0, n_count: int = 0):
        raw = np.ascontiguousarray(np.frombuffer(raw, dtype=np.uint8) if isinstance(raw, (bytes, bytearray))
                                   else raw).view(np.uint8).reshape(-1)
        h = _vp()
        _check(lib().tc_cuda_weight_upload(ctx.handle, ggml_type, n, k, raw.ctypes.data, raw.nbytes, n_begin,
                                           n_count, C.byref(h)), DecodeError)
        return cls(ctx, h)

    @classmethod
    def load_gguf(cls, ctx: Context, file: "GGUFFile", name_or_index, n_begin: int = 0, n_count: int = 0,
                  chunk_bytes: int = 0, cancel: CancelFlag | None = None):
        """Stream a K-quant tensor (or a row shard of it) from a GGUF file into
        HBM with read-ahead (tc_cuda_weight_load_gguf).  Returns (Weight,
        stats dict); raises Cancelled when `cancel` is set while it runs."""
        idx = name_or_index if isinstance(name_or_index, int) else file.tensor(name_or_index)["index"]
        h = _vp()
        st = LoadStats()
        _check(lib().tc_cuda_weight_load_gguf(ctx.handle, file._h, idx, n_begin, n_count, chunk_bytes,
                                              _cancel_ptr(cancel), C.byref(h), C.byref(st)), DecodeError)
        stats = {f: getattr(st, f) for f, _ in LoadStats._fields_}
        return cls(ctx, h), stats

    @classmethod
    def create(cls, ctx: Context, ggml_type: int, n: int, k: int):
        h = _vp()
        _check(lib().tc_cuda_weight_create(ctx.handle, ggml_type, n, k, C.byref(h)))
        return cls(ctx, h)

    def copy_panels(self, panels, stream=None):
        """Asynchronous copy of panel-layout bytes (tc_relayout_host output,
        pinned host or device torch uint8 tensor) into this weight."""
        _check(lib().tc_cuda_weight_copy_panels(self.ctx.handle, self._h, panels.data_ptr(), panels.numel(),
                                                _stream_ptr(stream)))

    def fill_device(self, raw_device, stream=None):
        """Re-layout raw GGUF rows already in device memory (torch uint8 tensor)."""
        _check(lib().tc_cuda_weight_fill_device(self.ctx.handle, self._h, raw_device.data_ptr(),
                                                raw_device.numel(), _stream_ptr(stream)))

    @property
    def handle(self):
        return self._h

    def free(self):
        if self._h:
            lib().tc_cuda_weight_free(self._h)
            self._h = _vp()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def dequant(ctx: Context, w: Weight, dtype: int = BF16, out=None, stream=None):
    """Dequantise an uploaded weight into a dense torch tensor [n, k]."""
    import torch
    tdt = {F32: torch.float32, F16: torch.float16, BF16: torch.bfloat16}[dtype]
    if out is None:
        out = torch.empty((w.n, w.k), dtype=tdt, device=f"cuda:{ctx.device}")
    _check(lib().tc_cuda_dequant(ctx.handle, w.handle, dtype, out.data_ptr(), out.stride(0), _stream_ptr(stream)))
    return out


def decode(ctx: Context, ggml_type: int, source, source_rows: int, source_columns: int, row_begin: int, rows: int,
           column_begin: int, columns: int, dtype: int, target, row_stride: int, column_stride: int,
           stream=None, check: bool = True):
    """Device mirror of decode_cpu_into on raw GGUF bytes (torch uint8 tensors).

    Raises DecodeError with the reference's message for geometry errors, and
    (when check=True, which synchronises) for nonfinite scales / fp16
    overflow detected by the kernel.
    """
    _check(lib().tc_cuda_decode(ctx.handle, ggml_type, source.data_ptr(), source.numel() * source.element_size(),
                                source_rows, source_columns, row_begin, rows, column_begin, columns, dtype,
                                target.data_ptr(), target.numel() * target.element_size(), row_stride,
                                column_stride, _stream_ptr(stream)), DecodeError)
    if check:
        bits = ctx.status(clear=True)
        if bits & STATUS_NONFINITE_SCALE:
            # The reference's checked copy (same floating type as the target,
            # contiguous columns) words this error differently from its
            # decoder (gguf_decode.cpp:136-158 vs :43).
            same = (ggml_type, dtype) in ((0, F32), (1, F16), (30, BF16))
            if same and column_stride == (4 if dtype == F32 else 2):
                raise DecodeError("nonfinite source float")
            raise DecodeError("nonfinite weight/scale or conversion overflow")
        if bits & STATUS_F16_OVERFLOW:
            raise DecodeError("FP16 conversion overflow")
        if bits & STATUS_BF16_OVERFLOW:
            raise DecodeError("BF16 conversion overflow")


def decode_gather(ctx: Context, ggml_type: int, source, source_rows: int, source_columns: int, indices,
                  column_begin: int, columns: int, dtype: int, target, row_stride: int, column_stride: int,
                  stream=None, check: bool = True):
    """Device mirror of decode_cpu_gather: target row r = source row
    indices[r] (device int64 / uint64 tensor).  Raises DecodeError with the
    reference's messages; with check=True (synchronises) also for an index
    past the matrix and for value errors detected by the kernel."""
    _check(lib().tc_cuda_decode_gather(ctx.handle, ggml_type, source.data_ptr(),
                                       source.numel() * source.element_size(), source_rows, source_columns,
                                       indices.data_ptr(), indices.numel(), column_begin, columns, dtype,
                                       target.data_ptr(), target.numel() * target.element_size(), row_stride,
                                       column_stride, _stream_ptr(stream)), DecodeError)
    if check:
        bits = ctx.status(clear=True)
        if bits & STATUS_GEOMETRY:
            raise DecodeError("gather row out of bounds")
        if bits & STATUS_NONFINITE_SCALE:
            raise DecodeError("nonfinite weight/scale or conversion overflow")
        if bits & STATUS_F16_OVERFLOW:
            raise DecodeError("FP16 conversion overflow")
        if bits & STATUS_BF16_OVERFLOW:
            raise DecodeError("BF16 conversion overflow")


def _torch_dtype(out_dtype: int):
    import torch
    return {F32: torch.float32, F16: torch.float16, BF16: torch.bfloat16}[out_dtype]


def qlinear(ctx: Context, weights, x, seg_offsets=None, seg_weight=None, out_dtype: int = BF16,
            stage: int = STAGE_BF16, out=None, stream=None, bias=None, activation: str | None = None,
            gate=None, residual=None, seg_gate=None, bias_up_offset: int | None = None, peers=None):
    """Y = X * W^T through tc_cuda_qlinear_ex.  `weights` is a Weight or a list
    of them; seg_offsets / seg_weight describe ragged request segments along M.

    Fused epilogue (all optional; f32 device tensors unless noted):
      bias        [rows] (SwiGLU weight: gate biases then up biases, up at
                  bias_up_offset, default n_out);
      activation  "gelu_tanh" | "gelu_erf" (SwiGLU weights always apply
                  silu(gate) * up);
      gate, residual  y = residual + gate[seg_gate[s]] * t; gate [G, n_out]
                  f32, residual [M, n_out] in the output dtype (may be `out`).
    peers: device addresses of replicas of `out` on other ranks (same layout;
    tc_cuda_qlinear_gather) -- every output is also stored there.
    """
    import torch
    ws = weights if isinstance(weights, (list, tuple)) else [weights]
    m = x.shape[0]
    if seg_offsets is None:
        seg_offsets = [0, m]
    seg_offsets = list(seg_offsets)
    n_seg = len(seg_offsets) - 1
    offs = (_i32 * len(seg_offsets))(*seg_offsets)
    sw = (_i32 * n_seg)(*seg_weight) if seg_weight is not None else None
    handles = (_vp * len(ws))(*[w.handle for w in ws])
    n_out = getattr(ws[0], "n_out", ws[0].n)
    if out is None:
        out = torch.empty((m, n_out), dtype=_torch_dtype(out_dtype), device=x.device)
    epi = Epilogue()
    if bias is not None:
        epi.flags |= EPI_BIAS
        epi.bias = bias.data_ptr()
        epi.bias_up_offset = n_out if bias_up_offset is None else bias_up_offset
    if activation is not None:
        epi.flags |= {"gelu_tanh": EPI_GELU_TANH, "gelu_erf": EPI_GELU_ERF}[activation]
    if getattr(ws[0], "glu", False):
        epi.flags |= EPI_SWIGLU
    if gate is not None or residual is not None:
        epi.flags |= EPI_GATE_RESIDUAL
        epi.gate = gate.data_ptr() if gate is not None else None
        epi.ld_gate = gate.stride(0) if gate is not None else 0
        epi.n_gate_rows = gate.shape[0] if gate is not None else 0
        epi.residual = residual.data_ptr() if residual is not None else None
        epi.ld_residual = residual.stride(0) if residual is not None else 0
        if seg_gate is not None:
            epi.seg_gate = (_i32 * n_seg)(*seg_gate)
    peers = list(peers or [])
    pv = (_vp * max(1, len(peers)))(*peers) if peers else None
    _check(lib().tc_cuda_qlinear_gather(ctx.handle, handles, len(ws), offs, sw, n_seg, x.data_ptr(),
                                        out.data_ptr(), out.stride(0), out_dtype, stage,
                                        C.byref(epi) if epi.flags else None, pv, len(peers), _stream_ptr(stream)))
    return out


def qlinear_batched(ctx: Context, weights, x, out_dtype: int = BF16, outs=None, stream=None):
    """[X * W_i^T for W_i in weights] in one GEMV launch per weight type (1..16
    rows of bf16 X, weights sharing K)."""
    import torch
    if outs is None:
        outs = [torch.empty((x.shape[0], w.n), dtype=_torch_dtype(out_dtype), device=x.device) for w in weights]
    handles = (_vp * len(weights))(*[w.handle for w in weights])
    ys = (_vp * len(outs))(*[o.data_ptr() for o in outs])
    lds = (_u64 * len(outs))(*[o.stride(0) for o in outs])
    _check(lib().tc_cuda_qlinear_batched(ctx.handle, handles, len(weights), x.data_ptr(), x.shape[0], ys, lds,
                                         out_dtype, _stream_ptr(stream)))
    return outs


def qlinear_small_static(weight: Weight, x, out_dtype: int = BF16, out=None, stream=None):
    """Y = X * W^T for 1..16 rows of X through the allocation-free entry point
    (static device scratch instead of a context workspace)."""
    import torch
    if out is None:
        out = torch.empty((x.shape[0], weight.n), dtype=_torch_dtype(out_dtype), device=x.device)
    _check(lib().tc_cuda_qlinear_small_static(weight.handle, x.data_ptr(), x.shape[0], out.data_ptr(),
                                              out.stride(0), out_dtype, _stream_ptr(stream)))
    return out


def small_static_status(device: int = 0, clear: bool = True) -> int:
    """TC_STATUS_* bits accumulated by qlinear_small_static on `device`
    (synchronises the device; clear resets them)."""
    bits = _u32()
    _check(lib().tc_cuda_small_static_status(device, C.byref(bits), int(clear)))
    return bits.value


class GGUFError(BackendError):
    """A GGUF file the reader rejects (message as the reference's gguf_invalid: ...)."""


class GGUFFile:
    """A parsed GGUF container (tc_gguf_*): directory, metadata lookup and
    row-range payload reads into host memory."""

    def __init__(self, path, limit: str | None = None):
        self._h = _vp()
        rc = lib().tc_gguf_open(str(path).encode(), limit.encode() if limit else None, C.byref(self._h))
        _check(rc, GGUFError)
        v, a, n, d, nm = _u32(), _u32(), _u64(), _u64(), _u64()
        _check(lib().tc_gguf_info(self._h, C.byref(v), C.byref(a), C.byref(n), C.byref(d), C.byref(nm)), GGUFError)
        self.version, self.alignment, self.data_offset = v.value, a.value, d.value
        self.tensors = [self._tensor(i) for i in range(n.value)]
        self.n_metadata = nm.value

    def _tensor(self, i: int) -> dict:
        name = C.create_string_buffer(4096)
        t, r, off, nb = _u32(), _u32(), _u64(), _u64()
        dims = (_u64 * 4)()
        _check(lib().tc_gguf_tensor(self._h, i, name, 4096, C.byref(t), C.byref(r), dims, C.byref(off),
                                    C.byref(nb)), GGUFError)
        d = list(dims)[:r.value]
        rows = 1
        for x in d[1:]:
            rows *= x
        return {"name": name.value.decode(), "type": t.value, "dims": d, "rows": rows, "columns": d[0],
                "file_offset": off.value, "bytes": nb.value}

    def tensor(self, name: str) -> dict:
        idx = _u64()
        _check(lib().tc_gguf_find(self._h, name.encode(), C.byref(idx)), GGUFError)
        return dict(self.tensors[idx.value], index=idx.value)

    def meta(self, key: str):
        t, u, i, f, cnt = _u32(), _u64(), C.c_int64(), C.c_double(), _u64()
        text = C.create_string_buffer(1 << 20)
        _check(lib().tc_gguf_meta(self._h, key.encode(), C.byref(t), C.byref(u), C.byref(i), C.byref(f), text,
                                  1 << 20, C.byref(cnt)), GGUFError)
        kind = t.value
        if kind == 8:
            return text.value.decode()
        if kind == 9:
            return ("array", cnt.value)
        if kind in (6, 12):
            return f.value
        if kind in (1, 3, 5, 11):
            return i.value
        return u.value

    def read(self, name_or_index, row_begin: int = 0, rows: int | None = None, out=None,
             cancel: CancelFlag | None = None) -> np.ndarray:
        """Raw block bytes of rows [row_begin, +rows) into `out` (a uint8
        numpy array or a pinned torch uint8 tensor; allocated if None).
        Raises Cancelled when `cancel` is set while it reads."""
        info = self.tensors[name_or_index] if isinstance(name_or_index, int) else self.tensor(name_or_index)
        idx = name_or_index if isinstance(name_or_index, int) else info["index"]
        rows = info["rows"] - row_begin if rows is None else rows
        nbytes = info["bytes"] // info["rows"] * rows
        if out is None:
            out = np.empty(nbytes, dtype=np.uint8)
        ptr = out.data_ptr() if hasattr(out, "data_ptr") else out.ctypes.data
        size = out.numel() if hasattr(out, "numel") else out.nbytes
        _check(lib().tc_gguf_read(self._h, idx, row_begin, rows, ptr, size, _cancel_ptr(cancel)), GGUFError)
        return out

    @staticmethod
    def validate_split(files) -> None:
        arr = (_vp * len(files))(*[f._h for f in files])
        _check(lib().tc_gguf_validate_split(arr, len(files)), GGUFError)

    def close(self):
        if self._h:
            lib().tc_gguf_close(self._h)
            self._h = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
