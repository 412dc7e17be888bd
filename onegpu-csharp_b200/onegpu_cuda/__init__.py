"""Host-side mirror of onegpu's quantized-matmul API over the C ABI of libonegpu_cuda.so.

The reference (recursive-ai-oss/onegpu-csharp) exposes this path as C# classes: ``Int8Gemm`` with ``EncodeInt32`` /
``EncodeFloat`` / ``EncodeRequantized`` (src/RecursiveAI.OneGpu.Kernels/Int8Gemm.cs:124-683), ``Int8GemmProblem``
(:43-95), ``Int8Operand<T>`` (:28), ``Int8Scratch`` (:37), ``Int8GemmOptions`` (:7-21) and ``DynamicQuantizeKernels``
(src/RecursiveAI.OneGpu.Kernels/DynamicQuantizeKernels.cs:20-110), written against ``GpuDevice`` / ``GpuBuffer<T>`` /
``GpuCommandEncoder`` (src/RecursiveAI.OneGpu/). This module keeps those names, argument meanings and error behaviour
(``GpuKernelShapeException`` with ``operation`` and ``argument``; ``GpuUnsupportedException``; ``ValueError`` for a
missing argument where C# throws ``ArgumentNullException``) and calls the CUDA library through ctypes. All work runs in
the CUDA kernels of the library; there is no fallback: importing this module fails when the library is missing.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import Optional

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY_PATH = os.path.join(os.path.dirname(_HERE), "lib", "libonegpu_cuda.so")

if not os.path.exists(LIBRARY_PATH):
    raise OSError(f"libonegpu_cuda.so is not built ({LIBRARY_PATH}); run `make -C onegpu-csharp_b200`")

_lib = ctypes.CDLL(LIBRARY_PATH)

# ---- C structures (include/onegpu_cuda.h) ------------------------------------------------------------------------

OG_OK = 0
OG_ERROR_SHAPE = 1
OG_ERROR_UNSUPPORTED = 2
OG_ERROR_ARGUMENT_NULL = 3
OG_ERROR_ARGUMENT_RANGE = 4
OG_ERROR_OUT_OF_MEMORY = 5
OG_ERROR_DEVICE_LOST = 6
OG_ERROR_COMMAND_FAILED = 7
OG_ERROR_CUDA = 8
OG_ERROR_INVALID_HANDLE = 9

U8, S8, I32, F32, F16, U32, U16, I16, I64 = 0, 1, 2, 3, 4, 5, 6, 7, 8
_NP = {U8: np.uint8, S8: np.int8, I32: np.int32, F32: np.float32, F16: np.float16, U32: np.uint32, U16: np.uint16,
       I16: np.int16, I64: np.int64}
_FROM_NP = {np.dtype(v): k for k, v in _NP.items()}

KERNEL_AUTO, KERNEL_TENSOR_CORE, KERNEL_PORTABLE = 0, 1, 2


class og_error_info(ctypes.Structure):
    _fields_ = [("status", ctypes.c_int32), ("operation", ctypes.c_char * 64), ("argument", ctypes.c_char * 64),
                ("message", ctypes.c_char * 512), ("capability", ctypes.c_char * 64),
                ("expected", ctypes.c_char * 128), ("actual", ctypes.c_char * 128)]


class og_buffer(ctypes.Structure):
    _fields_ = [("ptr", ctypes.c_void_p), ("length", ctypes.c_int64), ("type", ctypes.c_int32)]


class og_operand(ctypes.Structure):
    _fields_ = [("buffer", og_buffer), ("offset", ctypes.c_int32), ("is_vector", ctypes.c_int32)]


class og_device_info(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 256), ("ordinal", ctypes.c_int32), ("sm_count", ctypes.c_int32),
                ("cc_major", ctypes.c_int32), ("cc_minor", ctypes.c_int32), ("total_memory", ctypes.c_int64),
                ("max_shared_memory_per_block", ctypes.c_int32), ("tensor_core_i8", ctypes.c_int32)]


class og_int8_gemm_problem(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int32) for name in
                ("m", "n", "k", "batch", "transpose_b", "lda", "ldb", "offset_a", "offset_b", "offset_c",
                 "stride_a", "stride_b")]


class og_int8_gemm_options(ctypes.Structure):
    _fields_ = [("allow_packed_dot", ctypes.c_int32), ("kernel", ctypes.c_int32), ("tile", ctypes.c_int32),
                ("stream_k", ctypes.c_int32)]


_P = ctypes.c_void_p
_PP = ctypes.POINTER(ctypes.c_void_p)
_BUF = ctypes.POINTER(og_buffer)
_OPD = ctypes.POINTER(og_operand)
_PROB = ctypes.POINTER(og_int8_gemm_problem)

# x, offset, shape, rank, axis, per_axis, scale, offset, zero point, offset, output, offset
_QUANT_ARGS = [_BUF, ctypes.c_int32, ctypes.POINTER(ctypes.c_int32), ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
               _BUF, ctypes.c_int32, _BUF, ctypes.c_int32, _BUF, ctypes.c_int32]

EXPORTS = {
    "og_last_error": [ctypes.POINTER(og_error_info)],
    "og_device_count": [ctypes.POINTER(ctypes.c_int32)],
    "og_device_create": [ctypes.c_int32, _PP],
    "og_device_destroy": [_P],
    "og_device_info_get": [_P, ctypes.POINTER(og_device_info)],
    "og_device_wait_idle": [_P],
    "og_device_watchdog_selftest": [_P, ctypes.c_uint32],
    "og_device_stream": [_P, _PP],
    "og_device_set_stream": [_P, _P],
    "og_buffer_alloc": [_P, ctypes.c_uint64, _PP],
    "og_buffer_free": [_P, _P],
    "og_buffer_write": [_P, _P, _P, ctypes.c_uint64],
    "og_buffer_read": [_P, _P, _P, ctypes.c_uint64],
    "og_buffer_fill": [_P, _P, ctypes.c_int32, ctypes.c_uint64],
    "og_host_alloc": [ctypes.c_uint64, _PP],
    "og_host_free": [_P],
    "og_encoder_begin": [_P, _PP],
    "og_device_submit": [_P, _P],
    "og_encoder_discard": [_P],
    "og_encoder_dispatch_count": [_P, ctypes.POINTER(ctypes.c_int64)],
    "og_timestamps_create": [_P, ctypes.c_uint32, _PP],
    "og_timestamps_destroy": [_P],
    "og_encoder_timestamp": [_P, _P, ctypes.c_uint32],
    "og_device_timestamp": [_P, _P, ctypes.c_uint32],
    "og_device_capture_begin": [_P],
    "og_device_capture_end": [_P, _PP],
    "og_graph_launch": [_P],
    "og_graph_destroy": [_P],
    "og_timestamps_read": [_P, ctypes.c_uint32, ctypes.c_uint32, ctypes.POINTER(ctypes.c_double)],
    "og_int8_gemm_create": [_P, ctypes.POINTER(og_int8_gemm_options), _PP],
    "og_int8_gemm_destroy": [_P],
    "og_int8_gemm_variant": [_P, ctypes.c_char_p, ctypes.c_uint64],
    "og_int8_gemm_last_kernel": [_P, ctypes.c_char_p, ctypes.c_uint64],
    "og_int8_gemm_scratch_elements": [_PROB],
    "og_int8_gemm_reserve_scratch": [_P, ctypes.c_int64],
    "og_int8_gemm_bind_groups_created": [_P, ctypes.POINTER(ctypes.c_int32)],
    "og_int8_gemm_encode_int32": [_P, _P, _PROB, _BUF, _BUF, _BUF, _OPD, _OPD, _OPD],
    "og_int8_gemm_encode_float": [_P, _P, _PROB, _BUF, _BUF, _BUF, _OPD, _OPD, _OPD, _OPD, _OPD],
    "og_int8_gemm_encode_requantized": [_P, _P, _PROB, _BUF, _BUF, _BUF, _OPD, ctypes.c_int32, _OPD, _OPD, _OPD,
                                        _OPD],
    "og_int8_gemm_encode_dequantize": [_P, _P, _PROB, _BUF, _BUF, _BUF, _OPD, _OPD, _OPD, _OPD, _OPD, _OPD],
    "og_int8_gemm_check_dequantize": [_PROB, _BUF, _BUF, _BUF, _OPD, _OPD, _OPD, _OPD, _OPD, _OPD],
    "og_int8_gemm_int32_noalloc": [_P, _PROB, _BUF, _BUF, _BUF, _OPD, _OPD, _OPD],
    "og_int8_gemm_noalloc_status": [_P],
    "og_int8_gemm_noalloc_watchdog_selftest": [_P, ctypes.c_uint32],
    "og_int8_gemm_check_int32": [_PROB, _BUF, _BUF, _BUF, _OPD, _OPD, _OPD],
    "og_int8_gemm_check_float": [_PROB, _BUF, _BUF, _BUF, _OPD, _OPD, _OPD, _OPD, _OPD],
    "og_int8_gemm_check_requantized": [_PROB, _BUF, _BUF, _BUF, _OPD, ctypes.c_int32, _OPD, _OPD, _OPD, _OPD],
    "og_dynamic_quantize_create": [_P, _PP],
    "og_dynamic_quantize_destroy": [_P],
    "og_dynamic_quantize_encode": [_P, _P, _BUF, ctypes.c_int32, ctypes.c_int32, _BUF, ctypes.c_int32, _BUF,
                                   ctypes.c_int32, _BUF, ctypes.c_int32],
    "og_dynamic_quantize_check": [_BUF, ctypes.c_int32, ctypes.c_int32, _BUF, ctypes.c_int32, _BUF, ctypes.c_int32,
                                  _BUF, ctypes.c_int32],
    "og_buffer_write_async": [_P, _P, _P, ctypes.c_uint64],
    "og_buffer_read_async": [_P, _P, _P, ctypes.c_uint64, _PP],
    "og_readback_wait": [_P],
    "og_dequantize_create": [_P, _PP],
    "og_dequantize_destroy": [_P],
    "og_dequantize_encode": [_P, _P] + _QUANT_ARGS,
    "og_dequantize_encode_quantize": [_P, _P] + _QUANT_ARGS,
    "og_dequantize_check": _QUANT_ARGS,
    "og_dequantize_check_quantize": _QUANT_ARGS,
    "og_conv_integer_create": [_P, _P, _PP],
    "og_conv_integer_destroy": [_P],
    "og_conv_integer_variant": [_P, ctypes.c_char_p, ctypes.c_uint64],
    "og_conv_integer_bind_groups_created": [_P, ctypes.POINTER(ctypes.c_int32)],
    "og_conv_integer_scratch_bytes_per_image": [_P, ctypes.POINTER(ctypes.c_int64)],
    "og_conv_integer_encode": [_P, _P, _P, _BUF, _BUF, _BUF, _OPD, _OPD, _BUF, ctypes.c_int32],
    "og_conv_integer_check": [_P, _BUF, _BUF, _BUF, _OPD, _OPD, _BUF, ctypes.c_int32],
    "og_comm_unique_id": [_P],
    "og_comm_create": [_P, ctypes.c_int32, ctypes.c_int32, _P, _PP],
    "og_comm_destroy": [_P],
    "og_comm_gather_columns": [_P, _P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _P, _P, ctypes.c_int32],
    "og_comm_all_gather": [_P, _P, ctypes.c_uint64, _P],
}

for _name, _args in EXPORTS.items():
    _fn = getattr(_lib, _name)
    _fn.argtypes = _args
    _fn.restype = ctypes.c_int64 if _name == "og_int8_gemm_scratch_elements" else ctypes.c_int


# ---- exceptions ----------------------------------------------------------------------------------------------------

class GpuException(Exception):
    """Base of the errors the library reports."""


class GpuKernelShapeException(GpuException, ValueError):
    """A shape, stride, offset, range or operand type is invalid (GpuKernelShapeException.cs:7-25)."""

    def __init__(self, operation: str, argument: str, message: str):
        super().__init__(f"{operation}: {argument}: {message}")
        self.operation = operation
        self.argument = argument


class GpuUnsupportedException(GpuException):
    """The device cannot run what was asked (src/RecursiveAI.OneGpu/GpuDevice.cs:283-312)."""

    def __init__(self, message: str, capability: str, expected: str, actual: str):
        super().__init__(message)
        self.capability = capability
        self.expected = expected
        self.actual = actual


class ArgumentNullException(GpuException, ValueError):
    def __init__(self, argument: str, message: str):
        super().__init__(f"{message} (Parameter '{argument}')")
        self.argument = argument


class ArgumentOutOfRangeException(GpuException, ValueError):
    def __init__(self, argument: str, message: str):
        super().__init__(f"{argument}: {message}")
        self.argument = argument


class GpuOutOfMemoryException(GpuException, MemoryError):
    pass


class GpuDeviceLostException(GpuException):
    pass


class GpuCommandFailedException(GpuException):
    """A submission failed; ``reason`` is "Watchdog" when a kernel's bounded wait ran out (GpuDevice.cs:337-374)."""

    def __init__(self, message: str, reason: str = ""):
        super().__init__(message)
        self.reason = reason


def _raise(status: int) -> None:
    if status == OG_OK:
        return
    info = og_error_info()
    _lib.og_last_error(ctypes.byref(info))
    op, arg, msg = info.operation.decode(), info.argument.decode(), info.message.decode()
    if status == OG_ERROR_SHAPE:
        raise GpuKernelShapeException(op, arg, msg)
    if status == OG_ERROR_UNSUPPORTED:
        raise GpuUnsupportedException(f"{op}: {msg}", info.capability.decode(), info.expected.decode(),
                                      info.actual.decode())
    if status == OG_ERROR_ARGUMENT_NULL:
        raise ArgumentNullException(arg, msg)
    if status == OG_ERROR_ARGUMENT_RANGE:
        raise ArgumentOutOfRangeException(arg, msg)
    if status == OG_ERROR_OUT_OF_MEMORY:
        raise GpuOutOfMemoryException(f"{op}: {msg}")
    if status == OG_ERROR_DEVICE_LOST:
        raise GpuDeviceLostException(f"{op}: {msg}")
    if status == OG_ERROR_COMMAND_FAILED:
        raise GpuCommandFailedException(f"{op}: {msg}", info.capability.decode())
    raise GpuException(f"status {status}: {op}: {msg}")


def _check(status: int) -> None:
    if status != OG_OK:
        _raise(status)


# ---- device, buffers, encoders, timestamps ---------------------------------------------------------------------------

def device_count() -> int:
    n = ctypes.c_int32(0)
    _check(_lib.og_device_count(ctypes.byref(n)))
    return n.value


class GpuBuffer:
    """A typed device buffer (GpuBuffer<T>): `length` elements of `dtype`, owned by the caller."""

    def __init__(self, device: "GpuDevice", dtype, length: int, ptr: Optional[int] = None, owned: bool = True):
        self.device = device
        self.dtype = np.dtype(dtype)
        self.type = _FROM_NP[self.dtype]
        self.length = int(length)
        self.nbytes = self.length * self.dtype.itemsize
        self._owned = owned and ptr is None
        if ptr is None:
            p = ctypes.c_void_p()
            _check(_lib.og_buffer_alloc(device.handle, max(self.nbytes, 16), ctypes.byref(p)))
            ptr = p.value
        self.ptr = ptr

    @property
    def Length(self) -> int:  # noqa: N802 - the reference's property name
        return self.length

    def ref(self) -> og_buffer:
        return og_buffer(self.ptr, self.length, self.type)

    def write(self, data: np.ndarray, offset: int = 0) -> None:
        a = np.ascontiguousarray(np.asarray(data).view(self.dtype).reshape(-1))
        if offset < 0 or offset + a.size > self.length:
            raise ValueError("write past the end of the buffer")
        _check(_lib.og_buffer_write(self.device.handle, self.ptr + offset * self.dtype.itemsize,
                                    a.ctypes.data, a.nbytes))
        self.device._keep.append(a)  # the upload is asynchronous: keep the source alive until the next wait

    def read(self, count: Optional[int] = None) -> np.ndarray:
        n = self.length if count is None else count
        out = np.empty(n, dtype=self.dtype)
        _check(_lib.og_buffer_read(self.device.handle, out.ctypes.data, self.ptr, out.nbytes))
        self.device._keep.clear()
        return out

    def fill(self, byte_value: int) -> None:
        _check(_lib.og_buffer_fill(self.device.handle, self.ptr, int(byte_value), self.nbytes))

    def dispose(self) -> None:
        if self._owned and self.ptr:
            _check(_lib.og_buffer_free(self.device.handle, self.ptr))
        self.ptr = 0

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.dispose()


class GpuCommandEncoder:
    """Records work; nothing runs until GpuDevice.submit (GpuDevice.cs:155-161)."""

    def __init__(self, device: "GpuDevice"):
        self.device = device
        h = ctypes.c_void_p()
        _check(_lib.og_encoder_begin(device.handle, ctypes.byref(h)))
        self.handle = h.value

    @property
    def dispatch_count(self) -> int:
        n = ctypes.c_int64(0)
        _check(_lib.og_encoder_dispatch_count(self.handle, ctypes.byref(n)))
        return n.value

    def write_timestamp(self, stamps: "GpuTimestampSet", index: int) -> None:
        _check(_lib.og_encoder_timestamp(self.handle, stamps.handle, index))


class GpuGraph:
    """A CUDA graph of submitted work (og_graph): launch() replays it on the device stream."""

    def __init__(self, device: "GpuDevice", handle: ctypes.c_void_p):
        self.device = device
        self.handle = handle

    def launch(self) -> None:
        _check(_lib.og_graph_launch(self.handle))

    def dispose(self) -> None:
        if self.handle:
            _check(_lib.og_graph_destroy(self.handle))
            self.handle = None


class GpuTimestampSet:
    def __init__(self, device: "GpuDevice", count: int):
        self.device = device
        self.count = count
        h = ctypes.c_void_p()
        _check(_lib.og_timestamps_create(device.handle, count, ctypes.byref(h)))
        self.handle = h.value

    def read(self, first: int = 0, count: Optional[int] = None) -> np.ndarray:
        n = self.count - first if count is None else count
        out = (ctypes.c_double * n)()
        _check(_lib.og_timestamps_read(self.handle, first, n, out))
        return np.array(out, dtype=np.float64)

    def dispose(self) -> None:
        if self.handle:
            _check(_lib.og_timestamps_destroy(self.handle))
            self.handle = None


class PinnedHost:
    """Page-locked host memory (og_host_alloc) for asynchronous uploads and readbacks; `view` gives numpy arrays."""

    def __init__(self, nbytes: int):
        p = ctypes.c_void_p()
        _check(_lib.og_host_alloc(nbytes, ctypes.byref(p)))
        self.ptr = p.value
        self.nbytes = nbytes

    def view(self, dtype, count: int, offset: int = 0) -> np.ndarray:
        dt = np.dtype(dtype)
        if offset + count * dt.itemsize > self.nbytes:
            raise ValueError("view past the end of the pinned buffer")
        raw = (ctypes.c_uint8 * (count * dt.itemsize)).from_address(self.ptr + offset)
        return np.frombuffer(raw, dtype=dt, count=count)

    def dispose(self) -> None:
        if self.ptr:
            _check(_lib.og_host_free(ctypes.c_void_p(self.ptr)))
            self.ptr = None


class GpuReadback:
    """A readback queued by GpuDevice.read_async; wait() blocks until the bytes are in host memory."""

    def __init__(self, handle):
        self.handle = handle

    def wait(self) -> None:
        if self.handle:
            h, self.handle = self.handle, None
            _check(_lib.og_readback_wait(h))


class GpuDevice:
    """The CUDA backend's device (compute subset of GpuDevice, src/RecursiveAI.OneGpu/GpuDevice.cs:27-228)."""

    def __init__(self, ordinal: int = 0):
        h = ctypes.c_void_p()
        _check(_lib.og_device_create(ordinal, ctypes.byref(h)))
        self.handle = h.value
        self.ordinal = ordinal
        self._keep = []
        info = og_device_info()
        _check(_lib.og_device_info_get(self.handle, ctypes.byref(info)))
        self.name = info.name.decode()
        self.sm_count = info.sm_count
        self.compute_capability = (info.cc_major, info.cc_minor)
        self.total_memory = info.total_memory
        self.tensor_core_i8 = bool(info.tensor_core_i8)

    def create_buffer(self, dtype, length_or_data) -> GpuBuffer:
        if isinstance(length_or_data, (int, np.integer)):
            return GpuBuffer(self, dtype, int(length_or_data))
        data = np.asarray(length_or_data)
        buf = GpuBuffer(self, dtype, data.size)
        buf.write(data)
        return buf

    def wrap(self, ptr: int, dtype, length: int) -> GpuBuffer:
        """A view of device memory owned elsewhere (e.g. a framework tensor)."""
        return GpuBuffer(self, dtype, length, ptr=ptr, owned=False)

    def begin_commands(self) -> GpuCommandEncoder:
        return GpuCommandEncoder(self)

    def submit(self, encoder: GpuCommandEncoder) -> None:
        h, encoder.handle = encoder.handle, None
        _check(_lib.og_device_submit(self.handle, h))

    def timestamp(self, stamps: GpuTimestampSet, index: int) -> None:
        _check(_lib.og_device_timestamp(self.handle, stamps.handle, index))

    def capture_begin(self) -> None:
        """og_device_capture_begin: work submitted from now on is recorded into a CUDA graph, not run."""
        _check(_lib.og_device_capture_begin(self.handle))

    def capture_end(self) -> "GpuGraph":
        """og_device_capture_end: the recorded work as a graph to replay with GpuGraph.launch."""
        h = ctypes.c_void_p()
        _check(_lib.og_device_capture_end(self.handle, ctypes.byref(h)))
        return GpuGraph(self, h)

    def wait_idle(self) -> None:
        _check(_lib.og_device_wait_idle(self.handle))
        self._keep.clear()

    def write_async(self, dst_ptr: int, host_ptr: int, nbytes: int) -> None:
        """og_buffer_write_async: upload on the copy engine, overlapping earlier work that does not use `dst`;
        later submissions wait for it. `host_ptr` should be page-locked (og_host_alloc)."""
        _check(_lib.og_buffer_write_async(self.handle, ctypes.c_void_p(dst_ptr), ctypes.c_void_p(host_ptr), nbytes))

    def read_async(self, host_ptr: int, src_ptr: int, nbytes: int) -> "GpuReadback":
        """og_buffer_read_async: readback after the work submitted so far, without blocking; wait() on the result."""
        h = ctypes.c_void_p()
        _check(_lib.og_buffer_read_async(self.handle, ctypes.c_void_p(host_ptr), ctypes.c_void_p(src_ptr), nbytes,
                                         ctypes.byref(h)))
        return GpuReadback(h.value)

    def watchdog_selftest(self, limit_us: int) -> None:
        """Queues a kernel whose bounded wait runs out after ``limit_us``; the next wait_idle raises
        GpuCommandFailedException with reason "Watchdog" and the device stays usable."""
        _check(_lib.og_device_watchdog_selftest(self.handle, limit_us))

    @property
    def stream(self) -> int:
        s = ctypes.c_void_p()
        _check(_lib.og_device_stream(self.handle, ctypes.byref(s)))
        return s.value or 0

    def set_stream(self, stream: int) -> None:
        _check(_lib.og_device_set_stream(self.handle, ctypes.c_void_p(stream)))

    def dispose(self) -> None:
        if self.handle:
            _check(_lib.og_device_destroy(self.handle))
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.dispose()


# ---- several GPUs: NCCL over NVLink -----------------------------------------------------------------------------

COMM_ID_BYTES = 128


def comm_unique_id() -> bytes:
    """og_comm_unique_id: a new communicator id, made by one rank and handed to the others by the host."""
    buf = (ctypes.c_uint8 * COMM_ID_BYTES)()
    _check(_lib.og_comm_unique_id(buf))
    return bytes(buf)


class Communicator:
    """og_comm: this device's rank in an NCCL communicator of `nranks` GPUs of one node (one process per GPU). Every
    call is queued on the device's stream in order with submitted work; every rank makes the same calls in the same
    order. No counterpart in the reference (its devices never exchange data)."""

    def __init__(self, device: GpuDevice, nranks: int, rank: int, unique_id: bytes):
        if len(unique_id) != COMM_ID_BYTES:
            raise ValueError(f"the communicator id has {COMM_ID_BYTES} bytes")
        h = ctypes.c_void_p()
        idbuf = (ctypes.c_uint8 * COMM_ID_BYTES).from_buffer_copy(unique_id)
        _check(_lib.og_comm_create(device.handle, int(nranks), int(rank), idbuf, ctypes.byref(h)))
        self.handle = h.value
        self.device = device
        self.nranks = nranks
        self.rank = rank

    def gather_columns(self, shard_ptr: int, elem_bytes: int, batch: int, m: int, widths, out_ptr: int = 0,
                       root: int = 0) -> None:
        """og_comm_gather_columns: the column shards [batch][m][widths[r]] of every rank put together as the dense
        [batch][m][sum(widths)] result at `out_ptr` on `root`."""
        w = (ctypes.c_int32 * self.nranks)(*[int(x) for x in widths])
        _check(_lib.og_comm_gather_columns(self.handle, ctypes.c_void_p(shard_ptr), int(elem_bytes), int(batch),
                                           int(m), w, ctypes.c_void_p(out_ptr or None), int(root)))

    def all_gather(self, send_ptr: int, nbytes: int, recv_ptr: int) -> None:
        """og_comm_all_gather: recv (nranks * nbytes) receives every rank's nbytes of send, in rank order."""
        _check(_lib.og_comm_all_gather(self.handle, ctypes.c_void_p(send_ptr), int(nbytes), ctypes.c_void_p(recv_ptr)))

    def dispose(self) -> None:
        if self.handle:
            _check(_lib.og_comm_destroy(self.handle))
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.dispose()


# ---- Int8Gemm ------------------------------------------------------------------------------------------------------

@dataclass
class Int8GemmProblem:
    """Int8GemmProblem (Int8Gemm.cs:43-95): A is M x K, B is K x N (N x K with transpose_b), all row-major."""
    m: int
    n: int
    k: int
    batch: int = 1
    transpose_b: bool = False
    lda: int = 0
    ldb: int = 0
    offset_a: int = 0
    offset_b: int = 0
    offset_c: int = 0
    stride_a: int = 0
    stride_b: int = 0

    @property
    def ops(self) -> float:
        return 2.0 * self.batch * self.m * self.n * self.k

    def c_struct(self) -> og_int8_gemm_problem:
        return og_int8_gemm_problem(self.m, self.n, self.k, self.batch, int(bool(self.transpose_b)), self.lda,
                                    self.ldb, self.offset_a, self.offset_b, self.offset_c, self.stride_a,
                                    self.stride_b)


@dataclass
class Int8Operand:
    """Int8Operand<T> (Int8Gemm.cs:28): a zero point, scale or bias value (or vector) in a device buffer."""
    buffer: Optional[GpuBuffer]
    offset: int = 0
    is_vector: bool = False

    def c_struct(self) -> og_operand:
        ref = self.buffer.ref() if self.buffer is not None else og_buffer(None, 0, 0)
        return og_operand(ref, self.offset, int(bool(self.is_vector)))


@dataclass
class Int8Scratch:
    """Int8Scratch (Int8Gemm.cs:37): caller-placed int32 scratch."""
    buffer: Optional[GpuBuffer]
    offset: int = 0

    def c_struct(self) -> og_operand:
        ref = self.buffer.ref() if self.buffer is not None else og_buffer(None, 0, 0)
        return og_operand(ref, self.offset, 0)


@dataclass
class Int8GemmOptions:
    """Int8GemmOptions (Int8Gemm.cs:7-21); `kernel` (KERNEL_AUTO / _TENSOR_CORE / _PORTABLE) and `tile` (0, 128 or
    256 rows per tensor-core tile) are test hooks like the reference's internal Tile."""
    allow_packed_dot: bool = True
    kernel: int = KERNEL_AUTO
    tile: int = 0
    stream_k: int = 0  # test hook: 2 splits the (tile, K block) work evenly across the SM pairs (stream-K)


def _buf(b: Optional[GpuBuffer]):
    return ctypes.byref(b.ref()) if b is not None else None


def _opd(o):
    return ctypes.byref(o.c_struct()) if o is not None else None


class Int8Gemm:
    """Int8Gemm (Int8Gemm.cs:124-683) on the CUDA backend."""

    def __init__(self, device: GpuDevice, options: Optional[Int8GemmOptions] = None):
        self.device = device
        h = ctypes.c_void_p()
        opt = None
        if options is not None:
            opt = ctypes.byref(og_int8_gemm_options(int(bool(options.allow_packed_dot)), int(options.kernel),
                                                    int(options.tile), int(options.stream_k)))
        _check(_lib.og_int8_gemm_create(device.handle, opt, ctypes.byref(h)))
        self.handle = h.value

    @property
    def variant(self) -> str:
        s = ctypes.create_string_buffer(128)
        _check(_lib.og_int8_gemm_variant(self.handle, s, 128))
        return s.value.decode()

    @property
    def last_kernel(self) -> str:
        s = ctypes.create_string_buffer(64)
        _check(_lib.og_int8_gemm_last_kernel(self.handle, s, 64))
        return s.value.decode()

    @property
    def bind_groups_created(self) -> int:
        n = ctypes.c_int32(0)
        _check(_lib.og_int8_gemm_bind_groups_created(self.handle, ctypes.byref(n)))
        return n.value

    @staticmethod
    def scratch_elements(problem: Int8GemmProblem) -> int:
        p = problem.c_struct()
        return int(_lib.og_int8_gemm_scratch_elements(ctypes.byref(p)))

    def reserve_scratch(self, elements: int) -> None:
        _check(_lib.og_int8_gemm_reserve_scratch(self.handle, int(elements)))

    def encode_int32(self, encoder: GpuCommandEncoder, problem: Int8GemmProblem, a: GpuBuffer, b: GpuBuffer,
                     c: GpuBuffer, zero_point_a: Optional[Int8Operand] = None,
                     zero_point_b: Optional[Int8Operand] = None, bias: Optional[Int8Operand] = None) -> None:
        p = problem.c_struct()
        _check(_lib.og_int8_gemm_encode_int32(self.handle, encoder.handle if encoder else None, ctypes.byref(p),
                                              _buf(a), _buf(b), _buf(c), _opd(zero_point_a), _opd(zero_point_b),
                                              _opd(bias)))

    def encode_float(self, encoder: GpuCommandEncoder, problem: Int8GemmProblem, a: GpuBuffer, b: GpuBuffer,
                     c: GpuBuffer, scale: Int8Operand, zero_point_a: Optional[Int8Operand] = None,
                     zero_point_b: Optional[Int8Operand] = None, float_bias: Optional[Int8Operand] = None,
                     int_bias: Optional[Int8Operand] = None) -> None:
        p = problem.c_struct()
        _check(_lib.og_int8_gemm_encode_float(self.handle, encoder.handle if encoder else None, ctypes.byref(p),
                                              _buf(a), _buf(b), _buf(c), _opd(scale), _opd(zero_point_a),
                                              _opd(zero_point_b), _opd(float_bias), _opd(int_bias)))

    def encode_requantized(self, encoder: GpuCommandEncoder, problem: Int8GemmProblem, a: GpuBuffer, b: GpuBuffer,
                           y: GpuBuffer, multiplier: Int8Operand, zero_point_y: int,
                           zero_point_a: Optional[Int8Operand] = None, zero_point_b: Optional[Int8Operand] = None,
                           int_bias: Optional[Int8Operand] = None, scratch: Optional[Int8Scratch] = None) -> None:
        p = problem.c_struct()
        _check(_lib.og_int8_gemm_encode_requantized(self.handle, encoder.handle if encoder else None,
                                                    ctypes.byref(p), _buf(a), _buf(b), _buf(y), _opd(multiplier),
                                                    int(zero_point_y), _opd(zero_point_a), _opd(zero_point_b),
                                                    _opd(int_bias), _opd(scratch)))

    def encode_dequantize(self, encoder: GpuCommandEncoder, problem: Int8GemmProblem, a: GpuBuffer, b: GpuBuffer,
                          c: GpuBuffer, a_scale: Int8Operand, b_scale: Int8Operand,
                          zero_point_a: Optional[Int8Operand] = None, zero_point_b: Optional[Int8Operand] = None,
                          float_bias: Optional[Int8Operand] = None, int_bias: Optional[Int8Operand] = None) -> None:
        """MatMulIntegerToFloat in one call: float(sum + intBias) * (aScale * bScale[n]) (+ floatBias), the scale
        product formed in the epilogue (the reference forms it with a separate element-wise pass)."""
        p = problem.c_struct()
        _check(_lib.og_int8_gemm_encode_dequantize(self.handle, encoder.handle if encoder else None, ctypes.byref(p),
                                                   _buf(a), _buf(b), _buf(c), _opd(a_scale), _opd(b_scale),
                                                   _opd(zero_point_a), _opd(zero_point_b), _opd(float_bias),
                                                   _opd(int_bias)))

    # The reference's member names.
    EncodeInt32 = encode_int32
    EncodeFloat = encode_float
    EncodeRequantized = encode_requantized
    ScratchElements = scratch_elements
    ReserveScratch = reserve_scratch

    def dispose(self) -> None:
        if self.handle:
            _check(_lib.og_int8_gemm_destroy(self.handle))
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.dispose()


class _BufferSpec:
    """A buffer description without device memory, for the device-free argument checks."""

    def __init__(self, dtype, length: int, ptr: int = 0x1000):
        self.dtype = np.dtype(dtype)
        self.type = _FROM_NP[self.dtype]
        self.length = int(length)
        self.ptr = ptr

    def ref(self) -> og_buffer:
        return og_buffer(self.ptr, self.length, self.type)


def buffer_spec(dtype, length: int, null: bool = False) -> _BufferSpec:
    """Describes a buffer of `length` elements of `dtype` for check_* (no allocation, no device)."""
    return _BufferSpec(dtype, length, 0 if null else 0x1000)


def int8_gemm_int32_noalloc(stream: int, problem, a, b, c, zero_point_a=None, zero_point_b=None, bias=None) -> None:
    """EncodeInt32 for callers that cannot allocate device memory while they run products (a host whose pool owns
    the GPU's memory, an engine step that forbids allocation, a latency-bound loop): og_int8_gemm_int32_noalloc
    queues the product on `stream` of the current device, keeping the zero-point byte sums in the library's fixed
    array (at most 1,048,576 int32) instead of allocated scratch. No counterpart in the reference."""
    p = problem.c_struct()
    _check(_lib.og_int8_gemm_int32_noalloc(ctypes.c_void_p(stream), ctypes.byref(p), _buf(a), _buf(b), _buf(c),
                                           _opd(zero_point_a), _opd(zero_point_b), _opd(bias)))


def int8_gemm_noalloc_status(stream: int) -> None:
    """Waits for `stream` and raises GpuCommandFailedException (reason "Watchdog") if a kernel of an allocation-free
    product on the current device gave up a bounded wait since the last check (og_int8_gemm_noalloc_status); the
    failure word is cleared."""
    _check(_lib.og_int8_gemm_noalloc_status(ctypes.c_void_p(stream)))


def int8_gemm_noalloc_watchdog_selftest(stream: int, limit_us: int) -> None:
    """Queues a kernel whose bounded wait runs out after `limit_us` and raises the allocation-free products' failure
    word, with no fault (og_int8_gemm_noalloc_watchdog_selftest)."""
    _check(_lib.og_int8_gemm_noalloc_watchdog_selftest(ctypes.c_void_p(stream), int(limit_us)))


def check_int32(problem, a, b, c, zero_point_a=None, zero_point_b=None, bias=None) -> None:
    """The argument checks of EncodeInt32 alone (no device needed)."""
    p = problem.c_struct()
    _check(_lib.og_int8_gemm_check_int32(ctypes.byref(p), _buf(a), _buf(b), _buf(c), _opd(zero_point_a),
                                         _opd(zero_point_b), _opd(bias)))


def check_float(problem, a, b, c, scale, zero_point_a=None, zero_point_b=None, float_bias=None,
                int_bias=None) -> None:
    p = problem.c_struct()
    _check(_lib.og_int8_gemm_check_float(ctypes.byref(p), _buf(a), _buf(b), _buf(c), _opd(scale),
                                         _opd(zero_point_a), _opd(zero_point_b), _opd(float_bias), _opd(int_bias)))


def check_dequantize(problem, a, b, c, a_scale, b_scale, zero_point_a=None, zero_point_b=None, float_bias=None,
                     int_bias=None) -> None:
    p = problem.c_struct()
    _check(_lib.og_int8_gemm_check_dequantize(ctypes.byref(p), _buf(a), _buf(b), _buf(c), _opd(a_scale),
                                              _opd(b_scale), _opd(zero_point_a), _opd(zero_point_b),
                                              _opd(float_bias), _opd(int_bias)))


def check_requantized(problem, a, b, y, multiplier, zero_point_y, zero_point_a=None, zero_point_b=None,
                      int_bias=None, scratch=None) -> None:
    p = problem.c_struct()
    _check(_lib.og_int8_gemm_check_requantized(ctypes.byref(p), _buf(a), _buf(b), _buf(y), _opd(multiplier),
                                               int(zero_point_y), _opd(zero_point_a), _opd(zero_point_b),
                                               _opd(int_bias), _opd(scratch)))


def check_dynamic_quantize(x, offset_x, count, y, offset_y, scale, offset_scale, zero_point,
                           offset_zero_point) -> None:
    _check(_lib.og_dynamic_quantize_check(_buf(x), offset_x, count, _buf(y), offset_y, _buf(scale), offset_scale,
                                          _buf(zero_point), offset_zero_point))


def _shape(shape):
    dims = [int(v) for v in shape]
    return (ctypes.c_int32 * max(len(dims), 1))(*dims), len(dims)


def _quant_args(x, offset_x, shape, axis, per_axis, scale, offset_scale, zero_point, offset_zero_point, output,
                offset_output):
    dims, rank = _shape(shape)
    return [_buf(x), offset_x, dims, rank, axis, int(bool(per_axis)), _buf(scale), offset_scale, _buf(zero_point),
            offset_zero_point, _buf(output), offset_output]


def check_dequantize_linear(x, offset_x, shape, axis, per_axis, scale, offset_scale, zero_point, offset_zero_point,
                            output, offset_output) -> None:
    """The argument checks of DequantizeKernels.Encode alone (no device needed)."""
    _check(_lib.og_dequantize_check(*_quant_args(x, offset_x, shape, axis, per_axis, scale, offset_scale, zero_point,
                                                 offset_zero_point, output, offset_output)))


def check_quantize_linear(x, offset_x, shape, axis, per_axis, scale, offset_scale, zero_point, offset_zero_point,
                          output, offset_output) -> None:
    """The argument checks of DequantizeKernels.EncodeQuantize alone (no device needed)."""
    _check(_lib.og_dequantize_check_quantize(*_quant_args(x, offset_x, shape, axis, per_axis, scale, offset_scale,
                                                          zero_point, offset_zero_point, output, offset_output)))


# ---- DequantizeKernels ----------------------------------------------------------------------------------------------

class DequantizeKernels:
    """DequantizeKernels (DequantizeKernels.cs:29-298) on the CUDA backend: DequantizeLinear (encode) and
    QuantizeLinear (encode_quantize)."""

    def __init__(self, device: GpuDevice):
        self.device = device
        h = ctypes.c_void_p()
        _check(_lib.og_dequantize_create(device.handle, ctypes.byref(h)))
        self.handle = h.value

    def encode(self, encoder: GpuCommandEncoder, x: GpuBuffer, offset_x: int, shape, axis: int, per_axis: bool,
               scale: GpuBuffer, offset_scale: int, zero_point: Optional[GpuBuffer], offset_zero_point: int,
               output: GpuBuffer, offset_output: int) -> None:
        _check(_lib.og_dequantize_encode(self.handle, encoder.handle if encoder else None,
                                         *_quant_args(x, offset_x, shape, axis, per_axis, scale, offset_scale,
                                                      zero_point, offset_zero_point, output, offset_output)))

    def encode_quantize(self, encoder: GpuCommandEncoder, x: GpuBuffer, offset_x: int, shape, axis: int,
                        per_axis: bool, scale: GpuBuffer, offset_scale: int, zero_point: Optional[GpuBuffer],
                        offset_zero_point: int, output: GpuBuffer, offset_output: int) -> None:
        _check(_lib.og_dequantize_encode_quantize(self.handle, encoder.handle if encoder else None,
                                                  *_quant_args(x, offset_x, shape, axis, per_axis, scale,
                                                               offset_scale, zero_point, offset_zero_point, output,
                                                               offset_output)))

    Encode = encode
    EncodeQuantize = encode_quantize

    def dispose(self) -> None:
        if self.handle:
            _check(_lib.og_dequantize_destroy(self.handle))
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.dispose()


# ---- ConvIntegerKernels ---------------------------------------------------------------------------------------------

class og_conv_problem(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int32) for name in
                ("batch", "in_channels", "height", "width", "out_channels", "kernel_height", "kernel_width",
                 "stride_height", "stride_width", "dilation_height", "dilation_width", "pad_top", "pad_left",
                 "pad_bottom", "pad_right", "groups", "activation", "offset_x", "offset_w", "offset_bias",
                 "offset_residual", "offset_y")]


@dataclass
class ConvProblem:
    """ConvProblem (ConvProblem.cs): NCHW / OIHW geometry, offsets in elements."""
    batch: int
    in_channels: int
    height: int
    width: int
    out_channels: int
    kernel_height: int
    kernel_width: int
    stride_height: int = 1
    stride_width: int = 1
    dilation_height: int = 1
    dilation_width: int = 1
    pad_top: int = 0
    pad_left: int = 0
    pad_bottom: int = 0
    pad_right: int = 0
    groups: int = 1
    activation: int = 0
    offset_x: int = 0
    offset_w: int = 0
    offset_bias: int = 0
    offset_residual: int = 0
    offset_y: int = 0

    @staticmethod
    def conv1d(batch, in_channels, length, out_channels, kernel, stride=1, dilation=1, pad_begin=0, pad_end=0,
               groups=1) -> "ConvProblem":
        """ConvProblem.Conv1D: height 1."""
        return ConvProblem(batch, in_channels, 1, length, out_channels, 1, kernel, stride_width=stride,
                           dilation_width=dilation, pad_left=pad_begin, pad_right=pad_end, groups=groups)

    @staticmethod
    def _extent(input_, kernel, stride, dilation, pad_begin, pad_end) -> int:
        if input_ < 1 or kernel < 1 or stride < 1 or dilation < 1:
            return 0
        span = input_ + pad_begin + pad_end - (dilation * (kernel - 1) + 1)
        return 0 if span < 0 else span // stride + 1

    @property
    def out_height(self) -> int:
        return self._extent(self.height, self.kernel_height, self.stride_height, self.dilation_height, self.pad_top,
                            self.pad_bottom)

    @property
    def out_width(self) -> int:
        return self._extent(self.width, self.kernel_width, self.stride_width, self.dilation_width, self.pad_left,
                            self.pad_right)

    def c_struct(self) -> og_conv_problem:
        return og_conv_problem(*[int(getattr(self, name)) for name, _ in og_conv_problem._fields_])


def conv_scratch_bytes_per_image(problem: ConvProblem) -> int:
    """ConvIntegerKernels.ScratchBytesPerImage."""
    p = problem.c_struct()
    out = ctypes.c_int64()
    _check(_lib.og_conv_integer_scratch_bytes_per_image(ctypes.byref(p), ctypes.byref(out)))
    return out.value


def check_conv_integer(problem: ConvProblem, x, w, y, x_zero_point=None, w_zero_point=None, scratch=None,
                       scratch_offset: int = 0) -> None:
    """The argument checks of ConvIntegerKernels.Encode alone (no device needed)."""
    p = problem.c_struct()
    _check(_lib.og_conv_integer_check(ctypes.byref(p), _buf(x), _buf(w), _buf(y), _opd(x_zero_point),
                                      _opd(w_zero_point), _buf(scratch), scratch_offset))


class ConvIntegerKernels:
    """ConvIntegerKernels (ConvIntegerKernels.cs:25-351) on the CUDA backend."""

    def __init__(self, device: GpuDevice, options: Optional[Int8GemmOptions] = None):
        self.device = device
        h = ctypes.c_void_p()
        opt = None
        if options is not None:
            opt = ctypes.byref(og_int8_gemm_options(int(bool(options.allow_packed_dot)), int(options.kernel),
                                                    int(options.tile), int(options.stream_k)))
        _check(_lib.og_conv_integer_create(device.handle, opt, ctypes.byref(h)))
        self.handle = h.value

    @property
    def variant(self) -> str:
        buf = ctypes.create_string_buffer(256)
        _check(_lib.og_conv_integer_variant(self.handle, buf, 256))
        return buf.value.decode()

    @property
    def bind_groups_created(self) -> int:
        n = ctypes.c_int32()
        _check(_lib.og_conv_integer_bind_groups_created(self.handle, ctypes.byref(n)))
        return n.value

    scratch_bytes_per_image = staticmethod(conv_scratch_bytes_per_image)

    def encode(self, encoder: GpuCommandEncoder, problem: ConvProblem, x: GpuBuffer, w: GpuBuffer, y: GpuBuffer,
               x_zero_point=None, w_zero_point=None, scratch: Optional[GpuBuffer] = None,
               scratch_offset: int = 0) -> None:
        p = problem.c_struct()
        _check(_lib.og_conv_integer_encode(self.handle, encoder.handle if encoder else None, ctypes.byref(p), _buf(x),
                                           _buf(w), _buf(y), _opd(x_zero_point), _opd(w_zero_point), _buf(scratch),
                                           scratch_offset))

    Encode = encode

    def dispose(self) -> None:
        if self.handle:
            _check(_lib.og_conv_integer_destroy(self.handle))
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.dispose()


# ---- DynamicQuantizeKernels -----------------------------------------------------------------------------------------

class DynamicQuantizeKernels:
    """DynamicQuantizeKernels (DynamicQuantizeKernels.cs:20-110) on the CUDA backend."""

    def __init__(self, device: GpuDevice):
        self.device = device
        h = ctypes.c_void_p()
        _check(_lib.og_dynamic_quantize_create(device.handle, ctypes.byref(h)))
        self.handle = h.value

    def encode(self, encoder: GpuCommandEncoder, x: GpuBuffer, offset_x: int, count: int, y: GpuBuffer,
               offset_y: int, scale: GpuBuffer, offset_scale: int, zero_point: GpuBuffer,
               offset_zero_point: int) -> None:
        _check(_lib.og_dynamic_quantize_encode(self.handle, encoder.handle if encoder else None, _buf(x), offset_x,
                                               count, _buf(y), offset_y, _buf(scale), offset_scale, _buf(zero_point),
                                               offset_zero_point))

    Encode = encode

    def dispose(self) -> None:
        if self.handle:
            _check(_lib.og_dynamic_quantize_destroy(self.handle))
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.dispose()
