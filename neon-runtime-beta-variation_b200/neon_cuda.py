"""Python binding of libneon_cuda.so (include/neon_cuda.h) with the NEON
runtime's operator surface for the quantized matvec path.

The reference runs every projection of its decode loop through
``fwd::proj_all_positions(W, X, x_stride, Y, y_stride, seq, pool)`` and
``fwd::proj_all_positions_multi(targets, X, x_stride, seq, pool)``
(rawllm_forward.hpp:522-726) over ``loader::TensorInfo`` handles
(rawllm_loader.hpp:34-41). This module keeps those names, argument meanings and
error behaviour:

* :class:`TensorInfo` -- name, GGUF shape ``[cols, rows]``, GGML type and the raw
  tensor bytes (what ``data_ptr`` points at).
* :func:`proj_all_positions` / :func:`proj_all_positions_multi` -- host numpy
  buffers in and out, blocking, ``RuntimeError`` (the reference's
  ``std::runtime_error``) with the reference's message on a bad argument.
  Weights are uploaded to HBM on first use and stay there (a side table keyed
  by the TensorInfo object), the load-time hook of rawllm_loader.hpp:84-177.
* :class:`DeviceTensor` with :meth:`DeviceTensor.matvec` and :func:`matvec_multi`
  -- the device-pointer entry points for callers that keep activations on the
  GPU (torch tensors or raw pointers), asynchronous on a CUDA stream.

There is no CPU fallback: if the CUDA library cannot be loaded, every call
raises.
"""
from __future__ import annotations

import ctypes as C
import json
import struct
import os
import threading
import weakref

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libneon_cuda.so")

NEON_OK = 0
GGML_F32 = 0
GGML_F16 = 1
GGML_Q4_0 = 2
GGML_Q4_1 = 3
GGML_Q5_0 = 6
GGML_Q5_1 = 7
GGML_Q8_0 = 8
GGML_Q4_K = 12
GGML_Q5_K = 13
GGML_Q6_K = 14
GGML_BF16 = 30
SHARD_NONE = 0
SHARD_ROWS = 1
SHARD_COLS = 2

# Public C entry points, in the order include/neon_cuda.h declares them.
C_ENTRY_POINTS = (
    "neon_cuda_last_error",
    "neon_cuda_version",
    "neon_cuda_device_count",
    "neon_cuda_init",
    "neon_cuda_upload",
    "neon_cuda_quantize_rows",
    "neon_cuda_quantize_host",
    "neon_cuda_upload_quantized",
    "neon_cuda_tensor_info",
    "neon_cuda_free",
    "neon_cuda_quantize_q8_0",
    "neon_cuda_matvec",
    "neon_cuda_matvec_multi",
    "neon_cuda_proj_all_positions",
    "neon_cuda_proj_all_positions_multi",
    "neon_cuda_sync",
    "neon_cuda_launch_count",
    "neon_cuda_matvec_q4_0_noalloc",
    "neon_cuda_model_create",
    "neon_cuda_model_set_tensor",
    "neon_cuda_model_set_quantize",
    "neon_cuda_model_forward",
    "neon_cuda_model_generate",
    "neon_cuda_model_length",
    "neon_cuda_model_set_length",
    "neon_cuda_model_kv_shift",
    "neon_cuda_model_read_kv",
    "neon_cuda_model_decode_ms",
    "neon_cuda_model_forward_ms",
    "neon_cuda_model_free",
    "neon_cuda_comm_create",
    "neon_cuda_comm_ipc_handle",
    "neon_cuda_comm_connect",
    "neon_cuda_comm_connect_local",
    "neon_cuda_comm_set_timeout",
    "neon_cuda_comm_allreduce",
    "neon_cuda_matvec_allgather",
    "neon_cuda_comm_check",
    "neon_cuda_comm_free",
    "neon_cuda_model_comm_floats",
    "neon_cuda_tp_shard",
    "neon_cuda_model_create_tp",
    "neon_cuda_set_fused_collectives",
    "neon_cuda_set_pdl",
    "neon_cuda_set_prefill_mma",
    "neon_cuda_set_dq_ring",
    "neon_cuda_set_stream_tiles",
    "neon_cuda_set_resident",
    "neon_cuda_set_attn_rows",
    "neon_cuda_set_attn_head_split",
)

_sz = C.c_size_t
_vp = C.c_void_p


class _Target(C.Structure):
    _fields_ = [("W", _vp), ("Y", _vp), ("y_stride", _sz)]


class _ModelConfig(C.Structure):
    _fields_ = [(f, C.c_uint32) for f in ("n_vocab", "n_embd", "n_layer", "n_head", "n_kv_head", "head_dim",
                                          "n_ff", "ctx_len")] + [
        ("rope_base", C.c_float), ("rope_scale", C.c_float), ("rope_dim_count", C.c_uint32),
        ("norm_eps", C.c_float), ("plain_ffn", C.c_uint32)]


class NeonError(RuntimeError):
    """A failed library call; the message is the library's (or the reference's)."""


_lib = None
_lock = threading.Lock()


def load(path: str | None = None) -> C.CDLL:
    """Load libneon_cuda.so (building it first if it is missing)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            import importlib.util

            spec = importlib.util.spec_from_file_location("_neon_build", os.path.join(HERE, "build.py"))
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            mod.build()
        L = C.CDLL(p)
        L.neon_cuda_last_error.restype = C.c_char_p
        L.neon_cuda_version.restype = C.c_char_p
        L.neon_cuda_device_count.argtypes = [C.POINTER(C.c_int)]
        L.neon_cuda_init.argtypes = [C.c_int]
        L.neon_cuda_upload.argtypes = [_vp, C.c_int, _sz, _sz, C.c_int, C.c_int, C.c_int, C.POINTER(_vp)]
        L.neon_cuda_quantize_rows.argtypes = [_vp, C.c_int, _sz, _sz, C.c_int, _vp, _vp]
        L.neon_cuda_quantize_host.argtypes = [_vp, C.c_int, _sz, _sz, C.c_int, _vp]
        L.neon_cuda_upload_quantized.argtypes = [_vp, C.c_int, _sz, _sz, C.c_int, C.c_int, C.c_int, C.c_int,
                                                 C.POINTER(_vp)]
        L.neon_cuda_model_set_quantize.argtypes = [_vp, C.c_int]
        L.neon_cuda_tensor_info.argtypes = [_vp, C.POINTER(_sz), C.POINTER(_sz), C.POINTER(C.c_int),
                                            C.POINTER(_sz)]
        L.neon_cuda_free.argtypes = [_vp]
        L.neon_cuda_quantize_q8_0.argtypes = [_vp, _sz, _sz, _sz, _vp, _vp, _vp]
        L.neon_cuda_matvec.argtypes = [_vp, _vp, _sz, _vp, _sz, _sz, _vp]
        L.neon_cuda_matvec_multi.argtypes = [C.POINTER(_Target), _sz, _vp, _sz, _sz, _vp]
        L.neon_cuda_proj_all_positions.argtypes = [_vp, _vp, _sz, _vp, _sz, _sz]
        L.neon_cuda_proj_all_positions_multi.argtypes = [C.POINTER(_Target), _sz, _vp, _sz, _sz]
        L.neon_cuda_sync.argtypes = [_vp]
        L.neon_cuda_launch_count.restype = C.c_uint64
        L.neon_cuda_set_pdl.argtypes = [C.c_int]
        L.neon_cuda_set_prefill_mma.argtypes = [C.c_int]
        L.neon_cuda_set_dq_ring.argtypes = [C.c_int]
        L.neon_cuda_set_stream_tiles.argtypes = [C.c_int, C.c_int]
        L.neon_cuda_set_resident.argtypes = [C.c_int]
        L.neon_cuda_set_attn_rows.argtypes = [C.c_int, C.c_int]
        L.neon_cuda_set_attn_head_split.argtypes = [C.c_int]
        L.neon_cuda_matvec_q4_0_noalloc.argtypes = [_vp, _vp, _sz, _vp, _sz, _sz, _vp]
        L.neon_cuda_model_create.argtypes = [C.POINTER(_ModelConfig), C.POINTER(_vp)]
        L.neon_cuda_model_set_tensor.argtypes = [_vp, C.c_int, C.c_int, _vp, _sz, C.c_int, _sz, _sz]
        L.neon_cuda_model_forward.argtypes = [_vp, _vp, _sz, _vp]
        L.neon_cuda_model_generate.argtypes = [_vp, _vp, _sz, _sz, C.c_int32, _vp, C.POINTER(_sz)]
        L.neon_cuda_model_length.argtypes = [_vp, C.POINTER(_sz)]
        L.neon_cuda_model_set_length.argtypes = [_vp, _sz]
        L.neon_cuda_model_kv_shift.argtypes = [_vp, _sz, _sz]
        L.neon_cuda_model_read_kv.argtypes = [_vp, C.c_int, _sz, _vp, _vp]
        L.neon_cuda_model_decode_ms.argtypes = [_vp, C.POINTER(C.c_float)]
        L.neon_cuda_model_forward_ms.argtypes = [_vp, C.POINTER(C.c_float)]
        L.neon_cuda_model_free.argtypes = [_vp]
        L.neon_cuda_comm_create.argtypes = [C.c_int, C.c_int, _sz, C.POINTER(_vp)]
        L.neon_cuda_comm_ipc_handle.argtypes = [_vp, _vp, C.POINTER(_sz)]
        L.neon_cuda_comm_connect.argtypes = [_vp, _vp, _sz]
        L.neon_cuda_comm_connect_local.argtypes = [C.POINTER(_vp), C.c_int]
        L.neon_cuda_comm_set_timeout.argtypes = [_vp, C.c_double]
        L.neon_cuda_comm_allreduce.argtypes = [_vp, _vp, _vp, _sz, C.c_int, _vp]
        L.neon_cuda_matvec_allgather.argtypes = [_vp, _vp, _vp, _vp, _sz, _sz, _vp]
        L.neon_cuda_comm_check.argtypes = [_vp]
        L.neon_cuda_comm_free.argtypes = [_vp]
        L.neon_cuda_model_comm_floats.argtypes = [C.POINTER(_ModelConfig), C.c_int, C.POINTER(_sz)]
        L.neon_cuda_tp_shard.argtypes = [C.POINTER(_ModelConfig), C.c_int, C.c_int, C.c_int, C.POINTER(_sz)]
        L.neon_cuda_model_create_tp.argtypes = [C.POINTER(_ModelConfig), _vp, C.POINTER(_vp)]
        L.neon_cuda_set_fused_collectives.argtypes = [C.c_int]
        _lib = L
        return L


def _check(rc: int) -> None:
    if rc != NEON_OK:
        raise NeonError(load().neon_cuda_last_error().decode(errors="replace"))


def device_count() -> int:
    n = C.c_int(0)
    _check(load().neon_cuda_device_count(C.byref(n)))
    return n.value


def init(device: int = 0) -> None:
    _check(load().neon_cuda_init(int(device)))


def launch_count() -> int:
    return int(load().neon_cuda_launch_count())


def set_prefill_mma(enabled: bool) -> None:
    """Multi-position Q4_0 calls on the tensor cores (int8 MMA, bit-exact with
    dot_q4_0_q8_0) instead of the CUDA-core kernel; process-wide, off by default."""
    _check(load().neon_cuda_set_prefill_mma(1 if enabled else 0))


def set_dq_ring(enabled) -> None:
    """One-position calls of the dequantising types on the bulk-copy ring
    kernel (several row tiles in flight per CTA) instead of the register-buffer
    kernel: True for every such type, False for none, None (the default) for
    the types it measured faster for (Q4_1, F16, BF16). Process-wide."""
    _check(load().neon_cuda_set_dq_ring(-1 if enabled is None else 1 if enabled else 0))


def set_stream_tiles(rows_per_tile: int = 0, blocks_per_chunk: int = 0) -> None:
    """Tile shape of later one-position Q4_0 / Q8_0 launches (rows per tile,
    blocks per row chunk; 0 = whole rows); (0, 0) is the built-in planner.
    For tuning sweeps; process-wide."""
    _check(load().neon_cuda_set_stream_tiles(int(rows_per_tile), int(blocks_per_chunk)))


def set_resident(ctas_per_sm: int = 1) -> None:
    """One-position Q4_0 / Q8_0 launches that fit shared memory run on the
    resident kernel with this many CTAs per SM (default 1); 0 sends them all
    to the streaming kernel. Process-wide."""
    _check(load().neon_cuda_set_resident(int(ctas_per_sm)))


def set_attn_rows(min_rows: int = 32, share_rows: int = 128) -> None:
    """Decode attention: models created afterwards take the smallest cluster
    (up to 16 CTAs per KV head) whose share of ctx_len is at most share_rows
    rows; steps launched afterwards give each CTA at least min_rows rows.
    Multiples of 32. Process-wide."""
    _check(load().neon_cuda_set_attn_rows(int(min_rows), int(share_rows)))


def set_attn_head_split(max_split: int = 8) -> None:
    """Decode attention: spread each KV head's query heads over up to
    max_split clusters when one cluster per KV head leaves SMs idle (models
    created afterwards); 1 keeps one cluster per KV head. Process-wide."""
    _check(load().neon_cuda_set_attn_head_split(int(max_split)))


def set_pdl(enabled: bool) -> None:
    _check(load().neon_cuda_set_pdl(1 if enabled else 0))


def set_fused_collectives(enabled: bool) -> None:
    """Sharded decode: fold the all-reduces into the matvecs (default) or not."""
    _check(load().neon_cuda_set_fused_collectives(1 if enabled else 0))


def sync(stream: int = 0) -> None:
    _check(load().neon_cuda_sync(_vp(stream)))


def _ptr(a) -> int:
    """Address of a numpy array, a torch tensor or an int."""
    if a is None:
        return 0
    if isinstance(a, int):
        return a
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    if hasattr(a, "data_ptr"):
        return int(a.data_ptr())
    raise TypeError(f"cannot take the address of {type(a).__name__}")


def _stream(stream) -> int:
    if stream is None:
        return 0
    if isinstance(stream, int):
        return stream
    return int(getattr(stream, "cuda_stream", stream))


# ---------------------------------------------------------------------------
# device tensors
# ---------------------------------------------------------------------------

class DeviceTensor:
    """A weight tensor resident in HBM (an uploaded GGUF tensor or shard)."""

    def __init__(self, raw: np.ndarray, ggml_type: int, rows: int, cols: int,
                 shard_mode: int = SHARD_NONE, shard_index: int = 0, shard_count: int = 1):
        L = load()
        raw = np.ascontiguousarray(raw)
        h = _vp()
        _check(L.neon_cuda_upload(raw.ctypes.data, int(ggml_type), int(rows), int(cols), int(shard_mode),
                                  int(shard_index), int(shard_count), C.byref(h)))
        self.handle = h.value
        r, c, t, b = _sz(), _sz(), C.c_int(), _sz()
        _check(L.neon_cuda_tensor_info(self.handle, C.byref(r), C.byref(c), C.byref(t), C.byref(b)))
        self.rows, self.cols, self.type, self.device_bytes = r.value, c.value, t.value, b.value
        self._fin = weakref.finalize(self, L.neon_cuda_free, self.handle)

    @classmethod
    def _adopt(cls, handle) -> "DeviceTensor":
        """Wrap a tensor handle the library created."""
        L = load()
        self = cls.__new__(cls)
        self.handle = handle
        r, c, t, b = _sz(), _sz(), C.c_int(), _sz()
        _check(L.neon_cuda_tensor_info(self.handle, C.byref(r), C.byref(c), C.byref(t), C.byref(b)))
        self.rows, self.cols, self.type, self.device_bytes = r.value, c.value, t.value, b.value
        self._fin = weakref.finalize(self, L.neon_cuda_free, self.handle)
        return self

    def free(self) -> None:
        self._fin()

    def matvec(self, X, Y, seq: int = 1, x_stride: int | None = None, y_stride: int | None = None,
               stream=None) -> None:
        """Y[t*y_stride + r] = W_r . X_t on device buffers (torch tensors or pointers)."""
        x_stride = self.cols if x_stride is None else x_stride
        y_stride = self.rows if y_stride is None else y_stride
        _check(load().neon_cuda_matvec(self.handle, _ptr(X), x_stride, _ptr(Y), y_stride, seq,
                                       _vp(_stream(stream))))


_ROW_BYTES = {GGML_F32: (1, 4), GGML_F16: (1, 2), GGML_BF16: (1, 2), GGML_Q4_0: (32, 18), GGML_Q4_1: (32, 20),
              GGML_Q5_0: (32, 22), GGML_Q5_1: (32, 24), GGML_Q8_0: (32, 34), GGML_Q4_K: (256, 144),
              GGML_Q5_K: (256, 176), GGML_Q6_K: (256, 210)}


def row_bytes(ggml_type: int, cols: int) -> int:
    """Bytes of one GGUF row (GGUFLoader::bytes_for_type, rawllm_loader.hpp:367-386)."""
    be, bb = _ROW_BYTES[ggml_type]
    return cols // be * bb


def quantize(raw: np.ndarray, src_type: int, rows: int, cols: int, dst_type: int) -> np.ndarray:
    """Float rows (F32/F16/BF16 bytes) -> GGUF rows of dst_type, quantised on the
    device as gguf-py's gguf.quants.quantize writes them; shape (rows, row_bytes)."""
    raw = np.ascontiguousarray(raw)
    out = np.empty((rows, row_bytes(dst_type, cols)), np.uint8)
    _check(load().neon_cuda_quantize_host(raw.ctypes.data, int(src_type), rows, cols, int(dst_type),
                                          out.ctypes.data))
    return out


def upload_quantized(raw: np.ndarray, src_type: int, rows: int, cols: int, dst_type: int,
                     shard_mode: int = SHARD_NONE, shard_index: int = 0, shard_count: int = 1) -> "DeviceTensor":
    """A DeviceTensor of float rows quantised to dst_type on the device."""
    raw = np.ascontiguousarray(raw)
    h = _vp()
    _check(load().neon_cuda_upload_quantized(raw.ctypes.data, int(src_type), rows, cols, int(dst_type),
                                             int(shard_mode), int(shard_index), int(shard_count), C.byref(h)))
    return DeviceTensor._adopt(h.value)


def matvec_multi(targets, X, seq: int = 1, x_stride: int | None = None, stream=None) -> None:
    """targets: list of (DeviceTensor, Y device buffer, y_stride or None)."""
    n = len(targets)
    arr = (_Target * n)()
    for i, (w, y, ys) in enumerate(targets):
        arr[i].W = w.handle
        arr[i].Y = _ptr(y)
        arr[i].y_stride = w.rows if ys is None else ys
    x_stride = targets[0][0].cols if x_stride is None else x_stride
    _check(load().neon_cuda_matvec_multi(arr, n, _ptr(X), x_stride, seq, _vp(_stream(stream))))


def quantize_q8_0(X, cols: int, seq: int, d_out, q_out, x_stride: int | None = None, stream=None) -> None:
    """Device Q8_0 activation quantisation (bit-exact with quantize_rows_q8_0)."""
    x_stride = cols if x_stride is None else x_stride
    _check(load().neon_cuda_quantize_q8_0(_ptr(X), x_stride, cols, seq, _ptr(d_out), _ptr(q_out),
                                          _vp(_stream(stream))))


# ---------------------------------------------------------------------------
# the reference's operator surface
# ---------------------------------------------------------------------------

class TensorInfo:
    """Mirror of loader::TensorInfo (rawllm_loader.hpp:34-41): name, GGUF shape
    ``[cols, rows]`` (contiguous dim first), GGML type and the tensor's raw
    bytes (what ``data_ptr`` addresses)."""

    def __init__(self, name: str, shape, ggml_type: int, data: np.ndarray):
        self.name = name
        self.shape = list(shape)
        self.type = int(ggml_type)
        self.data = np.ascontiguousarray(data).reshape(-1).view(np.uint8)
        self.nbytes = self.data.nbytes


class ProjTarget:
    """Mirror of fwd::ProjTarget (rawllm_forward.hpp:626-630)."""

    def __init__(self, W: TensorInfo, Y: np.ndarray, y_stride: int):
        self.W, self.Y, self.y_stride = W, Y, y_stride


# values per block (block_size_for, rawllm_forward.hpp:289-299); float types: 1
_BLOCK = {GGML_Q4_0: 32, GGML_Q4_1: 32, GGML_Q5_0: 32, GGML_Q5_1: 32, GGML_Q8_0: 32,
          GGML_Q4_K: 256, GGML_Q5_K: 256, GGML_Q6_K: 256}
_uploaded: "weakref.WeakKeyDictionary[TensorInfo, DeviceTensor]" = weakref.WeakKeyDictionary()


def _check_shape(W: TensorInfo):
    """The reference's argument checks (rawllm_forward.hpp:527-534)."""
    if len(W.shape) < 2:
        raise RuntimeError("forward(): expected a 2D weight tensor: " + W.name)
    cols, rows = int(W.shape[0]), int(W.shape[1])
    bs = _BLOCK.get(W.type, 1)
    if cols % bs != 0:
        raise RuntimeError(f"forward(): {W.name} input dim ({cols}) isn't a multiple of its quant block "
                           f"size ({bs}) — can't dequantize safely.")
    return cols, rows


def upload(W: TensorInfo) -> DeviceTensor:
    """The one-time HBM upload of a tensor (cached per TensorInfo)."""
    dt = _uploaded.get(W)
    if dt is None:
        cols, rows = _check_shape(W)
        dt = DeviceTensor(W.data, W.type, rows, cols)
        _uploaded[W] = dt
    return dt


def proj_all_positions(W: TensorInfo, X: np.ndarray, x_stride: int, Y: np.ndarray, y_stride: int,
                       seq: int, pool=None) -> None:
    """Y[t*y_stride + r] = W_r . X_t (host buffers, blocking). ``pool`` is
    accepted for signature parity with the reference and ignored: the GPU grid
    replaces the CPU thread pool."""
    _check_shape(W)
    dt = upload(W)
    X = np.ascontiguousarray(X, dtype=np.float32)
    if Y.dtype != np.float32 or not Y.flags.c_contiguous:
        raise RuntimeError("Y must be a C-contiguous float32 array")
    _check(load().neon_cuda_proj_all_positions(dt.handle, X.ctypes.data, x_stride, Y.ctypes.data, y_stride,
                                               seq))


def proj_all_positions_multi(targets, X: np.ndarray, x_stride: int, seq: int, pool=None) -> None:
    """Several ProjTargets that share X (host buffers, blocking)."""
    n = len(targets)
    for t in targets:
        _check_shape(t.W)
    arr = (_Target * n)()
    for i, t in enumerate(targets):
        if t.Y.dtype != np.float32 or not t.Y.flags.c_contiguous:
            raise RuntimeError("Y must be a C-contiguous float32 array")
        arr[i].W = upload(t.W).handle
        arr[i].Y = t.Y.ctypes.data
        arr[i].y_stride = t.y_stride
    X = np.ascontiguousarray(X, dtype=np.float32)
    _check(load().neon_cuda_proj_all_positions_multi(arr, n, X.ctypes.data, x_stride, seq))


# ---------------------------------------------------------------------------
# the decode step (transformer_forward / run_generation on the device)
# ---------------------------------------------------------------------------

def _config(cfg) -> _ModelConfig:
    return _ModelConfig(*[getattr(cfg, f) for f in ("n_vocab", "n_embd", "n_layer", "n_head", "n_kv_head",
                                                    "head_dim", "n_ff", "ctx_len")],
                        cfg.rope_base, cfg.rope_scale, cfg.rope_dim_count, cfg.norm_eps,
                        1 if getattr(cfg, "plain_ffn", False) else 0)


def tp_shard(cfg, role: int, rank: int, world: int):
    """(row0, row1, col0, col1): the part of a GGUF tensor of ``role`` that
    tensor-parallel ``rank`` of ``world`` keeps (host-only, no GPU needed)."""
    r = (_sz * 4)()
    _check(load().neon_cuda_tp_shard(C.byref(_config(cfg)), int(role), int(rank), int(world), r))
    return tuple(int(v) for v in r)


def model_comm_floats(cfg, world: int) -> int:
    """Receive-slot size (floats) a communicator needs for this model."""
    n = _sz()
    _check(load().neon_cuda_model_comm_floats(C.byref(_config(cfg)), int(world), C.byref(n)))
    return n.value


class Comm:
    """Tensor-parallel communicator of one rank (neon_cuda_comm_*): a buffer
    in this GPU's HBM that every peer maps; collectives are one kernel each
    over peer memory. Create it with the rank's device current."""

    def __init__(self, rank: int, world: int, max_floats: int):
        L = load()
        h = _vp()
        _check(L.neon_cuda_comm_create(int(rank), int(world), int(max_floats), C.byref(h)))
        self.handle = h.value
        self.rank, self.world = int(rank), int(world)
        self._fin = weakref.finalize(self, L.neon_cuda_comm_free, self.handle)

    def ipc_handle(self) -> bytes:
        n = _sz(0)
        _check(load().neon_cuda_comm_ipc_handle(self.handle, None, C.byref(n)))
        buf = C.create_string_buffer(n.value)
        _check(load().neon_cuda_comm_ipc_handle(self.handle, buf, C.byref(n)))
        return buf.raw

    def connect(self, handles) -> None:
        """Open the peers' buffers from the IPC handles of ranks 0..world-1."""
        handles = list(handles)
        if len(handles) != self.world or len({len(h) for h in handles}) != 1:
            raise NeonError("connect() needs one IPC handle per rank, all of one size")
        blob = b"".join(handles)
        _check(load().neon_cuda_comm_connect(self.handle, blob, len(handles[0])))

    @classmethod
    def from_process_group(cls, max_floats: int, group=None) -> "Comm":
        """Create and connect over an initialised torch.distributed group (any
        backend; it only carries the IPC handles)."""
        import torch.distributed as dist

        c = cls(dist.get_rank(group), dist.get_world_size(group), max_floats)
        handles = [None] * c.world
        dist.all_gather_object(handles, c.ipc_handle(), group=group)
        c.connect(handles)
        return c

    @staticmethod
    def connect_local(comms) -> None:
        """Connect the communicators of ranks 0..n-1 created in this process."""
        arr = (_vp * len(comms))(*[c.handle for c in comms])
        _check(load().neon_cuda_comm_connect_local(arr, len(comms)))

    def set_timeout(self, seconds: float) -> None:
        _check(load().neon_cuda_comm_set_timeout(self.handle, float(seconds)))

    def allreduce(self, x, out, n: int | None = None, add: bool = False, stream=None) -> None:
        """out (+)= sum over ranks of x (device buffers, e.g. torch tensors)."""
        if n is None:
            n = x.numel()
        _check(load().neon_cuda_comm_allreduce(self.handle, _ptr(x), _ptr(out), int(n), 1 if add else 0,
                                               _stream(stream)))

    def matvec_allgather(self, w: "DeviceTensor", x, y, n_total: int, row0: int, stream=None) -> None:
        """y[0 .. n_total) = the whole matvec on every rank, from this rank's row
        shard w (rows row0 .. row0 + w.rows of the matrix) and x (device
        buffers); the ranks' shards must tile [0, n_total)."""
        _check(load().neon_cuda_matvec_allgather(self.handle, w.handle, _ptr(x), _ptr(y), int(n_total), int(row0),
                                                 _stream(stream)))

    def check(self) -> None:
        _check(load().neon_cuda_comm_check(self.handle))

    def free(self) -> None:
        self._fin()


# ---------------------------------------------------------------------------
# .gguf models
# ---------------------------------------------------------------------------

# Bytes of n values of a GGML type (nbytes_for, rawllm_loader.hpp:367-386),
# as (values per block, bytes per block); 0 bytes: a type the loader cannot size.
_GGUF_NBYTES = {0: (1, 4), 1: (1, 2), 30: (1, 2), 2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34),
                9: (32, 36), 10: (256, 84), 11: (256, 110), 12: (256, 144), 13: (256, 176), 14: (256, 210),
                25: (32, 18)}
# GGUF metadata value types (MetaType, rawllm_loader.hpp:66-69): struct code or None for string / array
_GGUF_SCALARS = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<B", 10: "<Q", 11: "<q",
                 12: "<d"}
_ROLE_NAMES = {"token_embd": 0, "output_norm": 1, "output": 2, "attn_norm": 3, "attn_q": 4, "attn_k": 5,
               "attn_v": 6, "attn_output": 7, "ffn_norm": 8, "ffn_gate": 9, "ffn_up": 10, "ffn_down": 11}


def _gguf_nbytes(t: int, n: int) -> int:
    be, bb = _GGUF_NBYTES.get(t, (1, 0))
    return n // be * bb


def load_gguf(path: str):
    """Open a NANITY .gguf file as (config, tensors) for :class:`Model`:
    restates GGUFLoader::open (rawllm_loader.hpp:84-177: header, metadata,
    tensor table, general.alignment, bounds) and validate_config (:197-330:
    the nanity.* keys, every tensor's shape), with their messages. ``tensors``
    are (role, layer, bytes, ggml type, ne0, ne1) views of a read-only memory
    map for the names ModelWeights::build looks up (rawllm_forward.hpp:847-866);
    ``config.ctx_len`` is the KV capacity kv_window = min(context_length, 4096),
    ``config.bos_id`` / ``eos_id`` / ``unk_id`` the tokenizer's ids."""
    mm = np.memmap(path, np.uint8, mode="r")
    size = mm.size
    if size < 16:
        raise RuntimeError("File too small to be GGUF (<16 bytes): " + path)
    pos = 0

    def rd(fmt):
        nonlocal pos
        n = struct.calcsize(fmt)
        if pos + n > size:
            raise RuntimeError("GGUF: unexpected EOF")
        v = struct.unpack(fmt, bytes(mm[pos:pos + n]))[0]
        pos += n
        return v

    def rd_str():
        nonlocal pos
        n = rd("<Q")
        if pos + n > size:
            raise RuntimeError("GGUF: string overflow")
        v = bytes(mm[pos:pos + n]).decode("utf-8", "replace")
        pos += n
        return v

    if bytes(mm[:4]) != b"GGUF":
        raise RuntimeError("Not a GGUF file: " + path)
    pos = 4
    ver = rd("<I")
    if ver < 2 or ver > 3:
        raise RuntimeError("Unsupported GGUF version")
    n_tensors, n_kv = rd("<Q"), rd("<Q")
    meta_num, meta_str, tok = {}, {}, {}

    def value(t, key):
        nonlocal pos
        if t in _GGUF_SCALARS:
            v = rd(_GGUF_SCALARS[t])
            return float(v != 0) if t == 7 else v
        if t == 8:
            return rd_str()
        if t == 9:
            et, cnt = rd("<I"), rd("<Q")
            for _ in range(cnt):  # arrays (the tokenizer's vocabulary and merges) are skipped
                value(et, key)
            return None
        raise RuntimeError("Unknown GGUF meta type")

    for _ in range(n_kv):
        key = rd_str()
        t = rd("<I")
        v = value(t, key)
        if key.startswith("tokenizer."):
            if isinstance(v, (int, float)) and t != 8:
                tok[key] = int(v) & 0xFFFFFFFF
        elif isinstance(v, str):
            meta_str[key] = v
        elif v is not None:
            meta_num[key] = float(v)
    infos = []
    for _ in range(n_tensors):
        name = rd_str()
        nd = rd("<I")
        shape = [rd("<Q") for _ in range(nd)]
        infos.append((name, shape, rd("<I"), rd("<Q")))
    alignment = int(meta_num.get("general.alignment", 32)) or 32
    data_start = (pos + alignment - 1) // alignment * alignment
    table = {}
    for name, shape, t, off in infos:
        n = int(np.prod(shape)) if shape else 1
        nbytes = _gguf_nbytes(t, n)
        if data_start + off + nbytes > size:
            raise RuntimeError(f"Tensor '{name}' OOB")
        table[name] = (shape, t, mm[data_start + off:data_start + off + nbytes])

    # validate_config
    def req_str(k):
        if not meta_str.get(k):
            raise RuntimeError(f"NANITY: missing required metadata string key '{k}'.")
        return meta_str[k]

    def req_num(k):
        if k not in meta_num:
            raise RuntimeError(f"NANITY: missing required metadata key '{k}'.")
        return meta_num[k]

    arch = req_str("general.architecture")
    if arch != "nanity":
        raise RuntimeError(f'NANITY: general.architecture="{arch}", expected "nanity" -- this file is not a '
                           "NANITY model.")
    spec = int(req_num("nanity.spec_version"))
    if spec != NCTR_SPEC_VERSION:
        raise RuntimeError(f"NANITY: nanity.spec_version={spec}, this runtime only supports version "
                           f"{NCTR_SPEC_VERSION}.")
    u32 = lambda v: int(v) & 0xFFFFFFFF  # noqa: E731
    n_embd, n_layer = u32(req_num("nanity.embedding_length")), u32(req_num("nanity.block_count"))
    n_head, n_kv = u32(req_num("nanity.attention.head_count")), u32(req_num("nanity.attention.head_count_kv"))
    head_dim, n_ff = u32(req_num("nanity.attention.key_length")), u32(req_num("nanity.feed_forward_length"))
    ctx_len = u32(req_num("nanity.context_length"))
    f32 = lambda v: float(np.float32(v))  # noqa: E731
    norm_eps = f32(meta_num.get("nanity.attention.layer_norm_rms_epsilon", 1e-5))
    rope_base = f32(meta_num.get("nanity.rope.freq_base", 10000.0))
    rope_scale = f32(meta_num.get("nanity.rope.scale_linear", 1.0))
    rope_dim = u32(meta_num.get("nanity.rope.dimension_count", 0.0))
    if 0 in (n_embd, n_layer, n_head, n_kv, head_dim, n_ff):
        raise RuntimeError("NANITY: one or more required hyperparameters is zero.")
    if n_head % n_kv:
        raise RuntimeError(f"NANITY: attention.head_count ({n_head}) must be an exact multiple of "
                           f"attention.head_count_kv ({n_kv}) -- GQA grouping requires it.")
    q_dim, kv_dim = n_head * head_dim, n_kv * head_dim

    def shape_str(sh):
        return "[" + ", ".join(str(v) for v in sh) + "]"

    def find(name):
        if name not in table:
            raise RuntimeError(f"NANITY: required tensor '{name}' is missing.")
        return table[name]

    def check(name, *dims):
        sh = find(name)[0]
        if list(sh) != list(dims):
            raise RuntimeError(f"NANITY: tensor '{name}' has shape {shape_str(sh)}, expected "
                               f"{shape_str(dims)}.")

    te = find("token_embd.weight")[0]
    if len(te) != 2 or te[0] != n_embd:
        raise RuntimeError(f"NANITY: 'token_embd.weight' shape {shape_str(te)} is inconsistent with "
                           f"nanity.embedding_length={n_embd}.")
    n_vocab = u32(te[1])
    if "nanity.vocab_size" in meta_num and u32(meta_num["nanity.vocab_size"]) != n_vocab:
        raise RuntimeError(f"NANITY: nanity.vocab_size={u32(meta_num['nanity.vocab_size'])} disagrees with "
                           f"token_embd.weight's vocab dimension ({n_vocab}).")
    check("output_norm.weight", n_embd)
    if "output.weight" in table:
        sh = table["output.weight"][0]
        if list(sh) != [n_embd, n_vocab]:
            raise RuntimeError(f"NANITY: 'output.weight' shape {shape_str(sh)} doesn't match "
                               f"[embedding_length, vocab_size] = [{n_embd}, {n_vocab}].")
    for i in range(n_layer):
        p = f"blk.{i}."
        check(p + "attn_norm.weight", n_embd)
        check(p + "attn_q.weight", n_embd, q_dim)
        check(p + "attn_k.weight", n_embd, kv_dim)
        check(p + "attn_v.weight", n_embd, kv_dim)
        check(p + "attn_output.weight", q_dim, n_embd)
        check(p + "ffn_norm.weight", n_embd)
        check(p + "ffn_gate.weight", n_embd, n_ff)
        check(p + "ffn_up.weight", n_embd, n_ff)
        check(p + "ffn_down.weight", n_ff, n_embd)

    tensors = []
    for name, (shape, t, raw) in table.items():
        parts = name.split(".")
        if len(parts) == 2 and parts[1] == "weight" and parts[0] in ("token_embd", "output_norm", "output"):
            role, layer = _ROLE_NAMES[parts[0]], -1
        elif (len(parts) == 4 and parts[0] == "blk" and parts[1].isdigit() and parts[3] == "weight"
              and parts[2] in _ROLE_NAMES and _ROLE_NAMES[parts[2]] >= 3):
            role, layer = _ROLE_NAMES[parts[2]], int(parts[1])
        else:
            continue
        tensors.append((role, layer, raw, t, int(shape[0]), int(shape[1]) if len(shape) > 1 else 0))
    cfg = NctrConfig(n_vocab=n_vocab, n_embd=n_embd, n_layer=n_layer, n_head=n_head, n_kv_head=n_kv,
                     head_dim=head_dim, n_ff=n_ff, ctx_len=min(ctx_len, 4096), context_length=ctx_len,
                     rope_base=rope_base, rope_scale=rope_scale, rope_dim_count=rope_dim, norm_eps=norm_eps,
                     plain_ffn=False, bos_id=tok.get("tokenizer.ggml.bos_token_id", 1),
                     eos_id=tok.get("tokenizer.ggml.eos_token_id", 2),
                     unk_id=tok.get("tokenizer.ggml.unknown_token_id", 0))
    return cfg, tensors


# ---------------------------------------------------------------------------
# .nctr models (the reference's F32 export container)
# ---------------------------------------------------------------------------

# NCTRHeader (rawllm_nctr_loader.hpp:32-62): 116 bytes, little-endian, packed.
_NCTR_HEADER = struct.Struct("<4s10Iff I f II 6Q")
_NCTR_SLOT = struct.Struct("<IQQ")  # quant_type, data_offset, nbytes (:70-71)
NCTR_SPEC_VERSION = 1               # engine::kSpecVersion (rawllm_common.hpp:111)
NCTR_FLAG_USE_SWIGLU, NCTR_FLAG_HAS_OUTPUT_WEIGHT, NCTR_FLAG_HAS_OPT_STATE = 1, 2, 4


class NctrConfig:
    """engine::Config as NCTRLoader::validate_config fills it
    (rawllm_nctr_loader.hpp:146-184): the header's fields, ``ctx_len`` the KV
    capacity (kv_window = min(ctx_len, 4096)) and ``context_length`` the
    header's value, ``plain_ffn`` = not use_swiglu."""

    def __init__(self, **kw):
        self.__dict__.update(kw)


def load_nctr(path: str):
    """Open a .nctr file -- the container export_nctr writes
    (train_nanity_fixed.py:1259-1433), F32 tensors -- as (config, tensors)
    for :class:`Model`: ``tensors`` are (role, layer, bytes, ggml type, ne0,
    ne1) views of a read-only memory map, in the positional order of
    NCTRLoader::build_tensor_table (rawllm_nctr_loader.hpp:217-264).
    The checks and messages are NCTRLoader::open's (:87-137) and
    validate_config's."""
    mm = np.memmap(path, np.uint8, mode="r")
    size = mm.size
    if size < _NCTR_HEADER.size:
        raise RuntimeError("File too small to be NCTR (<header size): " + path)
    (magic, _fmt, spec, n_vocab, n_embd, n_layer, n_head, n_kv, head_dim, n_ff, ctx_len, rope_base, rope_scale,
     rope_dim, eps, flags, _align, man_off, man_len, tok_off, tok_len, table_off,
     data_off) = _NCTR_HEADER.unpack(bytes(mm[:_NCTR_HEADER.size]))
    if magic != b"NCTR":
        raise RuntimeError("Not an NCTR file: " + path)
    if spec != NCTR_SPEC_VERSION:
        raise RuntimeError(f"NCTR: file declares spec_version {spec}, runtime built against {NCTR_SPEC_VERSION}")

    def in_bounds(off, length):
        if off > size or length > size - off:
            raise RuntimeError(f"NCTR: section out of bounds (offset={off} len={length} file_size={size})")

    in_bounds(man_off, man_len)
    in_bounds(tok_off, tok_len)
    swiglu, has_output = bool(flags & NCTR_FLAG_USE_SWIGLU), bool(flags & NCTR_FLAG_HAS_OUTPUT_WEIGHT)
    q_dim, kv_dim = n_head * head_dim, n_kv * head_dim
    slots = [(0, -1, n_embd, n_vocab), (1, -1, n_embd, 0)] + ([(2, -1, n_embd, n_vocab)] if has_output else [])
    for i in range(n_layer):
        slots += [(3, i, n_embd, 0), (4, i, n_embd, q_dim), (5, i, n_embd, kv_dim), (6, i, n_embd, kv_dim),
                  (7, i, q_dim, n_embd), (8, i, n_embd, 0)]
        slots += ([(9, i, n_embd, n_ff)] if swiglu else []) + [(10, i, n_embd, n_ff), (11, i, n_ff, n_embd)]
    in_bounds(table_off, len(slots) * _NCTR_SLOT.size)
    tensors = []
    for k, (role, layer, ne0, ne1) in enumerate(slots):
        o = table_off + k * _NCTR_SLOT.size
        qtype, off, nbytes = _NCTR_SLOT.unpack(bytes(mm[o:o + _NCTR_SLOT.size]))
        in_bounds(data_off + off, nbytes)
        tensors.append((role, layer, mm[data_off + off:data_off + off + nbytes], qtype, ne0, ne1))
    if n_head == 0 or n_kv == 0 or n_head % n_kv != 0:
        raise RuntimeError(f"NCTR: n_head must be a nonzero multiple of n_kv_head (got {n_head} / {n_kv})")
    tok = json.loads(bytes(mm[tok_off:tok_off + tok_len]).decode("utf-8"))
    cfg = NctrConfig(n_vocab=n_vocab, n_embd=n_embd, n_layer=n_layer, n_head=n_head, n_kv_head=n_kv,
                     head_dim=head_dim, n_ff=n_ff, ctx_len=min(ctx_len, 4096), context_length=ctx_len,
                     rope_base=rope_base, rope_scale=rope_scale, rope_dim_count=rope_dim, norm_eps=eps,
                     plain_ffn=not swiglu, has_optimizer_state=bool(flags & NCTR_FLAG_HAS_OPT_STATE),
                     bos_id=int(tok.get("bos_id", 1)), eos_id=int(tok.get("eos_id", 2)),
                     unk_id=int(tok.get("unk_id", 0)), n_tokens=len(tok.get("tokens", [])),
                     manifest_json=bytes(mm[man_off:man_off + man_len]).decode("utf-8", "replace"))
    return cfg, tensors


class Model:
    """A NANITY decoder on the current device (neon_cuda_model_*).

    ``cfg`` has the fields of engine::Config the forward pass reads (n_vocab,
    n_embd, n_layer, n_head, n_kv_head, head_dim, n_ff, ctx_len, rope_base,
    rope_scale, rope_dim_count, norm_eps); ``tensors`` yields (role, layer,
    GGUF bytes, ggml type, ne0, ne1); ``quantize`` (a GGML type) quantises
    float matrices on load. With a connected :class:`Comm`, the
    model is this rank's tensor-parallel share; every rank passes the WHOLE
    tensors and makes the same calls in the same order."""

    def __init__(self, cfg, tensors=(), comm: Comm | None = None, quantize: int | None = None):
        L = load()
        self.cfg = cfg
        self.comm = comm
        h = _vp()
        _check(L.neon_cuda_model_create_tp(C.byref(_config(cfg)), comm.handle if comm else None, C.byref(h)))
        self.handle = h.value
        self._fin = weakref.finalize(self, L.neon_cuda_model_free, self.handle)
        if quantize is not None:
            # float matrices (a .nctr model) quantised on load, as gguf-py exports them
            _check(L.neon_cuda_model_set_quantize(self.handle, int(quantize)))
        for t in tensors:
            self.set_tensor(*t)

    def set_tensor(self, role, layer, raw, ggml_type, ne0, ne1):
        raw = np.ascontiguousarray(raw)
        _check(load().neon_cuda_model_set_tensor(self.handle, int(role), int(layer), raw.ctypes.data, raw.nbytes,
                                                 int(ggml_type), int(ne0), int(ne1)))

    def forward(self, tokens) -> np.ndarray:
        """fwd::transformer_forward: append tokens, return the last logits."""
        t = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
        out = np.zeros(self.cfg.n_vocab, np.float32)
        _check(load().neon_cuda_model_forward(self.handle, t.ctypes.data, t.size, out.ctypes.data))
        return out

    def generate(self, prompt, max_new: int, eos_id: int = -1) -> np.ndarray:
        """Greedy run_generation on the device; returns the emitted tokens."""
        p = np.ascontiguousarray(prompt, dtype=np.int32).reshape(-1)
        out = np.zeros(max(1, max_new), np.int32)
        n = _sz()
        _check(load().neon_cuda_model_generate(self.handle, p.ctypes.data, p.size, max_new, int(eos_id),
                                               out.ctypes.data, C.byref(n)))
        return out[:n.value].copy()

    @property
    def length(self) -> int:
        n = _sz()
        _check(load().neon_cuda_model_length(self.handle, C.byref(n)))
        return n.value

    def set_length(self, n: int) -> None:
        _check(load().neon_cuda_model_set_length(self.handle, n))

    def kv_shift(self, keep: int, discard: int) -> None:
        """fwd::kv_cache_shift: forget positions [keep, keep+discard), slide the rest down."""
        _check(load().neon_cuda_model_kv_shift(self.handle, int(keep), int(discard)))

    def read_kv(self, layer: int, n: int):
        """K and V cache rows [0, n) of `layer` (this rank's KV heads)."""
        world = self.comm.world if self.comm else 1
        kv = self.cfg.n_kv_head // world * self.cfg.head_dim
        k = np.zeros((n, kv), np.float32)
        v = np.zeros((n, kv), np.float32)
        _check(load().neon_cuda_model_read_kv(self.handle, layer, n, k.ctypes.data, v.ctypes.data))
        return k, v

    @property
    def decode_ms(self) -> float:
        ms = C.c_float()
        _check(load().neon_cuda_model_decode_ms(self.handle, C.byref(ms)))
        return ms.value

    @property
    def forward_ms(self) -> float:
        """Device time of the last forward (for generate: the prompt pass), ms."""
        ms = C.c_float()
        _check(load().neon_cuda_model_forward_ms(self.handle, C.byref(ms)))
        return ms.value

    def free(self) -> None:
        self._fin()
