"""ctypes bindings for the test oracle -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.

Two libraries sit behind this module:

* ``oracle/liboracle.so`` -- the plain-C restatement of the reference's
  quantized matvec path (``oracle/neon_oracle.c``), single-threaded.
* ``oracle/_ref/libneon_ref.so`` -- the reference's own CPU path
  (``rawllm_forward.hpp``) compiled from the reference sources with the
  reference's flags by ``oracle/Makefile``; present wherever it was built.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` import this module. The product library never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libneon_ref.so")

GGML_Q4_0 = 2
GGML_Q8_0 = 8

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_sz = C.c_size_t


def build(with_ref: bool = False) -> None:
    """Compile the oracle (and, if asked and the reference tree exists, the
    reference harness) with oracle/Makefile."""
    subprocess.check_call(["make", "-s", "-C", HERE, "liboracle.so"])
    if with_ref:
        subprocess.check_call(["make", "-s", "-C", HERE, "ref"])


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build()
        L = C.CDLL(ORACLE_SO)
        L.oracle_fp16_to_fp32.argtypes = [C.c_uint16]
        L.oracle_fp16_to_fp32.restype = C.c_float
        L.oracle_quantize_rows_q8_0.argtypes = [_f32p, _sz, _sz, _sz, _f32p, _i8p]
        L.oracle_quantize_rows_q8_0.restype = None
        L.oracle_block_isum.argtypes = [_u8p, _i8p]
        L.oracle_block_isum.restype = C.c_int32
        L.oracle_dot_q4_0_q8_0.argtypes = [_u8p, _f32p, _i8p, _sz]
        L.oracle_dot_q4_0_q8_0.restype = C.c_float
        L.oracle_dot_f32.argtypes = [_f32p, _f32p, _sz]
        L.oracle_dot_f32.restype = C.c_float
        L.oracle_proj_all_positions.argtypes = [C.c_int, _u8p, _sz, _sz, _f32p, _sz, _f32p, _sz,
                                                _sz, _f32p, _i8p, _f32p]
        L.oracle_proj_all_positions.restype = C.c_int
        L.oracle_bf16_to_fp32.argtypes = [C.c_uint16]
        L.oracle_bf16_to_fp32.restype = C.c_float
        L.oracle_dequantize_row.argtypes = [C.c_int, _u8p, _sz, _f32p]
        L.oracle_dequantize_row.restype = C.c_int
        L.oracle_row_bytes.argtypes = [C.c_int, _sz]
        L.oracle_row_bytes.restype = _sz
        L.oracle_block_elems.argtypes = [C.c_int]
        L.oracle_block_elems.restype = _sz
        _lib = L
    return _lib


def ref_tree() -> str:
    """The reference source tree oracle/Makefile compiles from (its REF
    setting, overridable by the REF environment variable), or "" if absent."""
    path = os.environ.get("REF", "")
    if not path:
        with open(os.path.join(HERE, "Makefile")) as f:
            for line in f:
                if line.startswith("REF ?="):
                    path = line.split("=", 1)[1].strip()
    return path if path and os.path.isdir(path) else ""


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref():
    """The reference's own CPU path, or None when oracle/_ref was not built."""
    global _ref
    if _ref is None:
        if not ref_available():
            return None
        L = C.CDLL(REF_SO)
        L.ref_last_error.restype = C.c_char_p
        L.ref_pool_new.argtypes = [C.c_int]
        L.ref_pool_new.restype = C.c_void_p
        L.ref_pool_free.argtypes = [C.c_void_p]
        L.ref_pool_size.argtypes = [C.c_void_p]
        L.ref_fp16_to_fp32.argtypes = [C.c_uint16]
        L.ref_fp16_to_fp32.restype = C.c_float
        L.ref_quantize_rows_q8_0.argtypes = [_f32p, _sz, _sz, _sz, _f32p, _i8p]
        L.ref_quantize_rows_q8_0.restype = None
        L.ref_block_isum.argtypes = [_u8p, _i8p]
        L.ref_block_isum.restype = C.c_int32
        L.ref_block_isum_scalar.argtypes = [_u8p, _i8p]
        L.ref_block_isum_scalar.restype = C.c_int32
        L.ref_dot_q4_0_q8_0.argtypes = [_u8p, _f32p, _i8p, _sz]
        L.ref_dot_q4_0_q8_0.restype = C.c_float
        L.ref_dot_f32.argtypes = [_f32p, _f32p, _sz]
        L.ref_dot_f32.restype = C.c_float
        L.ref_proj_all_positions.argtypes = [C.c_void_p, _u8p, C.c_int, _sz, _sz, _f32p, _sz,
                                             _f32p, _sz, _sz]
        L.ref_proj_all_positions.restype = C.c_int
        L.ref_dequantize_row.argtypes = [C.c_int, _u8p, _sz, _f32p]
        L.ref_dequantize_row.restype = C.c_int
        L.ref_proj_all_positions_multi.argtypes = [
            C.c_void_p, _sz, C.POINTER(C.c_void_p), C.POINTER(C.c_int), C.POINTER(_sz),
            C.POINTER(_sz), C.POINTER(C.c_void_p), C.POINTER(_sz), _f32p, _sz, _sz]
        L.ref_proj_all_positions_multi.restype = C.c_int
        _ref = L
    return _ref


# ----------------------------------------------------------------------------
# numpy-facing helpers (oracle restatement)
# ----------------------------------------------------------------------------

def quantize_rows_q8_0(X: np.ndarray, cols: int | None = None):
    """X: (seq, x_stride) float32 -> (d (seq, cols/32) float32, q (seq, cols) int8)."""
    X = np.ascontiguousarray(X, dtype=np.float32)
    seq, stride = X.shape
    cols = stride if cols is None else cols
    d = np.empty((seq, cols // 32), np.float32)
    q = np.empty((seq, cols), np.int8)
    lib().oracle_quantize_rows_q8_0(X.reshape(-1), stride, cols, seq, d.reshape(-1), q.reshape(-1))
    return d, q


def dequantize_row(ggml_type: int, row: np.ndarray, n: int) -> np.ndarray:
    """Oracle fp32 values of the first n elements of raw GGUF bytes `row`."""
    out = np.empty(max(1, n), np.float32)
    if lib().oracle_dequantize_row(ggml_type, np.ascontiguousarray(row, np.uint8).reshape(-1), n, out) != 0:
        raise RuntimeError(f"oracle_dequantize_row: type {ggml_type} not supported")
    return out[:n]


def ref_dequantize_row(ggml_type: int, row: np.ndarray, n: int) -> np.ndarray:
    """The reference's own fwd::dequantize_row on the same bytes."""
    out = np.empty(max(1, n), np.float32)
    R = ref()
    if R.ref_dequantize_row(ggml_type, np.ascontiguousarray(row, np.uint8).reshape(-1), n, out) != 0:
        raise RuntimeError(R.ref_last_error().decode())
    return out[:n]


def proj_all_positions(ggml_type: int, W: np.ndarray, rows: int, cols: int, X: np.ndarray,
                       x_stride: int | None = None, y_stride: int | None = None,
                       seq: int | None = None) -> np.ndarray:
    """Oracle Y (seq, y_stride) for raw GGUF bytes W (rows * row_bytes uint8)."""
    X = np.ascontiguousarray(X, dtype=np.float32)
    if X.ndim == 1:
        X = X.reshape(1, -1)
    seq = X.shape[0] if seq is None else seq
    x_stride = X.shape[1] if x_stride is None else x_stride
    y_stride = rows if y_stride is None else y_stride
    Y = np.zeros((seq, y_stride), np.float32)
    sd = np.empty(max(1, seq * cols // 32), np.float32)
    sq = np.empty(max(1, seq * cols), np.int8)
    rb = np.empty(max(1, cols), np.float32)
    rc = lib().oracle_proj_all_positions(ggml_type, np.ascontiguousarray(W).reshape(-1), rows, cols,
                                         X.reshape(-1), x_stride, Y.reshape(-1), y_stride, seq,
                                         sd, sq, rb)
    if rc != 0:
        raise RuntimeError("oracle_proj_all_positions: bad argument")
    return Y


# ----------------------------------------------------------------------------
# numpy-facing helpers (reference's own CPU path)
# ----------------------------------------------------------------------------

class RefPool:
    """util::ThreadPool of the reference, kept alive across calls."""

    def __init__(self, n_threads: int):
        self.L = ref()
        if self.L is None:
            raise RuntimeError("reference CPU path not built (oracle/_ref missing)")
        self.h = self.L.ref_pool_new(int(n_threads))
        self.n = self.L.ref_pool_size(self.h)

    def close(self):
        if self.h:
            self.L.ref_pool_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def proj_all_positions(self, ggml_type, W, rows, cols, X, Y, x_stride=None, y_stride=None,
                           seq=None):
        seq = X.shape[0] if seq is None else seq
        x_stride = X.shape[-1] if x_stride is None else x_stride
        y_stride = Y.shape[-1] if y_stride is None else y_stride
        rc = self.L.ref_proj_all_positions(self.h, W.reshape(-1), ggml_type, rows, cols,
                                           X.reshape(-1), x_stride, Y.reshape(-1), y_stride, seq)
        if rc != 0:
            raise RuntimeError(self.L.ref_last_error().decode())
        return Y

    def proj_all_positions_multi(self, targets, X, x_stride=None, seq=None):
        """targets: list of (ggml_type, W bytes, rows, cols, Y (seq, y_stride) float32)."""
        n = len(targets)
        seq = X.shape[0] if seq is None else seq
        x_stride = X.shape[-1] if x_stride is None else x_stride
        Ws = (C.c_void_p * n)(*[t[1].ctypes.data for t in targets])
        types = (C.c_int * n)(*[t[0] for t in targets])
        rows = (_sz * n)(*[t[2] for t in targets])
        cols = (_sz * n)(*[t[3] for t in targets])
        Ys = (C.c_void_p * n)(*[t[4].ctypes.data for t in targets])
        ys = (_sz * n)(*[t[4].shape[-1] for t in targets])
        rc = self.L.ref_proj_all_positions_multi(self.h, n, Ws, types, rows, cols, Ys, ys,
                                                 X.reshape(-1), x_stride, seq)
        if rc != 0:
            raise RuntimeError(self.L.ref_last_error().decode())


# ----------------------------------------------------------------------------
# Decode step: the restatement (C) and the reference's transformer_forward
# ----------------------------------------------------------------------------

class _Config(C.Structure):
    _fields_ = [(f, C.c_uint32) for f in ("n_vocab", "n_embd", "n_layer", "n_head", "n_kv_head", "head_dim",
                                          "n_ff", "ctx_len")] + [
        ("rope_base", C.c_float), ("rope_scale", C.c_float), ("rope_dim_count", C.c_uint32),
        ("norm_eps", C.c_float), ("plain_ffn", C.c_uint32)]


def _config(cfg):
    return _Config(*[getattr(cfg, f) for f in ("n_vocab", "n_embd", "n_layer", "n_head", "n_kv_head",
                                               "head_dim", "n_ff", "ctx_len")],
                   cfg.rope_base, cfg.rope_scale, cfg.rope_dim_count, cfg.norm_eps,
                   1 if getattr(cfg, "plain_ffn", False) else 0)


class Model:
    """A decoder held by the oracle restatement (kind="port") or by the
    reference's own transformer_forward (kind="reference").

    forward(tokens) appends the tokens to the KV cache and returns the logits
    of the last one, as fwd::transformer_forward does."""

    def __init__(self, cfg, tensors, kind="port", threads=None):
        self.cfg, self.kind = cfg, kind
        if kind == "port":
            L = lib()
            L.oracle_model_new.restype = C.c_void_p
            L.oracle_model_new.argtypes = [C.POINTER(_Config)]
            L.oracle_model_free.argtypes = [C.c_void_p]
            L.oracle_model_set.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, _sz, C.c_int, _sz, _sz]
            L.oracle_model_forward.argtypes = [C.c_void_p, C.c_void_p, _sz, _f32p]
            L.oracle_model_length.argtypes = [C.c_void_p]
            L.oracle_model_length.restype = _sz
            L.oracle_model_set_length.argtypes = [C.c_void_p, _sz]
            L.oracle_model_kv.argtypes = [C.c_void_p, C.c_int, _sz, _f32p, _f32p]
            L.oracle_model_kv_shift.argtypes = [C.c_void_p, _sz, _sz]
            self._shift = L.oracle_model_kv_shift
            self.L, self.pool = L, None
            self._new, self._free, self._set = L.oracle_model_new, L.oracle_model_free, L.oracle_model_set
            self._len, self._setlen, self._kv = L.oracle_model_length, L.oracle_model_set_length, L.oracle_model_kv
            self._fwd = lambda h, t, n, out: L.oracle_model_forward(h, t, n, out)
        elif kind == "reference":
            L = ref()
            if L is None:
                raise RuntimeError("reference CPU path not built (oracle/_ref missing)")
            L.ref_model_new.restype = C.c_void_p
            L.ref_model_new.argtypes = [C.POINTER(_Config)]
            L.ref_model_free.argtypes = [C.c_void_p]
            L.ref_model_set.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, _sz, C.c_int, _sz, _sz]
            L.ref_model_forward.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, _sz, _f32p]
            L.ref_model_length.argtypes = [C.c_void_p]
            L.ref_model_length.restype = _sz
            L.ref_model_set_length.argtypes = [C.c_void_p, _sz]
            L.ref_model_kv.argtypes = [C.c_void_p, C.c_int, _sz, _f32p, _f32p]
            L.ref_model_kv_shift.argtypes = [C.c_void_p, _sz, _sz]
            self._shift = L.ref_model_kv_shift
            self.L = L
            self.pool = RefPool(threads or os.cpu_count() or 1)
            self._new, self._free, self._set = L.ref_model_new, L.ref_model_free, L.ref_model_set
            self._len, self._setlen, self._kv = L.ref_model_length, L.ref_model_set_length, L.ref_model_kv
            self._fwd = lambda h, t, n, out: L.ref_model_forward(h, self.pool.h, t, n, out)
        else:
            raise ValueError(kind)
        self._cfg = _config(cfg)
        self.h = self._new(C.byref(self._cfg))
        for role, layer, raw, typ, ne0, ne1 in tensors:
            raw = np.ascontiguousarray(raw)
            if self._set(self.h, role, layer, raw.ctypes.data, raw.nbytes, typ, ne0, ne1) != 0:
                raise RuntimeError(f"bad tensor role {role} layer {layer}")

    def forward(self, tokens):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.zeros(self.cfg.n_vocab, np.float32)
        rc = self._fwd(self.h, t.ctypes.data, t.size, out)
        if rc != 0:
            raise RuntimeError("forward failed" + (": " + self.L.ref_last_error().decode() if self.kind == "reference" else ""))
        return out

    @property
    def length(self):
        return int(self._len(self.h))

    def set_length(self, n):
        self._setlen(self.h, n)

    def kv_shift(self, keep, discard):
        """fwd::kv_cache_shift: forget positions [keep, keep+discard)."""
        self._shift(self.h, keep, discard)

    def kv(self, layer, n):
        k = np.zeros((n, self.cfg.kv_dim), np.float32)
        v = np.zeros((n, self.cfg.kv_dim), np.float32)
        self._kv(self.h, layer, n, k.reshape(-1), v.reshape(-1))
        return k, v

    def generate_greedy(self, prompt, n_new):
        """run_generation's loop (NEON-3.cpp:744-758) with greedy sampling
        (first maximum, NEON-3.cpp:471-474). Returns tokens and per-step logits."""
        logits = self.forward(prompt)
        toks, all_logits = [], [logits]
        nxt = int(np.argmax(logits))
        for _ in range(n_new):
            toks.append(nxt)
            logits = self.forward(np.array([nxt], np.int32))
            all_logits.append(logits)
            nxt = int(np.argmax(logits))
        return np.array(toks, np.int32), np.stack(all_logits)

    def close(self):
        if self.h:
            self._free(self.h)
            self.h = None
        if self.pool is not None:
            self.pool.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
