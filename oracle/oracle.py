"""ctypes binding of the CPU oracle (oracle/build/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, never by the sampler library or its binding.
The oracle restates the reference's DoSample (src/Gemma4.Model.pas:2615-2827)
and its helpers in C; see oracle/ref_sampler.h for the arithmetic model and
the parity status (unpinned by the reference; pinned by hand-derived
known-answer tests).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import POINTER, c_double, c_float, c_int32, c_int64, c_uint16, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "build", "liboracle.so")

TIE_HEAP, TIE_LOWER = 0, 1
PATH_TOPK, PATH_FULL = 0, 1
DTYPE_F32, DTYPE_BF16 = 0, 1
VARIANT_F32, VARIANT_F64, VARIANT_F32_LIBM = 0, 1, 2


class RefParams(ctypes.Structure):
    _fields_ = [("temperature", c_float), ("top_k", c_int32), ("top_p", c_float),
                ("repetition_penalty", c_float)]


class RefTrace(ctypes.Structure):
    _fields_ = [("token", c_int32), ("path", c_int32), ("count", c_int32), ("best", c_int32),
                ("fallback", c_int32), ("drawn", c_int32), ("thr", c_float), ("max_s", c_float),
                ("cum_prev", c_double), ("cum_at", c_double), ("sum", c_double),
                ("boundary", c_double)]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


_lib = None


def build():
    """Compiles the oracle with its Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        build()
    lib = ctypes.CDLL(LIB_PATH)
    lib.ref_bf16_to_f32.restype = c_float
    lib.ref_bf16_to_f32.argtypes = [c_uint16]
    lib.ref_f32_to_bf16_trunc.restype = c_uint16
    lib.ref_f32_to_bf16_trunc.argtypes = [c_float]
    lib.ref_f16_to_f32.restype = c_float
    lib.ref_f16_to_f32.argtypes = [c_uint16]
    lib.ref_f32_to_f16_trunc.restype = c_uint16
    lib.ref_f32_to_f16_trunc.argtypes = [c_float]
    lib.g4_expf.restype = c_float
    lib.g4_expf.argtypes = [c_float]
    lib.g4_tanhf.restype = c_float
    lib.g4_tanhf.argtypes = [c_float]
    for fn in (lib.ref_topk_heap, lib.ref_topk_lower):
        fn.restype = c_int32
        fn.argtypes = [c_void_p, c_int32, c_int32, c_void_p]
    lib.ref_sample.restype = c_int32
    lib.ref_sample.argtypes = [c_void_p, c_int32, POINTER(RefParams), c_float, c_double, c_int32,
                               c_int32, POINTER(RefTrace), c_void_p, c_void_p]
    lib.ref_sample_batch.restype = c_int32
    lib.ref_sample_batch.argtypes = [c_void_p, c_int32, c_int32, c_int32, c_int64, c_void_p, c_int32,
                                     c_float, c_void_p, c_int32, c_int32, c_void_p, c_int32]
    lib.ref_rmsnorm.restype = None
    lib.ref_rmsnorm.argtypes = [c_void_p, c_void_p, c_void_p, c_int32, c_float]
    lib.ref_matvec_q4.restype = None
    lib.ref_matvec_q4.argtypes = [c_void_p, c_void_p, c_void_p, c_int32, c_int32]
    lib.ref_matvec_q4_f64.restype = None
    lib.ref_matvec_q4_f64.argtypes = [c_void_p, c_void_p, c_void_p, c_int32, c_int32]
    lib.ref_matvec_q4_mt.restype = None
    lib.ref_matvec_q4_mt.argtypes = [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32]
    lib.ref_quantize_q8_1.restype = None
    lib.ref_quantize_q8_1.argtypes = [c_void_p, c_int32, c_void_p, c_void_p]
    lib.ref_matvec_q4q8.restype = None
    lib.ref_matvec_q4q8.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32]
    _lib = lib
    return lib


def _ptr(a):
    return c_void_p(a.ctypes.data)


def params(temperature=1.0, top_k=64, top_p=0.95, repetition_penalty=1.0) -> RefParams:
    return RefParams(float(temperature), int(top_k), float(top_p), float(repetition_penalty))


def as_f32(row, dtype=DTYPE_F32):
    """fp32 view of one row; bf16 rows (uint16 bits) widen like TBFloat16.ToSingle."""
    row = np.asarray(row)
    if dtype == DTYPE_BF16 or row.dtype == np.uint16:
        return (row.astype(np.uint32) << 16).view(np.float32)
    return np.ascontiguousarray(row, dtype=np.float32)


def sample(logits, p: RefParams, softcap: float, u: float, variant=VARIANT_F32, tie=TIE_LOWER,
           want_probs=False):
    """One DoSample on one fp32 row.  Returns (token, trace dict, ids, probs)."""
    lib = load()
    x = as_f32(logits)
    V = x.shape[0]
    tr = RefTrace()
    full = p.top_k <= 0 or p.top_k >= V
    n = V if full else max(p.top_k, 1)
    ids = np.full(n, -1, dtype=np.int32)
    probs = None
    if want_probs:
        probs = np.zeros(n, dtype=np.float64 if variant == VARIANT_F64 else np.float32)
    tok = lib.ref_sample(_ptr(x), V, ctypes.byref(p), softcap, float(u), variant, tie,
                         ctypes.byref(tr), _ptr(ids), _ptr(probs) if probs is not None else None)
    cnt = tr.count
    return tok, tr.as_dict(), ids[:cnt] if not full else None, (
        probs[:cnt] if probs is not None else None)


def sample_batch(logits, dtype, plist, softcap, u, variant=VARIANT_F32, tie=TIE_LOWER, nthreads=1):
    """Rows sampled independently on nthreads threads; logits [rows, stride]."""
    lib = load()
    logits = np.ascontiguousarray(logits)
    rows, stride = logits.shape
    if isinstance(plist, RefParams):
        parr, pstride = (RefParams * 1)(plist), 0
    else:
        parr, pstride = (RefParams * len(plist))(*plist), 1
    u = np.ascontiguousarray(u, dtype=np.float64)
    out = np.empty(rows, dtype=np.int32)
    lib.ref_sample_batch(_ptr(logits), dtype, rows, stride, stride, ctypes.cast(parr, c_void_p),
                         pstride, softcap, _ptr(u), variant, tie, _ptr(out), nthreads)
    return out


def topk(logits, K, tie=TIE_LOWER):
    lib = load()
    x = as_f32(logits)
    out = np.empty(max(K, 1), dtype=np.int32)
    fn = lib.ref_topk_heap if tie == TIE_HEAP else lib.ref_topk_lower
    n = fn(_ptr(x), x.shape[0], K, _ptr(out))
    return out[:n]


def matvec_q4(blocks: np.ndarray, vec: np.ndarray, rows: int, cols: int, f64=False):
    lib = load()
    vec = np.ascontiguousarray(vec, dtype=np.float32)
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    out = np.empty(rows, dtype=np.float64 if f64 else np.float32)
    (lib.ref_matvec_q4_f64 if f64 else lib.ref_matvec_q4)(_ptr(blocks), _ptr(vec), _ptr(out), rows, cols)
    return out


def matvec_q4_mt(blocks: np.ndarray, vec: np.ndarray, rows: int, cols: int, nthreads: int = 1):
    """CpuMatVecQ4 (src/Gemma4.Tensors.pas:546-590) on `nthreads` threads
    (same per-row arithmetic as matvec_q4)."""
    lib = load()
    vec = np.ascontiguousarray(vec, dtype=np.float32)
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    out = np.empty(rows, dtype=np.float32)
    lib.ref_matvec_q4_mt(_ptr(blocks), _ptr(vec), _ptr(out), rows, cols, nthreads)
    return out


def quantize_q8_1(x: np.ndarray):
    """gemma4_quantize_q8.comp: (int8 qs [n], fp16 bits ds [n/32, 2] = (d, d*sum(q)))."""
    lib = load()
    x = np.ascontiguousarray(x, dtype=np.float32)
    qs = np.empty(x.shape[0], dtype=np.int8)
    ds = np.empty((x.shape[0] // 32, 2), dtype=np.uint16)
    lib.ref_quantize_q8_1(_ptr(x), x.shape[0], _ptr(qs), _ptr(ds))
    return qs, ds


def matvec_q4q8(blocks: np.ndarray, vec: np.ndarray, rows: int, cols: int, nthreads: int = 1):
    """The reference's GPU LM head: Q8_1 activations and the DP4A matvec
    (gemma4_quantize_q8.comp, gemma4_matvec_q4q8.comp)."""
    lib = load()
    qs, ds = quantize_q8_1(vec)
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    out = np.empty(rows, dtype=np.float32)
    lib.ref_matvec_q4q8(_ptr(blocks), _ptr(qs), _ptr(ds), _ptr(out), rows, cols, nthreads)
    return out


def rmsnorm(x, w, eps=1e-6):
    """CpuRmsNorm on one fp32 vector."""
    lib = load()
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.empty_like(x)
    lib.ref_rmsnorm(_ptr(x), _ptr(w), _ptr(out), x.shape[0], eps)
    return out
