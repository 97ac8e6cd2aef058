"""ctypes binding of libg4sampler.so, the C ABI declared in include/g4sampler.h.

This is how the test suite and bench.py reach the CUDA sampler: exactly the
calls an Object Pascal host makes through its `external 'libg4sampler.so'`
declarations (pascal/G4Sampler.pas).  Device buffers are passed as raw
pointers (for example torch tensors' data_ptr()).  There is no fallback: if
the shared library is missing or no B200 is present, the calls fail loudly.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_double, c_float, c_int32, c_int64, c_uint32, c_void_p

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libg4sampler.so")

F32, BF16 = 0, 1
OK, ERR_ARG, ERR_CUDA, ERR_NOMEM, ERR_CAPACITY, ERR_NCCL, ERR_TIMEOUT, ERR_STATE, ERR_UNAVAILABLE = (
    0, -1, -2, -3, -4, -5, -6, -7, -8)
ROW_FALLBACK, ROW_EMPTY, ROW_FULL_PATH, ROW_GREEDY = 1, 2, 4, 8
PHASE_FULL_STREAM_ONLY, PHASE_LMHEAD_UNFUSED = 1, 2
FLAG_HOST_STAGING = 1


class Params(ctypes.Structure):
    """TSamplingParams (src/Gemma4.Model.pas:70-76), 16 bytes."""

    _fields_ = [("temperature", c_float), ("top_k", c_int32), ("top_p", c_float),
                ("repetition_penalty", c_float)]

    def __repr__(self):
        return (f"Params(T={self.temperature}, K={self.top_k}, P={self.top_p}, "
                f"rp={self.repetition_penalty})")


class TensorInfo(ctypes.Structure):
    """g4s_tensor_info: TTensorInfo (src/Gemma4.Types.pas:119-129)."""

    _fields_ = [("name", ctypes.c_char * 256), ("source_dtype", c_int32), ("output_dtype", c_int32),
                ("offset", ctypes.c_uint64), ("size", ctypes.c_uint64), ("ndim", c_int32),
                ("shape", c_int64 * 8)]

    @property
    def dims(self):
        return tuple(self.shape[i] for i in range(self.ndim))


DT_UNKNOWN, DT_BF16, DT_F16, DT_F32, DT_Q4_0 = 0, 1, 2, 3, 4


class Outputs(ctypes.Structure):
    _fields_ = [("token_prob", c_void_p), ("row_flags", c_void_p), ("cand_ids", c_void_p),
                ("cand_probs", c_void_p), ("cand_stride", c_int32), ("phase_mask", c_int32),
                ("full_probs", c_void_p)]


# every entry point include/g4sampler.h declares, with (restype, argtypes)
SIGNATURES = {
    "g4s_version": (c_int32, []),
    "g4s_params_defaults": (None, [POINTER(Params)]),
    "g4s_create": (c_int32, [c_int32, c_int32, c_int32, c_uint32, POINTER(c_void_p)]),
    "g4s_destroy": (c_int32, [c_void_p]),
    "g4s_last_error": (c_char_p, [c_void_p]),
    "g4s_stream": (c_void_p, [c_void_p]),
    "g4s_workspace_bytes": (c_int64, [c_void_p]),
    "g4s_sample": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int64, POINTER(Params),
                             c_int32, c_float, c_void_p, c_void_p, c_void_p]),
    "g4s_sample_ex": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int64,
                                POINTER(Params), c_int32, c_float, c_void_p, c_void_p,
                                POINTER(Outputs), c_void_p]),
    "g4s_sample_host": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int64,
                                  POINTER(Params), c_int32, c_float, c_void_p, c_void_p]),
    "g4s_sample_topk_noalloc": (c_int32, [c_void_p, c_int32, c_int32, c_int32, c_int64, POINTER(Params),
                                          c_float, c_void_p, c_void_p, c_void_p]),
    "g4s_device_status": (c_int32, [c_void_p]),
    "g4s_set_wait_limit": (c_int32, [c_void_p, c_int64]),
    "g4s_q4_repack": (c_int32, [c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_void_p]),
    "g4s_lmhead_sample": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_float, c_void_p, c_void_p,
                                    c_int32, POINTER(Params), c_int32, c_float, c_void_p, c_void_p,
                                    POINTER(Outputs), c_void_p, c_void_p]),
    "g4s_shard_lists": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int64, c_int32, c_int32,
                                  POINTER(Params), c_int32, c_float, c_void_p, c_void_p, c_void_p]),
    "g4s_shard_resolve": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int64, c_int32, c_int32,
                                    POINTER(Params), c_int32, c_float, c_void_p, c_void_p, POINTER(Outputs),
                                    c_void_p]),
    "g4s_shard_merge": (c_int32, [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, POINTER(Params),
                                  c_int32, c_float, c_void_p, c_void_p, POINTER(Outputs), c_void_p]),
    "g4s_shard_unique_id": (c_int32, [c_void_p]),
    "g4s_shard_set_timeout": (c_int32, [c_void_p, c_int64]),
    "g4s_shard_wait": (c_int32, [c_void_p, c_void_p, c_int64]),
    "g4s_shard_abort": (c_int32, [c_void_p]),
    "g4s_shard_init": (c_int32, [c_void_p, c_int32, c_int32, c_int32, c_void_p]),
    "g4s_shard_sample": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_int64, POINTER(Params), c_int32,
                                   c_float, c_void_p, c_void_p, POINTER(Outputs), c_void_p]),
    "g4s_vpk_open": (c_int32, [c_char_p, c_char_p, c_char_p, POINTER(c_void_p)]),
    "g4s_vpk_close": (c_int32, [c_void_p]),
    "g4s_vpk_tensor_count": (c_int32, [c_void_p]),
    "g4s_vpk_tensor_at": (c_int32, [c_void_p, c_int32, POINTER(TensorInfo)]),
    "g4s_vpk_find": (c_int32, [c_void_p, c_char_p, POINTER(TensorInfo)]),
    "g4s_vpk_data": (c_void_p, [c_void_p, POINTER(TensorInfo)]),
    "g4s_vpk_verify": (c_int32, [c_void_p, c_char_p]),
    "g4s_vpk_load_lmhead": (c_int32, [c_void_p, c_int32, c_void_p, c_void_p, c_int32, POINTER(c_int32),
                                      POINTER(c_int32), c_void_p]),
}
SHARD_LIST = 256       # G4S_SHARD_LIST
SHARD_UID_BYTES = 128  # G4S_SHARD_UID_BYTES


def shard_slices(vocab: int, world: int):
    """Rank r's [start, stop) of the vocabulary (contiguous, ceil(vocab/world) ids)."""
    S = -(-vocab // world)
    return [(r * S, min(vocab, (r + 1) * S)) for r in range(world)]

_lib = None


def load(path: str = LIB_PATH):
    """Loads the shared library (once) and declares every signature."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is not built: run `python -c 'import __graft_entry__ as g; g.build()'`")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def q4_repack(blocks_ptr: int, vocab: int, hidden: int, nib_ptr: int, scales_ptr: int, stream: int | None = None):
    """g4s_q4_repack: reference Q4_0 blocks -> nibble / scale planes (device pointers)."""
    lib = load()
    rc = lib.g4s_q4_repack(c_void_p(blocks_ptr), vocab, hidden, c_void_p(nib_ptr), c_void_p(scales_ptr),
                           c_void_p(stream) if stream else None)
    if rc != OK:
        raise G4SError(rc, lib.g4s_last_error(None).decode())


def shard_unique_id() -> bytes:
    """g4s_shard_unique_id: the 128 bytes every rank passes to shard_init."""
    lib = load()
    buf = ctypes.create_string_buffer(SHARD_UID_BYTES)
    rc = lib.g4s_shard_unique_id(buf)
    if rc != OK:
        raise G4SError(rc, lib.g4s_last_error(None).decode())
    return buf.raw


class G4SError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"g4s error {code}: {msg}")
        self.code = code


def make_params(temperature=1.0, top_k=64, top_p=0.95, repetition_penalty=1.0) -> Params:
    return Params(float(temperature), int(top_k), float(top_p), float(repetition_penalty))


def params_array(rows):
    """ctypes array of Params from a sequence of (T, K, P) or Params.  An array
    this function made is passed through unchanged, so a caller that samples
    the same per-row settings every step converts them once."""
    if isinstance(rows, ctypes.Array) and rows._type_ is Params:
        return rows
    arr = (Params * len(rows))()
    for i, r in enumerate(rows):
        arr[i] = r if isinstance(r, Params) else make_params(*r)
    return arr


class Sampler:
    """RAII wrapper of one g4s_ctx."""

    def __init__(self, device: int = 0, max_rows: int = 256, max_vocab: int = 262144, flags: int = 0):
        self.lib = load()
        h = c_void_p()
        rc = self.lib.g4s_create(device, max_rows, max_vocab, flags, ctypes.byref(h))
        if rc != OK:
            raise G4SError(rc, self.lib.g4s_last_error(None).decode())
        self.h = h
        self.max_rows, self.max_vocab = max_rows, max_vocab

    def close(self):
        if getattr(self, "h", None):
            self.lib.g4s_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def last_error(self) -> str:
        return self.lib.g4s_last_error(self.h).decode()

    @property
    def stream(self) -> int:
        return self.lib.g4s_stream(self.h) or 0

    def _check(self, rc):
        if rc != OK:
            raise G4SError(rc, self.last_error())

    def sample(self, logits_ptr: int, dtype: int, rows: int, vocab: int, row_stride: int, params,
               softcap: float, u_ptr: int, out_ptr: int, stream: int | None = None,
               outputs: Outputs | None = None, check: bool = True) -> int:
        """g4s_sample_ex on device pointers.  params: one Params (broadcast) or a list."""
        if isinstance(params, Params):
            parr, pstride = (Params * 1)(params), 0
        else:
            parr, pstride = params_array(params), 1
        rc = self.lib.g4s_sample_ex(self.h, c_void_p(logits_ptr), dtype, rows, vocab, row_stride,
                                    parr, pstride, softcap, c_void_p(u_ptr), c_void_p(out_ptr),
                                    ctypes.byref(outputs) if outputs is not None else None,
                                    c_void_p(stream) if stream else None)
        if check:
            self._check(rc)
        return rc

    @staticmethod
    def _params(params, rows):
        if isinstance(params, Params):
            return (Params * 1)(params), 0
        return params_array(params), 1

    def shard_lists(self, logits_ptr: int, dtype: int, rows: int, slice_vocab: int, row_stride: int,
                    id_offset: int, vocab_total: int, params, softcap: float, lists_ptr: int, counts_ptr: int,
                    stream: int | None = None, check: bool = True) -> int:
        parr, pstride = self._params(params, rows)
        rc = self.lib.g4s_shard_lists(self.h, c_void_p(logits_ptr), dtype, rows, slice_vocab, row_stride, id_offset,
                                      vocab_total, parr, pstride, softcap, c_void_p(lists_ptr),
                                      c_void_p(counts_ptr), c_void_p(stream) if stream else None)
        if check:
            self._check(rc)
        return rc

    def shard_resolve(self, logits_ptr: int, dtype: int, rows: int, slice_vocab: int, row_stride: int,
                      id_offset: int, rank: int, params, softcap: float, u_ptr: int, out_ptr: int,
                      outputs: Outputs | None = None, stream: int | None = None, check: bool = True) -> int:
        parr, pstride = self._params(params, rows)
        rc = self.lib.g4s_shard_resolve(self.h, c_void_p(logits_ptr), dtype, rows, slice_vocab, row_stride,
                                        id_offset, rank, parr, pstride, softcap, c_void_p(u_ptr), c_void_p(out_ptr),
                                        ctypes.byref(outputs) if outputs is not None else None,
                                        c_void_p(stream) if stream else None)
        if check:
            self._check(rc)
        return rc

    def shard_merge(self, lists_ptr: int, counts_ptr: int, world: int, rows: int, vocab_total: int, params,
                    softcap: float, u_ptr: int, out_ptr: int, outputs: Outputs | None = None,
                    stream: int | None = None, check: bool = True) -> int:
        parr, pstride = self._params(params, rows)
        rc = self.lib.g4s_shard_merge(self.h, c_void_p(lists_ptr), c_void_p(counts_ptr), world, rows, vocab_total,
                                      parr, pstride, softcap, c_void_p(u_ptr), c_void_p(out_ptr),
                                      ctypes.byref(outputs) if outputs is not None else None,
                                      c_void_p(stream) if stream else None)
        if check:
            self._check(rc)
        return rc

    def shard_init(self, world: int, rank: int, vocab_total: int, uid: bytes, check: bool = True) -> int:
        buf = ctypes.create_string_buffer(bytes(uid), SHARD_UID_BYTES)
        rc = self.lib.g4s_shard_init(self.h, world, rank, vocab_total, buf)
        if check:
            self._check(rc)
        return rc

    def shard_set_timeout(self, ms: int) -> None:
        """Host deadline (ms) of the rendezvous and of shard_wait; 0 restores the default."""
        self._check(self.lib.g4s_shard_set_timeout(self.h, ms))

    def shard_wait(self, stream: int | None = None, timeout_ms: int = 0, check: bool = True) -> int:
        """Waits for the queued sharded work; aborts the communicator when a peer
        stalls past the deadline (ERR_TIMEOUT) or fails (ERR_NCCL)."""
        rc = self.lib.g4s_shard_wait(self.h, c_void_p(stream) if stream else None, timeout_ms)
        if check:
            self._check(rc)
        return rc

    def shard_abort(self) -> None:
        self._check(self.lib.g4s_shard_abort(self.h))

    def shard_sample(self, logits_ptr: int, dtype: int, rows: int, row_stride: int, params, softcap: float,
                     u_ptr: int, out_ptr: int, outputs: Outputs | None = None, stream: int | None = None,
                     check: bool = True) -> int:
        parr, pstride = self._params(params, rows)
        rc = self.lib.g4s_shard_sample(self.h, c_void_p(logits_ptr), dtype, rows, row_stride, parr, pstride,
                                       softcap, c_void_p(u_ptr), c_void_p(out_ptr),
                                       ctypes.byref(outputs) if outputs is not None else None,
                                       c_void_p(stream) if stream else None)
        if check:
            self._check(rc)
        return rc

    def lmhead_sample(self, hidden_ptr: int, rows: int, hidden: int, nib_ptr: int, scales_ptr: int, vocab: int,
                      params, softcap: float, u_ptr: int, out_ptr: int, outputs: Outputs | None = None,
                      logits_ptr: int = 0, stream: int | None = None, check: bool = True, norm_ptr: int = 0,
                      norm_eps: float = 1e-6) -> int:
        """g4s_lmhead_sample: [final RMSNorm,] logits = hidden x W^T (Q4_0, repacked), sampling."""
        parr, pstride = self._params(params, rows)
        rc = self.lib.g4s_lmhead_sample(self.h, c_void_p(hidden_ptr), rows, hidden,
                                        c_void_p(norm_ptr) if norm_ptr else None, norm_eps, c_void_p(nib_ptr),
                                        c_void_p(scales_ptr), vocab, parr, pstride, softcap, c_void_p(u_ptr),
                                        c_void_p(out_ptr), ctypes.byref(outputs) if outputs is not None else None,
                                        c_void_p(logits_ptr) if logits_ptr else None,
                                        c_void_p(stream) if stream else None)
        if check:
            self._check(rc)
        return rc

    def sample_host(self, logits, dtype: int, params, softcap: float, u, tokens_out=None):
        """g4s_sample_host on numpy arrays (logits [rows, row_stride] f32 or uint16 bf16 bits)."""
        import numpy as np

        rows, stride = logits.shape
        vocab = stride
        if isinstance(params, Params):
            parr, pstride = (Params * 1)(params), 0
        else:
            parr, pstride = params_array(params), 1
        out = tokens_out if tokens_out is not None else np.empty(rows, dtype=np.int32)
        u = np.ascontiguousarray(u, dtype=np.float64)
        rc = self.lib.g4s_sample_host(self.h, c_void_p(logits.ctypes.data), dtype, rows, vocab, stride,
                                      parr, pstride, softcap, c_void_p(u.ctypes.data),
                                      c_void_p(out.ctypes.data))
        self._check(rc)
        return out


class Vpk:
    """A VPK weight archive opened through g4s_vpk_open (TWeightStore)."""

    def __init__(self, path: str, manifest: str | None = None, weights: str | None = None):
        self.lib = load()
        h = c_void_p()
        enc = lambda x: x.encode() if x is not None else None
        rc = self.lib.g4s_vpk_open(path.encode(), enc(manifest), enc(weights), ctypes.byref(h))
        if rc != OK:
            raise G4SError(rc, self.lib.g4s_last_error(None).decode())
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            self.lib.g4s_vpk_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __len__(self):
        return self.lib.g4s_vpk_tensor_count(self.h)

    def find(self, name: str) -> TensorInfo:
        ti = TensorInfo()
        rc = self.lib.g4s_vpk_find(self.h, name.encode(), ctypes.byref(ti))
        if rc != OK:
            raise G4SError(rc, self.lib.g4s_last_error(None).decode())
        return ti

    def tensor(self, name: str):
        """The tensor's bytes (a read-only view of the mapping, copied to numpy)."""
        import numpy as np

        ti = self.find(name)
        ptr = self.lib.g4s_vpk_data(self.h, ctypes.byref(ti))
        return np.ctypeslib.as_array((ctypes.c_uint8 * ti.size).from_address(ptr)).copy(), ti

    def verify(self, entry: str) -> int:
        return self.lib.g4s_vpk_verify(self.h, entry.encode())

    def load_lmhead(self, device: int, nib_ptr: int, scales_ptr: int, max_vocab: int, stream: int | None = None):
        v, hdim = c_int32(), c_int32()
        rc = self.lib.g4s_vpk_load_lmhead(self.h, device, c_void_p(nib_ptr), c_void_p(scales_ptr), max_vocab,
                                          ctypes.byref(v), ctypes.byref(hdim), c_void_p(stream) if stream else None)
        if rc != OK:
            raise G4SError(rc, self.lib.g4s_last_error(None).decode())
        return v.value, hdim.value

