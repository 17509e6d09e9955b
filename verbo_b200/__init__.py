"""verbo_b200 - B200 (sm_100a) drop-in for verbo's token sampler.

Python face of the C ABI in include/verbo_cuda.h, in the style of the
reference's ctypes bindings (python/verbo/__init__.py): one shared library,
``ctypes`` signatures, ``VerboCudaError`` carrying verbo_cuda_last_error().

The compute runs only in the CUDA library ``_lib/libverbo_cuda.so``; there is
no CPU fallback.  Importing this module does not need a GPU; calling a
batched entry point needs device tensors (torch is used here only to hold
device memory and streams).

Entry points
------------
``Sampling``        the option set of verbo::Sampling (include/verbo/verbo.hpp:56-64)
``Sampler``         the verbo::Sampler object (pick / accept / reset / cfg)
``sample``          Sampler::pick over a batch of device-resident rows
``shard_topk``      vocab-sharded step 1: a shard's k best (value, global id)
``merge_sample``    vocab-sharded step 2: merge shard candidates and draw
``seed_states``     per-row xoroshiro128+ states, seeded like Sampler::reset
``Batch``           B generation streams with device-side RNG states and windows
``Tail``            the logits producer tail: final RMSNorm + LM head on the device
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from pathlib import Path
from typing import Optional, Sequence

__all__ = ["Sampling", "Sampler", "VerboCudaError", "load_library", "sample", "sample_noalloc", "full_vocab_fallbacks", "shard_topk", "merge_sample",
           "seed_states", "check", "version", "ROW_STATS_FIELDS", "Batch", "Server", "Tail", "Comm"]
__version__ = "0.1.0"

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "_lib" / "libverbo_cuda.so"


class VerboCudaError(RuntimeError):
    pass


class _Sampling(ctypes.Structure):
    _fields_ = [
        ("temp", ctypes.c_float),
        ("top_k", ctypes.c_int),
        ("top_p", ctypes.c_float),
        ("min_p", ctypes.c_float),
        ("repeat", ctypes.c_float),
        ("repeat_last", ctypes.c_int),
        ("seed", ctypes.c_ulonglong),
    ]


class _RowStats(ctypes.Structure):
    _fields_ = [
        ("sum", ctypes.c_double),
        ("tot", ctypes.c_double),
        ("u", ctypes.c_double),
        ("draw_margin", ctypes.c_double),
        ("cut_margin", ctypes.c_double),
        ("k", ctypes.c_int),
        ("keep", ctypes.c_int),
        ("id", ctypes.c_int),
        ("greedy", ctypes.c_int),
    ]


ROW_STATS_FIELDS = [f for f, _ in _RowStats._fields_]
ROW_STATS_BYTES = ctypes.sizeof(_RowStats)


@dataclass
class Sampling:
    """verbo::Sampling with the reference defaults (include/verbo/verbo.hpp:56-64).

    Option names follow the CLI flags --temp/--top-k/--top-p/--min-p/--repeat/
    --seed (cli/common.hpp:72-77); ``repeat_last`` is the penalty window."""

    temp: float = 0.7
    top_k: int = 40
    top_p: float = 0.9
    min_p: float = 0.0
    repeat: float = 1.0
    repeat_last: int = 64
    seed: int = 0

    def _c(self) -> _Sampling:
        return _Sampling(self.temp, self.top_k, self.top_p, self.min_p, self.repeat, self.repeat_last, self.seed)


_lib = None
_P = ctypes.c_void_p


def load_library():
    """Loads libverbo_cuda.so (override with VERBO_CUDA_LIB).  Raises if it is
    missing: there is no fallback implementation."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("VERBO_CUDA_LIB", LIB_PATH))
    if not path.is_file():
        raise VerboCudaError(f"{path} not found: build it with `python -m verbo_b200.build`")
    lib = ctypes.CDLL(str(path))
    sig = {
        "verbo_cuda_last_error": (ctypes.c_char_p, []),
        "verbo_cuda_version": (ctypes.c_char_p, []),
        "verbo_cuda_default_sampling": (_Sampling, []),
        "verbo_cuda_rng_seed": (ctypes.c_int, [ctypes.c_ulonglong, _P]),
        "verbo_cuda_rng_unit": (ctypes.c_double, [_P]),
        "verbo_cuda_sample": (ctypes.c_int, [_P, ctypes.c_int, ctypes.c_int, ctypes.c_longlong, _P, _P,
                                             ctypes.POINTER(_Sampling), _P, _P, _P, _P]),
        "verbo_cuda_sample_noalloc": (ctypes.c_int, [_P, ctypes.c_int, ctypes.c_int, ctypes.c_longlong, _P, _P,
                                                     ctypes.POINTER(_Sampling), _P, _P, _P, _P]),
        "verbo_cuda_shard_topk": (ctypes.c_int, [_P, ctypes.c_int, ctypes.c_int, ctypes.c_longlong, ctypes.c_int,
                                                 ctypes.c_int, _P, _P, ctypes.POINTER(_Sampling), ctypes.c_int,
                                                 _P, _P, _P]),
        "verbo_cuda_merge_sample": (ctypes.c_int, [_P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                   ctypes.POINTER(_Sampling), _P, _P, _P, _P]),
        "verbo_cuda_check": (ctypes.c_int, [_P]),
        "verbo_cuda_full_vocab_fallbacks": (ctypes.c_int, [_P]),
        "verbo_cuda_comm_unique_id": (ctypes.c_int, [_P]),
        "verbo_cuda_comm_new": (_P, [_P, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
        "verbo_cuda_comm_free": (None, [_P]),
        "verbo_cuda_comm_wait": (ctypes.c_int, [_P, _P, ctypes.c_int]),
        "verbo_cuda_comm_mark_next": (ctypes.c_int, [_P, _P, _P]),
        "verbo_cuda_batch_decode": (ctypes.c_int, [_P, _P, _P, ctypes.c_longlong, _P, _P, _P]),
        "verbo_cuda_server_new": (_P, [ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, ctypes.c_int, ctypes.c_int]),
        "verbo_cuda_server_free": (None, [_P]),
        "verbo_cuda_server_submit": (ctypes.c_longlong, [_P, _P, ctypes.c_int, _P, ctypes.c_int]),
        "verbo_cuda_server_prepare": (ctypes.c_int, [_P, _P, _P]),
        "verbo_cuda_server_step": (ctypes.c_int, [_P, _P, ctypes.c_longlong, _P]),
        "verbo_cuda_server_result": (ctypes.c_int, [_P, ctypes.c_longlong, _P, ctypes.c_int, _P, _P, ctypes.c_int]),
        "verbo_cuda_sharded_sample": (ctypes.c_int, [_P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_longlong,
                                                     ctypes.c_int, ctypes.c_int, _P, _P, ctypes.POINTER(_Sampling),
                                                     ctypes.c_int, _P, _P, _P, _P]),
        "verbo_cuda_sampler_new": (_P, [ctypes.POINTER(_Sampling), ctypes.c_int]),
        "verbo_cuda_sampler_free": (None, [_P]),
        "verbo_cuda_sampler_pick": (ctypes.c_int, [_P, _P, ctypes.c_int]),
        "verbo_cuda_sampler_accept": (ctypes.c_int, [_P, ctypes.c_int]),
        "verbo_cuda_sampler_reset": (ctypes.c_int, [_P]),
        "verbo_cuda_sampler_cfg": (ctypes.c_int, [_P, ctypes.POINTER(_Sampling)]),
        "verbo_cuda_batch_new": (_P, [ctypes.POINTER(_Sampling), ctypes.c_int, ctypes.c_int]),
        "verbo_cuda_batch_free": (None, [_P]),
        "verbo_cuda_batch_reset": (ctypes.c_int, [_P, ctypes.c_int, ctypes.c_ulonglong, _P]),
        "verbo_cuda_batch_accept": (ctypes.c_int, [_P, ctypes.c_int, _P, ctypes.c_int, _P]),
        "verbo_cuda_batch_step": (ctypes.c_int, [_P, _P, ctypes.c_int, ctypes.c_longlong, _P, _P, _P]),
        "verbo_cuda_tail_new": (_P, [ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, _P, _P, ctypes.c_float,
                                     ctypes.c_int]),
        "verbo_cuda_tail_free": (None, [_P]),
        "verbo_cuda_tail_logits": (ctypes.c_int, [_P, _P, ctypes.c_int, ctypes.c_longlong, _P, ctypes.c_longlong, _P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def _err() -> VerboCudaError:
    return VerboCudaError(load_library().verbo_cuda_last_error().decode())


def _ok(rc: int) -> int:
    if rc < 0:
        raise _err()
    return rc


def version() -> str:
    return load_library().verbo_cuda_version().decode()


def _dptr(t, rows_strided: bool = False) -> Optional[int]:
    """Device address of a CUDA tensor.  With rows_strided, a 2-D view whose
    rows are contiguous but spaced by stride(0) (e.g. a column shard) is
    accepted; the caller passes stride(0) as the leading dimension."""
    if t is None:
        return None
    if not t.is_cuda:
        raise VerboCudaError("batched entry points take CUDA tensors")
    if rows_strided:
        if t.dim() != 2 or (t.shape[1] > 1 and t.stride(1) != 1):
            raise VerboCudaError("rows must be contiguous (stride(1) == 1)")
    elif not t.is_contiguous():
        raise VerboCudaError("tensors must be contiguous")
    return t.data_ptr()


def _stream(stream) -> Optional[int]:
    if stream is None:
        import torch

        return torch.cuda.current_stream().cuda_stream
    return getattr(stream, "cuda_stream", stream)


def seed_states(seeds: Sequence[int]):
    """Host list of per-row [s0, s1] states seeded like Sampler::reset
    (src/sampler.cpp:26-31; seed 0 takes the clock)."""
    lib = load_library()
    out = []
    st = (ctypes.c_ulonglong * 2)()
    for s in seeds:
        _ok(lib.verbo_cuda_rng_seed(int(s), st))
        out.append([st[0], st[1]])
    return out


def sample(logits, opts: Sampling, rng=None, hist=None, hist_off=None, out=None, stats=None, vocab=None,
           stream=None):
    """Sampler::pick for each row of `logits` (CUDA float32 [rows, ld]).

    rng: CUDA int64/uint64 tensor [rows, 2] advanced in place (required when
    temp > 0).  hist/hist_off: CUDA int32 ids and int64 CSR offsets [rows+1].
    stats: optional CUDA uint8 tensor of rows * ROW_STATS_BYTES.  Returns the
    int32 id tensor (asynchronous on `stream`)."""
    import torch

    rows, cols = logits.shape
    vocab = cols if vocab is None else vocab
    if logits.dtype != torch.float32:
        raise VerboCudaError("logits must be float32")
    if out is None:
        out = torch.empty(rows, dtype=torch.int32, device=logits.device)
    o = opts._c()
    rc = load_library().verbo_cuda_sample(_dptr(logits, True), rows, vocab, logits.stride(0), _dptr(hist),
                                          _dptr(hist_off),
                                          ctypes.byref(o), _dptr(rng), _dptr(out), _dptr(stats), _stream(stream))
    _ok(rc)
    return out


def sample_noalloc(logits, opts: Sampling, rng=None, hist=None, hist_off=None, out=None, stats=None, vocab=None,
                   stream=None):
    """``sample`` through verbo_cuda_sample_noalloc: for callers that cannot let
    the library allocate device memory (greedy and 0 < top_k <= 256 only; a
    fixed 8 MiB scratch inside the library, shared by all calls)."""
    import torch

    rows, cols = logits.shape
    vocab = cols if vocab is None else vocab
    if logits.dtype != torch.float32:
        raise VerboCudaError("logits must be float32")
    if out is None:
        out = torch.empty(rows, dtype=torch.int32, device=logits.device)
    o = opts._c()
    rc = load_library().verbo_cuda_sample_noalloc(_dptr(logits, True), rows, vocab, logits.stride(0), _dptr(hist),
                                                  _dptr(hist_off), ctypes.byref(o), _dptr(rng), _dptr(out),
                                                  _dptr(stats), _stream(stream))
    _ok(rc)
    return out


def shard_topk(shard, col_offset: int, vocab: int, opts: Sampling, k: int, hist=None, hist_off=None,
               cand_val=None, cand_id=None, stream=None):
    """A shard's k best (value, global id) per row: shard is CUDA float32
    [rows, ld] holding global columns [col_offset, col_offset + cols)."""
    import torch

    rows, cols = shard.shape
    if cand_val is None:
        cand_val = torch.empty(rows, k, dtype=torch.float32, device=shard.device)
    if cand_id is None:
        cand_id = torch.empty(rows, k, dtype=torch.int32, device=shard.device)
    o = opts._c()
    _ok(load_library().verbo_cuda_shard_topk(_dptr(shard, True), rows, cols, shard.stride(0), col_offset, vocab,
                                             _dptr(hist), _dptr(hist_off), ctypes.byref(o), k, _dptr(cand_val),
                                             _dptr(cand_id), _stream(stream)))
    return cand_val, cand_id


def merge_sample(cand_val, cand_id, vocab: int, opts: Sampling, rng=None, out=None, stats=None, stream=None):
    """Merges candidates laid out [nshards, rows, k] and finishes the pick."""
    import torch

    nshards, rows, k = cand_val.shape
    if out is None:
        out = torch.empty(rows, dtype=torch.int32, device=cand_val.device)
    o = opts._c()
    _ok(load_library().verbo_cuda_merge_sample(_dptr(cand_val), _dptr(cand_id), rows, nshards, k, vocab,
                                               ctypes.byref(o), _dptr(rng), _dptr(out), _dptr(stats),
                                               _stream(stream)))
    return out


def check(stream=None) -> None:
    """Synchronises the stream and raises if a kernel recorded a failure."""
    _ok(load_library().verbo_cuda_check(_stream(stream)))


def full_vocab_fallbacks(stream=None) -> int:
    """Rows of the last full-vocabulary call on the stream that the staged
    cluster kernel settled instead of the streaming one (synchronises)."""
    n = load_library().verbo_cuda_full_vocab_fallbacks(_stream(stream))
    _ok(0 if n >= 0 else -1)
    return n


class Sampler:
    """verbo::Sampler (include/verbo/verbo.hpp:116-132) on a CUDA device.

    ``pick`` takes a host buffer (numpy float32 or any object exposing the
    buffer protocol / a ctypes address) or a CUDA tensor."""

    def __init__(self, cfg: Optional[Sampling] = None, device: int = 0):
        self._lib = load_library()
        self._cfg = cfg if cfg is not None else Sampling()
        c = self._cfg._c()
        h = self._lib.verbo_cuda_sampler_new(ctypes.byref(c), device)
        if not h:
            raise _err()
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            self._lib.verbo_cuda_sampler_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def pick(self, logits, n: Optional[int] = None) -> int:
        if hasattr(logits, "is_cuda") and logits.is_cuda:
            ptr, size = logits.data_ptr(), logits.numel()
        else:
            import numpy as np

            arr = np.ascontiguousarray(logits, dtype=np.float32)
            self._keep = arr
            ptr, size = arr.ctypes.data, arr.size
        return _ok(self._lib.verbo_cuda_sampler_pick(self._h, ptr, size if n is None else n))

    def accept(self, tok: int) -> None:
        _ok(self._lib.verbo_cuda_sampler_accept(self._h, int(tok)))

    def reset(self) -> None:
        _ok(self._lib.verbo_cuda_sampler_reset(self._h))

    def cfg(self) -> Sampling:
        c = _Sampling()
        _ok(self._lib.verbo_cuda_sampler_cfg(self._h, ctypes.byref(c)))
        return Sampling(c.temp, c.top_k, c.top_p, c.min_p, c.repeat, c.repeat_last, c.seed)


class Batch:
    """B generation streams sampled together, their RNG states and penalty
    windows kept on the device (the batched form of verbo::generate's loop,
    src/sampler.cpp:111-181).  ``step`` takes CUDA float32 rows [B, ld]."""

    def __init__(self, cfg: Optional[Sampling], streams: int, device: int = 0):
        self._lib = load_library()
        self._cfg = cfg if cfg is not None else Sampling()
        c = self._cfg._c()
        h = self._lib.verbo_cuda_batch_new(ctypes.byref(c), int(streams), device)
        if not h:
            raise _err()
        self._h = h
        self.streams = int(streams)

    def close(self):
        if getattr(self, "_h", None):
            self._lib.verbo_cuda_batch_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self, stream: int, seed: int, cuda_stream=None) -> None:
        _ok(self._lib.verbo_cuda_batch_reset(self._h, int(stream), int(seed), _stream(cuda_stream)))

    def accept(self, stream: int, ids, cuda_stream=None) -> None:
        import numpy as np

        arr = np.ascontiguousarray(ids, dtype=np.int32)
        _ok(self._lib.verbo_cuda_batch_accept(self._h, int(stream), arr.ctypes.data if arr.size else None, arr.size,
                                              _stream(cuda_stream)))

    def step(self, logits, out=None, stats=None, vocab=None, cuda_stream=None):
        import torch

        rows, cols = logits.shape
        if rows != self.streams:
            raise VerboCudaError("logits must have one row per stream")
        if logits.dtype != torch.float32:
            raise VerboCudaError("logits must be float32")
        if out is None:
            out = torch.empty(rows, dtype=torch.int32, device=logits.device)
        _ok(self._lib.verbo_cuda_batch_step(self._h, _dptr(logits, True), cols if vocab is None else vocab,
                                            logits.stride(0), _dptr(out), _dptr(stats), _stream(cuda_stream)))
        return out

    def decode(self, tail: "Tail", hidden, out=None, stats=None, cuda_stream=None):
        """One decode step of the B generations (verbo_cuda_batch_decode):
        `hidden` [B, dim] float32 rows of final hidden state (a numpy array,
        a CPU tensor or a CUDA tensor) -> the tail's logits on the device ->
        pick + accept.  Returns the ids: a numpy int32 array when `hidden` is
        on the host (the call then waits for them), else a CUDA tensor; `out`
        may be either kind."""
        import numpy as np
        import torch

        if isinstance(hidden, np.ndarray):
            hidden = torch.from_numpy(np.ascontiguousarray(hidden, dtype=np.float32))
        if hidden.dim() != 2 or hidden.shape[0] != self.streams:
            raise VerboCudaError("hidden must have one row per stream")
        if hidden.dtype != torch.float32 or (hidden.shape[1] > 1 and hidden.stride(1) != 1):
            raise VerboCudaError("hidden rows must be contiguous float32")
        if out is None:
            out = (torch.empty(self.streams, dtype=torch.int32, device=hidden.device) if hidden.is_cuda
                   else np.empty(self.streams, dtype=np.int32))
        out_ptr = out.ctypes.data if isinstance(out, np.ndarray) else out.data_ptr()
        if isinstance(out, np.ndarray) and (out.dtype != np.int32 or out.size != self.streams):
            raise VerboCudaError("out must hold one int32 per stream")
        st_ptr = None if stats is None else (stats.ctypes.data if isinstance(stats, np.ndarray) else stats.data_ptr())
        _ok(self._lib.verbo_cuda_batch_decode(self._h, tail._h, hidden.data_ptr(), hidden.stride(0), out_ptr, st_ptr,
                                              _stream(cuda_stream)))
        return out



class Server:
    """Request batching with per-request options (verbo_cuda_server_*): up to
    `slots` requests in flight, each with its own Sampling (seed included) and
    sampler state on the device.  Per step: ``prepare()`` returns the request
    id of each row (-1 idle) and the active row count A; the caller writes each
    active request's next logits row into row r of a [>= A, vocab] float32
    array (CUDA tensor or numpy); ``step(logits)`` samples and accepts; a stop
    id or max_tokens finishes a request; ``result(id)`` reads it."""

    def __init__(self, slots: int, vocab: int, max_window: int = 256, stop_ids=(), device: int = 0):
        import numpy as np

        self._lib = load_library()
        st = np.ascontiguousarray(list(stop_ids), dtype=np.int32)
        h = self._lib.verbo_cuda_server_new(int(slots), int(vocab), int(max_window),
                                            st.ctypes.data if st.size else None, int(st.size), int(device))
        if not h:
            raise _err()
        self._h, self.slots, self.vocab = h, int(slots), int(vocab)
        self._rows = np.full(self.slots, -1, dtype=np.int64)

    def submit(self, prompt, opts: Sampling, max_tokens: int) -> int:
        import numpy as np

        p = np.ascontiguousarray(prompt, dtype=np.int32)
        c = opts._c()
        rid = self._lib.verbo_cuda_server_submit(self._h, p.ctypes.data if p.size else None, int(p.size),
                                                 ctypes.byref(c), int(max_tokens))
        if rid < 0:
            raise _err()
        return int(rid)

    def prepare(self, cuda_stream=None):
        """(row -> request id array, active rows A)."""
        n = self._lib.verbo_cuda_server_prepare(self._h, self._rows.ctypes.data, _stream(cuda_stream))
        if n < 0:
            raise _err()
        return self._rows.copy(), int(n)

    def step(self, logits, cuda_stream=None) -> int:
        import numpy as np

        if isinstance(logits, np.ndarray):
            arr = np.ascontiguousarray(logits, dtype=np.float32)
            ptr, ld = arr.ctypes.data, arr.shape[1]
        else:
            if logits.dtype.itemsize != 4 or (logits.shape[1] > 1 and logits.stride(1) != 1):
                raise VerboCudaError("logits rows must be contiguous float32")
            ptr, ld = logits.data_ptr(), logits.stride(0)
        n = self._lib.verbo_cuda_server_step(self._h, ptr, int(ld), _stream(cuda_stream))
        if n < 0:
            raise _err()
        return int(n)

    def result(self, rid: int, release: bool = False):
        """(finished, ids, stopped)."""
        import numpy as np

        n = ctypes.c_int(0)
        stopped = ctypes.c_int(0)
        rc = self._lib.verbo_cuda_server_result(self._h, int(rid), None, 0, ctypes.byref(n), ctypes.byref(stopped), 0)
        if rc < 0:
            raise _err()
        ids = np.zeros(max(n.value, 1), dtype=np.int32)
        rc = self._lib.verbo_cuda_server_result(self._h, int(rid), ids.ctypes.data, int(ids.size), ctypes.byref(n),
                                                ctypes.byref(stopped), 1 if release else 0)
        if rc < 0:
            raise _err()
        return bool(rc), ids[:n.value].tolist(), bool(stopped.value)

    def close(self):
        if getattr(self, "_h", None):
            self._lib.verbo_cuda_server_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


UNIQUE_ID_BYTES = 128


class Comm:
    """The library's communicator for vocab-sharded sampling (one per rank and
    GPU): NCCL, loaded by the library at run time.  Rank 0 makes an id with
    ``Comm.unique_id()``; every rank passes the same 128 bytes to the
    constructor (a collective call).  ``sample`` is verbo_cuda_sharded_sample:
    this rank's column shard -> its k best -> one all-gather -> the merge, on
    the given stream, with the same ids on every rank."""

    @staticmethod
    def unique_id() -> bytes:
        buf = (ctypes.c_ubyte * UNIQUE_ID_BYTES)()
        _ok(load_library().verbo_cuda_comm_unique_id(ctypes.addressof(buf)))
        return bytes(buf)

    def __init__(self, uid: bytes, nranks: int, rank: int, device: int = 0):
        if len(uid) != UNIQUE_ID_BYTES:
            raise VerboCudaError(f"the unique id has {UNIQUE_ID_BYTES} bytes")
        self._lib = load_library()
        buf = (ctypes.c_ubyte * UNIQUE_ID_BYTES).from_buffer_copy(uid)
        h = self._lib.verbo_cuda_comm_new(ctypes.addressof(buf), int(nranks), int(rank), int(device))
        if not h:
            raise _err()
        self._h, self.nranks, self.rank, self.device = h, int(nranks), int(rank), int(device)

    def sample(self, shard, col_offset: int, vocab: int, opts: Sampling, k: int, rng=None, hist=None, hist_off=None,
               out=None, stats=None, stream=None):
        import torch

        rows, cols = shard.shape
        if shard.dtype != torch.float32:
            raise VerboCudaError("logits must be float32")
        if out is None:
            out = torch.empty(rows, dtype=torch.int32, device=shard.device)
        o = opts._c()
        _ok(self._lib.verbo_cuda_sharded_sample(self._h, _dptr(shard, True), rows, cols, shard.stride(0),
                                                int(col_offset), int(vocab), _dptr(hist), _dptr(hist_off),
                                                ctypes.byref(o), int(k), _dptr(rng), _dptr(out), _dptr(stats),
                                                _stream(stream)))
        return out

    def wait(self, stream=None, timeout_ms: int = 10000) -> None:
        """Bounded wait for the stream; on timeout or a collective error the
        communicator is aborted and VerboCudaError raised."""
        _ok(self._lib.verbo_cuda_comm_wait(self._h, _stream(stream), int(timeout_ms)))

    def mark_next(self, after_shard=None, after_gather=None) -> None:
        """The next ``sample`` records these torch.cuda.Events (timing-enabled,
        recorded at least once so that they exist) on its stream after the
        shard's top-k kernel and after the all-gather."""
        def handle(e):
            if e is None:
                return None
            if not e.cuda_event:
                raise VerboCudaError("record the event once before passing it")
            return ctypes.c_void_p(e.cuda_event)
        _ok(self._lib.verbo_cuda_comm_mark_next(self._h, handle(after_shard), handle(after_gather)))

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.verbo_cuda_comm_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


TAIL_DTYPES = {"f32": 0, "q8": 1, "q4": 2}  # verbo::DType (include/verbo/verbo.hpp:13)


class Tail:
    """The logits producer tail of Session::Impl::batch (src/session.cpp:163-169)
    on the device: final RMSNorm (``norm``, ``eps``) then the LM head.

    ``q``/``s`` are host numpy arrays in verbo::Tensor layout
    (src/kernels.hpp:13-23): f32 (vocab, dim) float32; q8 (vocab, dim) int8;
    q4 (vocab, dim/2) uint8; s (vocab, dim/32) fp16 scales (float16 or their
    uint16 bits).  ``logits`` maps CUDA float32 hidden rows [n, >= dim] to
    logits rows [n, vocab] (or into ``out``, rows of stride(0) >= vocab)."""

    def __init__(self, dtype, q, s, norm, eps: float, device: int = 0):
        import numpy as np

        self._lib = load_library()
        dt = TAIL_DTYPES[dtype] if isinstance(dtype, str) else int(dtype)
        q = np.ascontiguousarray(q)
        norm = np.ascontiguousarray(norm, dtype=np.float32)
        vocab, dim = q.shape[0], norm.shape[0]
        sp = None
        if dt != 0:
            s = np.ascontiguousarray(s)
            if s.dtype == np.float16:
                s = s.view(np.uint16)
            s = np.ascontiguousarray(s, dtype=np.uint16)
            sp = s.ctypes.data
        h = self._lib.verbo_cuda_tail_new(dt, int(vocab), int(dim), q.ctypes.data, sp, norm.ctypes.data,
                                          float(eps), int(device))
        if not h:
            raise _err()
        self._h = h
        self.dtype, self.vocab, self.dim, self.device = dt, int(vocab), int(dim), int(device)

    def close(self):
        if getattr(self, "_h", None):
            self._lib.verbo_cuda_tail_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def logits(self, x, out=None, stream=None):
        import torch

        n, cols = x.shape
        if x.dtype != torch.float32:
            raise VerboCudaError("hidden rows must be float32")
        if out is None:
            out = torch.empty(n, self.vocab, dtype=torch.float32, device=x.device)
        if out.dtype != torch.float32 or out.shape[0] != n:
            raise VerboCudaError("out must be float32 with one row per hidden row")
        _ok(self._lib.verbo_cuda_tail_logits(self._h, _dptr(x, True), n, x.stride(0) if n else cols,
                                             _dptr(out, True), out.stride(0) if n else self.vocab,
                                             _stream(stream)))
        return out
