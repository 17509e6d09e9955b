"""ctypes access to the CPU checkers of the sampling path - TEST INFRASTRUCTURE.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU legs import this
module.  It wraps two libraries built by ``oracle/Makefile``:

* ``_build/liboracle.so``   - the C restatement of verbo's Sampler
  (src/sampler.cpp:11-109), with per-row diagnostics;
* ``_ref/libverbo_ref.so``  - the reference's own Sampler compiled from its
  sources, driven through ``ref_harness.cpp``.  Optional: it exists only where
  the reference sources were available at build time.

All array arguments are numpy arrays on the host.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Optional

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "_build" / "liboracle.so"
REF_LIB = HERE / "_ref" / "libverbo_ref.so"
REF_TAIL_LIBS = {"avx2": HERE / "_ref" / "libverbo_ref_tail.so", "scalar": HERE / "_ref" / "libverbo_ref_tail_scalar.so"}


class OracleSampling(ctypes.Structure):
    """Field-for-field verbo::Sampling (include/verbo/verbo.hpp:56-64)."""

    _fields_ = [
        ("temp", ctypes.c_float),
        ("top_k", ctypes.c_int),
        ("top_p", ctypes.c_float),
        ("min_p", ctypes.c_float),
        ("repeat", ctypes.c_float),
        ("repeat_last", ctypes.c_int),
        ("seed", ctypes.c_ulonglong),
    ]


class RowStats(ctypes.Structure):
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


STATS_DTYPE = np.dtype(
    [("sum", "f8"), ("tot", "f8"), ("u", "f8"), ("draw_margin", "f8"), ("cut_margin", "f8"),
     ("k", "i4"), ("keep", "i4"), ("id", "i4"), ("greedy", "i4")]
)
assert STATS_DTYPE.itemsize == ctypes.sizeof(RowStats)


def sampling(temp=0.7, top_k=40, top_p=0.9, min_p=0.0, repeat=1.0, repeat_last=64, seed=0) -> OracleSampling:
    """Defaults are verbo::Sampling's (include/verbo/verbo.hpp:56-64)."""
    return OracleSampling(temp, top_k, top_p, min_p, repeat, repeat_last, seed)


_P = ctypes.c_void_p
_oracle = None
_ref = None


def _ptr(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(_P)


def oracle_lib():
    global _oracle
    if _oracle is None:
        if not ORACLE_LIB.is_file():
            raise RuntimeError(f"{ORACLE_LIB} missing: run `make -C oracle`")
        lib = ctypes.CDLL(str(ORACLE_LIB))
        lib.oracle_seed.argtypes = [ctypes.c_uint64, _P]
        lib.oracle_unit.argtypes = [_P]
        lib.oracle_unit.restype = ctypes.c_double
        lib.oracle_sample_rows.argtypes = [_P, ctypes.c_int, ctypes.c_int, ctypes.c_longlong, _P, _P, _P, _P, _P, _P]
        lib.oracle_shard_topk.argtypes = [_P, ctypes.c_int, ctypes.c_int, ctypes.c_longlong, ctypes.c_int,
                                          ctypes.c_int, _P, _P, _P, ctypes.c_int, _P, _P]
        lib.oracle_logits_tail.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, _P, _P, ctypes.c_float, _P,
                                           ctypes.c_int, ctypes.c_longlong, _P, ctypes.c_longlong, _P, _P]
        lib.oracle_merge_sample.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                            _P, _P, _P, _P]
        _oracle = lib
    return _oracle


def ref_available() -> bool:
    return REF_LIB.is_file()


def ref_lib():
    global _ref
    if _ref is None:
        if not REF_LIB.is_file():
            raise RuntimeError(f"{REF_LIB} missing: build it with `make -C oracle ref REF=<verbo checkout>`")
        lib = ctypes.CDLL(str(REF_LIB))
        lib.ref_sample_rows.argtypes = [_P, ctypes.c_int, ctypes.c_int, ctypes.c_longlong, _P, _P, _P, _P,
                                        ctypes.c_int, _P, ctypes.c_int]
        _ref = lib
    return _ref


def seed_states(seeds: np.ndarray) -> np.ndarray:
    """(rows,) u64 seeds -> (rows, 2) u64 xoroshiro128+ states (Sampler::reset)."""
    lib = oracle_lib()
    seeds = np.ascontiguousarray(seeds, dtype=np.uint64)
    out = np.zeros((seeds.shape[0], 2), dtype=np.uint64)
    for r, s in enumerate(seeds):
        lib.oracle_seed(ctypes.c_uint64(int(s)), out[r].ctypes.data_as(_P))
    return out


def _hist(hist, hist_off):
    if hist is None:
        return None, None
    return (np.ascontiguousarray(hist, dtype=np.int32), np.ascontiguousarray(hist_off, dtype=np.int64))


def sample_rows(logits: np.ndarray, opts: OracleSampling, rng: Optional[np.ndarray] = None, hist=None,
                hist_off=None, vocab: Optional[int] = None):
    """C restatement of Sampler::pick over rows.  `rng` (rows,2) u64 is advanced
    in place for non-greedy picks.  Returns (ids, stats)."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    rows, ld = logits.shape
    vocab = ld if vocab is None else vocab
    h, ho = _hist(hist, hist_off)
    if rng is None:
        rng = np.zeros((rows, 2), dtype=np.uint64)
    assert rng.dtype == np.uint64 and rng.flags.c_contiguous
    ids = np.zeros(rows, dtype=np.int32)
    stats = np.zeros(rows, dtype=STATS_DTYPE)
    oracle_lib().oracle_sample_rows(_ptr(logits), rows, vocab, ld, _ptr(h), _ptr(ho), ctypes.byref(opts),
                                    _ptr(rng), _ptr(ids), _ptr(stats))
    return ids, stats


def shard_topk(shard: np.ndarray, col_offset: int, vocab: int, opts: OracleSampling, k: int, hist=None,
               hist_off=None):
    shard = np.ascontiguousarray(shard, dtype=np.float32)
    rows, cols = shard.shape
    h, ho = _hist(hist, hist_off)
    val = np.zeros((rows, k), dtype=np.float32)
    cid = np.zeros((rows, k), dtype=np.int32)
    oracle_lib().oracle_shard_topk(_ptr(shard), rows, cols, cols, col_offset, vocab, _ptr(h), _ptr(ho),
                                   ctypes.byref(opts), k, _ptr(val), _ptr(cid))
    return val, cid


def merge_sample(cand_val: np.ndarray, cand_id: np.ndarray, vocab: int, opts: OracleSampling,
                 rng: Optional[np.ndarray] = None):
    """cand_* shaped (nshards, rows, k)."""
    cand_val = np.ascontiguousarray(cand_val, dtype=np.float32)
    cand_id = np.ascontiguousarray(cand_id, dtype=np.int32)
    nshards, rows, k = cand_val.shape
    if rng is None:
        rng = np.zeros((rows, 2), dtype=np.uint64)
    ids = np.zeros(rows, dtype=np.int32)
    stats = np.zeros(rows, dtype=STATS_DTYPE)
    oracle_lib().oracle_merge_sample(_ptr(cand_val), _ptr(cand_id), rows, nshards, k, vocab,
                                     ctypes.byref(opts), _ptr(rng), _ptr(ids), _ptr(stats))
    return ids, stats


def ref_sample_rows(logits: np.ndarray, opts: OracleSampling, seeds: np.ndarray, hist=None, hist_off=None,
                    steps: int = 1, threads: int = 1, vocab: Optional[int] = None) -> np.ndarray:
    """The reference's own Sampler: row r seeded with seeds[r], history fed
    through accept(), then `steps` picks.  Returns (rows, steps) int32."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    rows, ld = logits.shape
    vocab = ld if vocab is None else vocab
    h, ho = _hist(hist, hist_off)
    seeds = np.ascontiguousarray(seeds, dtype=np.uint64)
    out = np.zeros((rows, steps), dtype=np.int32)
    ref_lib().ref_sample_rows(_ptr(logits), rows, vocab, ld, _ptr(h), _ptr(ho), ctypes.byref(opts),
                              _ptr(seeds), steps, _ptr(out), threads)
    return out


_ref_tail = {}


def ref_tail_available(build: str = "scalar") -> bool:
    return REF_TAIL_LIBS[build].is_file()


def _ref_tail_lib(build: str):
    if build not in _ref_tail:
        path = REF_TAIL_LIBS[build]
        if not path.is_file():
            raise RuntimeError(f"{path} missing: build it with `make -C oracle ref REF=<verbo checkout>`")
        lib = ctypes.CDLL(str(path))
        lib.ref_logits_tail.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, _P, _P, ctypes.c_float, _P,
                                        ctypes.c_int, ctypes.c_longlong, _P, ctypes.c_longlong, _P, _P, ctypes.c_int]
        lib.ref_model_tail.argtypes = [ctypes.c_char_p, ctypes.c_int, _P, ctypes.c_int, ctypes.c_int, _P, _P, _P, _P,
                                       _P, _P, _P]
        lib.ref_decode.argtypes = [ctypes.c_char_p, ctypes.c_int, _P, ctypes.c_int, ctypes.POINTER(OracleSampling),
                                   ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, _P, _P]
        _ref_tail[build] = lib
    return _ref_tail[build]


DTYPES = {"f32": 0, "q8": 1, "q4": 2}


def _tail_args(dtype, q, s, norm, x):
    dt = DTYPES[dtype] if isinstance(dtype, str) else int(dtype)
    q = np.ascontiguousarray(q)
    norm = np.ascontiguousarray(norm, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    s = None if dt == 0 else np.ascontiguousarray(s, dtype=np.uint16)
    n, dim = x.shape
    vocab = q.shape[0]
    return dt, q, s, norm, x, n, dim, vocab


def logits_tail(dtype, q, s, norm, eps, x):
    """Oracle logits tail: (n, dim) hidden rows -> ((n, vocab) logits, xq, xs).

    `q`/`s` hold the head in verbo::Tensor layout (src/kernels.hpp:13-23):
    f32 (vocab, dim) floats; q8 (vocab, dim) int8; q4 (vocab, dim/2) uint8;
    s (vocab, dim/32) fp16 bits as uint16.  xq/xs are None for f32 heads."""
    dt, q, s, norm, x, n, dim, vocab = _tail_args(dtype, q, s, norm, x)
    out = np.zeros((n, vocab), dtype=np.float32)
    xq = np.zeros((n, dim), dtype=np.int8) if dt else None
    xs = np.zeros((n, dim // 32), dtype=np.float32) if dt else None
    rc = oracle_lib().oracle_logits_tail(dt, vocab, dim, _ptr(q), _ptr(s), _ptr(norm), eps, _ptr(x), n, dim,
                                         _ptr(out), vocab, _ptr(xq), _ptr(xs))
    if rc != 0:
        raise ValueError("oracle_logits_tail rejected its arguments")
    return out, xq, xs


def ref_logits_tail(dtype, q, s, norm, eps, x, build: str = "scalar", threads: int = 1):
    """The reference's own tail (rmsnorm, quant_act, matmul) from the `build`
    ("scalar" = the VERBO_SCALAR option, "avx2" = the default x86 build)."""
    dt, q, s, norm, x, n, dim, vocab = _tail_args(dtype, q, s, norm, x)
    out = np.zeros((n, vocab), dtype=np.float32)
    xq = np.zeros((n, dim), dtype=np.int8) if dt else None
    xs = np.zeros((n, dim // 32), dtype=np.float32) if dt else None
    rc = _ref_tail_lib(build).ref_logits_tail(dt, vocab, dim, _ptr(q), _ptr(s), _ptr(norm), eps, _ptr(x), n, dim,
                                              _ptr(out), vocab, _ptr(xq), _ptr(xs), threads)
    if rc != 0:
        raise ValueError("ref_logits_tail rejected its arguments")
    return out, xq, xs


def ref_model_tail(model_dir, dtype, toks, build: str = "scalar", threads: int = 1) -> dict:
    """Session::eval_all of the reference on a checkpoint directory, with the
    final hidden rows read from the session: returns x (n, dim), logits
    (n, vocab), the head (dtype name, q, s), norm and eps."""
    lib = _ref_tail_lib(build)
    dt = DTYPES[dtype] if isinstance(dtype, str) else int(dtype)
    toks = np.ascontiguousarray(toks, dtype=np.int32)
    meta = np.zeros(3, dtype=np.int32)
    eps = np.zeros(1, dtype=np.float32)
    path = str(model_dir).encode()
    if lib.ref_model_tail(path, dt, None, 0, threads, _ptr(meta), _ptr(eps), None, None, None, None, None) != 0:
        raise RuntimeError(f"the reference could not load {model_dir}")
    dim, vocab, hdt = (int(v) for v in meta)
    n = toks.size
    x = np.zeros((n, dim), dtype=np.float32)
    logits = np.zeros((n, vocab), dtype=np.float32)
    if hdt == 0:
        q = np.zeros((vocab, dim), dtype=np.float32)
    elif hdt == 1:
        q = np.zeros((vocab, dim), dtype=np.int8)
    else:
        q = np.zeros((vocab, dim // 2), dtype=np.uint8)
    sc = np.zeros((vocab, dim // 32), dtype=np.uint16)
    norm = np.zeros(dim, dtype=np.float32)
    if lib.ref_model_tail(path, dt, _ptr(toks), n, threads, _ptr(meta), _ptr(eps), _ptr(x), _ptr(logits), _ptr(q),
                          _ptr(sc), _ptr(norm)) != 0:
        raise RuntimeError(f"the reference's session failed on {model_dir}")
    name = {0: "f32", 1: "q8", 2: "q4"}[hdt]
    return {"x": x, "logits": logits, "dtype": name, "q": q, "s": None if hdt == 0 else sc, "norm": norm,
            "eps": float(eps[0])}


def ref_decode(model_dir, dtype, prompt, opts: OracleSampling, max_tokens: int, build: str = "scalar",
               threads: int = 1) -> dict:
    """verbo::generate of the reference on a checkpoint (one generation), and
    for every pick its id and the hidden row its logits came from (the
    residual before the final rmsnorm).  Returns ids (picks,), x (picks, dim)
    and stopped (the last pick is a stop id)."""
    lib = _ref_tail_lib(build)
    dt = DTYPES[dtype] if isinstance(dtype, str) else int(dtype)
    meta = np.zeros(3, dtype=np.int32)
    eps = np.zeros(1, dtype=np.float32)
    path = str(model_dir).encode()
    if lib.ref_model_tail(path, dt, None, 0, threads, _ptr(meta), _ptr(eps), None, None, None, None, None) != 0:
        raise RuntimeError(f"the reference could not load {model_dir}")
    dim = int(meta[0])
    prompt = np.ascontiguousarray(prompt, dtype=np.int32)
    cap = max_tokens + 1
    ids = np.zeros(cap, dtype=np.int32)
    x = np.zeros((cap, dim), dtype=np.float32)
    stopped = np.zeros(1, dtype=np.int32)
    n = lib.ref_decode(path, dt, _ptr(prompt), prompt.size, ctypes.byref(opts), max_tokens, threads, cap, _ptr(ids),
                       _ptr(x), _ptr(stopped))
    if n == -2:
        raise RuntimeError("the replayed decode loop disagrees with verbo::generate")
    if n < 0:
        raise RuntimeError(f"ref_decode failed on {model_dir}")
    return {"ids": ids[:n].copy(), "x": x[:n].copy(), "stopped": bool(stopped[0])}


def random_head(dtype: str, vocab: int, dim: int, seed: int = 0):
    """A seeded head in verbo::Tensor layout with the value ranges the
    reference's quant_rows produces (src/kernels.cpp:133-175): Q8 codes in
    [-127, 127], Q4 nibbles in [0, 15], positive fp16 scales."""
    g = np.random.default_rng(seed)
    if dtype == "f32":
        return (g.standard_normal((vocab, dim)) * 0.05).astype(np.float32), None
    s = (np.abs(g.standard_normal((vocab, dim // 32))) * 0.004 + 1e-4).astype(np.float16).view(np.uint16)
    if dtype == "q8":
        return g.integers(-127, 128, size=(vocab, dim), dtype=np.int8), s
    return g.integers(0, 256, size=(vocab, dim // 2), dtype=np.uint8), s


def host_threads() -> int:
    return len(os.sched_getaffinity(0))
