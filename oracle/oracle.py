"""ctypes wrapper around the CPU oracle (``oracle/libbsoracle.so``).

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline / reference legs may import this module, and only
as the checker or as the timed CPU port of the reference's own decoders.  The
product package ``bigsmall_b200`` never imports it: the GPU path has no CPU
fallback.

Every function here is a thin call into ``bs_oracle.c``; each C function cites
the reference file:line it restates (BigSmall ``bigsmall/codecs/rans.py``,
``bf16_parallel.py``, ``single_kernel.py``, ``bf16_tans.py``/``numba_rans.py``)
or, for ``xc_*``, implements this project's own ``bf16_exp_chunked_v1`` format
whose parity anchor is the md5 of the raw tensor bytes.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "libbsoracle.so")
_lib = None

ERRORS = {
    -1: "bad argument", -2: "bad magic", -3: "count mismatch", -4: "truncated",
    -5: "precision mismatch", -6: "output capacity", -7: "corrupt stream",
    -8: "out of memory",
}


class OracleError(ValueError):
    pass


def build() -> str:
    """Compile the oracle with its Makefile (gcc only; a few seconds)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(
            os.path.join(_HERE, "bs_oracle.c")):
        build()
    L = ctypes.CDLL(_SO)
    P, I64, I32, U32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_uint32
    sigs = {
        "bso_quantise_ref": (I32, [P, I32, U32, P]),
        "bso_rans_encode": (I64, [P, I64, P, I32, U32, P, I64]),
        "bso_rans_decode": (I32, [P, I64, I64, P, I32, U32, P]),
        "bso_par_bound": (I64, [I64, I32]),
        "bso_par_encode": (I64, [P, I64, I32, P, I64]),
        "bso_par_decode": (I32, [P, I64, I64, P]),
        "bso_sk_bound": (I64, [I64]),
        "bso_sk_encode": (I64, [P, I64, P, I64]),
        "bso_sk_decode": (I32, [P, I64, I64, P]),
        "bso_sk_decode_many": (I32, [P, P, P, P, I32, I32]),
        "bso_tans_bound": (I64, [I64]),
        "bso_tans_encode": (I64, [P, I64, P, I64]),
        "bso_tans_decode": (I32, [P, I64, I64, P]),
        "bso_tans_decode_many": (I32, [P, P, P, P, I32, I32]),
        "bso_xc_bound": (I64, [I64, U32]),
        "bso_xc_encode": (I64, [P, I64, I32, I32, U32, P, I64]),
        "bso_xc_encode_groups": (I64, [P, I64, I32, I32, U32, U32, P, I64]),
        "bso_xc_decode": (I32, [P, I64, I64, P]),
        "bso_xc_quantise": (I32, [P, I32, P]),
        "bso_xc_decode_many": (I32, [P, P, P, P, I32, I32]),
        "bso_par_decode_many": (I32, [P, P, P, P, I32, I32]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _check(rc: int, what: str) -> int:
    if rc < 0:
        raise OracleError(f"{what}: {ERRORS.get(rc, rc)}")
    return rc


def _u16(raw) -> np.ndarray:
    if isinstance(raw, np.ndarray):
        return np.ascontiguousarray(raw).view(np.uint16).reshape(-1)
    return np.frombuffer(bytes(raw), dtype=np.uint16)


def _blob(blob) -> np.ndarray:
    if isinstance(blob, np.ndarray):
        return np.ascontiguousarray(blob).view(np.uint8).reshape(-1)
    return np.frombuffer(bytes(blob), dtype=np.uint8)


# ---- rans.py -----------------------------------------------------------------
def quantise_ref(counts, M: int) -> np.ndarray:
    c = np.ascontiguousarray(counts, dtype=np.int64)
    f = np.zeros(len(c), dtype=np.uint32)
    _check(lib().bso_quantise_ref(_ptr(c), len(c), M, _ptr(f)), "quantise")
    return f


def rans_encode(symbols, freqs, M: int) -> bytes:
    s = np.ascontiguousarray(symbols, dtype=np.int32)
    f = np.ascontiguousarray(freqs, dtype=np.uint32)
    cap = 16 + 2 * len(s) + 16
    out = np.empty(cap, dtype=np.uint8)
    n = _check(lib().bso_rans_encode(_ptr(s), len(s), _ptr(f), len(f), M, _ptr(out), cap), "rans_encode")
    return out[:n].tobytes()


def rans_decode(data: bytes, n: int, freqs, M: int) -> np.ndarray:
    d = _blob(data)
    f = np.ascontiguousarray(freqs, dtype=np.uint32)
    out = np.zeros(max(n, 1), dtype=np.uint32)
    _check(lib().bso_rans_decode(_ptr(d), len(d), n, _ptr(f), len(f), M, _ptr(out)), "rans_decode")
    return out[:n]


# ---- codecs: encode(raw) -> blob, decode(blob, n) -> raw ----------------------
def _enc(kind: str, raw, *args) -> bytes:
    w = _u16(raw)
    n = len(w)
    L = lib()
    bound = {"par": lambda: L.bso_par_bound(n, args[0]), "sk": lambda: L.bso_sk_bound(n),
             "tans": lambda: L.bso_tans_bound(n),
             "xc": lambda: L.bso_xc_bound(n, args[2])}[kind]()
    out = np.empty(max(bound, 16), dtype=np.uint8)
    fn = getattr(L, f"bso_{kind}_encode")
    nb = _check(fn(_ptr(w), n, *args, _ptr(out), len(out)), f"{kind}_encode")
    return out[:nb].tobytes()


def _dec(kind: str, blob, n_weights: int) -> bytes:
    b = _blob(blob)
    out = np.zeros(max(n_weights, 1), dtype=np.uint16)
    fn = getattr(lib(), f"bso_{kind}_decode")
    _check(fn(_ptr(b), len(b), n_weights, _ptr(out)), f"{kind}_decode")
    return out[:n_weights].tobytes()


def par_encode(raw, n_streams: int = 128) -> bytes:
    return _enc("par", raw, n_streams)


def par_decode(blob, n_weights: int) -> bytes:
    return _dec("par", blob, n_weights)


def sk_encode(raw) -> bytes:
    return _enc("sk", raw)


def sk_decode(blob, n_weights: int) -> bytes:
    return _dec("sk", blob, n_weights)


def tans_encode(raw) -> bytes:
    return _enc("tans", raw)


def tans_decode(blob, n_weights: int) -> bytes:
    return _dec("tans", blob, n_weights)


def xc_encode(raw, coder: int = 0, prec: int = 12, chunk_elems: int = 65536, groups: int = 1) -> bytes:
    """bf16_exp_chunked_v1 blob; `groups` > 1 cuts each chunk into that many
    state groups (format version 2)."""
    if groups == 1:
        return _enc("xc", raw, coder, prec, chunk_elems)
    w = _u16(raw)
    n = len(w)
    L = lib()
    ge = chunk_elems // groups if groups > 0 else 0
    out = np.empty(max(L.bso_xc_bound(n, ge) if ge else 16, 16), dtype=np.uint8)
    nb = _check(L.bso_xc_encode_groups(_ptr(w), n, coder, prec, chunk_elems, groups, _ptr(out), len(out)),
                "xc_encode_groups")
    return out[:nb].tobytes()


def xc_decode(blob, n_weights: int) -> bytes:
    return _dec("xc", blob, n_weights)


def xc_quantise(counts, prec: int = 12) -> np.ndarray:
    c = np.ascontiguousarray(counts, dtype=np.int64)
    assert len(c) == 256
    f = np.zeros(256, dtype=np.uint16)
    _check(lib().bso_xc_quantise(_ptr(c), prec, _ptr(f)), "xc_quantise")
    return f


def decode_many(kind: str, blobs, n_weights, threads: int) -> list[np.ndarray]:
    """Decode many blobs on `threads` host threads (kind 'sk', 'tans', 'xc' or 'par')."""
    arrs = [_blob(b) for b in blobs]
    outs = [np.empty(max(int(n), 1), dtype=np.uint16) for n in n_weights]
    cnt = len(arrs)
    bp = (ctypes.c_void_p * cnt)(*[a.ctypes.data for a in arrs])
    op = (ctypes.c_void_p * cnt)(*[o.ctypes.data for o in outs])
    lens = np.array([len(a) for a in arrs], dtype=np.int64)
    nw = np.array(list(n_weights), dtype=np.int64)
    fn = getattr(lib(), f"bso_{kind}_decode_many")
    _check(fn(bp, _ptr(lens), _ptr(nw), op, cnt, threads), f"{kind}_decode_many")
    return outs
