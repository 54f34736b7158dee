"""Device-resident API over libbsgpu.so (PyTorch supplies memory and streams).

Everything here runs on the CUDA device through the C ABI declared in
``include/bsgpu.h``; there is no CPU decode path.  Tensors handed to these
functions must be CUDA tensors; compressed blobs are ``torch.uint8`` device
tensors, decoded outputs ``torch.bfloat16`` (or a same-size 16-bit view).

Reference counterparts (BigSmall):
  * ``bigsmall/kernels/__init__.py:89-111`` decode_bf16_parallel  -> :func:`decode_par_into`
  * ``bigsmall/kernels/ac_triton.py:112-262`` (Triton SE + CPU mantissa) -> :class:`ParPlan`
  * ``bigsmall/decoder.py:128-136`` per-tensor decode loop -> :class:`XcPlan` (batched)
  * ``bigsmall/codecs/kv_cache.py:41-83`` CPU encode -> :func:`encode_xc`
"""
from __future__ import annotations

import ctypes
from typing import Iterable, Optional, Sequence

import torch

from . import _lib

# 64 KiB of bf16 per chunk (one warp-state group).  A chunk is the unit one
# warp decodes, so smaller chunks give more warps per tensor: a model layer
# or one GPU's share of an 8-GPU container then fills the SMs several times
# over instead of ~3 waves (1.6 % slower on a whole container on one GPU,
# 5.5 % faster on eight; ratio +0.0009).
DEFAULT_CHUNK_ELEMS = 32768
DEFAULT_PREC = 12             # M = 4096

CODERS = {"rans": _lib.CODER_RANS, "tans": _lib.CODER_TANS, "pair": _lib.CODER_RANS_PAIR}
# rANS over exponent pairs: half the coder steps per value for ~0.1 pp of ratio
DEFAULT_CODER = "pair"


def _as_cuda(t: torch.Tensor, name: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t


def _stream_ptr(stream, device) -> ctypes.c_void_p:
    if stream is None:
        stream = torch.cuda.current_stream(device)
    return ctypes.c_void_p(stream.cuda_stream)


def _dev_index(t: torch.Tensor) -> int:
    return t.device.index if t.device.index is not None else torch.cuda.current_device()


class _Plan:
    """Owns a ``bs_plan*``; keeps the tensors it points at alive."""

    def __init__(self, handle: ctypes.c_void_p, device: int, keep: list, n: int):
        self._h = handle
        self.device = device
        self._keep = keep
        self.n_tensors = n

    def decode(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Enqueue the decode on `stream` (default: current stream).  Async."""
        L = _lib.load()
        _lib.check(L.bs_plan_decode(self._h, _stream_ptr(stream, self.device)), "bs_plan_decode")

    def decode_timed(self, start: torch.cuda.Event, stop: torch.cuda.Event,
                     stream: Optional[torch.cuda.Stream] = None) -> None:
        """``decode`` with ``start`` / ``stop`` (timing events) recorded right
        before and after the decode kernels, so ``start.elapsed_time(stop)``
        is the decode kernels' time alone (without the per-launch table build)."""
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        for ev in (start, stop):
            if not ev.cuda_event:          # torch creates the event on first record
                ev.record(s)
        L = _lib.load()
        _lib.check(L.bs_plan_decode_timed(self._h, _stream_ptr(s, self.device), ctypes.c_void_p(start.cuda_event),
                                          ctypes.c_void_p(stop.cuda_event)), "bs_plan_decode_timed")

    def decode_after(self, stream: torch.cuda.Stream, wait: Optional[torch.cuda.Event] = None,
                     done: Optional[torch.cuda.Event] = None) -> None:
        """``stream`` waits for ``wait``, decodes, then records ``done``: one
        library call.  torch creates an event on its first record, so an event
        not yet created is recorded on ``stream`` first (a wait on it is then
        already satisfied, as a wait on an unrecorded event is)."""
        for ev in (wait, done):
            if ev is not None and not ev.cuda_event:
                ev.record(stream)
        L = _lib.load()
        _lib.check(L.bs_plan_decode_after(self._h, _stream_ptr(stream, self.device),
                                          ctypes.c_void_p(wait.cuda_event) if wait is not None else None,
                                          ctypes.c_void_p(done.cuda_event) if done is not None else None),
                   "bs_plan_decode_after")

    def handoff_call(self, side: torch.cuda.Stream, release: torch.cuda.Event, done: torch.cuda.Event,
                     next_ev: Optional[torch.cuda.Event] = None):
        """A prepared ``f(main_stream)`` for a two-stream prefetch: records
        ``release`` on ``main_stream``, makes ``side`` wait for it, decodes on
        ``side``, records ``done`` there, then makes ``main_stream`` wait for
        ``next_ev`` -- one library call per use, its arguments resolved once
        (events must have been recorded once, which creates them)."""
        for ev in (release, done, next_ev):
            if ev is not None and not ev.cuda_event:
                raise ValueError("hand-off events must have been recorded once")
        fn = _lib.load().bs_plan_decode_handoff
        h = self._h
        args = (ctypes.c_void_p(side.cuda_stream), ctypes.c_void_p(release.cuda_event),
                ctypes.c_void_p(done.cuda_event), ctypes.c_void_p(next_ev.cuda_event) if next_ev is not None else None)

        def call(main: torch.cuda.Stream) -> None:
            rc = fn(h, main.cuda_stream, *args)
            if rc:
                _lib.check(rc, "bs_plan_decode_handoff")
        return call

    def launch_count(self) -> int:
        """Kernels this plan has launched so far (a count kept by the library)."""
        v = ctypes.c_uint64()
        _lib.check(_lib.load().bs_plan_launch_count(self._h, ctypes.byref(v)), "bs_plan_launch_count")
        return int(v.value)

    def check(self, stream: Optional[torch.cuda.Stream] = None) -> list[int]:
        """Synchronise `stream` and raise BsCorruptError if any tensor failed."""
        L = _lib.load()
        st = (ctypes.c_uint32 * max(1, self.n_tensors))()
        rc = L.bs_plan_check(self._h, _stream_ptr(stream, self.device), st)
        words = [int(st[i]) for i in range(self.n_tensors)]
        if rc != _lib.BS_OK:
            bad = [(i, _lib.describe_device_status(w)) for i, w in enumerate(words) if w]
            _lib.check(rc, f"decode failed {bad}", words)
        return words

    def run(self, stream=None) -> None:
        self.decode(stream)
        self.check(stream)

    def close(self) -> None:
        if self._h:
            _lib.load().bs_plan_destroy(self._h)
            self._h = None
            self._keep = []

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def coder_mask(coder) -> int:
    """BS_CODER_* bit of a coder name or value; 0 (any coder) for None."""
    if coder is None:
        return 0
    c = CODERS[coder] if isinstance(coder, str) else int(coder)
    if c not in CODERS.values():
        raise ValueError(f"unknown coder {coder!r}")
    return 1 << c


class XcPlan(_Plan):
    """Decode plan for a batch of bf16_exp_chunked_v1 tensors.

    ``entries``: iterable of ``(blob, out, chunk_elems)`` with ``blob`` a
    1-D uint8 CUDA tensor (16-byte aligned) and ``out`` a contiguous 16-bit
    CUDA tensor receiving ``out.numel()`` values; or of
    ``(blob, out, chunk_elems, n_total, chunk_begin, chunk_count)`` to decode
    only chunks [chunk_begin, chunk_begin + chunk_count) of a tensor of
    ``n_total`` values into ``out`` (element chunk_begin * chunk_elems first).
    One plan decodes all entries with one prepare launch plus one decode
    launch per coder family present; it can be re-run any number of times.

    ``coders``: the coder each blob was written with ("rans", "tans", "pair"
    or a BS_CODER_* value), one for all entries or a sequence with one per
    entry; None (or a None element) means unknown, which launches every
    decode kernel.  A blob whose header names another coder fails with
    BS_DEV_HEADER rather than being skipped.

    ``groups``: state groups per chunk of each blob (the container's
    ``extra["groups"]``; 1 or None for a one-group, format-version-1 blob),
    one for all entries or a sequence with one per entry.
    """

    def __init__(self, entries: Iterable[tuple], device: Optional[int] = None, coders=None,
                 max_ctas: Optional[int] = None, groups=None):
        entries = list(entries)
        if coders is None or isinstance(coders, (str, int)):
            coders = [coders] * len(entries)
        coders = list(coders)
        if len(coders) != len(entries):
            raise ValueError("coders must have one element per entry")
        if groups is None or isinstance(groups, int):
            groups = [groups] * len(entries)
        groups = list(groups)
        if len(groups) != len(entries):
            raise ValueError("groups must have one element per entry")
        keep = []
        arr = (_lib.XcTensor * max(1, len(entries)))()
        dev = device
        for i, ent in enumerate(entries):
            blob, out, ce = ent[:3]
            n_total, c0, cc = (ent[3], ent[4], ent[5]) if len(ent) > 3 else (out.numel(), 0, 0)
            _as_cuda(blob, "blob")
            _as_cuda(out, "out")
            if blob.dtype != torch.uint8:
                raise TypeError("blob must be torch.uint8")
            if out.element_size() != 2:
                raise TypeError("out must be a 16-bit tensor (bfloat16)")
            d = _dev_index(out)
            if dev is None:
                dev = d
            if d != dev or _dev_index(blob) != dev:
                raise ValueError("all tensors of a plan must live on one device")
            arr[i].d_blob = blob.data_ptr() if blob.numel() else None
            arr[i].blob_bytes = blob.numel()
            arr[i].d_out = out.data_ptr() if out.numel() else None
            arr[i].n_elems = int(n_total)
            arr[i].chunk_elems = int(ce)
            arr[i].chunk_begin = int(c0)
            arr[i].chunk_count = int(cc)
            arr[i].coder_mask = coder_mask(coders[i])
            arr[i].groups = int(groups[i] or 1)
            keep += [blob, out]
        if dev is None:
            dev = torch.cuda.current_device()
        h = ctypes.c_void_p()
        L = _lib.load()
        _lib.check(L.bs_xc_plan_create(arr, len(entries), dev, ctypes.byref(h)), "bs_xc_plan_create")
        super().__init__(h, dev, keep, len(entries))
        if max_ctas:
            self.set_max_ctas(max_ctas)

    def set_max_ctas(self, max_ctas: int) -> None:
        """Cap the decode grid at ``max_ctas`` CTAs (0: uncapped) so kernels on
        other streams keep SM room while this plan decodes."""
        _lib.check(_lib.load().bs_plan_set_max_ctas(self._h, int(max_ctas)), "bs_plan_set_max_ctas")


class ParPlan(_Plan):
    """Decode plan for one bf16_parallel_v1 blob (the reference's GPU format).

    The framing is parsed from ``host_blob`` (bytes identical to ``d_blob``).
    """

    def __init__(self, host_blob: bytes, d_blob: torch.Tensor, out: torch.Tensor, n_weights: int):
        _as_cuda(out, "out")
        if n_weights and len(host_blob):
            _as_cuda(d_blob, "d_blob")
        if out.numel() < n_weights:
            raise ValueError("out is smaller than n_weights")
        dev = _dev_index(out)
        hb = ctypes.create_string_buffer(bytes(host_blob), len(host_blob)) if len(host_blob) else None
        h = ctypes.c_void_p()
        L = _lib.load()
        rc = L.bs_par_plan_create(hb, len(host_blob), int(n_weights),
                                  d_blob.data_ptr() if d_blob is not None and d_blob.numel() else None,
                                  out.data_ptr() if out.numel() else None, dev, ctypes.byref(h))
        _lib.check(rc, "bs_par_plan_create")
        super().__init__(h, dev, [d_blob, out], 1)


SE_CODECS = {"bf16_se_single_kernel": _lib.SE_SINGLE_KERNEL, "bf16_se_tans": _lib.SE_TANS}
# every format decoded by serial streams, batchable in one SePlan
SERIAL_CODECS = {**SE_CODECS, "bf16_parallel_v1": _lib.SE_PARALLEL}


class SePlan(_Plan):
    """Decode plan for blobs of the serial-stream formats: the legacy
    bf16_se_single_kernel / bf16_se_tans and the reference's bf16_parallel_v1.

    ``entries``: iterable of ``(codec, host_blob, d_blob, out, n_weights)``;
    the framing is parsed from ``host_blob`` (bytes identical to ``d_blob``,
    a 1-D uint8 CUDA tensor).  Every serial stream of every entry runs
    concurrently on the device, then the exponent un-sort, so the plan takes
    the time of its longest (sign,exp) stream."""

    def __init__(self, entries: Iterable[tuple], device: Optional[int] = None):
        entries = list(entries)
        arr = (_lib.SeBlob * max(1, len(entries)))()
        keep, dev = [], device
        for i, (codec, host_blob, d_blob, out, n_weights) in enumerate(entries):
            if codec not in SERIAL_CODECS:
                raise ValueError(f"not a serial-stream codec: {codec!r}")
            _as_cuda(out, "out")
            if out.element_size() != 2:
                raise TypeError("out must be a 16-bit tensor (bfloat16)")
            if out.numel() < n_weights:
                raise ValueError("out is smaller than n_weights")
            hb = bytes(host_blob)
            if n_weights and hb:
                _as_cuda(d_blob, "d_blob")
            d = _dev_index(out)
            if dev is None:
                dev = d
            if d != dev or (d_blob is not None and d_blob.numel() and _dev_index(d_blob) != dev):
                raise ValueError("all tensors of a plan must live on one device")
            cbuf = ctypes.create_string_buffer(hb, len(hb)) if hb else None
            arr[i].codec = SERIAL_CODECS[codec]
            arr[i].h_blob = ctypes.cast(cbuf, ctypes.c_void_p) if cbuf is not None else None
            arr[i].blob_bytes = len(hb)
            arr[i].n_weights = int(n_weights)
            arr[i].d_blob = d_blob.data_ptr() if d_blob is not None and d_blob.numel() else None
            arr[i].d_out = out.data_ptr() if out.numel() else None
            keep += [cbuf, d_blob, out]
        if dev is None:
            dev = torch.cuda.current_device()
        h = ctypes.c_void_p()
        L = _lib.load()
        _lib.check(L.bs_se_plan_create_many(arr, len(entries), dev, ctypes.byref(h)), "bs_se_plan_create_many")
        super().__init__(h, dev, [k for k in keep if k is not None and not isinstance(k, ctypes.Array)],
                         len(entries))


def decode_se_into(codec: str, host_blob: bytes, d_blob: torch.Tensor, out: torch.Tensor, n_weights: int,
                   stream=None) -> torch.Tensor:
    """Decode one legacy serial blob (device) into ``out`` (device)."""
    with SePlan([(codec, host_blob, d_blob, out, n_weights)]) as p:
        p.run(stream)
    return out


def decode_xc_into(blob: torch.Tensor, out: torch.Tensor, chunk_elems: int,
                   stream=None, check: bool = True, coder=None, groups: int = 1) -> torch.Tensor:
    """Decode one bf16_exp_chunked_v1 blob (device) into ``out`` (device)."""
    with XcPlan([(blob, out, chunk_elems)], coders=coder, groups=groups) as p:
        p.decode(stream)
        if check:
            p.check(stream)
    return out


def decode_par_into(host_blob: bytes, d_blob: torch.Tensor, out: torch.Tensor, n_weights: int,
                    stream=None) -> torch.Tensor:
    with ParPlan(host_blob, d_blob, out, n_weights) as p:
        p.run(stream)
    return out


# ---------------------------------------------------------------------------
# encoder
# ---------------------------------------------------------------------------
def encode_bound(n: int, chunk_elems: int = DEFAULT_CHUNK_ELEMS, groups: int = 1) -> int:
    v = ctypes.c_uint64()
    _lib.check(_lib.load().bs_xc_encode_bound(n, chunk_elems, groups, ctypes.byref(v)), "bs_xc_encode_bound")
    return int(v.value)


def encode_workspace(n: int, chunk_elems: int = DEFAULT_CHUNK_ELEMS, coder: str = DEFAULT_CODER,
                     groups: int = 1) -> int:
    v = ctypes.c_uint64()
    c = CODERS[coder] if isinstance(coder, str) else int(coder)
    _lib.check(_lib.load().bs_xc_encode_workspace(n, chunk_elems, groups, c, ctypes.byref(v)),
               "bs_xc_encode_workspace")
    return int(v.value)


class XcEncoder:
    """Reusable device encoder: owns an output buffer and a workspace sized for
    tensors of up to ``max_elems`` values (no allocation per call).  Chunks of
    ``chunk_elems`` values are cut into ``groups`` state groups."""

    def __init__(self, max_elems: int, chunk_elems: int = DEFAULT_CHUNK_ELEMS, coder: str = DEFAULT_CODER,
                 prec: int = DEFAULT_PREC, device=None, groups: int = 1):
        self.chunk_elems = int(chunk_elems)
        self.groups = int(groups or 1)
        self.coder = CODERS[coder] if isinstance(coder, str) else int(coder)
        self.prec = int(prec)
        self.max_elems = int(max_elems)
        dev = torch.device("cuda", device if device is not None else torch.cuda.current_device())
        self.device = dev
        self.out = torch.empty(max(16, encode_bound(max_elems, chunk_elems, self.groups)), dtype=torch.uint8,
                               device=dev)
        self.ws = torch.empty(max(16, encode_workspace(max_elems, chunk_elems, self.coder, self.groups)),
                              dtype=torch.uint8, device=dev)
        self.out_len = torch.zeros(2, dtype=torch.int64, device=dev)

    def encode_async(self, x: torch.Tensor, stream=None) -> None:
        """Enqueue the encode of ``x``; the blob is ``self.out[:self.out_len[0]]``."""
        _as_cuda(x, "x")
        if x.element_size() != 2:
            raise TypeError("x must be a 16-bit tensor (bfloat16)")
        n = x.numel()
        if n > self.max_elems:
            raise ValueError(f"tensor of {n} values exceeds encoder capacity {self.max_elems}")
        L = _lib.load()
        rc = L.bs_xc_encode(x.data_ptr() if n else None, n, self.coder, self.prec, self.chunk_elems, self.groups,
                            self.out.data_ptr(), self.out.numel(), self.out_len.data_ptr(),
                            self.ws.data_ptr(), self.ws.numel(), _stream_ptr(stream, self.device))
        _lib.check(rc, "bs_xc_encode")

    def encode_into(self, x: torch.Tensor, out: torch.Tensor, out_len: torch.Tensor, stream=None) -> None:
        """Enqueue the encode of ``x`` into ``out`` (uint8, >= encode_bound bytes);
        the blob length lands in ``out_len[0]`` (int64 device tensor).  Uses this
        encoder's workspace, so calls on one stream must not overlap others."""
        _as_cuda(x, "x")
        _as_cuda(out, "out")
        n = x.numel()
        if n > self.max_elems:
            raise ValueError(f"tensor of {n} values exceeds encoder capacity {self.max_elems}")
        L = _lib.load()
        rc = L.bs_xc_encode(x.data_ptr() if n else None, n, self.coder, self.prec, self.chunk_elems, self.groups,
                            out.data_ptr(), out.numel(), out_len.data_ptr(), self.ws.data_ptr(), self.ws.numel(),
                            _stream_ptr(stream, self.device))
        _lib.check(rc, "bs_xc_encode")

    def encode(self, x: torch.Tensor, stream=None) -> torch.Tensor:
        """Encode ``x`` and return a right-sized device copy of the blob."""
        self.encode_async(x, stream)
        n = int(self.out_len[0].item())
        return self.out[:n].clone()


def encode_xc(x: torch.Tensor, coder: str = DEFAULT_CODER, prec: int = DEFAULT_PREC,
              chunk_elems: int = DEFAULT_CHUNK_ELEMS, stream=None, groups: int = 1) -> torch.Tensor:
    """Encode a bf16 CUDA tensor into a bf16_exp_chunked_v1 blob on the device."""
    enc = XcEncoder(max(1, x.numel()), chunk_elems, coder, prec, device=_dev_index(x), groups=groups)
    return enc.encode(x.reshape(-1), stream)


def xc_extras(chunk_elems: int = DEFAULT_CHUNK_ELEMS, coder: str = DEFAULT_CODER, prec: int = DEFAULT_PREC,
              groups: int = 1) -> dict:
    """The per-tensor ``extra`` dict the container header stores for the codec
    (``groups`` only when a chunk holds more than one state group)."""
    d = {"chunk_elems": int(chunk_elems), "coder": coder, "prec": int(prec)}
    if int(groups or 1) > 1:
        d["groups"] = int(groups)
    return d


def extras_groups(extra: Optional[dict]) -> int:
    """State groups per chunk recorded in a tensor's ``extra`` dict (1 if absent)."""
    return int((extra or {}).get("groups", 1) or 1)


def aligned_view(buf: torch.Tensor, offset: int, nbytes: int) -> torch.Tensor:
    """A 16-byte aligned device view of buf[offset:offset+nbytes] (a copy if the
    slice is misaligned)."""
    v = buf[offset:offset + nbytes]
    if nbytes and v.data_ptr() % 16:
        v = v.clone()
    return v


def sync(device=None) -> None:
    torch.cuda.synchronize(device)


__all__: Sequence[str] = [
    "DEFAULT_CHUNK_ELEMS", "DEFAULT_PREC", "DEFAULT_CODER", "SePlan", "decode_se_into", "SE_CODECS", "SERIAL_CODECS", "XcPlan", "ParPlan", "XcEncoder", "decode_xc_into",
    "decode_par_into", "encode_xc", "encode_bound", "encode_workspace", "xc_extras", "extras_groups", "aligned_view",
]
