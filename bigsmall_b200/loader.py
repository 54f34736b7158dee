"""Container -> HBM loading with the compressed bytes as the only host->device
traffic.

The reference loads a container by decoding every tensor on the CPU and then
copying the *decoded* bytes to the device (BigSmall ``bigsmall/decoder.py:301-310``
``load``; ``bigsmall/streaming.py:183-191`` ``_to_torch``).  Here the
compressed data section is held in pinned host memory (:class:`ContainerImage`),
copied to the device group by group on a copy stream, and each group is decoded
on the compute stream as soon as its bytes have landed (:class:`DeviceLoader`),
so PCIe transfer of group i+1 overlaps the decode of group i.

Codecs handled on the device: ``bf16_exp_chunked_v1`` (batched per group),
``bf16_parallel_v1``, the legacy serial ``bf16_se_single_kernel`` and
``bf16_se_tans``, ``raw`` and ``tied_ref``.  Any other codec raises
``BigSmallVersionError`` exactly like the reference's dispatcher
(``bigsmall/decoder.py:89-97``); nothing is decoded on the CPU.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Iterable, Optional

import numpy as np
import torch

from . import container as _ct
from . import gpu
from .exceptions import BigSmallVersionError

DEVICE_CODECS = ("bf16_exp_chunked_v1", "bf16_parallel_v1", "bf16_se_single_kernel", "bf16_se_tans", "raw",
                 "tied_ref")

TORCH_DTYPES = {
    "BF16": torch.bfloat16, "bfloat16": torch.bfloat16, "F16": torch.float16, "float16": torch.float16,
    "F32": torch.float32, "float32": torch.float32, "I64": torch.int64, "int64": torch.int64,
    "I32": torch.int32, "int32": torch.int32, "I16": torch.int16, "int16": torch.int16,
    "I8": torch.int8, "int8": torch.int8, "U8": torch.uint8, "uint8": torch.uint8,
    "BOOL": torch.bool, "bool": torch.bool,
    "F8_E4M3": getattr(torch, "float8_e4m3fn", torch.uint8), "float8_e4m3fn": getattr(torch, "float8_e4m3fn", torch.uint8),
    "F8_E5M2": getattr(torch, "float8_e5m2", torch.uint8), "float8_e5m2": getattr(torch, "float8_e5m2", torch.uint8),
}


def _unknown_codec(codec: str):
    from . import __version__
    return BigSmallVersionError(required="newer-than-installed", installed=__version__,
                                detail=f"file references unknown codec {codec!r}")


class ContainerImage:
    """A container's header plus its data section in (pinned) host memory."""

    def __init__(self, header: dict, data, pin: bool = True):
        self.header = header
        self.tensors = {t["name"]: t for t in header["tensors"]}
        if isinstance(data, torch.Tensor):
            host = data.reshape(-1).view(torch.uint8)
        else:
            arr = np.frombuffer(data, dtype=np.uint8) if not isinstance(data, np.ndarray) else data.reshape(-1).view(np.uint8)
            if not arr.flags.writeable:
                arr = arr.copy()
            host = torch.from_numpy(arr)
        if pin and not host.is_pinned():
            pinned = torch.empty(host.numel(), dtype=torch.uint8, pin_memory=True)
            pinned.copy_(host)
            host = pinned
        self.host = host

    @classmethod
    def from_bytes(cls, buf: bytes, pin: bool = True) -> "ContainerImage":
        header, off = _ct.parse_header(buf)
        return cls(header, memoryview(buf)[off:], pin=pin)

    @classmethod
    def from_file(cls, path, pin: bool = True) -> "ContainerImage":
        header, off = _ct.read_header(path)
        with open(path, "rb") as f:
            f.seek(off)
            data = f.read()
        return cls(header, data, pin=pin)

    def blob_host(self, name: str) -> memoryview:
        t = self.tensors[name]
        return memoryview(self.host.numpy())[t["offset"]:t["offset"] + t["compressed_bytes"]]

    def raw_bytes(self) -> int:
        return sum(_ct.tensor_raw_bytes(t) for t in self.header["tensors"])

    def compressed_bytes(self) -> int:
        return sum(int(t["compressed_bytes"]) for t in self.header["tensors"])


@dataclass
class _Part:
    """One tensor (or chunk range of one) a loader decodes."""
    name: str
    meta: dict
    chunk_begin: int = 0
    chunk_count: int = 0          # 0: whole tensor
    out: Optional[torch.Tensor] = None


@dataclass
class _Group:
    lo: int                       # byte range of the data section copied to the device
    hi: int
    parts: list = field(default_factory=list)
    plans: list = field(default_factory=list)
    copies: list = field(default_factory=list)   # (dst, src view) device copies for raw tensors
    event: Optional[torch.cuda.Event] = None


class DeviceLoader:
    """Decode (part of) a :class:`ContainerImage` into device tensors.

    ``owned``: optional iterable of ``name`` or ``(name, chunk_begin, chunk_count)``
    selecting what this loader (e.g. one rank of several GPUs) decodes; default
    all tensors.  Output tensors are allocated once and reused by every
    :meth:`run`; the plans are built once.
    """

    def __init__(self, image: ContainerImage, device=None, owned: Optional[Iterable] = None,
                 group_bytes: int = 256 << 20, out: Optional[dict] = None):
        self.image = image
        self.device = torch.device("cuda", device if isinstance(device, int) else
                                   (torch.device(device).index if device is not None else torch.cuda.current_device()))
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        parts = []
        for item in (owned if owned is not None else image.tensors.keys()):
            name, c0, cc = (item, 0, 0) if isinstance(item, str) else (item[0], int(item[1]), int(item[2]))
            meta = image.tensors[name]
            if meta["codec"] not in DEVICE_CODECS:
                raise _unknown_codec(meta["codec"])
            if cc and meta["codec"] != "bf16_exp_chunked_v1":
                raise ValueError(f"chunk ranges apply to bf16_exp_chunked_v1 tensors only ({name})")
            parts.append(_Part(name, meta, c0, cc))
        # tied tensors need their master decoded here as well
        names = {p.name for p in parts}
        for p in list(parts):
            if p.meta["codec"] == "tied_ref":
                m = (p.meta.get("extra") or {})["tied_to"]
                if m not in names:
                    parts.append(_Part(m, image.tensors[m]))
                    names.add(m)
        self.parts = parts
        self.out: dict[str, torch.Tensor] = dict(out or {})
        self._alloc_outputs()
        self._build_groups(group_bytes)
        self.copy_stream = torch.cuda.Stream(self.device)

    # -- setup ---------------------------------------------------------------
    def _alloc_outputs(self):
        for p in self.parts:
            m = p.meta
            if m["codec"] == "tied_ref" or p.name in self.out:
                continue
            shape = m["shape"] or []
            if p.chunk_count:
                ce = int((m.get("extra") or {})["chunk_elems"])
                n = _ct.n_elements(shape)
                lo = p.chunk_begin * ce
                hi = min(n, (p.chunk_begin + p.chunk_count) * ce)
                t = torch.empty(hi - lo, dtype=TORCH_DTYPES[m["dtype"]], device=self.device)
            else:
                t = torch.empty(shape, dtype=TORCH_DTYPES.get(m["dtype"], torch.uint8), device=self.device)
            self.out[p.name] = t

    def _build_groups(self, group_bytes: int):
        # copy each part's blob once; lay the needed blobs out back to back
        # (16-byte aligned) in one device buffer, grouped by size
        spans = []
        seen = set()
        for p in self.parts:
            m = p.meta
            if m["codec"] == "tied_ref" or m["name"] in seen:
                continue
            seen.add(m["name"])
            spans.append((int(m["offset"]), int(m["compressed_bytes"]), m["name"]))
        spans.sort()
        layout, dev_off = {}, 0
        for off, nb, name in spans:
            layout[name] = (off, dev_off, nb)
            dev_off += (nb + 15) // 16 * 16
        self.dev_data = torch.empty(max(16, dev_off), dtype=torch.uint8, device=self.device)
        self.layout = layout
        groups, cur = [], None
        for off, nb, name in spans:
            d = layout[name][1]
            if cur is None or (d + nb - cur.lo) > group_bytes:
                cur = _Group(lo=d, hi=d)
                groups.append(cur)
            cur.hi = d + nb
            cur.parts += [p for p in self.parts if p.name == name]
        self.groups = groups
        # host copy plan: contiguous device range per group may map to several
        # host blobs (they are not contiguous on the host if others are skipped)
        for g in groups:
            g.host_spans = [(layout[p.name][0], layout[p.name][1], layout[p.name][2])
                            for p in g.parts if p.meta["codec"] != "tied_ref"]
            xc_entries, xc_coders, xc_groups, se_entries = [], [], [], []
            for p in g.parts:
                m = p.meta
                _, d, nb = layout[p.name]
                blob = self.dev_data[d:d + nb]
                if m["codec"] == "bf16_exp_chunked_v1":
                    ce = int((m.get("extra") or {})["chunk_elems"])
                    out = self.out[p.name].reshape(-1).view(torch.int16)
                    xc_entries.append((blob, out, ce, _ct.n_elements(m["shape"]), p.chunk_begin, p.chunk_count))
                    xc_coders.append((m.get("extra") or {}).get("coder"))
                    xc_groups.append(gpu.extras_groups(m.get("extra")))
                elif m["codec"] in gpu.SERIAL_CODECS:
                    n = _ct.n_elements(m["shape"])
                    out = self.out[p.name].reshape(-1).view(torch.int16)
                    se_entries.append((m["codec"], bytes(self.image.blob_host(p.name)), blob, out, n))
                elif m["codec"] == "raw":
                    dst = self.out[p.name].reshape(-1).view(torch.uint8)
                    if dst.numel() != nb:
                        raise ValueError(f"raw tensor {p.name}: {nb} bytes for {dst.numel()}")
                    g.copies.append((dst, blob))
            if se_entries:   # serial-stream tensors of the group: one plan, all streams concurrent
                g.plans.append(gpu.SePlan(se_entries, device=self.device.index))
            if xc_entries:
                g.plans.insert(0, gpu.XcPlan(xc_entries, device=self.device.index, coders=xc_coders,
                                             groups=xc_groups))
            g.event = torch.cuda.Event()

    # -- run -------------------------------------------------------------------
    def h2d_bytes(self) -> int:
        return sum(nb for g in self.groups for (_, _, nb) in g.host_spans)

    def run_async(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Enqueue H2D copies (copy stream) and decodes (``stream``)."""
        stream = stream or torch.cuda.current_stream(self.device)
        host = self.image.host
        self.copy_stream.wait_stream(stream)   # do not overwrite blobs still being decoded
        for g in self.groups:
            with torch.cuda.stream(self.copy_stream):
                for hoff, doff, nb in g.host_spans:
                    self.dev_data[doff:doff + nb].copy_(host[hoff:hoff + nb], non_blocking=True)
                g.event.record(self.copy_stream)
            stream.wait_event(g.event)
            for pl in g.plans:
                pl.decode(stream)
            with torch.cuda.stream(stream):
                for dst, src in g.copies:
                    dst.copy_(src, non_blocking=True)

    def decode_async(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Decode from the device-resident compressed bytes only (no H2D)."""
        stream = stream or torch.cuda.current_stream(self.device)
        for g in self.groups:
            for pl in g.plans:
                pl.decode(stream)
            with torch.cuda.stream(stream):
                for dst, src in g.copies:
                    dst.copy_(src, non_blocking=True)

    def upload(self) -> None:
        """Copy all compressed bytes to the device once (for decode_async)."""
        host = self.image.host
        for g in self.groups:
            for hoff, doff, nb in g.host_spans:
                self.dev_data[doff:doff + nb].copy_(host[hoff:hoff + nb])
        torch.cuda.synchronize(self.device)

    def check(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Synchronise and raise if any device decoder flagged a stream error."""
        for g in self.groups:
            for pl in g.plans:
                pl.check(stream)

    def tensors(self) -> dict[str, torch.Tensor]:
        out = {}
        for p in self.parts:
            if p.meta["codec"] == "tied_ref":
                out[p.name] = self.out[(p.meta.get("extra") or {})["tied_to"]]
            else:
                out[p.name] = self.out[p.name]
        return out

    def run(self, stream=None) -> dict[str, torch.Tensor]:
        self.run_async(stream)
        self.check(stream)
        return self.tensors()

    def close(self):
        for g in self.groups:
            for pl in g.plans:
                pl.close()
            g.plans = []


def load_image(image: ContainerImage, device="cuda", names=None) -> dict[str, torch.Tensor]:
    """Decode a container image into device tensors (one pipelined pass)."""
    ld = DeviceLoader(image, device=device, owned=names)
    try:
        return ld.run()
    finally:
        ld.close()


class Bundle:
    """A reusable decode of a fixed set of tensors (from a resident container)
    into fixed output buffers: device plans plus device copies for raw tensors."""

    def __init__(self, plans: list, copies: list):
        self.plans = plans
        self.copies = copies

    def decode_after(self, stream: torch.cuda.Stream, wait=None, done=None) -> None:
        """``stream`` waits for event ``wait``, decodes, records ``done``; a
        bundle of one plan and no copies does this in one library call."""
        if len(self.plans) == 1 and not self.copies:
            self.plans[0].decode_after(stream, wait, done)
            return
        if wait is not None:
            stream.wait_event(wait)
        self.decode(stream)
        if done is not None:
            done.record(stream)

    def handoff_call(self, side: torch.cuda.Stream, release, done, next_ev=None):
        """A prepared ``f(main_stream)``: ``release`` recorded on the main
        stream, ``side`` waits for it, decodes, records ``done``, and the main
        stream waits for ``next_ev``; one library call for a bundle of one plan
        and no copies."""
        if len(self.plans) == 1 and not self.copies:
            return self.plans[0].handoff_call(side, release, done, next_ev)

        def call(main: torch.cuda.Stream) -> None:
            release.record(main)
            self.decode_after(side, release, done)
            if next_ev is not None:
                main.wait_event(next_ev)
        return call

    def decode(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        for pl in self.plans:
            pl.decode(stream)
        if self.copies:
            ctx = torch.cuda.stream(stream) if stream is not None else _nullctx()
            with ctx:
                for dst, src in self.copies:
                    dst.copy_(src, non_blocking=True)

    def check(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        for pl in self.plans:
            pl.check(stream)

    def close(self) -> None:
        for pl in self.plans:
            pl.close()
        self.plans = []


class _nullctx:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


class ResidentContainer:
    """The compressed data section of a container uploaded to HBM once.

    Any subset of its tensors can then be decoded, any number of times, into
    caller-provided device buffers (:meth:`bundle`) or fresh tensors
    (:meth:`decode`).  Only tensors stored with a device codec are accepted.
    """

    def __init__(self, image: ContainerImage, device=None):
        self.image = image
        self.device = torch.device("cuda", device if isinstance(device, int) else
                                   (torch.device(device).index if device is not None else torch.cuda.current_device()))
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.layout = {}
        pos = 0
        for t in image.header["tensors"]:
            if t["codec"] == "tied_ref":
                continue
            if t["codec"] not in DEVICE_CODECS:
                raise _unknown_codec(t["codec"])
            self.layout[t["name"]] = (int(t["offset"]), pos, int(t["compressed_bytes"]))
            pos += (int(t["compressed_bytes"]) + 15) // 16 * 16
        self.data = torch.empty(max(16, pos), dtype=torch.uint8, device=self.device)
        host = image.host
        for hoff, doff, nb in self.layout.values():
            if nb:
                self.data[doff:doff + nb].copy_(host[hoff:hoff + nb], non_blocking=True)
        torch.cuda.synchronize(self.device)

    def resolve(self, name: str) -> str:
        seen = set()
        while self.image.tensors[name]["codec"] == "tied_ref":
            if name in seen:
                raise ValueError(f"Tied-ref cycle at {name!r}")
            seen.add(name)
            name = (self.image.tensors[name].get("extra") or {})["tied_to"]
        return name

    def blob(self, name: str) -> torch.Tensor:
        _, d, nb = self.layout[self.resolve(name)]
        return self.data[d:d + nb]

    def empty_like(self, name: str) -> torch.Tensor:
        m = self.image.tensors[self.resolve(name)]
        return torch.empty(m["shape"] or [], dtype=TORCH_DTYPES.get(m["dtype"], torch.uint8), device=self.device)

    def bundle(self, outputs: dict, max_ctas: Optional[int] = None) -> Bundle:
        """outputs: {name: device tensor of the tensor's shape/dtype}.
        ``max_ctas`` caps the bf16_exp_chunked_v1 decode grid (see
        :meth:`bigsmall_b200.gpu.XcPlan.set_max_ctas`)."""
        xc, coders, groups, se, plans, copies = [], [], [], [], [], []
        for name, out in outputs.items():
            real = self.resolve(name)
            m = self.image.tensors[real]
            blob = self.blob(real)
            flat = out.reshape(-1)
            if m["codec"] == "bf16_exp_chunked_v1":
                xc.append((blob, flat.view(torch.int16), int((m.get("extra") or {})["chunk_elems"])))
                coders.append((m.get("extra") or {}).get("coder"))
                groups.append(gpu.extras_groups(m.get("extra")))
            elif m["codec"] in gpu.SERIAL_CODECS:
                se.append((m["codec"], bytes(self.image.blob_host(real)), blob, flat.view(torch.int16),
                           _ct.n_elements(m["shape"])))
            else:   # raw
                copies.append((flat.view(torch.uint8), blob))
        if se:
            plans.append(gpu.SePlan(se, device=self.device.index))
        if xc:
            plans.insert(0, gpu.XcPlan(xc, device=self.device.index, coders=coders, max_ctas=max_ctas,
                                       groups=groups))
        return Bundle(plans, copies)

    def decode(self, names, stream=None) -> dict:
        """Decode `names` into fresh tensors (synchronous, checked)."""
        outs = {n: self.empty_like(n) for n in names}
        b = self.bundle(outs)
        try:
            b.decode(stream)
            b.check(stream)
        finally:
            b.close()
        return outs
