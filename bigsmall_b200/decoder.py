"""Reference-shaped decoding API backed by the device engine.

Mirrors BigSmall ``bigsmall/decoder.py``:
  * ``_decode_blob(t, blob) -> bytes``  (``:49-97``) per-tensor dispatch;
  * ``decompress(src, dst=None) -> {name: np.ndarray}`` (``:100-157``);
  * ``load(src, device) -> {name: torch.Tensor}`` (``:301-310``) -- here the
    compressed bytes go to the device and are decoded there (no host decode,
    no host->device copy of decoded bytes);
  * ``verify(src)`` header-md5 verification (``bigsmall/verify.py:14-51``).

Codecs outside the device set raise ``BigSmallVersionError`` like the
reference does for names it does not know; there is no CPU decoder here.
"""
from __future__ import annotations

import hashlib
from typing import Optional

import numpy as np

from . import codec_registry
from . import container as _ct
from .codecs import bf16_parallel, exp_chunked, se_legacy
from .loader import ContainerImage, DeviceLoader, _unknown_codec

_DTYPE_TO_NUMPY = {
    "F32": np.float32, "float32": np.float32, "F16": np.float16, "float16": np.float16,
    "BF16": None, "bfloat16": None,   # numpy has no bf16: uint16 view, as the reference returns
    "F8_E4M3": np.uint8, "float8_e4m3fn": np.uint8, "F8_E5M2": np.uint8, "float8_e5m2": np.uint8,
    "I64": np.int64, "int64": np.int64, "I32": np.int32, "int32": np.int32,
    "I16": np.int16, "int16": np.int16, "I8": np.int8, "int8": np.int8,
    "U8": np.uint8, "uint8": np.uint8, "BOOL": np.bool_, "bool": np.bool_,
}


def _decode_blob(t: dict, blob: bytes) -> Optional[bytes]:
    """Decode one tensor blob to raw bytes (bigsmall/decoder.py:49-97 contract)."""
    extras = t.get("extra") or {}
    codec = t["codec"]
    n_weights = _ct.n_elements(t["shape"])
    if codec == "tied_ref":
        return None
    if codec == "raw":
        return bytes(blob)
    if codec == exp_chunked.CODEC:
        return exp_chunked.decode(bytes(blob), extras, n_weights)
    if codec == bf16_parallel.CODEC:
        return bf16_parallel.decode(bytes(blob), extras, n_weights)
    if codec in se_legacy.CODECS:
        return se_legacy.decoder_for(codec)(bytes(blob), extras, n_weights)
    pair = codec_registry.get_codec(codec)
    if pair is not None:
        return pair[1](bytes(blob), extras, n_weights)
    raise _unknown_codec(codec)


def _raw_to_numpy(raw: bytes, dtype_str: str, shape) -> np.ndarray:
    np_dtype = _DTYPE_TO_NUMPY.get(dtype_str) or np.uint16
    arr = np.frombuffer(raw, dtype=np_dtype)
    return arr.reshape(shape) if shape else arr


def decompress(src, dst=None, progress: bool = False, device="cuda") -> dict[str, np.ndarray]:
    """Decode a .bs file to host numpy arrays (device decode, one D2H per tensor)."""
    image = ContainerImage.from_file(src, pin=False)
    tensors = _decode_image(image, device)
    out = {}
    for t in image.header["tensors"]:
        arr = tensors[t["name"]].reshape(-1).view(__import__("torch").uint8).cpu().numpy().tobytes()
        out[t["name"]] = _raw_to_numpy(arr, t["dtype"], t["shape"])
    if dst is not None:
        _write_safetensors(dst, out, image.header)
    return out


def _decode_image(image: ContainerImage, device) -> dict:
    ld = DeviceLoader(image, device=device)
    try:
        return ld.run()
    finally:
        ld.close()


def load(src, device: str = "cuda", progress: bool = False) -> dict:
    """Decode a .bs file straight into device tensors (compressed bytes only
    cross PCIe)."""
    import torch
    image = ContainerImage.from_file(src, pin=True)
    dev = torch.device(device)
    if dev.type != "cuda":
        raise ValueError("bigsmall_b200.load decodes on a CUDA device; use decompress() for host arrays")
    return _decode_image(image, dev)


def _write_safetensors(dst, tensors: dict, header: dict) -> None:
    import torch
    from safetensors.torch import save_file
    tt = {}
    for m in header["tensors"]:
        arr = tensors[m["name"]]
        if m["dtype"] in ("BF16", "bfloat16"):
            tt[m["name"]] = torch.from_numpy(arr.astype(np.uint16, copy=False).copy().view(np.int16)).view(torch.bfloat16)
        else:
            tt[m["name"]] = torch.from_numpy(arr.copy())
    save_file(tt, str(dst))


def verify(src) -> bool:
    """Decode and compare every tensor's md5 with the header's (bigsmall/verify.py:44-51)."""
    out = decompress(src)
    header, _ = _ct.read_header(src)
    ok = True
    for m in header["tensors"]:
        if hashlib.md5(out[m["name"]].tobytes()).hexdigest() != m["md5"]:
            print(f"  MISMATCH {m['name']}")
            ok = False
    return ok


def compress_tensors(tensors: dict, dst=None, coder: Optional[str] = None, prec: int = 12,
                     chunk_elems: int = exp_chunked.gpu.DEFAULT_CHUNK_ELEMS, raw_tiny: int = 512,
                     with_md5: bool = True, groups: int = 1):
    """Encode a {name: torch.Tensor} dict into a container on the device.

    bf16 tensors of at least ``raw_tiny`` bytes use bf16_exp_chunked_v1 (the
    reference stores tensors under 512 bytes raw, bigsmall/encoder.py:57,
    :386-388); everything else is stored raw.  Returns the container bytes
    (and writes ``dst`` if given).
    """
    import torch
    from . import gpu
    coder = coder or gpu.DEFAULT_CODER
    w = _ct.ContainerWriter(fmt="bf16")
    enc = None
    for name, t in tensors.items():
        tt = t.detach().contiguous()
        raw_dtype = {torch.bfloat16: "BF16", torch.float16: "F16", torch.float32: "F32", torch.int64: "I64",
                     torch.int32: "I32", torch.int16: "I16", torch.int8: "I8", torch.uint8: "U8",
                     torch.bool: "BOOL"}[tt.dtype]
        nbytes = tt.numel() * tt.element_size()
        md5 = ""
        if with_md5:
            md5 = hashlib.md5(tt.reshape(-1).view(torch.uint8).cpu().numpy().tobytes()).hexdigest()
        if tt.dtype == torch.bfloat16 and nbytes >= raw_tiny:
            x = tt.reshape(-1).cuda()
            if enc is None or enc.max_elems < x.numel():
                enc = gpu.XcEncoder(x.numel(), chunk_elems, coder, prec, device=x.device.index, groups=groups)
            blob = enc.encode(x).cpu().numpy().tobytes()
            w.add(name, tt.shape, raw_dtype, exp_chunked.CODEC, blob, md5,
                  gpu.xc_extras(chunk_elems, coder, prec, groups))
        else:
            w.add(name, tt.shape, raw_dtype, "raw", tt.reshape(-1).view(torch.uint8).cpu().numpy().tobytes(), md5)
    if dst is not None:
        w.write(dst)
    return w.to_bytes()
