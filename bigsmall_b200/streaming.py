"""Layer-at-a-time access to a container, decoded in HBM.

Same surface as BigSmall ``bigsmall/streaming.py:260-483`` ``StreamingLoader``
(``tensor_names``, ``layer_count``, ``layer_tensor_names``,
``non_layer_tensor_names``, ``load_tensor``, ``load_layer``,
``load_non_layer_tensors``, ``iter_layers``, context manager), with the same
layer-name rule (``:30-42``) and tied-reference resolution (``:163-181``).

The reference reads each blob from disk, decodes it on the CPU and copies
the decoded tensor to the device per call (``:158-191``).  Here the compressed
data section is uploaded to HBM once (:class:`~bigsmall_b200.loader.ResidentContainer`)
and every ``load_*`` call is a device decode.
"""
from __future__ import annotations

import re
from pathlib import Path
from typing import Iterator, Optional

import torch

from .loader import ContainerImage, ResidentContainer

_LAYER_RE = re.compile(r"(?:^|\.)(?:layers|h)\.(\d+)\.")


def layer_index(name: str) -> Optional[int]:
    m = _LAYER_RE.search(name)
    return int(m.group(1)) if m else None


class StreamingLoader:
    def __init__(self, path, device: str = "cuda", dtype=None):
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("StreamingLoader decodes on a CUDA device")
        self.dtype = dtype
        if isinstance(path, ContainerImage):
            image = path
            self.path = None
        else:
            self.path = Path(path)
            if self.path.is_dir():
                shards = sorted(self.path.glob("*.bs"))
                if len(shards) != 1:
                    raise FileNotFoundError(f"expected one .bs file in {self.path}, found {len(shards)}")
                self.path = shards[0]
            if not self.path.is_file():
                raise FileNotFoundError(f"Path not found: {self.path}")
            image = ContainerImage.from_file(self.path)
        self.image = image
        self.res = ResidentContainer(image, self.device)
        self._layers: dict[int, list[str]] = {}
        self._non_layer: list[str] = []
        for t in image.header["tensors"]:
            li = layer_index(t["name"])
            if li is None:
                self._non_layer.append(t["name"])
            else:
                self._layers.setdefault(li, []).append(t["name"])

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def close(self) -> None:
        self.res = None

    def tensor_names(self) -> list[str]:
        return list(self.image.tensors)

    def layer_count(self) -> int:
        return max(self._layers) + 1 if self._layers else 0

    def layer_tensor_names(self, layer_idx: int) -> list[str]:
        return list(self._layers.get(layer_idx, []))

    def non_layer_tensor_names(self) -> list[str]:
        return list(self._non_layer)

    def meta(self, name: str) -> dict:
        return self.image.tensors[name]

    def _cast(self, out: dict) -> dict:
        if self.dtype is not None:
            out = {k: (v.to(self.dtype) if v.is_floating_point() else v) for k, v in out.items()}
        return out

    def load_tensor(self, name: str) -> torch.Tensor:
        if name not in self.image.tensors:
            raise KeyError(f"Tensor {name!r} not in this BigSmall model")
        return self._cast(self.res.decode([name]))[name]

    def load_layer(self, layer_idx: int) -> dict:
        names = self._layers.get(layer_idx)
        if names is None:
            raise IndexError(f"Layer {layer_idx} not in this model (have {self.layer_count()} layers)")
        return self._cast(self.res.decode(names))

    def load_non_layer_tensors(self) -> dict:
        return self._cast(self.res.decode(self._non_layer)) if self._non_layer else {}

    def iter_layers(self, progress: bool = False) -> Iterator[tuple[int, dict]]:
        for i in sorted(self._layers):
            layer = self.load_layer(i)
            try:
                yield i, layer
            finally:
                layer.clear()
