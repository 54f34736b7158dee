"""Device-resident compressed KV cache.

Same API as BigSmall ``bigsmall/kv_cache_manager.py:22-91`` (``set``, ``get``,
``has``, ``memory_usage``, ``raw_size``, ``compression_ratio``, ``clear``,
``len``).  The reference keeps compressed bytes in host RAM and runs a CPU
codec (its docstring measures ~17-26 MB/s, unusable in a live decode loop);
here each layer's K and V are encoded on the GPU into bf16_exp_chunked_v1 blobs
that stay in HBM, and ``get`` decodes both with one device plan.
"""
from __future__ import annotations

from typing import Optional

import torch

from .kv_cache import KVEncoder, decode_kv


class CompressedKVCache:
    def __init__(self, device: str = "cuda"):
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("CompressedKVCache keeps its blobs on a CUDA device")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self._enc = KVEncoder(self.device)
        self._store: dict[int, tuple] = {}
        self._raw: dict[int, int] = {}

    def set(self, layer_idx: int, keys, values) -> None:
        if keys.dtype != torch.bfloat16 or values.dtype != torch.bfloat16:
            raise ValueError("CompressedKVCache.set: keys and values must be BF16")
        kb, vb = self._enc.encode_pair(keys, values)
        self._store[layer_idx] = (kb, vb, tuple(keys.shape), tuple(values.shape))
        self._raw[layer_idx] = keys.element_size() * keys.numel() + values.element_size() * values.numel()

    def get(self, layer_idx: int, out: Optional[tuple] = None):
        if layer_idx not in self._store:
            raise KeyError(f"layer {layer_idx} not in CompressedKVCache")
        kb, vb, ks, vs = self._store[layer_idx]
        return decode_kv(kb, vb, ks, vs, device=self.device, out=out, coder=self._enc.coder)

    def has(self, layer_idx: int) -> bool:
        return layer_idx in self._store

    def memory_usage(self) -> int:
        """Device bytes held by the compressed blobs."""
        return sum(int(kb.numel()) + int(vb.numel()) for kb, vb, _, _ in self._store.values())

    def raw_size(self) -> int:
        return sum(self._raw.values())

    def compression_ratio(self) -> Optional[float]:
        raw = self.raw_size()
        return None if raw == 0 else self.memory_usage() / raw

    def clear(self) -> None:
        self._store.clear()
        self._raw.clear()

    def __len__(self) -> int:
        return len(self._store)

    def __repr__(self) -> str:
        cr = self.compression_ratio()
        cr_str = f"{cr * 100:.2f}%" if cr is not None else "n/a"
        return (f"CompressedKVCache(layers={len(self)} compressed={self.memory_usage() / 1e6:.2f}MB "
                f"raw={self.raw_size() / 1e6:.2f}MB ratio={cr_str})")
