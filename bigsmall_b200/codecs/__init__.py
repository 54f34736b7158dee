"""Codec front-ends with the reference's per-codec contract:
``encode(raw: bytes, **ctx) -> (blob, extras)`` and
``decode(blob: bytes, extras: dict, n_weights: int) -> bytes``
(BigSmall ``bigsmall/codec_registry.py:38-41``).  Both run on the CUDA device."""
