"""Codec registry with the reference's contract (BigSmall
``bigsmall/codec_registry.py:38-55``): name -> (encode_fn, decode_fn).

Registered here: the device codecs of this package.  ``install_into`` adds
them to a reference ``bigsmall.codec_registry`` module so that
``verify_fast`` (``bigsmall/verify.py:124-139``) and encode-side selection
know the names.
"""
from __future__ import annotations

from typing import Callable, Optional

from .codecs import bf16_parallel, exp_chunked, se_legacy

_REGISTRY: dict[str, tuple[Callable, Callable]] = {}


def register_codec(name: str, encode_fn: Callable, decode_fn: Callable) -> None:
    _REGISTRY[name] = (encode_fn, decode_fn)


def get_codec(name: str) -> Optional[tuple[Callable, Callable]]:
    return _REGISTRY.get(name)


def registered_names() -> list[str]:
    return list(_REGISTRY)


def _enc_xc(raw, **ctx):
    return exp_chunked.encode(raw, **ctx)


def _dec_xc(blob, extras, n_weights):
    return exp_chunked.decode(blob, extras, n_weights)


def _dec_par(blob, extras, n_weights):
    return bf16_parallel.decode(blob, extras, n_weights)


register_codec(exp_chunked.CODEC, _enc_xc, _dec_xc)
register_codec(bf16_parallel.CODEC, bf16_parallel.encode, _dec_par)
for _name in se_legacy.CODECS:
    register_codec(_name, se_legacy.encode, se_legacy.decoder_for(_name))


def install_into(reference_registry, legacy: bool = False) -> None:
    """Register this package's codecs in a reference codec_registry module.
    The legacy serial formats are registered (device decode, the reference's
    encoder kept) only with ``legacy``."""
    for name, (enc, dec) in _REGISTRY.items():
        if name in se_legacy.CODECS and not legacy:
            continue
        if (name == bf16_parallel.CODEC or name in se_legacy.CODECS) and reference_registry.get_codec(name) is not None:
            enc = reference_registry.get_codec(name)[0]   # keep the reference encoder
        reference_registry.register_codec(name, enc, dec)
