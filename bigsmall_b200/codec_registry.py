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


def install_into(reference_registry, legacy: bool = False) -> dict:
    """Register this package's codecs in a reference codec_registry module.
    The legacy serial formats are registered (device decode, the reference's
    encoder kept) only with ``legacy``.  Returns {name: previous entry or None}
    for :func:`remove_from`."""
    previous = {}
    for name, (enc, dec) in _REGISTRY.items():
        if name in se_legacy.CODECS and not legacy:
            continue
        prev = reference_registry.get_codec(name)
        previous[name] = prev
        if (name == bf16_parallel.CODEC or name in se_legacy.CODECS) and prev is not None:
            enc = prev[0]   # keep the reference encoder
        reference_registry.register_codec(name, enc, dec)
    return previous


def remove_from(reference_registry, previous: dict) -> None:
    """Undo :func:`install_into`: entries that existed before get their
    original (encode, decode) pair back; names that did not exist are removed
    from the module's registry dict (the reference has no unregister call; its
    registry is the module-level ``_REGISTRY`` dict,
    bigsmall/codec_registry.py:42)."""
    table = getattr(reference_registry, "_REGISTRY", None)
    for name, prev in previous.items():
        if prev is not None:
            reference_registry.register_codec(name, prev[0], prev[1])
        elif isinstance(table, dict):
            table.pop(name, None)
