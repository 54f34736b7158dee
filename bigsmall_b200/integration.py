"""Install this engine behind an imported reference ``bigsmall`` package.

The three insertion points (BigSmall paths):
  * ``bigsmall/kernels/__init__.py:56-64`` imports ``bigsmall.kernels.ac_cuda``
    first and calls ``ac_cuda.decode(blob, extras, n) -> bytes`` for
    bf16_parallel_v1 -> this package's ``kernels.ac_cuda`` module is placed at
    that module name and the backend probe cache is reset;
  * ``bigsmall/decoder.py:49-97`` ``_decode_blob`` is an if-chain that raises
    for codec names it does not know -> it is wrapped so bf16_exp_chunked_v1
    (and bf16_parallel_v1) decode on the device, everything else is passed to
    the original function;
  * ``bigsmall/codec_registry.py:45-47`` ``register_codec`` -> the codec names
    are registered so ``verify_fast`` and encode-side selection know them.
``StreamingLoader`` (``bigsmall/streaming.py:22,181``) and the format migration
tool (``bigsmall/migrate.py:36,134``) import ``_decode_blob`` by name, so their
module attributes are patched too.
"""
from __future__ import annotations

import sys
import types

from . import codec_registry as _reg
from . import decoder as _dec
from .kernels import ac_cuda as _ac_cuda

DEVICE_CODECS = ("bf16_exp_chunked_v1", "bf16_parallel_v1")
# the reference's serial formats; their device decode is bit-exact but one
# serial stream per tensor, slower than the reference's CPU decoder per tensor
LEGACY_CODECS = ("bf16_se_single_kernel", "bf16_se_tans")


def install(bigsmall_pkg, legacy_on_device: bool = False) -> dict:
    """Wire the device engine into an imported reference package.  Returns the
    original callables so :func:`uninstall` can restore them.  With
    ``legacy_on_device`` the legacy serial formats decode on the device too
    (no CPU work; useful when host cores are busy); otherwise they keep the
    reference's CPU decoders."""
    name = bigsmall_pkg.__name__
    saved = {}
    device_codecs = DEVICE_CODECS + (LEGACY_CODECS if legacy_on_device else ())
    # 1. backend slot
    kern = sys.modules.get(f"{name}.kernels") or getattr(bigsmall_pkg, "kernels", None)
    sys.modules[f"{name}.kernels.ac_cuda"] = _ac_cuda
    if kern is not None:
        saved["ac_cuda"] = getattr(kern, "ac_cuda", None)
        kern.ac_cuda = _ac_cuda
        for attr, val in (("_GPU_BACKEND", None), ("_GPU_DECODE_FN", None)):
            if hasattr(kern, attr):
                setattr(kern, attr, val)
    # 2. dispatch
    dec = sys.modules.get(f"{name}.decoder") or getattr(bigsmall_pkg, "decoder")
    orig = dec._decode_blob
    saved["_decode_blob"] = orig

    def _decode_blob(t, blob):
        if t.get("codec") in device_codecs:
            return _dec._decode_blob(t, blob)
        return orig(t, blob)

    _decode_blob.__wrapped__ = orig
    dec._decode_blob = _decode_blob
    for mod_name in (f"{name}.streaming", f"{name}.migrate"):
        m = sys.modules.get(mod_name)
        if isinstance(m, types.ModuleType) and getattr(m, "_decode_blob", None) is orig:
            saved[mod_name] = orig
            m._decode_blob = _decode_blob
    # 3. registry
    reg = sys.modules.get(f"{name}.codec_registry") or getattr(bigsmall_pkg, "codec_registry", None)
    if reg is not None:
        saved["registry"] = _reg.install_into(reg, legacy=legacy_on_device)
    return saved


def uninstall(bigsmall_pkg, saved: dict) -> None:
    name = bigsmall_pkg.__name__
    dec = sys.modules.get(f"{name}.decoder") or getattr(bigsmall_pkg, "decoder")
    dec._decode_blob = saved["_decode_blob"]
    kern = sys.modules.get(f"{name}.kernels") or getattr(bigsmall_pkg, "kernels", None)
    if kern is not None:
        if saved.get("ac_cuda") is None:
            if hasattr(kern, "ac_cuda"):
                delattr(kern, "ac_cuda")
            sys.modules.pop(f"{name}.kernels.ac_cuda", None)
        else:
            kern.ac_cuda = saved["ac_cuda"]
            sys.modules[f"{name}.kernels.ac_cuda"] = saved["ac_cuda"]
    for mod_name, fn in saved.items():
        if mod_name.endswith((".streaming", ".migrate")) and mod_name in sys.modules:
            sys.modules[mod_name]._decode_blob = fn
    reg = sys.modules.get(f"{name}.codec_registry") or getattr(bigsmall_pkg, "codec_registry", None)
    if reg is not None and "registry" in saved:
        _reg.remove_from(reg, saved["registry"])
    if kern is not None:
        for attr in ("_GPU_BACKEND", "_GPU_DECODE_FN"):   # the next probe runs afresh
            if hasattr(kern, attr):
                setattr(kern, attr, None)
