"""The integration hook wires the engine into a reference-shaped `bigsmall`
package: the `ac_cuda` backend slot, the `_decode_blob` dispatch and the codec
registry.  A stand-in package with the reference's module layout and
behaviour (unknown codec -> BigSmallVersionError; kernels probe caches) is
built here; no decoding runs (CPU only)."""
from __future__ import annotations

import sys
import types

import pytest


def _fake_reference():
    pkg = types.ModuleType("fakebs")
    pkg.__path__ = []
    dec = types.ModuleType("fakebs.decoder")

    class VersionError(Exception):
        pass

    def _decode_blob(t, blob):
        if t["codec"] == "raw":
            return blob
        raise VersionError(t["codec"])

    dec._decode_blob = _decode_blob
    dec.VersionError = VersionError
    kern = types.ModuleType("fakebs.kernels")
    kern._GPU_BACKEND = ""
    kern._GPU_DECODE_FN = None
    reg = types.ModuleType("fakebs.codec_registry")
    reg._R = {}
    reg.register_codec = lambda n, e, d: reg._R.__setitem__(n, (e, d))
    reg.get_codec = lambda n: reg._R.get(n)
    reg.register_codec("bf16_parallel_v1", "ref-encoder", "ref-decoder")
    stream = types.ModuleType("fakebs.streaming")
    stream._decode_blob = _decode_blob
    pkg.decoder, pkg.kernels, pkg.codec_registry, pkg.streaming = dec, kern, reg, stream
    for m in (pkg, dec, kern, reg, stream):
        sys.modules[m.__name__] = m
    return pkg


def test_install_and_uninstall(monkeypatch):
    from bigsmall_b200 import integration
    from bigsmall_b200 import decoder as gdec
    pkg = _fake_reference()
    calls = []
    monkeypatch.setattr(gdec, "_decode_blob", lambda t, b: calls.append(t["codec"]) or b"device")
    saved = integration.install(pkg)
    try:
        assert sys.modules["fakebs.kernels.ac_cuda"].decode.__module__ == "bigsmall_b200.kernels.ac_cuda"
        assert pkg.kernels._GPU_BACKEND is None          # probe re-runs and finds ac_cuda
        assert pkg.decoder._decode_blob({"codec": "bf16_exp_chunked_v1"}, b"x") == b"device"
        assert pkg.decoder._decode_blob({"codec": "bf16_parallel_v1"}, b"x") == b"device"
        assert pkg.streaming._decode_blob({"codec": "bf16_exp_chunked_v1"}, b"x") == b"device"
        assert pkg.decoder._decode_blob({"codec": "raw"}, b"r") == b"r"
        with pytest.raises(pkg.decoder.VersionError):
            pkg.decoder._decode_blob({"codec": "bf16_se_rans"}, b"")
        assert calls == ["bf16_exp_chunked_v1", "bf16_parallel_v1", "bf16_exp_chunked_v1"]
        enc, dec = pkg.codec_registry.get_codec("bf16_parallel_v1")
        assert enc == "ref-encoder" and dec is not None and dec != "ref-decoder"
        assert pkg.codec_registry.get_codec("bf16_exp_chunked_v1") is not None
    finally:
        integration.uninstall(pkg, saved)
        for n in [m for m in sys.modules if m.startswith("fakebs")]:
            del sys.modules[n]
    assert "fakebs.kernels.ac_cuda" not in sys.modules


@pytest.mark.parametrize("legacy_on_device", [False, True])
def test_legacy_formats_stay_on_the_reference_cpu_unless_asked(monkeypatch, legacy_on_device):
    from bigsmall_b200 import integration
    from bigsmall_b200 import decoder as gdec
    pkg = _fake_reference()
    pkg.codec_registry.register_codec("bf16_se_single_kernel", "ref-sk-enc", "ref-sk-dec")
    orig = pkg.decoder._decode_blob

    def ref_decode(t, blob):
        if t["codec"] == "bf16_se_single_kernel":
            return b"cpu"
        return orig(t, blob)

    pkg.decoder._decode_blob = ref_decode
    monkeypatch.setattr(gdec, "_decode_blob", lambda t, b: b"device")
    saved = integration.install(pkg, legacy_on_device=legacy_on_device)
    try:
        got = pkg.decoder._decode_blob({"codec": "bf16_se_single_kernel"}, b"x")
        assert got == (b"device" if legacy_on_device else b"cpu")
        enc, dec = pkg.codec_registry.get_codec("bf16_se_single_kernel")
        assert enc == "ref-sk-enc"
        assert (dec != "ref-sk-dec") == legacy_on_device
    finally:
        integration.uninstall(pkg, saved)
        for n in [m for m in sys.modules if m.startswith("fakebs")]:
            del sys.modules[n]
