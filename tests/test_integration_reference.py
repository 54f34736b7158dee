"""The integration hook installed into the real reference package (CPU only).

Skipped unless the environment variable BIGSMALL_REFERENCE names a checkout of
the reference project (the directory that holds its ``bigsmall`` package).
The reference's optional native dependencies (constriction, zstandard, blosc2)
are replaced by empty stand-in modules, which the hook does not touch.  No
decoding runs: this checks the wiring against the reference's own modules
(bigsmall/decoder.py:49-97, bigsmall/streaming.py:22, bigsmall/migrate.py:36,
bigsmall/kernels/__init__.py:23-75, bigsmall/codec_registry.py:42-55).
"""
from __future__ import annotations

import os
import sys
import types

import pytest

REF = os.environ.get("BIGSMALL_REFERENCE", "")
pytestmark = pytest.mark.skipif(not os.path.isfile(os.path.join(REF, "bigsmall", "decoder.py")),
                                reason="BIGSMALL_REFERENCE does not name a reference checkout")


@pytest.fixture
def reference_pkg(monkeypatch):
    for m in ("constriction", "zstandard", "blosc2"):
        if m not in sys.modules:
            monkeypatch.setitem(sys.modules, m, types.ModuleType(m))
    monkeypatch.setenv("BIGSMALL_DISABLE_VERSION_CHECK", "1")
    monkeypatch.syspath_prepend(REF)
    before = set(sys.modules)
    import bigsmall
    import bigsmall.codec_registry  # noqa: F401
    import bigsmall.kernels  # noqa: F401  (the decoder imports it lazily)
    import bigsmall.migrate  # noqa: F401
    yield bigsmall
    for n in list(sys.modules):
        if n not in before and (n == "bigsmall" or n.startswith("bigsmall.")):
            del sys.modules[n]


def test_install_wires_every_insertion_point_and_uninstall_restores_them(reference_pkg):
    from bigsmall_b200 import integration
    from bigsmall_b200.kernels import ac_cuda
    bs = reference_pkg
    dec, stream, mig = sys.modules["bigsmall.decoder"], sys.modules["bigsmall.streaming"], sys.modules["bigsmall.migrate"]
    kern, reg = sys.modules["bigsmall.kernels"], sys.modules["bigsmall.codec_registry"]
    orig = dec._decode_blob
    assert stream._decode_blob is orig and mig._decode_blob is orig
    ref_par = reg.get_codec("bf16_parallel_v1")
    assert reg.get_codec("bf16_exp_chunked_v1") is None
    kern._GPU_BACKEND = ""                 # as after a CPU-only probe
    saved = integration.install(bs)
    try:
        for m in (dec, stream, mig):
            assert m._decode_blob is not orig and m._decode_blob.__wrapped__ is orig
        assert sys.modules["bigsmall.kernels.ac_cuda"] is ac_cuda and kern.ac_cuda is ac_cuda
        assert kern._GPU_BACKEND is None and kern._GPU_DECODE_FN is None   # the probe runs again
        assert reg.get_codec("bf16_exp_chunked_v1") is not None
        enc, dfn = reg.get_codec("bf16_parallel_v1")
        assert enc is ref_par[0] and dfn is not ref_par[1]   # reference encoder kept, device decoder
        # codecs the engine does not take still go to the reference's if-chain
        assert dec._decode_blob({"codec": "raw", "shape": [2], "extra": {}}, b"ab") == b"ab"
        with pytest.raises(bs.BigSmallVersionError):
            dec._decode_blob({"codec": "no_such_codec", "shape": [1], "extra": {}}, b"")
    finally:
        integration.uninstall(bs, saved)
    for m in (dec, stream, mig):
        assert m._decode_blob is orig
    assert "bigsmall.kernels.ac_cuda" not in sys.modules and not hasattr(kern, "ac_cuda")
    assert kern._GPU_BACKEND is None
    assert reg.get_codec("bf16_exp_chunked_v1") is None
    assert reg.get_codec("bf16_parallel_v1") == ref_par


def test_legacy_codecs_keep_the_reference_decoder_by_default(reference_pkg):
    from bigsmall_b200 import integration
    reg = sys.modules["bigsmall.codec_registry"]
    before = {n: reg.get_codec(n) for n in integration.LEGACY_CODECS}
    saved = integration.install(reference_pkg)
    try:
        assert {n: reg.get_codec(n) for n in integration.LEGACY_CODECS} == before
    finally:
        integration.uninstall(reference_pkg, saved)
    saved = integration.install(reference_pkg, legacy_on_device=True)
    try:
        for n in integration.LEGACY_CODECS:
            if before[n] is not None:
                assert reg.get_codec(n)[0] is before[n][0] and reg.get_codec(n)[1] is not before[n][1]
    finally:
        integration.uninstall(reference_pkg, saved)
    assert {n: reg.get_codec(n) for n in integration.LEGACY_CODECS} == before
