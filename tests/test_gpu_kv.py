"""Device KV-cache compression (reference tests/test_kv_cache.py:15-119 shapes
and gates), plus the config-5 distribution: device encode == CPU oracle bytes,
device decode bit-exact."""
from __future__ import annotations

import hashlib
import struct

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import oracle as O  # noqa: E402


def _md5(t):
    return hashlib.md5(t.contiguous().view(torch.uint8).cpu().numpy().tobytes()).hexdigest()


def test_kv_roundtrip_lossless():
    from bigsmall_b200.kv_cache import compress_kv_entry, decompress_kv_entry
    torch.manual_seed(0)
    k = torch.randn(1, 32, 64, 96).to(torch.bfloat16)
    v = torch.randn(1, 32, 64, 96).to(torch.bfloat16)
    k2, v2 = decompress_kv_entry(compress_kv_entry(k, v), device="cuda")
    assert _md5(k) == _md5(k2) and _md5(v) == _md5(v2)
    assert k2.shape == k.shape and k2.is_cuda


def test_kv_ratio_below_75pct():
    from bigsmall_b200.kv_cache import compress_kv_entry
    torch.manual_seed(0)
    k = (torch.randn(1, 32, 512, 96) * 0.5).to(torch.bfloat16)
    v = (torch.randn(1, 32, 512, 96) * 0.5).to(torch.bfloat16)
    raw = 2 * k.numel() * 2
    assert len(compress_kv_entry(k, v)) / raw < 0.75


def test_compressed_kv_cache_api():
    from bigsmall_b200.kv_cache_manager import CompressedKVCache
    torch.manual_seed(1)
    c = CompressedKVCache(device="cuda")
    assert len(c) == 0 and c.compression_ratio() is None
    layers = {}
    for i in range(3):
        k = torch.randn(1, 8, 33 + i, 64, device="cuda").to(torch.bfloat16)
        v = torch.randn(1, 8, 33 + i, 64, device="cuda").to(torch.bfloat16)
        c.set(i, k, v)
        layers[i] = (k, v)
    k = torch.randn(1, 8, 40, 64, device="cuda").to(torch.bfloat16)
    c.set(1, k, k)          # overwrite a layer
    layers[1] = (k, k)
    assert len(c) == 3 and c.has(2) and not c.has(5)
    for i, (k, v) in layers.items():
        k2, v2 = c.get(i)
        assert torch.equal(k.view(torch.int16), k2.view(torch.int16))
        assert torch.equal(v.view(torch.int16), v2.view(torch.int16))
    assert 0 < c.compression_ratio() < 0.8
    assert c.raw_size() == sum(2 * (a.numel() + b.numel()) for a, b in layers.values())
    assert "CompressedKVCache(layers=3" in repr(c)
    with pytest.raises(KeyError):
        c.get(9)
    with pytest.raises(ValueError):
        c.set(0, k.float(), k)
    c.clear()
    assert len(c) == 0 and c.memory_usage() == 0


def test_config5_distribution_device_encoder_matches_oracle():
    from bigsmall_b200 import gpu
    from bigsmall_b200.kv_cache import KVEncoder, decode_kv
    g = torch.Generator().manual_seed(0)
    scale = torch.exp(torch.randn(1, 8, 1, 128, generator=g))
    k = (torch.randn(2, 8, 256, 128, generator=g) * scale).to(torch.bfloat16)
    raw = k.view(torch.uint8).numpy().tobytes()
    for coder, cid in (("pair", 2), ("rans", 0)):
        enc = KVEncoder(0, coder=coder)
        kb = enc.encode(k.cuda())
        assert kb.cpu().numpy().tobytes() == O.xc_encode(raw, cid, 12, gpu.DEFAULT_CHUNK_ELEMS), coder
        k2, _ = decode_kv(kb, kb, k.shape, k.shape, coder=coder)
        assert torch.equal(k2.cpu().view(torch.int16), k.view(torch.int16)), coder


def test_config5_full_tensor_encode_matches_oracle_and_decodes_exactly():
    """One whole config-5 K/V tensor, [16, 8, 8192, 128] = 16.8M values (N(0,1)
    times a per-channel log-normal scale, seed 0): the device encoder's blob
    equals the CPU oracle's byte for byte and the device decode is bit-exact
    (reference bigsmall/codecs/kv_cache.py:41-117 round-trips the same layout)."""
    from bigsmall_b200 import gpu
    from bigsmall_b200.kv_cache import KVEncoder, decode_kv
    g = torch.Generator().manual_seed(0)
    scale = torch.exp(torch.randn(1, 8, 1, 128, generator=g))
    k = (torch.randn(16, 8, 8192, 128, generator=g) * scale).to(torch.bfloat16)
    raw = k.view(torch.uint8).numpy().tobytes()
    kd = k.cuda()
    for coder, cid in (("pair", 2), ("rans", 0)):
        enc = KVEncoder(0, coder=coder)
        kb = enc.encode(kd)
        assert kb.cpu().numpy().tobytes() == O.xc_encode(raw, cid, 12, gpu.DEFAULT_CHUNK_ELEMS), coder
        k2, v2 = decode_kv(kb, kb, k.shape, k.shape, coder=coder)
        assert torch.equal(k2.view(torch.int16), kd.view(torch.int16)), coder
        assert torch.equal(v2.view(torch.int16), kd.view(torch.int16)), coder


def test_legacy_kv_versions_rejected_clearly():
    from bigsmall_b200.kv_cache import decompress_kv_entry
    blob = struct.pack("<BB", 2, 1) + struct.pack("<i", 4) + struct.pack("<I", 0)
    with pytest.raises(ValueError, match="constriction"):
        decompress_kv_entry(blob + blob[1:])
