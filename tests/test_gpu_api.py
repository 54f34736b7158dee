"""Reference-shaped API on the device: container -> HBM, _decode_blob, the
ac_cuda backend slot and the codec registry (BigSmall bigsmall/decoder.py,
bigsmall/kernels/__init__.py, bigsmall/codec_registry.py contracts)."""
from __future__ import annotations

import hashlib

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import oracle as O  # noqa: E402
from tests.conftest import golden_bytes  # noqa: E402


def _model(seed=0):
    g = torch.Generator().manual_seed(seed)
    return {
        "model.embed_tokens.weight": (torch.randn(1000, 64, generator=g) * 0.02).to(torch.bfloat16),
        "model.layers.0.input_layernorm.weight": (1 + torch.randn(64, generator=g) * 0.01).to(torch.bfloat16),
        "model.layers.0.self_attn.q_proj.weight": (torch.randn(64, 64, generator=g) / 8).to(torch.bfloat16),
        "model.layers.1.mlp.up_proj.weight": (torch.randn(300, 64, generator=g) / 8).to(torch.bfloat16),
        "model.layers.1.tiny.bias": (torch.randn(7, generator=g)).to(torch.bfloat16),
        "model.positions": torch.arange(10, dtype=torch.int64),
    }


def test_compress_load_decompress_verify(tmp_path):
    from bigsmall_b200 import decoder
    sd = _model()
    p = tmp_path / "m.bs"
    decoder.compress_tensors(sd, p, chunk_elems=4096)
    out = decoder.load(p, device="cuda")
    for k, v in sd.items():
        assert out[k].dtype == v.dtype and tuple(out[k].shape) == tuple(v.shape)
        assert torch.equal(out[k].cpu().view(torch.uint8), v.view(torch.uint8)), k
    host = decoder.decompress(p)
    for k, v in sd.items():
        assert host[k].tobytes() == v.view(torch.uint8).numpy().tobytes()
    assert decoder.verify(p)


def test_loader_pipelined_groups_and_tied(tmp_path):
    from bigsmall_b200 import container as C, gpu
    from bigsmall_b200.loader import ContainerImage, DeviceLoader
    sd = _model(1)
    w = C.ContainerWriter()
    for k, v in sd.items():
        if v.dtype == torch.bfloat16 and v.numel() >= 256:
            blob = gpu.encode_xc(v.reshape(-1).cuda(), chunk_elems=256).cpu().numpy().tobytes()
            w.add(k, v.shape, "BF16", "bf16_exp_chunked_v1", blob, "", gpu.xc_extras(256))
        else:
            raw = v.reshape(-1).view(torch.uint8).numpy().tobytes()
            w.add(k, v.shape, {torch.bfloat16: "BF16", torch.int64: "I64"}[v.dtype], "raw", raw, "")
    # a bf16_parallel_v1 tensor from the reference format and a tied alias
    raw = golden_bytes("gauss_8k.raw")
    w.add("ref.par", [8192], "BF16", "bf16_parallel_v1", O.par_encode(raw, 32), "", {"n_streams": 32})
    w.add("lm_head.weight", [1000, 64], "BF16", "tied_ref", b"", "", {"tied_to": "model.embed_tokens.weight"})
    img = ContainerImage.from_bytes(w.to_bytes())
    ld = DeviceLoader(img, device=0, group_bytes=20_000)   # many small groups
    assert len(ld.groups) > 3
    for _ in range(2):
        out = ld.run()
    for k, v in sd.items():
        assert torch.equal(out[k].cpu().view(torch.uint8), v.view(torch.uint8)), k
    assert out["ref.par"].cpu().view(torch.uint8).numpy().tobytes() == raw
    assert out["lm_head.weight"].data_ptr() == out["model.embed_tokens.weight"].data_ptr()
    ld.close()


@pytest.mark.parametrize("ce,groups", [(256, 1), (1024, 4)])
def test_ranks_shares_cover_the_container(tmp_path, ce, groups):
    """sharding.owned_for + DeviceLoader(owned=...) for every rank of 2- and
    3-way partitions, run one after another on one GPU: chunked tensors split
    by chunk spans (chunks of one or of four state groups), raw /
    bf16_parallel_v1 tensors whole on one rank, tied aliases on none; together
    the ranks' outputs reproduce every tensor once."""
    from bigsmall_b200 import container as C, gpu
    from bigsmall_b200.loader import ContainerImage, DeviceLoader
    from bigsmall_b200.sharding import owned_for
    sd = _model(2)
    w = C.ContainerWriter()
    for k, v in sd.items():
        if v.dtype == torch.bfloat16 and v.numel() >= 256:
            blob = gpu.encode_xc(v.reshape(-1).cuda(), chunk_elems=ce, groups=groups).cpu().numpy().tobytes()
            w.add(k, v.shape, "BF16", "bf16_exp_chunked_v1", blob, "", gpu.xc_extras(ce, groups=groups))
        else:
            raw = v.reshape(-1).view(torch.uint8).numpy().tobytes()
            w.add(k, v.shape, {torch.bfloat16: "BF16", torch.int64: "I64"}[v.dtype], "raw", raw, "")
    raw = golden_bytes("gauss_8k.raw")
    w.add("ref.par", [8192], "BF16", "bf16_parallel_v1", O.par_encode(raw, 32), "", {"n_streams": 32})
    w.add("lm_head.weight", [1000, 64], "BF16", "tied_ref", b"", "", {"tied_to": "model.embed_tokens.weight"})
    img = ContainerImage.from_bytes(w.to_bytes())
    want = {k: v.reshape(-1).view(torch.uint8).numpy().tobytes() for k, v in sd.items()}
    want["ref.par"] = raw
    for world in (2, 3):
        got = {k: bytearray(len(b)) for k, b in want.items()}
        seen = {k: 0 for k in want}
        for rank in range(world):
            owned = owned_for(img.header, rank, world)
            assert all(name != "lm_head.weight" for name, _, _ in owned)
            ld = DeviceLoader(img, device=0, owned=owned)
            out = ld.run()
            for name, c0, cc in owned:
                b = out[name].reshape(-1).cpu().view(torch.uint8).numpy().tobytes()
                lo = 2 * ce * c0 if cc else 0
                got[name][lo:lo + len(b)] = b
                seen[name] += len(b)
            ld.close()
        for k in want:
            assert seen[k] == len(want[k]) and bytes(got[k]) == want[k], (world, k)


def test_unknown_codec_raises_version_error():
    from bigsmall_b200 import decoder
    from bigsmall_b200.exceptions import BigSmallVersionError
    with pytest.raises(BigSmallVersionError):
        decoder._decode_blob({"codec": "bf16_se_rans", "shape": [4], "extra": None}, b"1234")
    assert decoder._decode_blob({"codec": "raw", "shape": [2], "extra": None}, b"abcd") == b"abcd"
    assert decoder._decode_blob({"codec": "tied_ref", "shape": [2], "extra": None}, b"") is None


def test_ac_cuda_slot_and_registry(manifest):
    from bigsmall_b200 import codec_registry, kernels
    from bigsmall_b200.kernels import ac_cuda
    kernels._GPU_BACKEND = None          # re-probe, as the reference's tests do
    kernels._GPU_DECODE_FN = None
    assert kernels.use_gpu() is True and kernels.backend_name() == "cuda_c"
    c = manifest["cases"]["edge"]
    blob = golden_bytes(c["blobs"]["par128"]["file"])
    out = ac_cuda.decode(blob, {"n_streams": 128}, c["n"])
    assert hashlib.md5(out).hexdigest() == c["raw_md5"]
    assert kernels.decode_bf16_parallel(blob, {}, c["n"]) == out
    dev = ac_cuda.decode_to_device(blob, {"n_streams": 128}, c["n"])
    assert dev.is_cuda and dev.cpu().numpy().tobytes() == out
    enc, dec = codec_registry.get_codec("bf16_exp_chunked_v1")
    raw = golden_bytes("c1_head_16k.raw")
    b, extras = enc(raw, chunk_elems=4096)
    assert extras["coder"] == "pair"
    assert b == O.xc_encode(raw, 2, 12, 4096) and dec(b, extras, len(raw) // 2) == raw
    b0, extras0 = enc(raw, chunk_elems=4096, coder="rans")
    assert b0 == O.xc_encode(raw, 0, 12, 4096) and dec(b0, extras0, len(raw) // 2) == raw
    assert "bf16_parallel_v1" in codec_registry.registered_names()


def test_empty_tensors_on_every_path():
    """Zero-element tensors (the reference's codecs return b'' for them,
    bigsmall/codecs/bf16_parallel.py:270-271): the codec calls, a plan that
    mixes them with real tensors, a container holding one, and the KV cache."""
    from bigsmall_b200 import decoder, gpu
    from bigsmall_b200.codecs import bf16_parallel, exp_chunked
    from bigsmall_b200.kv_cache import compress_kv_entry, decompress_kv_entry
    from bigsmall_b200.loader import ContainerImage, DeviceLoader
    assert exp_chunked.decode(b"", gpu.xc_extras(), 0) == b""
    assert bf16_parallel.decode(b"", {"n_streams": 32}, 0) == b""
    blob, extras = exp_chunked.encode(b"")
    assert blob == b"" and extras["chunk_elems"] == gpu.DEFAULT_CHUNK_ELEMS
    x = (torch.randn(70_001) * 0.02).to(torch.bfloat16).cuda()
    b = gpu.encode_xc(x)
    empty_blob = torch.empty(0, dtype=torch.uint8, device="cuda")
    out, none = torch.empty_like(x), torch.empty(0, dtype=torch.bfloat16, device="cuda")
    with gpu.XcPlan([(empty_blob, none, 4096), (b, out, gpu.DEFAULT_CHUNK_ELEMS), (empty_blob, none, 256)]) as p:
        p.run()
        assert p.check() == [0, 0, 0]
    assert torch.equal(out.view(torch.int16), x.view(torch.int16))
    w = {"a.weight": x.cpu().reshape(70_001), "empty.weight": torch.empty(0, dtype=torch.bfloat16),
         "b.weight": torch.empty(0, 4, dtype=torch.bfloat16)}
    img = ContainerImage.from_bytes(decoder.compress_tensors(w, with_md5=False))
    ld = DeviceLoader(img, device=0)
    try:
        got = ld.run()
    finally:
        ld.close()
    assert torch.equal(got["a.weight"].cpu().view(torch.int16), w["a.weight"].view(torch.int16))
    assert got["empty.weight"].numel() == 0 and tuple(got["b.weight"].shape) == (0, 4)
    k = torch.empty(1, 8, 0, 64, dtype=torch.bfloat16)
    k2, v2 = decompress_kv_entry(compress_kv_entry(k, k), device="cuda")
    assert tuple(k2.shape) == (1, 8, 0, 64) and tuple(v2.shape) == (1, 8, 0, 64)


def test_tiny_tensors_stored_raw_at_the_reference_threshold(tmp_path):
    """Tensors under 512 bytes go raw, stored at their exact byte count; a bf16
    tensor of exactly 512 bytes takes the codec (reference
    tests/test_raw_tiny.py:30-110, bigsmall/encoder.py:57, :386-388)."""
    from bigsmall_b200 import decoder
    from bigsmall_b200.container import parse_header
    g = torch.Generator().manual_seed(0)
    w = {"tiny.bias": torch.randn(128, generator=g).to(torch.bfloat16),
         "very_tiny.scale": torch.tensor([1.5, -0.25], dtype=torch.float32),
         "norm.weight": torch.randn(2048, generator=g).to(torch.bfloat16),
         "matrix.weight": torch.randn(512, 512, generator=g).to(torch.bfloat16),
         "at_threshold.weight": torch.zeros(256, dtype=torch.bfloat16),
         "below_threshold.weight": torch.zeros(255, dtype=torch.bfloat16)}
    data = decoder.compress_tensors(w, tmp_path / "t.bs")
    header = parse_header(data)[0]
    codec = {t["name"]: t["codec"] for t in header["tensors"]}
    size = {t["name"]: int(t["compressed_bytes"]) for t in header["tensors"]}
    assert codec["tiny.bias"] == "raw" and size["tiny.bias"] == 256
    assert codec["very_tiny.scale"] == "raw" and size["very_tiny.scale"] == 8
    assert codec["below_threshold.weight"] == "raw"
    for n in ("norm.weight", "matrix.weight", "at_threshold.weight"):
        assert codec[n] == "bf16_exp_chunked_v1", n
    out = decoder.load(tmp_path / "t.bs", device="cuda")
    for k, v in w.items():
        got = out[k].cpu().contiguous().view(torch.uint8).numpy().tobytes()
        assert hashlib.md5(got).hexdigest() == hashlib.md5(v.view(torch.uint8).numpy().tobytes()).hexdigest(), k
