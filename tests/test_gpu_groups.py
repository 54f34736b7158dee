"""GPU parity of bf16_exp_chunked_v1 blobs with several state groups per chunk
(format version 2): a chunk of `chunk_elems` values is cut into `groups`
independently decodable groups, so chunk size (framing) and the number of
warps decoding a tensor are separate choices.

Checker: the CPU oracle (encoder bytes, decoder output) and the raw input
bytes.  Integer/byte work: every comparison is bit-exact.
"""
from __future__ import annotations

import ctypes
import struct

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import oracle as O  # noqa: E402
from tests.conftest import golden_bytes  # noqa: E402


def _dev(b: bytes):
    return torch.from_numpy(np.frombuffer(b, dtype=np.uint8).copy()).cuda()


def _normal(n, seed, scale=0.02):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, generator=g) * scale).to(torch.bfloat16).view(torch.uint8).numpy().tobytes()


def _wide(n, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal(n) * np.exp(rng.standard_normal(n) * 3)).astype(np.float32)
    return (w.view(np.uint32) >> 16).astype(np.uint16).tobytes()


def _decode(blob: bytes, n: int, ce: int, groups: int, coder=None) -> bytes:
    from bigsmall_b200 import gpu
    out = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    gpu.decode_xc_into(_dev(blob), out, ce, coder=coder, groups=groups)
    return out.cpu().view(torch.uint8).numpy().tobytes()


@pytest.mark.parametrize("coder", [0, 1, 2])
@pytest.mark.parametrize("ce,groups", [(8192, 2), (65536, 8), (1 << 20, 32), (1 << 21, 64)])
def test_golden_inputs_decode_and_device_encoder_matches_oracle(manifest, coder, ce, groups):
    from bigsmall_b200 import gpu
    for name, c in manifest["cases"].items():
        raw = golden_bytes(f"{name}.raw")
        n = c["n"]
        blob = O.xc_encode(raw, coder, 12, ce, groups)
        assert _decode(blob, n, ce, groups) == raw, (name, coder, ce, groups)
        x = torch.from_numpy(np.frombuffer(raw, dtype=np.int16).copy()).cuda()
        dev_blob = gpu.encode_xc(x, coder=coder, chunk_elems=ce, groups=groups)
        assert dev_blob.cpu().numpy().tobytes() == blob, (name, coder, ce, groups)


@pytest.mark.parametrize("n", [1, 255, 257, 8191, 8193, 300_001, (1 << 21) + 513])
@pytest.mark.parametrize("coder", [0, 2])
def test_ragged_sizes(n, coder):
    raw = _wide(n, n) if n % 2 else _normal(n, n)
    for ce, groups in ((8192, 4), (1 << 20, 128)):
        assert _decode(O.xc_encode(raw, coder, 12, ce, groups), n, ce, groups) == raw, (n, ce, groups)


def test_chunk_ranges_of_a_grouped_tensor():
    """chunk_begin / chunk_count count chunks (of `groups` groups each): the
    ranges of a split tensor decode exactly their values, as multi-GPU
    ownership uses them."""
    from bigsmall_b200 import gpu
    n, ce, groups = 5 * (1 << 20) + 12345, 1 << 20, 16
    raw = _normal(n, 3)
    words = np.frombuffer(raw, dtype=np.int16)
    blob = _dev(O.xc_encode(raw, 2, 12, ce, groups))
    nc = -(-n // ce)
    for c0, cc in ((0, 1), (1, 2), (3, 0), (5, 1), (0, 0)):
        cnt = cc if cc else nc - c0
        lo, hi = c0 * ce, min(n, (c0 + cnt) * ce)
        out = torch.full((hi - lo,), -1, dtype=torch.int16, device="cuda")
        with gpu.XcPlan([(blob, out, ce, n, c0, cc)], groups=groups) as p:
            p.run()
        assert np.array_equal(out.cpu().numpy(), words[lo:hi]), (c0, cc)


def test_grouped_and_one_group_tensors_in_one_plan():
    from bigsmall_b200 import gpu
    specs = [(300_001, 2, 65536, 8), (40_000, 0, 4096, 1), (1 << 20, 1, 1 << 20, 32), (123_457, 2, 32768, 1),
             (70_001, 0, 1 << 18, 64)]
    entries, outs, raws, gs = [], [], [], []
    for i, (n, coder, ce, g) in enumerate(specs):
        raw = _wide(n, i) if i % 2 else _normal(n, i)
        out = torch.empty(n, dtype=torch.bfloat16, device="cuda")
        entries.append((_dev(O.xc_encode(raw, coder, 12, ce, g)), out, ce))
        outs.append(out)
        raws.append(raw)
        gs.append(g)
    with gpu.XcPlan(entries, groups=gs) as plan:
        for _ in range(2):
            for o in outs:
                o.fill_(0)
            plan.run()
            for raw, o in zip(raws, outs):
                assert o.cpu().view(torch.uint8).numpy().tobytes() == raw


def test_groups_mismatch_is_a_header_error_without_fault():
    """A descriptor whose groups disagree with the blob header fails with
    BS_DEV_HEADER (no decode, no fault); the context stays usable."""
    from bigsmall_b200 import gpu
    from bigsmall_b200.exceptions import BsCorruptError
    n = 200_003
    raw = _normal(n, 9)
    v2 = O.xc_encode(raw, 2, 12, 65536, 8)
    v1 = O.xc_encode(raw, 2, 12, 8192)
    # 8192 values per group either way: only the header's framing differs
    for blob, ce, groups in ((v2, 65536, 4), (v2, 8192, 1), (v1, 65536, 8), (v2, 131072, 16)):
        out = torch.empty(n, dtype=torch.bfloat16, device="cuda")
        with pytest.raises(BsCorruptError) as ei:
            gpu.decode_xc_into(_dev(blob), out, ce, groups=groups)
        assert ei.value.device_status[0] & 0x01, (ce, groups)
    assert _decode(v2, n, 65536, 8) == raw and _decode(v1, n, 8192, 1) == raw
    with pytest.raises(ValueError):          # 65536 / 3 is not a multiple of 256
        gpu.decode_xc_into(_dev(v2), torch.empty(n, dtype=torch.bfloat16, device="cuda"), 65536, groups=3)
    bad = bytearray(v2)
    struct.pack_into("<I", bad, 60, 1)       # reserved word after the group count
    with pytest.raises(BsCorruptError):
        gpu.decode_xc_into(_dev(bytes(bad)), torch.empty(n, dtype=torch.bfloat16, device="cuda"), 65536,
                           groups=8)


def test_container_with_grouped_tensors_loads_exactly():
    """The container path (header extra "groups") decodes grouped tensors."""
    from bigsmall_b200 import decoder
    from bigsmall_b200.loader import ContainerImage, DeviceLoader
    g = torch.Generator(device="cuda").manual_seed(5)
    w = {f"layer.{i}.weight": (torch.randn(shape, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
         for i, shape in enumerate([(1024, 1024), (3000, 77), (4096, 1024)])}
    img = ContainerImage.from_bytes(decoder.compress_tensors(w, chunk_elems=1 << 20, groups=32, with_md5=False))
    for m in img.header["tensors"]:
        assert m["extra"]["groups"] == 32 and m["extra"]["chunk_elems"] == 1 << 20
    ld = DeviceLoader(img, device=0)
    try:
        out = ld.run()
    finally:
        ld.close()
    for k, v in w.items():
        assert torch.equal(out[k].view(torch.int16), v.view(torch.int16)), k


def test_noalloc_entry_point_takes_grouped_tensors():
    from bigsmall_b200 import _lib
    n, ce, groups = 300_001, 1 << 17, 8
    raw = _normal(n, 12)
    blob = _dev(O.xc_encode(raw, 2, 12, ce, groups))
    out = torch.empty(n, dtype=torch.int16, device="cuda")
    arr = (_lib.XcTensor * 1)()
    arr[0].d_blob, arr[0].blob_bytes, arr[0].d_out, arr[0].n_elems = blob.data_ptr(), blob.numel(), out.data_ptr(), n
    arr[0].chunk_elems, arr[0].groups = ce, groups
    st = (ctypes.c_uint32 * 1)()
    rc = _lib.load().bs_xc_decode_noalloc(arr, 1, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), st)
    assert rc == 0 and st[0] == 0
    assert out.cpu().numpy().tobytes() == raw


@pytest.mark.parametrize("n,ce,groups", [((1 << 21) + 513, 65536, 8), (3 << 20, 1 << 20, 32)])
def test_device_encoder_matches_oracle_on_sampled_tensors(n, ce, groups):
    """From 2^20 values on the pair coder counts an eighth of the tensor; with
    state groups the device encoder still writes the oracle's bytes."""
    from bigsmall_b200 import gpu
    raw = _wide(n, 21) if n % 2 else _normal(n, 21)
    x = torch.from_numpy(np.frombuffer(raw, dtype=np.int16).copy()).cuda()
    dev_blob = gpu.encode_xc(x, coder=2, chunk_elems=ce, groups=groups)
    assert dev_blob.cpu().numpy().tobytes() == O.xc_encode(raw, 2, 12, ce, groups)
    assert _decode(dev_blob.cpu().numpy().tobytes(), n, ce, groups) == raw
