"""GPU parity of coder 2 of bf16_exp_chunked_v1: rANS over exponent pairs
with a 15-exponent window and per-chunk escape bytes (sm_100a).

The checker is the CPU oracle (oracle/bs_oracle.c, ``xc2_*``); decode must
reproduce the raw bf16 bytes exactly and the device encoder must write the
oracle's bytes.  Integer/byte work: every comparison is bit-exact.
"""
from __future__ import annotations

import hashlib
import struct

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import oracle as O  # noqa: E402
from tests.conftest import golden_bytes  # noqa: E402


def _dev(b: bytes):
    return torch.from_numpy(np.frombuffer(b, dtype=np.uint8).copy()).cuda()


def _decode(blob: bytes, n: int, ce: int) -> bytes:
    from bigsmall_b200 import gpu
    out = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    gpu.decode_xc_into(_dev(blob), out, ce)
    return out.cpu().view(torch.uint8).numpy().tobytes()


def _normal(n, seed, scale=0.02) -> bytes:
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, generator=g) * scale).to(torch.bfloat16).view(torch.uint8).numpy().tobytes()


def _uniform(n, seed) -> bytes:
    return np.random.default_rng(seed).integers(0, 1 << 16, n, dtype=np.uint16).tobytes()


def _wide(n, seed) -> bytes:
    """Heavy-tailed values: a few percent of exponents fall outside any 15-wide window."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal(n) * np.exp(rng.standard_normal(n) * 3)).astype(np.float32)
    return (w.view(np.uint32) >> 16).astype(np.uint16).tobytes()


def test_decode_golden_inputs(manifest):
    for name, c in manifest["cases"].items():
        raw = golden_bytes(f"{name}.raw")
        for ce in (256, 65536):
            for prec in (11, 12):
                blob = O.xc_encode(raw, 2, prec, ce)
                assert hashlib.md5(_decode(blob, c["n"], ce)).hexdigest() == c["raw_md5"], (name, ce, prec)


@pytest.mark.parametrize("n", [1, 2, 3, 31, 255, 256, 257, 4095, 4097, 65535, 65536, 65537, 300_001])
def test_decode_ragged_sizes(n):
    for make in (_normal, _wide, _uniform):
        raw = make(n, n)
        for ce in (256, 32768, 65536):
            blob = O.xc_encode(raw, 2, 12, ce)
            assert _decode(blob, n, ce) == raw, (make.__name__, n, ce)


def test_device_encoder_matches_oracle_bytes(manifest):
    from bigsmall_b200 import gpu
    cases = [golden_bytes(f"{name}.raw") for name in manifest["cases"]]
    cases += [_normal(n, n) for n in (1, 3, 257, 65536, 200_003)]
    cases += [_wide(n, n) for n in (513, 100_001)]
    cases += [_uniform(70_001, 4)]
    for raw in cases:
        x = torch.from_numpy(np.frombuffer(raw, dtype=np.int16).copy()).view(torch.bfloat16).cuda()
        for ce in (256, 32768, 65536):
            for prec in (11, 12):
                d = gpu.encode_xc(x, coder="pair", prec=prec, chunk_elems=ce).cpu().numpy().tobytes()
                assert d == O.xc_encode(raw, 2, prec, ce), (len(raw) // 2, ce, prec)


def test_device_roundtrip_full_size_config1(manifest):
    from bigsmall_b200 import gpu
    from tests.golden.make_golden import c1_tensor
    full = manifest["full_size"]["c1"]
    x = c1_tensor().cuda()
    blob = gpu.encode_xc(x, coder="pair")
    out = torch.empty_like(x)
    gpu.decode_xc_into(blob, out, gpu.DEFAULT_CHUNK_ELEMS)
    assert hashlib.md5(out.cpu().view(torch.uint8).numpy().tobytes()).hexdigest() == full["raw_md5"]
    rans = gpu.encode_xc(x, coder="rans")
    # the pair coder spends at most a fraction of a percent more than per-exponent rANS
    assert blob.numel() <= rans.numel() * 1.005


def test_mixed_coders_in_one_plan():
    from bigsmall_b200 import gpu
    specs = [(300_001, 0, 65536), (40_000, 2, 256), (1, 2, 256), (123_457, 1, 4096), (65536 * 2, 2, 65536)]
    entries, outs, raws = [], [], []
    for i, (n, coder, ce) in enumerate(specs):
        raw = _wide(n, i) if i % 2 else _normal(n, i)
        blob = _dev(O.xc_encode(raw, coder, 12, ce))
        out = torch.empty(n, dtype=torch.bfloat16, device="cuda")
        entries.append((blob, out, ce))
        outs.append(out)
        raws.append(raw)
    with gpu.XcPlan(entries) as plan:
        for _ in range(2):
            for o in outs:
                o.fill_(0)
            plan.run()
            for raw, o in zip(raws, outs):
                assert o.cpu().view(torch.uint8).numpy().tobytes() == raw


def test_corrupt_pair_records_raise_without_fault():
    from bigsmall_b200 import gpu
    from bigsmall_b200.exceptions import BsCorruptError
    n = 100_000
    raw = _wide(n, 11)
    good = O.xc_encode(raw, 2, 12, 4096)
    co = struct.unpack_from("<Q", good, 32)[0]
    ne = struct.unpack_from("<I", good, co + 132)[0]
    assert ne > 0
    variants = {}
    b = bytearray(good); struct.pack_into("<I", b, 28, 250); variants["window"] = (bytes(b), 0x01)
    b = bytearray(good); struct.pack_into("<I", b, co + 132, ne - 1); variants["n_esc"] = (bytes(b), 0x08)
    b = bytearray(good); struct.pack_into("<I", b, co + 136, 1); variants["reserved"] = (bytes(b), 0x08)
    b = bytearray(good); b[co + 3] ^= 0x40; variants["lane_state"] = (bytes(b), 0x18)
    b = bytearray(good); struct.pack_into("<I", b, co + 128, 1 << 20); variants["n_words"] = (bytes(b), 0x08)
    # chunk 0's record cut to 128 bytes, shorter than its own 144-byte header
    b = bytearray(good); struct.pack_into("<I", b, 576 + 4, struct.unpack_from("<I", good, 576)[0] + 8)
    variants["short_record"] = (bytes(b), 0x08)
    for name, (blob, bits) in variants.items():
        out = torch.empty(n, dtype=torch.bfloat16, device="cuda")
        with pytest.raises(BsCorruptError) as ei:
            gpu.decode_xc_into(_dev(blob), out, 4096)
        st = ei.value.device_status[0]
        assert st and (st & bits), (name, hex(st))
    assert _decode(good, n, 4096) == raw


def test_coder_hint_selects_kernels_and_rejects_mismatch():
    """A plan given the blobs' coders launches only their decode kernels; a
    blob written with another coder fails with BS_DEV_HEADER, never skipped."""
    from bigsmall_b200 import gpu
    from bigsmall_b200.exceptions import BsCorruptError
    n = 70_001
    raw = _normal(n, 21)
    pair = O.xc_encode(raw, 2, 12, 4096)
    rans = O.xc_encode(raw, 0, 12, 4096)
    assert _decode(pair, n, 4096) == raw
    for blob, hint in ((pair, "pair"), (rans, "rans"), (pair, None), (rans, [None])):
        out = torch.empty(n, dtype=torch.bfloat16, device="cuda")
        with gpu.XcPlan([(_dev(blob), out, 4096)], coders=hint) as p:
            p.run()
        assert out.cpu().view(torch.uint8).numpy().tobytes() == raw, hint
    for blob, hint in ((pair, "rans"), (rans, "pair"), (pair, "tans")):
        out = torch.empty(n, dtype=torch.bfloat16, device="cuda")
        with pytest.raises(BsCorruptError) as ei:
            gpu.decode_xc_into(_dev(blob), out, 4096, coder=hint)
        assert ei.value.device_status[0] & 0x01, hint
    with pytest.raises(ValueError):
        gpu.XcPlan([(_dev(pair), torch.empty(n, dtype=torch.bfloat16, device="cuda"), 4096)], coders=["pair", "rans"])


@pytest.mark.parametrize("max_ctas", [1, 3, 150])
def test_capped_grid_walks_the_whole_work_list(max_ctas):
    """A plan capped at a few CTAs (bs_plan_set_max_ctas) still decodes every
    chunk of every tensor, for both decode kernels."""
    from bigsmall_b200 import gpu
    specs = [(300_001, 2, 65536), (40_000, 0, 256), (70_001, 2, 256), (123_457, 1, 4096)]
    entries, outs, raws = [], [], []
    for i, (n, coder, ce) in enumerate(specs):
        raw = _wide(n, 40 + i)
        entries.append((_dev(O.xc_encode(raw, coder, 12, ce)), torch.empty(n, dtype=torch.bfloat16, device="cuda"), ce))
        outs.append(entries[-1][1])
        raws.append(raw)
    with gpu.XcPlan(entries, max_ctas=max_ctas) as plan:
        for _ in range(2):
            for o in outs:
                o.fill_(0)
            plan.run()
            for raw, o in zip(raws, outs):
                assert o.cpu().view(torch.uint8).numpy().tobytes() == raw
        plan.set_max_ctas(0)
        plan.run()
        for raw, o in zip(raws, outs):
            assert o.cpu().view(torch.uint8).numpy().tobytes() == raw


def test_decode_timed_records_events_around_the_decode_kernels():
    from bigsmall_b200 import gpu
    n = 1_000_003
    raw = _normal(n, 77)
    out = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    with gpu.XcPlan([(_dev(O.xc_encode(raw, 2, 12, 65536)), out, 65536)], coders="pair") as p:
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        p.decode_timed(k0, k1)
        s1.record()
        p.check()
        assert 0 < k0.elapsed_time(k1) <= s0.elapsed_time(s1)
    assert out.cpu().view(torch.uint8).numpy().tobytes() == raw


@pytest.mark.parametrize("coder,name", [(0, "rans"), (1, "tans"), (2, "pair")])
@pytest.mark.parametrize("prec", [8, 10, 12])
def test_special_distributions_decode_and_device_encoder(coder, name, prec):
    """All-zero, NaN/Inf, subnormal, top-exponent (window base 241),
    two-cluster and many-rare-exponent tensors: device decode of oracle blobs and device encode,
    both bit-exact, at the format's small and default precisions."""
    from bigsmall_b200 import gpu
    from tests.test_oracle_xc import _special
    for kind in ("zeros", "nan_inf", "subnormal", "top_exponents", "two_clusters", "many_rare"):
        for n in (1, 300, 70_001):
            raw = _special(kind, n)
            blob = O.xc_encode(raw, coder, prec, 4096)
            assert _decode(blob, n, 4096) == raw, (kind, name, prec, n)
            x = torch.from_numpy(np.frombuffer(raw, dtype=np.int16).copy()).view(torch.bfloat16).cuda()
            d = gpu.encode_xc(x, coder=name, prec=prec, chunk_elems=4096).cpu().numpy().tobytes()
            assert d == blob, (kind, name, prec, n)


def test_handoff_call_chains_both_streams():
    """bs_plan_decode_handoff (the streaming prefetch's per-layer call): the
    side-stream decode follows the main stream's release point, and main-stream
    work enqueued after the call sees the decoded tensor."""
    from bigsmall_b200 import gpu
    n = 1_000_003
    raw = _normal(n, 21)
    blob = _dev(O.xc_encode(raw, 2, 12, 4096))
    out = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    main, side = torch.cuda.current_stream(), torch.cuda.Stream()
    rel, done = torch.cuda.Event(), torch.cuda.Event()
    with pytest.raises(ValueError):
        with gpu.XcPlan([(blob, out.view(torch.int16), 4096)], coders="pair") as p:
            p.handoff_call(side, rel, done, done)          # events not created yet
    for ev in (rel, done):
        ev.record(main)
    with gpu.XcPlan([(blob, out.view(torch.int16), 4096)], coders="pair") as p:
        call = p.handoff_call(side, rel, done, done)
        for _ in range(3):
            out.fill_(0)          # main-stream work the decode must follow
            call(main)
            got = out.clone()     # main-stream work after the hand-off's wait
            torch.cuda.synchronize()
            assert got.cpu().view(torch.uint8).numpy().tobytes() == raw
        p.check()


def test_tensor_past_2_32_values_round_trips():
    """Maximum size: one tensor of 2^32 + 1001 values (every element offset
    past 32 bits; odd, so the last pair is ragged), encoded and decoded on the
    device with the defaults, bit-exact, header count intact.  The reference's
    formats carry a u32 count; this one a u64.  About 40 GB of HBM."""
    from bigsmall_b200 import gpu
    free, _ = torch.cuda.mem_get_info()
    if free < 48 * 2 ** 30:
        pytest.skip("needs about 40 GB of free device memory")
    n = (1 << 32) + 1001
    x = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(7)
    step = 1 << 28
    for i in range(0, n, step):
        m = min(step, n - i)
        x[i:i + m] = (torch.randn(m, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    blob = gpu.encode_xc(x)
    assert struct.unpack_from("<Q", blob[:16].cpu().numpy().tobytes(), 8)[0] == n
    out = torch.empty_like(x)
    gpu.decode_xc_into(blob, out, gpu.DEFAULT_CHUNK_ELEMS)
    assert torch.equal(out.view(torch.int16), x.view(torch.int16))
    del x, out, blob
    torch.cuda.empty_cache()


def test_plan_counts_the_kernels_it_launches():
    """bs_plan_launch_count: the table build plus one decode kernel per coder
    family the plan may meet, per decode call (bench.py reports this count)."""
    from bigsmall_b200 import gpu
    n = 50_001
    raw = _normal(n, 5)
    pair, rans = _dev(O.xc_encode(raw, 2, 12, 4096)), _dev(O.xc_encode(raw, 0, 12, 4096))
    outs = [torch.empty(n, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    with gpu.XcPlan([(pair, outs[0], 4096), (rans, outs[1], 4096)], coders=["pair", "rans"]) as p:
        assert p.launch_count() == 0
        p.run()
        assert p.launch_count() == 3
        for _ in range(4):
            p.decode()
        p.check()
        assert p.launch_count() == 15
    with gpu.XcPlan([(pair, outs[0], 4096)], coders="pair") as p:
        p.run()
        p.run()
        assert p.launch_count() == 4
    for o in outs:
        assert o.cpu().view(torch.uint8).numpy().tobytes() == raw


@pytest.mark.parametrize("lead_scale", [None, 1e-6, 1e3])
def test_device_encoder_on_tensors_whose_scale_changes(lead_scale):
    """A tensor whose first 65,536 values have a far smaller or larger scale
    than the rest (so its exponents fall in two distant windows): the pair
    coder's device blob equals the CPU encoder's byte for byte, with one and
    with four state groups per chunk, and decodes exactly."""
    from bigsmall_b200 import gpu
    g = torch.Generator().manual_seed(17)
    body = torch.randn(1_000_003, generator=g)
    if lead_scale is not None:
        body = torch.cat([torch.randn(65_536, generator=g) * lead_scale, body])
    x = body.to(torch.bfloat16)
    raw = x.view(torch.uint8).numpy().tobytes()
    for ce, groups in ((32768, 1), (65536, 4)):
        blob = gpu.encode_xc(x.cuda(), coder="pair", chunk_elems=ce, groups=groups)
        assert blob.cpu().numpy().tobytes() == O.xc_encode(raw, 2, 12, ce, groups), (lead_scale, ce)
        assert _decode_g(blob, x.numel(), ce, groups) == raw


def _decode_g(blob, n, ce, groups):
    from bigsmall_b200 import gpu
    out = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    gpu.decode_xc_into(blob, out, ce, groups=groups)
    return out.cpu().view(torch.uint8).numpy().tobytes()


def test_event_chained_decode_runs_as_one_captured_graph():
    """bs_plan_decode_after runs the plan's table build and decode kernels as
    one CUDA graph (captured on first use, again after the CTA cap changes):
    outputs stay exact, events order it against the caller's stream, and the
    plan's launch count still counts both kernels per decode."""
    from bigsmall_b200 import gpu
    n = 500_001
    raw = _normal(n, 8)
    blob = _dev(O.xc_encode(raw, 2, 12, 4096))
    out = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    main = torch.cuda.current_stream()
    side = torch.cuda.Stream()
    go, done = torch.cuda.Event(), torch.cuda.Event()   # created by decode_after on first use
    with gpu.XcPlan([(blob, out, 4096)], coders="pair") as p:
        for k, cap in enumerate((0, 0, 3, 3, 0)):
            p.set_max_ctas(cap)
            out.fill_(0)
            go.record(main)
            p.decode_after(side, go, done)
            main.wait_event(done)
            assert out.cpu().view(torch.uint8).numpy().tobytes() == raw, (k, cap)
            assert p.launch_count() == 2 * (k + 1)
        p.check()


def test_event_chained_decode_inside_a_callers_graph_capture():
    """A plan's first event-chained decode issued while the caller captures
    its own CUDA graph (torch.cuda.graph, global capture mode): the library
    either nests its captured graph or, where it cannot capture, launches the
    kernels one by one into the caller's capture; replaying the caller's
    graph decodes exactly either way."""
    from bigsmall_b200 import gpu
    n = 300_001
    raw = _normal(n, 9)
    blob = _dev(O.xc_encode(raw, 2, 12, 4096))
    out = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    with gpu.XcPlan([(blob, out, 4096)], coders="pair") as p:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            p.decode_after(s)
        for _ in range(2):
            out.fill_(0)
            torch.cuda.synchronize()
            g.replay()
            torch.cuda.synchronize()
            assert out.cpu().view(torch.uint8).numpy().tobytes() == raw
        p.check()


def test_device_encoder_when_the_sample_is_unlike_the_rest():
    """The pair coder's statistics come from every eighth 2048-value block of a
    tensor of 2^20 values or more; with those blocks all zeros the device
    encoder still equals the oracle's bytes and decodes exactly."""
    from bigsmall_b200 import gpu
    n = (1 << 20) + 4097
    g = torch.Generator(device="cuda").manual_seed(11)
    x = (torch.randn(n, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    idx = torch.arange(n, device="cuda")
    x[((idx >> 11) & 7) == 0] = 0
    blob = gpu.encode_xc(x, coder=2, chunk_elems=32768)
    raw = x.cpu().view(torch.uint8).numpy().tobytes()
    assert blob.cpu().numpy().tobytes() == O.xc_encode(raw, 2, 12, 32768)
    out = torch.empty_like(x)
    gpu.decode_xc_into(blob, out, 32768)
    assert torch.equal(out.view(torch.int16), x.view(torch.int16))
