"""Property tests of the bf16_exp_chunked_v1 format on the CPU oracle (the
reference's property-test style, bigsmall tests/test_property_based.py:80-202,
applied to this project's format): any bf16 tensor, any coder, precision and
chunk size round-trips exactly, and the coded size stays within a small
margin of the exponent entropy (the reference's ratio gates,
tests/test_rans.py:52-62, restated for this format)."""
from __future__ import annotations

import math

import numpy as np
import pytest

hyp = pytest.importorskip("hypothesis")
from hypothesis import given, settings, strategies as st  # noqa: E402

from oracle import oracle as O  # noqa: E402


@st.composite
def bf16_tensors(draw):
    n = draw(st.integers(min_value=1, max_value=5000))
    kind = draw(st.sampled_from(["normal", "uniform_words", "few_values", "wide"]))
    seed = draw(st.integers(min_value=0, max_value=2 ** 31 - 1))
    rng = np.random.default_rng(seed)
    if kind == "normal":
        w = (rng.standard_normal(n).astype(np.float32) * draw(st.sampled_from([1e-3, 0.02, 1.0, 300.0])))
        words = (w.view(np.uint32) >> 16).astype(np.uint16)
    elif kind == "uniform_words":
        words = rng.integers(0, 1 << 16, n, dtype=np.uint16)
    elif kind == "few_values":
        words = rng.choice(rng.integers(0, 1 << 16, draw(st.integers(1, 4)), dtype=np.uint16), n)
    else:
        w = (rng.standard_normal(n) * np.exp(rng.standard_normal(n) * 4)).astype(np.float32)
        words = (w.view(np.uint32) >> 16).astype(np.uint16)
    return words.tobytes()


@settings(max_examples=150, deadline=None)
@given(raw=bf16_tensors(), coder=st.sampled_from([0, 1, 2]), prec=st.integers(8, 12),
       chunk=st.sampled_from([256, 512, 4096, 32768]), groups=st.sampled_from([1, 1, 2, 4, 16]))
def test_any_tensor_round_trips(raw, coder, prec, chunk, groups):
    chunk *= groups                       # `groups` state groups of `chunk` values per chunk
    blob = O.xc_encode(raw, coder, prec, chunk, groups)
    assert len(blob) % 16 == 0
    assert O.xc_decode(blob, len(raw) // 2) == raw


@pytest.mark.parametrize("coder", [0, 1, 2])
def test_coded_size_close_to_exponent_entropy(coder):
    """1M config-1-like values: the exponent stream costs at most 3 % more
    than its empirical entropy (plus record headers and the raw plane)."""
    n = 1 << 20
    rng = np.random.default_rng(0)
    x = rng.standard_normal(n).astype(np.float32) * 0.02
    x[rng.permutation(n)[: n // 1000]] *= 30
    words = (x.view(np.uint32) >> 16).astype(np.uint16)
    e = (words >> 7) & 0xFF
    p = np.bincount(e, minlength=256) / n
    h = -sum(q * math.log2(q) for q in p if q > 0)          # bits per value
    ce = 32768
    blob = O.xc_encode(words.tobytes(), coder, 12, ce)
    n_chunks = n // ce
    framing = 576 + 4 * (n_chunks + 1) + n_chunks * (144 if coder == 2 else 128) + 16 * n_chunks
    coded_bits = (len(blob) - n - framing) * 8
    assert coded_bits <= 1.03 * h * n, (coder, coded_bits / n, h)


@settings(max_examples=60, deadline=None)
@given(raw=bf16_tensors(), kind=st.sampled_from(["par", "sk", "tans"]),
       n_streams=st.sampled_from([1, 3, 32, 128]))
def test_reference_formats_round_trip_on_the_oracle(raw, kind, n_streams):
    """The reference's own formats through their C restatement: bf16_parallel_v1
    at any slice count, bf16_se_single_kernel and bf16_se_tans, on the same
    value distributions (the byte layouts are pinned separately against
    reference-minted golden blobs)."""
    blob = O.par_encode(raw, n_streams) if kind == "par" else getattr(O, f"{kind}_encode")(raw)
    assert getattr(O, f"{kind}_decode")(blob, len(raw) // 2) == raw


@settings(max_examples=200, deadline=None)
@given(sizes=st.lists(st.tuples(st.integers(0, 200_000), st.sampled_from([0, 256, 4096, 32768])),
                      min_size=1, max_size=40),
       world=st.integers(1, 9))
def test_partition_owns_every_unit_once(sizes, world):
    """sharding.partition_chunks on random containers: every chunk of a
    splittable tensor and every unsplittable tensor (chunk size 0) has exactly
    one owner, and per-rank value counts add up to the container."""
    from bigsmall_b200.sharding import partition_chunks
    items = [(f"t{i}", n, ce) for i, (n, ce) in enumerate(sizes)]
    owned, load = partition_chunks(items, world)
    assert len(owned) == world and sum(load) == sum(n for _, n, _ in items)
    for name, n, ce in items:
        nc = max(1, -(-n // ce)) if ce else 1
        parts = sorted((c0, cc or nc) for r in owned for nm, c0, cc in r if nm == name)
        pos = 0
        for c0, cc in parts:
            assert c0 == pos
            pos += cc
        assert pos == nc, (name, parts, nc)
