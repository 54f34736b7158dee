"""This project's bf16_exp_chunked_v1 encoder output, pinned: the CPU oracle's
blob md5 for every golden input, coder and framing, and for two seeded
tensors past 2^20 values (the pair coder's sampled statistics), as recorded by
tests/golden/make_xc_pins.py.  The GPU tests require the device encoder to
equal the oracle byte for byte, so these pins hold it too.  Regenerate the pins
only on purpose, when the encoder's choices change."""
from __future__ import annotations

import hashlib
import json
import os

import pytest

from oracle import oracle as O
from tests.conftest import ROOT, golden_bytes
from tests.golden.make_xc_pins import SEEDED, seeded

with open(os.path.join(ROOT, "tests", "golden", "xc_pins.json")) as _f:
    PINS = json.load(_f)


def _inputs():
    names = sorted({k.split("/")[0] for k in PINS["blobs"]})
    return names


@pytest.mark.parametrize("name", _inputs())
def test_oracle_encoder_matches_the_pins(name):
    raw = seeded(name) if name in SEEDED else golden_bytes(f"{name}.raw")
    for key, want in PINS["blobs"].items():
        n, coder, ce, groups = key.split("/")
        if n != name:
            continue
        blob = O.xc_encode(raw, int(coder), PINS["prec"], int(ce), int(groups))
        assert hashlib.md5(blob).hexdigest() == want, key
