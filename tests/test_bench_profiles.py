"""The committed traffic figure the bench's roofline line reports
(profiles/xc_decode_c2_pair.json) belongs to the current decode-kernel
sources, and is consistent with the algorithmic bytes of the capture it was
scaled from.  A change to the decode kernel's sources fails the first check
until the traffic is captured again (medium case, one pass)."""
from __future__ import annotations

import json
import os

from tests.conftest import ROOT


def _profile():
    with open(os.path.join(ROOT, "profiles", "xc_decode_c2_pair.json")) as f:
        return json.load(f)


def test_traffic_profile_matches_the_kernel_sources():
    import bench
    assert _profile()["kernel_sources_sha256_16"] == bench.kernel_sources_digest()


def test_traffic_profile_is_consistent():
    p = _profile()
    m = p["medium_case"]
    per_value = (m["dram_read"] + m["dram_write"]) / m["values"]
    # the decode reads the compressed bytes (ratio about 0.66 of 2 B) and writes 2 B per value
    assert 3.2 < per_value < 3.5
    assert abs(p["traffic_bytes_per_launch"] - per_value * 8_030_261_248) < 1e6
