"""Mint golden vectors from the reference BigSmall implementation.

Run once in a container where the reference source tree is available:

    python tests/golden/make_golden.py --reference <path-to-BigSmall-checkout>

The reference's optional native dependencies (constriction, zstandard,
blosc2) are not needed by the codecs pinned here; empty stand-in modules are
created in a temporary directory so that ``import bigsmall`` succeeds.  The
script imports the reference's own codecs
(``bigsmall/codecs/bf16_parallel.py``, ``single_kernel.py``, ``bf16_tans.py``,
``rans.py``), encodes seeded synthetic bf16 tensors with them, decodes them
again, and writes:

  * ``<case>.raw``            the input tensor bytes (little-endian bf16)
  * ``<case>.<codec>.bin``    the reference encoder's blob
  * ``manifest.json``         md5 of every input / blob / reference decode,
                              plus md5-only pins of full-size BASELINE config 1
                              blobs (too large to commit)

Tests compare the oracle (and, on a GPU, the CUDA decoders) against these.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import struct
import sys
import tempfile
import time

HERE = os.path.dirname(os.path.abspath(__file__))


def md5(b: bytes) -> str:
    return hashlib.md5(b).hexdigest()


def setup_reference(path: str):
    stubs = tempfile.mkdtemp(prefix="bs_stubs_")
    for m in ("constriction", "zstandard", "blosc2"):
        with open(os.path.join(stubs, m + ".py"), "w") as f:
            f.write("# empty stand-in: not used by the pinned codecs\n")
    os.environ["BIGSMALL_DISABLE_VERSION_CHECK"] = "1"
    os.environ["BIGSMALL_FORCE_CPU"] = "1"
    sys.path.insert(0, path)
    sys.path.insert(0, stubs)
    import bigsmall  # noqa: F401
    from bigsmall.codecs import bf16_parallel, bf16_tans, rans, single_kernel
    return bf16_parallel, single_kernel, bf16_tans, rans


def c1_tensor(n: int = 4096 * 4096):
    """N(0, 0.02) with 0.1 % of positions scaled by 30."""
    import torch
    g = torch.Generator().manual_seed(0)
    x = torch.randn(n, generator=g) * 0.02
    idx = torch.randperm(n, generator=g)[: n // 1000]
    x[idx] *= 30
    return x.to(torch.bfloat16)


def inputs():
    import numpy as np
    import torch
    cases = {}
    torch.manual_seed(0)
    cases["gauss_8k"] = (torch.randn(8192) * 0.02).to(torch.bfloat16)
    # the reference tests' edge-word fixture (tests/test_bf16_parallel.py:39-63)
    specials = [0x7FC0, 0x7F80, 0xFF80, 0x0000, 0x8000, 0x0001, 0x0080, 0x3F80]
    torch.manual_seed(1)
    normals = (torch.randn(4096) * 0.02).to(torch.bfloat16).view(torch.uint8).numpy()
    raw = b"".join(struct.pack("<H", w) for w in specials) + normals.tobytes()
    cases["edge"] = torch.from_numpy(np.frombuffer(raw, dtype=np.uint16).copy()).view(torch.bfloat16)
    g = torch.Generator().manual_seed(7)
    for n in (1, 2, 31, 33, 255, 257, 1000):
        cases[f"tiny_{n}"] = (torch.randn(n, generator=g) * 0.05).to(torch.bfloat16)
    cases["single_symbol"] = torch.full((3000,), 1.0, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(11)
    words = torch.randint(0, 65536, (4096,), generator=g, dtype=torch.int32).to(torch.int64)
    cases["all_words"] = torch.from_numpy(words.numpy().astype(np.uint16)).view(torch.bfloat16)
    g = torch.Generator().manual_seed(3)
    scale = torch.exp(torch.randn(1, 2, 1, 16, generator=g))
    kv = torch.randn(1, 2, 256, 16, generator=g) * scale
    cases["kv_small"] = kv.to(torch.bfloat16).reshape(-1)
    c1 = c1_tensor()
    cases["c1_head_16k"] = c1[: 1 << 14].clone()
    return cases, c1


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of a BigSmall source checkout")
    ap.add_argument("--skip-full", action="store_true", help="skip the full-size config-1 pins")
    a = ap.parse_args()
    import numpy as np
    import torch
    par, sk, tans, rans = setup_reference(a.reference)
    cases, c1 = inputs()
    manifest = {"generator": "tests/golden/make_golden.py", "reference_version": None,
                "cases": {}, "rans_vectors": [], "full_size": {}}
    try:
        import bigsmall
        manifest["reference_version"] = getattr(bigsmall, "__version__", None)
    except Exception:
        pass
    for name, t in cases.items():
        raw = t.contiguous().view(torch.uint8).numpy().tobytes()
        n = len(raw) // 2
        with open(os.path.join(HERE, f"{name}.raw"), "wb") as f:
            f.write(raw)
        entry = {"n": n, "raw_md5": md5(raw), "blobs": {}}
        blobs = {}
        for ns in (1, 32, 128):
            b, e = par.encode(raw, n_streams=ns)
            blobs[f"par{ns}"] = ("bf16_parallel_v1", b, e, lambda b=b, e=e: par.decode(b, e, n))
        b, e = sk.encode(raw)
        blobs["sk"] = ("bf16_se_single_kernel", b, e, lambda b=b, e=e: sk.decode(b, e, n))
        b, e = tans.encode(raw)
        blobs["tans"] = ("bf16_se_tans", b, e, lambda b=b, e=e: tans.decode(b, e, n))
        for key, (codec, b, e, dec) in blobs.items():
            fn = f"{name}.{key}.bin"
            with open(os.path.join(HERE, fn), "wb") as f:
                f.write(b)
            out = dec()
            assert out == raw, (name, key)
            entry["blobs"][key] = {"codec": codec, "file": fn, "len": len(b), "md5": md5(b),
                                   "extras": e, "decoded_md5": md5(out)}
        manifest["cases"][name] = entry
    # rans.py stream vectors, incl. the decoder's end-of-data quirks
    g = np.random.default_rng(5)
    for M, alphabet, n in ((4096, 512, 0), (4096, 512, 1), (4096, 512, 777), (1024, 128, 500),
                           (1024, 128, 64)):
        syms = g.integers(0, alphabet, n).astype(np.int32) if n else np.zeros(0, np.int32)
        if n == 64:
            syms[:] = 5   # single-symbol stream: freq == M
        counts = np.bincount(syms, minlength=alphabet).astype(np.int64)
        freqs = rans.quantise_frequencies(counts, M)
        data = rans.encode_stream(syms, freqs, M)
        s2s = rans.build_slot_to_symbol(freqs, M)
        dec = rans.decode_stream(data, n, freqs, s2s, M)
        assert (dec.astype(np.int64) == syms.astype(np.int64)).all()
        vec = {"M": M, "alphabet": alphabet, "n": n, "symbols_hex": syms.astype("<u2").tobytes().hex(),
               "freqs": [int(x) for x in freqs], "stream_hex": data.hex()}
        if len(data) > 6:
            # truncated streams: drop 1 byte (odd tail -> zero-pad) and 3 bytes
            for cut in (1, 3):
                dd = rans.decode_stream(data[:-cut], n, freqs, s2s, M)
                vec[f"decode_cut{cut}_hex"] = dd.astype("<u2").tobytes().hex()
        manifest["rans_vectors"].append(vec)
    if not a.skip_full:
        raw = c1.contiguous().view(torch.uint8).numpy().tobytes()
        n = len(raw) // 2
        full = {"n": n, "raw_md5": md5(raw)}
        t0 = time.time()
        b, _ = sk.encode(raw)
        full["sk"] = {"len": len(b), "md5": md5(b)}
        b, _ = tans.encode(raw)
        full["tans"] = {"len": len(b), "md5": md5(b)}
        b, _ = par.encode(raw, n_streams=128)
        full["par128"] = {"len": len(b), "md5": md5(b)}
        full["seconds"] = round(time.time() - t0, 1)
        manifest["full_size"]["c1"] = full
    with open(os.path.join(HERE, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)
    print("wrote", len(manifest["cases"]), "cases")


if __name__ == "__main__":
    main()
