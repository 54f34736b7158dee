"""The reference-shaped ``kernels`` module's backend probe, as the reference's
tests/test_gpu_kernel.py:54-80 drive it (probe cache reset through
``_GPU_BACKEND`` / ``_GPU_DECODE_FN``, ``BIGSMALL_FORCE_CPU``).  CPU-only: no
decode runs here."""
from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")


def _reset(kernels):
    kernels._GPU_BACKEND = None
    kernels._GPU_DECODE_FN = None


def test_force_cpu_env_disables_gpu(monkeypatch):
    from bigsmall_b200 import kernels
    _reset(kernels)
    monkeypatch.setenv("BIGSMALL_FORCE_CPU", "1")
    try:
        assert kernels.use_gpu() is False
        assert kernels.backend_name() == "cpu"
        with pytest.raises(RuntimeError, match="BIGSMALL_FORCE_CPU"):
            kernels.decode_bf16_parallel(b"PAR1", {}, 4)
    finally:
        _reset(kernels)


def test_probe_result_is_cached(monkeypatch):
    from bigsmall_b200 import kernels
    _reset(kernels)
    monkeypatch.setenv("BIGSMALL_FORCE_CPU", "yes")
    assert kernels.backend_name() == "cpu"
    monkeypatch.delenv("BIGSMALL_FORCE_CPU")
    assert kernels._GPU_BACKEND == ""                  # probed once, not again
    _reset(kernels)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device answer")
def test_no_device_means_no_backend():
    from bigsmall_b200 import kernels
    _reset(kernels)
    try:
        assert kernels.use_gpu() is False and kernels.backend_name() == "cpu"
        with pytest.raises(RuntimeError, match="no CUDA device"):
            kernels.decode_bf16_parallel(b"PAR1", {}, 4)
    finally:
        _reset(kernels)
