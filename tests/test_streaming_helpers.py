"""Helper functions of the streaming model, as the reference's
tests/test_streaming_inference.py:14-60 check them (CPU, no decode)."""
from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")
from torch import nn  # noqa: E402


def test_streaming_inference_imports():
    import bigsmall_b200.streaming_inference  # noqa: F401


def test_set_param_data_swaps_parameter():
    from bigsmall_b200.streaming_inference import _set_param_data
    m = nn.Linear(4, 4)
    _set_param_data(m, "weight", torch.zeros(4, 4))
    assert torch.equal(m.weight, torch.zeros(4, 4))
    assert isinstance(m.weight, nn.Parameter) and not m.weight.requires_grad


def test_set_param_data_nested_index_and_buffer():
    from bigsmall_b200.streaming_inference import _get_dotted_module, _set_param_data
    m = nn.ModuleList([nn.Linear(2, 2), nn.Linear(2, 2)])
    _set_param_data(m, "1.weight", torch.eye(2))
    assert torch.equal(m[1].weight, torch.eye(2))
    bn = nn.Sequential(nn.BatchNorm1d(3))
    _set_param_data(bn, "0.running_mean", torch.ones(3))
    assert torch.equal(bn[0].running_mean, torch.ones(3)) and not isinstance(bn[0].running_mean, nn.Parameter)
    assert _get_dotted_module(m, "1") is m[1]


def test_set_param_data_replaces_a_meta_parameter():
    from bigsmall_b200.streaming_inference import _set_param_data
    with torch.device("meta"):
        m = nn.Linear(3, 2)
    _set_param_data(m, "bias", torch.arange(2.0))
    assert m.bias.device.type == "cpu" and torch.equal(m.bias, torch.arange(2.0))


def test_layer_prefix_format():
    from bigsmall_b200.streaming_inference import _layer_prefix
    assert _layer_prefix(0) == "model.layers.0."
    assert _layer_prefix(31) == "model.layers.31."
    assert _layer_prefix(5, "h.{}") == "h.5."
