"""Seeded random-init weights of a Hugging Face decoder-only architecture,
generated on the device (BASELINE configs 2 and 4 use such models: linear
weights N(0, 1/sqrt(fan_in)), RMSNorm weights 1 + N(0, 0.01), biases
N(0, 0.02); one generator, tensors in parameter-name order)."""
from __future__ import annotations

import math

import torch


def param_specs(config, model_cls=None):
    """[(name, shape)] of the model's parameters, without allocating them."""
    from transformers import AutoModelForCausalLM
    ctor = model_cls or AutoModelForCausalLM.from_config
    with torch.device("meta"):
        m = ctor(config)
    return [(n, tuple(p.shape)) for n, p in m.named_parameters()]


def init_tensor(name: str, shape, g: torch.Generator, device) -> torch.Tensor:
    x = torch.randn(shape, generator=g, device=device)
    if name.endswith("norm.weight"):
        x = 1.0 + x * 0.01
    elif name.endswith(".bias"):
        x = x * 0.02
    else:
        x = x * (1.0 / math.sqrt(shape[-1]))
    return x.to(torch.bfloat16)


def random_weights(config, seed: int = 0, device="cuda", model_cls=None) -> dict:
    g = torch.Generator(device=device).manual_seed(seed)
    return {n: init_tensor(n, s, g, device) for n, s in param_specs(config, model_cls)}


def resident_model(config, weights: dict, device="cuda", model_cls=None):
    """An eval-mode model whose parameters are exactly `weights` (no copies)."""
    from transformers import AutoModelForCausalLM
    from .streaming_inference import _materialize_meta_buffers, _set_param_data
    ctor = model_cls or AutoModelForCausalLM.from_config
    with torch.device("meta"):
        m = ctor(config)
    for n, t in weights.items():
        _set_param_data(m, n, t)
    if getattr(config, "tie_word_embeddings", False) and "lm_head.weight" not in weights:
        m.get_output_embeddings().weight = m.get_input_embeddings().weight
    _materialize_meta_buffers(m, config, torch.device(device))
    return m.eval()


def greedy(model, input_ids: torch.Tensor, steps: int):
    """Prefill + `steps` greedy decode steps with a KV cache; returns
    (generated ids, per-step last-position logits, prefill ms, decode ms)."""
    s, m, e = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    logits, ids = [], []
    with torch.no_grad():
        s.record()
        out = model(input_ids=input_ids, use_cache=True)
        m.record()
        cache = out.past_key_values
        last = out.logits[:, -1, :]
        for _ in range(steps):
            logits.append(last)
            tok = last.argmax(dim=-1, keepdim=True)
            ids.append(tok)
            out = model(input_ids=tok, past_key_values=cache, use_cache=True)
            cache = out.past_key_values
            last = out.logits[:, -1, :]
        e.record()
    torch.cuda.synchronize()
    return torch.cat(ids, 1), torch.stack(logits), s.elapsed_time(m), m.elapsed_time(e)
