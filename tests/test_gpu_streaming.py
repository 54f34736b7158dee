"""Streaming layer-wise inference (reference bigsmall/streaming_inference.py,
bigsmall/streaming.py API): a random-init Qwen2-architecture model decoded
layer by layer on a side stream produces logits bit-identical to the fully
decoded model, and the StreamingLoader API returns exact tensors."""
from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")
transformers = pytest.importorskip("transformers")
pytestmark = pytest.mark.gpu


def _cfg(layers=4, tie=False):
    from transformers import Qwen2Config
    return Qwen2Config(vocab_size=512, hidden_size=128, intermediate_size=320, num_hidden_layers=layers,
                       num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=512,
                       tie_word_embeddings=tie, rope_theta=10000.0)


def _image(weights, chunk_elems=4096):
    from bigsmall_b200 import decoder
    from bigsmall_b200.loader import ContainerImage
    return ContainerImage.from_bytes(decoder.compress_tensors(weights, chunk_elems=chunk_elems, with_md5=False))


@pytest.mark.parametrize("layers,tie,prefetch", [(4, False, 1), (5, True, 1), (4, False, 0)])
def test_streaming_logits_bit_identical(layers, tie, prefetch):
    from bigsmall_b200 import synthetic
    from bigsmall_b200.streaming import StreamingLoader
    from bigsmall_b200.streaming_inference import BigSmallStreamingModel
    torch.use_deterministic_algorithms(True, warn_only=True)
    cfg = _cfg(layers, tie)
    w = synthetic.random_weights(cfg, seed=0)
    if tie:
        w.pop("lm_head.weight", None)
    g = torch.Generator(device="cuda").manual_seed(0)
    prompt = torch.randint(0, cfg.vocab_size, (1, 48), generator=g, device="cuda")
    ref = synthetic.resident_model(cfg, w)
    ids_r, lg_r, _, _ = synthetic.greedy(ref, prompt, 12)
    sm = BigSmallStreamingModel(StreamingLoader(_image(w)), cfg, prefetch=prefetch)
    for _ in range(2):      # the pipeline survives repeated generations
        ids_s, lg_s, _, _ = synthetic.greedy(sm.model, prompt, 12)
        sm.check()
        assert torch.equal(ids_r, ids_s)
        assert torch.equal(lg_r.view(torch.int16), lg_s.view(torch.int16))
    out = sm.generate(prompt, max_new_tokens=6)
    assert torch.equal(out[:, 48:], ids_r[:, :6])
    sm.close()


def test_streaming_loader_api():
    from bigsmall_b200 import synthetic
    from bigsmall_b200.streaming import StreamingLoader, layer_index
    cfg = _cfg(3)
    w = synthetic.random_weights(cfg, seed=1)
    with StreamingLoader(_image(w)) as ld:
        assert ld.layer_count() == 3
        assert set(ld.non_layer_tensor_names()) == {n for n in w if layer_index(n) is None}
        layer1 = ld.load_layer(1)
        assert set(layer1) == {n for n in w if layer_index(n) == 1}
        for n, t in layer1.items():
            assert torch.equal(t.view(torch.int16), w[n].view(torch.int16)), n
        assert torch.equal(ld.load_tensor("lm_head.weight").view(torch.int16), w["lm_head.weight"].view(torch.int16))
        seen = [i for i, _ in ld.iter_layers()]
        assert seen == [0, 1, 2]
        with pytest.raises(IndexError):
            ld.load_layer(7)
        with pytest.raises(KeyError):
            ld.load_tensor("nope")
    assert layer_index("transformer.h.11.mlp.c_fc.bias") == 11 and layer_index("model.norm.weight") is None


def test_streaming_config4_layer_width_logits_bit_identical():
    """BASELINE config 4's shapes (Qwen2.5-14B: hidden 5120, intermediate 13824,
    40 Q / 8 KV heads x 128, q/k/v biases, vocab 152064, untied embeddings) at 3
    layers, default chunk size: the side-stream pipeline's logits equal the
    resident model's bit for bit (reference bigsmall/streaming_inference.py:
    152-199, 272-348 swap decoded layers in the same way)."""
    from transformers import Qwen2Config
    from bigsmall_b200 import gpu, synthetic
    from bigsmall_b200.streaming import StreamingLoader
    from bigsmall_b200.streaming_inference import BigSmallStreamingModel
    torch.use_deterministic_algorithms(True, warn_only=True)
    cfg = Qwen2Config(vocab_size=152064, hidden_size=5120, intermediate_size=13824, num_hidden_layers=3,
                      num_attention_heads=40, num_key_value_heads=8, max_position_embeddings=4096,
                      tie_word_embeddings=False, rope_theta=1000000.0, rms_norm_eps=1e-6)
    w = synthetic.random_weights(cfg, seed=0)
    assert w["model.layers.0.mlp.gate_proj.weight"].shape == (13824, 5120)
    assert w["model.layers.0.self_attn.k_proj.weight"].shape == (1024, 5120)
    g = torch.Generator(device="cuda").manual_seed(0)
    prompt = torch.randint(0, cfg.vocab_size, (1, 64), generator=g, device="cuda")
    ref = synthetic.resident_model(cfg, w)
    ids_r, lg_r, _, _ = synthetic.greedy(ref, prompt, 4)
    del ref
    sm = BigSmallStreamingModel(StreamingLoader(_image(w, gpu.DEFAULT_CHUNK_ELEMS)), cfg, prefetch=1)
    try:
        for _ in range(2):
            ids_s, lg_s, _, _ = synthetic.greedy(sm.model, prompt, 4)
            sm.check()
            assert torch.equal(ids_r, ids_s)
            assert torch.equal(lg_r.view(torch.int16), lg_s.view(torch.int16))
    finally:
        sm.close()
