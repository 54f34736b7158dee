"""Streaming layer-wise inference with the layer decode overlapped on a side stream.

Same entry points as BigSmall ``bigsmall/streaming_inference.py``
(``BigSmallStreamingModel(bs_path, hf_config, device, dtype, layer_template,
prefetch)``, ``from_pretrained``, ``forward``, ``generate``, ``close``).  The
reference decodes each layer on the CPU every time the layer runs, optionally
in a GIL-bound prefetch thread (``:152-199``, ``:272-348``), and frees VRAM
with ``gc.collect`` + ``empty_cache`` after every layer.

Here:
  * the compressed container stays resident in HBM; non-layer tensors
    (embeddings, final norm, lm_head) are decoded once;
  * decoded layers live in ``slots`` (2) fixed device buffers allocated once;
  * ``forward``/``generate`` run the model on a higher-priority stream than
    the side-stream decode, so the block scheduler places the running layer's
    CTAs first; the decode can also be capped at ``decode_ctas_per_sm`` CTAs
    per SM (its kernels then walk their work list);
  * global layer execution k uses slot ``k % slots``.  After layer i runs on the
    main stream, the decode of the layer that runs ``slots`` executions later
    is enqueued on a side stream into the slot just released, ordered by CUDA
    events (side waits for "layer i done", main waits for "layer decoded"), so
    decoding layer i+1 overlaps the GEMMs of layer i with no host thread and
    no allocation in the loop;
  * a layer called out of the expected order drains the side stream and
    restarts the pipeline at that layer (still entirely on the device).
The weights the model computes with are bit-identical to a fully decoded
model, so logits match a resident run bit for bit when the kernels are
deterministic.
"""
from __future__ import annotations

from typing import Optional

import torch

from .streaming import StreamingLoader


def _get_dotted_module(root, dotted: str):
    """Walk a dotted module path, indexing ModuleLists by integer parts
    (BigSmall bigsmall/streaming_inference.py:350-358)."""
    obj = root
    for p in dotted.split("."):
        obj = obj[int(p)] if p.isdigit() else getattr(obj, p)
    return obj


def _set_param_data(root, dotted: str, tensor: torch.Tensor) -> None:
    """Swap the tensor behind a parameter (or buffer) by dotted name, whether
    it lives on ``meta`` or a real device; parameters stay ``nn.Parameter``
    (BigSmall bigsmall/streaming_inference.py:49-70)."""
    parts = dotted.split(".")
    mod = _get_dotted_module(root, ".".join(parts[:-1])) if len(parts) > 1 else root
    leaf = parts[-1]
    if isinstance(getattr(mod, leaf, None), torch.nn.Parameter) or leaf in dict(mod.named_parameters(recurse=False)):
        setattr(mod, leaf, torch.nn.Parameter(tensor, requires_grad=False))
    else:
        setattr(mod, leaf, tensor)


def _layer_prefix(layer_idx: int, layer_template: str = "model.layers.{}") -> str:
    """Dotted name prefix of one layer's tensors in the container
    (BigSmall bigsmall/streaming_inference.py:73-74)."""
    return layer_template.format(layer_idx) + "."


def _materialize_meta_buffers(model, config, device) -> None:
    """Re-create modules whose buffers are computed at construction (rotary
    embeddings) on the real device; other meta buffers become zeros."""
    for name, mod in list(model.named_modules()):
        bufs = [b for _, b in mod.named_buffers(recurse=False) if b.device.type == "meta"]
        if not bufs:
            continue
        if hasattr(mod, "inv_freq"):
            try:
                new = type(mod)(config=config, device=device)
            except TypeError:
                new = type(mod)(config, device=device)
            parent_name, _, leaf = name.rpartition(".")
            parent = _get_dotted_module(model, parent_name) if parent_name else model
            setattr(parent, leaf, new)
        else:
            for bname, b in list(mod.named_buffers(recurse=False)):
                if b.device.type == "meta":
                    mod.register_buffer(bname, torch.zeros_like(b, device=device), persistent=False)


class BigSmallStreamingModel:
    def __init__(self, bs_path, hf_config, device: str = "cuda", dtype=None,
                 layer_template: str = "model.layers.{}", prefetch: int = 1, slots: int = 2,
                 model_cls=None, decode_ctas_per_sm: Optional[int] = None, priority_compute: bool = True):
        from transformers import AutoConfig, AutoModelForCausalLM
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.dtype = dtype or torch.bfloat16
        self.layer_template = layer_template
        self.config = hf_config if not isinstance(hf_config, (str, bytes)) and hasattr(hf_config, "to_dict") \
            else AutoConfig.from_pretrained(str(hf_config))
        self.loader = bs_path if isinstance(bs_path, StreamingLoader) else StreamingLoader(bs_path, device=self.device)
        ctor = model_cls or AutoModelForCausalLM.from_config
        with torch.device("meta"):
            self.model = ctor(self.config)
        self.model.eval()
        self.n_layers = self.loader.layer_count()
        self.prefetch = bool(prefetch)
        self.n_slots = max(2, int(slots))
        # non-layer weights: decoded once, resident
        non_layer = self.loader.load_non_layer_tensors()
        for name, t in non_layer.items():
            _set_param_data(self.model, name, t)
        if getattr(self.config, "tie_word_embeddings", False) and "lm_head.weight" not in non_layer:
            emb = self.model.get_input_embeddings().weight
            self.model.get_output_embeddings().weight = emb
        _materialize_meta_buffers(self.model, self.config, self.device)
        # layer slots: one set of device buffers per slot, shaped like layer 0
        self._prefix = [_layer_prefix(i, layer_template) for i in range(self.n_layers)]
        self._local = []
        for i in range(self.n_layers):
            names = self.loader.layer_tensor_names(i)
            self._local.append({n[len(self._prefix[i]):]: n for n in names if n.startswith(self._prefix[i])})
        keys0 = set(self._local[0])
        for i, loc in enumerate(self._local):
            if set(loc) != keys0:
                raise ValueError(f"layer {i} tensors differ from layer 0's; streaming needs uniform layers")
            for k, n in loc.items():
                m0, mi = self.loader.meta(self._local[0][k]), self.loader.meta(n)
                if m0["shape"] != mi["shape"] or m0["dtype"] != mi["dtype"]:
                    raise ValueError(f"{n}: shape/dtype differs from layer 0")
        self._slots = [{k: self.loader.res.empty_like(self._local[0][k]) for k in sorted(keys0)}
                       for _ in range(self.n_slots)]
        # one prebuilt decode bundle per (layer, slot); the side-stream decode
        # can be capped at decode_ctas_per_sm CTAs per SM (a decode CTA is 16
        # warps, half an SM's resident decode warps) to leave the running layer
        # SM room; uncapped measured best with 16-warp CTAs (None: uncapped)
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.decode_max_ctas = sms * decode_ctas_per_sm if decode_ctas_per_sm else 0
        self._bundles = {}
        for i in range(self.n_layers):
            for s in range(self.n_slots):
                self._bundles[(i, s)] = self.loader.res.bundle(
                    {self._local[i][k]: self._slots[s][k] for k in self._local[i]},
                    max_ctas=self.decode_max_ctas)
        self._side = torch.cuda.Stream(self.device)
        # forward()/generate() run the model on a higher-priority stream than
        # the side-stream decode, so the block scheduler places the running
        # layer's CTAs first and the decode fills the gaps
        hi = torch.cuda.Stream.priority_range()[1]
        self.compute_stream = torch.cuda.Stream(self.device, priority=hi) if priority_compute else None
        self._decoded = [torch.cuda.Event() for _ in range(self.n_slots)]
        self._released = [torch.cuda.Event() for _ in range(self.n_slots)]
        for ev in self._decoded + self._released:   # create the CUDA events now
            ev.record(torch.cuda.current_stream(self.device))
        self._k = 0                 # global layer-execution counter (selects the slot)
        self._expect = 0            # layer expected to run next
        self._primed = False
        for i in range(self.n_layers):
            self._patch_layer(i)
        # bind layer i to slot i % slots once; with a layer count divisible by
        # the slot count every later pass finds the same slot and skips rebinding
        self._bound = [-1] * self.n_layers
        for i in range(self.n_layers):
            self._bind(i, i % self.n_slots)
        # per (layer, slot): the whole hand-off after the running layer as one
        # prepared library call -- "slot released" on the model stream, the
        # side stream decodes the layer into it, and the model stream waits for
        # the slot of the layer that runs next
        self._handoff = {(i, s): self._bundles[(i, s)].handoff_call(
                             self._side, self._released[s], self._decoded[s],
                             self._decoded[(s + 1) % self.n_slots])
                         for i in range(self.n_layers) for s in range(self.n_slots)}

    # ------------------------------------------------------------------
    def _bind(self, layer: int, slot: int) -> None:
        mod = _get_dotted_module(self.model, self.layer_template.format(layer))
        for k, t in self._slots[slot].items():
            _set_param_data(mod, k, t)
        self._bound[layer] = slot

    def _prime(self, first_layer: int = 0) -> None:
        """Enqueue the decodes of the next `slots` layer executions."""
        main = torch.cuda.current_stream(self.device)
        self._side.wait_stream(main)
        for d in range(self.n_slots):
            k = self._k + d
            i = (first_layer + d) % self.n_layers
            self._bundles[(i, k % self.n_slots)].decode(self._side)
            self._decoded[k % self.n_slots].record(self._side)
        self._primed = True

    def _patch_layer(self, layer_idx: int) -> None:
        mod = _get_dotted_module(self.model, self.layer_template.format(layer_idx))
        original = mod.forward
        outer = self

        def streaming_forward(*args, **kwargs):
            main = torch.cuda.current_stream(outer.device)
            if not outer.prefetch:
                slot = 0
                outer._bundles[(layer_idx, slot)].decode(main)
                if outer._bound[layer_idx] != slot:
                    outer._bind(layer_idx, slot)
                return original(*args, **kwargs)
            slot = outer._k % outer.n_slots
            if not outer._primed or outer._expect != layer_idx:
                # first call, or out of the expected order: drain the side
                # stream and restart the pipeline at this layer
                outer._side.synchronize()
                outer._prime(first_layer=layer_idx)
                main.wait_event(outer._decoded[slot])
            # (in order, the previous layer's hand-off made the model stream
            # wait for this layer's slot)
            if outer._bound[layer_idx] != slot:
                outer._bind(layer_idx, slot)
            out = original(*args, **kwargs)
            nxt = (layer_idx + outer.n_slots) % outer.n_layers
            outer._handoff[(nxt, slot)](main)
            outer._k += 1
            outer._expect = (layer_idx + 1) % outer.n_layers
            return out

        mod.forward = streaming_forward

    # ------------------------------------------------------------------
    @classmethod
    def from_pretrained(cls, bs_path, hf_config_path=None, device: str = "cuda", dtype=None,
                        layer_template: str = "model.layers.{}", prefetch: int = 1):
        from pathlib import Path
        p = Path(bs_path)
        if not p.exists():
            raise FileNotFoundError(f"BigSmallStreamingModel.from_pretrained: path {bs_path!r} does not exist")
        if hf_config_path is None:
            cand = p if p.is_dir() else p.parent
            if not (cand / "config.json").exists():
                raise FileNotFoundError(f"no config.json next to {bs_path!r}; pass hf_config_path")
            hf_config_path = cand
        return cls(p, hf_config_path, device=device, dtype=dtype, layer_template=layer_template, prefetch=prefetch)

    def _on_compute_stream(self, fn):
        if self.compute_stream is None:
            return fn()
        caller = torch.cuda.current_stream(self.device)
        self.compute_stream.wait_stream(caller)
        with torch.cuda.stream(self.compute_stream):
            out = fn()
        caller.wait_stream(self.compute_stream)
        return out

    def forward(self, *args, **kwargs):
        with torch.no_grad():
            return self._on_compute_stream(lambda: self.model(*args, **kwargs))

    def generate(self, input_ids, max_new_tokens: int = 20, **kwargs):
        kwargs.setdefault("do_sample", False)
        kwargs.setdefault("max_new_tokens", max_new_tokens)
        with torch.no_grad():
            return self._on_compute_stream(lambda: self.model.generate(input_ids.to(self.device), **kwargs))

    def check(self) -> None:
        """Synchronise and raise if any layer decode reported a stream error."""
        torch.cuda.synchronize(self.device)
        for b in self._bundles.values():
            b.check()

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        for b in self._bundles.values():
            b.close()
        self._bundles = {}
