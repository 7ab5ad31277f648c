"""The drop-in boundary, pinned against the reference engine's own source.

tests/golden/engine_contract.json lists, with file:line, what the
reference's engine (src/engine/model_runner.py, llm_engine.py), loader
(src/utils/loader.py) and bench.py ask of the decoder-path modules; it was
extracted from those files by tests/golden/make_engine_contract.py.  Here this
build's modules must satisfy every item (CPU only; the model is built on the
CPU with a tiny configuration, nothing runs a kernel):
  * each name the engine imports from a module this build provides exists;
  * each call the engine makes on the model, the sampler and the model class
    binds to this build's signatures with the same positional count and
    keyword names;
  * Context has every field the engine sets;
  * the KV-cache protocol: one module per layer with both k_cache and
    v_cache, empty until assigned;
  * the loader protocol: packed_modules_mapping targets exist and their
    weight_loaders take a shard id, the other parameters take (param, tensor).
The modules the reference keeps (its config, scheduler, logging, tokenizer)
are not part of the boundary.
"""
import importlib
import inspect
import json
import os

import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
PROVIDED = {"src.layers.linear", "src.layers.attention", "src.layers.layernorm",
            "src.layers.pos_embedding", "src.layers.activation", "src.layers.llm_head",
            "src.layers.sampler", "src.models.qwen3", "src.utils.context", "src.utils.loader",
            "src.utils.math"}


@pytest.fixture(scope="module")
def contract():
    with open(os.path.join(HERE, "golden", "engine_contract.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def model():
    from oracle.weights import Qwen3Shape
    from src.models.qwen3 import Qwen3ForCausalLM
    shape = Qwen3Shape(hidden=256, layers=3, heads=4, kv_heads=2, head_dim=128, inter=512,
                       vocab=1000, max_pos=512)
    return Qwen3ForCausalLM(shape.hf_config(), tp=(0, 1))


def _binds(fn, positional: int, keywords: list[str]):
    args = [object()] * positional
    inspect.signature(fn).bind(*args, **{k: object() for k in keywords})


def test_imports_of_the_engine_resolve(contract):
    seen = 0
    for imp in contract["imports"]:
        if imp["module"] not in PROVIDED:
            continue
        mod = importlib.import_module(imp["module"])
        assert hasattr(mod, imp["name"]), imp
        seen += 1
    assert seen >= 3  # Sampler, Context, Qwen3ForCausalLM


def test_engine_calls_bind(contract, model):
    from src.layers.sampler import Sampler
    from src.models.qwen3 import Qwen3ForCausalLM
    methods = set()
    for c in contract["model_calls"]:
        m = c["method"]
        methods.add(m)
        if m == "__init__":
            _binds(Qwen3ForCausalLM, c["positional"], c["keywords"])
        elif m == "__call__":
            _binds(model.forward, c["positional"], c["keywords"])
        elif m == "Sampler":
            _binds(Sampler, c["positional"], c["keywords"])
        elif m == "sampler":
            _binds(Sampler(seed=0).forward, c["positional"], c["keywords"])
        else:
            _binds(getattr(model, m), c["positional"], c["keywords"])
    assert {"__init__", "load", "__call__", "compute_logits", "modules", "sampler"} <= methods


def test_context_has_the_fields_the_engine_sets(contract):
    import dataclasses
    from src.utils.context import Context
    fields = {f.name for f in dataclasses.fields(Context)}
    for c in contract["context_kwargs"]:
        assert set(c["keywords"]) <= fields, c
        Context(**{k: None for k in c["keywords"]})


def test_kv_cache_protocol(contract, model):
    attrs = {a["attr"] for a in contract["module_attrs"] if a["at"].startswith("src/engine/model_runner")}
    assert {"k_cache", "v_cache"} <= attrs
    holders = [m for m in model.modules() if all(hasattr(m, a) for a in ("k_cache", "v_cache"))]
    assert len(holders) == len(model.model.layers)
    assert all(m.k_cache.numel() == 0 and m.v_cache.numel() == 0 for m in holders)


def test_loader_protocol(contract, model):
    calls = {(c["call"], c["positional"]) for c in contract["loader"]}
    assert ("weight_loader", 3) in calls and ("weight_loader", 2) in calls
    packed = model.packed_modules_mapping
    names = dict(model.named_parameters())
    hf = ["model.layers.0.self_attn.q_proj.weight", "model.layers.0.self_attn.k_proj.weight",
          "model.layers.0.self_attn.v_proj.weight", "model.layers.0.mlp.gate_proj.weight",
          "model.layers.0.mlp.up_proj.weight", "model.layers.0.self_attn.o_proj.weight",
          "model.layers.0.mlp.down_proj.weight", "model.embed_tokens.weight", "lm_head.weight",
          "model.norm.weight", "model.layers.0.input_layernorm.weight"]
    for weight_name in hf:
        for k, (v, shard_id) in packed.items():
            if k in weight_name:
                p = model.get_parameter(weight_name.replace(k, v))
                inspect.signature(p.weight_loader).bind(p, torch.empty(0), shard_id)
                break
        else:
            p = model.get_parameter(weight_name)
            wl = getattr(p, "weight_loader", None)
            if wl is not None:
                inspect.signature(wl).bind(p, torch.empty(0))
    assert "model.layers.0.self_attn.qkv_proj.weight" in names
