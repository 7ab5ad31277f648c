"""Extract, from the reference's engine sources, what the engine asks of the
decoder-path modules (the drop-in boundary), into engine_contract.json.

Run where the reference checkout is available, with its path in REF_DIR
(required).  Reads src/engine/*.py, src/utils/loader.py and bench.py of the
reference with Python's ast module (nothing is imported or executed) and
records, with file:line:
  * every `from src.<pkg>.<mod> import <name>` of the path's packages
    (layers, models, utils);
  * the calls the engine makes on the model object (self.model.<attr>(...),
    self.model(...), modelClass(...)) with their positional count and
    keyword names;
  * the keyword names of every Context(...) construction;
  * the attributes read from modules (k_cache / v_cache protocol) and the
    loader's weight protocol (packed_modules_mapping, get_parameter,
    weight_loader call shapes).
tests/test_engine_contract.py checks this build's modules against it.
"""
import ast
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.environ.get("REF_DIR", "")
FILES = ["src/engine/model_runner.py", "src/engine/llm_engine.py", "src/utils/loader.py", "bench.py"]
PATH_PKGS = ("src.layers", "src.models", "src.utils")


def call_shape(node: ast.Call) -> dict:
    return {"positional": len(node.args), "keywords": sorted(k.arg for k in node.keywords if k.arg)}


def main():
    if not REF_DIR or not os.path.isdir(os.path.join(REF_DIR, "src")):
        raise SystemExit("set REF_DIR to the reference checkout (the directory holding src/)")
    out = {"imports": [], "model_calls": [], "context_kwargs": [], "module_attrs": [], "loader": []}
    for rel in FILES:
        path = os.path.join(REF_DIR, rel)
        tree = ast.parse(open(path).read(), rel)
        for node in ast.walk(tree):
            where = f"{rel}:{getattr(node, 'lineno', 0)}"
            if isinstance(node, ast.ImportFrom) and node.module and node.module.startswith(PATH_PKGS):
                for a in node.names:
                    out["imports"].append({"module": node.module, "name": a.name, "at": where})
            if not isinstance(node, ast.Call):
                continue
            f = node.func
            # self.model(...), self.model.<attr>(...)
            if isinstance(f, ast.Attribute) and isinstance(f.value, ast.Name) and f.value.id == "self" \
                    and f.attr == "model":
                out["model_calls"].append({"method": "__call__", **call_shape(node), "at": where})
            if isinstance(f, ast.Attribute) and isinstance(f.value, ast.Attribute) \
                    and isinstance(f.value.value, ast.Name) and f.value.value.id == "self" \
                    and f.value.attr == "model":
                out["model_calls"].append({"method": f.attr, **call_shape(node), "at": where})
            if isinstance(f, ast.Name) and f.id == "modelClass":
                out["model_calls"].append({"method": "__init__", **call_shape(node), "at": where})
            if isinstance(f, ast.Name) and f.id == "Sampler":
                out["model_calls"].append({"method": "Sampler", **call_shape(node), "at": where})
            if isinstance(f, ast.Attribute) and f.attr == "sampler":
                out["model_calls"].append({"method": "sampler", **call_shape(node), "at": where})
            if isinstance(f, ast.Name) and f.id == "Context":
                out["context_kwargs"].append({"keywords": sorted(k.arg for k in node.keywords), "at": where})
            if isinstance(f, ast.Name) and f.id == "hasattr" and len(node.args) == 2 \
                    and isinstance(node.args[1], ast.Constant):
                out["module_attrs"].append({"attr": node.args[1].value, "at": where})
            if rel.endswith("loader.py"):
                if isinstance(f, ast.Name) and f.id in ("weight_loader", "getattr"):
                    out["loader"].append({"call": f.id, **call_shape(node), "at": where,
                                          "args": [a.value for a in node.args if isinstance(a, ast.Constant)]})
                if isinstance(f, ast.Attribute) and f.attr == "get_parameter":
                    out["loader"].append({"call": "get_parameter", **call_shape(node), "at": where, "args": []})
    with open(os.path.join(HERE, "engine_contract.json"), "w") as fh:
        json.dump(out, fh, indent=1)
    print({k: len(v) for k, v in out.items()})


if __name__ == "__main__":
    sys.exit(main())
