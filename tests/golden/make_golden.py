"""Generate the golden fixtures that pin the oracle to the reference itself.

Run where a checkout of the LlamaMPS sources is available (it is only read),
giving its path as the argument or in ``$LLAMAMPS_REF``:

    python tests/golden/make_golden.py <path to the LlamaMPS checkout>

It imports the reference's own Python functions and records their outputs on
seeded inputs:

* ``utils/pack_weights.py::pack_tensor_4bit`` -- the Q4 packer that defines
  the weight format.  The function reads a safetensors file and writes
  ``<project>/weights/<name>_4bit.bin`` / ``_scales.bin`` next to its own
  module, so it is run from a temporary copy of ``utils/pack_weights.py``.
* ``utils/verify_attention.py::verify_attention_indexing`` -- GQA scores for
  one cached position.
* ``utils/verify_swiglu.py::verify_swiglu`` -- SiLU(gate) * up, fp16 out.

* ``scripts/extract_all.py`` with ``extract_layernorm``, ``extract_attn``,
  ``extract_post_norm``, ``extract_mlp``, ``copy_layer_weights`` and
  ``scripts/extract_global.py::extract_tied_weights`` -- the checkpoint
  converter that writes the flat-.bin layout the engine loads.  They run
  from a temporary copy of ``scripts/`` and ``utils/pack_weights.py`` (they
  read and write ``<project>/weights``) on a small seeded Qwen2-named
  checkpoint (``llamamps_b200.convert.write_synthetic_checkpoint``), and the
  sha256 of every file they write is recorded.

Outputs (small files, committed): ``pack_cases.npz``, ``verify_cases.npz``,
``reference_layout.json``.  Nothing at test time reads the reference; the
tests read these files.
"""
from __future__ import annotations

import importlib.util
import os
import shutil
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF = ""  # the LlamaMPS checkout, set in __main__ from argv[1] or $LLAMAMPS_REF


def _load_module(path: str, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def pack_cases():
    """Seeded tensors, including a padded odd size, half-way ties, dead groups
    and negative-max groups, packed by the reference function."""
    import torch
    from safetensors.torch import save_file

    rng = np.random.default_rng(20240601)
    cases = {
        "normal_64x96": rng.normal(0, 0.02, (64, 96)).astype(np.float32),
        "odd_7x33": rng.normal(0, 1.0, (7, 33)).astype(np.float32),
        "kproj_64x1536": rng.normal(0, 0.02, (64, 1536)).astype(np.float32),
    }
    # groups of 32 with exact .5 ties after division by scale = 1.0 (max 7),
    # a dead all-zero group, a group whose max-|w| element is negative, and a
    # group with tiny values (subnormal fp16 scale).
    ties = np.array([7.0, 0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 3.5, -3.5, 4.5, 5.5, 6.5, -6.5,
                     0.0, -0.0, 6.9] + [0.25 * i for i in range(16)], np.float32)
    dead = np.zeros(32, np.float32)
    negmax = np.linspace(-3.5, 1.0, 32).astype(np.float32)
    tiny = (rng.normal(0, 1e-6, 32)).astype(np.float32)
    cases["edge_4x32"] = np.stack([ties, dead, negmax, tiny])

    tmp = tempfile.mkdtemp(prefix="lmps_golden_")
    try:
        os.makedirs(os.path.join(tmp, "utils"))
        shutil.copy(os.path.join(REF, "utils", "pack_weights.py"), os.path.join(tmp, "utils", "pack_weights.py"))
        mod = _load_module(os.path.join(tmp, "utils", "pack_weights.py"), "ref_pack_weights")
        st_path = os.path.join(tmp, "tensors.safetensors")
        save_file({f"model.case.{k}.weight": torch.from_numpy(v) for k, v in cases.items()}, st_path)
        out = {}
        for name, w in cases.items():
            mod.pack_tensor_4bit(st_path, f"model.case.{name}.weight")
            packed = np.fromfile(os.path.join(tmp, "weights", f"{name}_4bit.bin"), np.uint8)
            scales = np.fromfile(os.path.join(tmp, "weights", f"{name}_scales.bin"), np.float16)
            out[f"{name}__w"] = w
            out[f"{name}__packed"] = packed
            out[f"{name}__scales"] = scales
        np.savez_compressed(os.path.join(HERE, "pack_cases.npz"), **out)
        print("pack cases:", ", ".join(cases))
    finally:
        shutil.rmtree(tmp)


def verify_cases():
    att = _load_module(os.path.join(REF, "utils", "verify_attention.py"), "ref_verify_attention")
    swi = _load_module(os.path.join(REF, "utils", "verify_swiglu.py"), "ref_verify_swiglu")
    rng = np.random.default_rng(7)
    out = {}
    for i in range(3):
        q = rng.normal(0, 1, 1536).astype(np.float16)
        k = rng.normal(0, 1, 256).astype(np.float16)
        out[f"attn{i}__q"] = q
        out[f"attn{i}__k"] = k
        out[f"attn{i}__scores"] = att.verify_attention_indexing(q, k)
    for i in range(2):
        g = (rng.normal(0, 3, 8960)).astype(np.float16)
        u = (rng.normal(0, 1, 8960)).astype(np.float16)
        out[f"swiglu{i}__gate"] = g
        out[f"swiglu{i}__up"] = u
        out[f"swiglu{i}__out"] = swi.verify_swiglu(g, u)
    np.savez_compressed(os.path.join(HERE, "verify_cases.npz"), **out)
    print("verify cases written")


# The checkpoint of the layout case: small enough to convert in seconds, the
# smallest shape the persistent decode kernel takes (hidden a multiple of 512,
# head_dim 128).
LAYOUT_CASE = {"hidden": 512, "intermediate": 512, "vocab": 1024, "n_layers": 2, "n_q_heads": 4,
               "n_kv_heads": 2, "head_dim": 128, "seed": 11}


def layout_case_config():
    from llamamps_b200.config import ModelConfig
    c = {k: v for k, v in LAYOUT_CASE.items() if k != "seed"}
    return ModelConfig(**c)


def reference_layout_case():
    """Run the reference's extraction scripts on the seeded checkpoint and
    record the sha256 of every file they write."""
    import hashlib
    import json
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from llamamps_b200.convert import write_synthetic_checkpoint
    cfg = layout_case_config()
    tmp = tempfile.mkdtemp(prefix="lmps_layout_")
    saved_path = list(sys.path)
    try:
        os.makedirs(os.path.join(tmp, "utils"))
        os.makedirs(os.path.join(tmp, "scripts"))
        os.makedirs(os.path.join(tmp, "weights"))
        shutil.copy(os.path.join(REF, "utils", "pack_weights.py"), os.path.join(tmp, "utils"))
        for f in ("extract_all.py", "extract_attn.py", "extract_mlp.py", "extract_layernorm.py",
                  "extract_postnorm.py", "extract_global.py"):
            shutil.copy(os.path.join(REF, "scripts", f), os.path.join(tmp, "scripts"))
        model = os.path.join(tmp, "weights", "model.safetensors")
        write_synthetic_checkpoint(model, cfg, LAYOUT_CASE["seed"])
        for m in [m for m in sys.modules if m == "utils" or m.startswith(("utils.", "scripts"))]:
            del sys.modules[m]
        sys.path.insert(0, tmp)
        ext_all = _load_module(os.path.join(tmp, "scripts", "extract_all.py"), "ref_extract_all")
        ext_glob = _load_module(os.path.join(tmp, "scripts", "extract_global.py"), "ref_extract_global")
        for layer in range(cfg.n_layers):      # extract_all.py:53-60
            ext_all.extract_layernorm(layer)
            ext_all.extract_attn(layer)
            ext_all.extract_post_norm(layer)
            ext_all.extract_mlp(layer)
            ext_all.copy_layer_weights(layer)
        ext_glob.extract_tied_weights(model, os.path.join(tmp, "weights", "global"))
        files = {}
        root = os.path.join(tmp, "weights")
        for dirpath, _, names in os.walk(root):
            for n in names:
                path = os.path.join(dirpath, n)
                if path == model:
                    continue
                with open(path, "rb") as f:
                    files[os.path.relpath(path, root)] = hashlib.sha256(f.read()).hexdigest()
        with open(os.path.join(HERE, "reference_layout.json"), "w") as f:
            json.dump({"case": LAYOUT_CASE, "files": dict(sorted(files.items()))}, f, indent=1)
        print("reference layout case:", len(files), "files")
    finally:
        sys.path[:] = saved_path
        shutil.rmtree(tmp)


if __name__ == "__main__":
    REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("LLAMAMPS_REF", "")
    if not REF or not os.path.isdir(REF):
        sys.exit("usage: make_golden.py <path to the LlamaMPS checkout> (or set LLAMAMPS_REF)")
    pack_cases()
    verify_cases()
    reference_layout_case()
