"""A checkpoint converted to the reference's layout, loaded through the
reference API and decoded, against the oracle built from the checkpoint's own
tensors; and the demo flow (demo.py:14-20 with the forward pass) on it."""
import numpy as np
import pytest
import torch

from oracle import mirror as M
from tests._util import greedy_ids_match
from tests.test_host_cpu import _layout_case

pytestmark = pytest.mark.gpu


def _oracle_weights(st, cfg):
    def q4(name):
        return M.q4_pack(st[name].float().numpy())

    def f16(name):
        return st[name].to(torch.float16).numpy()
    layers = []
    for i in range(cfg.n_layers):
        p = f"model.layers.{i}."
        lw = {"in_norm": f16(p + "input_layernorm.weight"), "post_norm": f16(p + "post_attention_layernorm.weight"),
              "bq": f16(p + "self_attn.q_proj.bias"), "bk": f16(p + "self_attn.k_proj.bias"),
              "bv": f16(p + "self_attn.v_proj.bias")}
        for key, name in (("q", "self_attn.q_proj"), ("k", "self_attn.k_proj"), ("v", "self_attn.v_proj"),
                          ("o", "self_attn.o_proj"), ("gt", "mlp.gate_proj"), ("up", "mlp.up_proj"),
                          ("dn", "mlp.down_proj")):
            lw[key], lw[key + "s"] = q4(p + name + ".weight")
        layers.append(lw)
    lp, ls = q4("model.embed_tokens.weight")
    return {"layers": layers, "final_norm": f16("model.norm.weight"), "lm_packed": lp, "lm_scales": ls,
            "embed": f16("model.embed_tokens.weight")}


def test_converted_checkpoint_decodes_like_the_oracle(cuda, tmp_path):
    from llamamps_b200 import demo
    from llamamps_b200.convert import convert_state_dict, synthetic_state_dict
    from llamamps_b200.engine import QwenEngine
    cfg, seed, _ = _layout_case()
    st = synthetic_state_dict(cfg, seed)
    convert_state_dict(st, str(tmp_path))
    prompt = [5, 1000, 77, 1023, 300]
    eng = QwenEngine(str(tmp_path), config=cfg, max_seq_len=64)
    assert eng.decoder == "persistent"
    got = demo.generate(eng, prompt, 6)
    host = _oracle_weights(st, cfg)
    ocfg = M.OracleConfig(hidden=cfg.hidden, intermediate=cfg.intermediate, vocab=cfg.vocab, n_layers=cfg.n_layers,
                          n_q_heads=cfg.n_q_heads, n_kv_heads=cfg.n_kv_heads, head_dim=cfg.head_dim)
    rec = []
    ref = M.OracleModel(host, ocfg).generate(prompt, 6, record=rec)
    assert greedy_ids_match(got, ref, rec) >= 3
    kern = QwenEngine(str(tmp_path), config=cfg, max_seq_len=64, decoder="kernels")
    assert greedy_ids_match(kern.generate(prompt, 6), ref, rec) >= 3
    # the reference's entry points: first token's embedding row, one forward, host argmax
    vec, ids = demo.get_input_vector(prompt, str(tmp_path / "global" / "embed_tokens.bin"), hidden=cfg.hidden)
    assert ids == prompt and np.array_equal(vec, host["embed"][prompt[0]])
    lg = QwenEngine(str(tmp_path), config=cfg, max_seq_len=64).run_inference(vec)
    first = M.OracleModel(host, ocfg).step_vector(vec)
    assert float(np.max(np.abs(lg.astype(np.float32) - first.astype(np.float32)))) <= 2e-2
    # the command-line flow
    out = demo.main(["--weights", str(tmp_path), "--ids", ",".join(map(str, prompt)), "--new", "6"], config=cfg)
    assert out == got
