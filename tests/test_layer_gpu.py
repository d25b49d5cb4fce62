"""One decoder layer, one decode step (seeded synthetic case: Qwen2.5-1.5B
layer shapes, biases, 31 cached positions, new token at position 31) through
the engine's kernels, against the oracle layer."""
import dataclasses

import numpy as np
import pytest
import torch

from oracle import mirror as M
from tests._util import assert_close

pytestmark = pytest.mark.gpu


def _one_layer_engine(parts, cfg, max_seq=128, page_order=None):
    from llamamps_b200.engine import QwenEngine
    from llamamps_b200.weights import ModelWeights, layer_from_parts
    small = dataclasses.replace(cfg, vocab=256, n_layers=1)
    lw = layer_from_parts(small, {k: torch.from_numpy(v) for k, v in parts.items()}, "cuda")
    rng = np.random.default_rng(9)
    embed = torch.from_numpy(rng.normal(0, 0.02, (256, cfg.hidden)).astype(np.float16)).cuda()
    from llamamps_b200.quant import pack_q4
    lp, ls = pack_q4(embed.float())
    mw = ModelWeights(small, [lw], torch.ones(cfg.hidden, dtype=torch.float16, device="cuda"), lp, ls, embed)
    return QwenEngine(weights=mw, max_seq_len=max_seq, page_order=page_order)


@pytest.mark.parametrize("seed,prefix", [(0, 31), (1, 0), (2, 63), (3, 64)])
def test_one_layer_decode_step(cuda, seed, prefix):
    from llamamps_b200.config import QWEN2_5_1_5B as cfg
    from llamamps_b200.weights import parts_host_arrays, synth_one_layer_case
    parts, x, kp, vp = synth_one_layer_case(cfg, seed=seed, prefix=prefix)
    order = list(np.random.default_rng(seed).permutation(2))
    eng = _one_layer_engine(parts, cfg, max_seq=128, page_order=order)
    eng.reset(1, start_pos=prefix)
    if prefix:
        eng.cache.write_positions(0, 0, 0, torch.from_numpy(kp), torch.from_numpy(vp))
    eng.buf_residual[0].copy_(torch.from_numpy(x))
    eng._layers(1)
    torch.cuda.synchronize()
    got = eng.buf_residual[0].cpu().numpy()

    ocfg = M.OracleConfig()
    cache = M.KVCache(1, ocfg.kv_dim)
    if prefix:
        cache.set_prefix(0, kp, vp)
    tr = {}
    ref = M.decoder_layer(x, parts_host_arrays(parts), cache, 0, prefix, ocfg, trace=tr)
    assert_close(got, ref, what="layer output")
    kk, vv = eng.cache.read_positions(0, 0, prefix + 1)
    assert_close(kk[-1].cpu().numpy(), tr["k"], what="appended k")
    assert_close(vv[-1].cpu().numpy(), tr["v"], what="appended v")
    assert_close(eng.buf_attn[0].cpu().numpy(), tr["attn"], what="attention output")
    assert_close(eng.buf_mlp[0].cpu().numpy(), tr["a"], what="swiglu output")
