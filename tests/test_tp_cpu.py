"""Tensor-parallel split on the host: the Q4 weight sharding and the
partial-sum + all-reduce decomposition of a decoder layer, run as two gloo
ranks with the oracle's arithmetic per rank, against the unsplit oracle layer
(config 0: one layer, one step, 31 cached positions)."""
import dataclasses
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import mirror as M
from tests._util import assert_close


def _cfgs():
    from llamamps_b200.config import QWEN2_5_1_5B
    from llamamps_b200.tp import local_config
    return QWEN2_5_1_5B, local_config(QWEN2_5_1_5B, 2)


def _layer_cpu():
    from llamamps_b200.weights import layer_from_parts, synth_one_layer_case
    cfg, _ = _cfgs()
    parts, x, kp, vp = synth_one_layer_case(cfg, seed=0, prefix=31)
    lw = layer_from_parts(cfg, {k: torch.from_numpy(v) for k, v in parts.items()}, "cpu")
    return parts, lw, x, kp, vp


def test_shard_rows_and_columns_are_slices_of_the_dequantised_matrix():
    from llamamps_b200.tp import shard_layer
    from llamamps_b200.weights import layer_host_arrays
    cfg, loc = _cfgs()
    _, lw, _, _, _ = _layer_cpu()
    full = layer_host_arrays(lw, cfg)
    for r in (0, 1):
        sh = layer_host_arrays(shard_layer(lw, cfg, r, 2), loc)
        q = M.q4_dequant(full["q"], full["qs"], cfg.q_dim, cfg.hidden)
        assert np.array_equal(M.q4_dequant(sh["q"], sh["qs"], loc.q_dim, cfg.hidden),
                              q[r * loc.q_dim:(r + 1) * loc.q_dim])
        k = M.q4_dequant(full["k"], full["ks"], cfg.kv_dim, cfg.hidden)
        assert np.array_equal(M.q4_dequant(sh["k"], sh["ks"], loc.kv_dim, cfg.hidden),
                              k[r * loc.kv_dim:(r + 1) * loc.kv_dim])
        o = M.q4_dequant(full["o"], full["os"], cfg.hidden, cfg.q_dim)
        assert np.array_equal(M.q4_dequant(sh["o"], sh["os"], cfg.hidden, loc.q_dim),
                              o[:, r * loc.q_dim:(r + 1) * loc.q_dim])
        d = M.q4_dequant(full["dn"], full["dns"], cfg.hidden, cfg.intermediate)
        assert np.array_equal(M.q4_dequant(sh["dn"], sh["dns"], cfg.hidden, loc.intermediate),
                              d[:, r * loc.intermediate:(r + 1) * loc.intermediate])
        assert np.array_equal(sh["bv"], full["bv"][r * loc.kv_dim:(r + 1) * loc.kv_dim])


def _rank_layer(rank, world, port, out):
    """One rank: its slice of the layer with the oracle's arithmetic and
    gloo all-reduces where the GPU engine uses NCCL."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from llamamps_b200.tp import shard_layer
        from llamamps_b200.weights import layer_host_arrays
        cfg, loc = _cfgs()
        _, lw, x, kp, vp = _layer_cpu()
        hl = layer_host_arrays(shard_layer(lw, cfg, rank, world), loc)
        ocfg = M.OracleConfig(n_layers=1, n_q_heads=loc.n_q_heads, n_kv_heads=loc.n_kv_heads,
                              intermediate=loc.intermediate)
        D, pos = cfg.hidden, 31
        sl = slice(rank * loc.kv_dim, (rank + 1) * loc.kv_dim)
        xn = M.rms_norm(x, hl["in_norm"], cfg.eps)
        accq = M._gemv_acc(hl, "q", xn, ocfg.q_dim, D, None)
        acck = M._gemv_acc(hl, "k", xn, ocfg.kv_dim, D, None)
        accv = M._gemv_acc(hl, "v", xn, ocfg.kv_dim, D, None)
        q = M.rope(M.add_bias(accq.astype(np.float16), accq, hl["bq"]), pos, 128, cfg.rope_theta, cfg.rope_style)
        k = M.rope(M.add_bias(acck.astype(np.float16), acck, hl["bk"]), pos, 128, cfg.rope_theta, cfg.rope_style)
        v = M.add_bias(accv.astype(np.float16), accv, hl["bv"])
        kc = np.concatenate([kp[:, sl], k[None]]).astype(np.float16)
        vc = np.concatenate([vp[:, sl], v[None]]).astype(np.float16)
        s = M.attention_scores(q, kc, ocfg.n_q_heads, ocfg.n_kv_heads, 128)
        attn = M.attn_weighted_sum(M.softmax(s), vc, ocfg.n_q_heads, ocfg.n_kv_heads, 128)
        o_part = torch.from_numpy(M._gemv_acc(hl, "o", attn, D, ocfg.q_dim, None).astype(np.float16).astype(np.float32))
        dist.all_reduce(o_part)
        x1 = M.residual_add(x, o_part.numpy().astype(np.float16))
        hn = M.rms_norm(x1, hl["post_norm"], cfg.eps)
        g = M._gemv_acc(hl, "gt", hn, ocfg.intermediate, D, None).astype(np.float16)
        u = M._gemv_acc(hl, "up", hn, ocfg.intermediate, D, None).astype(np.float16)
        a = M.swiglu(g, u)
        d_part = torch.from_numpy(M._gemv_acc(hl, "dn", a, D, ocfg.intermediate, None).astype(np.float16).astype(np.float32))
        dist.all_reduce(d_part)
        x2 = M.residual_add(x1, d_part.numpy().astype(np.float16))
        out[rank] = torch.from_numpy(x2.astype(np.float32))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_layer_matches_unsplit_oracle():
    from llamamps_b200.weights import parts_host_arrays
    parts, _, x, kp, vp = _layer_cpu()
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank_layer, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        assert p.exitcode == 0
    ocfg = M.OracleConfig(n_layers=1)
    cache = M.KVCache(1, ocfg.kv_dim)
    cache.set_prefix(0, kp, vp)
    ref = M.decoder_layer(x, parts_host_arrays(parts), cache, 0, 31, ocfg)
    r0, r1 = out[0].numpy(), out[1].numpy()
    assert np.array_equal(r0, r1), "ranks disagree on the replicated residual"
    assert_close(r0, ref, what="2-rank layer output vs unsplit oracle")
