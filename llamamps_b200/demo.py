"""The reference's generate flow (demo.py:14-20, utils/tokenizer.py:13-28) on B200.

The reference's ``demo.main`` tokenises a prompt, looks up the embedding row
of the FIRST token only (``utils/tokenizer.py:24-26``) and hands that vector
straight to ``predict_next_token`` (``demo.py:17-18``): the forward pass never
runs.  Here every prompt id goes through the model (prefill), then greedy
decode continues from the last position:

    engine = QwenEngine(weights_dir)
    input_vec, ids = get_input_vector(prompt_ids, embed_path)   # the reference's contract
    out = engine.generate(ids, max_new_tokens)                   # all ids, then greedy

``get_input_vector`` keeps the reference's return value (the first token's
fp16 embedding row and the token ids).  The Hugging Face tokenizer the
reference downloads at import time (``utils/tokenizer.py:10``) needs the
network; a caller that has one passes it (anything with ``encode(text,
add_special_tokens=True)``), otherwise the prompt is given as token ids.

    python -m llamamps_b200.demo --weights DIR --ids 785,6722,315,6864,374 --new 16
    python -m llamamps_b200.demo --synthetic --ids 1,2,3 --new 8     # random-init model
"""
from __future__ import annotations

import argparse
import os
import sys
from typing import List, Optional, Sequence, Tuple, Union

import numpy as np

from .config import QWEN2_5_1_5B, ModelConfig


def _ids(prompt: Union[str, Sequence[int]], tokenizer=None) -> List[int]:
    if isinstance(prompt, str):
        if tokenizer is None:
            raise ValueError("a text prompt needs a tokenizer (the Qwen2.5 files are not available offline); "
                             "pass token ids instead")
        return [int(t) for t in tokenizer.encode(prompt, add_special_tokens=True)]   # utils/tokenizer.py:18
    return [int(t) for t in prompt]


def get_input_vector(prompt: Union[str, Sequence[int]], embed_path: Optional[str] = None, tokenizer=None,
                     hidden: int = QWEN2_5_1_5B.hidden) -> Tuple[np.ndarray, List[int]]:
    """utils/tokenizer.py:13-28: the fp16 embedding row of the prompt's first
    token (read from ``<weights>/global/embed_tokens.bin``) and the token ids.
    Reads only that row, where the reference loads the whole 466 MB table."""
    ids = _ids(prompt, tokenizer)
    if not ids:
        raise ValueError("empty prompt")
    if embed_path is None:
        raise ValueError("embed_path is the weights directory's global/embed_tokens.bin")
    n_rows = os.path.getsize(embed_path) // (2 * hidden)
    if not 0 <= ids[0] < n_rows:
        raise ValueError(f"token id {ids[0]} outside the {n_rows}-row embedding table")
    table = np.memmap(embed_path, dtype=np.float16, mode="r", shape=(n_rows, hidden))
    return np.array(table[ids[0]]), ids


def generate(engine, prompt: Union[str, Sequence[int]], max_new_tokens: int, tokenizer=None) -> List[int]:
    """demo.py:14-20 with the forward pass: every prompt id through the model,
    then ``max_new_tokens`` greedy tokens (engine.predict_next_token's
    first-index argmax, on the device)."""
    return engine.generate(_ids(prompt, tokenizer), max_new_tokens)


def main(argv: Optional[Sequence[str]] = None, config: ModelConfig = QWEN2_5_1_5B) -> List[int]:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--weights", default=None, help="directory in the reference's flat-.bin layout")
    ap.add_argument("--synthetic", action="store_true", help="random-init weights instead (seeded)")
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--ids", required=True, help="comma-separated prompt token ids")
    ap.add_argument("--new", type=int, default=16, help="tokens to generate")
    a = ap.parse_args(argv)
    import torch
    from .engine import QwenEngine
    ids = [int(t) for t in a.ids.split(",") if t.strip()]
    max_seq = len(ids) + a.new + 1
    if a.synthetic:
        from .weights import synth_model
        engine = QwenEngine(weights=synth_model(config, seed=a.seed, device="cuda"), max_seq_len=max_seq)
        embed_row = engine.weights.embed[ids[0]].cpu().numpy()
    elif a.weights:
        engine = QwenEngine(a.weights, config=config, max_seq_len=max_seq)
        embed_row, _ = get_input_vector(ids, os.path.join(a.weights, "global", "embed_tokens.bin"),
                                        hidden=config.hidden)
    else:
        ap.error("give --weights DIR or --synthetic")
    # the reference's single-token step (run_inference on the first token's
    # row, then the host argmax) -- what demo.py meant to print
    first = engine.predict_next_token(engine.run_inference(embed_row))
    out = generate(engine, ids, a.new)
    torch.cuda.synchronize()
    print(f"Input token IDs: {ids}")
    print(f"Predicted token ID after the first token: {first}")
    print(f"Generated token IDs: {out}")
    return out


if __name__ == "__main__":
    main(sys.argv[1:])
