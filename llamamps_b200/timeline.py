"""Stage timeline of the persistent decode kernel.

``capture(engine, steps)`` runs ``steps`` decode steps in one traced launch
(``lmps_decode_state.trace``: a %globaltimer stamp per CTA at the start of
every stage, once its input is staged in shared memory, once its compute is
done and at its end; the
producer's first/last chunk issue per stage and the consumers' cumulative
wait for weights) and reduces it to per-stage-kind numbers: the hand-off
latency (last CTA's end of the previous stage to the first CTA's start), the
stage span, the median per-CTA compute time and its staging part, the median
time spent waiting for the weight ring, and how far ahead of the consumers the
producer finished issuing.
"""
from __future__ import annotations

from typing import Dict

import numpy as np
import torch

KINDS = ("QKV", "ATT", "O", "GU", "DN")
WEIGHT_KINDS = ("QKV", "O", "GU", "DN")
# consumer stamps per stage: start (inputs polled from here), input staged,
# compute done (the ring chunks consumed), end (epilogue published)
EV = 4


def capture(engine, steps: int = 4) -> Dict:
    if engine.pdec is None:
        raise ValueError("the stage timeline belongs to the persistent decoder")
    L = engine.layers
    sms = torch.cuda.get_device_properties(engine.device).multi_processor_count
    n_stage = L * len(KINDS) + 1
    events = steps * n_stage * EV + 8
    trace = torch.zeros(3 * sms, events, dtype=torch.int64, device=engine.device)
    B = engine.batch
    engine.pdec.run(B, engine.tokens, engine.pos, steps, trace=trace)
    torch.cuda.synchronize(engine.device)
    engine.pdec.check_error()
    engine.host_pos += steps
    t = trace.cpu().numpy().astype(np.int64)
    cons, prod, wait = t[:sms], t[sms:2 * sms], t[2 * sms:3 * sms]
    # CTAs dedicated to attention (short contexts) record no stage events
    active = (cons != 0).any(axis=1)
    cons, prod, wait = cons[active], prod[active], wait[active]
    names = [f"L{l}.{k}" for l in range(L) for k in KINDS] + ["HEAD"]
    pnames = [f"L{l}.{k}" for l in range(L) for k in WEIGHT_KINDS] + ["HEAD"]
    step = steps // 2  # a middle step
    agg: Dict[str, Dict[str, list]] = {}
    prev_end = None
    for i, n in enumerate(names):
        e = (step * n_stage + i) * EV
        st, sg, cm, en = cons[:, e], cons[:, e + 1], cons[:, e + 2], cons[:, e + 3]
        kind = n.split(".")[-1]
        a = agg.setdefault(kind, {"handoff_us": [], "span_us": [], "cta_us": [], "staging_us": [],
                                  "compute_us": [], "epilogue_us": [], "ring_wait_us": []})
        if prev_end is not None:
            a["handoff_us"].append((st.min() - prev_end) / 1e3)
        a["span_us"].append((en.max() - st.min()) / 1e3)
        a["cta_us"].append(float(np.median((en - st) / 1e3)))
        a["staging_us"].append(float(np.median((sg - st) / 1e3)))
        a["compute_us"].append(float(np.median((cm - sg) / 1e3)))
        a["epilogue_us"].append(float(np.median((en - cm) / 1e3)))
        a["ring_wait_us"].append(float(np.median((wait[:, e + 3] - wait[:, e]) / 1e3)))
        prev_end = en.max()
    for i, n in enumerate(pnames):
        e = (step * len(pnames) + i) * 2
        kind = n.split(".")[-1]
        ci = names.index(n)
        ce = (step * n_stage + ci) * EV
        lead = np.median((cons[:, ce] - prod[:, e + 1]) / 1e3)
        agg.setdefault(kind, {}).setdefault("producer_lead_us", []).append(float(lead))
    step_us = []
    for s in range(steps):
        e0, e1 = (s * n_stage) * EV, (s * n_stage + n_stage - 1) * EV + EV - 1
        step_us.append(float((cons[:, e1].max() - cons[:, e0].min()) / 1e3))
    out = {"steps": steps, "step_span_us": step_us, "stages": {}}
    for k, a in agg.items():
        out["stages"][k] = {m: round(float(np.mean(v)), 3) for m, v in a.items() if v}
        if "span_us" in a:
            out["stages"][k]["count_per_step"] = len(a["span_us"])
    return out
