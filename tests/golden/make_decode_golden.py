"""Generate tests/golden/decode_8b.json: 64 greedy tokens of the synthetic
Llama-3-8B-architecture Q4_K_M model, decoded by the CPU oracle (the
reference's Transformer.Forward restated in oracle/oracle.cpp) from a KV cache
prefilled with 4096 seeded f16 positions.

The weights are the library's seeded recipe (si_model_tensor_recipe): Q4_K
projections and token embedding, Q6_K lm_head, f32 norms 1 + 0.01 N(0,1).
Per step the file records the token, the top-1/top-2 logit margin and the
top-1 logit, so a GPU run can be judged against margins.

Run from the repository root (about 10 minutes on 8 cores, ~6 GB RAM):
    python tests/golden/make_decode_golden.py [--steps 64]
"""
import argparse
import json
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from sharpinfer_b200.model import llama3_8b  # noqa: E402

SEED = 20261201
KV_LEN = 4096
START_TOKEN = 128000  # Llama-3 <|begin_of_text|> id; any id < vocab works


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--out", default=os.path.join(os.path.dirname(os.path.abspath(__file__)), "decode_8b.json"))
    args = ap.parse_args()
    cfg = llama3_8b(max_seq=KV_LEN + args.steps)
    t0 = time.time()
    om = oracle.synthetic_model(cfg, SEED, n_seq=1, kv_len=KV_LEN)
    print("model built in %.1fs" % (time.time() - t0), flush=True)
    tok = START_TOKEN
    rec = []
    for s in range(args.steps):
        t1 = time.time()
        logits = om.forward(0, tok, KV_LEN + s)
        nxt = oracle.argmax(logits)
        top = np.sort(logits)[-2:]
        rec.append({"pos": KV_LEN + s, "input": int(tok), "token": int(nxt), "top1": float(top[1]),
                    "margin": float(top[1] - top[0])})
        print("step %d token %d margin %.5f (%.1fs)" % (s, nxt, top[1] - top[0], time.time() - t1), flush=True)
        tok = nxt
    out = {"seed": SEED, "kv_len": KV_LEN, "start_token": START_TOKEN, "steps": args.steps,
           "config": {f: getattr(cfg, f) for f, _ in cfg._fields_}, "records": rec,
           "tokens": [r["token"] for r in rec], "min_margin": min(r["margin"] for r in rec)}
    json.dump(out, open(args.out, "w"), indent=1)
    print("wrote", args.out, "min margin", out["min_margin"])


if __name__ == "__main__":
    main()
