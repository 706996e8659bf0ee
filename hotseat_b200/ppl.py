"""Mean negative log-likelihood over a token stream, the protocol of
hs-engine examples/ppl.rs (and llama-perplexity): independent windows of
`ctx` tokens, each decoded from position 0; only the second half of each
window is scored, so every scored token has at least ctx/2 tokens of
context behind it. A token's score is -log softmax(logits)[next] computed on
the device (hs_scratch_nll / hs_batch_nll: max-shifted, exp_f32, f64 sum).

    python -m hotseat_b200.ppl MODEL.gguf TEXT [ctx] [--numeric reference|fast|tc] [--ids]

TEXT is tokenized by the model's own byte-level BPE (hotseat_b200.tok), or,
with --ids, read as whitespace-separated token ids. On the tensor-core path
the windows are decoded together as one batch, position by position.
"""
import argparse
import math
import sys

import numpy as np

import hotseat_b200 as hs

NUMERIC = {"reference": hs.NUMERIC_REFERENCE, "fast": hs.NUMERIC_FAST, "tc": hs.NUMERIC_TC}


def score(model, ids, ctx=256):
    """ppl.rs on `model` (a hs.Model loaded with max_ctx >= ctx) over token
    ids: returns tokens, windows, scored, mean_nll and ppl."""
    ids = [int(t) for t in ids]
    chunks = len(ids) // ctx
    windows = [ids[c * ctx:(c + 1) * ctx] for c in range(chunks)]
    terms = [[] for _ in windows]  # per window, in position order
    if model.cfg.numeric == hs.NUMERIC_TC:
        if windows:
            b = hs.Batch(model, len(windows))
            kvs = [model.kv() for _ in windows]
            for p in range(ctx):
                b.forward(kvs, [w[p] for w in windows], [p] * len(windows))
                if p >= ctx // 2 and p + 1 < ctx:
                    for c, v in enumerate(b.nll([w[p + 1] for w in windows])):
                        terms[c].append(float(v))
            for kv in kvs:
                kv.close()
            b.close()
    else:
        kv, s = model.kv(), model.scratch()
        for c, w in enumerate(windows):
            for p, t in enumerate(w):
                model.forward(kv, t, p, s)
                if p >= ctx // 2 and p + 1 < len(w):
                    terms[c].append(s.nll(w[p + 1]))
        kv.close()
        s.close()
    nll = 0.0
    counted = 0
    for ws in terms:  # the reference's order: window by window, position by position
        for v in ws:
            nll += v
            counted += 1
    mean = nll / counted if counted else float("nan")
    return {"tokens": len(ids), "windows": chunks, "ctx": ctx, "scored": counted, "mean_nll": mean,
            "ppl": math.exp(mean) if counted else float("nan")}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("model")
    ap.add_argument("text")
    ap.add_argument("ctx", nargs="?", type=int, default=256)
    ap.add_argument("--numeric", default="fast", choices=sorted(NUMERIC))
    ap.add_argument("--ids", action="store_true", help="TEXT holds token ids, not text")
    ap.add_argument("--device", type=int, default=0)
    a = ap.parse_args(argv)
    raw = open(a.text, encoding="utf-8").read()
    if a.ids:
        ids = [int(x) for x in raw.split()]
    else:
        from hotseat_b200 import tok
        ids = tok.Tokenizer.from_gguf(a.model).encode(raw)
    m = hs.Model.load(a.model, max_ctx=a.ctx, device=a.device, numeric=NUMERIC[a.numeric])
    r = score(m, ids, a.ctx)
    print(f"tokens {r['tokens']} | windows {r['windows']} of {r['ctx']} | scored {r['scored']} | "
          f"mean NLL {r['mean_nll']:.5f} | ppl {r['ppl']:.5f}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
