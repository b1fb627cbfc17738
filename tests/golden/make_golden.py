"""Generate the golden fixtures in tests/golden/ from the reference itself.

Runs the reference's own CPU code (oracle/_ref/libdqmref.so, compiled from the
reference sources by oracle/Makefile) on the seeded synthetic inputs that the
tests and bench.py regenerate on any machine, and stores its outputs:

  gemv_cases.npz        LinearQ80 / LinearQ40 outputs for the standalone GEMV
                        shapes (the reference's own test shapes plus the
                        Qwen2-0.5B projection shapes; lm_head sampled).
  mini_model.npz        Per-token logits of a 2-layer Qwen2-shaped model
                        (Q8_0 and Q4_0) over a 12-token prompt, ForwardBatch.
  qwen2_0_5b_q8_0.json  Full-size Qwen2-0.5B-architecture Q8_0 model: 32 random
                        prompt ids, then 64 greedy decode steps; the tokens,
                        each step's top-1/top-2 logit margin and top-5, plus
                        sha256 digests of reference-quantized weight blocks.
  qwen2_0_5b_q4_0_ctx2048.json  Qwen2-0.5B-architecture with ggml-convention
                        Q4_0 weights: a 2048-id random prompt fills the KV cache,
                        then 128 greedy steps (same fields).

  qwen2_0_5b_q8_0_logits.npz  Whole logit vectors of the full-size Q8_0 model:
                        after the 32-id prompt (step 0), after 16 further
                        greedy tokens (step 16), and after a 602-id prompt run
                        through the reference's per-token ForwardBatch (the
                        batched-prefill workload), with that prompt's digest.
  qwen2_0_5b_q4_0_ctx2048_logits.npz  Whole logit vectors of the Q4_0 model
                        after its 2048-id prompt (step 0) and at step 64.

Usage: python tests/golden/make_golden.py [--skip-full] [--q4-long] [--logits] [--q4-logits]
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
import __graft_entry__ as ge  # noqa: E402

S = ge.load_package().synth
O = ge.load_oracle()

GEMV_CASES = [
    # (qtype, out, in, seed): tests/test_cuda_quant.cc:304-411 shapes, a tail
    # case (tests/quant_test.cc:168-197) and the Qwen2-0.5B projections.
    (S.Q80, 5, 13, 1), (S.Q80, 32, 64, 2), (S.Q80, 17, 65, 3), (S.Q80, 2, 42, 4),
    (S.Q80, 896, 896, 10), (S.Q80, 128, 896, 11), (S.Q80, 4864, 896, 12),
    (S.Q80, 896, 4864, 13), (S.Q80, 151936, 896, 14),
    (S.Q40, 5, 13, 21), (S.Q40, 17, 65, 22), (S.Q40, 896, 896, 30), (S.Q40, 4864, 896, 31),
    (S.Q40, 896, 4864, 32),
]


def sample_idx(n: int) -> np.ndarray:
    step = max(1, n // 4096)
    return np.arange(0, n, step, dtype=np.int64)


def make_gemv():
    out = {}
    for qt, o, i, seed in GEMV_CASES:
        blocks, x = S.gemv_case(o, i, seed, qt)
        y = O.linear(qt, x, blocks, o, use_ref=True)
        idx = sample_idx(o)
        key = f"q{qt}_{o}x{i}_s{seed}"
        out[key + "_idx"] = idx
        out[key + "_y"] = y[idx]
    np.savez_compressed(os.path.join(HERE, "gemv_cases.npz"), **out)


def make_mini():
    out = {}
    for qt in (S.Q80, S.Q40):
        w = S.make_model(S.QWEN2_MINI, qt, 2024, quantize_q80=lambda a: O.quantize_q80(a, True))
        toks = S.prompt_tokens(w.cfg["vocab"], 12, 77)
        rm = O.RefModel(w, 64)
        logits = np.stack([rm.forward_batch([int(t)], i) for i, t in enumerate(toks)])
        out[f"q{qt}_tokens"] = toks
        out[f"q{qt}_logits"] = logits
    np.savez_compressed(os.path.join(HERE, "mini_model.npz"), **out)


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def make_full(threads: int):
    t0 = time.time()
    seed, prompt_seed, n_prompt, n_steps = 20261201, 1, 32, 64
    quant = lambda a: O.quantize_q80(a, True)  # the reference's QuantizeToQ80
    w = S.make_model(S.QWEN2_0_5B, S.Q80, seed, quantize_q80=quant)
    t1 = time.time()
    rm = O.RefModel(w, n_prompt + n_steps, threads=threads)
    prompt = S.prompt_tokens(w.cfg["vocab"], n_prompt, prompt_seed)
    logits = rm.forward_batch(prompt, 0)
    t2 = time.time()
    tokens, margins, top5 = [], [], []
    pos = n_prompt
    for step in range(n_steps):
        order = np.argsort(-logits, kind="stable")[:5]
        nxt = int(O.argmax(logits, use_ref=True))
        assert nxt == int(order[0])
        tokens.append(nxt)
        margins.append(float(logits[order[0]] - logits[order[1]]))
        top5.append([[int(k), float(logits[k])] for k in order])
        if step + 1 < n_steps:
            logits = rm.forward_batch([nxt], pos)
            pos += 1
    t3 = time.time()
    res = {
        "workload": "qwen2-0.5b-architecture, random-init N(0,0.02), Q8_0 (reference "
                    "QuantizeToQ80), tied embeddings; 32 prompt ids then 64 greedy steps",
        "model_seed": seed, "prompt_seed": prompt_seed, "prompt": [int(t) for t in prompt],
        "greedy_tokens": tokens, "top1_top2_margin": margins, "top5": top5,
        "logit_range_first_step": float(top5[0][0][1]),
        "digests": {"token_embd": digest(w.token_embd), "layers.0.wq": digest(w.layers[0].wq),
                    "layers.23.w_down": digest(w.layers[23].w_down)},
        "reference_threads": threads,
        "seconds": {"synth": t1 - t0, "prefill_32": t2 - t1, "decode_64": t3 - t2},
    }
    with open(os.path.join(HERE, "qwen2_0_5b_q8_0.json"), "w") as f:
        json.dump(res, f, indent=1)
    print(json.dumps(res["seconds"]))


def make_q4_long(threads: int):
    t0 = time.time()
    seed, prompt_seed, n_prompt, n_steps = 20261202, 3, 2048, 128
    w = S.make_model(S.QWEN2_0_5B, S.Q40, seed)
    rm = O.RefModel(w, n_prompt + n_steps, threads=threads)
    prompt = S.prompt_tokens(w.cfg["vocab"], n_prompt, prompt_seed)
    t1 = time.time()
    logits = rm.forward_batch(prompt, 0)
    t2 = time.time()
    tokens, margins, top5 = [], [], []
    pos = n_prompt
    for step in range(n_steps):
        order = np.argsort(-logits, kind="stable")[:5]
        nxt = int(order[0])
        tokens.append(nxt)
        margins.append(float(logits[order[0]] - logits[order[1]]))
        top5.append([[int(k), float(logits[k])] for k in order])
        if step + 1 < n_steps:
            logits = rm.forward_batch([nxt], pos)
            pos += 1
    t3 = time.time()
    res = {
        "workload": "qwen2-0.5b-architecture, random-init N(0,0.02), Q4_0 (ggml convention), "
                    "tied embeddings; 2048 prompt ids then 128 greedy steps",
        "model_seed": seed, "prompt_seed": prompt_seed, "n_prompt": n_prompt,
        "prompt_sha256": digest(prompt), "greedy_tokens": tokens, "top1_top2_margin": margins,
        "top5": top5, "digests": {"token_embd": digest(w.token_embd),
                                  "layers.0.wq": digest(w.layers[0].wq)},
        "reference_threads": threads,
        "seconds": {"build": t1 - t0, "prefill_2048": t2 - t1, "decode_128": t3 - t2},
    }
    with open(os.path.join(HERE, "qwen2_0_5b_q4_0_ctx2048.json"), "w") as f:
        json.dump(res, f, indent=1)
    print(json.dumps(res["seconds"]))


def make_full_logits(threads: int):
    t0 = time.time()
    seed, prompt_seed = 20261201, 1
    w = S.make_model(S.QWEN2_0_5B, S.Q80, seed, quantize_q80=lambda a: O.quantize_q80(a, True))
    rm = O.RefModel(w, 602, threads=threads)
    prompt = S.prompt_tokens(w.cfg["vocab"], 32, prompt_seed)
    logits = rm.forward_batch(prompt, 0)
    out = {"step0": logits.astype(np.float32)}
    pos, steps = 32, 16
    for _ in range(steps):
        tok = int(O.argmax(logits, use_ref=True))
        logits = rm.forward_batch([tok], pos)
        pos += 1
    out["step16"] = logits.astype(np.float32)
    t1 = time.time()
    rm.reset()
    p602 = S.prompt_tokens(w.cfg["vocab"], 602, 4)
    out["prefill602"] = rm.forward_batch(p602, 0).astype(np.float32)
    t2 = time.time()
    out["prefill602_prompt_sha256"] = np.frombuffer(digest(p602).encode(), np.uint8)
    out["prefill602_seconds"] = np.array([t2 - t1, threads], np.float64)
    np.savez_compressed(os.path.join(HERE, "qwen2_0_5b_q8_0_logits.npz"), **out)
    print(json.dumps({"decode_s": t1 - t0, "prefill602_s": t2 - t1, "threads": threads}))


def make_q4_logits(threads: int):
    seed, prompt_seed, n_prompt = 20261202, 3, 2048
    w = S.make_model(S.QWEN2_0_5B, S.Q40, seed)
    rm = O.RefModel(w, n_prompt + 65, threads=threads)
    prompt = S.prompt_tokens(w.cfg["vocab"], n_prompt, prompt_seed)
    logits = rm.forward_batch(prompt, 0)
    out = {"step0": logits.astype(np.float32)}
    pos = n_prompt
    for _ in range(64):
        tok = int(np.argmax(logits))
        logits = rm.forward_batch([tok], pos)
        pos += 1
    out["step64"] = logits.astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "qwen2_0_5b_q4_0_ctx2048_logits.npz"), **out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--skip-full", action="store_true")
    ap.add_argument("--q4-long", action="store_true")
    ap.add_argument("--threads", type=int, default=os.cpu_count())
    ap.add_argument("--logits", action="store_true")
    ap.add_argument("--q4-logits", action="store_true")
    args = ap.parse_args()
    if args.logits:
        make_full_logits(args.threads)
        return
    if args.q4_logits:
        make_q4_logits(args.threads)
        return
    if args.q4_long:
        make_q4_long(args.threads)
        return
    make_gemv()
    make_mini()
    if not args.skip_full:
        make_full(args.threads)


if __name__ == "__main__":
    main()
