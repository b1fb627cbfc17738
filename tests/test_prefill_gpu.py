"""GPU parity of the batched prefill (ForwardBatch over consecutive positions).

The reference's ForwardBatch runs ForwardToken once per token
(src/batch.cc:35-40).  Here a prompt runs layer by layer as tcgen05
tensor-core GEMMs (two-term fp16 activations times exact two-term fp16
weights, fp32 accumulation) plus causal attention, so its logits and KV
cache are compared with the reference within the logit tolerance
(max |logit - ref| <= 1e-3 x the reference's logit range), and decoding
after it must continue exactly as the reference does.
"""
import os

import numpy as np
import pytest

from conftest import golden_path

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3


def check_logits(got, ref, label):
    rng = float(ref.max() - ref.min())
    err = float(np.abs(got - ref).max())
    assert err <= LOGIT_TOL * rng, f"{label}: max err {err:.3e} > {LOGIT_TOL} * range {rng:.3f}"
    return err / rng


@pytest.fixture(scope="module")
def minis(pkg, S, cuda):
    return {qt: S.make_model(S.QWEN2_MINI, qt, 2024,
                             quantize_q80=lambda a: pkg.QuantizeToQ80(a).cpu().numpy())
            for qt in (pkg.Q80, pkg.Q40)}


@pytest.fixture(scope="module")
def mini_q8(minis, pkg):
    return minis[pkg.Q80]


class env_var:
    """Sets one environment variable for the duration of a block."""

    def __init__(self, name, value):
        self.name, self.value = name, value

    def __enter__(self):
        self.old = os.environ.get(self.name)
        os.environ[self.name] = self.value

    def __exit__(self, *exc):
        if self.old is None:
            del os.environ[self.name]
        else:
            os.environ[self.name] = self.old


class per_token_path:
    """DQMK_PREFILL=0: ForwardBatch replays the decode graph per token."""

    def __enter__(self):
        self.old = os.environ.get("DQMK_PREFILL")
        os.environ["DQMK_PREFILL"] = "0"

    def __exit__(self, *exc):
        if self.old is None:
            del os.environ["DQMK_PREFILL"]
        else:
            os.environ["DQMK_PREFILL"] = self.old


@pytest.mark.parametrize("qt", [1, 2])
def test_prefill_then_decode_matches_reference_golden(pkg, minis, cuda, qt):
    """8 prompt tokens batched, then 4 ForwardToken steps that attend over the
    KV cache the prefill wrote; every logits vector against the reference
    (Q8_0, and Q4_0 whose dequantized values the prefill splits into fp16
    planes once)."""
    g = np.load(golden_path("mini_model.npz"))
    toks = g[f"q{qt}_tokens"]
    ref = g[f"q{qt}_logits"]
    ctx = pkg.Context(pkg.Model.from_synth(minis[qt], max_seq_len=64))
    worst = check_logits(ctx.ForwardBatch([int(t) for t in toks[:8]], 0), ref[7], "prefill")
    for i in range(8, len(toks)):
        worst = max(worst, check_logits(ctx.ForwardToken(int(toks[i]), i), ref[i], f"step {i}"))
    print(f"worst relative logit error {worst:.2e}")


def test_prefill_matches_per_token_path(pkg, mini_q8, cuda):
    """Batched and per-token ForwardBatch agree (the reference asserts exact
    equality, tests/batch_test.cc:157-217, because its batch IS per-token; the
    per-token path here is still exact, the batched one within tolerance)."""
    model = pkg.Model.from_synth(mini_q8, max_seq_len=64)
    toks = [1, 104, 101, 108, 108, 111, 7, 900, 3, 44]
    with per_token_path():
        a = pkg.Context(model)
        la = a.ForwardBatch(toks, 0)
        manual = pkg.Context(model)
        for i, t in enumerate(toks):
            lm = manual.ForwardToken(t, i)
        assert np.array_equal(la, lm)
    b = pkg.Context(model)
    lb = b.ForwardBatch(toks, 0)
    check_logits(lb, la, "batched vs per-token")
    assert b.token_history == toks and b.pos == len(toks) - 1
    # the caches agree too: one more token through the decode path
    check_logits(b.ForwardToken(5, len(toks)), a.ForwardToken(5, len(toks)), "next token")


def test_prefill_offset_start_and_second_batch(pkg, mini_q8, orc, cuda):
    """A batch that starts mid-sequence attends over what earlier calls cached."""
    model = pkg.Model.from_synth(mini_q8, max_seq_len=64)
    toks = [9, 8, 7, 6, 5, 4, 3, 2, 1, 10, 11, 12, 13]
    om = orc.OracleModel(mini_q8, 64)
    for i, t in enumerate(toks):
        ref = om.forward_token(t, i)
    ctx = pkg.Context(model)
    ctx.ForwardBatch(toks[:5], 0)
    ctx.ForwardBatch(toks[5:9], 5)
    check_logits(ctx.ForwardBatch(toks[9:], 9), ref, "three batches")


@pytest.mark.parametrize("attn", ["tc", "fma"])
def test_prefill_chunked_long_prompt_matches_reference(pkg, orc, S, mini_q8, cuda, attn):
    """1100 tokens: two chunks (1024 + 76 rows, the second starting at cache
    position 1024) of the batched path under either causal attention kernel;
    last logits against the reference's own ForwardBatch, then 16 greedy
    steps must equal the reference's."""
    n, steps = 1100, 16
    prompt = S.prompt_tokens(mini_q8.cfg["vocab"], n, 5).tolist()
    rm = orc.RefModel(mini_q8, n + steps)
    ref = rm.forward_batch(prompt, 0)
    ref_tokens, tok, margins = [], None, []
    lg = ref
    for i in range(steps):
        top2 = np.sort(lg)[-2:]
        margins.append(float(top2[1] - top2[0]))
        tok = int(np.argmax(lg))
        ref_tokens.append(tok)
        if i + 1 < steps:
            lg = rm.forward_batch([tok], n + i)
    ctx = pkg.Context(pkg.Model.from_synth(mini_q8, max_seq_len=n + steps))
    with env_var("DQMK_PREFILL_ATTN", attn):
        got = ctx.ForwardBatch(prompt, 0)
    print(f"{attn} attention: relative logit error {check_logits(got, ref, 'chunked prefill'):.2e}, "
          f"min margin {min(margins):.2e}")
    first = int(np.argmax(got))
    assert first == ref_tokens[0]
    rest = ctx.decode_greedy(first, n, steps - 1).tolist()
    assert [first] + rest == ref_tokens


def test_qwen2_0_5b_q4_0_ctx2048_prefill_then_128_greedy(pkg, S, cuda):
    """Qwen2-0.5B-architecture with ggml-convention Q4_0 weights: a 2048-id
    prompt through the batched prefill (two 1024-row chunks) fills the KV
    cache; the whole logit vector after the prompt and after 64 greedy steps
    must sit within 1e-3 x logit range of the reference's, and 128 greedy
    steps over the cache must equal the reference's tokens."""
    import hashlib
    import json

    g = json.load(open(golden_path("qwen2_0_5b_q4_0_ctx2048.json")))
    whole = np.load(golden_path("qwen2_0_5b_q4_0_ctx2048_logits.npz"))
    w = S.make_model(S.QWEN2_0_5B, S.Q40, g["model_seed"])
    sha = lambda a: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()
    assert sha(w.token_embd) == g["digests"]["token_embd"]
    n = g["n_prompt"]
    prompt = S.prompt_tokens(w.cfg["vocab"], n, g["prompt_seed"])
    assert sha(prompt) == g["prompt_sha256"]
    ctx = pkg.Context(pkg.Model.from_synth(w, max_seq_len=n + len(g["greedy_tokens"])))
    logits = ctx.ForwardBatch(prompt.tolist(), 0)
    err0 = check_logits(logits, whole["step0"], "2048-id prefill")
    first = int(np.argmax(logits))
    # greedy tokens 1..63, then the logits after 64 fed tokens
    tokens = [first] + ctx.decode_greedy(first, n, 63).tolist()
    logits = ctx.ForwardBatch([tokens[63]], n + 63)
    err64 = check_logits(logits, whole["step64"], "step 64 over the 2048-id cache")
    print(f"relative logit error: step 0 {err0:.2e}, step 64 {err64:.2e}")
    tok64 = int(np.argmax(logits))
    tokens += [tok64] + ctx.decode_greedy(tok64, n + 64, len(g["greedy_tokens"]) - 65).tolist()
    assert tokens == g["greedy_tokens"], (
        f"first divergence at {next(i for i, (a, b) in enumerate(zip(tokens, g['greedy_tokens'])) if a != b)}"
        f", reference min margin {min(g['top1_top2_margin']):.3e}")


@pytest.mark.parametrize("attn", ["tc", "fma"])
def test_qwen2_0_5b_q8_0_prefill_602_whole_logits(pkg, S, cuda, attn):
    """Configuration 4 at full size: the Qwen2-0.5B-architecture Q8_0 model
    (reference-quantized weights) runs one 602-id prompt as a single batched
    ForwardBatch (tensor-core GEMMs, causal attention); its whole 151936-entry
    logit vector must sit within 1e-3 x logit range of the reference's own
    per-token ForwardBatch loop over the same prompt.  Both causal attention
    kernels: tcgen05 (the default at head_dim 64) and fp32 FMA
    (DQMK_PREFILL_ATTN=fma)."""
    import hashlib

    g = np.load(golden_path("qwen2_0_5b_q8_0_logits.npz"))
    w = S.make_model(S.QWEN2_0_5B, S.Q80, 20261201,
                     quantize_q80=lambda a: pkg.QuantizeToQ80(a).cpu().numpy())
    prompt = S.prompt_tokens(w.cfg["vocab"], 602, 4)
    sha = hashlib.sha256(np.ascontiguousarray(prompt).tobytes()).hexdigest()
    assert sha == bytes(g["prefill602_prompt_sha256"]).decode()
    model = pkg.Model.from_synth(w, max_seq_len=602)
    ctx = pkg.Context(model)
    with env_var("DQMK_PREFILL_ATTN", attn):
        logits = ctx.ForwardBatch(prompt.tolist(), 0)
    err = check_logits(logits, g["prefill602"], f"602-token batched prefill ({attn} attention)")
    print(f"602-token prefill, {attn} attention: relative logit error {err:.2e}")
    assert int(np.argmax(logits)) == int(np.argmax(g["prefill602"]))
    ctx.close()
    model.close()



def test_prefix_reuse_matches_full_prefill(pkg, S, minis, cuda):
    """Prefix reuse (dqmk_forward_batch_prefix, the reference chat loop's
    reuse at src/main.cc:887-913): after a 300-token prompt and 6 greedy
    tokens, a second prompt that shares the first 200 tokens keeps those 200
    positions and batched-prefills only the rest; its logits and next greedy
    tokens equal a fresh context's full prefill of the second prompt (logits
    within 1e-3 x range).  The same prompt again, or one sharing nothing,
    recomputes from position 0."""
    w = minis[pkg.Q80]
    vocab = w.cfg["vocab"]
    p1 = S.prompt_tokens(vocab, 300, 21).tolist()
    p2 = p1[:200] + S.prompt_tokens(vocab, 150, 22).tolist()
    model = pkg.Model.from_synth(w, max_seq_len=512)
    ctx = pkg.Context(model)
    first = int(np.argmax(ctx.ForwardBatch(p1, 0)))
    ctx.decode_greedy(first, 300, 6)
    got, reused = ctx.ForwardBatchReuse(p2)
    assert reused == 200
    assert ctx.pos == len(p2) - 1
    fresh = pkg.Context(model)
    ref = fresh.ForwardBatch(p2, 0)
    check_logits(got, ref, "prefix reuse")
    nxt = int(np.argmax(got))
    assert ctx.decode_greedy(nxt, len(p2), 4).tolist() == fresh.decode_greedy(nxt, len(p2), 4).tolist()
    again, reused = ctx.ForwardBatchReuse(p2)
    assert reused == 0
    check_logits(again, ref, "same prompt, recomputed")
    other = S.prompt_tokens(vocab, 40, 23).tolist()
    _, reused = ctx.ForwardBatchReuse(other)
    assert reused == 0 and ctx.pos == 39
    ctx.close()
    fresh.close()
    model.close()
