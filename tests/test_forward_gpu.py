"""GPU parity of the whole decode path (engine + fused kernels) against the
reference: ForwardToken logits, ForwardBatch side effects, greedy tokens, and
the runtime counters the reference's CUDA tests assert.

Logit tolerance: max |logit - ref| <= 1e-3 * (max - min
of the reference logits).  Greedy decoding must produce identical tokens; the
smallest top-1/top-2 margin of each run is reported alongside.
"""
import json
import os

import numpy as np
import pytest

from conftest import golden_path

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3  # relative to the logit range


def check_logits(got, ref, label):
    rng = float(ref.max() - ref.min())
    err = float(np.abs(got - ref).max())
    assert err <= LOGIT_TOL * rng, f"{label}: max err {err:.3e} > {LOGIT_TOL} * range {rng:.3f}"
    return err / rng


@pytest.fixture(scope="module")
def mini(pkg, orc, S, cuda):
    out = {}
    for qt in (pkg.Q80, pkg.Q40):
        out[qt] = S.make_model(S.QWEN2_MINI, qt, 2024,
                               quantize_q80=lambda a: pkg.QuantizeToQ80(a).cpu().numpy())
    return out


@pytest.mark.parametrize("qt", [1, 2])
def test_forward_token_matches_reference_golden(pkg, mini, cuda, qt):
    g = np.load(golden_path("mini_model.npz"))
    w = mini[qt]
    model = pkg.Model.from_synth(w, max_seq_len=64)
    ctx = pkg.Context(model)
    toks = g[f"q{qt}_tokens"]
    worst = 0.0
    for i, t in enumerate(toks):
        logits = ctx.ForwardToken(int(t), i)
        worst = max(worst, check_logits(logits, g[f"q{qt}_logits"][i], f"q{qt} step {i}"))
    print(f"q{qt} worst relative logit error {worst:.2e}")


def test_forward_batch_semantics(pkg, mini, cuda):
    """tests/batch_test.cc:157-217: batched == per-token, pos / history updates."""
    w = mini[pkg.Q80]
    model = pkg.Model.from_synth(w, max_seq_len=64)
    toks = [1, 104, 101, 108, 108, 111]
    manual = pkg.Context(model)
    for i, t in enumerate(toks):
        manual_logits = manual.ForwardToken(t, i)
    batched = pkg.Context(model)
    os.environ["DQMK_PREFILL"] = "0"  # per-token replays: bit-identical to ForwardToken
    try:
        batch_logits = batched.ForwardBatch(toks, 0)
    finally:
        del os.environ["DQMK_PREFILL"]
    assert np.array_equal(batch_logits, manual_logits)
    assert batched.token_history == toks and batched.pos == 5
    assert manual.token_history == [] and manual.pos == 0  # ForwardToken touches neither
    batched.ForwardBatch([42], positions=[6])
    assert batched.token_history == toks + [42] and batched.pos == 6
    with pytest.raises(RuntimeError, match="ForwardBatch: empty token"):
        batched.ForwardBatch([], 0)
    with pytest.raises(pkg.OutOfRange, match="token id out of range"):
        batched.ForwardToken(w.cfg["vocab"], 0)
    with pytest.raises(pkg.OutOfRange, match="position out of range"):
        batched.ForwardToken(0, 64)


def test_runtime_counters(pkg, mini, cuda):
    """Per-logical-op counters as TestCudaForwardQuant asserts them
    (tests/test_cuda_quant.cc:442-472): Linear 7L+1, attention L per token,
    one logits download, no activation uploads."""
    w = mini[pkg.Q80]
    L = w.cfg["n_layers"]
    model = pkg.Model.from_synth(w, max_seq_len=16)
    s = model.stats()
    assert s["uploaded_weight_count"] == 2 + 12 * L  # embedding, final norm, 12 per layer
    model.reset_stats()
    ctx = pkg.Context(model)
    ctx.ForwardToken(3, 0)
    s = model.stats()
    assert s["linear_calls"] == 7 * L + 1
    assert s["attention_calls"] == L
    assert s["activation_calls"] == 10 * L + 1  # bias adds present in Qwen2
    assert s["device_to_host_copies"] == 1 and s["device_to_host_bytes"] == 4 * w.cfg["vocab"]
    assert s["host_to_device_copies"] == 0
    for i in range(1, 3):
        ctx.ForwardToken(3, i)
    assert model.stats()["linear_calls"] == 3 * (7 * L + 1)
    # packed weights occupy exactly the ggml block bytes plus resident F32
    c = w.cfg
    hd = c["dim"] // c["n_heads"]
    blocks = w.token_embd.nbytes + sum(getattr(Ly, n).nbytes for Ly in w.layers
                                       for n in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down"))
    f32 = 4 * (c["dim"] + L * (2 * c["dim"] + c["n_heads"] * hd + 2 * c["n_kv_heads"] * hd))
    assert model.memory_bytes() == blocks + f32
    # the first batched ForwardBatch builds the tensor-core side tables --
    # two fp16 planes per weight (4 bytes per weight, rows padded to 32
    # values) and a float scale per row -- and the accounting grows by them
    ctx.ForwardBatch([3, 4, 5, 6], 3)
    kp = lambda k: (k + 31) // 32 * 32
    rows_k = [(c["dim"] + 2 * c["n_kv_heads"] * hd, c["dim"]), (c["dim"], c["n_heads"] * hd),
              (2 * c["hidden"], c["dim"]), (c["dim"], c["hidden"])]
    planes = L * sum(r * 4 + 4 * r * kp(k) for r, k in rows_k)
    assert model.memory_bytes() == blocks + f32 + planes


@pytest.mark.parametrize("qt", [1, 2])
def test_greedy_decode_matches_oracle(pkg, orc, mini, cuda, qt):
    w = mini[qt]
    prompt = [5, 77, 300]
    n_steps = 20
    om = orc.OracleModel(w, 64)
    for i, t in enumerate(prompt[:-1]):
        om.forward_token(t, i)
    tok, ref_tokens, margins = prompt[-1], [], []
    for i in range(n_steps):
        lg = om.forward_token(tok, len(prompt) - 1 + i)
        top2 = np.sort(lg)[-2:]
        margins.append(float(top2[1] - top2[0]))
        tok = orc.argmax(lg)
        ref_tokens.append(tok)
    model = pkg.Model.from_synth(w, max_seq_len=64)
    ctx = pkg.Context(model)
    ctx.ForwardBatch(prompt[:-1], 0)
    got = ctx.decode_greedy(prompt[-1], len(prompt) - 1, n_steps)
    print(f"q{qt} min top1/top2 margin {min(margins):.3e}")
    assert got.tolist() == ref_tokens


@pytest.mark.parametrize("qt", [1, 2], ids=["q8_0", "q4_0"])
def test_tall_weights_match_oracle(pkg, orc, S, cuda, qt):
    """A model with tall gate/up (16384 rows x 2048) and lm_head (16384 x
    2048) weights: in Q8_0 both take the tensor-core GEMV (tcgen05 kind::i8,
    per-block sums in tensor memory) with its fused RMSNorm + SwiGLU and final
    RMSNorm + logits + device argmax epilogues; Q4_0 runs the same model on
    the register GEMV.  One layer; an 8-id prompt through ForwardBatch, then 8 greedy
    steps.  Prompt logits within 1e-3 x logit range of the oracle, greedy
    tokens equal to the oracle's."""
    cfg = dict(S.QWEN2_7B, name="tall", vocab=16384, dim=2048, hidden=8192, n_layers=1,
               n_heads=16, n_kv_heads=2)
    w = S.make_model(cfg, qt, 41, quantize_q80=lambda a: pkg.QuantizeToQ80(a).cpu().numpy())
    prompt = S.prompt_tokens(cfg["vocab"], 8, 6).tolist()
    n_steps = 8
    om = orc.OracleModel(w, 32)
    for i, t in enumerate(prompt):
        lg = om.forward_token(t, i)
    first = lg.copy()
    tok, ref_tokens = orc.argmax(lg), []
    for i in range(n_steps):
        ref_tokens.append(tok)
        lg = om.forward_token(tok, len(prompt) + i)
        tok = orc.argmax(lg)
    model = pkg.Model.from_synth(w, max_seq_len=32)
    ctx = pkg.Context(model)
    logits = ctx.ForwardBatch(prompt, 0)
    rng = float(first.max() - first.min())
    assert float(np.abs(logits - first).max()) <= 1e-3 * rng
    got = [int(np.argmax(logits))] + ctx.decode_greedy(int(np.argmax(logits)), len(prompt),
                                                       n_steps - 1).tolist()
    assert got == ref_tokens
    ctx.close()
    model.close()


def test_long_cache_head_dim_128_matches_oracle(pkg, orc, S, cuda):
    """Decode attention over a cache longer than 128 positions at the Qwen2-7B
    head shape (head_dim 128, 7 query heads per KV head; the split kernel with
    its cache rows requested into L2 before the dependency wait, and the
    last-CTA merge of the splits): a two-layer Q4_0 model with that head shape
    (dim 896, 7 / 1 heads), a 200-id prompt through ForwardBatch, then 16
    greedy steps.  Prompt logits within 1e-3 x logit range of the oracle and
    greedy tokens equal to the oracle's."""
    cfg = dict(S.QWEN2_7B, name="qwen2-7b-heads", vocab=2048, dim=896, hidden=1216, n_layers=2,
               n_heads=7, n_kv_heads=1)
    w = S.make_model(cfg, S.Q40, 31)
    prompt = S.prompt_tokens(cfg["vocab"], 200, 4).tolist()
    n_steps = 16
    om = orc.OracleModel(w, 224)
    for i, t in enumerate(prompt):
        lg = om.forward_token(t, i)
    first = lg.copy()
    tok, ref_tokens = orc.argmax(lg), []
    for i in range(n_steps):
        ref_tokens.append(tok)
        lg = om.forward_token(tok, len(prompt) + i)
        tok = orc.argmax(lg)
    model = pkg.Model.from_synth(w, max_seq_len=224)
    ctx = pkg.Context(model)
    logits = ctx.ForwardBatch(prompt, 0)
    rng = float(first.max() - first.min())
    assert float(np.abs(logits - first).max()) <= 1e-3 * rng
    got = [int(np.argmax(logits))] + ctx.decode_greedy(int(np.argmax(logits)), len(prompt),
                                                       n_steps - 1).tolist()
    assert got == ref_tokens
    ctx.close()
    model.close()


def test_qwen2_0_5b_q8_0_greedy_64_matches_reference(pkg, S, cuda):
    """Full-size Qwen2-0.5B-architecture Q8_0 (configuration 1): 32 random prompt
    ids, 64 greedy steps; tokens must equal the reference's, and the whole
    151936-entry logit vectors after the prompt (step 0) and after 16 greedy
    tokens (step 16) must sit within 1e-3 x logit range of the reference's."""
    g = json.load(open(golden_path("qwen2_0_5b_q8_0.json")))
    full = np.load(golden_path("qwen2_0_5b_q8_0_logits.npz"))
    w = S.make_model(S.QWEN2_0_5B, S.Q80, g["model_seed"],
                     quantize_q80=lambda a: pkg.QuantizeToQ80(a).cpu().numpy())
    model = pkg.Model.from_synth(w, max_seq_len=96)
    ctx = pkg.Context(model)
    prompt = g["prompt"]
    assert prompt == S.prompt_tokens(w.cfg["vocab"], 32, g["prompt_seed"]).tolist()
    logits = ctx.ForwardBatch(prompt, 0)
    err0 = check_logits(logits, full["step0"], "step 0")
    first = int(np.argmax(logits))
    assert first == g["greedy_tokens"][0]
    # step 16 through ForwardToken replays, then the greedy run from position 32
    tok = first
    for i in range(16):
        lg = ctx.ForwardToken(tok, 32 + i)
        tok = int(np.argmax(lg))
    err16 = check_logits(lg, full["step16"], "step 16")
    print(f"relative logit error: step 0 {err0:.2e}, step 16 {err16:.2e}")
    rest = ctx.decode_greedy(first, 32, 63)
    tokens = [first] + rest.tolist()
    assert tokens == g["greedy_tokens"], (
        f"first divergence at {next(i for i, (a, b) in enumerate(zip(tokens, g['greedy_tokens'])) if a != b)}"
        f", reference min margin {min(g['top1_top2_margin']):.3e}")


@pytest.mark.parametrize("qt", [1, 2])
def test_gguf_model_matches_reference_gguf_load(pkg, orc, S, cuda, tmp_path, qt):
    """A model loaded from a GGUF v3 file by the library (dqmk_model_load_gguf)
    against the reference's own LoadGgufModel of the same file: the prompt's
    logits within 1e-3 x logit range, and the library keeps the token
    embedding quantized (memory = block bytes + F32 norms and biases, where the
    reference holds the embedding -- and a tied lm_head -- as F32)."""
    w = S.make_model(dict(S.QWEN2_MINI, tied=qt == 1), qt, 41,
                     quantize_q80=lambda a: orc.quantize_q80(a, True))
    path = str(tmp_path / "mini.gguf")
    S.write_gguf(path, w, context_length=64)
    c = w.cfg
    toks = S.prompt_tokens(c["vocab"], 9, 5)
    _, ref = orc.ref_gguf_forward(path, toks)
    model = pkg.Model.from_gguf(path)
    hd = c["dim"] // c["n_heads"]
    blocks = w.token_embd.nbytes + (0 if w.lm_head is None else w.lm_head.nbytes) + sum(
        getattr(Ly, n).nbytes for Ly in w.layers
        for n in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down"))
    L = c["n_layers"]
    f32 = 4 * (c["dim"] + L * (2 * c["dim"] + c["n_heads"] * hd + 2 * c["n_kv_heads"] * hd))
    assert model.memory_bytes() == blocks + f32
    ctx = pkg.Context(model)
    got = ctx.ForwardBatch(toks.tolist(), 0)
    check_logits(got, ref, f"gguf q{qt}")
    ctx.close()
    model.close()
