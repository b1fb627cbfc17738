"""GPU parity of multi-sequence decode (dqmk_batch and its GEMM).

The reference decodes one sequence per context (ForwardToken,
src/forward.cc:667-754); a dqmk_batch runs up to 64 (slot, position, token)
columns per step, every projection as one tensor-core GEMM over the packed
Q8_0 / Q4_0 blocks (dequantized on chip into exact two-term fp16 operands).
Each column must compute what ForwardToken computes for its sequence:

  * the GEMM against the oracle's F32 LinearQ80 / LinearQ40 with the bound
    |y - ref| <= 1e-5 * sum_k |W[o,k] x[k]| per output (fp32 summation order,
    the 2^-22 activation split, the dropped lo*lo term), on ragged shapes:
    one column, column counts that are not multiples of 16, K tails, row
    counts across the 256-row tile, split-K, bias and an in-place residual;
  * whole models: per-sequence logits within 1e-3 x logit range of the
    oracle (the logit tolerance of the whole path), and greedy tokens identical to the
    oracle's, with sequences at different positions in the same step, one
    slot taking several prompt positions in one step, and the 7B layer
    widths (head_dim 128, K = 3584 / 18944) on a one-layer model.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3

CASES = [
    # (qtype, columns, in, out)
    (1, 1, 896, 896), (1, 64, 896, 1152), (1, 17, 896, 4864), (1, 64, 4864, 896),
    (1, 7, 96, 300), (1, 33, 13, 5), (1, 64, 896, 151936),
    (2, 64, 3584, 2304), (2, 64, 1792, 3584), (2, 5, 65, 17), (2, 48, 896, 1000),
    (2, 64, 4736, 3584), (2, 16, 18944, 512),
]


def make_x(m, k, seed):
    g = np.random.default_rng(seed)
    x = g.standard_normal((m, k), dtype=np.float32)
    if m > 2:
        x[1] = 0.0                      # a zero column: every scale is 0
        x[2, ::97] *= 300.0             # outliers dominate their blocks
    return x


def error_bound(orc, qt, x, blocks, o):
    w = orc.dequantize(qt, blocks, o, x.shape[1])
    return 1e-5 * (np.abs(x).astype(np.float64) @ np.abs(w).astype(np.float64).T) + 1e-30


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"q{c[0]}_c{c[1]}_{c[2]}to{c[3]}")
def test_linear_cols_matches_oracle(pkg, orc, S, cuda, case):
    torch = cuda
    qt, m, k, o = case
    blocks, _ = S.gemv_case(o, k, 300 + m, qt)
    x = make_x(m, k, 5 * m + k)
    packed = pkg.pack_weight(qt, blocks, o, k)
    y = pkg.linear_cols_packed(qt, torch.from_numpy(x).cuda(), packed, o).cpu().numpy()
    ref = orc.linear(qt, x, blocks, o)
    bound = error_bound(orc, qt, x, blocks, o)
    err = np.abs(y.astype(np.float64) - ref)
    worst = np.unravel_index(np.argmax(err - bound), err.shape)
    assert np.all(err <= bound), (f"column {worst[0]} row {worst[1]}: err {err[worst]:.3e} "
                                  f"> bound {bound[worst]:.3e}")
    if m > 2:
        assert np.all(y[1] == 0.0)
    assert pkg.lib().dqmk_device_error(1) == 0
    print(f"{case}: max err / max |ref| = {float(err.max() / max(1e-30, np.abs(ref).max())):.2e}")


def test_linear_cols_bias_and_inplace_residual(pkg, orc, S, cuda):
    torch = cuda
    m, k, o = 40, 896, 896
    blocks, _ = S.gemv_case(o, k, 3)
    x = make_x(m, k, 11)
    g = np.random.default_rng(5)
    bias = g.standard_normal(o, dtype=np.float32)
    res = g.standard_normal((m, o), dtype=np.float32)
    packed = pkg.pack_weight(pkg.Q80, blocks, o, k)
    rd = torch.from_numpy(res).cuda()
    pkg.linear_cols_packed(pkg.Q80, torch.from_numpy(x).cuda(), packed, o,
                           bias=torch.from_numpy(bias).cuda(), residual=rd, y=rd)
    got = rd.cpu().numpy()
    ref = orc.linear(pkg.Q80, x, blocks, o) + bias[None, :] + res
    bound = error_bound(orc, pkg.Q80, x, blocks, o) + 1e-6 * (np.abs(res) + np.abs(bias))
    assert np.all(np.abs(got - ref) <= bound)


def test_linear_cols_rejects_bad_shapes(pkg, cuda):
    torch = cuda
    x = torch.zeros(65, 64, device="cuda")
    packed = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    with pytest.raises(RuntimeError):
        pkg.linear_cols_packed(pkg.Q80, x, packed, 32)


def check_logits(got, ref, label):
    rng = float(ref.max() - ref.min())
    err = float(np.abs(got - ref).max())
    assert err <= LOGIT_TOL * rng, f"{label}: max err {err:.3e} > {LOGIT_TOL} * range {rng:.3f}"
    return err / rng


def oracle_run(orc, w, prompt, n_greedy, max_seq):
    """Logits after the prompt and the greedy continuation (oracle)."""
    om = orc.OracleModel(w, max_seq)
    for i, t in enumerate(prompt):
        logits = om.forward_token(int(t), i)
    first = logits.copy()
    toks, margins = [], []
    pos = len(prompt)
    for _ in range(n_greedy):
        top2 = np.sort(logits)[-2:]
        margins.append(float(top2[1] - top2[0]))
        t = int(orc.argmax(logits))
        toks.append(t)
        logits = om.forward_token(t, pos)
        pos += 1
    return first, toks, min(margins)


def run_batch(pkg, w, prompts, n_greedy, max_seq):
    model = pkg.Model.from_synth(w, max_seq_len=max_seq)
    b = pkg.Batch(model, len(prompts), max_seq)
    for s, p in enumerate(prompts):  # several positions of one slot per step
        if len(p) > 1:
            b.prefill(s, p[:-1])
    # one step over every slot at its own position
    logits, nxt = b.step(list(range(len(prompts))), [int(p[-1]) for p in prompts],
                         [len(p) - 1 for p in prompts])
    toks = b.decode_greedy(nxt, [len(p) for p in prompts], n_greedy - 1)
    b.close()
    model.close()
    return logits, nxt, toks


@pytest.fixture(scope="module")
def mini(pkg, S, cuda):
    return {qt: S.make_model(S.QWEN2_MINI, qt, 2024,
                             quantize_q80=lambda a: pkg.QuantizeToQ80(a).cpu().numpy())
            for qt in (pkg.Q80, pkg.Q40)}


@pytest.mark.parametrize("qt", [1, 2])
def test_batch_matches_oracle_per_sequence(pkg, orc, S, mini, cuda, qt):
    w = mini[qt]
    vocab = S.QWEN2_MINI["vocab"]
    lens = [5, 12, 1, 70]  # ragged; the 70-token prompt takes two prefill steps
    prompts = [S.prompt_tokens(vocab, n, 40 + i) for i, n in enumerate(lens)]
    n_greedy, max_seq = 12, 96
    logits, nxt, toks = run_batch(pkg, w, prompts, n_greedy, max_seq)
    worst = 0.0
    for s, p in enumerate(prompts):
        first, ref_toks, margin = oracle_run(orc, w, p, n_greedy, max_seq)
        worst = max(worst, check_logits(logits[s], first, f"q{qt} slot {s}"))
        got = [int(nxt[s])] + [int(t) for t in toks[:, s]]
        assert got == ref_toks, (s, got, ref_toks, margin)
    print(f"q{qt}: worst relative logit error {worst:.2e}")


def test_batch_7b_widths_matches_oracle(pkg, orc, S, cuda):
    """Qwen2-7B layer widths (dim 3584, FFN 18944, 28/4 heads of 128), one
    layer, 8192 vocabulary ids, untied Q4_0 lm_head."""
    import tp_worker
    w, _ = tp_worker.reduced_7b(S)
    vocab = tp_worker.REDUCED_7B["vocab"]
    prompts = [S.prompt_tokens(vocab, n, 90 + i) for i, n in enumerate([6, 3, 9])]
    n_greedy, max_seq = 6, 32
    logits, nxt, toks = run_batch(pkg, w, prompts, n_greedy, max_seq)
    for s, p in enumerate(prompts):
        first, ref_toks, margin = oracle_run(orc, w, p, n_greedy, max_seq)
        check_logits(logits[s], first, f"7b slot {s}")
        got = [int(nxt[s])] + [int(t) for t in toks[:, s]]
        assert got == ref_toks, (s, got, ref_toks, margin)


def test_batch_rejects_bad_columns(pkg, mini, cuda):
    model = pkg.Model.from_synth(mini[pkg.Q80], max_seq_len=32)
    b = pkg.Batch(model, 2, 32)
    with pytest.raises(IndexError):
        b.step([2], [1], [0])          # slot out of range
    with pytest.raises(IndexError):
        b.step([0], [1], [32])         # position out of range
    with pytest.raises(RuntimeError):
        b.step([0, 0], [1, 2], [3, 3])  # the same (slot, position) twice
    with pytest.raises(RuntimeError):
        b.step(list(range(65)), [1] * 65, [0] * 65)
    b.close()
    model.close()
