"""CPU: the oracle restatement pinned to the reference.

Three anchors: the known-answer values of the reference's own tests
(tests/quant_test.cc, tests/quantized_tensor_test.cc), the reference's CPU
code compiled from its sources (oracle/_ref, when present) and the golden
fixtures that code produced (tests/golden/make_golden.py).
"""
import json
import os

import numpy as np
import pytest

from conftest import golden_path

FP16_ONE, FP16_TWO, FP16_HALF = 0x3C00, 0x4000, 0x3800  # tests/quant_test.cc:12-14


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def block_q80(d, qs):
    b = np.zeros(34, np.uint8)
    b[:2] = np.array([d], np.uint16).view(np.uint8)
    b[2:] = np.asarray(qs, np.int8).view(np.uint8)
    return b


# ------------------------------------------------ known answers (reference tests)
def test_fp16_known_patterns(orc):
    assert orc.fp16_to_fp32(FP16_ONE) == 1.0
    assert orc.fp16_to_fp32(FP16_TWO) == 2.0
    assert orc.fp16_to_fp32(FP16_HALF) == 0.5
    assert orc.fp32_to_fp16(1.0) == FP16_ONE
    # reference rounding: bit 12 set rounds up even on an exact tie (not RNE)
    tie = np.array([0x3F801000], np.uint32).view(np.float32)[0]  # 1 + 2^-11
    assert orc.fp32_to_fp16(float(tie)) == 0x3C01
    assert orc.fp32_to_fp16(1e6) == 0x7C00  # overflow -> inf
    assert orc.fp32_to_fp16(1e-9) == 0      # underflow -> 0
    # subnormal round trip
    assert orc.fp16_to_fp32(0x0001) == 2.0 ** -24


def test_quantize_q80_kats(orc):
    # QuantizeQ80ScaleIsOne (tests/quant_test.cc:262-273)
    src = np.zeros(32, np.float32)
    src[0] = 127.0
    b = orc.quantize_q80(src)
    assert b[:2].view(np.uint16)[0] == FP16_ONE and b[2] == 127
    # QuantizeQ80ZeroBlock (:276-287)
    b = orc.quantize_q80(np.zeros(32, np.float32))
    assert b[:2].view(np.uint16)[0] == 0 and not b[2:].any()
    # QuantizeQ80PartialBlock (:290-301): 40 values -> 2 blocks, tail zero
    b = orc.quantize_q80(np.ones(40, np.float32))
    assert b.size == 68
    out = orc.dequantize(orc.Q80, b, 1, 40)[0]
    assert np.allclose(out, 1.0, atol=0.01)
    assert not b[34 + 2 + 8:].any()
    # QuantizeQ80Empty (:304-307)
    assert orc.quantize_q80(np.zeros((0, 32), np.float32)).size == 0
    # round trip within d/2 (:244-259)
    src = (np.arange(32, dtype=np.float32) - 16) / 16
    out = orc.dequantize(orc.Q80, orc.quantize_q80(src), 1, 32)[0]
    assert np.abs(out - src).max() <= (1 / 127) * 0.5 + 1e-6


def test_quantize_q40_kats(orc):
    # QuantizeQ40ScaleAndPacking (tests/quant_test.cc:345-356)
    src = np.zeros(32, np.float32)
    src[0] = 7.0
    b = orc.quantize_q40(src)
    assert b[:2].view(np.uint16)[0] == FP16_ONE
    assert b[2] == (15 | (8 << 4))
    assert orc.dequantize(orc.Q40, b, 1, 32)[0, 0] == 7.0
    # zero block (:359-370)
    b = orc.quantize_q40(np.zeros(32, np.float32))
    assert not b.any()


def test_dequant_and_linear_kats(orc):
    # DequantizeQ80Basic (:20-35)
    b = block_q80(FP16_ONE, np.arange(32) - 16)
    assert np.array_equal(orc.dequantize(orc.Q80, b, 1, 32)[0], np.arange(32) - 16.0)
    # DequantizeQ40Basic (:82-101)
    q = np.zeros(18, np.uint8)
    q[:2] = np.array([FP16_ONE], np.uint16).view(np.uint8)
    for j in range(16):
        q[2 + j] = ((15 - j) << 4) | j
    out = orc.dequantize(orc.Q40, q, 1, 32)[0]
    assert np.array_equal(out[:16], np.arange(16) - 8.0)
    assert np.array_equal(out[16:], (15 - np.arange(16)) - 8.0)
    # LinearQ80Basic (:127-144)
    w = np.concatenate([block_q80(FP16_ONE, np.ones(32)), block_q80(FP16_TWO, np.ones(32))])
    y = orc.linear(orc.Q80, np.ones(32, np.float32), w, 2)
    assert y.tolist() == [32.0, 64.0]
    # LinearQ80PartialBlockTail (:168-197)
    blocks = np.concatenate([block_q80(FP16_ONE, [(i + 7 * b) % 17 - 8 for i in range(32)])
                             for b in range(4)])
    x = (0.25 * (np.arange(42) % 5)).astype(np.float32)
    y = orc.linear(orc.Q80, x, blocks, 2)
    for j in range(2):
        exp = sum(((k % 32 + 7 * (j * 2 + k // 32)) % 17 - 8) * x[k] for k in range(42))
        assert abs(y[j] - exp) < 1e-4


def test_block_sizes(orc):
    # tests/quantized_tensor_test.cc:31-52
    assert orc.Q80_BYTES == 34 and orc.Q40_BYTES == 18


# ------------------------------------------------ bit-exact vs compiled reference
needs_ref = pytest.mark.skipif(not os.path.exists(os.path.join(
    os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
    "libdqmref.so")), reason="reference library not built")


@needs_ref
@pytest.mark.parametrize("shape", [(5, 13), (32, 64), (17, 65), (3, 40), (64, 896)])
def test_quant_and_linear_match_reference(orc, shape):
    rng = np.random.default_rng(sum(shape))
    x = (rng.standard_normal(shape) * rng.uniform(1e-3, 50)).astype(np.float32)
    x[0, :5] = 0.0
    for qt, fn in ((orc.Q80, orc.quantize_q80), (orc.Q40, orc.quantize_q40)):
        a, b = fn(x), fn(x, use_ref=True)
        assert np.array_equal(a, b)
        assert np.array_equal(bits(orc.dequantize(qt, a, *shape)),
                              bits(orc.dequantize(qt, a, *shape, use_ref=True)))
        for rows in (1, 3):
            xx = rng.standard_normal((rows, shape[1])).astype(np.float32)
            assert np.array_equal(bits(orc.linear(qt, xx, a, shape[0])),
                                  bits(orc.linear(qt, xx, a, shape[0], use_ref=True)))


@needs_ref
@pytest.mark.parametrize("n", [8, 9, 13, 16, 21, 896, 897])
def test_f32_simd_linear_matches_reference(orc, n):
    rng = np.random.default_rng(n)
    w = rng.standard_normal((64, n)).astype(np.float32)
    x = rng.standard_normal(n).astype(np.float32)
    assert np.array_equal(bits(orc.linear(orc.F32, x, w, 64)),
                          bits(orc.linear(orc.F32, x, w, 64, use_ref=True)))


@needs_ref
def test_ops_match_reference(orc):
    rng = np.random.default_rng(3)
    for _ in range(20):
        x = rng.standard_normal(896).astype(np.float32)
        w = rng.standard_normal(896).astype(np.float32)
        assert np.array_equal(bits(orc.rmsnorm(x, w, 1e-6)), bits(orc.rmsnorm(x, w, 1e-6, True)))
    q = rng.standard_normal((14, 64)).astype(np.float32)
    k = rng.standard_normal((2, 64)).astype(np.float32)
    for pos in (0, 1, 7, 95, 2047, 2175):
        for neox in (True, False):
            qa, ka = orc.rope(q, k, pos, 1e6, neox)
            qb, kb = orc.rope(q, k, pos, 1e6, neox, True)
            assert np.array_equal(bits(qa), bits(qb)) and np.array_equal(bits(ka), bits(kb))
    s = rng.standard_normal(97).astype(np.float32)
    assert np.array_equal(bits(orc.softmax(s)), bits(orc.softmax(s, True)))
    g = rng.standard_normal(4864).astype(np.float32)
    u = rng.standard_normal(4864).astype(np.float32)
    assert np.array_equal(bits(orc.swiglu(g, u)), bits(orc.swiglu(g, u, True)))
    t = np.array([1.0, 3.0, 3.0, 2.0], np.float32)  # first max wins
    assert orc.argmax(t) == 1 == orc.argmax(t, True)


@needs_ref
@pytest.mark.parametrize("qt", [1, 2])
def test_whole_model_matches_reference(orc, S, qt):
    w = S.make_model(S.QWEN2_MINI, qt, 99, quantize_q80=orc.quantize_q80)
    om, rm = orc.OracleModel(w, 32), orc.RefModel(w, 32)
    toks = S.prompt_tokens(w.cfg["vocab"], 6, 5)
    for i, t in enumerate(toks):
        assert np.array_equal(bits(om.forward_token(int(t), i)),
                              bits(rm.forward_batch([int(t)], i)))
    # ForwardBatch side effects (tests/batch_test.cc:196-217)
    rm.reset()
    rm.forward_batch(toks[:3], 0)
    assert rm.pos() == 2 and rm.history().tolist() == toks[:3].tolist()


# ------------------------------------------------ oracle vs committed goldens
def _gemv_cases():
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", golden_path("make_golden.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.GEMV_CASES


@pytest.mark.parametrize("case", range(11))
def test_oracle_gemv_golden(orc, S, case):
    cases = [c for c in _gemv_cases() if c[1] * c[2] <= 5_000_000]
    if case >= len(cases):
        pytest.skip("fewer small cases")
    qt, o, i, seed = cases[case]
    g = np.load(golden_path("gemv_cases.npz"))
    blocks, x = S.gemv_case(o, i, seed, qt)
    y = orc.linear(qt, x, blocks, o)
    key = f"q{qt}_{o}x{i}_s{seed}"
    assert np.array_equal(bits(y[g[key + "_idx"]]), bits(g[key + "_y"]))


@pytest.mark.parametrize("qt", [1, 2])
def test_oracle_mini_model_golden(orc, S, qt):
    g = np.load(golden_path("mini_model.npz"))
    w = S.make_model(S.QWEN2_MINI, qt, 2024, quantize_q80=orc.quantize_q80)
    om = orc.OracleModel(w, 64)
    toks = g[f"q{qt}_tokens"]
    assert np.array_equal(toks, S.prompt_tokens(w.cfg["vocab"], 12, 77))
    for i, t in enumerate(toks):
        assert np.array_equal(bits(om.forward_token(int(t), i)), bits(g[f"q{qt}_logits"][i]))


def test_full_model_golden_is_consistent():
    d = json.load(open(golden_path("qwen2_0_5b_q8_0.json")))
    assert len(d["prompt"]) == 32 and len(d["greedy_tokens"]) == 64
    assert all(t[0][0] == tok for t, tok in zip(d["top5"], d["greedy_tokens"]))
    assert min(d["top1_top2_margin"]) > 0


@needs_ref
@pytest.mark.parametrize("shape", [(5, 13), (32, 64), (17, 65), (64, 896)])
def test_q41_dequant_and_linear_match_reference(orc, S, shape):
    """Q4_1 (20-byte blocks, d * q + m): the restatement's dequantization and
    Linear equal the reference's DequantizeFromQ41 / LinearQ41
    (src/quant.cc:192-235, 256-262, 362-366) bit for bit."""
    o, i = shape
    blocks, _ = S.gemv_case(o, i, 91 + o, S.Q41)
    assert np.array_equal(bits(orc.dequantize(orc.Q41, blocks, o, i)),
                          bits(orc.dequantize(orc.Q41, blocks, o, i, use_ref=True)))
    rng = np.random.default_rng(o * i)
    for rows in (1, 3):
        x = rng.standard_normal((rows, i)).astype(np.float32)
        assert np.array_equal(bits(orc.linear(orc.Q41, x, blocks, o)),
                              bits(orc.linear(orc.Q41, x, blocks, o, use_ref=True)))


@needs_ref
@pytest.mark.parametrize("qt", [1, 2])
def test_gguf_writer_read_by_reference(orc, S, tmp_path, qt):
    """The synthetic GGUF v3 writer (synth.write_gguf) produces files the
    reference's own reader and LoadGgufModel accept (src/gguf.cc,
    src/gguf_loader.cc:279-364): the configuration comes back from the
    metadata and the loaded model's ForwardBatch logits equal, bit for bit,
    those of the same weights handed to the reference directly."""
    w = S.make_model(dict(S.QWEN2_MINI, tied=qt == 1), qt, 31,
                     quantize_q80=lambda a: orc.quantize_q80(a, True))
    path = str(tmp_path / "mini.gguf")
    S.write_gguf(path, w, context_length=64)
    c = w.cfg
    toks = S.prompt_tokens(c["vocab"], 7, 3)
    cfg, logits = orc.ref_gguf_forward(path, toks)
    assert cfg == {"vocab": c["vocab"], "dim": c["dim"], "hidden": c["hidden"],
                   "n_layers": c["n_layers"], "n_heads": c["n_heads"],
                   "n_kv_heads": c["n_kv_heads"], "max_seq": 64, "neox": 1}
    direct = orc.RefModel(w, 64)
    assert np.array_equal(bits(logits), bits(direct.forward_batch(toks, 0)))


@pytest.mark.parametrize("qt", [1, 2])
def test_gguf_config_read_by_library(pkg, orc, S, tmp_path, qt):
    """The library's own GGUF reader (dqmk_gguf_read_config, no device work)
    builds the configuration the reference's BuildConfig does from the same
    file: qwen2 => NeoX RoPE, vocabulary = tokenizer.ggml.tokens length,
    head_dim = dim / n_heads."""
    w = S.make_model(dict(S.QWEN2_MINI, tied=qt == 1), qt, 31,
                     quantize_q80=lambda a: orc.quantize_q80(a))
    path = str(tmp_path / "mini.gguf")
    S.write_gguf(path, w, context_length=96)
    c = w.cfg
    got = pkg.Model.gguf_config(path)
    assert got == {"vocab": c["vocab"], "dim": c["dim"], "hidden": c["hidden"],
                   "n_layers": c["n_layers"], "n_heads": c["n_heads"],
                   "n_kv_heads": c["n_kv_heads"], "head_dim": c["dim"] // c["n_heads"],
                   "max_seq_len": 96, "rope_theta": np.float32(c["rope_theta"]),
                   "eps": np.float32(c["eps"]), "rope_neox": 1}
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUF\x02\x00\x00\x00" + b"\x00" * 16)
    with pytest.raises(RuntimeError, match="LoadGgufModel: GGUF version 3 expected"):
        pkg.Model.gguf_config(str(bad))
