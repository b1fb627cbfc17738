"""GPU parity of the individual kernels, through the C ABI, against the oracle.

Integer / byte work (quantize, dequantize, repack, embedding gather, argmax)
must be bit-exact.  Float reductions (GEMV, RMSNorm, attention) are checked
with the reference's own CUDA-test tolerance: |err| <= 1e-3 absolute or
relative to max(1, |expected|) (tests/test_cuda_quant.cc:28-41).
"""
import numpy as np
import pytest

from conftest import golden_path

pytestmark = pytest.mark.gpu

ABS_TOL = 1e-3
REL_TOL = 1e-3


def assert_close(actual, expected, label=""):
    actual = np.asarray(actual, np.float32)
    expected = np.asarray(expected, np.float32)
    assert actual.shape == expected.shape, label
    err = np.abs(actual - expected)
    scale = np.maximum(1.0, np.abs(expected))
    bad = ~((err <= ABS_TOL) | (err / scale <= REL_TOL))
    assert not bad.any(), f"{label}: {bad.sum()} mismatches, max err {err.max():.3e}"


def pattern(shape, scale, shift):
    """MakePatternTensor (tests/test_cuda_quant.cc:56-64)."""
    n = int(np.prod(shape))
    i = np.arange(n)
    return ((((i * 19 + 7) % 31) - 15) * scale + shift).astype(np.float32).reshape(shape)


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


# ------------------------------------------------------------ quantization
def quant_inputs():
    rng = np.random.default_rng(0)
    cases = {
        "normal": (rng.standard_normal((64, 896)) * 0.02).astype(np.float32),
        "tail": rng.standard_normal((7, 45)).astype(np.float32),
        "wide_range": (rng.standard_normal((16, 128)) *
                       np.exp(rng.uniform(-20, 12, (16, 1)))).astype(np.float32),
        "zeros_and_ties": np.concatenate([np.zeros((1, 64), np.float32),
                                          np.tile(np.float32([127.0, -63.5, 0.5, 1.5]),
                                                  (1, 16))], 0),
        "subnormal_scale": (rng.standard_normal((4, 64)) * 1e-6).astype(np.float32),
        "pattern": pattern((32, 64), 0.019, 0.04),
    }
    return cases


@pytest.mark.parametrize("name", list(quant_inputs().keys()))
def test_quantize_bit_exact(pkg, orc, cuda, name):
    x = quant_inputs()[name]
    for fn_dev, fn_orc, qt in ((pkg.QuantizeToQ80, orc.quantize_q80, pkg.Q80),
                               (pkg.QuantizeToQ40, orc.quantize_q40, pkg.Q40)):
        dev = fn_dev(x).cpu().numpy()
        ref = fn_orc(x)
        assert np.array_equal(dev, ref), f"{name} q{qt}: {np.count_nonzero(dev != ref)} bytes differ"
        deq = (pkg.DequantizeFromQ80 if qt == pkg.Q80 else pkg.DequantizeFromQ40)(
            ref, x.shape).cpu().numpy()
        assert np.array_equal(bits(deq), bits(orc.dequantize(qt, ref, *x.shape)))


def test_quantize_full_size_digest_matches_reference(pkg, S, cuda):
    """Device QuantizeToQ80 of the full-size synthetic Qwen2-0.5B tensors gives the
    same bytes the reference's QuantizeToQ80 gave when the golden was made."""
    import hashlib
    import json
    g = json.load(open(golden_path("qwen2_0_5b_q8_0.json")))
    seed = g["model_seed"]
    c = S.QWEN2_0_5B
    hd = c["dim"] // c["n_heads"]
    checks = {"token_embd": (0, (c["vocab"], c["dim"])),
              "layers.0.wq": (16 + 1, (c["n_heads"] * hd, c["dim"])),
              "layers.23.w_down": (16 + 16 * 23 + 11, (c["dim"], c["hidden"]))}
    for name, (idx, shape) in checks.items():
        blocks = pkg.QuantizeToQ80(S.normal(seed, idx, shape)).cpu().numpy()
        assert hashlib.sha256(blocks.tobytes()).hexdigest() == g["digests"][name], name


def test_pack_roundtrip(pkg, orc, S, cuda):
    for qt, o, i in ((pkg.Q80, 33, 70), (pkg.Q40, 9, 96), (pkg.Q80, 128, 896)):
        blocks, _ = S.gemv_case(o, i, 5, qt)
        packed = pkg.pack_weight(qt, blocks, o, i).cpu().numpy()
        nb = (i + 31) // 32
        bb = blocks.reshape(o * nb, 34 if qt == pkg.Q80 else 18)
        qbytes = o * nb * (32 if qt == pkg.Q80 else 16)
        d = packed[qbytes:].view(np.uint16)
        assert np.array_equal(d, bb[:, :2].copy().view(np.uint16).reshape(-1))
        q = packed[:qbytes].reshape(o, -1)
        if qt == pkg.Q80:
            exp = bb[:, 2:].reshape(o, nb * 32).copy()
            exp[:, i:] = 0  # values past in_features are zeroed
        else:
            exp = bb[:, 2:].reshape(o, nb * 16)
        assert np.array_equal(q, exp)


# ------------------------------------------------------------ Linear / GEMV
@pytest.mark.parametrize("qt", [1, 2])
def test_linear_reference_cases(pkg, orc, cuda, qt):
    """TestCudaQ80LinearCases / TestCudaQ40LinearCases (tests/test_cuda_quant.cc:304-372)."""
    quant = orc.quantize_q80 if qt == 1 else orc.quantize_q40
    lin = pkg.CudaQ80Linear if qt == 1 else pkg.CudaQ40Linear
    w1, x1, b1 = pattern((5, 13), 0.037, -0.11), pattern((13,), 0.071, 0.03), pattern((5,), 0.013, -0.02)
    q1 = quant(w1)
    exp1 = orc.linear(qt, x1, q1, 5)
    assert_close(lin(x1, q1, (5, 13)), exp1, "1D no bias")
    assert_close(lin(x1, q1, (5, 13), bias=b1), exp1 + b1, "1D bias")
    w2, x2 = pattern((32, 64), 0.019, 0.04), pattern((3, 64), 0.029, -0.06)
    q2 = quant(w2)
    assert_close(lin(x2, q2, (32, 64)), orc.linear(qt, x2, q2, 32), "2D batch")
    w3, x3 = pattern((17, 65), 0.019, 0.04), pattern((3, 65), 0.029, -0.06)
    q3 = quant(w3)
    dev = (pkg.CudaQ80LinearDeviceInput if qt == 1 else pkg.CudaQ40LinearDeviceInput)(
        cuda.from_numpy(x3).cuda(), cuda.from_numpy(q3).cuda(), 17 * 3, (17, 65))
    assert_close(dev.cpu().numpy(), orc.linear(qt, x3, q3, 17), "device input 17x65")
    with pytest.raises(RuntimeError, match="block count mismatch"):
        lin(x3, q3[:-34], (17, 65))


def test_q41_linear_reference_cases(pkg, orc, S, cuda):
    """The Q4_1 cases of tests/test_cuda_quant.cc:373-411 (pattern shapes
    5x13 with and without bias, 32x64 with 3 input rows, 17x65 device input)
    against the reference's LinearQ41, abs/rel tolerance 1e-3."""
    for (o, i), rows in (((5, 13), 1), ((32, 64), 3), ((17, 65), 3), ((896, 896), 1)):
        blocks, _ = S.gemv_case(o, i, 300 + o, S.Q41)
        x = pattern((rows, i) if rows > 1 else (i,), 0.029, -0.06)
        ref = orc.linear(orc.Q41, x, blocks, o, use_ref=True)
        assert_close(pkg.CudaQ41Linear(x, blocks, (o, i)), ref, f"q4_1 {o}x{i}")
    b = pattern((5,), 0.013, -0.02)
    blocks, _ = S.gemv_case(5, 13, 305, S.Q41)
    x = pattern((13,), 0.071, 0.03)
    assert_close(pkg.CudaQ41Linear(x, blocks, (5, 13), bias=b),
                 orc.linear(orc.Q41, x, blocks, 5, use_ref=True) + b, "q4_1 bias")
    dev = pkg.CudaQ41LinearDeviceInput(cuda.zeros(3, 65, device="cuda"),
                                       cuda.from_numpy(S.gemv_case(17, 65, 1, S.Q41)[0]).cuda(),
                                       17 * 3, (17, 65))
    assert float(dev.abs().max()) == 0.0
    with pytest.raises(RuntimeError, match="CudaQ41Linear: block count mismatch"):
        pkg.CudaQ41Linear(x, blocks[:-20], (5, 13))


@pytest.mark.parametrize("shape", [(64, 13), (896, 896), (17, 65), (151936, 896)])
def test_f32_linear_matches_reference(pkg, orc, cuda, shape):
    """F32-weight Linear (the reference's cuBLAS path, tests/test_cuda_matmul.cc:
    112-163) against the reference's threaded-simd LinearDispatch, abs/rel
    tolerance 1e-3; 1 and 3 input rows, bias on one case; the 151936 x 896
    shape is the reference's tied F32 lm_head."""
    o, i = shape
    rng = np.random.default_rng(o + i)
    w = (rng.standard_normal((o, i)) * 0.02).astype(np.float32)
    x = rng.standard_normal(i).astype(np.float32)
    ref = orc.linear(orc.F32, x, w, o, use_ref=True)
    assert_close(pkg.CudaLinear(x, w), ref, f"f32 {o}x{i}")
    if o <= 896:
        x3 = rng.standard_normal((3, i)).astype(np.float32)
        ref3 = np.stack([orc.linear(orc.F32, r, w, o, use_ref=True) for r in x3])
        bias = rng.standard_normal(o).astype(np.float32)
        assert_close(pkg.CudaLinear(x3, w, bias=bias), ref3 + bias, f"f32 {o}x{i} x3 bias")


def gemv_cases():
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", golden_path("make_golden.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.GEMV_CASES


@pytest.mark.parametrize("case", gemv_cases(), ids=lambda c: f"q{c[0]}_{c[1]}x{c[2]}")
def test_gemv_sweep_vs_golden_and_oracle(pkg, orc, S, cuda, case):
    """Standalone GEMV sweep: packed (engine) kernel and ggml-layout kernel against
    the reference's outputs stored in the golden fixture, and against the live
    oracle wherever that finishes in seconds."""
    qt, o, i, seed = case
    g = np.load(golden_path("gemv_cases.npz"))
    key = f"q{qt}_{o}x{i}_s{seed}"
    idx, gy = g[key + "_idx"], g[key + "_y"]
    blocks, x = S.gemv_case(o, i, seed, qt)
    xd = cuda.from_numpy(x).cuda()
    bd = cuda.from_numpy(blocks).cuda()
    packed = pkg.pack_weight(qt, bd, o, i)
    y_packed = pkg.gemv_packed(qt, xd, packed, o).cpu().numpy()
    y_ggml = pkg._linear_device(qt, xd, bd, o * ((i + 31) // 32), (o, i)).cpu().numpy()
    cuda.cuda.synchronize()
    assert_close(y_packed[idx], gy, key + " packed vs golden")
    assert_close(y_ggml[idx], gy, key + " ggml vs golden")
    if o * i <= 5_000_000:
        ref = orc.linear(qt, x, blocks, o)
        assert np.array_equal(bits(ref[idx]), bits(gy))  # the oracle reproduces the golden
        assert_close(y_packed, ref, key + " packed vs oracle")


@pytest.mark.parametrize("qt", [1, 2], ids=["q8_0", "q4_0"])
@pytest.mark.parametrize("rows,k", [(4100, 3584), (1000, 18944), (520, 2048), (65600, 2048)])
def test_gemv_wide_rows_vs_oracle(pkg, orc, S, cuda, qt, rows, k):
    """Rows of 2048 values and more (the Qwen2-7B widths; ragged row counts that
    leave a partial tile; a tall Q8_0 weight, which takes the tensor-core
    GEMV, and a tall Q4_0 weight and wide Q8_0 rows, which take the
    shared-memory ring form): packed GEMV with a residual add, and the
    chained form with RMSNorm and SwiGLU over interleaved gate/up rows, both
    against the oracle within the reference's CUDA-test tolerance (1e-3
    absolute or relative)."""
    blocks, x = S.gemv_case(rows, k, 40 + rows % 7, qt)
    rng = np.random.default_rng(rows)
    res = rng.standard_normal(rows).astype(np.float32)
    packed = pkg.pack_weight(qt, cuda.from_numpy(blocks).cuda(), rows, k)
    xd = cuda.from_numpy(x).cuda()
    rd = cuda.from_numpy(res).cuda()
    y = pkg.gemv_packed(qt, xd, packed, rows, residual=rd, y=rd).cpu().numpy()
    assert_close(y, res + orc.linear(qt, x, blocks, rows), f"q{qt} {rows}x{k} residual")
    nw = (1 + 0.02 * rng.standard_normal(k)).astype(np.float32)
    yo = cuda.empty(rows // 2, dtype=cuda.float32, device="cuda")
    pkg.gemv_packed_chained(qt, xd, packed, rows, yo, norm=cuda.from_numpy(nw).cuda(),
                            swiglu=True)
    lin = orc.linear(qt, orc.rmsnorm(x, nw, 1e-6), blocks, rows)
    assert_close(yo.cpu().numpy(), orc.swiglu(lin[0::2], lin[1::2]), f"q{qt} {rows}x{k} swiglu")


def test_gemv_residual_and_bias(pkg, orc, S, cuda):
    blocks, x = S.gemv_case(300, 896, 9)
    rng = np.random.default_rng(1)
    bias = rng.standard_normal(300).astype(np.float32)
    res = rng.standard_normal(300).astype(np.float32)
    packed = pkg.pack_weight(pkg.Q80, blocks, 300, 896)
    rd = cuda.from_numpy(res).cuda()
    y = pkg.gemv_packed(pkg.Q80, cuda.from_numpy(x).cuda(), packed, 300,
                        bias=cuda.from_numpy(bias).cuda(), residual=rd, y=rd).cpu().numpy()
    assert_close(y, res + (orc.linear(pkg.Q80, x, blocks, 300) + bias))


# ------------------------------------------------------------ memory-bound ops
def test_rmsnorm(pkg, orc, cuda):
    rng = np.random.default_rng(2)
    for dim in (32, 896, 3584):
        x = rng.standard_normal(dim).astype(np.float32)
        w = (1 + 0.02 * rng.standard_normal(dim)).astype(np.float32)
        y = pkg.CudaRmsNormDeviceWeight(cuda.from_numpy(x).cuda(), cuda.from_numpy(w).cuda(), 1e-6)
        assert_close(y.cpu().numpy(), orc.rmsnorm(x, w, 1e-6), f"rmsnorm {dim}")


@pytest.mark.parametrize("neox", [True, False])
def test_rope(pkg, orc, cuda, neox):
    rng = np.random.default_rng(4)
    q = rng.standard_normal((14, 64)).astype(np.float32)
    k = rng.standard_normal((2, 64)).astype(np.float32)
    for pos in (0, 1, 31, 95, 2047):
        qd, kd = cuda.from_numpy(q.copy()).cuda(), cuda.from_numpy(k.copy()).cuda()
        pkg.CudaRopeDeviceInput(qd, kd, 14, 2, 64, pos, 1e6, neox)
        qr, kr = orc.rope(q, k, pos, 1e6, neox)
        # same angles bit for bit; rotation rounding pinned to the reference's
        assert np.array_equal(bits(qd.cpu().numpy()), bits(qr)), f"pos {pos}"
        assert np.array_equal(bits(kd.cpu().numpy()), bits(kr)), f"pos {pos}"


def test_swiglu_add_embedding_argmax(pkg, orc, S, cuda):
    rng = np.random.default_rng(5)
    g = rng.standard_normal(4864).astype(np.float32)
    u = rng.standard_normal(4864).astype(np.float32)
    y = pkg.CudaSiluMulDeviceInput(cuda.from_numpy(g).cuda(), cuda.from_numpy(u).cuda())
    assert_close(y.cpu().numpy(), orc.swiglu(g, u), "swiglu")
    a = cuda.from_numpy(g).cuda()
    assert np.array_equal(pkg.CudaElementwiseAddDeviceInput(a, a).cpu().numpy(), g + g)
    blocks, _ = S.gemv_case(100, 96, 3)
    table = orc.dequantize(pkg.Q80, blocks, 100, 96)
    for tok in (0, 57, 99):
        e = pkg.embedding_lookup_blocks(pkg.Q80, cuda.from_numpy(blocks).cuda(), 100, 96, tok)
        assert np.array_equal(bits(e.cpu().numpy()), bits(table[tok]))
        e2 = pkg.CudaEmbeddingLookupDeviceWeight(cuda.from_numpy(table).cuda(), tok)
        assert np.array_equal(bits(e2.cpu().numpy()), bits(table[tok]))
    with pytest.raises(pkg.OutOfRange):
        pkg.embedding_lookup_blocks(pkg.Q80, cuda.from_numpy(blocks).cuda(), 100, 96, 100)
    x = rng.standard_normal(151936).astype(np.float32)
    x[[5000, 90000]] = 50.0  # tie: the first index wins
    assert pkg.argmax(cuda.from_numpy(x).cuda()) == 5000 == orc.argmax(x)
    x[:] = -1.0
    assert pkg.argmax(cuda.from_numpy(x).cuda()) == 0


# ------------------------------------------------------------ attention
@pytest.mark.parametrize("cfg", [(14, 2, 64), (4, 2, 64), (28, 4, 128), (4, 4, 8)],
                         ids=lambda c: f"h{c[0]}_kv{c[1]}_hd{c[2]}")
def test_attention_decode(pkg, orc, cuda, cfg):
    n_heads, n_kv, hd = cfg
    n_layers, max_seq = 2, 300
    rng = np.random.default_rng(n_heads + hd)
    kv = pkg.CudaKvCache(n_layers, max_seq, n_kv, hd)
    keys = rng.standard_normal((n_layers, max_seq, n_kv, hd)).astype(np.float32)
    vals = rng.standard_normal((n_layers, max_seq, n_kv, hd)).astype(np.float32)
    kv.keys.copy_(cuda.from_numpy(keys))
    kv.values.copy_(cuda.from_numpy(vals))
    q = rng.standard_normal(n_heads * hd).astype(np.float32)
    qd = cuda.from_numpy(q).cuda()
    for layer, pos in ((0, 0), (1, 1), (1, 31), (0, 32), (1, 200), (0, 299)):
        out = pkg.CudaAttentionDecodeDeviceInput(qd, kv, layer, pos, n_heads, n_kv, hd)
        ref = orc.attention(q, keys, vals, layer, pos, n_heads)
        assert_close(out.cpu().numpy(), ref, f"layer {layer} pos {pos}")
    # KV write then read back through attention at pos 0 (softmax of one = 1)
    k = cuda.from_numpy(rng.standard_normal(n_kv * hd).astype(np.float32)).cuda()
    v = cuda.from_numpy(rng.standard_normal(n_kv * hd).astype(np.float32)).cuda()
    kv.WriteDevice(1, 0, k, v)
    out = pkg.CudaAttentionDecodeDeviceInput(qd, kv, 1, 0, n_heads, n_kv, hd).cpu().numpy()
    vv = v.cpu().numpy().reshape(n_kv, hd)
    exp = np.concatenate([vv[h // (n_heads // n_kv)] for h in range(n_heads)])
    assert np.array_equal(bits(out), bits(exp))
    with pytest.raises(pkg.OutOfRange):
        pkg.CudaAttentionDecodeDeviceInput(qd, kv, 2, 0, n_heads, n_kv, hd)


@pytest.mark.parametrize("cfg", [(14, 2, 64, 96), (28, 4, 128, 128), (4, 4, 64, 64)])
def test_attention_decode_short_cache(pkg, orc, cuda, cfg):
    """Caches of at most 128 positions take the one-pass short kernel (one CTA
    per query head, all loads issued together): outputs within the CUDA
    tests' 1e-3 tolerance of the oracle at the first, middle and last
    positions, and exactly V at position 0."""
    n_heads, n_kv, hd, max_seq = cfg
    n_layers = 2
    rng = np.random.default_rng(n_heads * hd + max_seq)
    kv = pkg.CudaKvCache(n_layers, max_seq, n_kv, hd)
    keys = rng.standard_normal((n_layers, max_seq, n_kv, hd)).astype(np.float32)
    vals = rng.standard_normal((n_layers, max_seq, n_kv, hd)).astype(np.float32)
    kv.keys.copy_(cuda.from_numpy(keys))
    kv.values.copy_(cuda.from_numpy(vals))
    q = rng.standard_normal(n_heads * hd).astype(np.float32)
    qd = cuda.from_numpy(q).cuda()
    for layer, pos in ((0, 1), (1, 31), (0, max_seq // 2 + 3), (1, max_seq - 1)):
        out = pkg.CudaAttentionDecodeDeviceInput(qd, kv, layer, pos, n_heads, n_kv, hd)
        ref = orc.attention(q, keys, vals, layer, pos, n_heads)
        assert_close(out.cpu().numpy(), ref, f"layer {layer} pos {pos}")
    out = pkg.CudaAttentionDecodeDeviceInput(qd, kv, 1, 0, n_heads, n_kv, hd).cpu().numpy()
    exp = np.concatenate([vals[1, 0, h // (n_heads // n_kv)] for h in range(n_heads)])
    assert np.array_equal(bits(out), bits(exp))


@pytest.mark.parametrize("cfg", [(2, 1, 3, 4), (12, 1, 6, 300), (4, 2, 260, 40), (18, 1, 64, 64)])
def test_attention_decode_any_shape(pkg, orc, cuda, cfg):
    """Head configurations outside the fast kernels (head_dim not a multiple
    of 4 or above 256, more than 8 query heads per KV head -- the reference's
    CUDA attention takes any): the general kernel, within the CUDA tests'
    tolerance of the oracle, exactly V at position 0.  (2, 1, 3) is the
    reference test's own GQA case (tests/test_cuda_attention.cc:106-145)."""
    n_heads, n_kv, hd, max_seq = cfg
    n_layers = 2
    rng = np.random.default_rng(n_heads * hd + max_seq)
    kv = pkg.CudaKvCache(n_layers, max_seq, n_kv, hd)
    keys = rng.standard_normal((n_layers, max_seq, n_kv, hd)).astype(np.float32)
    vals = rng.standard_normal((n_layers, max_seq, n_kv, hd)).astype(np.float32)
    kv.keys.copy_(cuda.from_numpy(keys))
    kv.values.copy_(cuda.from_numpy(vals))
    q = rng.standard_normal(n_heads * hd).astype(np.float32)
    qd = cuda.from_numpy(q).cuda()
    for layer, pos in ((0, 1), (1, max_seq // 2), (1, max_seq - 1)):
        out = pkg.CudaAttentionDecodeDeviceInput(qd, kv, layer, pos, n_heads, n_kv, hd)
        ref = orc.attention(q, keys, vals, layer, pos, n_heads)
        assert_close(out.cpu().numpy(), ref, f"layer {layer} pos {pos}")
    out = pkg.CudaAttentionDecodeDeviceInput(qd, kv, 1, 0, n_heads, n_kv, hd).cpu().numpy()
    exp = np.concatenate([vals[1, 0, h // (n_heads // n_kv)] for h in range(n_heads)])
    assert np.array_equal(bits(out), bits(exp))


@pytest.mark.parametrize("qt", [1, 2])
def test_lm_head_block_sums_exact(pkg, orc, S, cuda, qt):
    """The TMA-staged GEMV's integer path, bit for bit: x split into three int8
    terms per 32-value block (terms and scales equal to the host integer
    restatement), and the int32 dp4a sums of every block of every row against
    each term equal to exact integer sums -- at the five Qwen2-0.5B GEMV
    shapes.  The terms also reconstruct x to within 1e-7 of each block's
    largest magnitude."""
    torch = cuda
    L = pkg.lib()
    for o, i in ((896, 896), (128, 896), (4864, 896), (896, 4864), (151936, 896)):
        blocks, x = S.gemv_case(o, i, 5 + o % 97, qt)
        packed = pkg.pack_weight(qt, blocks, o, i)
        nb = (i + 31) // 32
        q = torch.empty(3 * nb * 32, dtype=torch.int8, device="cuda")
        sc = torch.empty(3 * nb, dtype=torch.float32, device="cuda")
        sums = torch.empty(o * 3 * nb, dtype=torch.int32, device="cuda")
        xd = torch.from_numpy(x).cuda()
        pkg.check(L.dqmk_lm_head_block_sums(qt, xd.data_ptr(), i, packed.data_ptr(), o,
                                            q.data_ptr(), sc.data_ptr(), sums.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        rq, rsc = orc.x_terms(x)
        assert np.array_equal(q.cpu().numpy().reshape(3, nb, 32), rq), (o, i)
        assert np.array_equal(sc.cpu().numpy().view(np.uint32), rsc.reshape(-1).view(np.uint32))
        ref = orc.block_term_sums(qt, blocks, o, i, rq)
        assert np.array_equal(sums.cpu().numpy().reshape(o, 3, nb).astype(np.int64), ref), (o, i)
        recon = np.einsum("tbj,tb->bj", rq.astype(np.float64), rsc.astype(np.float64))
        xb = np.zeros((nb, 32))
        xb.reshape(-1)[:i] = x
        assert np.all(np.abs(recon - xb) <= 1e-7 * np.abs(xb).max(axis=1, keepdims=True) + 1e-30)
