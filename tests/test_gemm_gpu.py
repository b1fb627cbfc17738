"""GPU parity of the batched (prefill) linear on the tensor cores.

dqmk_linear_batch_packed computes the rows of LinearQ80 / LinearQ40
(src/quant.cc:350-360) for m activation rows at once.  Each dequantized
weight d*q is exact as two fp16 terms once its row is scaled by a power of
two; each activation row is scaled likewise and split into two fp16 terms
(x 2^-e = hi + lo, relative error <= 2^-22); the tensor core accumulates
hi*hi + hi*lo + lo*hi in fp32 over all of K.  The test bound per output is

    |y - ref| <= 1e-5 * sum_k |W[o,k] x[k]|

(fp32 summation in a different order than the reference's per-element FMA
chain, plus the 2^-22 split and the dropped lo*lo term), against the
oracle's F32 LinearQ80 / LinearQ40 (itself pinned to the reference), on
ragged shapes: single rows, rows across
the 128-row tile boundary, K tails (in % 32 != 0, in % 128 != 0),
out % 128 != 0, split-K (few output tiles), a zero row, rows with outliers,
bias and an in-place residual.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CASES = [
    # (qtype, m, in, out)
    (1, 1, 896, 896), (1, 3, 13, 5), (1, 64, 65, 17), (1, 128, 896, 1152),
    (1, 129, 704, 300), (1, 602, 896, 4864), (1, 257, 4864, 896),
    (2, 33, 896, 896), (2, 130, 896, 4864), (2, 5, 65, 17), (2, 300, 4864, 896),
]


def make_x(m, k, seed):
    g = np.random.default_rng(seed)
    x = g.standard_normal((m, k), dtype=np.float32)
    if m > 2:
        x[1] = 0.0                      # a zero row: every block scale is 0
        x[2, ::97] *= 300.0             # outliers dominate their blocks
    return x


def error_bound(orc, qt, x, blocks, o):
    w = orc.dequantize(qt, blocks, o, x.shape[1])  # [o, k] F32, exact block values
    return 1e-5 * (np.abs(x).astype(np.float64) @ np.abs(w).astype(np.float64).T) + 1e-30


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"q{c[0]}_m{c[1]}_{c[2]}to{c[3]}")
def test_linear_batch_matches_oracle(pkg, orc, S, cuda, case):
    torch = cuda
    qt, m, k, o = case
    blocks, _ = S.gemv_case(o, k, 100 + m, qt)
    x = make_x(m, k, 7 * m + k)
    packed = pkg.pack_weight(qt, blocks, o, k)
    y = pkg.linear_batch_packed(qt, torch.from_numpy(x).cuda(), packed, o).cpu().numpy()
    ref = orc.linear(qt, x, blocks, o)
    bound = error_bound(orc, qt, x, blocks, o)
    err = np.abs(y.astype(np.float64) - ref)
    worst = np.unravel_index(np.argmax(err - bound), err.shape)
    assert np.all(err <= bound), (f"row {worst[0]} col {worst[1]}: err {err[worst]:.3e} "
                                  f"> bound {bound[worst]:.3e}")
    if m > 2:
        assert np.all(y[1] == 0.0)
    rel = float(err.max() / max(1e-30, np.abs(ref).max()))
    print(f"{case}: max err / max |ref| = {rel:.2e}")


def test_linear_batch_bias_and_inplace_residual(pkg, orc, S, cuda):
    torch = cuda
    m, k, o = 200, 896, 896
    blocks, _ = S.gemv_case(o, k, 3)
    x = make_x(m, k, 11)
    g = np.random.default_rng(5)
    bias = g.standard_normal(o, dtype=np.float32)
    res = g.standard_normal((m, o), dtype=np.float32)
    packed = pkg.pack_weight(pkg.Q80, blocks, o, k)
    rd = torch.from_numpy(res).cuda()
    pkg.linear_batch_packed(pkg.Q80, torch.from_numpy(x).cuda(), packed, o,
                            bias=torch.from_numpy(bias).cuda(), residual=rd, y=rd)
    got = rd.cpu().numpy()
    ref = orc.linear(pkg.Q80, x, blocks, o)
    bound = error_bound(orc, pkg.Q80, x, blocks, o) + 1e-6 * (np.abs(res) + np.abs(bias))
    assert np.all(np.abs(got - (res + (ref + bias))) <= bound)


def test_linear_batch_validation(pkg, cuda):
    torch = cuda
    L = pkg.lib()
    x = torch.zeros(4, 32, device="cuda")
    y = torch.zeros(4, 32, device="cuda")
    packed = torch.zeros(64 * 34, dtype=torch.uint8, device="cuda")
    assert L.dqmk_linear_batch_packed(0, x.data_ptr(), 4, 32, packed.data_ptr(), 32, None, None,
                                      y.data_ptr(), None) == pkg._lib.DQMK_ERR_UNSUPPORTED
    assert L.dqmk_linear_batch_packed(1, x.data_ptr(), 0, 32, packed.data_ptr(), 32, None, None,
                                      y.data_ptr(), None) == pkg._lib.DQMK_ERR_INVALID
    assert L.dqmk_linear_batch_packed(1, x.data_ptr(), 4, 32, packed.data_ptr() + 1, 32, None,
                                      None, y.data_ptr(), None) == pkg._lib.DQMK_ERR_INVALID
