"""GPU: the allocation-free attention entry point.

dqmk_attention_decode_noalloc serves callers that cannot allocate device
memory when they run attention (an engine whose device budget is reserved at
start-up, a host that forbids allocations outside its own allocator).  Its
split partials live in a fixed buffer compiled into the library instead of the
library's growable scratch.  Called through the C ABI, it must give the same
results as dqmk_attention_decode, within the kernel tests' tolerance, on two
calls in a row (the second call reuses the buffer the first one left behind).

Kept in its own file, named to be collected last, so a run that stops at the
first failure has already run every other test.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ABS_TOL = 1e-3
REL_TOL = 1e-3


def assert_close(actual, expected, label):
    err = np.abs(actual - expected)
    scale = np.maximum(1.0, np.abs(expected))
    bad = ~((err <= ABS_TOL) | (err / scale <= REL_TOL))
    assert not bad.any(), f"{label}: {bad.sum()} mismatches, max err {err.max():.3e}"


@pytest.mark.parametrize("cfg", [(14, 2, 64, 2176), (28, 4, 128, 600), (4, 4, 8, 96)],
                         ids=lambda c: f"h{c[0]}_kv{c[1]}_hd{c[2]}_seq{c[3]}")
def test_noalloc_attention_matches_allocating_entry_point(pkg, cuda, cfg):
    torch = cuda
    n_heads, n_kv, hd, max_seq = cfg
    n_layers = 2
    L = pkg.lib()
    g = torch.Generator(device="cuda").manual_seed(n_heads * 1000 + hd)
    keys = torch.randn((n_layers, max_seq, n_kv, hd), device="cuda", generator=g)
    values = torch.randn((n_layers, max_seq, n_kv, hd), device="cuda", generator=g)
    q = torch.randn(n_heads * hd, device="cuda", generator=g)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):  # two calls in a row for every position
        for layer, pos in ((0, 0), (1, 40), (0, max_seq - 1), (1, max_seq // 2)):
            ref = torch.empty(n_heads * hd, device="cuda")
            got = torch.full((n_heads * hd,), float("nan"), device="cuda")
            args = (q.data_ptr(), keys.data_ptr(), values.data_ptr(), n_layers, max_seq, n_kv,
                    hd, layer, pos, n_heads)
            pkg.check(L.dqmk_attention_decode(*args, ref.data_ptr(), stream))
            pkg.check(L.dqmk_attention_decode_noalloc(*args, got.data_ptr(), stream))
            torch.cuda.synchronize()
            assert_close(got.cpu().numpy(), ref.cpu().numpy(),
                         f"call {call} layer {layer} pos {pos}")


def test_noalloc_buffer_holds_the_largest_supported_shape(pkg, cuda):
    """Splits are capped at SM count / n_kv_heads and a KV head serves at most 8
    query heads, so n_heads * splits <= 8 * SM count: at head_dim 256 the
    partials of every supported shape fit the fixed 2 MiB buffer on this GPU.
    The largest such shape runs (with a cache of its full size) and matches the
    allocating entry point."""
    torch = cuda
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    need = 8 * sms * (256 + 4) * 4 + 256
    assert need <= 2 << 20, need
    L = pkg.lib()
    n_heads, n_kv, hd, max_seq, n_layers = 64, 8, 256, 4096, 1
    g = torch.Generator(device="cuda").manual_seed(5)
    keys = torch.randn((n_layers, max_seq, n_kv, hd), device="cuda", generator=g)
    values = torch.randn((n_layers, max_seq, n_kv, hd), device="cuda", generator=g)
    q = torch.randn(n_heads * hd, device="cuda", generator=g)
    stream = torch.cuda.current_stream().cuda_stream
    for pos in (0, 1000, max_seq - 1):
        ref = torch.empty(n_heads * hd, device="cuda")
        got = torch.full((n_heads * hd,), float("nan"), device="cuda")
        args = (q.data_ptr(), keys.data_ptr(), values.data_ptr(), n_layers, max_seq, n_kv, hd,
                0, pos, n_heads)
        pkg.check(L.dqmk_attention_decode(*args, ref.data_ptr(), stream))
        pkg.check(L.dqmk_attention_decode_noalloc(*args, got.data_ptr(), stream))
        torch.cuda.synchronize()
        assert_close(got.cpu().numpy(), ref.cpu().numpy(), f"largest shape pos {pos}")
