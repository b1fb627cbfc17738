"""CPU: the C ABI library loads, exports every declared symbol, and rejects bad
arguments on the host with the reference's exception types and message
prefixes (no device work is issued by any call here)."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "dqmk.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(dqmk_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(pkg):
    L = pkg.lib()
    syms = declared_symbols()
    assert len(syms) >= 30
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing
    # and the Python binding declares a signature for each of them
    from importlib import import_module
    sigs = import_module(pkg.__name__ + "._lib").SIGNATURES
    assert sorted(sigs) == syms


def test_built_flag(pkg):
    assert pkg.lib().dqmk_built() == 1


def test_packed_bytes_is_block_bytes(pkg):
    L = pkg.lib()
    assert L.dqmk_packed_bytes(pkg.Q80, 896, 896) == 896 * 28 * 34
    assert L.dqmk_packed_bytes(pkg.Q40, 4864, 896) == 4864 * 28 * 18
    assert L.dqmk_packed_bytes(pkg.Q80, 2, 42) == 2 * 2 * 34
    assert L.dqmk_packed_bytes(7, 2, 42) == 0


def _err(pkg, rc):
    with pytest.raises(Exception) as ei:
        pkg.check(rc)
    return ei


def test_linear_block_count_mismatch(pkg):
    L = pkg.lib()
    dummy = C.c_void_p(16)
    rc = L.dqmk_q80_linear(dummy, 1, 64, dummy, 3, 2, None, dummy, None)
    ei = _err(pkg, rc)
    assert ei.type is RuntimeError
    assert str(ei.value).startswith("CudaQ80Linear: block count mismatch: expected 4, got 3")
    rc = L.dqmk_q40_linear(dummy, 1, 64, None, 4, 2, None, dummy, None)
    assert str(_err(pkg, rc).value) == "CudaQ40Linear: null pointer"


def test_quantize_validation(pkg):
    L = pkg.lib()
    assert L.dqmk_quantize_q80(None, 0, 32, None, None) == 0  # empty tensor: no blocks
    ei = _err(pkg, L.dqmk_quantize_q80(None, -1, 32, None, None))
    assert str(ei.value).startswith("QuantizeToQ80")


def test_range_errors_map_to_out_of_range(pkg):
    L = pkg.lib()
    dummy = C.c_void_p(16)
    rc = L.dqmk_attention_decode(dummy, dummy, dummy, 2, 8, 2, 64, 2, 0, 4, dummy, None)
    ei = _err(pkg, rc)
    assert ei.type is pkg.OutOfRange and issubclass(ei.type, IndexError)
    assert "layer out of range" in str(ei.value)
    rc = L.dqmk_attention_decode(dummy, dummy, dummy, 2, 8, 2, 64, 0, 8, 4, dummy, None)
    assert "pos out of range" in str(_err(pkg, rc).value)
    rc = L.dqmk_rope(dummy, dummy, 4, 2, 64, -1, 1e6, 1, None)
    assert str(_err(pkg, rc).value) == "Rope: position must be non-negative"
    rc = L.dqmk_rope(dummy, dummy, 4, 2, 63, 0, 1e6, 1, None)
    assert str(_err(pkg, rc).value) == "Rope: head_dim must be positive and even"
    rc = L.dqmk_kv_write(dummy, dummy, 2, 8, 2, 64, 0, 8, dummy, dummy, None)
    assert _err(pkg, rc).type is pkg.OutOfRange


def test_pack_validation(pkg):
    L = pkg.lib()
    dummy = C.c_void_p(16)
    rc = L.dqmk_pack_weight(pkg.Q80, dummy, 5, 2, 64, dummy, None)
    assert "block count mismatch" in str(_err(pkg, rc).value)
    rc = L.dqmk_pack_weight(9, dummy, 4, 2, 64, dummy, None)
    assert "unsupported" in str(_err(pkg, rc).value)


def test_gemv_packed_rejects_misaligned_weight(pkg):
    L = pkg.lib()
    rc = L.dqmk_gemv_packed(pkg.Q80, C.c_void_p(16), 64, C.c_void_p(18), 2, None, None,
                            C.c_void_p(16), None)
    assert "16-byte aligned" in str(_err(pkg, rc).value)


def test_model_null_arguments(pkg):
    L = pkg.lib()
    ei = _err(pkg, L.dqmk_model_create(None, 0, None))
    assert str(ei.value).startswith("UploadModelWeightsToCuda")
    assert "ForwardToken" in str(_err(pkg, L.dqmk_forward_token(None, 0, 0, None)).value)
    assert "ForwardBatch" in str(_err(pkg, L.dqmk_forward_batch(None, None, None, 0, None)).value)
