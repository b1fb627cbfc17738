"""ctypes binding of libdqmk.so (the C ABI in include/dqmk.h).

The library is built in-tree by csrc/Makefile.  Loading fails loudly when it
is missing: there is no CPU or eager fallback for any entry point.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdqmk.so")

DQMK_OK = 0
DQMK_ERR_INVALID = 1
DQMK_ERR_RANGE = 2
DQMK_ERR_CUDA = 3
DQMK_ERR_TIMEOUT = 4
DQMK_ERR_UNSUPPORTED = 5
DQMK_ERR_NOMEM = 6

F32, Q80, Q40, Q41 = 0, 1, 2, 3

# Every symbol include/dqmk.h declares, with its ctypes signature.
_vp, _i, _i64, _sz, _f = C.c_void_p, C.c_int, C.c_int64, C.c_size_t, C.c_float
_ip = C.POINTER(C.c_int)
_fp = C.POINTER(C.c_float)


class ModelConfig(C.Structure):
    """dqmk_model_config = ModelConfig (include/dqm_llama/model.h:23-35)."""
    _fields_ = [("vocab_size", _i), ("dim", _i), ("hidden_dim", _i), ("n_layers", _i),
                ("n_heads", _i), ("n_kv_heads", _i), ("head_dim", _i), ("max_seq_len", _i),
                ("rope_theta", _f), ("rms_norm_eps", _f), ("rope_neox", _i)]


class ModelStats(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in (
        "uploaded_weight_count", "uploaded_bytes", "linear_calls", "activation_calls",
        "attention_calls", "kv_cache_write_bytes", "kv_cache_read_bytes",
        "host_to_device_copies", "device_to_host_copies", "host_to_device_bytes",
        "device_to_host_bytes")]


class TpPlan(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("rank", "world", "q_head0", "n_q_heads", "kv_head0",
                                         "n_kv_heads", "hidden0", "hidden", "vocab0", "vocab",
                                         "vocab_stride")]


SIGNATURES = {
    "dqmk_last_error": ([], C.c_char_p),
    "dqmk_built": ([], _i),
    "dqmk_quantize_q80": ([_vp, _i64, _i64, _vp, _vp], _i),
    "dqmk_quantize_q40": ([_vp, _i64, _i64, _vp, _vp], _i),
    "dqmk_dequantize_q80": ([_vp, _i64, _i64, _vp, _vp], _i),
    "dqmk_dequantize_q40": ([_vp, _i64, _i64, _vp, _vp], _i),
    "dqmk_q80_linear": ([_vp, _i, _i, _vp, _sz, _i, _vp, _vp, _vp], _i),
    "dqmk_q40_linear": ([_vp, _i, _i, _vp, _sz, _i, _vp, _vp, _vp], _i),
    "dqmk_q41_linear": ([_vp, _i, _i, _vp, _sz, _i, _vp, _vp, _vp], _i),
    "dqmk_f32_linear": ([_vp, _i, _i, _vp, _i, _vp, _vp, _vp], _i),
    "dqmk_packed_bytes": ([_i, _i, _i], _sz),
    "dqmk_pack_weight": ([_i, _vp, _sz, _i, _i, _vp, _vp], _i),
    "dqmk_gemv_packed": ([_i, _vp, _i, _vp, _i, _vp, _vp, _vp, _vp], _i),
    "dqmk_linear_batch_packed": ([_i, _vp, _i, _i, _vp, _i, _vp, _vp, _vp, _vp], _i),
    "dqmk_linear_cols_packed": ([_i, _vp, _i, _i, _vp, _i, _vp, _vp, _vp, _vp], _i),
    "dqmk_device_error": ([_i], _i),
    "dqmk_gemv_packed_withhold_tile": ([_i, _vp, _i, _vp, _i, _vp, _i, _vp], _i),
    "dqmk_context_withhold_lm_head": ([_vp, _i], _i),
    "dqmk_forward_batch_prefix": ([_vp, _vp, _i, _vp, _vp], _i),
    "dqmk_gguf_read_config": ([C.c_char_p, _vp], _i),
    "dqmk_model_load_gguf": ([C.c_char_p, _i, _i, _vp], _i),
    "dqmk_gemv_packed_chained": ([_i, _vp, _i, _vp, _i, _vp, _f, _i, _vp, _vp], _i),
    "dqmk_lm_head_block_sums": ([_i, _vp, _i, _vp, _i, _vp, _vp, _vp, _vp], _i),
    "dqmk_rmsnorm": ([_vp, _vp, _i, _f, _vp, _vp], _i),
    "dqmk_silu_mul": ([_vp, _vp, _i, _vp, _vp], _i),
    "dqmk_add": ([_vp, _vp, _i, _vp, _vp], _i),
    "dqmk_silu": ([_vp, _i, _vp, _vp], _i),
    "dqmk_mul": ([_vp, _vp, _i, _vp, _vp], _i),
    "dqmk_softmax": ([_vp, _i, _vp, _vp], _i),
    "dqmk_rope": ([_vp, _vp, _i, _i, _i, _i, _f, _i, _vp], _i),
    "dqmk_embedding_lookup": ([_vp, _i, _i, _i, _vp, _vp], _i),
    "dqmk_embedding_lookup_blocks": ([_i, _vp, _i, _i, _i, _vp, _vp], _i),
    "dqmk_argmax": ([_vp, _i, _vp, _vp], _i),
    "dqmk_kv_write": ([_vp, _vp, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp], _i),
    "dqmk_attention_decode": ([_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _vp], _i),
    "dqmk_attention_decode_noalloc": ([_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _vp], _i),
    "dqmk_model_create": ([C.POINTER(ModelConfig), _i, C.POINTER(_vp)], _i),
    "dqmk_model_destroy": ([_vp], _i),
    "dqmk_model_upload": ([_vp, C.c_char_p, _i, _vp, _sz, _i, _i], _i),
    "dqmk_model_finalize": ([_vp], _i),
    "dqmk_tp_plan_get": ([C.POINTER(ModelConfig), _i, _i, C.POINTER(TpPlan)], _i),
    "dqmk_nccl_unique_id": ([C.c_char_p], _i),
    "dqmk_model_set_tp": ([_vp, _i, _i, C.c_char_p], _i),
    "dqmk_context_tp_ipc_handle": ([_vp, C.c_char_p], _i),
    "dqmk_context_tp_connect": ([_vp, C.c_char_p], _i),
    "dqmk_model_stats_get": ([_vp, C.POINTER(ModelStats)], _i),
    "dqmk_model_stats_reset": ([_vp], _i),
    "dqmk_model_memory_bytes": ([_vp], _sz),
    "dqmk_context_create": ([_vp, C.POINTER(_vp)], _i),
    "dqmk_context_destroy": ([_vp], _i),
    "dqmk_context_reset": ([_vp], _i),
    "dqmk_context_pos": ([_vp], _i),
    "dqmk_context_history": ([_vp, _ip, _i], _i),
    "dqmk_forward_token": ([_vp, _i, _i, _fp], _i),
    "dqmk_forward_batch": ([_vp, _ip, _ip, _i, _fp], _i),
    "dqmk_decode_greedy": ([_vp, _i, _i, _i, _ip], _i),
    "dqmk_decode_enqueue": ([_vp, _i, _i, _i], _i),
    "dqmk_context_stream": ([_vp], _vp),
    "dqmk_batch_create": ([_vp, _i, _i, C.POINTER(_vp)], _i),
    "dqmk_batch_destroy": ([_vp], _i),
    "dqmk_batch_reset": ([_vp], _i),
    "dqmk_batch_step": ([_vp, _ip, _ip, _ip, _i, _fp, _ip], _i),
    "dqmk_batch_decode_greedy": ([_vp, _ip, _ip, _i, _i, _ip], _i),
    "dqmk_batch_decode_enqueue": ([_vp, _ip, _ip, _i, _i], _i),
    "dqmk_batch_stream": ([_vp], _vp),
    "dqmk_batch_history": ([_vp, _i, _i, _i, _ip], _i),
}

_lib = None


class OutOfRange(IndexError):
    """Status DQMK_ERR_RANGE: the reference throws std::out_of_range here."""


class CudaError(RuntimeError):
    pass


def build(quiet: bool = True) -> None:
    """Compile libdqmk.so for sm_100a (nvcc cross-compiles without a GPU)."""
    cmd = ["make", "-C", os.path.join(HERE, "csrc"), "-j8"]
    if quiet:
        cmd.insert(1, "-s")
    subprocess.run(cmd, check=True)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                "libdqmk.so is not built (run __graft_entry__.build()); the CUDA path has no "
                "fallback")
        L = C.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def check(status: int) -> None:
    """Raise the exception the reference would throw for a failed call."""
    if status == DQMK_OK:
        return
    msg = lib().dqmk_last_error().decode(errors="replace")
    if status == DQMK_ERR_RANGE:
        raise OutOfRange(msg)
    if status in (DQMK_ERR_CUDA, DQMK_ERR_NOMEM, DQMK_ERR_TIMEOUT):
        raise CudaError(msg)
    raise RuntimeError(msg)
