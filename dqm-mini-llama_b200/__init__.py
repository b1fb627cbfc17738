"""B200 (sm_100a) block-quantized matmul path for the dqm-mini-llama engine.

Host-side mirror of the reference's CUDA operator interface (names, argument
meaning and exceptions follow include/dqm_llama/cuda_quant.h, cuda_ops.h,
cuda_attention.h, cuda_kv_cache.h, forward.h).  Every call goes through the
C ABI of libdqmk.so (include/dqmk.h); torch is used only to own device memory
and to hand its pointers over.  Errors surface as RuntimeError, or OutOfRange
(an IndexError) where the reference throws std::out_of_range.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence

import numpy as np

from . import synth
from ._lib import (F32, Q40, Q41, Q80, CudaError, ModelConfig, ModelStats, OutOfRange, TpPlan,
                   build, check, lib)

__all__ = [
    "F32", "Q80", "Q40", "Q41", "OutOfRange", "CudaError", "build", "lib", "synth",
    "QuantizeToQ80", "QuantizeToQ40", "DequantizeFromQ80", "DequantizeFromQ40",
    "CudaQ80Linear", "CudaQ40Linear", "CudaQ80LinearDeviceInput", "CudaQ40LinearDeviceInput",
    "pack_weight", "gemv_packed", "CudaRmsNormDeviceWeight", "CudaSiluMulDeviceInput",
    "CudaElementwiseAddDeviceInput", "CudaRopeDeviceInput", "CudaEmbeddingLookupDeviceWeight",
    "embedding_lookup_blocks", "argmax", "CudaKvCache", "CudaAttentionDecodeDeviceInput",
    "Model", "Context", "Batch", "BLOCK_BYTES", "linear_batch_packed", "linear_cols_packed",
    "CudaQ41Linear", "CudaQ41LinearDeviceInput", "CudaLinear", "CudaLinearDeviceInput",
]

BLOCK_BYTES = {Q80: 34, Q40: 18, Q41: 20}


def _torch():
    import torch
    return torch


def _stream(stream=None) -> Optional[int]:
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream if hasattr(s, "cuda_stream") else s


def _ptr(t) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _dev(x, dtype=None):
    """numpy / torch -> contiguous CUDA tensor."""
    torch = _torch()
    if isinstance(x, np.ndarray):
        x = torch.from_numpy(np.ascontiguousarray(x))
    if dtype is not None and x.dtype != dtype:
        x = x.to(dtype)
    return x.cuda().contiguous()


def _nblocks(rows: int, cols: int) -> int:
    return rows * ((cols + 31) // 32)


# ------------------------------------------------------------ quantization
def _quantize(qtype: int, src):
    torch = _torch()
    src = _dev(src, torch.float32)
    cols = src.shape[-1] if src.dim() else 0
    rows = src.numel() // cols if cols else 0
    out = torch.zeros(_nblocks(rows, cols) * BLOCK_BYTES[qtype], dtype=torch.uint8, device="cuda")
    fn = lib().dqmk_quantize_q80 if qtype == Q80 else lib().dqmk_quantize_q40
    check(fn(_ptr(src), rows, cols, _ptr(out), _stream()))
    return out


def QuantizeToQ80(src):
    """QuantizeToQ80 (src/quant.cc:372-418) on the device; returns uint8 blocks."""
    return _quantize(Q80, src)


def QuantizeToQ40(src):
    """QuantizeToQ40 (src/quant.cc:420-476) on the device; returns uint8 blocks."""
    return _quantize(Q40, src)


def _dequantize(qtype, blocks, shape):
    torch = _torch()
    blocks = _dev(blocks, torch.uint8)
    cols = shape[-1]
    rows = int(np.prod(shape[:-1])) if len(shape) > 1 else 1
    out = torch.empty(tuple(shape), dtype=torch.float32, device="cuda")
    fn = lib().dqmk_dequantize_q80 if qtype == Q80 else lib().dqmk_dequantize_q40
    if blocks.numel() != _nblocks(rows, cols) * BLOCK_BYTES[qtype]:
        raise RuntimeError(("DequantizeFromQ80" if qtype == Q80 else "DequantizeFromQ40") +
                           ": block count mismatch")
    check(fn(_ptr(blocks), rows, cols, _ptr(out), _stream()))
    return out


def DequantizeFromQ80(blocks, shape):
    return _dequantize(Q80, blocks, shape)


def DequantizeFromQ40(blocks, shape):
    return _dequantize(Q40, blocks, shape)


# ------------------------------------------------------------ Linear
def _linear_device(qtype, x, blocks, block_count, weight_shape, bias=None):
    torch = _torch()
    if len(weight_shape) != 2:
        raise RuntimeError("LinearQuantized: expected 2D weight shape")
    out_f, in_f = weight_shape
    name = {Q80: "CudaQ80Linear", Q40: "CudaQ40Linear", Q41: "CudaQ41Linear"}[qtype]
    if x.shape[-1] != in_f:
        raise RuntimeError(name + ": dimension mismatch")
    rows = 1 if x.dim() == 1 else x.shape[0]
    y = torch.empty((out_f,) if x.dim() == 1 else (rows, out_f), dtype=torch.float32,
                    device=x.device)
    fn = {Q80: lib().dqmk_q80_linear, Q40: lib().dqmk_q40_linear,
          Q41: lib().dqmk_q41_linear}[qtype]
    check(fn(_ptr(x), rows, in_f, _ptr(blocks), block_count, out_f, _ptr(bias), _ptr(y),
             _stream()))
    return y


def CudaQ80LinearDeviceInput(x, q8_0_device, block_count: int, weight_shape):
    """include/dqm_llama/cuda_quant.h:27-31: device x, device ggml blocks -> device y."""
    return _linear_device(Q80, x, q8_0_device, block_count, weight_shape)


def CudaQ40LinearDeviceInput(x, q4_0_device, block_count: int, weight_shape):
    return _linear_device(Q40, x, q4_0_device, block_count, weight_shape)


def CudaQ41LinearDeviceInput(x, q4_1_device, block_count: int, weight_shape):
    """include/dqm_llama/cuda_quant.h:59-63."""
    return _linear_device(Q41, x, q4_1_device, block_count, weight_shape)


def CudaLinearDeviceInput(x, w_device, weight_shape, bias=None):
    """include/dqm_llama/cuda_matmul.h:35-41: F32 weight [out, in] on the device."""
    torch = _torch()
    out_f, in_f = weight_shape
    if x.shape[-1] != in_f:
        raise RuntimeError("CudaLinear: dimension mismatch")
    rows = 1 if x.dim() == 1 else x.shape[0]
    y = torch.empty((out_f,) if x.dim() == 1 else (rows, out_f), dtype=torch.float32,
                    device=x.device)
    check(lib().dqmk_f32_linear(_ptr(x), rows, in_f, _ptr(w_device), out_f, _ptr(bias), _ptr(y),
                                _stream()))
    return y


def CudaLinear(x, weight, bias=None):
    """include/dqm_llama/cuda_matmul.h:25-27: host x and F32 weight [out, in]."""
    torch = _torch()
    w = _dev(weight, torch.float32)
    y = CudaLinearDeviceInput(_dev(x, torch.float32), w, tuple(w.shape),
                              None if bias is None else _dev(bias, torch.float32))
    torch.cuda.current_stream().synchronize()
    return y.cpu().numpy()


def _linear_host(qtype, x, blocks, weight_shape, bias=None):
    torch = _torch()
    xd = _dev(x, torch.float32)
    bd = _dev(blocks, torch.uint8)
    biasd = None if bias is None else _dev(bias, torch.float32)
    y = _linear_device(qtype, xd, bd, bd.numel() // BLOCK_BYTES[qtype], weight_shape, biasd)
    torch.cuda.current_stream().synchronize()
    return y.cpu().numpy()


def CudaQ80Linear(x, weight_blocks, weight_shape, bias=None):
    """include/dqm_llama/cuda_quant.h:17-19: host tensors in, host tensor out."""
    return _linear_host(Q80, x, weight_blocks, weight_shape, bias)


def CudaQ40Linear(x, weight_blocks, weight_shape, bias=None):
    return _linear_host(Q40, x, weight_blocks, weight_shape, bias)


def CudaQ41Linear(x, weight_blocks, weight_shape, bias=None):
    """include/dqm_llama/cuda_quant.h:49-51."""
    return _linear_host(Q41, x, weight_blocks, weight_shape, bias)


def pack_weight(qtype: int, blocks, out_features: int, in_features: int):
    """ggml blocks -> the planar layout the engine streams (include/dqmk.h)."""
    torch = _torch()
    blocks = _dev(blocks, torch.uint8)
    nbytes = lib().dqmk_packed_bytes(qtype, out_features, in_features)
    packed = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    check(lib().dqmk_pack_weight(qtype, _ptr(blocks), blocks.numel() // BLOCK_BYTES[qtype],
                                 out_features, in_features, _ptr(packed), _stream()))
    return packed


def gemv_packed(qtype: int, x, packed, out_features: int, bias=None, residual=None, y=None,
                stream=None):
    torch = _torch()
    if y is None:
        y = torch.empty(out_features, dtype=torch.float32, device=x.device)
    check(lib().dqmk_gemv_packed(qtype, _ptr(x), x.shape[-1], _ptr(packed), out_features,
                                 _ptr(bias), _ptr(residual), _ptr(y), _stream(stream)))
    return y


def gemv_packed_chained(qtype: int, x, packed, out_features: int, y, norm=None, eps=1e-6,
                        swiglu=False, stream=None):
    """The decode step's GEMV launched as the step chains it (programmatic
    dependent launch), with optional RMSNorm prologue and SwiGLU epilogue."""
    check(lib().dqmk_gemv_packed_chained(qtype, _ptr(x), x.shape[-1], _ptr(packed), out_features,
                                         _ptr(norm), float(eps), 1 if swiglu else 0, _ptr(y),
                                         _stream(stream)))
    return y


def linear_batch_packed(qtype: int, x, packed, out_features: int, bias=None, residual=None,
                        y=None, stream=None):
    """x [m, in] (device, float32) times a packed weight on the tensor cores."""
    torch = _torch()
    m, k = x.shape
    if y is None:
        y = torch.empty(m, out_features, dtype=torch.float32, device=x.device)
    check(lib().dqmk_linear_batch_packed(qtype, _ptr(x), m, k, _ptr(packed), out_features,
                                         _ptr(bias), _ptr(residual), _ptr(y), _stream(stream)))
    return y


def linear_cols_packed(qtype: int, x, packed, out_features: int, bias=None, residual=None,
                       y=None, stream=None):
    """x [cols, in] (device, float32, 1..64 columns, one per sequence) times a
    packed weight the way a multi-sequence decode step runs it: the quantized
    blocks stream once and become tensor-core operands on chip."""
    torch = _torch()
    m, k = x.shape
    if y is None:
        y = torch.empty(m, out_features, dtype=torch.float32, device=x.device)
    check(lib().dqmk_linear_cols_packed(qtype, _ptr(x), m, k, _ptr(packed), out_features,
                                        _ptr(bias), _ptr(residual), _ptr(y), _stream(stream)))
    return y


# ------------------------------------------------------------ ops
def CudaRmsNormDeviceWeight(x, weight, eps: float):
    torch = _torch()
    y = torch.empty_like(x)
    if weight.numel() != x.numel():
        raise RuntimeError("ops: RmsNorm: dim not compare")
    check(lib().dqmk_rmsnorm(_ptr(x), _ptr(weight), x.numel(), eps, _ptr(y), _stream()))
    return y


def CudaSiluMulDeviceInput(gate, up):
    """CudaSiluDeviceInput + CudaElementwiseMulDeviceInput = SwiGlu."""
    torch = _torch()
    if gate.shape != up.shape:
        raise RuntimeError("SwiGlu: shape mismatch")
    y = torch.empty_like(gate)
    check(lib().dqmk_silu_mul(_ptr(gate), _ptr(up), gate.numel(), _ptr(y), _stream()))
    return y


def CudaElementwiseAddDeviceInput(a, b):
    torch = _torch()
    if a.shape != b.shape:
        raise RuntimeError("CudaElementwiseAdd: shape mismatch")
    y = torch.empty_like(a)
    check(lib().dqmk_add(_ptr(a), _ptr(b), a.numel(), _ptr(y), _stream()))
    return y


def CudaRopeDeviceInput(q, k, n_heads: int, n_kv_heads: int, head_dim: int, pos: int,
                        theta: float, neox: bool = True):
    """In place, like the reference (include/dqm_llama/cuda_ops.h:57-61)."""
    check(lib().dqmk_rope(_ptr(q), _ptr(k), n_heads, n_kv_heads, head_dim, pos, theta,
                          1 if neox else 0, _stream()))


def CudaEmbeddingLookupDeviceWeight(table, token: int):
    torch = _torch()
    vocab, dim = table.shape
    y = torch.empty(dim, dtype=torch.float32, device=table.device)
    check(lib().dqmk_embedding_lookup(_ptr(table), vocab, dim, token, _ptr(y), _stream()))
    return y


def embedding_lookup_blocks(qtype: int, blocks, vocab: int, dim: int, token: int):
    torch = _torch()
    y = torch.empty(dim, dtype=torch.float32, device=blocks.device)
    check(lib().dqmk_embedding_lookup_blocks(qtype, _ptr(blocks), vocab, dim, token, _ptr(y),
                                             _stream()))
    return y


def argmax(x) -> int:
    torch = _torch()
    out = torch.zeros(1, dtype=torch.int32, device=x.device)
    check(lib().dqmk_argmax(_ptr(x), x.numel(), _ptr(out), _stream()))
    return int(out.item())


class CudaKvCache:
    """include/dqm_llama/cuda_kv_cache.h:17-72: f32 [layers][max_seq][kv][hd]."""

    def __init__(self, n_layers: int, max_seq_len: int, n_kv_heads: int, head_dim: int):
        torch = _torch()
        shape = (n_layers, max_seq_len, n_kv_heads, head_dim)
        self.keys = torch.zeros(shape, dtype=torch.float32, device="cuda")
        self.values = torch.zeros(shape, dtype=torch.float32, device="cuda")
        self.n_layers, self.max_seq_len = n_layers, max_seq_len
        self.n_kv_heads, self.head_dim = n_kv_heads, head_dim

    def WriteDevice(self, layer: int, pos: int, k, v):
        check(lib().dqmk_kv_write(_ptr(self.keys), _ptr(self.values), self.n_layers,
                                  self.max_seq_len, self.n_kv_heads, self.head_dim, layer, pos,
                                  _ptr(k), _ptr(v), _stream()))


def CudaAttentionDecodeDeviceInput(q, kv: CudaKvCache, layer: int, pos: int, n_heads: int,
                                   n_kv_heads: int, head_dim: int):
    torch = _torch()
    out = torch.empty(n_heads * head_dim, dtype=torch.float32, device=q.device)
    if n_kv_heads != kv.n_kv_heads or head_dim != kv.head_dim:
        raise RuntimeError("CudaAttentionDecode: cache shape mismatch")
    check(lib().dqmk_attention_decode(_ptr(q), _ptr(kv.keys), _ptr(kv.values), kv.n_layers,
                                      kv.max_seq_len, n_kv_heads, head_dim, layer, pos, n_heads,
                                      _ptr(out), _stream()))
    return out


# ------------------------------------------------------------ engine
def nccl_unique_id() -> bytes:
    """A fresh NCCL unique id (128 bytes) for Model.set_tp."""
    buf = C.create_string_buffer(128)
    check(lib().dqmk_nccl_unique_id(buf))
    return buf.raw


def tp_plan(cfg: dict, rank: int, world: int, max_seq_len: int = 1) -> dict:
    """This rank's tensor-parallel shard of a model shape (host only)."""
    c = ModelConfig()
    c.vocab_size, c.dim, c.hidden_dim = cfg["vocab"], cfg["dim"], cfg["hidden"]
    c.n_layers, c.n_heads, c.n_kv_heads = cfg["n_layers"], cfg["n_heads"], cfg["n_kv_heads"]
    c.head_dim = cfg["dim"] // cfg["n_heads"]
    c.max_seq_len = max_seq_len
    c.rope_theta, c.rms_norm_eps, c.rope_neox = cfg["rope_theta"], cfg["eps"], 1
    p = TpPlan()
    check(lib().dqmk_tp_plan_get(C.byref(c), rank, world, C.byref(p)))
    return {n: getattr(p, n) for n, _ in TpPlan._fields_}


class Model:
    """A device-resident model: UploadModelWeightsToCuda + the fused layouts.

    ``tensors`` maps the reference's weight names to (qtype, array, rows,
    cols); arrays may be numpy (host) or torch CUDA tensors.
    """

    def __init__(self, cfg: dict, max_seq_len: int, device: int = 0):
        self.cfg = dict(cfg)
        c = ModelConfig()
        c.vocab_size, c.dim, c.hidden_dim = cfg["vocab"], cfg["dim"], cfg["hidden"]
        c.n_layers, c.n_heads, c.n_kv_heads = cfg["n_layers"], cfg["n_heads"], cfg["n_kv_heads"]
        c.head_dim = cfg["dim"] // cfg["n_heads"]
        c.max_seq_len = max_seq_len
        c.rope_theta, c.rms_norm_eps = cfg["rope_theta"], cfg["eps"]
        c.rope_neox = 1
        self.max_seq_len = max_seq_len
        self._c = c
        h = C.c_void_p()
        check(lib().dqmk_model_create(C.byref(c), device, C.byref(h)))
        self.h = h

    def set_tp(self, rank: int, world: int, nccl_id: Optional[bytes]) -> None:
        """Tensor parallelism before finalize (collective: all ranks call it)."""
        check(lib().dqmk_model_set_tp(self.h, rank, world, nccl_id))

    def upload(self, name: str, qtype: int, data, rows: int, cols: int) -> None:
        if hasattr(data, "data_ptr"):
            ptr, nbytes = data.data_ptr(), data.numel() * data.element_size()
            keep = data
        else:
            keep = np.ascontiguousarray(data)
            ptr, nbytes = keep.ctypes.data, keep.nbytes
        check(lib().dqmk_model_upload(self.h, name.encode(), qtype, ptr, nbytes, rows, cols))
        del keep

    def finalize(self) -> None:
        check(lib().dqmk_model_finalize(self.h))

    @staticmethod
    def gguf_config(path: str) -> dict:
        """The model configuration a GGUF file's metadata gives (BuildConfig,
        src/gguf_loader.cc:202-273), without touching a device."""
        c = ModelConfig()
        check(lib().dqmk_gguf_read_config(path.encode(), C.byref(c)))
        return {"vocab": c.vocab_size, "dim": c.dim, "hidden": c.hidden_dim,
                "n_layers": c.n_layers, "n_heads": c.n_heads, "n_kv_heads": c.n_kv_heads,
                "head_dim": c.head_dim, "max_seq_len": c.max_seq_len,
                "rope_theta": c.rope_theta, "eps": c.rms_norm_eps, "rope_neox": c.rope_neox}

    @classmethod
    def from_gguf(cls, path: str, max_seq_len: int = 0, device: int = 0) -> "Model":
        """LoadGgufModel + UploadModelWeightsToCuda: a finalized model from a
        GGUF v3 file (quantized tensors kept as stored)."""
        cfg = cls.gguf_config(path)
        m = cls.__new__(cls)
        m.cfg = {k: cfg[k] for k in ("vocab", "dim", "hidden", "n_layers", "n_heads",
                                     "n_kv_heads", "rope_theta", "eps")}
        m.max_seq_len = max_seq_len or cfg["max_seq_len"]
        h = C.c_void_p()
        check(lib().dqmk_model_load_gguf(path.encode(), int(max_seq_len), device, C.byref(h)))
        m.h = h
        return m

    @classmethod
    def from_synth(cls, w: "synth.SynthModel", max_seq_len: int, device: int = 0,
                   tp: Optional[tuple] = None) -> "Model":
        """tp = (rank, world, nccl_id): keep this rank's tensor-parallel shard."""
        c = w.cfg
        m = cls(c, max_seq_len, device)
        if tp is not None:
            m.set_tp(*tp)
        qt, hd = w.qtype, c["dim"] // c["n_heads"]
        qd, kvd = c["n_heads"] * hd, c["n_kv_heads"] * hd
        m.upload("token_embedding", qt, w.token_embd, c["vocab"], c["dim"])
        m.upload("final_norm", F32, w.final_norm, 1, c["dim"])
        if w.lm_head is not None:
            m.upload("lm_head", qt, w.lm_head, c["vocab"], c["dim"])
        shapes = {"wq": (qd, c["dim"]), "wk": (kvd, c["dim"]), "wv": (kvd, c["dim"]),
                  "wo": (c["dim"], qd), "w_gate": (c["hidden"], c["dim"]),
                  "w_up": (c["hidden"], c["dim"]), "w_down": (c["dim"], c["hidden"])}
        for i, L in enumerate(w.layers):
            p = f"layers.{i}."
            m.upload(p + "attention_norm", F32, L.attention_norm, 1, c["dim"])
            m.upload(p + "ffn_norm", F32, L.ffn_norm, 1, c["dim"])
            for n, (r, cc) in shapes.items():
                m.upload(p + n, qt, getattr(L, n), r, cc)
            for n, size in (("bq", qd), ("bk", kvd), ("bv", kvd)):
                b = getattr(L, n)
                if b is not None:
                    m.upload(p + n, F32, b, 1, size)
        m.finalize()
        return m

    def stats(self) -> dict:
        s = ModelStats()
        check(lib().dqmk_model_stats_get(self.h, C.byref(s)))
        return {n: getattr(s, n) for n, _ in ModelStats._fields_}

    def reset_stats(self) -> None:
        check(lib().dqmk_model_stats_reset(self.h))

    def memory_bytes(self) -> int:
        return lib().dqmk_model_memory_bytes(self.h)

    def close(self) -> None:
        if getattr(self, "h", None):
            lib().dqmk_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Context:
    """MiniLlamaContext + ForwardToken / ForwardBatch (forward.h:11-17)."""

    def __init__(self, model: Model):
        self.model = model
        h = C.c_void_p()
        check(lib().dqmk_context_create(model.h, C.byref(h)))
        self.h = h
        self.vocab = model.cfg["vocab"]

    def reset(self) -> None:
        check(lib().dqmk_context_reset(self.h))

    @property
    def pos(self) -> int:
        return lib().dqmk_context_pos(self.h)

    @property
    def token_history(self):
        n = lib().dqmk_context_history(self.h, None, 0)
        buf = (C.c_int * max(n, 1))()
        lib().dqmk_context_history(self.h, buf, n)
        return list(buf)[:n]

    def ForwardToken(self, token: int, pos: int, logits: Optional[np.ndarray] = None):
        out = logits if logits is not None else np.empty(self.vocab, np.float32)
        check(lib().dqmk_forward_token(self.h, int(token), int(pos),
                                       out.ctypes.data_as(C.POINTER(C.c_float))))
        return out

    def ForwardBatch(self, tokens: Sequence[int], start_pos: int = 0,
                     positions: Optional[Sequence[int]] = None,
                     logits: Optional[np.ndarray] = None):
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        if positions is None:
            positions = np.arange(start_pos, start_pos + toks.size, dtype=np.int32)
        pos = np.ascontiguousarray(np.asarray(positions, dtype=np.int32))
        if pos.size != toks.size:
            raise RuntimeError("ForwardBatch: tokens and positions size mismatch")
        out = logits if logits is not None else np.empty(self.vocab, np.float32)
        ip = C.POINTER(C.c_int)
        check(lib().dqmk_forward_batch(self.h, toks.ctypes.data_as(ip), pos.ctypes.data_as(ip),
                                       toks.size, out.ctypes.data_as(C.POINTER(C.c_float))))
        return out

    def ForwardBatchReuse(self, tokens: Sequence[int]):
        """A new prompt on this context, reusing the longest common prefix
        of its token history (dqmk_forward_batch_prefix); returns (logits,
        number of prompt tokens whose KV entries were kept)."""
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        out = np.empty(self.vocab, np.float32)
        reused = C.c_int(0)
        check(lib().dqmk_forward_batch_prefix(self.h, toks.ctypes.data_as(C.POINTER(C.c_int)),
                                              toks.size, out.ctypes.data_as(C.POINTER(C.c_float)),
                                              C.byref(reused)))
        return out, reused.value

    def decode_greedy(self, token: int, pos: int, n_steps: int) -> np.ndarray:
        out = np.zeros(n_steps, np.int32)
        check(lib().dqmk_decode_greedy(self.h, int(token), int(pos), int(n_steps),
                                       out.ctypes.data_as(C.POINTER(C.c_int))))
        return out

    def decode_enqueue(self, token: int, pos: int, n_steps: int) -> None:
        check(lib().dqmk_decode_enqueue(self.h, int(token), int(pos), int(n_steps)))

    def tp_ipc_handle(self) -> bytes:
        """This rank's exchange buffer as a 64-byte CUDA IPC handle."""
        buf = C.create_string_buffer(64)
        check(lib().dqmk_context_tp_ipc_handle(self.h, buf))
        return buf.raw

    def tp_connect(self, handles) -> None:
        """Map every rank's exchange buffer (handles in rank order): the decode
        step then exchanges partial sums over peer memory instead of NCCL."""
        check(lib().dqmk_context_tp_connect(self.h, b"".join(handles)))

    @property
    def stream_handle(self) -> int:
        return lib().dqmk_context_stream(self.h)

    def close(self) -> None:
        if getattr(self, "h", None):
            lib().dqmk_context_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Batch:
    """Many sequences decoded together over one model (dqmk_batch): n_slots
    independent KV caches; each step runs up to 64 (slot, position, token)
    columns, streaming every weight once per step."""

    MAX_COLS = 64

    def __init__(self, model: Model, n_slots: int, max_seq: Optional[int] = None):
        self.model = model
        self.n_slots = int(n_slots)
        self.max_seq = int(max_seq if max_seq is not None else model.max_seq_len)
        h = C.c_void_p()
        check(lib().dqmk_batch_create(model.h, self.n_slots, self.max_seq, C.byref(h)))
        self.h = h
        self.vocab = model.cfg["vocab"]

    @staticmethod
    def _i32(a):
        return np.ascontiguousarray(np.asarray(a, dtype=np.int32))

    def reset(self) -> None:
        check(lib().dqmk_batch_reset(self.h))

    def step(self, slots: Optional[Sequence[int]], tokens: Sequence[int],
             positions: Sequence[int], want_logits: bool = True):
        """One step over columns (slot, token, position); returns (logits
        [n, vocab] or None, next greedy tokens [n])."""
        toks, pos = self._i32(tokens), self._i32(positions)
        n = toks.size
        if pos.size != n:
            raise RuntimeError("DecodeBatch: tokens and positions size mismatch")
        ip = C.POINTER(C.c_int)
        sl = None if slots is None else self._i32(slots)
        logits = np.empty((n, self.vocab), np.float32) if want_logits else None
        nxt = np.zeros(n, np.int32)
        check(lib().dqmk_batch_step(
            self.h, None if sl is None else sl.ctypes.data_as(ip), toks.ctypes.data_as(ip),
            pos.ctypes.data_as(ip), n,
            None if logits is None else logits.ctypes.data_as(C.POINTER(C.c_float)),
            nxt.ctypes.data_as(ip)))
        return logits, nxt

    def prefill(self, slot: int, tokens: Sequence[int], pos0: int = 0) -> None:
        """The prompt of one slot, up to 64 positions per step."""
        toks = self._i32(tokens)
        for i0 in range(0, toks.size, self.MAX_COLS):
            chunk = toks[i0:i0 + self.MAX_COLS]
            self.step([slot] * chunk.size, chunk, np.arange(pos0 + i0, pos0 + i0 + chunk.size),
                      want_logits=False)

    def decode_greedy(self, tokens: Sequence[int], positions: Sequence[int],
                      n_steps: int) -> np.ndarray:
        """Slots 0..n-1 decode together; returns [n_steps, n] tokens."""
        toks, pos = self._i32(tokens), self._i32(positions)
        out = np.zeros((n_steps, toks.size), np.int32)
        ip = C.POINTER(C.c_int)
        check(lib().dqmk_batch_decode_greedy(self.h, toks.ctypes.data_as(ip),
                                             pos.ctypes.data_as(ip), toks.size, int(n_steps),
                                             out.ctypes.data_as(ip)))
        return out

    def decode_enqueue(self, tokens: Sequence[int], positions: Sequence[int],
                       n_steps: int) -> None:
        toks, pos = self._i32(tokens), self._i32(positions)
        ip = C.POINTER(C.c_int)
        check(lib().dqmk_batch_decode_enqueue(self.h, toks.ctypes.data_as(ip),
                                              pos.ctypes.data_as(ip), toks.size, int(n_steps)))

    def history(self, slot: int, pos0: int, count: int) -> np.ndarray:
        out = np.zeros(count, np.int32)
        check(lib().dqmk_batch_history(self.h, int(slot), int(pos0), int(count),
                                       out.ctypes.data_as(C.POINTER(C.c_int))))
        return out

    @property
    def stream_handle(self) -> int:
        return lib().dqmk_batch_stream(self.h)

    def close(self) -> None:
        if getattr(self, "h", None):
            lib().dqmk_batch_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
