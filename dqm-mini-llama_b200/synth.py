"""Seeded synthetic inputs: random-init Qwen2-architecture weights and GEMV cases.

No checkpoints or datasets exist on this machine, so every workload runs on
weights drawn here from a fixed seed.  Each tensor gets its own numpy PCG64
stream keyed by (seed, tensor index), so a tensor can be regenerated alone and
the same seed gives the same bits on every machine with the same numpy.

Weights follow the shapes of the dqm-mini-llama engine
(include/dqm_llama/model.h:38-51): linears are [out_features, in_features],
stored as ggml blocks (34-byte Q8_0 / 18-byte Q4_0, row-major, 32 values per
block along in_features).  Linear weights and the token embedding are drawn
N(0, 0.02); norm weights are 1 + N(0, 0.02); QKV biases N(0, 0.02).

Q8_0 quantization is delegated to a caller-supplied function (the device
quantizer in the product, the oracle on CPU) because it must match the
reference's QuantizeToQ80 bit for bit.  Q4_0 model weights use the ggml
convention (scale = signed absmax / -8, q = trunc(x/d + 8.5) clipped to 15),
which is what GGUF files carry; the forward pass reads any valid Q4_0 block.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import Callable, List, Optional

import numpy as np

F32, Q80, Q40, Q41 = 0, 1, 2, 3
BLOCK_BYTES = {Q80: 34, Q40: 18, Q41: 20}

QWEN2_0_5B = dict(name="qwen2-0.5b", vocab=151936, dim=896, hidden=4864, n_layers=24,
                  n_heads=14, n_kv_heads=2, rope_theta=1e6, eps=1e-6, bias=True, tied=True)
QWEN2_7B = dict(name="qwen2-7b", vocab=152064, dim=3584, hidden=18944, n_layers=28,
                n_heads=28, n_kv_heads=4, rope_theta=1e6, eps=1e-6, bias=True, tied=False)
# Small Qwen2-style shape for fast parity cases (same GQA ratio, head_dim 64).
QWEN2_MINI = dict(name="qwen2-mini", vocab=1024, dim=256, hidden=704, n_layers=2,
                  n_heads=4, n_kv_heads=2, rope_theta=1e6, eps=1e-6, bias=True, tied=True)

_FIELDS = ("attention_norm", "wq", "wk", "wv", "bq", "bk", "bv", "wo", "ffn_norm",
           "w_gate", "w_up", "w_down")


def rng_for(seed: int, index: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, index])))


def normal(seed: int, index: int, shape, std: float = 0.02) -> np.ndarray:
    x = rng_for(seed, index).standard_normal(shape, dtype=np.float32)
    return x * np.float32(std)


def quantize_q40_ggml(src: np.ndarray) -> np.ndarray:
    """ggml's Q4_0 rule, vectorised: d = m / -8 where m is the signed value of
    largest magnitude; id = 1/d; q = min(15, trunc(x*id + 8.5)); the stored
    scale is d rounded to fp16 (round-to-nearest-even).  Rows must be a
    multiple of 32 long."""
    src = np.ascontiguousarray(src, dtype=np.float32)
    rows, cols = src.reshape(-1, src.shape[-1]).shape
    assert cols % 32 == 0, "ggml Q4_0 synthesis expects in_features % 32 == 0"
    blk = src.reshape(-1, 32)
    idx = np.abs(blk).argmax(axis=1)
    m = blk[np.arange(blk.shape[0]), idx]
    d = m / np.float32(-8.0)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    q = np.trunc(blk * inv[:, None] + np.float32(8.5)).astype(np.int32)
    q = np.minimum(q, 15).astype(np.uint8)
    packed = (q[:, :16] | (q[:, 16:] << 4)).astype(np.uint8)
    out = np.empty((blk.shape[0], 18), dtype=np.uint8)
    out[:, :2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = packed
    return out.reshape(-1)


@dataclass
class SynthLayer:
    attention_norm: np.ndarray
    wq: np.ndarray
    wk: np.ndarray
    wv: np.ndarray
    bq: Optional[np.ndarray]
    bk: Optional[np.ndarray]
    bv: Optional[np.ndarray]
    wo: np.ndarray
    ffn_norm: np.ndarray
    w_gate: np.ndarray
    w_up: np.ndarray
    w_down: np.ndarray


@dataclass
class SynthModel:
    cfg: dict
    qtype: int
    token_embd: np.ndarray          # blocks [vocab, dim]
    final_norm: np.ndarray          # f32 [dim]
    lm_head: Optional[np.ndarray]   # blocks [vocab, dim]; None when tied
    layers: List[SynthLayer] = field(default_factory=list)

    @property
    def head_dim(self) -> int:
        return self.cfg["dim"] // self.cfg["n_heads"]


def make_model(cfg: dict, qtype: int, seed: int,
               quantize_q80: Optional[Callable[[np.ndarray], np.ndarray]] = None,
               n_layers: Optional[int] = None) -> SynthModel:
    """Draw a whole model.  ``quantize_q80`` maps a 2-D float32 array to its
    Q8_0 blocks (uint8); it is required when qtype is Q8_0."""
    cfg = dict(cfg)
    if n_layers is not None:
        cfg["n_layers"] = n_layers
    if qtype == Q80:
        if quantize_q80 is None:
            raise ValueError("make_model: a Q8_0 quantizer is required")
        quant = quantize_q80
    else:
        quant = quantize_q40_ggml
    dim, hid = cfg["dim"], cfg["hidden"]
    hd = dim // cfg["n_heads"]
    qd, kvd = cfg["n_heads"] * hd, cfg["n_kv_heads"] * hd
    token_embd = quant(normal(seed, 0, (cfg["vocab"], dim)))
    final_norm = np.float32(1.0) + normal(seed, 1, (dim,))
    lm_head = None if cfg["tied"] else quant(normal(seed, 2, (cfg["vocab"], dim)))
    layers = []
    for li in range(cfg["n_layers"]):
        base = 16 + 16 * li
        shapes = {"wq": (qd, dim), "wk": (kvd, dim), "wv": (kvd, dim), "wo": (dim, qd),
                  "w_gate": (hid, dim), "w_up": (hid, dim), "w_down": (dim, hid)}
        vals = {}
        for fi, name in enumerate(_FIELDS):
            idx = base + fi
            if name in shapes:
                vals[name] = quant(normal(seed, idx, shapes[name]))
            elif name in ("attention_norm", "ffn_norm"):
                vals[name] = np.float32(1.0) + normal(seed, idx, (dim,))
            else:  # biases
                n = qd if name == "bq" else kvd
                vals[name] = normal(seed, idx, (n,)) if cfg["bias"] else None
        layers.append(SynthLayer(**vals))
    return SynthModel(cfg=cfg, qtype=qtype, token_embd=token_embd, final_norm=final_norm,
                      lm_head=lm_head, layers=layers)


def prompt_tokens(vocab: int, n: int, seed: int) -> np.ndarray:
    """n token ids drawn uniformly from [0, vocab)."""
    return rng_for(seed, 999).integers(0, vocab, size=n, dtype=np.int64).astype(np.int32)


def gemv_case(out_features: int, in_features: int, seed: int, qtype: int = Q80):
    """Standalone GEMV inputs: int8 values uniform in [-127, 127] (Q4_0 / Q4_1:
    nibbles uniform in [0, 15]; Q4_1 minima uniform in [-0.08, 0]), fp16 scales
    uniform in [1e-4, 1e-2], x ~ N(0, 1).
    Returns (blocks uint8, x float32)."""
    g = rng_for(seed, 7000 + qtype)
    nb = (in_features + 31) // 32
    n = out_features * nb
    d = g.uniform(1e-4, 1e-2, size=n).astype(np.float16).view(np.uint8).reshape(n, 2)
    if qtype == Q80:
        qs = g.integers(-127, 128, size=(n, 32), dtype=np.int16).astype(np.int8).view(np.uint8)
        blocks = np.concatenate([d, qs], axis=1)
    elif qtype == Q41:
        m = g.uniform(-0.08, 0.0, size=n).astype(np.float16).view(np.uint8).reshape(n, 2)
        qs = g.integers(0, 256, size=(n, 16), dtype=np.int16).astype(np.uint8)
        blocks = np.concatenate([d, m, qs], axis=1)
    else:
        qs = g.integers(0, 256, size=(n, 16), dtype=np.int16).astype(np.uint8)
        blocks = np.concatenate([d, qs], axis=1)
    x = g.standard_normal(in_features, dtype=np.float32)
    return np.ascontiguousarray(blocks.reshape(-1)), x


# ---------------------------------------------------------------- GGUF files
# GGUF version 3 (the llama.cpp model container, the input format of every
# workload here): header "GGUF", u32 version, u64 tensor count, u64 metadata
# count; metadata as (string key, u32 type, value); tensor infos as (string
# name, u32 n_dims, u64 dims innermost first, u32 ggml type, u64 offset into
# the data section); the data section starts at the next multiple of
# general.alignment (32 here).  Strings are u64 length + bytes, little endian.
GGUF_U32, GGUF_F32, GGUF_STRING, GGUF_ARRAY = 4, 6, 8, 9
GGML_TYPE = {F32: 0, Q40: 2, Q41: 3, Q80: 8}


def _gguf_str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def gguf_tensors(w: SynthModel):
    """(GGUF name, ggml qtype, data bytes, [rows, cols] or [n]) of a model, in
    the llama.cpp naming the reference's loader maps (src/gguf_loader.cc:21-59)."""
    c = w.cfg
    hd = c["dim"] // c["n_heads"]
    qd, kvd = c["n_heads"] * hd, c["n_kv_heads"] * hd
    out = [("token_embd.weight", w.qtype, w.token_embd, [c["vocab"], c["dim"]]),
           ("output_norm.weight", F32, w.final_norm, [c["dim"]])]
    if w.lm_head is not None:
        out.append(("output.weight", w.qtype, w.lm_head, [c["vocab"], c["dim"]]))
    for i, L in enumerate(w.layers):
        p = f"blk.{i}."
        out += [(p + "attn_norm.weight", F32, L.attention_norm, [c["dim"]]),
                (p + "attn_q.weight", w.qtype, L.wq, [qd, c["dim"]]),
                (p + "attn_k.weight", w.qtype, L.wk, [kvd, c["dim"]]),
                (p + "attn_v.weight", w.qtype, L.wv, [kvd, c["dim"]])]
        for nm, b, n in (("attn_q.bias", L.bq, qd), ("attn_k.bias", L.bk, kvd),
                         ("attn_v.bias", L.bv, kvd)):
            if b is not None:
                out.append((p + nm, F32, b, [n]))
        out += [(p + "attn_output.weight", w.qtype, L.wo, [c["dim"], qd]),
                (p + "ffn_norm.weight", F32, L.ffn_norm, [c["dim"]]),
                (p + "ffn_gate.weight", w.qtype, L.w_gate, [c["hidden"], c["dim"]]),
                (p + "ffn_up.weight", w.qtype, L.w_up, [c["hidden"], c["dim"]]),
                (p + "ffn_down.weight", w.qtype, L.w_down, [c["dim"], c["hidden"]])]
    return out


def write_gguf(path: str, w: SynthModel, context_length: int, alignment: int = 32) -> None:
    """Write a model as a GGUF v3 file with qwen2 metadata: block count,
    widths, head counts, context length, RoPE base, RMSNorm epsilon and a
    tokenizer.ggml.tokens array whose length is the vocabulary."""
    c = w.cfg
    kv = [("general.architecture", GGUF_STRING, "qwen2"),
          ("general.alignment", GGUF_U32, alignment),
          ("qwen2.block_count", GGUF_U32, c["n_layers"]),
          ("qwen2.context_length", GGUF_U32, context_length),
          ("qwen2.embedding_length", GGUF_U32, c["dim"]),
          ("qwen2.feed_forward_length", GGUF_U32, c["hidden"]),
          ("qwen2.attention.head_count", GGUF_U32, c["n_heads"]),
          ("qwen2.attention.head_count_kv", GGUF_U32, c["n_kv_heads"]),
          ("qwen2.rope.freq_base", GGUF_F32, c["rope_theta"]),
          ("qwen2.attention.layer_norm_rms_epsilon", GGUF_F32, c["eps"])]
    tensors = gguf_tensors(w)
    head = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kv) + 1))
    for key, t, v in kv:
        head += _gguf_str(key) + struct.pack("<I", t)
        if t == GGUF_STRING:
            head += _gguf_str(v)
        elif t == GGUF_U32:
            head += struct.pack("<I", int(v))
        else:
            head += struct.pack("<f", float(v))
    head += _gguf_str("tokenizer.ggml.tokens") + struct.pack("<IIQ", GGUF_ARRAY, GGUF_STRING,
                                                            c["vocab"])
    head += b"".join(_gguf_str(f"tok_{i}") for i in range(c["vocab"]))
    offset, blobs = 0, []
    for name, qt, data, shape in tensors:
        raw = np.ascontiguousarray(data).view(np.uint8).tobytes()
        dims = list(reversed(shape))  # innermost first: [in, out]
        head += _gguf_str(name) + struct.pack("<I", len(dims))
        head += b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", GGML_TYPE[qt], offset)
        pad = (-len(raw)) % alignment
        blobs.append(raw + b"\0" * pad)
        offset += len(raw) + pad
    head += b"\0" * ((-len(head)) % alignment)
    with open(path, "wb") as f:
        f.write(head)
        for b in blobs:
            f.write(b)
