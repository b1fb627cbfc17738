"""ctypes view of the checker libraries built by oracle/Makefile.

TEST INFRASTRUCTURE.  Only tests/, ``__graft_entry__.smoke()`` and the CPU
legs of ``bench.py`` import this module.  Two libraries sit behind it:

* ``liboracle.so`` -- the C restatement (dqm_oracle.c) of the reference's
  quantized-matmul path, each function citing the reference file:line.
* ``_ref/libdqmref.so`` -- the reference's own CPU sources compiled as its
  CMake Release build does, plus ref_shim.cc.  Present where it was built
  (it travels with the source tree); ``ref_available()`` says whether it is.

Arrays are numpy; quantized blocks are raw uint8 arrays in the ggml layouts
(34-byte Q8_0 blocks, 18-byte Q4_0 blocks).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
Q80_BYTES = 34
Q40_BYTES = 18
Q41_BYTES = 20
F32, Q80, Q40, Q41 = 0, 1, 2, 3

_fp = C.POINTER(C.c_float)
_vp = C.c_void_p
_ip = C.POINTER(C.c_int)

_lib = None
_ref = None


def build() -> None:
    """Compile liboracle.so (and _ref when the reference sources exist)."""
    subprocess.run(["make", "-s", "-C", HERE, "-j8"], check=True)


def _f(a: np.ndarray):
    return a.ctypes.data_as(_fp)


def _v(a: np.ndarray):
    return a.ctypes.data_as(_vp)


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        L.orc_fp16_to_fp32.argtypes = [C.c_uint16]
        L.orc_fp16_to_fp32.restype = C.c_float
        L.orc_fp32_to_fp16.argtypes = [C.c_float]
        L.orc_fp32_to_fp16.restype = C.c_uint16
        for n in ("orc_quantize_q80", "orc_quantize_q40"):
            getattr(L, n).argtypes = [_fp, C.c_int64, C.c_int64, _vp]
        for n in ("orc_dequantize_q80", "orc_dequantize_q40", "orc_dequantize_q41"):
            getattr(L, n).argtypes = [_vp, C.c_int64, C.c_int64, _fp]
        for n in ("orc_linear_q80", "orc_linear_q40", "orc_linear_q41"):
            getattr(L, n).argtypes = [_fp, C.c_int, C.c_int, _vp, C.c_int, _fp]
        L.orc_linear_f32_simd.argtypes = [_fp, C.c_int, _fp, C.c_int, _fp]
        L.orc_rmsnorm.argtypes = [_fp, _fp, C.c_int, C.c_float, _fp]
        L.orc_rope.argtypes = [_fp, C.c_int, _fp, C.c_int, C.c_int, C.c_int, C.c_float, C.c_int]
        L.orc_softmax.argtypes = [_fp, C.c_int, _fp]
        L.orc_swiglu.argtypes = [_fp, _fp, C.c_int, _fp]
        L.orc_argmax.argtypes = [_fp, C.c_int]
        L.orc_argmax.restype = C.c_int
        L.orc_kv_write.argtypes = [_fp, _fp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _fp, _fp]
        L.orc_attention.argtypes = [_fp, _fp, _fp, C.c_int, C.c_int, C.c_int, C.c_int,
                                    C.c_int, C.c_int, _fp, _fp]
        L.orc_forward_scratch_floats.argtypes = [_vp]
        L.orc_forward_scratch_floats.restype = C.c_int64
        L.orc_forward_token.argtypes = [_vp, _fp, _fp, C.c_int, C.c_int, _fp, _fp]
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(os.path.join(HERE, "_ref", "libdqmref.so"))


def ref():
    global _ref
    if _ref is None:
        path = os.path.join(HERE, "_ref", "libdqmref.so")
        if not os.path.exists(path):
            raise RuntimeError("reference library not built: " + path)
        R = C.CDLL(path)
        R.ref_last_error.restype = C.c_char_p
        R.ref_set_threads.argtypes = [C.c_int]
        R.ref_get_threads.restype = C.c_int
        for n in ("ref_quantize_q80", "ref_quantize_q40"):
            getattr(R, n).argtypes = [_fp, C.c_int, C.c_int, _vp]
        for n in ("ref_dequantize_q80", "ref_dequantize_q40", "ref_dequantize_q41"):
            getattr(R, n).argtypes = [_vp, C.c_int, C.c_int, _fp]
        R.ref_linear.argtypes = [C.c_int, _fp, C.c_int, C.c_int, _vp, C.c_int, _fp]
        R.ref_rmsnorm.argtypes = [_fp, _fp, C.c_int, C.c_float, _fp]
        R.ref_rope.argtypes = [_fp, C.c_int, _fp, C.c_int, C.c_int, C.c_int, C.c_float, C.c_int]
        R.ref_softmax.argtypes = [_fp, C.c_int, _fp]
        R.ref_swiglu.argtypes = [_fp, _fp, C.c_int, _fp]
        R.ref_argmax.argtypes = [_fp, C.c_int]
        R.ref_model_create.argtypes = [C.c_int] * 7 + [C.c_float, C.c_float, C.c_int]
        R.ref_model_create.restype = _vp
        R.ref_model_destroy.argtypes = [_vp]
        R.ref_model_set_embedding.argtypes = [_vp, C.c_int, _vp, C.c_int]
        R.ref_model_set_lm_head.argtypes = [_vp, C.c_int, _vp]
        R.ref_model_set_final_norm.argtypes = [_vp, _fp]
        R.ref_model_set_layer.argtypes = [_vp, C.c_int, C.c_int, _fp, _vp, _vp, _vp,
                                          _fp, _fp, _fp, _vp, _fp, _vp, _vp, _vp]
        R.ref_model_finish.argtypes = [_vp]
        R.ref_context_reset.argtypes = [_vp]
        R.ref_forward_batch.argtypes = [_vp, _ip, C.c_int, C.c_int, _fp]
        R.ref_context_pos.argtypes = [_vp]
        R.ref_context_history.argtypes = [_vp, _ip, C.c_int]
        _ref = R
    return _ref


def ref_set_threads(n: int) -> None:
    """SetThreadCount of the reference's CPU thread pool (src/thread_pool.cc:186)."""
    ref().ref_set_threads(int(n))


def _check_ref(rc: int) -> None:
    if rc != 0:
        raise RuntimeError(ref().ref_last_error().decode())


# ---------------------------------------------------------------- helpers
def _nblocks(rows: int, cols: int) -> int:
    return rows * ((cols + 31) // 32)


def _rows_cols(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.ndim == 1:
        return x, 1, x.shape[0]
    return x, int(np.prod(x.shape[:-1])), x.shape[-1]


def fp16_to_fp32(h: int) -> float:
    return lib().orc_fp16_to_fp32(h)


def fp32_to_fp16(v: float) -> int:
    return lib().orc_fp32_to_fp16(v)


def quantize_q80(src: np.ndarray, use_ref: bool = False) -> np.ndarray:
    src, rows, cols = _rows_cols(src)
    out = np.zeros(_nblocks(rows, cols) * Q80_BYTES, dtype=np.uint8)
    if src.size:
        if use_ref:
            _check_ref(ref().ref_quantize_q80(_f(src), rows, cols, _v(out)))
        else:
            lib().orc_quantize_q80(_f(src), rows, cols, _v(out))
    return out


def quantize_q40(src: np.ndarray, use_ref: bool = False) -> np.ndarray:
    src, rows, cols = _rows_cols(src)
    out = np.zeros(_nblocks(rows, cols) * Q40_BYTES, dtype=np.uint8)
    if src.size:
        if use_ref:
            _check_ref(ref().ref_quantize_q40(_f(src), rows, cols, _v(out)))
        else:
            lib().orc_quantize_q40(_f(src), rows, cols, _v(out))
    return out


def dequantize(qtype: int, blocks: np.ndarray, rows: int, cols: int,
               use_ref: bool = False) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    out = np.zeros((rows, cols), dtype=np.float32)
    names = {Q80: "q80", Q40: "q40", Q41: "q41"}
    if use_ref:
        fn = getattr(ref(), "ref_dequantize_" + names[qtype])
        _check_ref(fn(_v(blocks), rows, cols, _f(out)))
    else:
        fn = getattr(lib(), "orc_dequantize_" + names[qtype])
        fn(_v(blocks), rows, cols, _f(out))
    return out


def linear(qtype: int, x: np.ndarray, w: np.ndarray, out_features: int,
           use_ref: bool = False) -> np.ndarray:
    """y = x W^T for W [out_features, in] as blocks (or F32 for qtype F32)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows = 1 if x.ndim == 1 else x.shape[0]
    inf = x.shape[-1]
    y = np.zeros((rows, out_features), dtype=np.float32)
    w = np.ascontiguousarray(w)
    if use_ref:
        _check_ref(ref().ref_linear(qtype, _f(x), rows, inf, _v(w), out_features, _f(y)))
    elif qtype == Q80:
        lib().orc_linear_q80(_f(x), rows, inf, _v(w), out_features, _f(y))
    elif qtype == Q40:
        lib().orc_linear_q40(_f(x), rows, inf, _v(w), out_features, _f(y))
    elif qtype == Q41:
        lib().orc_linear_q41(_f(x), rows, inf, _v(w), out_features, _f(y))
    else:
        assert rows == 1
        lib().orc_linear_f32_simd(_f(x), inf, w.ctypes.data_as(_fp), out_features, _f(y))
    return y[0] if x.ndim == 1 else y


# ---- integer restatement of the decode GEMV's int8 path (numpy) ----------
# The reference's Linear has no integer dot product; the TMA-staged decode
# GEMV (the lm_head form) quantizes x per 32-value block into three int8 terms
# and sums int8 x int8 products exactly in int32.  These functions restate
# that arithmetic on the host so its terms, scales and block sums can be
# compared bit for bit.

def x_terms(x: np.ndarray):
    """x [k] -> (q [3, nb, 32] int8, s [3, nb] float32), x ~= sum_t s_t q_t per
    block.  s_1 = absmax / 127 (0 for a zero block); term t: inv = 1 / s_t,
    q_t = clamp(round-half-even(r * inv), -127, 127), r <- fl(r - s_t q_t)
    (one rounding: s_t q_t is exact in float64, so the float64 difference is
    exact and rounds once to float32), s_{t+1} = s_t * fl(1 / 254)."""
    x = np.asarray(x, dtype=np.float32)
    nb = (x.size + 31) // 32
    r = np.zeros((nb, 32), np.float32)
    r.reshape(-1)[: x.size] = x
    m = np.abs(r).max(axis=1)
    s = np.where(m > 0, m / np.float32(127.0), np.float32(0.0)).astype(np.float32)
    step = np.float32(1.0) / np.float32(254.0)
    q = np.zeros((3, nb, 32), np.int8)
    sc = np.zeros((3, nb), np.float32)
    for t in range(3):
        with np.errstate(divide="ignore"):
            inv = np.where(s > 0, np.float32(1.0) / s, np.float32(0.0)).astype(np.float32)
        qq = np.clip(np.rint((r * inv[:, None]).astype(np.float32)), -127, 127)
        r = (r.astype(np.float64) - s.astype(np.float64)[:, None] * qq).astype(np.float32)
        q[t] = qq.astype(np.int8)
        sc[t] = s
        s = (s * step).astype(np.float32)
    return q, sc


def block_term_sums(qtype: int, blocks: np.ndarray, rows: int, cols: int,
                    q: np.ndarray) -> np.ndarray:
    """Exact sums[row, t, b] = sum_j w[row, 32 b + j] q[t, b, j] with the
    block's integer weights (Q8_0: int8; Q4_0: nibble - 8), int64."""
    nb = (cols + 31) // 32
    bl = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(rows, nb, -1)
    if qtype == Q80:
        w = bl[:, :, 2:34].view(np.int8).astype(np.int64)
    else:
        lo = (bl[:, :, 2:18] & 0x0F).astype(np.int64) - 8
        hi = (bl[:, :, 2:18] >> 4).astype(np.int64) - 8
        w = np.concatenate([lo, hi], axis=2)
    return np.einsum("rbj,tbj->rtb", w, q.astype(np.int64))


def rmsnorm(x, w, eps, use_ref=False):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    y = np.zeros_like(x)
    if use_ref:
        _check_ref(ref().ref_rmsnorm(_f(x), _f(w), x.size, eps, _f(y)))
    else:
        lib().orc_rmsnorm(_f(x), _f(w), x.size, eps, _f(y))
    return y


def rope(q, k, pos, theta, neox=True, use_ref=False):
    q = np.array(q, np.float32, copy=True, order="C")
    k = np.array(k, np.float32, copy=True, order="C")
    fn = ref().ref_rope if use_ref else lib().orc_rope
    rc = fn(_f(q), q.shape[0], _f(k), k.shape[0], q.shape[1], pos, theta, 1 if neox else 0)
    if use_ref:
        _check_ref(rc)
    return q, k


def softmax(x, use_ref=False):
    x = np.ascontiguousarray(x, np.float32)
    y = np.zeros_like(x)
    if use_ref:
        _check_ref(ref().ref_softmax(_f(x), x.size, _f(y)))
    else:
        lib().orc_softmax(_f(x), x.size, _f(y))
    return y


def swiglu(g, u, use_ref=False):
    g = np.ascontiguousarray(g, np.float32)
    u = np.ascontiguousarray(u, np.float32)
    y = np.zeros_like(g)
    if use_ref:
        _check_ref(ref().ref_swiglu(_f(g), _f(u), g.size, _f(y)))
    else:
        lib().orc_swiglu(_f(g), _f(u), g.size, _f(y))
    return y


def argmax(x, use_ref=False):
    x = np.ascontiguousarray(x, np.float32)
    return (ref().ref_argmax if use_ref else lib().orc_argmax)(_f(x), x.size)


def attention(q, keys, values, layer, pos, n_heads):
    """keys/values: [n_layers, max_seq, n_kv, hd] float32."""
    q = np.ascontiguousarray(q, np.float32)
    _, max_seq, n_kv, hd = keys.shape
    out = np.zeros(n_heads * hd, np.float32)
    scratch = np.zeros(2 * (pos + 1), np.float32)
    lib().orc_attention(_f(q), _f(keys), _f(values), max_seq, n_kv, hd, layer, pos,
                        n_heads, _f(out), _f(scratch))
    return out


# ------------------------------------------------------------ whole model
class _Layer(C.Structure):
    _fields_ = [(n, _vp) for n in ("attention_norm", "wq", "wk", "wv", "bq", "bk", "bv",
                                    "wo", "ffn_norm", "w_gate", "w_up", "w_down")]


class _Model(C.Structure):
    _fields_ = [("vocab", C.c_int), ("dim", C.c_int), ("hidden_dim", C.c_int),
                ("n_layers", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("head_dim", C.c_int), ("max_seq", C.c_int), ("rope_theta", C.c_float),
                ("eps", C.c_float), ("rope_neox", C.c_int), ("qtype", C.c_int),
                ("lm_head_qtype", C.c_int), ("token_embedding", _vp), ("final_norm", _vp),
                ("lm_head", _vp), ("layers", C.POINTER(_Layer))]


class OracleModel:
    """The C restatement of ForwardToken over a SynthModel-like weight set.

    ``w`` must expose ``cfg`` (dict) and the arrays documented in
    dqm_mini_llama_b200.synth.SynthModel.  The tied lm_head is the F32
    dequantization of the token_embd blocks, as the reference loader builds
    it.
    """

    def __init__(self, w, max_seq: int):
        c = w.cfg
        self.cfg = c
        self.max_seq = max_seq
        self._keep = []
        qt = w.qtype
        self.emb = dequantize(qt, w.token_embd, c["vocab"], c["dim"])
        self._keep.append(self.emb)
        layers = (_Layer * c["n_layers"])()
        for i, L in enumerate(w.layers):
            lay = layers[i]
            for name in ("attention_norm", "wq", "wk", "wv", "wo", "ffn_norm",
                         "w_gate", "w_up", "w_down", "bq", "bk", "bv"):
                arr = getattr(L, name)
                if arr is None:
                    setattr(lay, name, None)
                    continue
                arr = np.ascontiguousarray(arr)
                self._keep.append(arr)
                setattr(lay, name, arr.ctypes.data)
        self._layers = layers
        m = _Model()
        m.vocab, m.dim, m.hidden_dim = c["vocab"], c["dim"], c["hidden"]
        m.n_layers, m.n_heads, m.n_kv_heads = c["n_layers"], c["n_heads"], c["n_kv_heads"]
        m.head_dim = c["dim"] // c["n_heads"]
        m.max_seq = max_seq
        m.rope_theta, m.eps, m.rope_neox = c["rope_theta"], c["eps"], 1
        m.qtype = qt
        fn = np.ascontiguousarray(w.final_norm, np.float32)
        self._keep.append(fn)
        m.token_embedding = self.emb.ctypes.data
        m.final_norm = fn.ctypes.data
        if w.lm_head is None:
            m.lm_head_qtype = F32
            m.lm_head = self.emb.ctypes.data
        else:
            lm = np.ascontiguousarray(w.lm_head)
            self._keep.append(lm)
            m.lm_head_qtype = qt
            m.lm_head = lm.ctypes.data
        m.layers = C.cast(layers, C.POINTER(_Layer))
        self._m = m
        hd = m.head_dim
        self.keys = np.zeros((c["n_layers"], max_seq, c["n_kv_heads"], hd), np.float32)
        self.values = np.zeros_like(self.keys)
        self._scratch = np.zeros(lib().orc_forward_scratch_floats(C.byref(m)), np.float32)

    def reset(self):
        self.keys[:] = 0
        self.values[:] = 0

    def forward_token(self, token: int, pos: int) -> np.ndarray:
        logits = np.zeros(self.cfg["vocab"], np.float32)
        lib().orc_forward_token(C.byref(self._m), _f(self.keys), _f(self.values), pos,
                                token, _f(logits), _f(self._scratch))
        return logits


class RefModel:
    """The reference's own ForwardBatch/ForwardToken over the same weights."""

    def __init__(self, w, max_seq: int, threads: int = 0):
        R = ref()
        c = w.cfg
        if threads:
            R.ref_set_threads(threads)
        self.cfg = c
        self.h = R.ref_model_create(c["vocab"], c["dim"], c["hidden"], c["n_layers"],
                                    c["n_heads"], c["n_kv_heads"], max_seq,
                                    c["rope_theta"], c["eps"], 1)
        qt = w.qtype
        tied = w.lm_head is None
        _check_ref(R.ref_model_set_embedding(self.h, qt, _v(np.ascontiguousarray(w.token_embd)),
                                             1 if tied else 0))
        if not tied:
            _check_ref(R.ref_model_set_lm_head(self.h, qt, _v(np.ascontiguousarray(w.lm_head))))
        _check_ref(R.ref_model_set_final_norm(self.h, _f(np.ascontiguousarray(w.final_norm,
                                                                              np.float32))))

        def fp(a):
            return None if a is None else _f(np.ascontiguousarray(a, np.float32))

        for i, L in enumerate(w.layers):
            _check_ref(R.ref_model_set_layer(
                self.h, i, qt, fp(L.attention_norm), _v(L.wq), _v(L.wk), _v(L.wv),
                fp(L.bq), fp(L.bk), fp(L.bv), _v(L.wo), fp(L.ffn_norm), _v(L.w_gate),
                _v(L.w_up), _v(L.w_down)))
        _check_ref(R.ref_model_finish(self.h))

    def __del__(self):
        try:
            if self.h:
                ref().ref_model_destroy(self.h)
                self.h = None
        except Exception:
            pass

    def reset(self):
        _check_ref(ref().ref_context_reset(self.h))

    def forward_batch(self, tokens, start_pos: int) -> np.ndarray:
        toks = np.ascontiguousarray(tokens, dtype=np.int32)
        logits = np.zeros(self.cfg["vocab"], np.float32)
        _check_ref(ref().ref_forward_batch(self.h, toks.ctypes.data_as(_ip), toks.size,
                                           start_pos, _f(logits)))
        return logits

    def pos(self) -> int:
        return ref().ref_context_pos(self.h)

    def history(self):
        n = ref().ref_context_history(self.h, None, 0)
        out = np.zeros(max(n, 1), np.int32)
        ref().ref_context_history(self.h, out.ctypes.data_as(_ip), n)
        return out[:n]


_GGUF_CHILD = r"""
import ctypes as C, struct, sys
path, out, threads = sys.argv[1], sys.argv[2], int(sys.argv[3])
toks = [int(t) for t in sys.argv[4].split(",")]
R = C.CDLL(sys.argv[5])
R.ref_last_error.restype = C.c_char_p
R.ref_set_threads.argtypes = [C.c_int]
R.ref_model_load_gguf.argtypes = [C.c_char_p, C.c_void_p]
R.ref_model_load_gguf.restype = C.c_void_p
R.ref_forward_batch.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
if threads:
    R.ref_set_threads(threads)
cfg = (C.c_int * 8)()
h = R.ref_model_load_gguf(path.encode(), cfg)
if not h:
    sys.stderr.write(R.ref_last_error().decode())
    sys.exit(2)
arr = (C.c_int * len(toks))(*toks)
logits = (C.c_float * cfg[0])()
if R.ref_forward_batch(h, arr, len(toks), 0, logits):
    sys.stderr.write(R.ref_last_error().decode())
    sys.exit(3)
with open(out, "wb") as f:
    f.write(struct.pack("<8i", *cfg))
    f.write(bytes(logits))
"""


def ref_gguf_forward(path: str, tokens, threads: int = 0):
    """The reference's own LoadGgufModel (src/gguf_loader.cc:279-364) over a
    GGUF file, then its ForwardBatch over `tokens` from position 0: returns
    (config dict, last-token logits).  Runs in a child interpreter that loads
    only ctypes: inside a process that has imported numpy, the reference's
    reader faulted in its console output (std::cout), while plain hosts read
    the same files cleanly."""
    import subprocess
    import sys
    import tempfile
    with tempfile.NamedTemporaryFile(suffix=".bin") as tf:
        r = subprocess.run([sys.executable, "-c", _GGUF_CHILD, path, tf.name, str(threads),
                            ",".join(str(int(t)) for t in tokens),
                            os.path.join(HERE, "_ref", "libdqmref.so")],
                           capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("reference GGUF load failed: " + r.stderr[-2000:])
        raw = open(tf.name, "rb").read()
    cfg = np.frombuffer(raw[:32], np.int32)
    keys = ("vocab", "dim", "hidden", "n_layers", "n_heads", "n_kv_heads", "max_seq", "neox")
    return dict(zip(keys, (int(v) for v in cfg))), np.frombuffer(raw[32:], np.float32).copy()

