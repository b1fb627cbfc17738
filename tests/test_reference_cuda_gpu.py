"""The reference's own CUDA tests, run through this library.

oracle/Makefile (target dropin) compiles the reference's engine sources with
its CUDA backend switched on, leaves out its CUDA kernels (src/cuda_quant.cu,
cuda_ops.cu, cuda_attention.cu) and its cuBLAS matmul (src/cuda_matmul.cc),
links in their drop-in replacement over libdqmk
(dqm-mini-llama_b200/engine_shim/dqmk_backend.cc) and the reference's own
gtest files tests/test_cuda_*.cc: quantized Linear cases at the CUDA tests'
1e-3 tolerance (tests/test_cuda_quant.cc:304-411), ops, decode attention,
the KV cache, F32 matmul, and the tiny model's forward pass against its CPU
forward with the runtime counters the reference asserts
(tests/test_cuda_quant.cc:413-473: 21 uploaded weights, 15 Linear calls, 2
attention calls, one logits download).  The engine code above the kernels --
tensors, KV cache, weight upload, ForwardToken's device branch -- is the
reference's, unchanged.

Those forward tests load models/tiny/model.json + model.bin relative to the
working directory; the test writes a tiny model of the same shape (random
weights) in that manifest format into a temporary directory and runs the
binary there (seeded random weights with the value distribution of the
reference's tiny model)."""
import json
import os
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BINARY = os.path.join(ROOT, "oracle", "_ref", "reference_cuda_tests")

TINY = {"vocab_size": 128, "dim": 32, "hidden_dim": 86, "n_layers": 2, "n_heads": 4,
        "n_kv_heads": 4, "max_seq_len": 128, "rope_theta": 10000.0, "rms_norm_eps": 1e-05}


def write_tiny_manifest(root: str, seed: int = 7) -> None:
    """models/tiny/{model.json, model.bin}: the reference's F32 manifest
    layout (config, tokenizer, tensors with name / shape / dtype / offset /
    byte_size into one raw little-endian float32 file)."""
    c = TINY
    d, h, v = c["dim"], c["hidden_dim"], c["vocab_size"]
    rng = np.random.default_rng(seed)
    shapes = [("token_embedding", [v, d])]
    for i in range(c["n_layers"]):
        p = f"layers.{i}."
        shapes += [(p + "attention_norm", [d]), (p + "wq", [d, d]), (p + "wk", [d, d]),
                   (p + "wv", [d, d]), (p + "wo", [d, d]), (p + "ffn_norm", [d]),
                   (p + "w_gate", [h, d]), (p + "w_up", [h, d]), (p + "w_down", [d, h])]
    shapes += [("final_norm", [d]), ("lm_head", [v, d])]
    tensors, blobs, off = [], [], 0
    for name, shape in shapes:
        # the value distribution of the reference's own tiny model (unit norm
        # weights, matrices of standard deviation ~0.0115), for which its
        # CUDA tests' absolute tolerances (1e-6 on KV-cache entries) are set
        if name.endswith("norm"):
            a = np.ones(shape, np.float32)
        else:
            a = (0.0115 * rng.standard_normal(shape)).astype(np.float32)
        raw = a.tobytes()
        tensors.append({"name": name, "shape": shape, "dtype": "float32", "offset": off,
                        "byte_size": len(raw)})
        blobs.append(raw)
        off += len(raw)
    d_ = os.path.join(root, "models", "tiny")
    os.makedirs(d_, exist_ok=True)
    manifest = {"config": c, "tokenizer": {"type": "ascii", "bos_id": 1, "eos_id": 2,
                                           "unk_id": 0}, "tensors": tensors}
    with open(os.path.join(d_, "model.json"), "w") as f:
        json.dump(manifest, f, indent=2)
    with open(os.path.join(d_, "model.bin"), "wb") as f:
        f.write(b"".join(blobs))


def test_reference_cuda_tests_pass_through_dqmk(cuda, tmp_path):
    if not os.path.exists(BINARY):
        pytest.skip("reference CUDA tests not built (oracle/Makefile dropin needs the "
                    "reference sources)")
    write_tiny_manifest(str(tmp_path))
    r = subprocess.run([BINARY, "--gtest_filter=-*CpuBuild*:*MissingCuda*:*NotBuilt*"],
                       cwd=str(tmp_path), capture_output=True, text=True, timeout=600)
    print(r.stdout[-4000:])
    assert r.returncode == 0, r.stdout[-6000:] + r.stderr[-3000:]
    assert "[  PASSED  ]" in r.stdout
    assert "FAILED" not in r.stdout
