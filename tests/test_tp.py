"""Tensor-parallel host logic on CPU: the shard plan of the Qwen2-7B shape
(column-parallel heads / FFN rows, row-parallel K splits at 32-value blocks,
vocabulary-parallel lm_head) and its exchange between world-size-2 gloo
ranks, including the NCCL unique-id broadcast the GPU ranks use."""
import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_plan_partitions_qwen2_7b(pkg, S):
    c = S.QWEN2_7B
    for world in (1, 2, 4):
        plans = [pkg.tp_plan(c, r, world) for r in range(world)]
        assert sum(p["n_q_heads"] for p in plans) == c["n_heads"]
        assert sum(p["n_kv_heads"] for p in plans) == c["n_kv_heads"]
        assert sum(p["hidden"] for p in plans) == c["hidden"]
        assert sum(p["vocab"] for p in plans) == c["vocab"]
        for p in plans:
            assert p["hidden"] % 32 == 0 and (p["n_q_heads"] * c["dim"] // c["n_heads"]) % 32 == 0
            assert p["vocab_stride"] == -(-c["vocab"] // world)
    # 4 key/value heads do not split 8 ways; 0.5B's 2 do not split 4 ways
    for cfg, world in ((c, 8), (S.QWEN2_0_5B, 4)):
        with pytest.raises(RuntimeError, match="split evenly"):
            pkg.tp_plan(cfg, 0, world)
    with pytest.raises(RuntimeError, match="invalid rank"):
        pkg.tp_plan(c, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_gloo_world2_plan_and_nccl_id_exchange():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.join(ROOT, "tests", "tp_worker.py"), "--mode", "plan"]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=240, env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "plan ok 2" in r.stdout
