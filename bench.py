"""Benchmark: batch-1 decode of the Qwen2-0.5B-architecture Q8_0 model on B200.

Workload (one "step" = one decoded token at batch 1): the Qwen2-0.5B shape
(24 layers, dim 896, FFN 4864, 14/2 heads, vocab 151936, tied embeddings),
random-init N(0, 0.02) weights quantized to Q8_0, 32 random prompt ids, then
greedy decoding at positions 32..95 (64 decode positions, cycled so a timed
run can hold any number of steps).  Synthetic weights: no checkpoint exists
here.  Each step streams ~525 MB of weights, more than the 126 MB L2, so no
flush is needed between steps.

Reported (one JSON line on rank 0):
  value      decode tok/s with weights resident, tokens chosen by the device
             argmax, the step graph replayed back to back (CUDA events);
  e2e        the same through the public decode entry point with host
             buffers: each call uploads the token and position, runs one step
             with the argmax on the device and returns the chosen token
             (dqmk_decode_greedy, n_steps = 1); e2e.logits_path is the same
             through ForwardToken with the 151936 logits downloaded and
             argmaxed on the host every step, as the reference engine does;
  roofline   the dominant kernel (the Q8_0 GEMV) timed live at the lm_head
             shape 151936 x 896 (145.25 MB per launch, two rotating copies);
  cpu_baseline  the reference's own CPU path (compiled from its sources) on
             this host's cores, a bounded sample of decode steps.
With --impl reference only the reference arm runs and prints its line.
Under torchrun every rank runs an independent replica (the 0.5B model does
not shard); value = tokens of all ranks / max-over-ranks time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
import __graft_entry__ as ge  # noqa: E402

N_PROMPT = 32
N_DECODE_POS = 64
MODEL_SEED = 20261201
PROMPT_SEED = 1
LM_HEAD_BYTES = 151936 * 28 * 34 + 896 * 4 + 151936 * 4  # blocks + x + logits
METRIC = "decode tok/s, Qwen2-0.5B Q8_0, batch 1"
SWEEP_SHAPES = ((896, 896), (128, 896), (4864, 896), (896, 4864), (151936, 896))
ROTATE_BYTES = 1_050_000_000  # rotating weight copies per timed shape: > 8 x the 126 MB L2
REF_MAX_STEPS = 512           # reference arm: at ~12 tokens/s, under a minute of host time


def decode_launches_per_step(n_layers: int) -> int:
    """Kernels of one batch-1 decode step: embedding, per layer QKV GEMV,
    attention, O GEMV, gate/up GEMV, down GEMV, then the lm_head GEMV."""
    return 1 + 5 * n_layers + 1


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during a timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def build_model(pkg, torch, n_layers=None):
    S = pkg.synth
    w = S.make_model(S.QWEN2_0_5B, S.Q80, MODEL_SEED, n_layers=n_layers,
                     quantize_q80=lambda a: pkg.QuantizeToQ80(a).cpu().numpy())
    torch.cuda.synchronize()
    return w


def time_decode(pkg, torch, ctx, first_token, steps: int, warmup: int):
    """Device-resident greedy decode: positions cycle through 32..95."""
    stream = torch.cuda.ExternalStream(ctx.stream_handle)

    def run(n):
        done = 0
        while done < n:
            chunk = min(N_DECODE_POS, n - done)
            ctx.decode_enqueue(first_token, N_PROMPT, chunk)
            done += chunk

    run(warmup)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    run(steps)
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end) / 1000.0


def time_e2e(ctx, first_token, steps: int):
    """ForwardToken through the C ABI with host buffers; host argmax picks the
    next token, like the reference's CPU sampler after ComputeLogitsDevice."""
    logits = np.empty(151936, np.float32)
    tok = first_token
    for i in range(4):  # warm-up
        ctx.ForwardToken(tok, N_PROMPT + i, logits)
    t0 = time.perf_counter()
    for i in range(steps):
        ctx.ForwardToken(tok, N_PROMPT + (i % N_DECODE_POS), logits)
        tok = int(np.argmax(logits))
    return time.perf_counter() - t0


def time_e2e_greedy(ctx, first_token, steps: int):
    """One greedy token per call of the public decode entry point
    (dqmk_decode_greedy with n_steps = 1): the token and position go host to
    device, the step graph runs with the argmax on the device, and the chosen
    token (4 bytes) comes back to the host, which feeds it to the next call."""
    tok = first_token
    for i in range(4):  # warm-up
        tok = int(ctx.decode_greedy(tok, N_PROMPT + i, 1)[0])
    tok = first_token
    t0 = time.perf_counter()
    for i in range(steps):
        tok = int(ctx.decode_greedy(tok, N_PROMPT + (i % N_DECODE_POS), 1)[0])
    return time.perf_counter() - t0


def graph_time(torch, launch, n: int, reps: int = 3):
    """Device seconds per launch of launch(i), i = 0..n-1, captured back to back
    in one CUDA graph (no host launch overhead between kernels) and replayed;
    CUDA events on the replay stream, best of `reps` replays after one warm-up."""
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for i in range(min(n, 4)):
            launch(i)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    with torch.cuda.graph(g):
        for i in range(n):
            launch(i)
    g.replay()
    torch.cuda.synchronize()
    best = None
    stream = torch.cuda.current_stream()
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        g.replay()
        e1.record(stream)
        e1.synchronize()
        dt = e0.elapsed_time(e1) / 1000.0 / n
        best = dt if best is None else min(best, dt)
    del g
    return best


def time_gemv(pkg, torch, w):
    """The lm_head GEMV (151936 x 896 Q8_0, 145.25 MB per launch: the largest
    single kernel by bytes, 5% of the step) standalone: rotating weight copies
    (> 8 x L2) back to back in a CUDA graph, CUDA events."""
    blocks = torch.from_numpy(w.token_embd).cuda()
    copies = -(-ROTATE_BYTES // w.token_embd.nbytes)
    packs = [pkg.pack_weight(pkg.Q80, blocks, 151936, 896) for _ in range(copies)]
    x = torch.randn(896, device="cuda")
    y = torch.empty(151936, device="cuda")
    dt = graph_time(torch, lambda i: pkg.gemv_packed(pkg.Q80, x, packs[i % copies], 151936, y=y),
                    4 * copies)
    del packs
    torch.cuda.empty_cache()
    peak, _ = peaks()
    gbs = LM_HEAD_BYTES / dt / 1e9
    return {"kernel": "gemv_tma_kernel<Q8_0> 151936x896", "us_per_launch": round(dt * 1e6, 2),
            "GB_s": round(gbs, 1), "frac": round(gbs / peak, 4),
            "algorithmic_bytes": LM_HEAD_BYTES, "traffic": profile_traffic()}


def time_dominant(pkg, torch, ctx):
    """The decode step's largest kernel by share of the step (the fused gate/up
    GEMV: RMSNorm of x, 9728 interleaved gate/up rows x 896 Q8_0, SwiGLU
    epilogue) in its in-graph form: launched with programmatic dependent launch
    back to back, each launch on the next of rotating weight copies totalling
    > 8 x L2, captured in a CUDA graph; CUDA events around the replay."""
    rows, k = 9728, 896
    gen = torch.Generator(device="cuda")
    gen.manual_seed(9)
    nb = rows * k // 32
    one = torch.cat([(torch.rand(nb, device="cuda", generator=gen) * 0.01 + 1e-4).half()
                     .view(torch.uint8).view(nb, 2),
                     torch.randint(0, 256, (nb, 32), dtype=torch.uint8, device="cuda",
                                   generator=gen)], dim=1).contiguous()
    copies = -(-ROTATE_BYTES // one.numel())
    packs = [pkg.pack_weight(pkg.Q80, one, rows, k) for _ in range(copies)]
    x = torch.randn(k, device="cuda")
    nw = torch.ones(k, device="cuda")
    y = torch.empty(rows // 2, device="cuda")
    dt = graph_time(torch, lambda i: pkg.gemv_packed_chained(pkg.Q80, x, packs[i % copies], rows,
                                                               y, norm=nw, swiglu=True), copies)
    nbytes = rows * k // 32 * 34 + 4 * k * 2 + 4 * rows // 2
    del packs
    torch.cuda.empty_cache()
    return {"kernel": "gemv_kernel<Q8_0> gate/up 9728x896 (RMSNorm + SwiGLU), chained",
            "achieved": round(nbytes / dt / 1e9, 1), "algorithmic_bytes": nbytes,
            "us_per_launch": round(dt * 1e6, 3), "launches": copies,
            "traffic": profile_traffic("gemv_q8_0_layer_projections.md", "gate_up_dram_bytes:")}


def gemv_sweep(pkg, torch, S):
    """Configuration 2 (Q8_0 GEMV sweep): per shape, rotating weight copies
    totalling more than 8 x L2 (so every launch reads its weight from HBM),
    one launch per copy back to back in a CUDA graph (device time, no host
    launch overhead); GB/s and fraction of the measured HBM peak."""
    peak, kind = peaks()
    out = {"rotating_bytes_per_shape": ROTATE_BYTES, "peak_GB_s": peak, "peak_source": kind}
    for o, i in SWEEP_SHAPES:
        blocks, x = S.gemv_case(o, i, 7)
        bd = torch.from_numpy(blocks).cuda()
        nbytes = blocks.nbytes + 4 * (i + o)
        copies = max(2, -(-ROTATE_BYTES // blocks.nbytes))
        packs = [pkg.pack_weight(pkg.Q80, bd, o, i) for _ in range(copies)]
        xd = torch.from_numpy(x).cuda()
        y = torch.empty(o, device="cuda")
        dt = graph_time(torch, lambda k: pkg.gemv_packed(pkg.Q80, xd, packs[k % copies], o, y=y),
                        copies)
        gbs = nbytes / dt / 1e9
        out[f"{o}x{i}"] = {"us": round(dt * 1e6, 2), "GB_s": round(gbs, 1),
                           "frac": round(gbs / peak, 4), "copies": copies}
        del packs
        torch.cuda.empty_cache()
    return out


def profile_traffic(name="gemv_q8_0_lm_head_151936x896.md", key="dram_bytes_per_launch:"):
    """DRAM bytes per launch of a kernel from its committed ncu summary."""
    path = os.path.join(ROOT, "profiles", name)
    try:
        for ln in open(path):
            if ln.startswith(key):
                return int(float(ln.split(":")[1].strip()))
    except OSError:
        pass
    return None


def int8_peak(torch):
    """Dense int8 tensor-core throughput measured here: torch._int_mm (cuBLASLt
    int8 x int8 -> int32) at 8192^3, best of 10 after warm-up, CUDA events;
    None where the call is unavailable."""
    try:
        n = 8192
        a = torch.randint(-127, 127, (n, n), dtype=torch.int8, device="cuda")
        b = torch.randint(-127, 127, (n, n), dtype=torch.int8, device="cuda").t()
        for _ in range(3):
            torch._int_mm(a, b)
        best = None
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._int_mm(a, b)
            e1.record()
            e1.synchronize()
            t = e0.elapsed_time(e1) / 1e3
            best = t if best is None else min(best, t)
        del a, b
        torch.cuda.empty_cache()
        return round(2.0 * n ** 3 / best / 1e12, 1)
    except Exception:
        return None


def tensor_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured (cuBLAS bf16 burst; fp16 same rate)"
    except Exception:
        return 1590.0, "fallback"


def time_prefill(pkg, torch, S, w, n_tokens: int = 602):
    """ForwardBatch over an n_tokens prompt (median of 5, cache reset between)
    plus the batched linear alone at the gate/up shape."""
    pmodel = pkg.Model.from_synth(w, max_seq_len=n_tokens)
    pctx = pkg.Context(pmodel)
    ptoks = S.prompt_tokens(w.cfg["vocab"], n_tokens, 4)
    stream = torch.cuda.ExternalStream(pctx.stream_handle)
    pctx.ForwardBatch(ptoks, 0)  # first call allocates the prefill buffers
    walls, devs = [], []
    for _ in range(5):
        pctx.reset()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        t0 = time.perf_counter()
        pctx.ForwardBatch(ptoks, 0)
        walls.append(time.perf_counter() - t0)
        e1.record(stream)
        e1.synchronize()
        devs.append(e0.elapsed_time(e1) / 1e3)
    pctx.close()
    pmodel.close()
    wall, dev = statistics.median(walls), statistics.median(devs)

    # the batched linear at the gate/up shape: m x 896 -> 9728
    c = w.cfg
    m, k, o = n_tokens, c["dim"], 2 * c["hidden"]
    blocks, _ = S.gemv_case(o, k, 41)
    packed = pkg.pack_weight(pkg.Q80, blocks, o, k)
    x = torch.randn(m, k, device="cuda")
    y = torch.empty(m, o, device="cuda")
    for _ in range(3):
        pkg.linear_batch_packed(pkg.Q80, x, packed, o, y=y)
    reps = 50
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        pkg.linear_batch_packed(pkg.Q80, x, packed, o, y=y)
    e1.record()
    e1.synchronize()
    t = e0.elapsed_time(e1) / 1e3 / reps
    kp64 = (k + 63) // 64 * 64
    m_tiles, n_tiles = (m + 127) // 128, (o + 127) // 128
    useful = 2.0 * m * k * o / t / 1e12
    # three fp16 products per weight: A_hi B_hi, A_hi B_lo, A_lo B_hi
    issued = 2.0 * 3 * (m_tiles * 128) * kp64 * (n_tiles * 128) / t / 1e12
    peak, src = tensor_peak()
    i8 = int8_peak(torch)
    # useful work of the whole prefill: every linear over all rows, the
    # lm_head on the last row, causal attention (QK^T and PV)
    hd = c["dim"] // c["n_heads"]
    per_layer = (c["dim"] + 2 * c["n_kv_heads"] * hd) * c["dim"] + c["dim"] * c["dim"] \
        + 2 * c["hidden"] * c["dim"] + c["dim"] * c["hidden"]
    attn = 4 * hd * c["n_heads"] * (n_tokens * (n_tokens + 1) // 2) * c["n_layers"]
    ops = 2 * n_tokens * per_layer * c["n_layers"] + 2 * c["vocab"] * c["dim"] + attn
    whole = ops / dev / 1e12
    return {
        "tokens": n_tokens, "tok_s": round(n_tokens / wall, 1),
        "useful_tops": round(whole, 2), "useful_ops": ops,
        "frac_of_int8_peak": round(whole / i8, 4) if i8 else None,
        "int8_peak_tops": i8, "int8_peak_source": "measured here: torch._int_mm (cuBLASLt "
                                                   "int8) at 8192^3, best of 10",
        "frac_of_bf16_peak": round(whole / peak, 4), "bf16_peak_source": src,
        "device_tok_s": round(n_tokens / dev, 1), "ms": round(wall * 1e3, 3),
        "device_ms": round(dev * 1e3, 3),
        "path": "ForwardBatch: per layer RMSNorm + two-term fp16 split, persistent tcgen05 "
                "kind::f16 GEMM over two-term fp16 weights (QKV, O, gate/up, down; split-K where "
                "output tiles are few) + causal attention (tcgen05 kind::f16, two-term Q/K/V/P, "
                "cache range split across CTAs); lm_head GEMV on the last row",
        "linear_batch": {"shape": f"{m}x{k}->{o}", "us_per_call": round(t * 1e6, 2),
                         "useful_tflops": round(useful, 1), "issued_tflops": round(issued, 1),
                         "peak_tflops": peak, "peak_source": src,
                         "frac_useful_of_bf16_peak": round(useful / peak, 4),
                         "frac_useful_of_int8_peak": round(useful / i8, 4) if i8 else None,
                         "note": "standalone op per call: activation split and weight "
                                 "two-term split launches included"},
    }


def time_q4_ctx2048(pkg, torch, S, n_prompt: int = 2048, n_steps: int = 128):
    """Qwen2-0.5B-architecture with Q4_0 weights: a 2048-id prompt through the
    batched prefill, then 128 greedy decode steps over the 2048-long KV cache
    (device argmax, graph replays), each timed with CUDA events."""
    w = S.make_model(S.QWEN2_0_5B, S.Q40, 20261202)
    model = pkg.Model.from_synth(w, max_seq_len=n_prompt + n_steps)
    ctx = pkg.Context(model)
    stream = torch.cuda.ExternalStream(ctx.stream_handle)
    prompt = S.prompt_tokens(w.cfg["vocab"], n_prompt, 3).tolist()
    ctx.ForwardBatch(prompt[:64], 0)  # allocates the prefill buffers
    ctx.reset()
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    e0.record(stream)
    logits = ctx.ForwardBatch(prompt, 0)
    e1.record(stream)
    first = int(np.argmax(logits))
    ctx.decode_enqueue(first, n_prompt, n_steps)
    e2.record(stream)
    e2.synchronize()
    pre, dec = e0.elapsed_time(e1) / 1e3, e1.elapsed_time(e2) / 1e3
    ctx.close()
    model.close()
    bytes_per_token = (sum(getattr(L, n).nbytes for L in w.layers
                           for n in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down"))
                       + w.token_embd.nbytes + 24576 * (n_prompt + n_steps // 2))
    return {"workload": "qwen2-0.5b-architecture Q4_0, 2048-id prompt (batched prefill) then "
                        "128 greedy decode steps at positions 2048..2175",
            "prefill_tok_s": round(n_prompt / pre, 1), "decode_tok_s": round(n_steps / dec, 1),
            "decode_ms_per_token": round(dec / n_steps * 1e3, 4),
            "decode_bytes_per_token": bytes_per_token,
            "decode_GB_s": round(bytes_per_token * n_steps / dec / 1e9, 1)}


def random_q40_blocks(torch, rows: int, cols: int, gen) -> "torch.Tensor":
    """Q4_0 blocks on the device: uniform nibbles, fp16 scales in [0.003, 0.006]
    (weights of std ~0.02, like the N(0, 0.02) models), generated in place."""
    nb = rows * ((cols + 31) // 32)
    d = (torch.rand(nb, device="cuda", generator=gen) * 0.003 + 0.003).half()
    q = torch.randint(0, 256, (nb, 16), dtype=torch.uint8, device="cuda", generator=gen)
    return torch.cat([d.view(torch.uint8).view(nb, 2), q], dim=1).contiguous()


def build_7b(pkg, torch, max_seq: int, local: int, tp_rank: int, tp_world: int, nccl_id):
    """Qwen2-7B-architecture Q4_0 model with random device blocks (uniform
    nibbles, fp16 scales 0.003-0.006), unit norms, N(0, 0.02) QKV biases,
    untied lm_head; this rank's tensor-parallel shard."""
    c = dict(pkg.synth.QWEN2_7B)
    model = pkg.Model(c, max_seq, local)
    model.set_tp(tp_rank, tp_world, nccl_id)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(20261205)
    hd = c["dim"] // c["n_heads"]
    qd, kvd = c["n_heads"] * hd, c["n_kv_heads"] * hd
    model.upload("token_embedding", pkg.Q40, random_q40_blocks(torch, c["vocab"], c["dim"], gen),
                 c["vocab"], c["dim"])
    model.upload("lm_head", pkg.Q40, random_q40_blocks(torch, c["vocab"], c["dim"], gen),
                 c["vocab"], c["dim"])
    ones = np.ones(c["dim"], np.float32)
    model.upload("final_norm", pkg.F32, ones, 1, c["dim"])
    shapes = {"wq": (qd, c["dim"]), "wk": (kvd, c["dim"]), "wv": (kvd, c["dim"]),
              "wo": (c["dim"], qd), "w_gate": (c["hidden"], c["dim"]),
              "w_up": (c["hidden"], c["dim"]), "w_down": (c["dim"], c["hidden"])}
    brng = np.random.default_rng(5)
    for i in range(c["n_layers"]):
        p = f"layers.{i}."
        model.upload(p + "attention_norm", pkg.F32, ones, 1, c["dim"])
        model.upload(p + "ffn_norm", pkg.F32, ones, 1, c["dim"])
        for n, (r, cc) in shapes.items():
            model.upload(p + n, pkg.Q40, random_q40_blocks(torch, r, cc, gen), r, cc)
        for n, size in (("bq", qd), ("bk", kvd), ("bv", kvd)):
            model.upload(p + n, pkg.F32, brng.normal(0, 0.02, size).astype(np.float32), 1, size)
        torch.cuda.synchronize()
    model.finalize()
    return model


def seven_b_bytes(c: dict):
    hd = c["dim"] // c["n_heads"]
    qd, kvd = c["n_heads"] * hd, c["n_kv_heads"] * hd
    weights = (c["n_layers"] * (qd + 2 * kvd + qd + 3 * c["hidden"]) * c["dim"] * 18 // 32
               + c["vocab"] * c["dim"] * 18 // 32)
    return weights, kvd


def block_7b_tp(pkg, torch, dist, world, rank, local, ctx_len=2048, n_steps=64, warm=8,
                p2p=False):
    """Qwen2-7B-architecture Q4_0 (untied lm_head), one sequence, tensor
    parallel over the ranks (one GPU each): a ctx_len prompt through
    ForwardBatch fills the KV cache, then n_steps greedy decode steps are timed
    (device argmax, captured step graph with the NCCL all-reduces inside).
    Returns the result dict on rank 0."""
    S = pkg.synth
    c = dict(S.QWEN2_7B)
    nccl_id = None
    if world > 1:
        obj = [pkg.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nccl_id = obj[0]
    model = build_7b(pkg, torch, ctx_len + n_steps + warm, local, rank, world, nccl_id)
    ctx = pkg.Context(model)
    exchange = "none"
    if world > 1:
        exchange = "nccl"
        if p2p:
            handles = [None] * world
            dist.all_gather_object(handles, ctx.tp_ipc_handle())
            ctx.tp_connect(handles)
            dist.barrier()
            exchange = "peer memory"
    stream = torch.cuda.ExternalStream(ctx.stream_handle)
    prompt = S.prompt_tokens(c["vocab"], ctx_len, 11).tolist()
    logits = ctx.ForwardBatch(prompt, 0)
    first = int(np.argmax(logits))
    ctx.decode_enqueue(first, ctx_len, warm)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        ctx.decode_enqueue(first, ctx_len + warm, n_steps)
        e1.record(stream)
        e1.synchronize()
    dt = e0.elapsed_time(e1) / 1e3
    if dist:
        t = torch.tensor([dt], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t.item())
    ctx.close()
    model.close()
    torch.cuda.synchronize()
    if rank != 0:
        return None
    weights, kvd = seven_b_bytes(c)
    kv = c["n_layers"] * 2 * kvd * 4 * (ctx_len + warm + n_steps // 2)
    per_gpu = (weights + kv) / world
    peak, peak_kind = peaks()
    gbs = per_gpu * n_steps / dt / 1e9
    return {
        "workload": f"qwen2-7b-architecture Q4_0, untied lm_head, {ctx_len}-token prompt then "
                    f"batch-1 greedy decode ({n_steps} timed steps after {warm})",
        "value": round(n_steps / dt, 2), "unit": "tok/s", "ms_per_step": round(dt / n_steps * 1e3, 4),
        "parallelism": f"tp{world}", "exchange": exchange,
        "hbm": {"bytes_per_token_per_gpu": int(per_gpu), "GB_s_per_gpu": round(gbs, 1),
                "frac_of_peak": round(gbs / peak, 4), "peak_source": peak_kind},
        "clocks": clk.summary()}


def block_7b_batch(pkg, torch, dist, world, rank, local, seqs=64, ctx_len=2048, n_steps=32,
                   warm=8, tp=0, kv_fill="zero", e2e_steps=8):
    """Configuration 5: Qwen2-7B-architecture Q4_0, `seqs` sequences decoded
    together (dqmk_batch), tensor parallel over `tp` ranks (default min(world,
    4)), world / tp independent groups splitting the sequences (2 x TP4 at 8
    GPUs).  Every slot's KV cache holds ctx_len positions -- filled by a
    random prompt (kv_fill "prompt", batched steps of 64 positions of one slot)
    or left zero (kv_fill "zero": the step reads the same bytes) -- then `warm`
    greedy steps run and n_steps are timed (one captured step graph per step,
    argmax and position advanced on the device), max over ranks.  Then
    e2e_steps through the public step call with host tokens.  Returns the
    result dict on rank 0."""
    S = pkg.synth
    c = dict(S.QWEN2_7B)
    tp = tp or min(world, 4)
    if world % tp or seqs % (world // tp):
        raise SystemExit("the GPU count must be a multiple of the TP size and the sequences of "
                         "the group count")
    groups = world // tp
    group, tp_rank = rank // tp, rank % tp
    my_seqs = seqs // groups
    nccl_id = None
    if tp > 1:
        mine = pkg.nccl_unique_id() if tp_rank == 0 else None
        ids = [None] * world
        dist.all_gather_object(ids, mine)
        nccl_id = ids[group * tp]
    max_seq = ctx_len + warm + n_steps + e2e_steps + 1
    model = build_7b(pkg, torch, max_seq, local, tp_rank, tp, nccl_id)
    batch = pkg.Batch(model, my_seqs, max_seq)
    stream = torch.cuda.ExternalStream(batch.stream_handle)
    prompts = [S.prompt_tokens(c["vocab"], ctx_len, 1000 + group * my_seqs + i)
               for i in range(my_seqs)]
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    if kv_fill == "prompt":
        for i in range(my_seqs):
            batch.prefill(i, prompts[i][:-1])
    torch.cuda.synchronize()
    fill_s = time.perf_counter() - t0
    last = [int(p[-1]) for p in prompts]
    batch.decode_enqueue(last, [ctx_len - 1] * my_seqs, warm)
    torch.cuda.synchronize()
    pos0 = ctx_len - 1 + warm
    cont = [int(batch.history(i, pos0 - 1, 1)[0]) for i in range(my_seqs)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("timed")  # lets a profiler select the timed steps
        e0.record(stream)
        batch.decode_enqueue(cont, [pos0] * my_seqs, n_steps)
        e1.record(stream)
        e1.synchronize()
        torch.cuda.nvtx.range_pop()
    dt = e0.elapsed_time(e1) / 1e3
    # end to end through the public step call: host tokens in, host tokens out
    pos1 = pos0 + n_steps
    toks = [int(batch.history(i, pos1 - 1, 1)[0]) for i in range(my_seqs)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        _, nxt = batch.step(None, toks, [pos1 + i] * my_seqs, want_logits=False)
        toks = nxt.tolist()
    e2e_dt = time.perf_counter() - t0
    if dist:
        t = torch.tensor([dt, e2e_dt, fill_s], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt, e2e_dt, fill_s = (float(v) for v in t.tolist())
    batch.close()
    model.close()
    torch.cuda.synchronize()
    if rank != 0:
        return None
    weights, kvd = seven_b_bytes(c)
    mean_pos = pos0 + n_steps / 2
    kv = c["n_layers"] * 2 * kvd * 4 * (mean_pos + 1) * my_seqs
    per_gpu = (weights + kv) / tp
    peak, peak_kind = peaks()
    gbs = per_gpu * n_steps / dt / 1e9
    per_layer = 9 + (4 if tp > 1 else 0)
    return {
        "workload": f"qwen2-7b-architecture Q4_0, untied lm_head, {seqs} sequences each with "
                    f"{ctx_len} positions in its KV cache, greedy steps of all sequences "
                    f"together ({n_steps} timed after {warm})",
        "value": round(seqs * n_steps / dt, 1), "unit": "tok/s",
        "ms_per_step": round(dt / n_steps * 1e3, 4),
        "parallelism": f"{groups}x tp{tp}" if groups > 1 else f"tp{tp}",
        "tp": tp, "groups": groups, "nccl_ranks_per_communicator": tp,
        "collectives_per_step": (2 * c["n_layers"] + 1) if tp > 1 else 0,
        "allreduce_bytes": my_seqs * c["dim"] * 4 if tp > 1 else 0,
        "kv_fill": ({"tokens": seqs * (ctx_len - 1), "s": round(fill_s, 3)}
                    if kv_fill == "prompt" else "zero (not filled; the step reads the same bytes)"),
        "hbm": {"bytes_per_step_per_gpu": int(per_gpu), "GB_s_per_gpu": round(gbs, 1),
                "frac_of_peak": round(gbs / peak, 4), "peak_source": peak_kind},
        "e2e": {"value": round(seqs * e2e_steps / e2e_dt, 1), "unit": "tok/s",
                "h2d_bytes_per_step": 3 * 64 * 4, "d2h_bytes_per_step": my_seqs * 4,
                "steps": e2e_steps},
        "gpu_launches": n_steps * (1 + c["n_layers"] * per_layer + 3),
        "clocks": clk.summary()}


def time_cols_gemm(pkg, torch, launches: int = 10):
    """dqmk_linear_cols_packed at the Qwen2-7B gate/up shape: 64 columns x
    37888 rows x 3584, Q4_0 (76 MB of blocks), after 3 warm-up calls; CUDA
    events around `launches` back-to-back calls (each call includes its
    stream-ordered scratch and side tables)."""
    gen = torch.Generator(device="cuda")
    gen.manual_seed(3)
    rows, k = 37888, 3584
    packed = pkg.pack_weight(pkg.Q40, random_q40_blocks(torch, rows, k, gen), rows, k)
    x = torch.randn(64, k, device="cuda")
    y = torch.empty(64, rows, device="cuda")
    for _ in range(3):
        pkg.linear_cols_packed(pkg.Q40, x, packed, rows, y=y)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(launches):
        pkg.linear_cols_packed(pkg.Q40, x, packed, rows, y=y)
    e1.record()
    e1.synchronize()
    return {"shape": "64x3584->37888 Q4_0", "us_per_call": round(e0.elapsed_time(e1) / launches * 1e3, 2)}


def gemv_sample(pkg, torch, spec: str):
    """A few launches of one decode GEMV for profiling: spec "q8_0:37888x3584"
    (quant type, rows x in_features); random blocks (int8 / nibbles uniform,
    fp16 scales in [1e-4, 1e-2]), RMSNorm prologue and SwiGLU epilogue as in
    the decode step's gate/up projection, a 256 MB buffer written between
    launches so the weight is read from HBM."""
    name, shape = spec.split(":")
    qt = {"q8_0": pkg.Q80, "q4_0": pkg.Q40}[name]
    rows, k = (int(v) for v in shape.split("x"))
    gen = torch.Generator(device="cuda")
    gen.manual_seed(5)
    nb = rows * k // 32
    d = (torch.rand(nb, device="cuda", generator=gen) * 0.01 + 1e-4).half().view(torch.uint8)
    q = torch.randint(0, 256, (nb, 32 if qt == pkg.Q80 else 16), dtype=torch.uint8, device="cuda",
                      generator=gen)
    packed = pkg.pack_weight(qt, torch.cat([d.view(nb, 2), q], dim=1).contiguous(), rows, k)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    x = torch.randn(k, device="cuda")
    nw = torch.ones(k, device="cuda")
    y = torch.empty(rows // 2, device="cuda")
    for _ in range(3):
        flush.fill_(1)
        pkg.gemv_packed_chained(qt, x, packed, rows, y, norm=nw, swiglu=True)
    torch.cuda.synchronize()
    return {"gemv_sample": spec, "y0": float(y[0])}


def kernel_sample(pkg, torch):
    """One small launch of every kernel kind of the library, for profiling
    runs (ncu -k regex:... on this mode): quantize / dequantize / pack, the
    ggml-layout Linears (Q8_0, Q4_0, Q4_1, F32), the packed GEMV, the
    TMA-staged lm_head GEMV and the shared-memory ring GEMV, the standalone ops (RMSNorm, SiLU, SwiGLU, add,
    multiply, softmax, argmax, RoPE, embedding lookup, KV write), decode
    attention over a 2048-position cache and over an odd head shape, one Qwen2-0.5B-architecture decode step (embed,
    QKV / O / gate-up / down GEMVs, short-cache attention, lm_head), a
    128-token batched prefill (activation split, tensor-core GEMM, split-K
    epilogue, causal attention, weight split), and one 64-column step of a
    one-layer Qwen2-7B-shaped multi-sequence batch over a 2048-position cache
    (split, batch GEMM, split-K reduce, streaming attention, greedy
    advance)."""
    S = pkg.synth
    x = torch.randn(4096, 4096, device="cuda")
    for qt in (pkg.Q80, pkg.Q40):
        q = pkg.QuantizeToQ80(x) if qt == pkg.Q80 else pkg.QuantizeToQ40(x)
        (pkg.DequantizeFromQ80 if qt == pkg.Q80 else pkg.DequantizeFromQ40)(q, (4096, 4096))
        pkg.pack_weight(qt, q, 4096, 4096)
    del x
    for qt in (pkg.Q80, pkg.Q40, pkg.Q41):
        blocks, xs = S.gemv_case(4864, 896, 3, qt)
        fn = {pkg.Q80: pkg.CudaQ80Linear, pkg.Q40: pkg.CudaQ40Linear, pkg.Q41: pkg.CudaQ41Linear}
        fn[qt](xs, blocks, (4864, 896))
    pkg.CudaLinear(np.random.default_rng(0).standard_normal(896).astype(np.float32),
                   np.random.default_rng(1).standard_normal((4864, 896)).astype(np.float32))
    # the tensor-core GEMV: a tall Q8_0 weight (16384 x 2048, 35 MB)
    blocks, xs = S.gemv_case(16384, 2048, 5, pkg.Q80)
    pkg.gemv_packed(pkg.Q80, torch.from_numpy(xs).cuda(),
                    pkg.pack_weight(pkg.Q80, torch.from_numpy(blocks).cuda(), 16384, 2048), 16384)
    # the shared-memory ring GEMV: a tall Q4_0 weight (65600 x 2048, 75 MB)
    blocks, xs = S.gemv_case(65600, 2048, 5, pkg.Q40)
    pkg.gemv_packed(pkg.Q40, torch.from_numpy(xs).cuda(),
                    pkg.pack_weight(pkg.Q40, torch.from_numpy(blocks).cuda(), 65600, 2048), 65600)
    # the standalone ops of the drop-in boundary
    v = torch.randn(4864, device="cuda")
    w = torch.randn(4864, device="cuda")
    pkg.CudaRmsNormDeviceWeight(v, w, 1e-6)
    pkg.CudaSiluMulDeviceInput(v, w)
    pkg.CudaElementwiseAddDeviceInput(v, w)
    out = torch.empty_like(v)
    for name, args in (("dqmk_silu", (v.data_ptr(), v.numel(), out.data_ptr(), None)),
                       ("dqmk_mul", (v.data_ptr(), w.data_ptr(), v.numel(), out.data_ptr(), None)),
                       ("dqmk_softmax", (v.data_ptr(), v.numel(), out.data_ptr(), None))):
        pkg.check(getattr(pkg.lib(), name)(*args))
    pkg.argmax(v)
    q, k = torch.randn(14 * 64, device="cuda"), torch.randn(2 * 64, device="cuda")
    pkg.CudaRopeDeviceInput(q, k, 14, 2, 64, 5, 1e6)
    pkg.CudaEmbeddingLookupDeviceWeight(torch.randn(1024, 896, device="cuda"), 7)
    # decode attention outside the chain: a 2048-position cache (split over
    # the SMs, merged by the last CTA) and a head shape only the general
    # kernel takes
    for n_heads, n_kv, hd, max_seq, pos in ((14, 2, 64, 2048, 2047), (2, 1, 3, 4, 1)):
        kv = pkg.CudaKvCache(1, max_seq, n_kv, hd)
        kv.keys.normal_()
        kv.values.normal_()
        q = torch.randn(n_heads * hd, device="cuda")
        pkg.CudaAttentionDecodeDeviceInput(q, kv, 0, pos, n_heads, n_kv, hd)
        kv.WriteDevice(0, 0, torch.randn(n_kv * hd, device="cuda"),
                       torch.randn(n_kv * hd, device="cuda"))
    w = S.make_model(S.QWEN2_0_5B, S.Q80, MODEL_SEED,
                     quantize_q80=lambda a: pkg.QuantizeToQ80(a).cpu().numpy())
    model = pkg.Model.from_synth(w, max_seq_len=N_PROMPT + N_DECODE_POS)
    ctx = pkg.Context(model)
    prompt = S.prompt_tokens(w.cfg["vocab"], 128, 5).tolist()
    first = int(np.argmax(ctx.ForwardBatch(prompt[:N_PROMPT], 0)))
    ctx.decode_enqueue(first, N_PROMPT, 1)
    torch.cuda.synchronize()
    ctx.close()
    model.close()
    c7 = dict(S.QWEN2_7B, vocab=8192)
    w7 = S.make_model(c7, S.Q40, 77, n_layers=1)
    m7 = pkg.Model.from_synth(w7, max_seq_len=2048 + 4)
    b7 = pkg.Batch(m7, 64, 2048 + 4)
    b7.decode_enqueue([3] * 64, [2047] * 64, 1)
    torch.cuda.synchronize()
    b7.close()
    m7.close()
    return {"kernel_sample": "done"}


def decode_config(world: int) -> dict:
    """The headline workload, shared by the GPU arm and the reference arm."""
    return {"workload": "qwen2-0.5b-architecture Q8_0, 32-token prompt then batch-1 greedy "
                        "decode at positions 32..95 (cycled)",
            "model": "qwen2-0.5b", "global_batch": world, "seq_len": N_PROMPT + N_DECODE_POS,
            "parallelism": "replicas" if world > 1 else "single",
            "l2": "per-step weight stream 525 MB > 126 MB L2; no flush needed"}


def cpu_model() -> str:
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def reference_decode(w, steps: int, warmup: int, threads: int):
    """The reference's CPU decode (oracle/_ref) on this host: returns s/token."""
    orc = ge.load_oracle()
    if not orc.ref_available():
        return None, "reference library missing"
    rm = orc.RefModel(w, N_PROMPT + N_DECODE_POS, threads=threads)
    S = ge.load_package().synth
    prompt = S.prompt_tokens(w.cfg["vocab"], N_PROMPT, PROMPT_SEED)
    # the same workload as the GPU arm: the 32-token prompt (untimed, the
    # reference's per-token ForwardBatch), then greedy steps from position 32
    logits = rm.forward_batch(prompt, 0)
    tok = int(np.argmax(logits))
    for i in range(warmup):
        logits = rm.forward_batch([tok], N_PROMPT + i)
        tok = int(np.argmax(logits))
    t0 = time.perf_counter()
    for i in range(steps):
        logits = rm.forward_batch([tok], N_PROMPT + (warmup + i) % N_DECODE_POS)
        tok = int(np.argmax(logits))
    dt = time.perf_counter() - t0
    return dt / steps, "ok"


def reference_prefill_sample(w, threads: int, n_tokens: int = 96):
    """The reference's ForwardBatch (src/batch.cc:26-42, a per-token
    ForwardToken loop) over the first n_tokens of the 602-token prefill prompt,
    on this host: tokens/s of the per-token loop."""
    orc = ge.load_oracle()
    S = ge.load_package().synth
    rm = orc.RefModel(w, n_tokens, threads=threads)
    prompt = S.prompt_tokens(w.cfg["vocab"], 602, 4)[:n_tokens]
    t0 = time.perf_counter()
    rm.forward_batch(prompt, 0)
    return n_tokens / (time.perf_counter() - t0)


def reference_linear_sweep(S, threads: int):
    """The reference's LinearQ80 / LinearQ40 (src/quant.cc:350-366) at the
    GEMV-sweep shapes on this host: median of 3 calls after one warm-up."""
    orc = ge.load_oracle()
    orc.ref_set_threads(threads)
    out = {}
    for qt, name in ((S.Q80, "q8_0"), (S.Q40, "q4_0")):
        for o, i in SWEEP_SHAPES:
            blocks, x = S.gemv_case(o, i, 7, qt)
            orc.linear(qt, x, blocks, o, use_ref=True)
            ts = []
            for _ in range(3):
                t0 = time.perf_counter()
                orc.linear(qt, x, blocks, o, use_ref=True)
                ts.append(time.perf_counter() - t0)
            t = statistics.median(ts)
            nbytes = blocks.nbytes + 4 * (i + o)
            out[f"{name} {o}x{i}"] = {"ms": round(t * 1e3, 3), "GB_s": round(nbytes / t / 1e9, 2)}
    return out


def reference_arm(args, rank):
    if rank != 0:
        return
    pkg = ge.load_package()
    S = pkg.synth
    orc = ge.load_oracle()
    if not orc.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libdqmref.so not built"}))
        return
    threads = os.cpu_count() or 1
    w = S.make_model(S.QWEN2_0_5B, S.Q80, MODEL_SEED,
                     quantize_q80=lambda a: orc.quantize_q80(a, use_ref=True))
    # every timed step is one decode token of the same workload; the run is
    # kept to a few minutes on the host cores (about 12 tokens/s)
    steps = max(1, min(args.steps, REF_MAX_STEPS))
    warm = max(3, min(args.warmup, 8))
    spt, _ = reference_decode(w, steps, warm, threads)
    v = 1.0 / spt
    line = {
        "impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "tok/s",
        "n_gpus": args.gpus, "steps": steps, "warmup": warm, "ms_per_step": round(spt * 1e3, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "q8_0xf32",
        "data": "synthetic: random-init N(0,0.02) weights quantized to Q8_0, random prompt ids",
        "config": decode_config(args.gpus),
        "path": "the reference's CPU ForwardBatch / ForwardToken (compiled from its sources: "
                "threaded scalar LinearQ80, AVX2 F32 lm_head) on the host cores",
        "cpu_baseline": {"value": round(v, 4), "unit": "tok/s", "cores": threads,
                         "kind": "reference", "cpu": cpu_model(),
                         "sample": f"{steps} decode steps after {warm} warm-up"},
        "e2e": {"value": round(v, 4), "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    if steps < args.steps:
        line["steps_note"] = f"{args.steps} steps asked; {steps} run (bounded CPU sample)"
    print(json.dumps(line))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4096)
    ap.add_argument("--warmup", type=int, default=64)
    ap.add_argument("--impl", default="dqmk", choices=["dqmk", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-7b", action="store_true", help="skip the Qwen2-7B blocks")
    ap.add_argument("--decode-only", action="store_true",
                    help="time only the decode steps (small runs for profiling)")
    ap.add_argument("--prefill-only", action="store_true",
                    help="time only the 602-token prefill and the batched linear (profiling)")
    ap.add_argument("--model", default="qwen2-0.5b", choices=["qwen2-0.5b", "qwen2-7b"],
                    help="qwen2-7b: only the 7B workload, as its own line")
    ap.add_argument("--ctx", type=int, default=2048, help="qwen2-7b: KV length before decoding")
    ap.add_argument("--seqs", type=int, default=64,
                    help="qwen2-7b: sequences decoded together (64: configuration 5; 1: "
                         "batch-1 decode)")
    ap.add_argument("--tp", type=int, default=0,
                    help="qwen2-7b with --seqs > 1: tensor-parallel group size (default: "
                         "min(ranks, 4)); ranks / tp independent groups split the sequences")
    ap.add_argument("--kv-fill", default="zero", choices=["prompt", "zero"],
                    help="qwen2-7b --seqs > 1: fill every KV cache with a random prompt "
                         "(prompt) or leave it zero and start decoding at position --ctx - 1 "
                         "(zero: the step reads the same bytes)")
    ap.add_argument("--kernel-sample", action="store_true",
                    help="one small launch of every kernel kind (for profiling)")
    ap.add_argument("--gemv-sample", default="",
                    help="a few launches of one decode GEMV (profiling), e.g. q8_0:37888x3584")
    ap.add_argument("--cols-gemm", action="store_true",
                    help="time only the standalone multi-sequence GEMM at the Qwen2-7B gate/up "
                         "shape (64 columns x 37888 x 3584 Q4_0; profiling)")
    ap.add_argument("--p2p", action="store_true",
                    help="qwen2-7b batch 1 under tensor parallelism: exchange partial sums over "
                         "peer memory instead of NCCL all-reduces")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        reference_arm(args, rank)
        return

    import torch
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    pkg = ge.load_package()
    S = pkg.synth
    if args.gemv_sample:
        print(json.dumps(gemv_sample(pkg, torch, args.gemv_sample)))
        return
    if args.cols_gemm:
        print(json.dumps({"cols_gemm": time_cols_gemm(pkg, torch)}))
        return
    if args.kernel_sample:
        print(json.dumps(kernel_sample(pkg, torch)))
        return
    if args.model == "qwen2-7b":
        if args.seqs > 1:
            r = block_7b_batch(pkg, torch, dist, world, rank, local, seqs=args.seqs,
                               ctx_len=args.ctx, n_steps=args.steps, warm=args.warmup, tp=args.tp,
                               kv_fill=args.kv_fill)
        else:
            r = block_7b_tp(pkg, torch, dist, world, rank, local, ctx_len=args.ctx,
                            n_steps=args.steps, warm=args.warmup, p2p=args.p2p)
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps(dict(r, n_gpus=world, steps=args.steps, warmup=args.warmup)))
        return
    w = build_model(pkg, torch)
    if args.prefill_only:
        print(json.dumps({"prefill": time_prefill(pkg, torch, S, w)}))
        return
    model = pkg.Model.from_synth(w, max_seq_len=N_PROMPT + N_DECODE_POS, device=local)
    ctx = pkg.Context(model)
    prompt = S.prompt_tokens(w.cfg["vocab"], N_PROMPT, PROMPT_SEED)
    logits = ctx.ForwardBatch(prompt, 0)
    first = int(np.argmax(logits))
    launches_per_step = decode_launches_per_step(w.cfg["n_layers"])

    # ---- timed region: K device-resident decode steps
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        dt = time_decode(pkg, torch, ctx, first, args.steps, args.warmup)
    clocks = clk.summary()
    if dist:
        t = torch.tensor([dt], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t.item())
    value = world * args.steps / dt

    if args.decode_only:
        if dist:
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": round(value, 2), "unit": "tok/s",
                              "steps": args.steps, "ms_per_step": dt / args.steps * 1e3,
                              "decode_only": True, "clocks": clocks}))
        return

    # ---- e2e through the C ABI with host buffers
    e2e_steps = min(args.steps, 256)
    e2e_dt = time_e2e_greedy(ctx, first, e2e_steps)
    e2e_logits_dt = time_e2e(ctx, first, e2e_steps)
    if dist:
        t = torch.tensor([e2e_dt, e2e_logits_dt], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_dt, e2e_logits_dt = (float(v) for v in t.tolist())
    e2e = world * e2e_steps / e2e_dt

    # ---- the dominant kernel of the step, timed in its in-graph (chained) form
    peak, peak_kind = peaks()
    dom = time_dominant(pkg, torch, ctx)
    bytes_per_token = (sum(getattr(L, n).nbytes for L in w.layers
                           for n in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down"))
                       + w.token_embd.nbytes + 896 * 4 * 2)
    ctx.close()
    model.close()
    lm = time_gemv(pkg, torch, w) if rank == 0 else None
    sweep = None if (args.no_sweep or rank != 0) else gemv_sweep(pkg, torch, S)

    # ---- prefill (ForwardBatch) of a 602-token prompt: the batched path
    prefill = time_prefill(pkg, torch, S, w) if rank == 0 else None
    q4_ctx2048 = time_q4_ctx2048(pkg, torch, S) if rank == 0 else None
    torch.cuda.synchronize()

    # ---- Qwen2-7B: configuration 5 (64 sequences) on every run; batch 1 at N=1
    seven_b = None
    if not args.no_7b:
        seven_b = {"config5": block_7b_batch(pkg, torch, dist, world, rank, local)}
        if world == 1:
            seven_b["batch1_tp1"] = block_7b_tp(pkg, torch, dist, world, rank, local)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        spt, status = reference_decode(w, 8, 3, threads)
        if spt is not None:
            pre_tok_s = reference_prefill_sample(w, threads)
            cpu = {"value": round(1.0 / spt, 4), "unit": "tok/s", "cores": threads,
                   "kind": "reference", "cpu": cpu_model(),
                   "sample": "8 decode steps (after 3 warm-up steps) of the same model and "
                             "positions on the reference's CPU path, threaded over all host "
                             "cores",
                   "prefill_per_token_loop": {
                       "tok_s": round(pre_tok_s, 3), "sample": "the reference's ForwardBatch "
                       "(per-token loop) over the first 96 ids of the 602-token prompt",
                       "gpu_batched_over_reference": (round(prefill["tok_s"] / pre_tok_s, 1)
                                                      if prefill else None)},
                   "linear_sweep": reference_linear_sweep(S, threads)}

    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "q8_0xf32",
        "data": "synthetic: random-init N(0,0.02) weights quantized to Q8_0, random prompt ids",
        "config": decode_config(world),
        "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 8,
                "d2h_bytes_per_step": 4,
                "path": "dqmk_decode_greedy, one token per call: token and position in, the "
                        "device argmax's token out",
                "logits_path": {"value": round(world * e2e_steps / e2e_logits_dt, 2),
                                "unit": "tok/s", "h2d_bytes_per_step": 8,
                                "d2h_bytes_per_step": 151936 * 4,
                                "path": "ForwardToken with the 151936 logits copied to the "
                                        "host and argmaxed there, as the reference engine "
                                        "samples"}},
        "gpu_launches": args.steps * launches_per_step,
        "decode_hbm": {"bytes_per_token": bytes_per_token,
                       "GB_s": round(bytes_per_token * value / world / 1e9, 1),
                       "frac_of_peak": round(bytes_per_token * value / world / 1e9 / peak, 4),
                       "peak_source": peak_kind},
        "roofline": dict(dom, bound="hbm", peak=peak, unit="GB/s",
                         frac=round(dom["achieved"] / peak, 4),
                         peak_source=f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"),
        "lm_head_gemv": lm,
        "gemv_sweep": sweep,
        "prefill": prefill,
        "q4_0_ctx2048": q4_ctx2048,
        "qwen2_7b": seven_b,
        "cpu_baseline": cpu,
        "clocks": clocks,
    }
    print(json.dumps(line))


if __name__ == "__main__":
    main()
