"""One rank of a tensor-parallel run, launched by torchrun from the TP tests.

--mode plan (CPU, gloo): every rank asks the library for its shard plan of
    the Qwen2-7B shape; rank 0 draws an NCCL unique id and broadcasts it;
    rank 0 checks that the plans partition heads, FFN rows and vocabulary and
    that every rank received the same id.
--mode gpu (one GPU per rank): every rank builds the same reduced
    Qwen2-7B-shaped model (full layer widths, fewer layers, smaller
    vocabulary), keeps its shard (Model.from_synth(..., tp=...)), runs
    ForwardBatch over the prompt and greedy decoding; rank 0 writes the
    gathered logits and the tokens to --out.  With --p2p the contexts
    exchange IPC handles and connect, so the decode step's partial sums
    travel over peer memory instead of NCCL; without it a two-slot
    multi-sequence batch (dqmk_batch) also decodes the prompt on the same
    shards.
"""
import argparse
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import __graft_entry__ as ge  # noqa: E402

REDUCED_7B = dict(vocab=8192, n_layers=1, seed=77, prompt_seed=9, n_prompt=8, n_steps=8)


def reduced_7b(S):
    r = REDUCED_7B
    w = S.make_model(dict(S.QWEN2_7B, vocab=r["vocab"]), S.Q40, r["seed"], n_layers=r["n_layers"])
    prompt = S.prompt_tokens(r["vocab"], r["n_prompt"], r["prompt_seed"]).tolist()
    return w, prompt


def mode_plan(pkg, rank, world):
    S = pkg.synth
    plan = pkg.tp_plan(S.QWEN2_7B, rank, world)
    obj = [pkg.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    plans, ids = [None] * world, [None] * world
    dist.all_gather_object(plans, plan)
    dist.all_gather_object(ids, obj[0])
    if rank == 0:
        assert all(i == ids[0] and len(i) == 128 for i in ids)
        c = S.QWEN2_7B
        for key0, key, total in (("q_head0", "n_q_heads", c["n_heads"]),
                                 ("kv_head0", "n_kv_heads", c["n_kv_heads"]),
                                 ("hidden0", "hidden", c["hidden"]),
                                 ("vocab0", "vocab", c["vocab"])):
            covered = []
            for p in plans:
                covered.extend(range(p[key0], p[key0] + p[key]))
            assert covered == list(range(total)), key
        # each rank's query heads use only its own key/value heads
        g = c["n_heads"] // c["n_kv_heads"]
        for p in plans:
            assert p["q_head0"] // g == p["kv_head0"]
            assert (p["q_head0"] + p["n_q_heads"] - 1) // g == p["kv_head0"] + p["n_kv_heads"] - 1
        print("plan ok", world)


def mode_gpu(pkg, rank, world, local, out, p2p):
    S = pkg.synth
    torch.cuda.set_device(local)
    w, prompt = reduced_7b(S)
    obj = [pkg.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    r = REDUCED_7B
    model = pkg.Model.from_synth(w, max_seq_len=r["n_prompt"] + r["n_steps"], device=local,
                                 tp=(rank, world, obj[0]))
    ctx = pkg.Context(model)
    if p2p:
        handles = [None] * world
        dist.all_gather_object(handles, ctx.tp_ipc_handle())
        ctx.tp_connect(handles)
        dist.barrier()
    logits = ctx.ForwardBatch(prompt, 0)
    first = int(np.argmax(logits))
    tokens = [first] + ctx.decode_greedy(first, r["n_prompt"], r["n_steps"] - 1).tolist()
    # one more host-visible step: ForwardToken logits after the decoded tokens
    step_logits = ctx.ForwardToken(tokens[-1], r["n_prompt"] + r["n_steps"] - 1)
    ctx.close()
    batch_tokens = []
    if not p2p:
        # the multi-sequence step on the same shards (NCCL all-reduces inside
        # its captured graph): two slots fed the same prompt must both follow
        # the single-sequence greedy path
        batch = pkg.Batch(model, 2, r["n_prompt"] + r["n_steps"])
        for slot in range(2):
            batch.prefill(slot, prompt[:-1])
        _, nxt = batch.step(None, [prompt[-1]] * 2, [r["n_prompt"] - 1] * 2, want_logits=False)
        seq = batch.decode_greedy(nxt.tolist(), [r["n_prompt"]] * 2, r["n_steps"] - 1)
        batch_tokens = [[int(nxt[c])] + seq[:, c].tolist() for c in range(2)]
        batch.close()
    model.close()
    gathered = [None] * world
    dist.all_gather_object(gathered, (tokens, batch_tokens))
    if rank == 0:
        assert all(t == (tokens, batch_tokens) for t in gathered), gathered
        np.savez(out, logits=logits, tokens=np.array(tokens), step_logits=step_logits,
                 batch_tokens=np.array(batch_tokens))
        print("gpu ok", world, tokens, batch_tokens)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", choices=["plan", "gpu"], required=True)
    ap.add_argument("--out", default="")
    ap.add_argument("--p2p", action="store_true",
                    help="exchange partial sums over peer memory instead of NCCL")
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    pkg = ge.load_package()
    try:
        if args.mode == "plan":
            mode_plan(pkg, rank, world)
        else:
            mode_gpu(pkg, rank, world, local, args.out, args.p2p)
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
