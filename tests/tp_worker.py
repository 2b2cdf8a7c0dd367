"""One rank of a tensor-parallel parity run (launched by test_gpu_tp.py through
torch.distributed.run): loads its shard of a bundle, runs a prefill + greedy decode and a
batched decode over seeded random KV contexts, and rank 0 saves the results to --out."""
import argparse
import os
import sys
from pathlib import Path

import numpy as np

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--bundle", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--vocab", type=int, required=True)
    args = ap.parse_args()
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from soc_b200 import runtime as R

    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=timedelta(seconds=120))
    ctx = R.Context(local)
    comm = R.tensor_parallel_comm(ctx)
    m = R.Model(ctx, args.bundle, tp_rank=rank, tp_size=world, comm=comm)
    assert m.info.tp_size == world and m.info.tp_rank == rank
    out = {}
    # prefill + greedy decode of one sequence
    prompt = np.random.default_rng(61).integers(0, args.vocab, 9).astype(np.int32)
    kv = R.KVCache(m, 1, 128)
    lg, nid = m.forward_logits_cached(kv, 0, prompt)
    out["prefill_logits"], out["prefill_id"] = lg, nid
    # the no-alloc decode step is single-GPU only: refused on a shard, with nothing changed
    try:
        m.decode_noalloc(kv, 0, nid)
        out["noalloc_refusal"] = np.array("")
    except R.SocError as e:
        out["noalloc_refusal"] = np.array(str(e))
    out["length_after_refusal"] = np.array(kv.length(0))
    toks, logits = [nid], []
    for i in range(3):
        lg, nxt = m.decode(kv, [0], [toks[-1]])
        logits.append(lg[0])
        toks.append(int(nxt[0]))
        if i == 0:  # the sampler's candidates over the gathered vocab shards (every rank calls)
            out["topk_vals"], out["topk_ids"] = m.topk(0, 8)
    out["decode_logits"], out["decode_ids"] = np.stack(logits), np.array(toks)
    out["generate"] = np.array(m.generate(kv, 0, prompt, 5))
    kv.free()
    # batched decode over random contexts (global kv-head indexing of the fill)
    ctxs = np.array([40, 77, 120, 33, 96, 150])
    kv = R.KVCache(m, len(ctxs), int(ctxs.sum()) + 64 * len(ctxs))
    for s, c in enumerate(ctxs):
        kv.fill_random(s, int(c), 700 + s)
    first = np.random.default_rng(62).integers(0, args.vocab, len(ctxs)).astype(np.int32)
    lg1, n1 = m.decode(kv, list(range(len(ctxs))), first)
    lg2, n2 = m.decode(kv, list(range(len(ctxs))), n1)
    out.update(batch_ctx=ctxs, batch_first=first, batch_logits1=lg1, batch_ids1=n1, batch_logits2=lg2, batch_ids2=n2)
    kv.free()
    m.free()
    R.Context.nccl_comm_destroy(comm)
    ctx.close()
    if rank == 0:
        np.savez(args.out, prompt=prompt, **out)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
