"""CPU (gloo, world size 2) check of the tensor-parallel decomposition the library uses.

Each rank takes the shard soc_b200_load_bundle gives it (q/k/v and gate/up rows, o_proj and
down_proj columns, lm_head vocab rows), computes one Qwen3 block and the lm_head in
float64, and the ranks combine the way the CUDA path does: rank 0 adds its o_proj/down_proj
partial to the residual stream and the others contribute their bare partial to an
all-reduce; the greedy pick all-gathers per-shard (value, global index) keys and takes the
largest, the lowest global index winning ties.  The result must equal the unsharded block.
"""
import os

import numpy as np
import pytest
import torch.multiprocessing as mp

from soc_b200.bundle import layer_tensor_names, load_tensor, read_manifest, tiny_config, write_synthetic_bundle


def argmax_key(v: float, idx: int) -> int:
    b = int(np.float32(v).view(np.uint32))
    b = (~b & 0xFFFFFFFF) if b & 0x80000000 else (b | 0x80000000)
    return (b << 32) | (0x7FFFFFFF - idx)


def block(x, W, cfg, pos0, shard=None):
    """One block + lm_head logits of rows x [T, H] (float64); shard = (rank, world) keeps that
    rank's part and returns partial o/down products instead of residual sums."""
    H, D = cfg["hidden_size"], cfg["head_dim"]
    hq, hkv, I = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["intermediate_size"]
    r, w = shard or (0, 1)
    ql, kl, il = hq // w, hkv // w, I // w
    eps = cfg["rms_norm_eps"]

    def rms(a, g):
        return a / np.sqrt((a * a).mean(-1, keepdims=True) + eps) * g

    T = x.shape[0]
    xn = rms(x, W["in"])
    q = xn @ W["q"][r * ql * D:(r + 1) * ql * D].T
    k = xn @ W["k"][r * kl * D:(r + 1) * kl * D].T
    v = xn @ W["v"][r * kl * D:(r + 1) * kl * D].T
    q = q.reshape(T, ql, D)
    k = k.reshape(T, kl, D)
    v = v.reshape(T, kl, D)
    att = np.zeros((T, ql, D))
    for h in range(ql):
        kh = h // (ql // kl)
        s = q[:, h] @ k[:, kh].T / np.sqrt(D)
        s = np.where(np.tril(np.ones((T, T), bool)), s, -np.inf)
        p = np.exp(s - s.max(-1, keepdims=True))
        att[:, h] = (p / p.sum(-1, keepdims=True)) @ v[:, kh]
    o = att.reshape(T, ql * D) @ W["o"][:, r * ql * D:(r + 1) * ql * D].T
    return xn, o, (r, w, il)


def mlp(h, W, cfg, shard=None):
    r, w = shard or (0, 1)
    il = cfg["intermediate_size"] // w
    hn = h / np.sqrt((h * h).mean(-1, keepdims=True) + cfg["rms_norm_eps"]) * W["post"]
    g = hn @ W["gate"][r * il:(r + 1) * il].T
    u = hn @ W["up"][r * il:(r + 1) * il].T
    a = g / (1 + np.exp(-g)) * u
    return a @ W["down"][:, r * il:(r + 1) * il].T


def weights(path):
    m = read_manifest(path)
    names = layer_tensor_names(0)
    keys = ["in", "q", "k", "v", "o", "qn", "kn", "post", "gate", "up", "down"]
    W = {k: np.asarray(load_tensor(m, n), dtype=np.float64) for k, n in zip(keys, names)}
    W["embed"] = np.asarray(load_tensor(m, "model.embed_tokens.weight"), dtype=np.float64)
    return m["config"], W


def _rank(rank, world, path, port, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg, W = weights(path)
    x = W["embed"][[3, 17, 256, 999, 5]]
    _, o, _ = block(x, W, cfg, 0, (rank, world))
    h = torch.from_numpy((x + o) if rank == 0 else o)
    dist.all_reduce(h)
    part = mlp(h.numpy(), W, cfg, (rank, world))
    h2 = torch.from_numpy((h.numpy() + part) if rank == 0 else part)
    dist.all_reduce(h2)
    V = cfg["vocab_size"]
    vl = V // world
    logits = h2.numpy() @ W["embed"][rank * vl:(rank + 1) * vl].T
    logits[0, 7] = 1000.0  # the same maximum in both shards of row 0 (global 7 and V/2 + 7)
    # keys shifted by 2^63 so that signed int64 order is the unsigned key order
    keys = torch.tensor([argmax_key(np.float32(row.max()), rank * vl + int(np.argmax(row))) - (1 << 63) for row in
                         logits.astype(np.float32)], dtype=torch.int64)
    got = [torch.zeros_like(keys) for _ in range(world)]
    dist.all_gather(got, keys)
    merged = [0x7FFFFFFF - ((max(int(g[i]) for g in got) + (1 << 63)) & 0xFFFFFFFF) for i in range(len(keys))]
    if rank == 0:
        q.put((h2.numpy(), merged))
    dist.destroy_process_group()


def test_two_rank_decomposition_equals_whole_block(tmp_path):
    path = write_synthetic_bundle(tmp_path / "b", tiny_config(num_attention_heads=4, num_key_value_heads=2), seed=3)
    ctxm = mp.get_context("spawn")
    q = ctxm.Queue()
    port = 29700 + os.getpid() % 200
    ps = [ctxm.Process(target=_rank, args=(r, 2, str(path), port, q)) for r in range(2)]
    for p in ps:
        p.start()
    h2, merged = q.get(timeout=120)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    cfg, W = weights(path)
    x = W["embed"][[3, 17, 256, 999, 5]]
    _, o, _ = block(x, W, cfg, 0)
    h = x + o
    ref = h + mlp(h, W, cfg)
    assert np.allclose(h2, ref, rtol=1e-10, atol=1e-12)
    logits = (ref @ W["embed"].T).astype(np.float32)
    V = cfg["vocab_size"]
    logits[0, 7] = logits[0, V // 2 + 7] = 1000.0
    expect = [int(np.argmax(row)) for row in logits]  # numpy: first (lowest) index of the maximum
    assert merged[1:] == expect[1:]
    assert merged[0] == 7
