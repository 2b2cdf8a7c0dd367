"""Tensor parallelism on 2 GPUs: each rank holds a Megatron-style shard (q/k/v and gate/up
rows, o_proj/down_proj columns, lm_head vocab rows), the residual stream is all-reduced
after o_proj and down_proj and the greedy pick merges per-shard argmax keys.  A 2-rank run
(tests/tp_worker.py under torch.distributed.run) is compared with the CPU oracle on the
whole model: logits within 2e-2 max-abs, identical greedy ids.  Skipped with fewer than 2
visible GPUs."""
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from soc_b200.bundle import QWEN3_8B, tiny_config

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-2
HERE = Path(__file__).resolve().parent

CASES = {
    "tiny_untied_bf16": (tiny_config(tie_word_embeddings=False), "bfloat16"),
    "tiny_tied_f16_gqa4": (tiny_config(num_attention_heads=8, num_key_value_heads=4, head_dim=64), "float16"),
    "qwen8b_shape_2layer_bf16": (dict(QWEN3_8B, num_hidden_layers=2), "bfloat16"),
}


def _gpus():
    import torch
    return torch.cuda.device_count()


@pytest.mark.parametrize("allreduce", ["nccl", "p2p"])
@pytest.mark.parametrize("case", sorted(CASES))
def test_tensor_parallel_two_ranks_match_oracle(make_bundle, tmp_path, case, allreduce):
    """allreduce "p2p": the residual sums of decode-sized steps go through the peer-memory
    all-reduce (SOC_B200_TP_ALLREDUCE=p2p) instead of NCCL's."""
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    cfg, dt = CASES[case]
    p = make_bundle("tp_" + case, cfg, seed=5, dtype=dt)
    out = tmp_path / "tp.npz"
    port = 29500 + (os.getpid() % 1000)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2", "--master-addr",
           "127.0.0.1", "--master-port", str(port), str(HERE / "tp_worker.py"), "--bundle", str(p), "--out", str(out),
           "--vocab", str(cfg["vocab_size"])]
    env = dict(os.environ)
    if allreduce == "p2p":
        env["SOC_B200_TP_ALLREDUCE"] = "p2p"
    else:
        env.pop("SOC_B200_TP_ALLREDUCE", None)
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = np.load(out)
    prompt = res["prompt"]
    assert "not available for a tensor-parallel shard" in str(res["noalloc_refusal"])
    assert int(res["length_after_refusal"]) == len(prompt)
    om = O.OracleModel(p, 256)
    ref = om.forward(prompt, 0, last_only=True)[0]
    assert np.abs(res["prefill_logits"] - ref).max() <= LOGIT_TOL
    assert int(res["prefill_id"]) == O.argmax(ref)
    ids = res["decode_ids"]
    row0 = res["decode_logits"][0]
    order = np.lexsort((np.arange(row0.size), -row0))[:8]
    assert np.array_equal(res["topk_ids"], order)
    assert np.array_equal(res["topk_vals"], row0[order])
    for i in range(3):
        ref = om.forward([int(ids[i])], len(prompt) + i, last_only=True)[0]
        assert np.abs(res["decode_logits"][i] - ref).max() <= LOGIT_TOL
        assert int(ids[i + 1]) == O.argmax(ref)
    gen, _ = O.OracleModel(p, 256).generate(prompt, 5)
    assert list(res["generate"]) == gen
    # batched decode over the seeded random contexts
    L, hkv, hd = cfg["num_hidden_layers"], cfg["num_key_value_heads"], cfg["head_dim"]
    for s, c in enumerate(res["batch_ctx"]):
        if s % 2:
            continue
        om = O.OracleModel(p, 256)
        for layer in range(L):
            om.set_cache(layer, O.kv_random(700 + s, s, layer, 0, int(c), hkv, hd, L),
                         O.kv_random(700 + s, s, layer, 1, int(c), hkv, hd, L))
        om.set_length(int(c))
        ref1 = om.forward([int(res["batch_first"][s])], int(c), last_only=True)[0]
        assert np.abs(res["batch_logits1"][s] - ref1).max() <= LOGIT_TOL
        assert int(res["batch_ids1"][s]) == O.argmax(ref1)
        ref2 = om.forward([int(res["batch_ids1"][s])], int(c) + 1, last_only=True)[0]
        assert np.abs(res["batch_logits2"][s] - ref2).max() <= LOGIT_TOL
        assert int(res["batch_ids2"][s]) == O.argmax(ref2)
