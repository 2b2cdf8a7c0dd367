"""Batched ragged decode over seeded random KV contexts (the shape of the batched-decode
benchmark: many sequences, each with its own context length, paged fp16 cache).

soc_b200_kv_fill_random writes the contexts on the device; its values are restated in
numpy (oracle.kv_random) and compared bit for bit.  The oracle then gets the same cache
contents per sequence and decodes one sequence at a time; the GPU decodes all sequences in
one batch.  Logits within 2e-2 max-abs, greedy ids identical.
"""
import numpy as np
import pytest

from oracle import oracle as O
from soc_b200 import runtime as R
from soc_b200.bundle import QWEN3_0_6B, tiny_config

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-2


def test_kv_fill_random_matches_restatement(gpu_ctx, make_bundle):
    cfg = dict(QWEN3_0_6B, num_hidden_layers=2)
    p = make_bundle("batched_qwen06_2layer", cfg, seed=41, dtype="float16")
    m = R.Model(gpu_ctx, p)
    kv = R.KVCache(m, 3, 2048)
    for seq, n, seed in ((0, 37, 5), (2, 300, 123456789012345)):
        kv.fill_random(seq, n, seed)
        assert kv.length(seq) == n
        for layer in range(2):
            k, v = kv.read(seq, layer, 0, n)
            rk = O.kv_random(seed, seq, layer, 0, n, cfg["num_key_value_heads"], cfg["head_dim"], 2)
            rv = O.kv_random(seed, seq, layer, 1, n, cfg["num_key_value_heads"], cfg["head_dim"], 2)
            assert np.array_equal(k, rk.astype(np.float32))
            assert np.array_equal(v, rv.astype(np.float32))
    # refilling a sequence replaces it (pages are reused, length resets)
    kv.fill_random(0, 5, 9)
    assert kv.length(0) == 5
    kv.free()
    m.free()


CASES = {
    "tiny_f16": (tiny_config(), None, 24),
    "qwen06_2layer_f16": (dict(QWEN3_0_6B, num_hidden_layers=2), None, 12),
    "qwen06_2layer_int8": (dict(QWEN3_0_6B, num_hidden_layers=2), "int8_g64", 20),
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_batched_ragged_decode_over_random_contexts(gpu_ctx, make_bundle, case):
    cfg, quant, n = CASES[case]
    p = make_bundle("batched_" + case, cfg, seed=43, dtype="float16", quant=quant)
    m = R.Model(gpu_ctx, p)
    L, hkv, hd = cfg["num_hidden_layers"], cfg["num_key_value_heads"], cfg["head_dim"]
    rng = np.random.default_rng(44)
    ctx = rng.integers(16, 300, n)
    kv = R.KVCache(m, n, int(ctx.sum()) + 16 * n + 64 * n)
    for s in range(n):
        kv.fill_random(s, int(ctx[s]), 1000 + s)
    toks = rng.integers(0, cfg["vocab_size"], n).astype(np.int32)
    oracles = []
    for s in (0, n // 2, n - 1):
        om = O.OracleModel(p, 400)
        for layer in range(L):
            om.set_cache(layer, O.kv_random(1000 + s, s, layer, 0, int(ctx[s]), hkv, hd, L),
                         O.kv_random(1000 + s, s, layer, 1, int(ctx[s]), hkv, hd, L))
        om.set_length(int(ctx[s]))
        oracles.append((s, om))
    for step in range(3):
        lg, nxt = m.decode(kv, list(range(n)), toks)
        for s, om in oracles:
            ref = om.forward([int(toks[s])], int(ctx[s]) + step, last_only=True)[0]
            assert np.abs(lg[s] - ref).max() <= LOGIT_TOL, (s, step, np.abs(lg[s] - ref).max())
            assert int(nxt[s]) == O.argmax(ref)
        toks = nxt.astype(np.int32)
    for s in range(n):
        assert kv.length(s) == int(ctx[s]) + 3
    kv.free()
    m.free()


@pytest.mark.parametrize("kernel", ["lanes", "mma"])
def test_batched_decode_long_contexts_cycle_the_page_ring(gpu_ctx, make_bundle, kernel):
    """40 sequences at contexts 700-1100: one attention split streams 20-35 pages through the
    shared-memory ring (several times around it), for both page-attention kernels."""
    import os
    cfg = dict(QWEN3_0_6B, num_hidden_layers=2)
    p = make_bundle("batched_qwen06_2layer_f16", cfg, seed=43, dtype="float16")
    old = os.environ.get("SOC_B200_ATTENTION")
    os.environ["SOC_B200_ATTENTION"] = kernel
    try:
        m = R.Model(gpu_ctx, p)
        L, hkv, hd = cfg["num_hidden_layers"], cfg["num_key_value_heads"], cfg["head_dim"]
        n = 40
        rng = np.random.default_rng(46)
        ctx = rng.integers(700, 1100, n)
        kv = R.KVCache(m, n, int(ctx.sum()) + 32 * n)
        for s in range(n):
            kv.fill_random(s, int(ctx[s]), 2000 + s)
        toks = rng.integers(0, cfg["vocab_size"], n).astype(np.int32)
        lg, nxt = m.decode(kv, list(range(n)), toks)
        for s in (0, 19, 39):
            om = O.OracleModel(p, 1200)
            for layer in range(L):
                om.set_cache(layer, O.kv_random(2000 + s, s, layer, 0, int(ctx[s]), hkv, hd, L),
                             O.kv_random(2000 + s, s, layer, 1, int(ctx[s]), hkv, hd, L))
            om.set_length(int(ctx[s]))
            ref = om.forward([int(toks[s])], int(ctx[s]), last_only=True)[0]
            assert np.abs(lg[s] - ref).max() <= LOGIT_TOL, (s, np.abs(lg[s] - ref).max())
            assert int(nxt[s]) == O.argmax(ref)
        kv.free()
        m.free()
    finally:
        if old is None:
            os.environ.pop("SOC_B200_ATTENTION", None)
        else:
            os.environ["SOC_B200_ATTENTION"] = old


def test_batched_int8_decode_contexts_near_4096(gpu_ctx, make_bundle):
    """The config-3 form at its longest contexts: int8 g64 linears, 6 sequences with contexts
    in [3800, 4096) of seeded random KV, two batched decode steps; three sequences against the
    oracle (logits within 2e-2, greedy ids identical)."""
    cfg, quant, _ = CASES["qwen06_2layer_int8"]
    p = make_bundle("batched_qwen06_2layer_int8", cfg, seed=43, dtype="float16", quant=quant)
    m = R.Model(gpu_ctx, p)
    L, hkv, hd = cfg["num_hidden_layers"], cfg["num_key_value_heads"], cfg["head_dim"]
    n = 6
    rng = np.random.default_rng(48)
    ctx = rng.integers(3800, 4096, n)
    kv = R.KVCache(m, n, int(ctx.sum()) + 32 * n)
    for s in range(n):
        kv.fill_random(s, int(ctx[s]), 3000 + s)
    toks = rng.integers(0, cfg["vocab_size"], n).astype(np.int32)
    oracles = []
    for s in (0, 3, 5):
        om = O.OracleModel(p, 4128)
        for layer in range(L):
            om.set_cache(layer, O.kv_random(3000 + s, s, layer, 0, int(ctx[s]), hkv, hd, L),
                         O.kv_random(3000 + s, s, layer, 1, int(ctx[s]), hkv, hd, L))
        om.set_length(int(ctx[s]))
        oracles.append((s, om))
    for step in range(2):
        lg, nxt = m.decode(kv, list(range(n)), toks)
        for s, om in oracles:
            ref = om.forward([int(toks[s])], int(ctx[s]) + step, last_only=True)[0]
            assert np.abs(lg[s] - ref).max() <= LOGIT_TOL, (s, step, np.abs(lg[s] - ref).max())
            assert int(nxt[s]) == O.argmax(ref)
        toks = nxt.astype(np.int32)
    kv.free()
    m.free()
