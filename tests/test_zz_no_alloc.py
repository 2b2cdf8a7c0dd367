"""The decode step that allocates no device memory (soc_b200_decode_noalloc).

It exists for hosts that cannot call cudaMalloc while serving -- an engine that
hands the whole GPU to its own memory pool at start-up, or a latency path that
must not take cudaMalloc's implicit device synchronisation.  Its scratch lives
in a static device array, so its output must equal the allocating entry point's
(soc_b200_decode) on the same inputs, call after call, and the device's free
memory must not move while it runs.  This file is collected last so that a
failure here comes after every other test has run.
"""
import numpy as np
import pytest

from oracle import oracle as O
from soc_b200 import runtime as R
from soc_b200.bundle import QWEN3_0_6B, tiny_config, write_synthetic_bundle

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-2


def _cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test selected but no CUDA device is visible")
    return torch


def test_decode_noalloc_matches_decode_two_calls(tmp_path):
    torch = _cuda()
    cfg = dict(QWEN3_0_6B, num_hidden_layers=2)
    p = write_synthetic_bundle(tmp_path / "b", cfg, seed=9)
    ctx = R.Context(0)
    model = R.Model(ctx, p)
    kv = R.KVCache(model, 2, 512)
    prompt = np.random.default_rng(3).integers(0, cfg["vocab_size"], 11).astype(np.int32)
    _, ta = model.forward_logits_cached(kv, 0, prompt)
    _, tb = model.forward_logits_cached(kv, 1, prompt)
    assert ta == tb
    om = O.OracleModel(p, 64)
    om.forward(prompt, 0, last_only=True)
    free = []
    for i in range(2):  # two calls in a row: the shared array must not carry state over
        la, na = model.decode(kv, [0], [ta])
        lb, nb = model.decode_noalloc(kv, 1, tb)
        ctx.synchronize()
        free.append(torch.cuda.mem_get_info(0)[0])
        # the same persistent kernel with the same split count: bit-identical results
        assert np.array_equal(la[0], lb)
        assert int(na[0]) == nb
        # and both match the CPU oracle
        ref = om.forward([tb], len(prompt) + i, last_only=True)[0]
        assert np.abs(lb - ref).max() <= LOGIT_TOL
        assert nb == O.argmax(ref)
        ta, tb = int(na[0]), nb
    # the first call has loaded every module it needs; the second takes no device memory
    assert free[1] == free[0]
    assert kv.length(0) == kv.length(1) == len(prompt) + 2
    kv.free()
    model.free()
    ctx.close()


def test_decode_noalloc_rejects_before_side_effects(tmp_path):
    """A model loaded without the persistent kernel (the CUDA-graph decode path) is refused
    before the cache reserves a page for the step: the sequence length and the pages held
    are unchanged, and the ordinary decode still runs."""
    import os
    _cuda()
    cfg = tiny_config()
    p = write_synthetic_bundle(tmp_path / "t", cfg, seed=4)
    ctx = R.Context(0)
    old = os.environ.get("SOC_B200_DECODE_PATH")
    os.environ["SOC_B200_DECODE_PATH"] = "graph"
    try:
        model = R.Model(ctx, p)
    finally:
        if old is None:
            os.environ.pop("SOC_B200_DECODE_PATH", None)
        else:
            os.environ["SOC_B200_DECODE_PATH"] = old
    kv = R.KVCache(model, 1, 64)
    prompt = np.arange(3, 19, dtype=np.int32)  # 16 ids: the next step needs a new page
    _, t = model.forward_logits_cached(kv, 0, prompt)
    with pytest.raises(R.SocError, match="without the persistent decode kernel"):
        model.decode_noalloc(kv, 0, t)
    assert kv.length(0) == len(prompt)
    # the page the refused call did not take is still free: a full cache's worth of decode fits
    for _ in range(64 - len(prompt)):
        _, nxt = model.decode(kv, [0], [t], want_logits=False)
        t = int(nxt[0])
    assert kv.length(0) == 64
    kv.free()
    model.free()
    ctx.close()
