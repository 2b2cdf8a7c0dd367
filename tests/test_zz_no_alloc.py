"""The decode step that allocates no device memory (soc_b200_decode_noalloc).

It exists for hosts that cannot call cudaMalloc while serving -- an engine that
hands the whole GPU to its own memory pool at start-up, or a latency path that
must not take cudaMalloc's implicit device synchronisation.  Its scratch lives
in a static device array, so its output must equal the allocating entry point's
(soc_b200_decode) on the same inputs, call after call.  This file is collected
last so that a failure here comes after every other test has run.
"""
import numpy as np
import pytest

from soc_b200 import runtime as R
from soc_b200.bundle import QWEN3_0_6B, write_synthetic_bundle

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-2


def test_decode_noalloc_matches_decode_two_calls(tmp_path):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test selected but no CUDA device is visible")
    cfg = dict(QWEN3_0_6B, num_hidden_layers=2)
    p = write_synthetic_bundle(tmp_path / "b", cfg, seed=9)
    ctx = R.Context(0)
    model = R.Model(ctx, p)
    kv = R.KVCache(model, 2, 512)
    prompt = np.random.default_rng(3).integers(0, cfg["vocab_size"], 11).astype(np.int32)
    _, ta = model.forward_logits_cached(kv, 0, prompt)
    _, tb = model.forward_logits_cached(kv, 1, prompt)
    assert ta == tb
    for _ in range(2):  # two calls in a row: the shared array must not carry state over
        la, na = model.decode(kv, [0], [ta])
        lb, nb = model.decode_noalloc(kv, 1, tb)
        assert np.abs(la[0] - lb).max() <= LOGIT_TOL
        assert int(na[0]) == nb
        ta, tb = int(na[0]), nb
    assert kv.length(0) == kv.length(1) == len(prompt) + 2
    kv.free()
    model.free()
    ctx.close()
