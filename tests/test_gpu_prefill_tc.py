"""The tcgen05 prefill attention (attn_prefill_tc.cu, SOC_B200_PREFILL_ATTENTION=tc) against the
CPU oracle: the same prompt prefilled in one chunk and in two, last-row logits within the parity
tolerance, identical greedy ids, and the cached keys within fp16 rounding of the oracle's.
The tcgen05 kernel is the default flash step; the mma.sync kernel it replaced
(SOC_B200_PREFILL_ATTENTION=mma) stays selectable and is checked the same way."""
import os

import numpy as np
import pytest

from oracle import oracle as O
from soc_b200 import runtime as R
from soc_b200.bundle import tiny_config

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-2

CASES = {
    "d64_gqa2": (tiny_config(), "float16"),
    "d128_gqa4_bf16": (tiny_config(num_attention_heads=8, num_key_value_heads=2, head_dim=128), "bfloat16"),
}


def _prefill(ctx, path, prompt, chunks, kernel):
    old = os.environ.get("SOC_B200_PREFILL_ATTENTION")
    os.environ["SOC_B200_PREFILL_ATTENTION"] = kernel
    try:
        m = R.Model(ctx, path)
        kv = R.KVCache(m, 1, 1024)
        at, logits, nid = 0, None, None
        for n in chunks:
            logits, nid = m.forward_logits_cached(kv, 0, prompt[at:at + n])
            at += n
        ctx.synchronize()
        k = kv.read(0, 1, 0, at)[0]
        kv.free()
        m.free()
        return logits, nid, k
    finally:
        if old is None:
            os.environ.pop("SOC_B200_PREFILL_ATTENTION", None)
        else:
            os.environ["SOC_B200_PREFILL_ATTENTION"] = old


@pytest.mark.parametrize("kernel", ["tc", "mma"])
@pytest.mark.parametrize("case", sorted(CASES))
@pytest.mark.parametrize("chunks", [(40,), (200,), (150, 130), (33, 300)], ids=str)
def test_tc_prefill_matches_oracle(gpu_ctx, make_bundle, case, chunks, kernel):
    cfg, dt = CASES[case]
    p = make_bundle("tc_" + case, cfg, seed=11, dtype=dt)
    prompt = np.random.default_rng(7).integers(0, cfg["vocab_size"], sum(chunks)).astype(np.int32)
    om = O.OracleModel(p, 1024)
    at = 0
    for n in chunks:
        ref = om.forward(prompt[at:at + n], at, last_only=True)[0]
        at += n
    ref_k = om.kv_read(1, 0, at)[0]
    logits, nid, k = _prefill(gpu_ctx, p, prompt, chunks, kernel)
    assert np.isfinite(logits).all()
    assert np.abs(logits - ref).max() <= LOGIT_TOL
    assert nid == O.argmax(ref)
    assert np.abs(k - ref_k).max() < 1e-2
