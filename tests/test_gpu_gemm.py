"""Tensor-core (tcgen05) GEMM of the prefill / batched-row linears.

soc_b200_linear and the forward switch to the tcgen05 kernel from 16 rows (fp16/bf16
weights; 32 rows for int8/int4, expanded to fp16 first); fewer rows run on the CUDA-core
GEMV (the 4-row cases below).  Up to 512 rows the input rows are
carried as hi + lo halves (fp32-level products); above that they are rounded once to the
weight type (fp16: 11-bit, bf16: 8-bit significand) and accumulated in fp32, so the kernel
cases compare against an fp64 product with tolerances scaled by that rounding; the model cases compare prefill logits with the
CPU oracle at the 2e-2 logit tolerance and greedy ids exactly.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O
from soc_b200 import runtime as R
from soc_b200.bundle import QWEN3_0_6B, tiny_config

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-2


@pytest.mark.parametrize("rows", [4, 16, 64, 100, 256, 1000])
@pytest.mark.parametrize("shape", [(2048, 1024), (1024, 2048), (6144, 1024), (1024, 3072), (1000, 1024), (4096, 4096)],
                         ids=["q", "o", "gate_up", "down", "ragged_n", "h4096"])
@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_tc_linear_against_fp64(gpu_ctx, dtype, rows, shape):
    import torch
    out_f, in_f = shape
    g = torch.Generator().manual_seed(out_f * 7 + rows)
    tdt = torch.float16 if dtype == "fp16" else torch.bfloat16
    w = (torch.randn(out_f, in_f, generator=g) * 0.02).to(tdt)
    x = torch.randn(rows, in_f, generator=g)
    ref = x.double() @ w.double().T
    # the GEMM rounds x to the weight type; the reference of that rounding alone
    ref_r = x.to(tdt).double() @ w.double().T
    wd, xd = w.cuda(), x.cuda()
    y = torch.full((rows, out_f), float("nan"), device="cuda")
    fmt = R.WEIGHTS_F16 if dtype == "fp16" else R.WEIGHTS_BF16
    gpu_ctx.linear(fmt, wd.data_ptr(), None, out_f, in_f, xd.data_ptr(), rows, y.data_ptr(),
                   torch.cuda.current_stream().cuda_stream)
    gpu_ctx.synchronize()
    torch.cuda.synchronize()
    yc = y.double().cpu()
    assert torch.isfinite(yc).all()
    if rows <= 512:
        # hi + lo input halves: fp32-level agreement with the exact product
        assert (yc - ref).abs().max().item() <= 2e-5 * in_f ** 0.5
    else:
        # one rounded half per input: fp32 accumulation of exactly-rounded products
        assert (yc - ref_r).abs().max().item() <= 2e-5 * in_f ** 0.5
        rel = 2.0 ** -11 if dtype == "fp16" else 2.0 ** -8
        assert (yc - ref).abs().max().item() <= 6 * rel * 0.02 * in_f ** 0.5 + 2e-5 * in_f ** 0.5


CASES = {
    "qwen06_shape_2layer": (dict(QWEN3_0_6B, num_hidden_layers=2), "float16"),
    "bf16_gqa4_d128": (tiny_config(num_attention_heads=8, num_key_value_heads=2, head_dim=128), "bfloat16"),
    "tied_f16_gqa2_d64": (tiny_config(), "float16"),
}


@pytest.fixture
def tc_rows():
    old = os.environ.get("SOC_B200_TC_MIN_ROWS")

    def set_(v):
        os.environ["SOC_B200_TC_MIN_ROWS"] = str(v)

    yield set_
    if old is None:
        os.environ.pop("SOC_B200_TC_MIN_ROWS", None)
    else:
        os.environ["SOC_B200_TC_MIN_ROWS"] = old


@pytest.mark.parametrize("case", sorted(CASES))
def test_tc_prefill_logits_match_oracle(gpu_ctx, make_bundle, tc_rows, case):
    cfg, dt = CASES[case]
    p = make_bundle("tc_" + case, cfg, seed=9, dtype=dt)
    m = R.Model(gpu_ctx, p)
    om = O.OracleModel(p, 512)
    prompt = np.random.default_rng(12).integers(0, cfg["vocab_size"], 200).astype(np.int32)
    ref = om.forward(prompt, 0, last_only=True)[0]
    out = {}
    for mode, v in (("tc", 64), ("cuda_cores", 0)):
        tc_rows(v)
        kv = R.KVCache(m, 1, 512)
        lg, nid = m.forward_logits_cached(kv, 0, prompt)
        out[mode] = lg
        assert np.abs(lg - ref).max() <= LOGIT_TOL, (mode, np.abs(lg - ref).max())
        assert nid == O.argmax(ref), mode
        kv.free()
    m.free()


def test_prefill_2048_then_greedy_matches_oracle(gpu_ctx, make_bundle):
    """Config-2 length on a 2-layer Qwen3-0.6B-shape fp16 bundle: one 2048-token prefill
    (tensor-core GEMMs above 512 rows, flash attention over the whole causal triangle) with
    the default kernel choices, its last-row logits and greedy id against the oracle, then 8
    greedy decode steps against a 2048-entry cache, each step's logits and id against the
    oracle's."""
    cfg, dt = CASES["qwen06_shape_2layer"]
    p = make_bundle("tc_qwen06_shape_2layer", cfg, seed=9, dtype=dt)
    prompt = np.random.default_rng(31).integers(0, cfg["vocab_size"], 2048).astype(np.int32)
    om = O.OracleModel(p, 2080)
    ref = om.forward(prompt, 0, last_only=True)[0]
    m = R.Model(gpu_ctx, p)
    kv = R.KVCache(m, 1, 2080)
    lg, nid = m.forward_logits_cached(kv, 0, prompt)
    assert np.abs(lg - ref).max() <= LOGIT_TOL, np.abs(lg - ref).max()
    assert nid == O.argmax(ref)
    tok = nid
    for i in range(8):
        ref = om.forward([tok], 2048 + i, last_only=True)[0]
        lg, nxt = m.decode(kv, [0], [tok])
        assert np.abs(lg[0] - ref).max() <= LOGIT_TOL, (i, np.abs(lg[0] - ref).max())
        assert int(nxt[0]) == O.argmax(ref), i
        tok = int(nxt[0])
    kv.free()
    m.free()


def test_tc_prefill_then_greedy_matches_oracle(gpu_ctx, make_bundle, tc_rows):
    """A 160-token prompt through the tensor-core prefill, then 24 decode steps: the greedy
    ids equal the oracle's."""
    tc_rows(64)
    cfg, dt = CASES["qwen06_shape_2layer"]
    p = make_bundle("tc_qwen06_shape_2layer", cfg, seed=9, dtype=dt)
    m = R.Model(gpu_ctx, p)
    prompt = np.random.default_rng(13).integers(0, cfg["vocab_size"], 160).astype(np.int32)
    toks, _ = O.OracleModel(p, 256).generate(prompt, 24)
    kv = R.KVCache(m, 1, 256)
    assert m.generate(kv, 0, prompt, 24) == toks
    kv.free()
    m.free()


def test_tc_batched_decode_rows(gpu_ctx, make_bundle, tc_rows):
    """80 sequences decoded in one batch (80 rows >= 64: tensor-core linears) equal the same
    sequences decoded one at a time."""
    tc_rows(64)
    cfg = tiny_config()
    p = make_bundle("tc_batch_tiny", cfg, seed=3, dtype="float16")
    m = R.Model(gpu_ctx, p)
    n = 80
    rng = np.random.default_rng(5)
    kv = R.KVCache(m, n, 64 * n)
    firsts = []
    for s in range(n):
        _, nid = m.forward_logits_cached(kv, s, rng.integers(0, cfg["vocab_size"], 3 + s % 7).astype(np.int32))
        firsts.append(nid)
    lg, nxt = m.decode(kv, list(range(n)), firsts)
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, cfg["vocab_size"], 3 + s % 7).astype(np.int32) for s in range(n)]
    for s in (0, 17, 41, 79):
        om = O.OracleModel(p, 64)
        om.forward(prompts[s], 0, last_only=True)
        ref = om.forward([firsts[s]], len(prompts[s]), last_only=True)[0]
        assert np.abs(lg[s] - ref).max() <= LOGIT_TOL
        assert int(nxt[s]) == O.argmax(ref)
    kv.free()
    m.free()


FLASH_CASES = {
    "tied_f16_gqa2_d64": (tiny_config(), "float16"),
    "f16_gqa4_d128": (tiny_config(num_attention_heads=8, num_key_value_heads=2, head_dim=128), "float16"),
    "mha_d128": (tiny_config(num_attention_heads=2, num_key_value_heads=2, head_dim=128), "float16"),
    "qwen06_shape_2layer": (dict(QWEN3_0_6B, num_hidden_layers=2), "float16"),
}


@pytest.fixture
def flash_rows():
    old = os.environ.get("SOC_B200_FLASH_MIN_ROWS")

    def set_(v):
        os.environ["SOC_B200_FLASH_MIN_ROWS"] = str(v)

    yield set_
    if old is None:
        os.environ.pop("SOC_B200_FLASH_MIN_ROWS", None)
    else:
        os.environ["SOC_B200_FLASH_MIN_ROWS"] = old


@pytest.mark.parametrize("case", sorted(FLASH_CASES))
def test_flash_prefill_two_chunks_match_oracle(gpu_ctx, make_bundle, flash_rows, case):
    """Prefill in two calls (45 then 83 rows: the second starts at position 45, ragged
    64-row blocks) through the flash kernel; last-row logits and greedy id vs the oracle,
    and every layer's KV cache vs the oracle's cache."""
    flash_rows(32)
    cfg, dt = FLASH_CASES[case]
    p = make_bundle("flash_" + case, cfg, seed=21, dtype=dt)
    m = R.Model(gpu_ctx, p)
    prompt = np.random.default_rng(22).integers(0, cfg["vocab_size"], 128).astype(np.int32)
    om = O.OracleModel(p, 256)
    om.forward(prompt[:45], 0, last_only=True)
    ref = om.forward(prompt[45:], 45, last_only=True)[0]
    kv = R.KVCache(m, 1, 256)
    m.forward_logits_cached(kv, 0, prompt[:45])
    lg, nid = m.forward_logits_cached(kv, 0, prompt[45:])
    assert np.abs(lg - ref).max() <= LOGIT_TOL
    assert nid == O.argmax(ref)
    kv.free()
    m.free()


def test_flash_and_row_attention_agree(gpu_ctx, make_bundle, flash_rows):
    """The flash kernel and the per-row split-K kernel give the same prefill logits within
    the fp16 rounding of q and of the softmax weights."""
    cfg, dt = FLASH_CASES["qwen06_shape_2layer"]
    p = make_bundle("flash_qwen06_shape_2layer", cfg, seed=21, dtype=dt)
    m = R.Model(gpu_ctx, p)
    prompt = np.random.default_rng(23).integers(0, cfg["vocab_size"], 700).astype(np.int32)
    out = []
    for v in (32, 0):
        flash_rows(v)
        kv = R.KVCache(m, 1, 1024)
        out.append(m.forward_logits_cached(kv, 0, prompt)[0])
        kv.free()
    assert np.abs(out[0] - out[1]).max() <= LOGIT_TOL
    m.free()
