"""Parity of the B200 path (through the C ABI) with the CPU oracle / reference goldens.

Tolerances: logits within 2e-2 max-abs (fp32 accumulation, fp16 KV cache);
greedy ids identical; KV-cache indexing bit-exact (kv_write -> kv_read).
"""
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from soc_b200 import runtime as R
from soc_b200.bundle import QWEN3_0_6B, tiny_config

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-2
GOLDEN = Path(__file__).resolve().parent / "golden"

CASES = {
    "tied_f16_gqa2_d64": (tiny_config(), "float16"),
    "untied_f16": (tiny_config(tie_word_embeddings=False), "float16"),
    "bf16_gqa4_d128": (tiny_config(num_attention_heads=8, num_key_value_heads=2, head_dim=128), "bfloat16"),
    "mha_d128": (tiny_config(num_attention_heads=2, num_key_value_heads=2, head_dim=128), "float16"),
    "qwen06_shape_2layer": (dict(QWEN3_0_6B, num_hidden_layers=2), "float16"),
}


@pytest.fixture(scope="module")
def models(gpu_ctx, make_bundle):
    """(case, decode path) -> (manifest, Model).  Path "mk" is the persistent batch-1 decode
    kernel (the default where the shape allows it), "graph" the CUDA-graph of modular kernels."""
    import os
    cache = {}

    def get(case, path="mk"):
        if (case, path) not in cache:
            cfg, dt = CASES[case]
            p = make_bundle(case, cfg, seed=7, dtype=dt)
            old = os.environ.get("SOC_B200_DECODE_PATH")
            os.environ["SOC_B200_DECODE_PATH"] = path
            try:
                cache[(case, path)] = (p, R.Model(gpu_ctx, p))
            finally:
                if old is None:
                    os.environ.pop("SOC_B200_DECODE_PATH")
                else:
                    os.environ["SOC_B200_DECODE_PATH"] = old
        return cache[(case, path)]

    yield get
    for _, m in cache.values():
        m.free()


def _prompt(cfg, n, seed):
    return np.random.default_rng(seed).integers(0, cfg["vocab_size"], n).astype(np.int32)


@pytest.mark.parametrize("path", ["mk", "graph"])
@pytest.mark.parametrize("case", sorted(CASES))
def test_prefill_and_decode_logits_match_oracle(models, case, path):
    p, m = models(case, path)
    cfg = CASES[case][0]
    kv = R.KVCache(m, 1, 256)
    om = O.OracleModel(p, 256)
    prompt = _prompt(cfg, 13, 1)
    lg, nid = m.forward_logits_cached(kv, 0, prompt)
    ref = om.forward(prompt, 0, last_only=True)[0]
    assert np.abs(lg - ref).max() <= LOGIT_TOL
    assert nid == O.argmax(ref)
    tok, pos = nid, len(prompt)
    for _ in range(6):
        lg, nxt = m.decode(kv, [0], [tok])
        ref = om.forward([tok], pos, last_only=True)[0]
        assert np.abs(lg[0] - ref).max() <= LOGIT_TOL
        assert int(nxt[0]) == O.argmax(ref)
        tok, pos = int(nxt[0]), pos + 1
    assert kv.length(0) == pos
    kv.free()


@pytest.mark.parametrize("path", ["mk", "graph"])
@pytest.mark.parametrize("case", ["tied_f16_gqa2_d64", "bf16_gqa4_d128", "qwen06_shape_2layer", "mha_d128"])
def test_generate_matches_oracle_greedy(models, case, path):
    p, m = models(case, path)
    cfg = CASES[case][0]
    kv = R.KVCache(m, 2, 512)
    prompt = _prompt(cfg, 9, 2)
    toks, _ = O.OracleModel(p, 256).generate(prompt, 12)
    assert m.generate(kv, 1, prompt, 12) == toks
    assert kv.length(1) == len(prompt) + 11
    # a second run on the same cache re-uses the captured decode graph
    assert m.generate(kv, 1, prompt, 12) == toks
    kv.free()


@pytest.mark.parametrize("path", ["mk", "graph"])
def test_captured_graphs_follow_their_cache_and_buffers(models, path):
    """Short prefills and graph-path decode steps replay captured CUDA graphs.  A graph bakes in
    the device pointers of its KV cache and of the model's scratch: a new cache (which the host
    allocator often places at the freed one's address) and a longer prompt (which regrows the
    scratch) must each capture again instead of replaying against freed memory."""
    p, m = models("qwen06_shape_2layer", path)
    cfg = CASES["qwen06_shape_2layer"][0]
    short, long_ = _prompt(cfg, 40, 31), _prompt(cfg, 300, 32)
    toks, _ = O.OracleModel(p, 512).generate(short, 6)
    long_toks, _ = O.OracleModel(p, 512).generate(long_, 3)
    for i in range(3):
        kv = R.KVCache(m, 1, 512)
        assert m.generate(kv, 0, short, 6) == toks, f"fresh cache {i}"
        kv.free()
    kv = R.KVCache(m, 1, 512)
    assert m.generate(kv, 0, long_, 3) == long_toks
    kv.reset(0)
    assert m.generate(kv, 0, short, 6) == toks
    kv.free()


@pytest.mark.parametrize("path", ["mk", "graph"])
def test_generate_long_context_split_k(models, path):
    """Decode at contexts 300..340 (several attention splits per kv head)."""
    p, m = models("tied_f16_gqa2_d64", path)
    prompt = _prompt(CASES["tied_f16_gqa2_d64"][0], 300, 6)
    toks, _ = O.OracleModel(p, 400).generate(prompt, 40)
    kv = R.KVCache(m, 1, 512)
    assert m.generate(kv, 0, prompt, 40) == toks
    kv.free()


@pytest.mark.parametrize("path", ["mk", "graph"])
@pytest.mark.parametrize("at", [0, 3, 7])
def test_generate_eos_stops_and_truncates_cache(models, path, at):
    """EOS at the prefill's pick (0), mid-way (3) and at the last step (7).  On the persistent
    kernel the stop happens on the device; the cache must then hold exactly the prompt and
    the ids before the EOS, so decoding the EOS next continues the oracle's sequence."""
    p, m = models("tied_f16_gqa2_d64", path)
    prompt = _prompt(CASES["tied_f16_gqa2_d64"][0], 5, 3)
    toks, _ = O.OracleModel(p, 64).generate(prompt, 10)
    kv = R.KVCache(m, 1, 64)
    eos = toks[at]
    first = toks.index(eos)
    out = m.generate(kv, 0, prompt, 8, eos=eos)
    assert out == toks[: first + 1]
    assert kv.length(0) == len(prompt) + first
    _, nxt = m.decode(kv, [0], [eos])
    assert int(nxt[0]) == toks[first + 1]
    assert kv.length(0) == len(prompt) + first + 1
    # the next generation on the same model runs every step again
    n0 = R.kernel_launches()
    assert m.generate(kv, 0, prompt, 8) == toks[:8]
    full = R.kernel_launches() - n0
    if path == "graph":
        # the graph loop stops on the device too: its launch count, corrected by the device's
        # own step counter, shows that the seven steps after an EOS at the prefill's pick never ran
        n0 = R.kernel_launches()
        assert m.generate(kv, 0, prompt, 8, eos=toks[0]) == toks[:1]
        assert full - (R.kernel_launches() - n0) >= 7 * 10  # at least ten kernels per step
    kv.free()


@pytest.mark.parametrize("path", ["mk", "graph"])
@pytest.mark.parametrize("temperature", [0.7, 3.0])
def test_sampler_temperature_on_every_pick_path(models, path, temperature):
    """With Sampler(temperature, top_k) set, every pick (prefill, batch-1 decode, batched
    decode, the on-device generate loop, decode_noalloc) is the reference rule applied to the
    logits the device returns: bit-exact, since both divide the same floats."""
    p, m = models("tied_f16_gqa2_d64", path)
    cfg = CASES["tied_f16_gqa2_d64"][0]
    with pytest.raises(R.SocError, match="sampler temperature must be positive"):
        m.set_sampler(-1.0, 1)
    with pytest.raises(R.SocError, match="sampler top_k must be positive"):
        m.set_sampler(1.0, 0)
    m.set_sampler(temperature, 4)
    try:
        kv = R.KVCache(m, 2, 256)
        prompt = _prompt(cfg, 7, 11)
        logits, nid = m.forward_logits_cached(kv, 0, prompt)
        assert nid == O.sample_rule(logits, temperature)
        picks, last = [nid], nid
        for _ in range(6):
            lg, nxt = m.decode(kv, [0], [last])
            assert int(nxt[0]) == O.sample_rule(lg[0], temperature)
            last = int(nxt[0])
            picks.append(last)
        assert m.generate(kv, 1, prompt, 7) == picks
        lg, nxt = m.decode(kv, [0, 1], [last, last])
        for r in range(2):
            assert int(nxt[r]) == O.sample_rule(lg[r], temperature)
        if path == "mk":
            lg, nid2 = m.decode_noalloc(kv, 0, int(nxt[0]))
            assert nid2 == O.sample_rule(lg, temperature)
        kv.free()
    finally:
        m.set_sampler(1.0, 1)


def test_batched_ragged_decode(models):
    p, m = models("bf16_gqa4_d128")
    cfg = CASES["bf16_gqa4_d128"][0]
    kv = R.KVCache(m, 4, 1024)
    lens = [3, 17, 40]
    oms, toks, pos = [], [], []
    for s, n in enumerate(lens):
        pr = _prompt(cfg, n, 10 + s)
        om = O.OracleModel(p, 128)
        ref = om.forward(pr, 0, last_only=True)[0]
        _, nid = m.forward_logits_cached(kv, s, pr)
        assert nid == O.argmax(ref)
        oms.append(om)
        toks.append(nid)
        pos.append(n)
    for _ in range(4):
        lg, nxt = m.decode(kv, [0, 1, 2], toks)
        for s in range(3):
            ref = oms[s].forward([toks[s]], pos[s], last_only=True)[0]
            assert np.abs(lg[s] - ref).max() <= LOGIT_TOL
            assert int(nxt[s]) == O.argmax(ref)
        toks = [int(t) for t in nxt]
        pos = [q + 1 for q in pos]
    kv.free()


def test_long_prompt_and_chunk_consistency(models):
    """600-token prompt: one prefill == two half prefills == prefill(599) + decode(1) == oracle."""
    p, m = models("tied_f16_gqa2_d64")
    cfg = CASES["tied_f16_gqa2_d64"][0]
    pr = _prompt(cfg, 600, 4)
    kv = R.KVCache(m, 3, 4096)
    a, _ = m.forward_logits_cached(kv, 0, pr)
    m.forward_logits_cached(kv, 1, pr[:300])
    b, _ = m.forward_logits_cached(kv, 1, pr[300:])
    m.forward_logits_cached(kv, 2, pr[:599])
    c, _ = m.decode(kv, [2], [pr[599]])
    ref = O.OracleModel(p, 700).forward(pr, 0, last_only=True)[0]
    for x in (a, b, c[0]):
        assert np.abs(x - ref).max() <= LOGIT_TOL
    kv.free()


def test_kv_cache_matches_oracle(models):
    p, m = models("tied_f16_gqa2_d64")
    cfg = CASES["tied_f16_gqa2_d64"][0]
    pr = _prompt(cfg, 21, 5)
    kv = R.KVCache(m, 1, 64)
    m.forward_logits_cached(kv, 0, pr)
    om = O.OracleModel(p, 64)
    om.forward(pr, 0, last_only=True)
    for layer in range(cfg["num_hidden_layers"]):
        k, v = kv.read(0, layer, 0, 21)
        ko, vo = om.kv_read(layer, 0, 21)
        # fp16 storage (half an fp16 ulp of the fp32 value) plus the fp32 rounding the
        # earlier layers carry in (amplified by the k RMSNorm); indexing itself is pinned
        # bit-exactly by test_kv_write_read_bit_exact_across_pages.
        assert np.all(np.abs(k - ko) <= np.abs(ko) * 2.0 ** -10 + 5e-3), np.abs(k - ko).max()
        assert np.all(np.abs(v - vo) <= np.abs(vo) * 2.0 ** -10 + 5e-3), np.abs(v - vo).max()
    kv.free()


def test_kv_write_read_bit_exact_across_pages(models):
    _, m = models("bf16_gqa4_d128")
    hkv, hd = m.info.kv_heads, m.info.head_dim
    kv = R.KVCache(m, 3, 512)
    rng = np.random.default_rng(0)
    for seq, n in [(0, 5), (2, 37), (1, 16)]:
        k = rng.standard_normal((n, hkv, hd)).astype(np.float16).astype(np.float32)
        v = rng.standard_normal((n, hkv, hd)).astype(np.float16).astype(np.float32)
        kv.write(seq, 1, 0, k, v)
        k2, v2 = kv.read(seq, 1, 0, n)
        assert np.array_equal(k, k2) and np.array_equal(v, v2)
        assert kv.length(seq) == n
        # a window that straddles a 16-token page boundary
        if n > 20:
            k3, _ = kv.read(seq, 1, 14, 19)
            assert np.array_equal(k3, k[14:19])
    kv.free()


def test_error_paths(models, gpu_ctx, tmp_path):
    p, m = models("tied_f16_gqa2_d64")
    kv = R.KVCache(m, 1, 32)
    with pytest.raises(R.SocError, match="token id out of range") as e:
        m.forward_logits_cached(kv, 0, [1, 1000])
    assert e.value.code == R.ERR_RANGE
    with pytest.raises(R.SocError, match="prefilled KV cache"):
        m.decode(kv, [0], [1])
    with pytest.raises(R.SocError) as e:
        m.forward_logits_cached(kv, 0, list(range(40)))
    assert e.value.code == R.ERR_CAPACITY
    with pytest.raises(R.SocError, match="read range exceeds"):
        kv.read(0, 0, 0, 5)
    kv.free()
    # manifest validation text follows the reference loader
    import json
    import shutil
    bad = tmp_path / "bad"
    shutil.copytree(Path(p).parent, bad)
    man = json.loads((bad / "manifest.json").read_text())
    man["format"] = "other"
    (bad / "manifest.json").write_text(json.dumps(man))
    with pytest.raises(R.SocError, match="manifest format must be soc.cpp.llm_export") as e:
        R.Model(gpu_ctx, bad / "manifest.json")
    assert e.value.code == R.ERR_FORMAT
    man["format"] = "soc.cpp.llm_export"
    man["tensors"] = [t for t in man["tensors"] if "k_norm" not in t["name"]]
    (bad / "manifest.json").write_text(json.dumps(man))
    with pytest.raises(R.SocError, match="missing tensor in manifest: model.layers.0.self_attn.k_norm.weight"):
        R.Model(gpu_ctx, bad / "manifest.json")
    man = json.loads((Path(p).parent / "manifest.json").read_text())
    rec = next(t for t in man["tensors"] if t["name"].endswith("layers.1.mlp.up_proj.weight"))
    with open(bad / rec["file"], "r+b") as f:
        f.truncate(10)
    (bad / "manifest.json").write_text(json.dumps(man))
    with pytest.raises(R.SocError, match="smaller than expected byte_size") as e:
        R.Model(gpu_ctx, bad / "manifest.json")
    assert e.value.code == R.ERR_IO


def test_generation_context_api(models):
    p, m = models("tied_f16_gqa2_d64")
    gc = R.GenerationContext(m, max_sequence_length=24)
    prompt = _prompt(CASES["tied_f16_gqa2_d64"][0], 6, 8)
    gc.prefill(prompt)
    first = O.argmax(gc._last_logits)
    gc.running_token_ids.append(first)
    with pytest.raises(R.SocError, match="match the current sequence tail"):
        gc.decode_next_token(first + 1)
    r = gc.decode_next_token(first)
    toks, _ = O.OracleModel(p, 64).generate(prompt, 2)
    assert [first, r.token_id] == toks
    assert gc.generate(prompt, 4) == O.OracleModel(p, 64).generate(prompt, 4)[0]


@pytest.mark.parametrize("fixture", sorted(GOLDEN.glob("tiny_*.npz")), ids=lambda q: q.stem)
def test_reference_golden_vectors_on_gpu(gpu_ctx, fixture, tmp_path):
    from tests.golden.make_golden import bundle_for, load_fixture
    fx = load_fixture(fixture)
    p = bundle_for(fx, tmp_path)
    m = R.Model(gpu_ctx, p)
    kv = R.KVCache(m, 1, 64)
    lg, nid = m.forward_logits_cached(kv, 0, fx["prompt"])
    assert np.abs(lg - fx["prefill_logits"][-1]).max() <= LOGIT_TOL
    assert nid == int(fx["greedy"][0])
    for i, tok in enumerate(fx["decode_inputs"]):
        lg, nxt = m.decode(kv, [0], [int(tok)])
        assert np.abs(lg[0] - fx["decode_logits"][i]).max() <= LOGIT_TOL
        assert int(nxt[0]) == int(fx["greedy"][i + 1])
    kv.free()
    m.free()


def test_config0_greedy_matches_reference(gpu_ctx):
    """Benchmark config 0 at full Qwen3-0.6B shape: 16-token prompt + 32 greedy tokens,
    token-for-token equal to the reference CPU runtime's run (tests/golden/config0_greedy.npz)."""
    path = GOLDEN / "config0_greedy.npz"
    if not path.exists():
        pytest.skip("config-0 golden not generated")
    from soc_b200.bundle import cached_bundle
    from tests.golden.make_golden import load_fixture, weights_digest
    fx = load_fixture(path)
    meta = fx["meta"]
    p = cached_bundle("config0", meta["cfg"], seed=meta["seed"], dtype=meta["dtype"])
    assert weights_digest(p) == meta["weights_sha256"]
    m = R.Model(gpu_ctx, p)
    kv = R.KVCache(m, 1, 256)
    out = m.generate(kv, 0, fx["prompt"], len(fx["greedy"]))
    assert out == fx["greedy"].tolist()
    # logits of the first step agree with the reference's top-16
    kv.reset(0)
    lg, _ = m.forward_logits_cached(kv, 0, fx["prompt"])
    assert np.abs(lg[fx["top_ids"][0]] - fx["top_logits"][0]).max() <= LOGIT_TOL
    kv.free()
    m.free()


@pytest.mark.parametrize("rows", [1, 4, 16, 64])
@pytest.mark.parametrize("shape", [(2048, 1024), (1024, 2048), (6144, 1024), (1024, 3072), (151936, 1024)],
                         ids=["q", "o", "gate_up", "down", "lm_head"])
def test_linear_kernel_against_fp64(gpu_ctx, rows, shape):
    import torch
    out_f, in_f = shape
    g = torch.Generator().manual_seed(out_f + rows)
    w = (torch.randn(out_f, in_f, generator=g) * 0.02).half()
    x = torch.randn(rows, in_f, generator=g)
    ref = x.double() @ w.double().T
    wd, xd = w.cuda(), x.cuda()
    y = torch.empty(rows, out_f, device="cuda")
    gpu_ctx.linear(R.WEIGHTS_F16, wd.data_ptr(), None, out_f, in_f, xd.data_ptr(), rows, y.data_ptr(),
                   torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    err = (y.double().cpu() - ref).abs().max().item()
    assert err <= 1e-4 * (in_f ** 0.5), err


def _topk_ref(row, k, temperature=1.0):
    """The sampler's candidates from a logits row: larger logit / temperature first, lower id
    first among equal values (Mac/gpu/src/runtime/sampler.cpp:36-68 with that tie rule)."""
    v = (row / np.float32(temperature)).astype(np.float32)
    order = np.lexsort((np.arange(row.size), -v))
    return order[:k]


@pytest.mark.parametrize("path", ["mk", "graph"])
def test_topk_candidates_match_the_logits_row(models, path):
    """soc_b200_topk after a prefill and after decode steps: the k candidates are exactly the k
    largest of the row the same call returned (ids and raw logits), the first one is the
    greedy pick, and under a temperature the order is that of logit / temperature."""
    p, m = models("qwen06_shape_2layer", path)
    cfg = CASES["qwen06_shape_2layer"][0]
    kv = R.KVCache(m, 1, 256)
    prompt = _prompt(cfg, 9, 4)
    lg, nid = m.forward_logits_cached(kv, 0, prompt)
    vals, ids = m.topk(0, 16)
    ref = _topk_ref(lg, 16)
    assert np.array_equal(ids, ref)
    assert np.array_equal(vals, lg[ref])
    assert int(ids[0]) == nid
    tok = nid
    for k in (1, 8, 64):
        lgd, nxt = m.decode(kv, [0], [tok])
        vals, ids = m.topk(0, k)
        ref = _topk_ref(lgd[0], k)
        assert np.array_equal(ids, ref), k
        assert np.array_equal(vals, lgd[0][ref])
        assert int(ids[0]) == int(nxt[0])
        tok = int(nxt[0])
    m.set_sampler(0.7, 8)
    try:
        lgd, nxt = m.decode(kv, [0], [tok])
        vals, ids = m.topk(0, 8)
        assert np.array_equal(ids, _topk_ref(lgd[0], 8, 0.7))
        assert int(ids[0]) == int(nxt[0])
    finally:
        m.set_sampler(1.0, 1)
    with pytest.raises(R.SocError, match="k must be in"):
        m.topk(0, 65)
    with pytest.raises(R.SocError, match="no logits row 1"):
        m.topk(1, 4)
    kv.free()


def test_generation_context_step_carries_top_candidates(models):
    p, m = models("qwen06_shape_2layer", "mk")
    cfg = CASES["qwen06_shape_2layer"][0]
    m.set_sampler(1.0, 8)
    try:
        gc = R.GenerationContext(m, 64)
        prompt = _prompt(cfg, 7, 5)
        gc.prefill(prompt)
        first = O.argmax(gc._last_logits)
        gc.running_token_ids.append(first)
        res = gc.decode_next_token(first)
        assert res.top_token_ids.shape == (8,) and res.top_logits.shape == (8,)
        assert int(res.top_token_ids[0]) == res.token_id
        assert np.array_equal(res.top_token_ids, _topk_ref(res.logits, 8))
    finally:
        m.set_sampler(1.0, 1)
