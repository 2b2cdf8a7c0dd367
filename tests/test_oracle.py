"""Pins the CPU oracle (oracle/soc_oracle.c) before it is trusted as the checker.

1. Known-answer cases of the reference's own unit tests
   (Mac/cpu/test/test_nn_modules.cpp), restated against the oracle.
2. Bit-exact agreement with the reference CPU runtime itself (oracle/_ref, the
   reference sources compiled unchanged) on synthetic bundles -- skipped where
   the reference build is absent.
3. Bit-exact agreement with golden vectors the reference produced
   (tests/golden/*.npz, made by tests/golden/make_golden.py).
"""
import math
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from soc_b200.bundle import tiny_config, write_synthetic_bundle

GOLDEN = Path(__file__).resolve().parent / "golden"


def near(a, b, tol=1e-5):
    return abs(float(a) - float(b)) <= tol


# ---- 1. known answers (test_nn_modules.cpp) ---------------------------------
def test_linear_known_answer():
    # test_nn_modules.cpp:106-137 (its bias dropped: Qwen3 linears have none)
    w = np.array([[1.0, 2.0, 3.0], [-1.0, 0.5, 4.0]], np.float32)
    x = np.array([[1.0, 0.0, -1.0], [2.0, 1.0, 0.5]], np.float32)
    y = O.linear(x, w)
    assert np.allclose(y, [[-2.0, -5.0], [5.5, 0.5]], atol=1e-5)


def test_linear_fp16_weights():
    # test_nn_modules.cpp:139-155 (fp16 weights decoded exactly)
    w = np.array([[1.0, -0.5], [0.25, 2.0]], np.float16)
    y = O.linear(np.array([[2.0, 4.0]], np.float32), w)
    assert np.allclose(y, [[0.0, 8.5]], atol=1e-6)


def test_rmsnorm_known_answer():
    # test_nn_modules.cpp:157-186
    w = np.array([1.0, 1.5, 0.5], np.float32)
    x = np.array([[3.0, 4.0, 0.0], [1.0, 2.0, 2.0]], np.float32)
    y = O.rmsnorm(x, w, 1e-6)
    s0 = 1.0 / math.sqrt((9 + 16 + 0) / 3.0 + 1e-6)
    s1 = 1.0 / math.sqrt((1 + 4 + 4) / 3.0 + 1e-6)
    assert near(y[0, 0], 3 * s0) and near(y[0, 1], 4 * s0 * 1.5)
    assert near(y[1, 0], 1 * s1) and near(y[1, 2], 2 * s1 * 0.5)


def test_rope_known_answer():
    # test_nn_modules.cpp:201-240 (head_dim 4, theta 1e4, positions 0/1 and offset 3)
    x = np.array([[[1, 2, 10, 20]], [[3, 4, 30, 40]]], np.float32)
    y = O.rope(x, 10000.0, 0)
    assert np.allclose(y[0, 0], [1, 2, 10, 20], atol=1e-5)
    a0, a1 = 1.0, 0.01
    exp = [3 * math.cos(a0) - 30 * math.sin(a0), 4 * math.cos(a1) - 40 * math.sin(a1),
           3 * math.sin(a0) + 30 * math.cos(a0), 4 * math.sin(a1) + 40 * math.cos(a1)]
    assert np.allclose(y[1, 0], exp, atol=1e-5)
    z = O.rope(np.array([[[5, 6, 7, 8]]], np.float32), 10000.0, 3)
    assert near(z[0, 0, 0], 5 * math.cos(3.0) - 7 * math.sin(3.0))
    assert near(z[0, 0, 1], 6 * math.cos(0.03) - 8 * math.sin(0.03))


def test_gqa_known_answer():
    # test_nn_modules.cpp:252-300: 2 query heads share 1 kv head, causal.
    q = np.array([[[1, 0], [0, 1]], [[0.5, 0.5], [1, 0]]], np.float32)
    k = np.array([[[1, 0]], [[0, 1]]], np.float32)
    v = np.array([[[10, 1]], [[2, 20]]], np.float32)
    out = O.attention(q, k, v, 0)
    assert np.allclose(out[0, 0], [10, 1]) and np.allclose(out[0, 1], [10, 1])
    sc = 1 / math.sqrt(2.0)

    def mix(s0, s1):
        m = max(s0, s1)
        w0, w1 = math.exp(s0 - m), math.exp(s1 - m)
        return [(w0 * 10 + w1 * 2) / (w0 + w1), (w0 * 1 + w1 * 20) / (w0 + w1)]

    assert np.allclose(out[1, 0], mix(0.5 * sc, 0.5 * sc), atol=1e-5)
    assert np.allclose(out[1, 1], mix(1 * sc, 0.0), atol=1e-5)


def test_sampler_first_strict_maximum():
    # test_nn_modules.cpp:619-628 and the tie rule of sampler.cpp:38-45 (top_k = 1)
    assert O.argmax(np.array([0.1, 3.0, 2.0], np.float32)) == 1
    assert O.argmax(np.array([1.0, 5.0, 5.0, 2.0], np.float32)) == 1


def test_fp16_decode_is_exact():
    vals = np.array([0.0, -0.0, 1.0, -2.5, 65504.0, 6.1035156e-05, 5.96e-08, np.inf], np.float16)
    for v in vals:
        got = O.oracle_lib().oracle_f16_to_f32(int(v.view(np.uint16)))
        assert got == float(v) or (math.isinf(got) and math.isinf(float(v)))


def _block_bundle(tmp_path, **kw):
    cfg = tiny_config(hidden_size=256, intermediate_size=256, num_hidden_layers=1, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=64, vocab_size=40, **kw)
    return write_synthetic_bundle(tmp_path, cfg, seed=3)


def test_cached_equals_uncached(tmp_path):
    # test_nn_modules.cpp:535-590: prefix-cached logits equal the full forward's.
    p = _block_bundle(tmp_path)
    full = O.OracleModel(p, 16).forward([3, 7, 11], 0)
    m = O.OracleModel(p, 16)
    m.forward([3, 7], 0)
    cached = m.forward([11], 2)
    assert np.allclose(cached[0], full[2], atol=1e-5)


def test_embedding_rejects_out_of_range(tmp_path):
    # test_nn_modules.cpp:82-86 / embedding.cpp:66-68
    m = O.OracleModel(_block_bundle(tmp_path), 8)
    with pytest.raises(ValueError, match="out of range"):
        m.forward([40], 0)


# ---- 2. bit-exact against the reference build ---------------------------------
CASES = {
    "tied_f16_gqa2": (tiny_config(), "float16"),
    "untied_f16": (tiny_config(tie_word_embeddings=False), "float16"),
    "bf16_gqa4_d128": (tiny_config(num_attention_heads=8, num_key_value_heads=2, head_dim=128,
                                   hidden_size=256, num_hidden_layers=1), "bfloat16"),
    "f32_mha": (tiny_config(num_attention_heads=4, num_key_value_heads=4, num_hidden_layers=1), "float32"),
}


@pytest.mark.skipif(not O.ref_available(), reason="reference build oracle/_ref absent")
@pytest.mark.parametrize("case", sorted(CASES))
def test_oracle_bit_exact_vs_reference(case, tmp_path):
    cfg, dtype = CASES[case]
    p = write_synthetic_bundle(tmp_path / case, cfg, seed=11, dtype=dtype)
    om, rm = O.OracleModel(p, 64), O.RefModel(p, 64)
    ids = np.random.default_rng(5).integers(0, cfg["vocab_size"], 9).astype(np.int32)
    a, b = om.forward(ids, 0), rm.forward(ids, 0)
    assert np.array_equal(a, b)
    for step, tok in enumerate([int(ids[-1]), 17, 3]):
        a, b = om.forward([tok], 9 + step), rm.forward([tok], 9 + step)
        assert np.array_equal(a, b)
        assert O.argmax(a[0]) == rm.sample(b[0])
    for layer in range(cfg["num_hidden_layers"]):
        ka, va = om.kv_read(layer, 0, 12)
        kb, vb = rm.kv_read(layer, 0, 12)
        assert np.array_equal(ka, kb) and np.array_equal(va, vb)


@pytest.mark.skipif(not O.ref_available(), reason="reference build oracle/_ref absent")
def test_module_ops_bit_exact_vs_reference():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((3, 64), dtype=np.float32)
    w = rng.standard_normal((40, 64), dtype=np.float32) * np.float32(0.1)
    assert np.array_equal(O.linear(x, w), O.ref_linear(x, w))
    nw = rng.standard_normal(64, dtype=np.float32)
    assert np.array_equal(O.rmsnorm(x, nw), O.ref_rmsnorm(x, nw))
    r = rng.standard_normal((5, 3, 128), dtype=np.float32)
    assert np.array_equal(O.rope(r, 1e6, 37), O.ref_rope(r, 1e6, 37))
    q = rng.standard_normal((4, 4, 64), dtype=np.float32)
    k = rng.standard_normal((9, 2, 64), dtype=np.float32)
    v = rng.standard_normal((9, 2, 64), dtype=np.float32)
    assert np.array_equal(O.attention(q, k, v, 5), O.ref_attention(q, k, v, 5))


@pytest.mark.skipif(not O.ref_available(), reason="reference build oracle/_ref absent")
@pytest.mark.parametrize("theta", [1e4, 1e6])
@pytest.mark.parametrize("offset", [0, 2047, 4095, 40959])
def test_rope_bit_exact_at_long_positions(theta, offset):
    """The positions the long-context benchmarks reach (4K contexts, the 40,960-row RoPE table):
    the oracle's angles (double precision, as the reference) stay bit-exact there too."""
    r = np.random.default_rng(offset).standard_normal((3, 2, 128), dtype=np.float32)
    assert np.array_equal(O.rope(r, theta, offset), O.ref_rope(r, theta, offset))


@pytest.mark.skipif(not O.ref_available(), reason="reference build oracle/_ref absent")
@pytest.mark.parametrize("keys,prefix", [(300, 290), (1030, 1000), (64, 0)])
def test_attention_bit_exact_long_context(keys, prefix):
    rng = np.random.default_rng(keys)
    T = keys - prefix if prefix else 8
    q = rng.standard_normal((T, 8, 128), dtype=np.float32)
    k = rng.standard_normal((keys, 2, 128), dtype=np.float32)
    v = rng.standard_normal((keys, 2, 128), dtype=np.float32)
    assert np.array_equal(O.attention(q, k, v, prefix), O.ref_attention(q, k, v, prefix))


# ---- 3. golden vectors produced by the reference -------------------------------
def _golden_files():
    return sorted(GOLDEN.glob("tiny_*.npz"))


@pytest.mark.parametrize("path", _golden_files(), ids=lambda p: p.stem)
def test_oracle_matches_reference_golden(path, tmp_path):
    from tests.golden.make_golden import bundle_for, load_fixture
    fx = load_fixture(path)
    p = bundle_for(fx, tmp_path)
    m = O.OracleModel(p, 64)
    pre = m.forward(fx["prompt"], 0)
    assert np.array_equal(pre, fx["prefill_logits"])
    pos = len(fx["prompt"])
    for i, tok in enumerate(fx["decode_inputs"]):
        lg = m.forward([int(tok)], pos + i)
        assert np.array_equal(lg[0], fx["decode_logits"][i])
    k, v = m.kv_read(0, 0, pos + len(fx["decode_inputs"]))
    assert np.array_equal(k, fx["kv_k_layer0"]) and np.array_equal(v, fx["kv_v_layer0"])
