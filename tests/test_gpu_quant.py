"""Group-quantised linears on the B200 path (int8 group 64 / int4 group 32, fp16 scales).

The oracle dequantises every quantised record to float32 (``float(q) * float(s)``), so the
GPU result is compared with the reference arithmetic on the dequantised weights: logits
within 2e-2 max-abs and identical greedy ids.  The kernel-level cases compare against an
fp64 product with the dequantised matrix.
"""
import numpy as np
import pytest

from oracle import oracle as O
from soc_b200 import runtime as R
from soc_b200.bundle import QWEN3_0_6B, dequantize_groupwise, quantize_bundle, quantize_groupwise, tiny_config

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-2
FORMATS = {"int8_g64": R.WEIGHTS_INT8_G64, "int4_g32": R.WEIGHTS_INT4_G32}


@pytest.mark.parametrize("rows", [1, 4, 16, 64])
@pytest.mark.parametrize("shape", [(2048, 1024), (1024, 2048), (6144, 1024), (1024, 3072), (151936, 1024)],
                         ids=["q", "o", "gate_up", "down", "lm_head"])
@pytest.mark.parametrize("fmt", sorted(FORMATS))
def test_quant_linear_kernel_against_fp64(gpu_ctx, fmt, rows, shape):
    import torch
    out_f, in_f = shape
    if out_f > 100000 and rows > 4:
        pytest.skip("lm_head shape covered at rows 1 and 4")
    rng = np.random.default_rng(out_f + rows)
    w = rng.standard_normal((out_f, in_f), dtype=np.float32) * np.float32(0.02)
    q, s = quantize_groupwise(w, fmt)
    wd = dequantize_groupwise(q, s, fmt).astype(np.float64)
    x = rng.standard_normal((rows, in_f), dtype=np.float32)
    ref = x.astype(np.float64) @ wd.T
    qt = torch.from_numpy(np.ascontiguousarray(q).view(np.uint8)).cuda()
    st = torch.from_numpy(np.ascontiguousarray(s)).cuda()
    xt = torch.from_numpy(x).cuda()
    y = torch.empty(rows, out_f, device="cuda")
    gpu_ctx.linear(FORMATS[fmt], qt.data_ptr(), st.data_ptr(), out_f, in_f, xt.data_ptr(), rows, y.data_ptr(),
                   torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    err = np.abs(y.cpu().numpy().astype(np.float64) - ref).max()
    assert err <= 1e-4 * (in_f ** 0.5), err


@pytest.mark.parametrize("rows", [2, 3, 5, 13, 37])
@pytest.mark.parametrize("shape", [(1000, 384), (1000, 320), (40, 256)], ids=["ragged_tile", "off_chunk", "tiny"])
@pytest.mark.parametrize("fmt", ["fp16", "int8_g64", "int4_g32"])
def test_small_batch_linear_ragged_shapes(gpu_ctx, fmt, rows, shape):
    """Row counts that leave row blocks part-empty, output counts that leave the last 16-row tile
    part-empty, and an in_features (320) that is not a whole number of int4 chunks (128): the
    tensor-core small-batch kernel or the CUDA-core GEMV, whichever takes the shape, against an
    fp64 product."""
    import torch
    out_f, in_f = shape
    rng = np.random.default_rng(out_f * 7 + in_f + rows)
    w = rng.standard_normal((out_f, in_f), dtype=np.float32) * np.float32(0.02)
    x = (rng.standard_normal((rows, in_f), dtype=np.float32) * np.float32(30.0)).astype(np.float32)
    if fmt == "fp16":
        wh = w.astype(np.float16)
        wd, code, sc = wh.astype(np.float64), R.WEIGHTS_F16, None
        qt = torch.from_numpy(wh).cuda()
    else:
        q, s = quantize_groupwise(w, fmt)
        wd, code = dequantize_groupwise(q, s, fmt).astype(np.float64), FORMATS[fmt]
        qt = torch.from_numpy(np.ascontiguousarray(q).view(np.uint8)).cuda()
        sc = torch.from_numpy(np.ascontiguousarray(s)).cuda()
    ref = x.astype(np.float64) @ wd.T
    xt = torch.from_numpy(x).cuda()
    y = torch.full((rows, out_f), float("nan"), device="cuda")
    gpu_ctx.linear(code, qt.data_ptr(), sc.data_ptr() if sc is not None else None, out_f, in_f, xt.data_ptr(),
                   rows, y.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    err = np.abs(y.cpu().numpy().astype(np.float64) - ref).max()
    assert err <= 1e-4 * 30.0 * (in_f ** 0.5), err


def test_quant_linear_rejects_missing_scales(gpu_ctx):
    import torch
    w = torch.zeros(64, 256, dtype=torch.uint8, device="cuda")
    x = torch.zeros(1, 256, device="cuda")
    y = torch.empty(1, 64, device="cuda")
    with pytest.raises(R.SocError):
        gpu_ctx.linear(R.WEIGHTS_INT8_G64, w.data_ptr(), None, 64, 256, x.data_ptr(), 1, y.data_ptr())


CASES = {
    "tiny": tiny_config(),
    "qwen06_shape_2layer": dict(QWEN3_0_6B, num_hidden_layers=2),
}


@pytest.fixture(scope="module")
def qmodels(gpu_ctx, make_bundle):
    cache = {}

    def get(case, quant):
        if (case, quant) not in cache:
            p = make_bundle(f"q_{case}_{quant}", CASES[case], seed=11, dtype="float16", quant=quant)
            cache[(case, quant)] = (p, R.Model(gpu_ctx, p))
        return cache[(case, quant)]

    yield get
    for _, m in cache.values():
        m.free()


@pytest.mark.parametrize("quant", sorted(FORMATS))
@pytest.mark.parametrize("case", sorted(CASES))
def test_quantized_bundle_logits_match_oracle(qmodels, case, quant):
    p, m = qmodels(case, quant)
    assert m.info.weight_format == FORMATS[quant]
    cfg = CASES[case]
    kv = R.KVCache(m, 1, 256)
    om = O.OracleModel(p, 256)
    prompt = np.random.default_rng(3).integers(0, cfg["vocab_size"], 11).astype(np.int32)
    lg, nid = m.forward_logits_cached(kv, 0, prompt)
    ref = om.forward(prompt, 0, last_only=True)[0]
    assert np.abs(lg - ref).max() <= LOGIT_TOL
    assert nid == O.argmax(ref)
    tok, pos = nid, len(prompt)
    for _ in range(5):
        lg, nxt = m.decode(kv, [0], [tok])
        ref = om.forward([tok], pos, last_only=True)[0]
        assert np.abs(lg[0] - ref).max() <= LOGIT_TOL
        assert int(nxt[0]) == O.argmax(ref)
        tok, pos = int(nxt[0]), pos + 1
    kv.free()


@pytest.mark.parametrize("quant", sorted(FORMATS))
def test_quantized_generate_matches_oracle_greedy(qmodels, quant):
    p, m = qmodels("qwen06_shape_2layer", quant)
    prompt = np.random.default_rng(4).integers(0, QWEN3_0_6B["vocab_size"], 8).astype(np.int32)
    toks, _ = O.OracleModel(p, 128).generate(prompt, 10)
    kv = R.KVCache(m, 1, 128)
    assert m.generate(kv, 0, prompt, 10) == toks
    kv.free()


@pytest.mark.parametrize("quant", sorted(FORMATS))
def test_load_time_quantisation_equals_exported_bundle(gpu_ctx, make_bundle, tmp_path, quant):
    """A float bundle loaded with weight_format=int8/int4 gives the same device weights as
    the exporter's quantised bundle: logits are bit-identical."""
    src = make_bundle("q_src_f16", tiny_config(), seed=5, dtype="float16")
    exported = quantize_bundle(src, tmp_path / quant, quant)
    a = R.Model(gpu_ctx, src, weight_format=FORMATS[quant])
    b = R.Model(gpu_ctx, exported)
    prompt = np.arange(1, 10, dtype=np.int32) * 37
    ka, kb = R.KVCache(a, 1, 64), R.KVCache(b, 1, 64)
    la, ia = a.forward_logits_cached(ka, 0, prompt)
    lb, ib = b.forward_logits_cached(kb, 0, prompt)
    assert ia == ib
    assert np.array_equal(la, lb)
    for m_ in (ka, kb):
        m_.free()
    a.free()
    b.free()


@pytest.mark.parametrize("quant", sorted(FORMATS))
def test_quantized_prefill_tensor_core_path(qmodels, quant):
    """40 prompt rows (>= 32): the quantised linears run as an fp16 expansion of each
    matrix feeding the tensor-core GEMM.  Logits vs the oracle, then greedy decode."""
    p, m = qmodels("qwen06_shape_2layer", quant)
    prompt = np.random.default_rng(31).integers(0, QWEN3_0_6B["vocab_size"], 40).astype(np.int32)
    om = O.OracleModel(p, 128)
    ref = om.forward(prompt, 0, last_only=True)[0]
    kv = R.KVCache(m, 1, 128)
    lg, nid = m.forward_logits_cached(kv, 0, prompt)
    assert np.abs(lg - ref).max() <= LOGIT_TOL
    assert nid == O.argmax(ref)
    kv.free()
    toks, _ = O.OracleModel(p, 128).generate(prompt, 8)
    kv = R.KVCache(m, 1, 128)
    assert m.generate(kv, 0, prompt, 8) == toks
    kv.free()
