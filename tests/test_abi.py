"""CPU-side checks of the C-ABI library and the bundle format (no kernels run)."""
import ctypes
import json

import numpy as np
import pytest

from soc_b200 import bundle as B
from soc_b200 import runtime as R


def test_library_exports_every_declared_symbol():
    names = R.header_functions()
    assert len(names) >= 19
    lib = ctypes.CDLL(str(R.LIB_PATH))
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # the ctypes front end binds exactly the declared set
    assert set(names) == set(R._SIGNATURES)


def test_open_without_device_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    with pytest.raises(R.SocError) as e:
        R.Context(0)
    assert e.value.code in (R.ERR_CUDA, R.ERR_INVALID)


def test_null_arguments_rejected():
    lib = R.lib()
    assert lib.soc_b200_open(0, None) == R.ERR_INVALID
    assert b"null" in lib.soc_b200_last_error()
    assert lib.soc_b200_kv_length(None, 0) == R.ERR_INVALID
    assert lib.soc_b200_prefill(None, None, 0, None, 0, None, None) == R.ERR_INVALID


def test_bundle_layout_matches_reference_format(tmp_path):
    p = B.write_synthetic_bundle(tmp_path / "b", B.tiny_config(), seed=1)
    m = json.loads(p.read_text())
    assert m["format"] == "soc.cpp.llm_export" and m["format_version"] == 2
    assert m["tokenizer_runtime_file"] == "tokenizer/tokenizer_runtime.json"
    names = [t["name"] for t in m["tensors"]]
    assert names[0] == "model.embed_tokens.weight" and "model.norm.weight" in names
    for t in m["tensors"]:
        assert set(t) >= {"name", "file", "dtype", "shape", "byte_size", "source_shard"}
        assert (p.parent / t["file"]).stat().st_size == t["byte_size"]
        assert t["byte_size"] == int(np.prod(t["shape"])) * 2
    tok = json.loads((p.parent / m["tokenizer_runtime_file"]).read_text())
    assert tok["format"] == "soc.cpp.tokenizer_runtime" and tok["template_runtime"]["type"] == "qwen3"


def test_synthetic_values_are_seeded(tmp_path):
    a = B.write_synthetic_bundle(tmp_path / "a", B.tiny_config(), seed=4)
    b = B.write_synthetic_bundle(tmp_path / "b", B.tiny_config(), seed=4)
    ma, mb = B.read_manifest(a), B.read_manifest(b)
    for name in ["model.embed_tokens.weight", "model.layers.1.mlp.down_proj.weight"]:
        assert np.array_equal(B.load_tensor(ma, name), B.load_tensor(mb, name))
    w = np.asarray(B.load_tensor(ma, "model.layers.0.self_attn.q_proj.weight"), dtype=np.float32)
    assert abs(float(w.std()) - 0.02) < 2e-3
    assert np.all(np.asarray(B.load_tensor(ma, "model.layers.0.input_layernorm.weight")) == 1)


@pytest.mark.parametrize("fmt", ["int8_g64", "int4_g32"])
def test_groupwise_quantisation_roundtrip(fmt):
    rng = np.random.default_rng(0)
    w = rng.standard_normal((64, 256), dtype=np.float32) * np.float32(0.02)
    q, s = B.quantize_groupwise(w, fmt)
    g = B.QUANT_GROUP[fmt]
    assert s.dtype == np.float16 and s.shape == (64, 256 // g)
    dq = B.dequantize_groupwise(q, s, fmt)
    # error of symmetric rounding: at most half a step per group (plus fp16 scale rounding)
    step = np.repeat(s.astype(np.float32), g, axis=1)
    assert np.all(np.abs(dq - w) <= 0.5 * step * 1.01 + 1e-7)
    qmax = 127 if fmt == "int8_g64" else 7
    if fmt == "int8_g64":
        assert q.dtype == np.int8 and int(np.abs(q).max()) <= qmax
    else:
        assert q.dtype == np.uint8 and q.shape == (64, 128)
        lo = (q & 0xF).astype(np.int16)
        lo = np.where(lo > 7, lo - 16, lo)
        assert int(np.abs(lo).max()) <= qmax


def test_reference_loads_synthetic_bundle(tmp_path):
    from oracle import oracle as O
    if not O.ref_available():
        pytest.skip("reference build absent")
    p = B.write_synthetic_bundle(tmp_path / "b", B.tiny_config(num_hidden_layers=1), seed=2)
    rm = O.RefModel(p, 8)
    assert rm.forward([1, 2], 0).shape == (2, 1000)


@pytest.mark.parametrize("fmt", ["int8_g64", "int4_g32"])
def test_quantize_bundle_exporter(tmp_path, fmt):
    """The exporter option re-encodes only the block linears; the oracle decodes them."""
    from oracle import oracle as O
    src = B.write_synthetic_bundle(tmp_path / "src", B.tiny_config(), seed=2)
    out = B.quantize_bundle(src, tmp_path / fmt, fmt)
    ms, mq = B.read_manifest(src), B.read_manifest(out)
    assert mq["export_dtype"] == fmt
    recs = {r["name"]: r for r in mq["tensors"]}
    name = "model.layers.1.mlp.down_proj.weight"
    assert recs[name]["dtype"] == fmt and recs[name + ".scales"]["dtype"] == "float16"
    assert recs["model.embed_tokens.weight"]["dtype"] == "float16"
    w = np.asarray(B.load_tensor(ms, name), dtype=np.float32)
    q, s = B.quantize_groupwise(w, fmt)
    assert np.array_equal(np.asarray(B.load_tensor(mq, name)), q)
    assert np.array_equal(np.asarray(B.load_tensor(mq, name + ".scales")), s)
    lg = O.OracleModel(out, 32).forward([5, 6, 7], 0, last_only=True)[0]
    assert np.isfinite(lg).all()
