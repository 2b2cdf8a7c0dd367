"""Bundle validation on the host (soc_b200_validate_bundle) against the reference's own
RuntimePipeline::LoadBundle (oracle/_ref) on the same broken bundles: the first problem each
finds, and its message, must be the same.  No GPU needed."""
import json
import shutil

import pytest

from oracle import oracle as O
from soc_b200 import runtime as R
from soc_b200.bundle import quantize_bundle, tiny_config, write_synthetic_bundle


@pytest.fixture(scope="module")
def good(tmp_path_factory):
    root = tmp_path_factory.mktemp("val")
    return {
        "tied": write_synthetic_bundle(root / "tied", tiny_config(), seed=4, tokenizer="bpe"),
        "untied": write_synthetic_bundle(root / "untied", tiny_config(tie_word_embeddings=False), seed=5,
                                         dtype="bfloat16"),
    }


def _copy(src, dst):
    shutil.copytree(src.parent, dst)
    return dst / "manifest.json"


def _edit_manifest(path, fn):
    m = json.loads(path.read_text())
    fn(m)
    path.write_text(json.dumps(m))


def _record(m, suffix):
    return next(t for t in m["tensors"] if t["name"].endswith(suffix))


def _drop(suffix):
    return lambda m: m.update(tensors=[t for t in m["tensors"] if not t["name"].endswith(suffix)])


def _set_config(**kw):
    return lambda m: m["config"].update(kw)


def _set_shape(suffix, shape):
    return lambda m: _record(m, suffix).update(shape=shape)


def _truncate(suffix):
    def f(path):
        m = json.loads(path.read_text())
        with open(path.parent / _record(m, suffix)["file"], "r+b") as fh:
            fh.truncate(10)
    return f


def _tokenizer(fn):
    def f(path):
        m = json.loads(path.read_text())
        tp = path.parent / m["tokenizer_runtime_file"]
        doc = json.loads(tp.read_text())
        fn(doc)
        tp.write_text(json.dumps(doc))
    return f


MANIFEST_EDITS = {
    "format": lambda m: m.update(format="other"),
    "format_version": lambda m: m.update(format_version=1),
    "config_not_object": lambda m: m.update(config=[1, 2]),
    "no_tensors": lambda m: m.update(tensors=[]),
    "model_type": _set_config(model_type="llama"),
    "heads_not_divisible": _set_config(num_key_value_heads=3),
    "zero_vocab": _set_config(vocab_size=0),
    "missing_k_norm": _drop("layers.1.self_attn.k_norm.weight"),
    "missing_final_norm": _drop("model.norm.weight"),
    "missing_down": _drop("layers.0.mlp.down_proj.weight"),
    "shape_q": _set_shape("layers.0.self_attn.q_proj.weight", [128, 256]),
    "shape_q_consistent": lambda m: _record(m, "layers.0.self_attn.q_proj.weight").update(shape=[128, 256],
                                                                                          byte_size=128 * 256 * 2),
    "shape_norm_consistent": lambda m: _record(m, "layers.1.self_attn.q_norm.weight").update(shape=[32],
                                                                                             byte_size=32 * 2),
    "shape_embed": _set_shape("model.embed_tokens.weight", [999, 256]),
    "byte_size": lambda m: _record(m, "layers.1.mlp.up_proj.weight").update(byte_size=123),
    "int_dtype": lambda m: _record(m, "layers.0.self_attn.q_proj.weight").update(dtype="int32"),
}
FILE_EDITS = {
    "truncated_up": _truncate("layers.1.mlp.up_proj.weight"),
    "tokenizer_vocab_too_big": _tokenizer(lambda d: d.update(vocab_size=5000)),
    "tokenizer_version": _tokenizer(lambda d: d.update(format_version=3)),
    "tokenizer_template": _tokenizer(lambda d: d["template_runtime"].update(type="chatml")),
}


def _compare(path):
    if not O.ref_available():
        pytest.skip("reference library not built (oracle/_ref)")
    expect = O.ref_load_bundle(path)
    if expect is None:
        R.validate_bundle(path)
        return None
    with pytest.raises(R.SocError) as got:
        R.validate_bundle(path)
    assert str(got.value).endswith(expect), (str(got.value), expect)
    return expect


@pytest.mark.parametrize("kind", ["tied", "untied"])
def test_good_bundles_pass(good, kind):
    assert _compare(good[kind]) is None


def test_quantised_bundle_passes(good, tmp_path):
    p = quantize_bundle(good["tied"], tmp_path / "q8", "int8_g64")
    R.validate_bundle(p)  # the reference does not read group-quantised records
    m = json.loads(p.read_text())
    m["tensors"] = [t for t in m["tensors"] if not t["name"].endswith("layers.0.mlp.up_proj.weight.scales")]
    p.write_text(json.dumps(m))
    with pytest.raises(R.SocError, match="missing tensor in manifest: model.layers.0.mlp.up_proj.weight.scales"):
        R.validate_bundle(p)


@pytest.mark.parametrize("name", sorted(MANIFEST_EDITS))
def test_manifest_faults_match_reference(good, tmp_path, name):
    p = _copy(good["tied"], tmp_path / "b")
    _edit_manifest(p, MANIFEST_EDITS[name])
    assert _compare(p) is not None


@pytest.mark.parametrize("name", sorted(FILE_EDITS))
def test_file_faults_match_reference(good, tmp_path, name):
    p = _copy(good["tied"], tmp_path / "b")
    FILE_EDITS[name](p)
    assert _compare(p) is not None


def test_untied_lm_head_checked(good, tmp_path):
    p = _copy(good["untied"], tmp_path / "b")
    _edit_manifest(p, _drop("lm_head.weight"))
    assert _compare(p) == "missing tensor in manifest: lm_head.weight"


def test_empty_tokenizer_reference(good, tmp_path):
    """A manifest whose tokenizer_runtime_file is empty: the reference resolves it to the
    manifest's own directory and fails parsing that as JSON, before its own "must reference"
    check can run; this library reports that check's message directly."""
    p = _copy(good["tied"], tmp_path / "b")
    _edit_manifest(p, lambda m: m.update(tokenizer_runtime_file=""))
    if O.ref_available():
        assert O.ref_load_bundle(p) is not None
    with pytest.raises(R.SocError, match="manifest must reference tokenizer_runtime_file"):
        R.validate_bundle(p)
