"""soc_b200_cli against the reference's own command-line runner (Mac/cpu/main.cpp compiled
unchanged into oracle/_ref/soc_ref_cli): argument handling and error lines on the CPU, and
the full output (serialized prompt, prompt ids, generated ids and text) on the GPU."""
import subprocess

import pytest

from soc_b200.bundle import tiny_config, write_synthetic_bundle

from .conftest import ROOT

OURS = ROOT / "soc_b200" / "soc_b200_cli"
REF = ROOT / "oracle" / "_ref" / "soc_ref_cli"


def _run(exe, *args, timeout=600):
    if not exe.exists():
        pytest.skip(f"{exe.name} not built")
    p = subprocess.run([str(exe), *map(str, args)], capture_output=True, timeout=timeout)
    # generated_text may hold any bytes: surrogateescape keeps them distinct and comparable
    return p.returncode, p.stdout.decode("utf-8", "surrogateescape"), p.stderr.decode("utf-8", "surrogateescape")


@pytest.fixture(scope="module")
def bpe_bundle(tmp_path_factory):
    """Weights spread wide enough (std 0.1) that greedy generations vary; on this bundle the
    smallest top-2 logit gap over the cases below is 0.04, well above the device path's
    logit error."""
    return write_synthetic_bundle(tmp_path_factory.mktemp("cli") / "b", tiny_config(), seed=3, tokenizer="bpe",
                                  std=0.1)


def test_help_lists_the_reference_options():
    rc, _, err = _run(OURS, "--help")
    rc_r, _, err_r = _run(REF, "--help")
    assert rc == rc_r == 0
    ours = err.splitlines()[1:]
    for line in err_r.splitlines()[1:]:
        assert line in ours


@pytest.mark.parametrize("args", [
    [],
    ["--prompt", "hi"],
    ["--manifest", "m.json"],
    ["--manifest", "m.json", "--prompt", "hi", "--bogus"],
    ["--manifest", "m.json", "--prompt"],
    ["--manifest", "m.json", "--prompt", "hi", "--max-new-tokens", "many"],
    ["--manifest", "m.json", "--prompt", "hi", "--eos-token-id", "x"],
    ["--manifest", "m.json", "--prompt", "hi", "--temperature", "warm"],
], ids=range(8))
def test_argument_errors_match_reference(args):
    rc, out, err = _run(OURS, *args)
    rc_r, out_r, err_r = _run(REF, *args)
    assert rc == rc_r == 1
    assert out == out_r == ""
    assert err.splitlines()[0] == err_r.splitlines()[0]


def test_bad_tokenizer_is_reported_before_the_device_is_touched(tmp_path, bpe_bundle):
    import json
    import shutil
    d = tmp_path / "b"
    shutil.copytree(bpe_bundle.parent, d)
    tok = d / "tokenizer" / "tokenizer_runtime.json"
    doc = json.loads(tok.read_text())
    doc["template_runtime"]["type"] = "llama"
    tok.write_text(json.dumps(doc))
    rc, _, err = _run(OURS, "--manifest", d / "manifest.json", "--prompt", "hi")
    rc_r, _, err_r = _run(REF, "--manifest", d / "manifest.json", "--prompt", "hi")
    assert rc == rc_r == 1
    assert err.splitlines()[0] == err_r.splitlines()[0] == \
        "runtime error: tokenizer template runtime type must be qwen3"


CASES = [
    ["--prompt", "Hello world, the quick brown fox", "--max-new-tokens", "8"],
    ["--prompt", "Tell me a story.", "--max-new-tokens", "6", "--apply-chat-template"],
    ["--prompt", "Think less", "--max-new-tokens", "5", "--apply-chat-template", "--disable-thinking",
     "--system-prompt", "Be brief."],
    ["--prompt", "numbers 12 and 345", "--max-new-tokens", "0"],
    ["--prompt", "cold", "--max-new-tokens", "6", "--temperature", "0.5", "--top-k", "4"],
]


@pytest.mark.gpu
@pytest.mark.parametrize("args", CASES, ids=range(len(CASES)))
def test_cli_output_matches_reference(bpe_bundle, args):
    rc, out, err = _run(OURS, "--manifest", bpe_bundle, *args)
    assert rc == 0, err
    rc_r, out_r, err_r = _run(REF, "--manifest", bpe_bundle, *args)
    assert rc_r == 0, err_r
    assert out == out_r


@pytest.mark.gpu
def test_cli_eos_and_capacity_match_reference(bpe_bundle):
    rc, out, _ = _run(OURS, "--manifest", bpe_bundle, "--prompt", "abc", "--max-new-tokens", "4")
    assert rc == 0
    ids = out.split("generated_token_ids: [")[1].split("]")[0].split(", ")
    eos = ids[1]
    args = ["--manifest", bpe_bundle, "--prompt", "abc", "--max-new-tokens", "4", "--eos-token-id", eos]
    rc, out, _ = _run(OURS, *args)
    rc_r, out_r, _ = _run(REF, *args)
    assert rc == rc_r == 0 and out == out_r
    assert f"generated_token_ids: [{ids[0]}, {eos}]" in out or ids[0] == eos
    # The prompt fills the cache: the reference fails at the first write past it.
    n_prompt = len(out.split("prompt_token_ids: [")[1].split("]")[0].split(", "))
    for max_seq, max_new in [(n_prompt + 1, 2), (n_prompt + 1, 3), (n_prompt - 1, 1)]:
        args = ["--manifest", bpe_bundle, "--prompt", "abc", "--max-new-tokens", max_new, "--max-seq-len", max_seq]
        rc, out, err = _run(OURS, *args)
        rc_r, out_r, err_r = _run(REF, *args)
        assert rc == rc_r, (max_seq, max_new, err, err_r)
        assert out == out_r
        if rc:
            assert err.splitlines()[0] == err_r.splitlines()[0]


@pytest.mark.parametrize("fault", ["missing_tensor", "byte_size", "config", "tokenizer_vocab"])
def test_broken_bundle_reported_like_reference(bpe_bundle, tmp_path, fault):
    """Broken bundles fail in both runners with the same first line, before any device work
    (so this runs without a GPU)."""
    import json
    import shutil
    d = tmp_path / "b"
    shutil.copytree(bpe_bundle.parent, d)
    mp = d / "manifest.json"
    m = json.loads(mp.read_text())
    if fault == "missing_tensor":
        m["tensors"] = [t for t in m["tensors"] if not t["name"].endswith("layers.1.mlp.gate_proj.weight")]
    elif fault == "byte_size":
        next(t for t in m["tensors"] if t["name"] == "model.norm.weight")["byte_size"] = 3
    elif fault == "config":
        m["config"]["num_key_value_heads"] = 3
    else:
        tp = d / m["tokenizer_runtime_file"]
        doc = json.loads(tp.read_text())
        doc["vocab_size"] = 4096
        tp.write_text(json.dumps(doc))
    mp.write_text(json.dumps(m))
    rc, out, err = _run(OURS, "--manifest", mp, "--prompt", "hi")
    rc_r, out_r, err_r = _run(REF, "--manifest", mp, "--prompt", "hi")
    assert rc == rc_r == 1 and out == out_r == ""
    assert err.splitlines()[0] == err_r.splitlines()[0]
