"""The header-only C++ mirror (include/soc_b200_generation_context.hpp) compiles against the
C ABI and behaves like the Python front end on the host (no GPU): tokenizer wrappers,
generation options, and GenerationContext's argument checks with the reference's messages."""
import shutil
import subprocess

import pytest

from soc_b200 import runtime as R
from soc_b200.bundle import tiny_config, write_synthetic_bundle

from .conftest import ROOT


@pytest.fixture(scope="module")
def mirror(tmp_path_factory):
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    out = tmp_path_factory.mktemp("mirror") / "mirror_check"
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", str(ROOT / "include"), str(ROOT / "tests/cpp/mirror_check.cpp"),
                    "-o", str(out), "-L", str(ROOT / "soc_b200"), "-lsoc_b200",
                    f"-Wl,-rpath,{ROOT / 'soc_b200'}"], check=True)
    return out


def test_cpp_mirror_matches_python(mirror, tmp_path):
    p = write_synthetic_bundle(tmp_path / "b", tiny_config(), seed=1, tokenizer="bpe")
    text = "Hello there, the quick brown fox 42!"
    res = subprocess.run([str(mirror), str(p), text], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stderr
    got = dict(line.split(": ", 1) for line in res.stdout.splitlines())
    tok = R.Tokenizer(p)
    assert got["ids"] == str(tok.encode(text))
    assert got["roundtrip"] == "ok"
    assert got["prompt_ids"] == str(tok.encode(tok.chat_prompt([("user", text)], True, False, "Be brief.")))
    assert got["options"] == "32 1 1 -1 4352"
    assert got["decode_error"] == f"unknown token id: {1 << 30}"
    assert got["prefill_empty"] == "0 GenerationContext prefill requires at least one token"
    assert got["decode_unprefilled"] == "0 GenerationContext decode requires a prefilled KV cache"
    assert got["generate_too_long"] == "0 GenerationContext sequence length would exceed max_sequence_length"
    assert got["generate_null"] == "0 GenerationContext generate requires a non-null generated_token_ids output"
    tok.free()
