"""String pipeline (host only): the library's tokenizer and chat template against the
reference's TokenizerRuntime / Qwen3TemplateBuilder compiled from its own sources
(oracle/_ref).  Token ids, decoded bytes and prompt text must be identical."""
import json

import pytest

from oracle import oracle as O
from soc_b200 import runtime as R
from soc_b200.bundle import synthetic_bpe_tokenizer, tiny_config, write_synthetic_bundle

TEXTS = [
    "",
    "Hello world!",
    "Hello again, world. The quick brown fox jumps over the lazy dog.",
    "  leading spaces and\ttabs\nnewlines\r\n  trailing  ",
    "numbers 2048 151936 3.14159 and x2y3z",
    "punctuation !?;:,.() [] {} <> -- == ++",
    "UTF-8: café naïve 東京 🙂 ñ",
    "<|im_start|>user\nHi there<|im_end|>\n<|im_start|>assistant\n<think>\n",
    "special tokens inside<|im_end|>text<|endoftext|>and<think>more</think>",
    "thinking andand the then there these",
    "a",
    " ",
    "\x00\x01 control bytes \x7f",
]


@pytest.fixture(scope="module")
def bpe_path(tmp_path_factory):
    p = tmp_path_factory.mktemp("tok") / "tokenizer_runtime.json"
    p.write_text(json.dumps(synthetic_bpe_tokenizer(1000)))
    return p


@pytest.fixture(scope="module")
def byte_bundle(tmp_path_factory):
    return write_synthetic_bundle(tmp_path_factory.mktemp("tb") / "b", tiny_config(), seed=1)


def _pair(path):
    if not O.ref_available():
        pytest.skip("reference library not built (oracle/_ref)")
    return R.Tokenizer(path), O.RefTokenizer(path)


@pytest.mark.parametrize("text", TEXTS, ids=range(len(TEXTS)))
def test_bpe_encode_decode_matches_reference(bpe_path, text):
    ours, ref = _pair(bpe_path)
    ids = ours.encode(text)
    assert ids == ref.encode(text)
    assert ours.decode_bytes(ids) == ref.decode_bytes(ids) == text.encode("utf-8")
    ours.free()
    ref.free()


def test_bpe_merges_are_used(bpe_path):
    ours, _ = _pair(bpe_path)
    text = "the then there and"
    assert len(ours.encode(text)) < len(text.encode())
    ours.free()


@pytest.mark.parametrize("text", ["<|im_start|>", "plain <|im_end|>", "x"], ids=range(3))
def test_placeholder_tokenizer_matches_reference(byte_bundle, text):
    """The placeholder tokenizer of the synthetic bundles (no BPE model): longest-match over
    its tokens, and the reference's error text where nothing matches."""
    import json as _j
    path = byte_bundle.parent / _j.loads(byte_bundle.read_text())["tokenizer_runtime_file"]
    ours, ref = _pair(path)
    try:
        expect = ref.encode(text)
    except ValueError as e:
        with pytest.raises(R.SocError) as got:
            ours.encode(text)
        assert str(e) in str(got.value)
    else:
        assert ours.encode(text) == expect
    ours.free()
    ref.free()


@pytest.mark.parametrize("gen,think,system", [(True, True, ""), (True, False, ""), (False, False, "Be terse."),
                                              (True, True, "Du bist hilfreich.")])
def test_chat_prompt_matches_reference(bpe_path, gen, think, system):
    ours, ref = _pair(bpe_path)
    for user in ("Hello!", "Explain 2+2.\nThen stop.", ""):
        assert ours.chat_prompt([("user", user)], gen, think, system) == ref.chat_prompt(user, gen, think, system)
    ours.free()
    ref.free()


def test_chat_prompt_keeps_a_given_system_message(bpe_path):
    ours, _ = _pair(bpe_path)
    p = ours.chat_prompt([("system", "S"), ("user", "U")], True, False)
    assert p == "<|im_start|>system\nS<|im_end|>\n<|im_start|>user\nU<|im_end|>\n<|im_start|>assistant\n"
    ours.free()


def test_tokenizer_errors(tmp_path, bpe_path):
    doc = json.loads(bpe_path.read_text())
    doc["format_version"] = 2
    bad = tmp_path / "bad.json"
    bad.write_text(json.dumps(doc))
    with pytest.raises(R.SocError, match="format_version must be 1"):
        R.Tokenizer(bad)
    with pytest.raises(R.SocError, match="failed to open file"):
        R.Tokenizer(tmp_path / "missing.json")
    ours = R.Tokenizer(bpe_path)
    with pytest.raises(R.SocError, match="unknown token id"):
        ours.decode([10 ** 6])
    ours.free()


def test_generation_options_from_manifest(tmp_path, byte_bundle):
    o = R.GenerationOptions.from_manifest(byte_bundle)
    doc = json.loads(byte_bundle.read_text())
    g = doc["generation_config"]
    assert (o.max_new_tokens, o.temperature, o.top_k, o.eos_token_id, o.max_sequence_length) == \
        (g["max_new_tokens"], g["temperature"], g["top_k"], g["eos_token_id"], g["max_length"])
    # defaults when absent; an eos list takes its first id (runtime_pipeline.cpp ReadOptionalInt)
    doc["generation_config"] = {"eos_token_id": [151645, 151643], "temperature": 0.7}
    p = tmp_path / "manifest.json"
    p.write_text(json.dumps(doc))
    o = R.GenerationOptions.from_manifest(p)
    assert (o.max_new_tokens, o.top_k, o.eos_token_id, o.max_sequence_length) == (32, 1, 151645, 256)
    assert abs(o.temperature - 0.7) < 1e-7
    del doc["generation_config"]
    p.write_text(json.dumps(doc))
    o = R.GenerationOptions.from_manifest(p)
    assert (o.max_new_tokens, o.temperature, o.top_k, o.eos_token_id, o.max_sequence_length) == (32, 1.0, 1, -1, 256)
    o.temperature = 0.0
    with pytest.raises(R.SocError, match="sampler temperature must be positive"):
        o.check()
    o.temperature, o.top_k = 1.0, 0
    with pytest.raises(R.SocError, match="sampler top_k must be positive"):
        o.check()
    assert R.manifest_tokenizer_path(byte_bundle) == str(byte_bundle.parent / doc["tokenizer_runtime_file"])


def test_tokenizer_vocab_checked_against_model(bpe_path):
    t = R.Tokenizer(bpe_path)
    t.check_model(1000)
    t.check_model(4096)
    with pytest.raises(R.SocError, match="must not exceed qwen3 config vocab_size"):
        t.check_model(999)
    t.free()


def _variant(name):
    """Tokenizer documents that switch on the options the synthetic tokenizer leaves off."""
    from soc_b200.bundle import bytes_to_unicode
    doc = synthetic_bpe_tokenizer(2000)
    if name == "prefix_space":
        doc["pre_tokenizer"]["byte_level"]["add_prefix_space"] = True
    elif name == "no_regex":
        doc["pre_tokenizer"]["byte_level"]["use_regex"] = False
    elif name == "subword_prefix_unk":
        doc["bpe_model"]["continuing_subword_prefix"] = "##"
        doc["bpe_model"]["unk_token"] = "<|endoftext|>"
    elif name == "word_suffix":
        doc["bpe_model"]["end_of_word_suffix"] = "</w>"
        doc["decoder"]["bpe"] = {"enabled": True, "suffix": "</w>"}
        b2u = bytes_to_unicode()
        first = 256 + len(doc["bpe_model"]["merges"])
        for b in range(256):  # replace filler ids by the suffixed byte symbols
            doc["vocab"][first + b]["token"] = b2u[b] + "</w>"
    elif name == "no_byte_level":
        doc["pre_tokenizer"] = None
        doc["decoder"] = None
    return doc


VARIANT_TEXTS = ["Hello world, the quick brown fox!", "  two  spaces", "abc", "x", "end.", "café 12",
                 "<|im_start|>user\nhi<|im_end|>", ""]


@pytest.mark.parametrize("name", ["prefix_space", "no_regex", "subword_prefix_unk", "word_suffix", "no_byte_level"])
def test_tokenizer_options_match_reference(tmp_path, name):
    p = tmp_path / "tok.json"
    p.write_text(json.dumps(_variant(name)))
    ours, ref = _pair(p)
    for text in VARIANT_TEXTS:
        try:
            expect = ref.encode(text)
        except ValueError as e:
            with pytest.raises(R.SocError) as got:
                ours.encode(text)
            assert str(e) in str(got.value), (name, text)
            continue
        ids = ours.encode(text)
        assert ids == expect, (name, text)
        assert ours.decode_bytes(ids) == ref.decode_bytes(ids), (name, text)
    ours.free()
    ref.free()


def test_missing_unk_token_rejected_like_reference(tmp_path):
    doc = synthetic_bpe_tokenizer(1000)
    doc["bpe_model"]["unk_token"] = "<nope>"
    p = tmp_path / "tok.json"
    p.write_text(json.dumps(doc))
    if not O.ref_available():
        pytest.skip("reference library not built (oracle/_ref)")
    with pytest.raises(ValueError) as ref_err:
        O.RefTokenizer(p)
    with pytest.raises(R.SocError) as ours_err:
        R.Tokenizer(p)
    assert str(ref_err.value) in str(ours_err.value)


@pytest.mark.parametrize("gen,think,system", [(True, True, ""), (True, False, "Custom system prompt."),
                                              (False, True, "")])
def test_multi_turn_chat_prompt_matches_reference(bpe_path, gen, think, system):
    """The reference's own template test conversation (user, assistant, user), and one that
    brings its own system message."""
    ours, ref = _pair(bpe_path)
    convs = [[("user", "Say hello."), ("assistant", "Hello."), ("user", "Now think first.")],
             [("system", "Only facts."), ("user", "2+2?"), ("assistant", "4"), ("user", "And 3+3?")],
             []]
    for msgs in convs:
        assert ours.chat_prompt(msgs, gen, think, system) == ref.chat_prompt_messages(msgs, gen, think, system)
    ours.free()
    ref.free()
