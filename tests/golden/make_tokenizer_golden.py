"""Generates tests/golden/string_pipeline.json from the REFERENCE's own tokenizer, chat
template and sampler (oracle/_ref/libsocref.so, ``make -C oracle ref``).

    python tests/golden/make_tokenizer_golden.py

The tokenizer documents are not stored: each case records how the synthetic writer makes
it (``soc_b200.bundle.synthetic_bpe_tokenizer`` with the options of ``tests/test_tokenizer.py``)
and a SHA-256 of its JSON, which the test regenerates and checks before comparing.
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from oracle import oracle as O  # noqa: E402
from soc_b200.bundle import bytes_to_unicode, synthetic_bpe_tokenizer  # noqa: E402

OUT = HERE / "string_pipeline.json"

TEXTS = ["", "Hello world!", "  leading spaces and\ttabs\nnewlines\r\n  trailing  ",
         "numbers 2048 151936 3.14159 and x2y3z", "UTF-8: café naïve 東京 🙂 ñ",
         "special tokens inside<|im_end|>text<|endoftext|>and<think>more</think>",
         "the quick brown fox jumps over the lazy dog, then the fox sleeps."]
VARIANTS = ["plain", "prefix_space", "no_regex", "subword_prefix_unk", "word_suffix"]
CHATS = [
    ([["user", "Say hello."], ["assistant", "Hello."], ["user", "Now think first."]], True, True, ""),
    ([["user", "Say hello."]], True, False, "Custom system prompt."),
    ([["system", "Only facts."], ["user", "2+2?"]], False, True, ""),
]


def tokenizer_doc(variant: str) -> dict:
    """The synthetic tokenizer (vocab 2000) with one of the reference's optional behaviours on."""
    doc = synthetic_bpe_tokenizer(2000)
    if variant == "prefix_space":
        doc["pre_tokenizer"]["byte_level"]["add_prefix_space"] = True
    elif variant == "no_regex":
        doc["pre_tokenizer"]["byte_level"]["use_regex"] = False
    elif variant == "subword_prefix_unk":
        doc["bpe_model"]["continuing_subword_prefix"] = "##"
        doc["bpe_model"]["unk_token"] = "<|endoftext|>"
    elif variant == "word_suffix":
        doc["bpe_model"]["end_of_word_suffix"] = "</w>"
        doc["decoder"]["bpe"] = {"enabled": True, "suffix": "</w>"}
        b2u = bytes_to_unicode()
        first = 256 + len(doc["bpe_model"]["merges"])
        for b in range(256):
            doc["vocab"][first + b]["token"] = b2u[b] + "</w>"
    elif variant != "plain":
        raise ValueError(variant)
    return doc


def doc_digest(doc: dict) -> str:
    return hashlib.sha256(json.dumps(doc, sort_keys=True).encode()).hexdigest()


def sampler_rows():
    rng = np.random.default_rng(31)
    rows = [(rng.standard_normal(997) * 3).astype(np.float32) for _ in range(6)]
    rows[0][[5, 400]] = rows[0].max() + 1.0  # a repeated maximum
    return rows


def main() -> None:
    import tempfile
    if not O.ref_available():
        raise SystemExit("build the reference first: make -C oracle ref")
    out = {"tokenizers": [], "chats": [], "sampler": []}
    with tempfile.TemporaryDirectory() as d:
        for v in VARIANTS:
            doc = tokenizer_doc(v)
            p = Path(d) / f"{v}.json"
            p.write_text(json.dumps(doc))
            ref = O.RefTokenizer(p)
            cases = []
            for text in TEXTS:
                try:
                    ids = ref.encode(text)
                    cases.append({"text": text, "ids": ids, "decoded_hex": ref.decode_bytes(ids).hex()})
                except ValueError as e:
                    cases.append({"text": text, "error": str(e)})
            out["tokenizers"].append({"variant": v, "sha256": doc_digest(doc), "cases": cases})
            if v == "plain":
                for msgs, gen, think, system in CHATS:
                    out["chats"].append({"messages": msgs, "add_generation_prompt": gen, "enable_thinking": think,
                                         "system_prompt": system,
                                         "prompt": ref.chat_prompt_messages([tuple(m) for m in msgs], gen, think,
                                                                            system)})
            ref.free()
    for row in sampler_rows():
        for t in (1.0, 0.7, 2.5):
            for k in (1, 4):
                s = row / np.float32(t)
                out["sampler"].append({"temperature": t, "top_k": k, "pick": O.ref_sample(row, t, k),
                                       "maximum_repeats": int((s == s.max()).sum())})
    OUT.write_text(json.dumps(out, indent=1, ensure_ascii=False) + "\n")
    print(OUT)


if __name__ == "__main__":
    main()
