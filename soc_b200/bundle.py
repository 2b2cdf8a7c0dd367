"""Bundle I/O in the reference's on-disk format (``soc.cpp.llm_export`` v2).

A bundle is a directory holding

* ``manifest.json`` -- ``format``, ``format_version``, ``export_dtype``, the HF
  ``config`` object, ``generation_config``, ``tokenizer_runtime_file`` and one
  record per tensor ``{name, file, dtype, shape, byte_size, source_shard}``
  (reference writer: ``LLM_interpreter/convert_py_to_cpp.py:507-551``; reader:
  ``Mac/cpu/src/runtime_assets.cpp:138-168``);
* ``weights/<sanitised name>.bin`` -- one raw little-endian array per tensor
  (``convert_py_to_cpp.py:478-504``, file stems from ``sanitize_tensor_name``
  at ``convert_py_to_cpp.py:123-135``);
* ``tokenizer/tokenizer_runtime.json`` (``convert_py_to_cpp.py:445-475``).

The reference exporter needs a Hugging Face snapshot and the network; this
module instead writes *synthetic* bundles of the same layout with seeded
random weights, so the B200 runtime and the reference CPU runtime can load the
very same files.

Quantised formats (this library's own extension; the reference has no
group-wise layout): a linear weight record with ``dtype`` ``int8_g64`` or
``int4_g32`` holds the packed integers, and a companion record named
``<name>.scales`` (``float16``, shape ``[out, in / group]``) holds one scale per
group.  ``int8_g64``: ``s = fp16(max|w_g| / 127)``, ``q = clamp(round(w / s),
-127, 127)``, one signed byte per weight.  ``int4_g32``: ``s = fp16(max|w_g| /
7)``, ``q = clamp(round(w / s), -7, 7)``, two weights per byte, low nibble first
(two's complement nibbles).  Dequantised value: ``float(q) * float(s)``.
"""
from __future__ import annotations

import json
import os
import re
from pathlib import Path
from typing import Any

import numpy as np

FORMAT = "soc.cpp.llm_export"
FORMAT_VERSION = 2

# Qwen3-0.6B architecture (config 0/2/3 of the benchmark set).
QWEN3_0_6B: dict[str, Any] = {
    "architectures": ["Qwen3ForCausalLM"],
    "model_type": "qwen3",
    "hidden_size": 1024,
    "intermediate_size": 3072,
    "num_hidden_layers": 28,
    "num_attention_heads": 16,
    "num_key_value_heads": 8,
    "head_dim": 128,
    "rms_norm_eps": 1e-6,
    "rope_theta": 1000000.0,
    "tie_word_embeddings": True,
    "torch_dtype": "float16",
    "vocab_size": 151936,
    "max_position_embeddings": 40960,
    "hidden_act": "silu",
}

# Qwen3-8B architecture (config 4): untied lm_head.
QWEN3_8B: dict[str, Any] = dict(
    QWEN3_0_6B,
    hidden_size=4096,
    intermediate_size=12288,
    num_hidden_layers=36,
    num_attention_heads=32,
    num_key_value_heads=8,
    tie_word_embeddings=False,
    torch_dtype="bfloat16",
)

DTYPE_NP = {
    "float32": np.float32,
    "float16": np.float16,
    "bfloat16": np.uint16,  # raw bits
    "int8_g64": np.int8,
    "int4_g32": np.uint8,
}

QUANT_GROUP = {"int8_g64": 64, "int4_g32": 32}


def tiny_config(**overrides: Any) -> dict[str, Any]:
    """A small Qwen3-shaped config for fast CPU-oracle parity cases."""
    cfg = dict(
        QWEN3_0_6B,
        hidden_size=256,
        intermediate_size=512,
        num_hidden_layers=2,
        num_attention_heads=4,
        num_key_value_heads=2,
        head_dim=64,
        vocab_size=1000,
    )
    cfg.update(overrides)
    return cfg


def sanitize_tensor_name(name: str, used: set[str]) -> str:
    """File stem for a tensor name, as the reference exporter derives it."""
    stem = re.sub(r"[^a-zA-Z0-9._-]+", "_", name).strip("._-") or "tensor"
    candidate, suffix = stem, 1
    while candidate in used:
        suffix += 1
        candidate = f"{stem}_{suffix}"
    used.add(candidate)
    return candidate


def layer_tensor_names(layer: int) -> list[str]:
    """Per-layer HF tensor names in the order the synthetic generator draws them."""
    p = f"model.layers.{layer}."
    return [
        p + "input_layernorm.weight",
        p + "self_attn.q_proj.weight",
        p + "self_attn.k_proj.weight",
        p + "self_attn.v_proj.weight",
        p + "self_attn.o_proj.weight",
        p + "self_attn.q_norm.weight",
        p + "self_attn.k_norm.weight",
        p + "post_attention_layernorm.weight",
        p + "mlp.gate_proj.weight",
        p + "mlp.up_proj.weight",
        p + "mlp.down_proj.weight",
    ]


def tensor_shapes(cfg: dict[str, Any]) -> list[tuple[str, tuple[int, ...]]]:
    """(name, shape) of every tensor of a Qwen3 checkpoint, in draw order.

    Shapes follow ``QwenModelLoader::LoadModel`` (``Mac/cpu/src/qwen_model_loader.cpp:35-93``).
    """
    H, I = cfg["hidden_size"], cfg["intermediate_size"]
    D = cfg["head_dim"]
    q = cfg["num_attention_heads"] * D
    kv = cfg["num_key_value_heads"] * D
    V = cfg["vocab_size"]
    out: list[tuple[str, tuple[int, ...]]] = [("model.embed_tokens.weight", (V, H))]
    for layer in range(cfg["num_hidden_layers"]):
        n = layer_tensor_names(layer)
        out += [
            (n[0], (H,)),
            (n[1], (q, H)),
            (n[2], (kv, H)),
            (n[3], (kv, H)),
            (n[4], (H, q)),
            (n[5], (D,)),
            (n[6], (D,)),
            (n[7], (H,)),
            (n[8], (I, H)),
            (n[9], (I, H)),
            (n[10], (H, I)),
        ]
    out.append(("model.norm.weight", (H,)))
    if not cfg["tie_word_embeddings"]:
        out.append(("lm_head.weight", (V, H)))
    return out


def is_norm(name: str) -> bool:
    return name.endswith("norm.weight") or name.endswith("layernorm.weight")


def is_quantizable(name: str) -> bool:
    """Linear projections inside the blocks (q/k/v/o/gate/up/down)."""
    return name.endswith("_proj.weight")


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 bit pattern (``dtype.cpp:158-163``)."""
    bits = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    bias = np.uint32(0x7FFF) + ((bits >> np.uint32(16)) & np.uint32(1))
    return ((bits + bias) >> np.uint32(16)).astype(np.uint16)


def bf16_bits_to_f32(a: np.ndarray) -> np.ndarray:
    return (np.asarray(a, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def quantize_groupwise(w: np.ndarray, fmt: str) -> tuple[np.ndarray, np.ndarray]:
    """Symmetric group-wise quantisation of a float ``[out, in]`` matrix.

    Extends the per-column int8 prototype of the reference
    (``Mac/cpu/header/matrix_ops.h:42-73``: ``scale = max|w| / 127``,
    ``round``, clamp to ``[-127, 127]``) to groups along ``in``.
    Returns (packed integers, fp16 scales ``[out, in / group]``).
    """
    g = QUANT_GROUP[fmt]
    qmax = 127.0 if fmt == "int8_g64" else 7.0
    out_f, in_f = w.shape
    if in_f % g:
        raise ValueError(f"in_features {in_f} is not a multiple of group {g}")
    wg = w.astype(np.float32).reshape(out_f, in_f // g, g)
    scale = (np.abs(wg).max(axis=2) / np.float32(qmax)).astype(np.float16)
    s32 = scale.astype(np.float32)
    safe = np.where(s32 == 0, np.float32(1), s32)
    q = np.clip(np.rint(wg / safe[..., None]), -qmax, qmax).astype(np.int8)
    q = np.where(s32[..., None] == 0, np.int8(0), q).reshape(out_f, in_f)
    if fmt == "int8_g64":
        return q, scale
    nib = (q.astype(np.int16) & 0xF).astype(np.uint8)
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)
    return packed, scale


def dequantize_groupwise(q: np.ndarray, scale: np.ndarray, fmt: str) -> np.ndarray:
    """float32 ``[out, in]`` = ``float(q) * float(scale)`` (same arithmetic as the GPU)."""
    g = QUANT_GROUP[fmt]
    if fmt == "int8_g64":
        qi = q.astype(np.float32)
    else:
        lo = (q & 0xF).astype(np.int8)
        hi = ((q >> 4) & 0xF).astype(np.int8)
        lo = np.where(lo > 7, lo - 16, lo)
        hi = np.where(hi > 7, hi - 16, hi)
        qi = np.empty((q.shape[0], q.shape[1] * 2), dtype=np.float32)
        qi[:, 0::2] = lo
        qi[:, 1::2] = hi
    out_f, in_f = qi.shape
    s = scale.astype(np.float32).reshape(out_f, in_f // g, 1)
    return (qi.reshape(out_f, in_f // g, g) * s).reshape(out_f, in_f)


# Text the synthetic BPE tokenizer learns its merges from (own words; any text works).
BPE_TRAINING_TEXT = (
    "The quick brown fox jumps over the lazy dog. A tokenizer splits text into pieces, and the model "
    "reads those pieces as numbers. Byte pairs that appear together often are merged first: th, he, in, "
    "er, an, the, and, ing, tion. Numbers like 2048, 151936 and 3.14159 stay as digit runs; punctuation "
    "such as !?;:,.() stays apart from words. Hello world! Hello again, world. Decoding joins the pieces "
    "back into the same bytes, including UTF-8 text like café, naïve, 東京 and emoji 🙂.\n\tTabs and "
    "  double  spaces are kept. Qwen3 models chat with im_start and im_end markers around each turn."
)


def bytes_to_unicode() -> list[str]:
    """The byte-level BPE alphabet (GPT-2's published mapping): printable Latin-1 bytes stand
    for themselves, the other bytes for code points 256, 257, ... in byte order."""
    keep = list(range(ord("!"), ord("~") + 1)) + list(range(ord("\u00a1"), ord("\u00ac") + 1)) + \
        list(range(ord("\u00ae"), ord("\u00ff") + 1))
    table, extra = {}, 0
    for b in range(256):
        if b in keep:
            table[b] = chr(b)
        else:
            table[b] = chr(256 + extra)
            extra += 1
    return [table[b] for b in range(256)]


def _pretokenize(text: str) -> list[bytes]:
    """Whitespace run + one run of letters, digits or other non-space bytes (the reference's
    byte-level pre-tokenizer rule, ``tokenizer_runtime.cpp`` PreTokenizeText), on bytes."""
    data, out, i = text.encode("utf-8"), [], 0
    isspace = lambda c: c in b" \t\n\r\x0b\x0c"
    isalpha = lambda c: (65 <= c <= 90) or (97 <= c <= 122)
    isdigit = lambda c: 48 <= c <= 57
    while i < len(data):
        start = i
        while i < len(data) and isspace(data[i]):
            i += 1
        if i == len(data):
            out.append(data[start:])
            break
        if isalpha(data[i]):
            while i < len(data) and isalpha(data[i]):
                i += 1
        elif isdigit(data[i]):
            while i < len(data) and isdigit(data[i]):
                i += 1
        else:
            while i < len(data) and not isspace(data[i]) and not isalpha(data[i]) and not isdigit(data[i]):
                i += 1
        out.append(data[start:i])
    return out


def synthetic_bpe_tokenizer(vocab_size: int, n_merges: int = 300, text: str = BPE_TRAINING_TEXT) -> dict[str, Any]:
    """A ``soc.cpp.tokenizer_runtime`` v1 byte-level BPE document: 256 byte symbols (ids 0-255),
    up to ``n_merges`` merges learned greedily from ``text`` (most frequent adjacent pair, ties
    to the smaller pair), merged symbols as ids 256.., filler symbols of printable bytes up to the added
    tokens, and the chat / control tokens as added tokens at the top of the id range."""
    b2u = bytes_to_unicode()
    words: dict[tuple[str, ...], int] = {}
    for piece in _pretokenize(text):
        key = tuple(b2u[b] for b in piece)
        words[key] = words.get(key, 0) + 1
    merges: list[tuple[str, str]] = []
    vocab = list(b2u)
    specials = ["<|endoftext|>", "<|im_start|>", "<|im_end|>", "<think>", "</think>"]
    limit = vocab_size - len(specials) - 256
    while len(merges) < min(n_merges, limit):
        pairs: dict[tuple[str, str], int] = {}
        for w, c in words.items():
            for a, b in zip(w, w[1:]):
                pairs[(a, b)] = pairs.get((a, b), 0) + c
        if not pairs:
            break
        best = min(pairs, key=lambda pr: (-pairs[pr], pr))
        if pairs[best] < 2:
            break
        merges.append(best)
        vocab.append(best[0] + best[1])
        new_words: dict[tuple[str, ...], int] = {}
        for w, c in words.items():
            out, i = [], 0
            while i < len(w):
                if i + 1 < len(w) and (w[i], w[i + 1]) == best:
                    out.append(w[i] + w[i + 1])
                    i += 2
                else:
                    out.append(w[i])
                    i += 1
            new_words[tuple(out)] = new_words.get(tuple(out), 0) + c
        words = new_words
    # Fill the rest of the id range below the added tokens with multi-byte symbols no merge
    # produces, so that every id a model of this vocab_size can emit decodes to bytes.
    have = set(vocab)
    k = 94
    while len(vocab) < vocab_size - len(specials):
        digits, n = [], k  # k in base 94 over the printable bytes '!'..'~' (two or more symbols)
        while n:
            digits.append(b2u[0x21 + n % 94])
            n //= 94
        tok = "".join(reversed(digits))
        k += 1
        if tok not in have:
            have.add(tok)
            vocab.append(tok)
    doc = _tokenizer_runtime(vocab_size)
    doc["tokenizer_class"] = "SyntheticByteLevelBPE"
    doc["vocab"] = [{"id": i, "token": t} for i, t in enumerate(vocab)]
    doc["bpe_model"] = {"type": "bpe", "unk_token": None, "continuing_subword_prefix": None,
                        "end_of_word_suffix": None, "merges": [{"left": a, "right": b} for a, b in merges]}
    doc["pre_tokenizer"] = {"type": "ByteLevel", "byte_level": {"enabled": True, "add_prefix_space": False,
                                                                 "use_regex": True}}
    doc["decoder"] = {"type": "ByteLevel", "byte_level": {"enabled": True, "add_prefix_space": False,
                                                           "trim_offsets": False, "use_regex": True,
                                                           "byte_to_unicode": b2u}}
    return doc


def _tokenizer_runtime(vocab_size: int) -> dict[str, Any]:
    """A minimal ``soc.cpp.tokenizer_runtime`` v1 document that passes the
    reference validator (``Mac/cpu/src/startup_validator.cpp:25-75``).

    The synthetic bundles carry random weights, so the vocabulary is only a
    byte-level placeholder; chat-boundary tokens sit at the top of the id range.
    """
    byte_tokens = [{"id": i, "token": f"<0x{i:02X}>"} for i in range(min(256, vocab_size - 5))]
    specials = ["<|endoftext|>", "<|im_start|>", "<|im_end|>", "<think>", "</think>"]
    added = [
        {"id": vocab_size - len(specials) + k, "content": s, "special": True,
         "single_word": False, "lstrip": False, "rstrip": False, "normalized": False}
        for k, s in enumerate(specials)
    ]
    return {
        "format": "soc.cpp.tokenizer_runtime",
        "format_version": 1,
        "tokenizer_class": "SyntheticByteTokenizer",
        "vocab_size": vocab_size,
        "model_max_length": 40960,
        "special_tokens_map": {"eos_token": "<|im_end|>", "pad_token": "<|endoftext|>"},
        "special_token_ids": {"eos_token": vocab_size - 3, "pad_token": vocab_size - 5},
        "added_tokens": added,
        "vocab": byte_tokens,
        "chat_template": None,
        "template_runtime": {
            "type": "qwen3",
            "im_start": "<|im_start|>",
            "im_end": "<|im_end|>",
            "think_start": "<think>",
            "think_end": "</think>",
            "default_system_prompt": "You are a helpful assistant.",
        },
        "bpe_model": None,
        "pre_tokenizer": None,
        "decoder": None,
        "copied_files": [],
    }


def write_synthetic_bundle(
    out_dir: str | os.PathLike,
    cfg: dict[str, Any],
    seed: int = 0,
    dtype: str = "float16",
    quant: str | None = None,
    std: float = 0.02,
    model_id: str = "synthetic/qwen3",
    torch_device: str | None = None,
    tokenizer: str = "placeholder",
) -> Path:
    """Write a seeded random Qwen3 bundle in the reference format.

    Values: every non-norm tensor ~ N(0, std) drawn with
    ``numpy.random.default_rng(seed).standard_normal(shape, float32) * std`` in
    ``tensor_shapes`` order; every norm weight is 1.0.  ``dtype`` is the stored
    float type (``float16``/``bfloat16``/``float32``).  ``quant`` (``int8_g64``
    or ``int4_g32``) stores the block linears group-quantised instead, with
    embeddings, norms and the lm_head kept in ``dtype``.
    ``torch_device`` (e.g. ``"cuda"``) draws the values with
    ``torch.randn(shape, generator=torch.Generator(device).manual_seed(seed))`` on that
    device instead (same order, same std), for multi-billion-parameter bundles.
    ``tokenizer``: ``"placeholder"`` (chat and control tokens only) or ``"bpe"``
    (``synthetic_bpe_tokenizer``, a byte-level BPE over the config's vocab_size).
    Returns the manifest path.
    """
    out = Path(out_dir)
    (out / "weights").mkdir(parents=True, exist_ok=True)
    (out / "tokenizer").mkdir(parents=True, exist_ok=True)
    rng = np.random.default_rng(seed)
    tgen = None
    if torch_device is not None:
        import torch
        tgen = torch.Generator(device=torch_device).manual_seed(seed)
    used: set[str] = set()
    records = []

    def emit(name: str, arr: np.ndarray, dt: str) -> None:
        stem = sanitize_tensor_name(name, used)
        rel = f"weights/{stem}.bin"
        data = np.ascontiguousarray(arr)
        data.tofile(out / rel)
        records.append({
            "name": name, "file": rel, "dtype": dt, "shape": list(arr.shape) if dt != "int4_g32" else [arr.shape[0], arr.shape[1] * 2],
            "byte_size": int(data.nbytes), "source_shard": "synthetic.safetensors",
        })

    for name, shape in tensor_shapes(cfg):
        if is_norm(name):
            w = np.ones(shape, dtype=np.float32)
        elif tgen is not None:
            import torch
            t = torch.randn(tuple(shape), generator=tgen, device=torch_device, dtype=torch.float32) * std
            if dtype == "bfloat16" and quant is None:
                emit(name, t.to(torch.bfloat16).view(torch.int16).cpu().numpy().view(np.uint16), "bfloat16")
                continue
            w = t.cpu().numpy()
        else:
            w = rng.standard_normal(shape, dtype=np.float32)
            w *= np.float32(std)
        if quant is not None and is_quantizable(name):
            q, s = quantize_groupwise(w, quant)
            emit(name, q, quant)
            emit(name + ".scales", s, "float16")
        elif dtype == "float16":
            emit(name, w.astype(np.float16), "float16")
        elif dtype == "bfloat16":
            emit(name, f32_to_bf16_bits(w), "bfloat16")
        elif dtype == "float32":
            emit(name, w, "float32")
        else:
            raise ValueError(f"unsupported bundle dtype {dtype}")
        del w

    if tokenizer == "bpe":
        tok = synthetic_bpe_tokenizer(cfg["vocab_size"])
    elif tokenizer == "placeholder":
        tok = _tokenizer_runtime(cfg["vocab_size"])
    else:
        raise ValueError(f"unknown synthetic tokenizer {tokenizer}")
    (out / "tokenizer" / "tokenizer_runtime.json").write_text(json.dumps(tok, indent=1))
    manifest = {
        "format": FORMAT,
        "format_version": FORMAT_VERSION,
        "model_id": model_id,
        "source_dir": "synthetic",
        "export_dtype": quant or dtype,
        "tensor_count": len(records),
        "config": cfg,
        "generation_config": {"max_new_tokens": 32, "temperature": 1.0, "top_k": 1,
                              "eos_token_id": -1, "max_length": 4352},
        "source_index": None,
        "tokenizer_runtime_file": "tokenizer/tokenizer_runtime.json",
        "tensors": records,
        "tokenizer": {"runtime_file": "tokenizer_runtime.json"},
        "synthetic": {"seed": seed, "std": std, "dtype": dtype, "quant": quant,
                      "generator": "numpy.default_rng" if torch_device is None else f"torch.randn({torch_device})"},
    }
    path = out / "manifest.json"
    path.write_text(json.dumps(manifest, indent=1))
    return path


def quantize_bundle(src_manifest: str | os.PathLike, out_dir: str | os.PathLike, quant: str) -> Path:
    """Export an existing float bundle with its block linears group-quantised.

    The exporter option of the quantised layout: every ``*_proj.weight`` record is
    decoded to float32 (``float16``/``bfloat16``/``float32``), quantised with
    ``quantize_groupwise`` and written as a ``quant`` record plus its ``.scales``
    record; every other record and the tokenizer asset are copied unchanged.
    Returns the new manifest path.
    """
    if quant not in QUANT_GROUP:
        raise ValueError(f"unknown quantisation {quant}")
    src = read_manifest(src_manifest)
    out = Path(out_dir)
    (out / "weights").mkdir(parents=True, exist_ok=True)
    (out / "tokenizer").mkdir(parents=True, exist_ok=True)
    used: set[str] = set()
    records = []

    def emit(name: str, data: np.ndarray, dt: str, shape: list[int]) -> None:
        rel = f"weights/{sanitize_tensor_name(name, used)}.bin"
        data = np.ascontiguousarray(data)
        data.tofile(out / rel)
        records.append({"name": name, "file": rel, "dtype": dt, "shape": shape, "byte_size": int(data.nbytes),
                        "source_shard": "quantized.safetensors"})

    for rec in src["tensors"]:
        name = rec["name"]
        arr = load_tensor(src, name)
        if is_quantizable(name) and rec["dtype"] in ("float16", "bfloat16", "float32"):
            w = bf16_bits_to_f32(arr) if rec["dtype"] == "bfloat16" else np.asarray(arr, dtype=np.float32)
            q, s = quantize_groupwise(w, quant)
            emit(name, q, quant, list(rec["shape"]))
            emit(name + ".scales", s, "float16", list(s.shape))
        else:
            emit(name, np.asarray(arr), rec["dtype"], list(rec["shape"]))
    tok_src = Path(src["_dir"]) / src["tokenizer_runtime_file"]
    (out / "tokenizer" / "tokenizer_runtime.json").write_bytes(tok_src.read_bytes())
    manifest = {k: v for k, v in src.items() if not k.startswith("_")}
    manifest.update({"export_dtype": quant, "tensor_count": len(records), "tensors": records,
                     "tokenizer_runtime_file": "tokenizer/tokenizer_runtime.json"})
    path = out / "manifest.json"
    path.write_text(json.dumps(manifest, indent=1))
    return path


def read_manifest(path: str | os.PathLike) -> dict[str, Any]:
    """Parse ``manifest.json`` and resolve tensor files against its directory."""
    p = Path(path)
    m = json.loads(p.read_text())
    base = p.parent
    for rec in m["tensors"]:
        rec["path"] = str((base / rec["file"]).resolve())
    m["_dir"] = str(base.resolve())
    return m


def load_tensor(manifest: dict[str, Any], name: str) -> np.ndarray:
    """Memory-map one tensor of a parsed manifest as its stored numpy dtype."""
    for rec in manifest["tensors"]:
        if rec["name"] == name:
            dt = DTYPE_NP[rec["dtype"]]
            shape = list(rec["shape"])
            if rec["dtype"] == "int4_g32":
                shape[-1] //= 2
            return np.memmap(rec["path"], dtype=dt, mode="r", shape=tuple(shape))
    raise KeyError(f"missing tensor in manifest: {name}")


def cached_bundle(name: str, cfg: dict[str, Any], seed: int, dtype: str = "float16",
                  quant: str | None = None, root: str | None = None, torch_device: str | None = None) -> Path:
    """Write a synthetic bundle once under ``root`` (default: a temp dir) and reuse it."""
    root = root or os.environ.get("SOC_B200_BUNDLE_DIR", os.path.join(os.environ.get("TMPDIR", "/tmp"), "soc_b200_bundles"))
    out = Path(root) / name
    manifest = out / "manifest.json"
    stamp = out / ".complete"
    if manifest.exists() and stamp.exists():
        return manifest
    tmp = Path(root) / (name + f".tmp{os.getpid()}")
    write_synthetic_bundle(tmp, cfg, seed=seed, dtype=dtype, quant=quant, torch_device=torch_device)
    (tmp / ".complete").write_text("ok")
    out.parent.mkdir(parents=True, exist_ok=True)
    if out.exists():
        import shutil
        shutil.rmtree(out)
    os.replace(tmp, out)
    return manifest
