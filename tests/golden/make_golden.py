"""Generates the golden vectors under tests/golden/ from the REFERENCE CPU runtime.

    python tests/golden/make_golden.py            # tiny fixtures (seconds)
    python tests/golden/make_golden.py --config0  # Qwen3-0.6B config-0 greedy run (minutes)

Runs the reference's own sources compiled unchanged (oracle/_ref/libsocref.so,
``make -C oracle ref``) on seeded synthetic bundles.  The bundles are not
committed: each fixture records the writer's (config, seed, dtype) and a
SHA-256 of the weight files, and ``bundle_for`` regenerates and verifies them.
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

from soc_b200.bundle import QWEN3_0_6B, tiny_config, write_synthetic_bundle  # noqa: E402

TINY = {
    "tiny_tied_f16": dict(cfg=tiny_config(), dtype="float16", seed=21, prompt_len=7, steps=5),
    "tiny_untied_bf16_d128": dict(cfg=tiny_config(tie_word_embeddings=False, num_attention_heads=8,
                                                  num_key_value_heads=2, head_dim=128),
                                  dtype="bfloat16", seed=22, prompt_len=5, steps=4),
}

CONFIG0 = dict(cfg=QWEN3_0_6B, dtype="float16", seed=0, prompt_seed=1, prompt_len=16, new_tokens=32)


def weights_digest(manifest_path: Path) -> str:
    m = json.loads(Path(manifest_path).read_text())
    h = hashlib.sha256()
    for rec in m["tensors"]:
        with open(Path(manifest_path).parent / rec["file"], "rb") as f:
            while True:
                b = f.read(1 << 24)
                if not b:
                    break
                h.update(b)
    return h.hexdigest()


def load_fixture(path) -> dict:
    z = np.load(path, allow_pickle=False)
    fx = {k: z[k] for k in z.files}
    fx["meta"] = json.loads(str(fx["meta"]))
    return fx


def bundle_for(fx: dict, out_dir) -> Path:
    """Re-create the fixture's bundle and check it is byte-identical to the one used."""
    meta = fx["meta"]
    p = write_synthetic_bundle(Path(out_dir) / meta["name"], meta["cfg"], seed=meta["seed"], dtype=meta["dtype"])
    got = weights_digest(p)
    if got != meta["weights_sha256"]:
        raise AssertionError(f"synthetic bundle differs from the golden one ({got} != {meta['weights_sha256']})")
    return p


def make_tiny(name: str, spec: dict, tmp: Path) -> None:
    from oracle.oracle import RefModel
    p = write_synthetic_bundle(tmp / name, spec["cfg"], seed=spec["seed"], dtype=spec["dtype"])
    rm = RefModel(p, 64)
    rng = np.random.default_rng(spec["seed"] + 1000)
    prompt = rng.integers(0, spec["cfg"]["vocab_size"], spec["prompt_len"]).astype(np.int32)
    pre = rm.forward(prompt, 0)
    inputs, logits, greedy = [], [], [rm.sample(pre[-1])]
    pos = len(prompt)
    for i in range(spec["steps"]):
        tok = greedy[-1]
        inputs.append(tok)
        lg = rm.forward([tok], pos + i)[0]
        logits.append(lg)
        greedy.append(rm.sample(lg))
    k, v = rm.kv_read(0, 0, pos + spec["steps"])
    meta = dict(name=name, cfg=spec["cfg"], seed=spec["seed"], dtype=spec["dtype"], weights_sha256=weights_digest(p),
                source="reference Mac/cpu/src via oracle/_ref/libsocref.so")
    np.savez_compressed(HERE / f"{name}.npz", meta=json.dumps(meta), prompt=prompt, prefill_logits=pre,
                        decode_inputs=np.array(inputs, np.int32), decode_logits=np.stack(logits),
                        greedy=np.array(greedy, np.int32), kv_k_layer0=k, kv_v_layer0=v)
    print("wrote", HERE / f"{name}.npz")


def config0_prompt() -> np.ndarray:
    c = CONFIG0
    return np.random.default_rng(c["prompt_seed"]).integers(0, c["cfg"]["vocab_size"], c["prompt_len"]).astype(np.int32)


def make_config0(tmp: Path) -> None:
    """Greedy ids of benchmark config 0 (16-token prompt + 32 tokens) from the reference,
    with the top-16 logits of every step (the CPU top-2 gap flags near-ties)."""
    import time
    from oracle.oracle import RefModel
    c = CONFIG0
    p = write_synthetic_bundle(tmp / "config0", c["cfg"], seed=c["seed"], dtype=c["dtype"])
    rm = RefModel(p, 64)
    prompt = config0_prompt()
    t0 = time.time()
    lg = rm.forward(prompt, 0)[-1]
    t_prefill = time.time() - t0
    toks, tops_v, tops_i = [], [], []
    pos = len(prompt)
    step_times = []
    for i in range(c["new_tokens"]):
        order = np.argsort(-lg, kind="stable")[:16]
        tops_i.append(order.astype(np.int32))
        tops_v.append(lg[order])
        toks.append(rm.sample(lg))
        if i + 1 < c["new_tokens"]:
            t1 = time.time()
            lg = rm.forward([toks[-1]], pos + i)[0]
            step_times.append(time.time() - t1)
    meta = dict(name="config0", cfg=c["cfg"], seed=c["seed"], dtype=c["dtype"], weights_sha256=weights_digest(p),
                prompt_seed=c["prompt_seed"], source="reference Mac/cpu/src via oracle/_ref/libsocref.so",
                ref_prefill_s=t_prefill, ref_decode_s_per_token=float(np.mean(step_times)) if step_times else None)
    np.savez_compressed(HERE / "config0_greedy.npz", meta=json.dumps(meta), prompt=prompt,
                        greedy=np.array(toks, np.int32), top_ids=np.stack(tops_i), top_logits=np.stack(tops_v))
    print("wrote", HERE / "config0_greedy.npz", meta)


if __name__ == "__main__":
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        if "--config0" in sys.argv:
            make_config0(Path(d))
        else:
            for name, spec in TINY.items():
                make_tiny(name, spec, Path(d))
