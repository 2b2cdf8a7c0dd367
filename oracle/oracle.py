"""TEST INFRASTRUCTURE ONLY -- ctypes front end of the two CPU checkers.

* ``Oracle*``: this repository's C restatement (``oracle/soc_oracle.c``) of the
  reference CPU runtime's Qwen3 forward.
* ``Ref*``: the reference CPU runtime itself (``oracle/_ref/libsocref.so``,
  its ``Mac/cpu/src`` compiled unchanged, driven by ``oracle/ref_driver.cpp``).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs use
this module, as the checker; the soc_b200 product never imports it.
"""
from __future__ import annotations

import ctypes as C
import json
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "libsoc_oracle.so"
REF_SO = HERE / "_ref" / "libsocref.so"

_F = C.POINTER(C.c_float)
_I = C.POINTER(C.c_int32)
DT_CODE = {"float32": 0, "float16": 1, "bfloat16": 2}


def _fp(a: np.ndarray):
    return a.ctypes.data_as(_F)


def _ip(a: np.ndarray):
    return a.ctypes.data_as(_I)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


_olib = None
_rlib = None


def oracle_lib() -> C.CDLL:
    """Load (building if needed) the C restatement."""
    global _olib
    if _olib is None:
        if not ORACLE_SO.exists():
            import subprocess
            subprocess.run(["make", "-s", "-C", str(HERE), "oracle"], check=True)
        lib = C.CDLL(str(ORACLE_SO))
        lib.oracle_linear.argtypes = [_F, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_int, _F]
        lib.oracle_rmsnorm.argtypes = [_F, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_float, _F]
        lib.oracle_rope.argtypes = [_F, C.c_int, C.c_int, C.c_int, C.c_double, C.c_int]
        lib.oracle_attention.argtypes = [_F, C.c_int, C.c_int, _F, _F, C.c_int, C.c_int, C.c_int, C.c_int, _F]
        lib.oracle_argmax.argtypes = [_F, C.c_int]
        lib.oracle_argmax.restype = C.c_int
        lib.oracle_f16_to_f32.argtypes = [C.c_uint16]
        lib.oracle_f16_to_f32.restype = C.c_float
        lib.oracle_forward_cached.argtypes = [C.c_void_p, _I, C.c_int, C.c_int, _F, C.c_int]
        lib.oracle_forward_cached.restype = C.c_int
        _olib = lib
    return _olib


def ref_available() -> bool:
    return REF_SO.exists()


def ref_lib() -> C.CDLL:
    """Load the reference CPU runtime shim (built from the reference sources)."""
    global _rlib
    if _rlib is None:
        if not REF_SO.exists():
            raise FileNotFoundError(f"{REF_SO} missing: build it with `make -C oracle ref` where the reference is mounted")
        lib = C.CDLL(str(REF_SO))
        lib.socref_last_error.restype = C.c_char_p
        lib.socref_load.argtypes = [C.c_char_p]
        lib.socref_load.restype = C.c_void_p
        lib.socref_free.argtypes = [C.c_void_p]
        lib.socref_cache_new.argtypes = [C.c_void_p, C.c_int]
        lib.socref_cache_new.restype = C.c_void_p
        lib.socref_cache_free.argtypes = [C.c_void_p]
        lib.socref_cache_length.argtypes = [C.c_void_p]
        lib.socref_forward_cached.argtypes = [C.c_void_p, C.c_void_p, _I, C.c_int, C.c_int, _F]
        lib.socref_sample_greedy.argtypes = [_F, C.c_int]
        lib.socref_sample.argtypes = [_F, C.c_int, C.c_float, C.c_int]
        lib.socref_load_bundle.argtypes = [C.c_char_p]
        lib.socref_kv_read.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, _F, _F]
        lib.socref_linear.argtypes = [_F, C.c_int, C.c_int, _F, C.c_int, _F]
        lib.socref_rmsnorm.argtypes = [_F, C.c_int, C.c_int, _F, C.c_float, _F]
        lib.socref_rope.argtypes = [_F, C.c_int, C.c_int, C.c_int, C.c_double, C.c_int]
        lib.socref_attention.argtypes = [_F, C.c_int, C.c_int, _F, _F, C.c_int, C.c_int, C.c_int, C.c_int, _F]
        _rlib = lib
    return _rlib


# ---------------------------------------------------------------- module ops
def linear(x, w) -> np.ndarray:
    """y = x . W^T with W float32/float16 ``[out, in]`` (Linear::Forward)."""
    x = _f32(x)
    w = np.ascontiguousarray(w)
    dt = {np.dtype(np.float32): 0, np.dtype(np.float16): 1}[w.dtype]
    rows = x.size // w.shape[1]
    y = np.empty((rows, w.shape[0]), dtype=np.float32)
    oracle_lib().oracle_linear(_fp(x), rows, w.shape[1], w.ctypes.data, dt, w.shape[0], _fp(y))
    return y.reshape(x.shape[:-1] + (w.shape[0],))


def rmsnorm(x, w, eps=1e-6) -> np.ndarray:
    x = _f32(x)
    w = np.ascontiguousarray(w)
    dt = {np.dtype(np.float32): 0, np.dtype(np.float16): 1}[w.dtype]
    y = np.empty_like(x)
    oracle_lib().oracle_rmsnorm(_fp(x), x.size // w.shape[0], w.shape[0], w.ctypes.data, dt, eps, _fp(y))
    return y


def rope(x, theta, pos0) -> np.ndarray:
    """x: [T, heads, D]; returns the rotated copy."""
    y = _f32(x).copy()
    T, Hh, D = y.shape
    oracle_lib().oracle_rope(_fp(y), T, Hh, D, float(theta), int(pos0))
    return y


def attention(q, k, v, prefix) -> np.ndarray:
    """q [T, Hq, D]; k, v [S, Hkv, D]; causal with ``prefix`` cached positions."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.empty_like(q)
    oracle_lib().oracle_attention(_fp(q), q.shape[0], q.shape[1], _fp(k), _fp(v), k.shape[0], k.shape[1],
                                  k.shape[2], int(prefix), _fp(out))
    return out


def argmax(logits) -> int:
    x = _f32(logits)
    return int(oracle_lib().oracle_argmax(_fp(x), x.size))


# --------------------------------------------------------------- whole model
class _OracleModelStruct(C.Structure):
    _fields_ = [
        ("hidden", C.c_int), ("inter", C.c_int), ("layers", C.c_int), ("hq", C.c_int), ("hkv", C.c_int),
        ("hd", C.c_int), ("vocab", C.c_int), ("max_seq", C.c_int),
        ("eps", C.c_float), ("theta", C.c_double),
        ("embed", C.c_void_p), ("embed_dt", C.c_int),
        ("fnorm", C.c_void_p), ("fnorm_dt", C.c_int),
        ("lm_head", C.c_void_p), ("lm_head_dt", C.c_int),
        ("lw", C.POINTER(C.c_void_p)), ("lw_dt", C.POINTER(C.c_int)),
        ("kcache", _F), ("vcache", _F), ("length", C.c_int),
    ]


def _read_manifest(path):
    p = Path(path)
    m = json.loads(p.read_text())
    recs = {r["name"]: r for r in m["tensors"]}
    return m, recs, p.parent


def _load_weight(recs, base, name):
    """Returns (array, dtype code).  Group-quantised linears are dequantised to
    float32 here (``float(q) * float(scale)``), the oracle of the int8/int4 paths."""
    r = recs[name]
    path = base / r["file"]
    if r["dtype"] in ("int8_g64", "int4_g32"):
        s = recs[name + ".scales"]
        scale = np.fromfile(base / s["file"], dtype=np.float16).reshape(s["shape"])
        if r["dtype"] == "int8_g64":
            q = np.fromfile(path, dtype=np.int8).reshape(r["shape"])
        else:
            q = np.fromfile(path, dtype=np.uint8).reshape(r["shape"][0], r["shape"][1] // 2)
        from soc_b200.bundle import dequantize_groupwise  # same formula as the writer
        return np.ascontiguousarray(dequantize_groupwise(q, scale, r["dtype"]), dtype=np.float32), 0
    dt = {"float32": np.float32, "float16": np.float16, "bfloat16": np.uint16}[r["dtype"]]
    arr = np.fromfile(path, dtype=dt).reshape(r["shape"])
    return arr, DT_CODE[r["dtype"]]


class OracleModel:
    """The C restatement over a bundle: ``forward(ids, pos)`` = ForwardLogitsCached."""

    def __init__(self, manifest_path, max_seq=256):
        m, recs, base = _read_manifest(manifest_path)
        cfg = m["config"]
        from soc_b200.bundle import layer_tensor_names
        self.cfg = cfg
        self._keep = []
        L = cfg["num_hidden_layers"]
        ptrs = (C.c_void_p * (L * 11))()
        dts = (C.c_int * (L * 11))()
        for layer in range(L):
            for j, name in enumerate(layer_tensor_names(layer)):
                a, d = _load_weight(recs, base, name)
                self._keep.append(a)
                ptrs[layer * 11 + j] = a.ctypes.data
                dts[layer * 11 + j] = d
        emb, emb_dt = _load_weight(recs, base, "model.embed_tokens.weight")
        fn, fn_dt = _load_weight(recs, base, "model.norm.weight")
        self._keep += [emb, fn, ptrs, dts]
        lm, lm_dt = (None, 0)
        if not cfg["tie_word_embeddings"]:
            lm, lm_dt = _load_weight(recs, base, "lm_head.weight")
            self._keep.append(lm)
        self.hd, self.hkv = cfg["head_dim"], cfg["num_key_value_heads"]
        self.vocab = cfg["vocab_size"]
        self.max_seq = max_seq
        self.kc = np.zeros((L, self.hkv, max_seq, self.hd), dtype=np.float32)
        self.vc = np.zeros_like(self.kc)
        s = _OracleModelStruct()
        s.hidden, s.inter, s.layers = cfg["hidden_size"], cfg["intermediate_size"], L
        s.hq, s.hkv, s.hd, s.vocab, s.max_seq = cfg["num_attention_heads"], self.hkv, self.hd, self.vocab, max_seq
        s.eps = float(np.float32(cfg["rms_norm_eps"]))
        s.theta = float(cfg["rope_theta"])
        s.embed, s.embed_dt = emb.ctypes.data, emb_dt
        s.fnorm, s.fnorm_dt = fn.ctypes.data, fn_dt
        s.lm_head, s.lm_head_dt = (lm.ctypes.data if lm is not None else None), lm_dt
        s.lw = ptrs
        s.lw_dt = dts
        s.kcache, s.vcache = _fp(self.kc), _fp(self.vc)
        s.length = 0
        self.s = s

    @property
    def length(self) -> int:
        return self.s.length

    def reset(self):
        self.s.length = 0

    def forward(self, ids, pos, last_only=False) -> np.ndarray:
        """Logits ``[T, vocab]`` (or ``[1, vocab]`` for the last row only)."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        T = ids.size
        first = T - 1 if last_only else 0
        out = np.empty((T - first, self.vocab), dtype=np.float32)
        rc = oracle_lib().oracle_forward_cached(C.byref(self.s), _ip(ids), T, int(pos), _fp(out), first)
        if rc == -1:
            raise ValueError("embedding input token id out of range")
        if rc == -2:
            raise ValueError("kv cache write position out of range")
        return out

    def set_cache(self, layer, k, v):
        """Overwrite positions [0, S) of `layer` with [S, Hkv, D] K and V (TensorKVCache::Write
        of a whole prefix, kv_cache.cpp:50-80); set_length() then makes them visible."""
        S = k.shape[0]
        self.kc[layer, :, :S, :] = np.asarray(k, dtype=np.float32).transpose(1, 0, 2)
        self.vc[layer, :, :S, :] = np.asarray(v, dtype=np.float32).transpose(1, 0, 2)

    def set_length(self, n):
        self.s.length = int(n)

    def kv_read(self, layer, start, end):
        """[S, Hkv, D] float32 K and V, like TensorKVCache::Read."""
        if end > self.length or start > end:
            raise ValueError("kv cache read range exceeds cached sequence length")
        k = self.kc[layer, :, start:end, :].transpose(1, 0, 2).copy()
        v = self.vc[layer, :, start:end, :].transpose(1, 0, 2).copy()
        return k, v

    def generate(self, prompt, n_new):
        """Prefill then greedy decode; returns (generated ids, per-step last-row logits)."""
        self.reset()
        lg = self.forward(prompt, 0, last_only=True)[0]
        toks, logits = [argmax(lg)], [lg]
        pos = len(prompt)
        for _ in range(n_new - 1):
            lg = self.forward([toks[-1]], pos, last_only=True)[0]
            pos += 1
            toks.append(argmax(lg))
            logits.append(lg)
        return toks, np.stack(logits)


class RefModel:
    """The reference CPU runtime over a bundle (QwenModelLoader + ForwardLogitsCached)."""

    def __init__(self, manifest_path, max_seq=256):
        lib = ref_lib()
        self.lib = lib
        self.h = lib.socref_load(str(manifest_path).encode())
        if not self.h:
            raise RuntimeError(lib.socref_last_error().decode("utf-8", "replace"))
        self.cfg = json.loads(Path(manifest_path).read_text())["config"]
        self.vocab = self.cfg["vocab_size"]
        self.c = lib.socref_cache_new(self.h, max_seq)

    def __del__(self):
        try:
            self.lib.socref_cache_free(self.c)
            self.lib.socref_free(self.h)
        except Exception:
            pass

    @property
    def length(self) -> int:
        return self.lib.socref_cache_length(self.c)

    def forward(self, ids, pos) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty((ids.size, self.vocab), dtype=np.float32)
        if self.lib.socref_forward_cached(self.h, self.c, _ip(ids), ids.size, int(pos), _fp(out)) != 0:
            raise RuntimeError(self.lib.socref_last_error().decode("utf-8", "replace"))
        return out

    def sample(self, logits_row) -> int:
        x = _f32(logits_row)
        return int(self.lib.socref_sample_greedy(_fp(x), x.size))

    def kv_read(self, layer, start, end):
        hkv, hd = self.cfg["num_key_value_heads"], self.cfg["head_dim"]
        k = np.empty((end - start, hkv, hd), dtype=np.float32)
        v = np.empty_like(k)
        if self.lib.socref_kv_read(self.c, layer, start, end, _fp(k), _fp(v)) != 0:
            raise RuntimeError(self.lib.socref_last_error().decode("utf-8", "replace"))
        return k, v


def ref_linear(x, w):
    x, w = _f32(x), _f32(w)
    y = np.empty((x.size // w.shape[1], w.shape[0]), dtype=np.float32)
    if ref_lib().socref_linear(_fp(x), y.shape[0], w.shape[1], _fp(w), w.shape[0], _fp(y)) != 0:
        raise RuntimeError(ref_lib().socref_last_error().decode("utf-8", "replace"))
    return y


def ref_rmsnorm(x, w, eps=1e-6):
    x, w = _f32(x), _f32(w)
    y = np.empty_like(x)
    if ref_lib().socref_rmsnorm(_fp(x), x.size // w.size, w.size, _fp(w), eps, _fp(y)) != 0:
        raise RuntimeError(ref_lib().socref_last_error().decode("utf-8", "replace"))
    return y


def ref_rope(x, theta, pos0):
    y = _f32(x).copy()
    T, Hh, D = y.shape
    if ref_lib().socref_rope(_fp(y), T, Hh, D, float(theta), int(pos0)) != 0:
        raise RuntimeError(ref_lib().socref_last_error().decode("utf-8", "replace"))
    return y


def ref_attention(q, k, v, prefix):
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.empty_like(q)
    if ref_lib().socref_attention(_fp(q), q.shape[0], q.shape[1], _fp(k), _fp(v), k.shape[0], k.shape[1],
                                  k.shape[2], int(prefix), _fp(out)) != 0:
        raise RuntimeError(ref_lib().socref_last_error().decode("utf-8", "replace"))
    return out


def host_cores() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count() or 1


def _mix64(x: np.ndarray) -> np.ndarray:
    """splitmix64 output function of x + 0x9E3779B97F4A7C15 (uint64, wrapping)."""
    z = x + np.uint64(0x9E3779B97F4A7C15)
    z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def kv_random(seed: int, seq: int, layer: int, kind: int, n_tokens: int, hkv: int, hd: int, layers: int) -> np.ndarray:
    """The seeded K (kind 0) or V (kind 1) contents that soc_b200_kv_fill_random writes for
    one layer of one sequence, [n_tokens, hkv, hd] float16 (restated for the parity tests)."""
    with np.errstate(over="ignore"):
        stream = np.uint64((seq * layers + layer) * 2 + kind)
        e = np.arange(n_tokens * hkv * hd, dtype=np.uint64)
        x = np.uint64(seed) + stream * np.uint64(0xD1B54A32D192ED03) + np.uint64(3) * e
        total = np.zeros(e.shape, dtype=np.uint64)
        for w in range(3):
            z = _mix64(x + np.uint64(w))
            for sh in (0, 16, 32, 48):
                total += (z >> np.uint64(sh)) & np.uint64(0xFFFF)
    val = total.astype(np.float32) * np.float32(1.0 / 65536.0) - np.float32(6.0)
    return val.astype(np.float16).reshape(n_tokens, hkv, hd)


class RefTokenizer:
    """The reference's TokenizerRuntime + Qwen3TemplateBuilder (oracle/_ref), for parity tests."""

    def __init__(self, path):
        lib = ref_lib()
        if not hasattr(lib, "_tok_bound"):
            lib.socref_tokenizer_load.argtypes = [C.c_char_p]
            lib.socref_tokenizer_load.restype = C.c_void_p
            lib.socref_tokenizer_free.argtypes = [C.c_void_p]
            lib.socref_tokenizer_encode.argtypes = [C.c_void_p, C.c_char_p, C.c_int, C.POINTER(C.c_int32), C.c_int]
            lib.socref_tokenizer_decode.argtypes = [C.c_void_p, C.POINTER(C.c_int32), C.c_int, C.c_char_p, C.c_int]
            lib.socref_chat_prompt.argtypes = [C.c_void_p, C.c_char_p, C.c_int, C.c_int, C.c_char_p, C.c_char_p,
                                               C.c_int]
            lib.socref_chat_prompt_messages.argtypes = [C.c_void_p, C.POINTER(C.c_char_p), C.POINTER(C.c_char_p),
                                                        C.c_int, C.c_int, C.c_int, C.c_char_p, C.c_char_p, C.c_int]
            lib._tok_bound = True
        self.lib = lib
        self.h = lib.socref_tokenizer_load(str(path).encode())
        if not self.h:
            raise ValueError(lib.socref_last_error().decode("utf-8", "replace"))

    def free(self):
        if self.h:
            self.lib.socref_tokenizer_free(self.h)
            self.h = None

    def encode(self, text):
        data = text.encode("utf-8") if isinstance(text, str) else bytes(text)
        cap = len(data) + 16
        ids = (C.c_int32 * cap)()
        n = self.lib.socref_tokenizer_encode(self.h, data, len(data), ids, cap)
        if n < 0:
            raise ValueError(self.lib.socref_last_error().decode("utf-8", "replace"))
        return list(ids[:n])

    def decode_bytes(self, ids):
        arr = (C.c_int32 * max(1, len(ids)))(*ids)
        cap = 64 + 64 * len(ids)
        buf = C.create_string_buffer(cap)
        n = self.lib.socref_tokenizer_decode(self.h, arr, len(ids), buf, cap)
        if n < 0:
            raise ValueError(self.lib.socref_last_error().decode("utf-8", "replace"))
        return buf.raw[:n]

    def chat_prompt(self, user, add_generation_prompt=True, enable_thinking=True, system_prompt=""):
        cap = 1024 + 4 * len(user.encode()) + len(system_prompt.encode())
        buf = C.create_string_buffer(cap)
        n = self.lib.socref_chat_prompt(self.h, user.encode(), int(add_generation_prompt), int(enable_thinking),
                                        system_prompt.encode(), buf, cap)
        if n < 0:
            raise ValueError(self.lib.socref_last_error().decode("utf-8", "replace"))
        return buf.raw[:n].decode("utf-8")

    def chat_prompt_messages(self, messages, add_generation_prompt=True, enable_thinking=True, system_prompt=""):
        n = len(messages)
        roles = (C.c_char_p * max(n, 1))(*[r.encode() for r, _ in messages])
        contents = (C.c_char_p * max(n, 1))(*[c.encode() for _, c in messages])
        cap = 1024 + sum(4 * len(c.encode()) + len(r) for r, c in messages) + len(system_prompt.encode())
        buf = C.create_string_buffer(cap)
        k = self.lib.socref_chat_prompt_messages(self.h, roles, contents, n, int(add_generation_prompt),
                                                 int(enable_thinking), system_prompt.encode(), buf, cap)
        if k < 0:
            raise ValueError(self.lib.socref_last_error().decode("utf-8", "replace"))
        return buf.raw[:k].decode("utf-8")


def ref_sample(logits_row, temperature=1.0, top_k=1) -> int:
    """The reference Sampler::SampleFromLogits (Mac/cpu/src/sampler.cpp:22-57) on one row."""
    x = _f32(logits_row)
    r = int(ref_lib().socref_sample(_fp(x), x.size, float(temperature), int(top_k)))
    if r < 0:
        raise ValueError(ref_lib().socref_last_error().decode("utf-8", "replace"))
    return r


def sample_rule(logits_row, temperature=1.0) -> int:
    """The pick the device kernels make: first index of the maximum of logit / temperature
    (float32 IEEE division, as the reference's comparator computes it)."""
    x = _f32(logits_row)
    return int(np.argmax(x / np.float32(temperature)))


def ref_load_bundle(manifest_path) -> str | None:
    """The reference's RuntimePipeline::LoadBundle: None when it loads, else its error message."""
    lib = ref_lib()
    if lib.socref_load_bundle(str(manifest_path).encode()) == 0:
        return None
    return lib.socref_last_error().decode("utf-8", "replace")
