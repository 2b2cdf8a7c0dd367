"""Python front end of the soc_b200 C ABI (``include/soc_b200.h``), via ctypes.

The classes mirror the reference runtime's objects so host code reads the same:

* ``Context``           -- device + stream (reference: ``MetalContext``)
* ``Model``             -- a loaded bundle (``QwenModelLoader::LoadModel`` -> ``QwenCausalLM``),
                           with ``forward_logits_cached`` (``QwenCausalLM::ForwardLogitsCached``,
                           ``Mac/cpu/src/qwen_causal_lm.cpp:74-80``)
* ``KVCache``           -- paged fp16 cache (``TensorKVCache``, ``Mac/cpu/src/kv_cache.cpp``)
* ``GenerationContext`` -- ``Prefill / DecodeNextToken / Generate / Reset``
                           (``Mac/gpu/src/runtime/generation_context.cpp:17-179``)

Errors raise ``SocError`` (the reference throws ``std::runtime_error``) carrying the
library's status code and message.  There is no CPU fallback: without the CUDA
library or a GPU every entry point fails loudly.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libsoc_b200.so"
HEADER = PKG.parent / "include" / "soc_b200.h"

OK = 0
ERR_INVALID, ERR_CUDA, ERR_IO, ERR_FORMAT, ERR_CAPACITY, ERR_RANGE, ERR_DEVICE = -1, -2, -3, -4, -5, -6, -7
WEIGHTS_NATIVE, WEIGHTS_F16, WEIGHTS_BF16, WEIGHTS_INT8_G64, WEIGHTS_INT4_G32 = 0, 1, 2, 3, 4


class SocError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class ModelInfo(C.Structure):
    _fields_ = [
        ("layers", C.c_int), ("hidden", C.c_int), ("intermediate", C.c_int), ("q_heads", C.c_int),
        ("kv_heads", C.c_int), ("head_dim", C.c_int), ("vocab", C.c_int), ("tied_embeddings", C.c_int),
        ("weight_format", C.c_int), ("max_position", C.c_int), ("rms_norm_eps", C.c_float),
        ("rope_theta", C.c_double), ("tp_rank", C.c_int), ("tp_size", C.c_int),
    ]


_lib = None
_VP = C.c_void_p
_I32P = C.POINTER(C.c_int32)
_FP = C.POINTER(C.c_float)

_SIGNATURES = {
    "soc_b200_last_error": (C.c_char_p, []),
    "soc_b200_kernel_launches": (C.c_longlong, []),
    "soc_b200_open": (C.c_int, [C.c_int, C.POINTER(_VP)]),
    "soc_b200_close": (None, [_VP]),
    "soc_b200_synchronize": (C.c_int, [_VP]),
    "soc_b200_stream": (_VP, [_VP]),
    "soc_b200_load_bundle": (C.c_int, [_VP, C.c_char_p, C.c_int, C.c_int, C.c_int, _VP, C.POINTER(_VP)]),
    "soc_b200_model_info": (C.c_int, [_VP, C.POINTER(ModelInfo)]),
    "soc_b200_free_model": (None, [_VP]),
    "soc_b200_kv_create": (C.c_int, [_VP, C.c_int, C.c_int, C.c_int, C.POINTER(_VP)]),
    "soc_b200_free_kv": (None, [_VP]),
    "soc_b200_kv_reset": (C.c_int, [_VP, C.c_int]),
    "soc_b200_kv_length": (C.c_int, [_VP, C.c_int]),
    "soc_b200_kv_read": (C.c_int, [_VP, C.c_int, C.c_int, C.c_int, C.c_int, _FP, _FP]),
    "soc_b200_kv_write": (C.c_int, [_VP, C.c_int, C.c_int, C.c_int, C.c_int, _FP, _FP]),
    "soc_b200_kv_fill_random": (C.c_int, [_VP, C.c_int, C.c_int, C.c_ulonglong]),
    "soc_b200_nccl_unique_id": (C.c_int, [_VP]),
    "soc_b200_nccl_comm_create": (C.c_int, [_VP, C.c_int, C.c_int, _VP, C.POINTER(_VP)]),
    "soc_b200_nccl_comm_destroy": (C.c_int, [_VP]),
    "soc_b200_prefill": (C.c_int, [_VP, _VP, C.c_int, _I32P, C.c_int, _FP, _I32P]),
    "soc_b200_decode": (C.c_int, [_VP, _VP, C.c_int, _I32P, _I32P, _FP, _I32P]),
    "soc_b200_generate": (C.c_int, [_VP, _VP, C.c_int, _I32P, C.c_int, C.c_int, C.c_int, _I32P,
                                    C.POINTER(C.c_int)]),
    "soc_b200_generate_device": (C.c_int, [_VP, _VP, C.c_int, _VP, C.c_int, C.c_int, _VP]),
    "soc_b200_linear": (C.c_int, [_VP, C.c_int, _VP, _VP, C.c_int, C.c_int, _VP, C.c_int, _VP, _VP]),
    "soc_b200_decode_noalloc": (C.c_int, [_VP, _VP, C.c_int, C.c_int32, _FP, _I32P]),
    "soc_b200_topk": (C.c_int, [_VP, C.c_int, C.c_int, _FP, _I32P]),
    "soc_b200_tokenizer_load": (C.c_int, [C.c_char_p, C.POINTER(_VP)]),
    "soc_b200_tokenizer_free": (None, [_VP]),
    "soc_b200_tokenizer_encode": (C.c_int, [_VP, C.c_char_p, C.c_size_t, _I32P, C.c_int, C.POINTER(C.c_int)]),
    "soc_b200_tokenizer_decode": (C.c_int, [_VP, _I32P, C.c_int, C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t)]),
    "soc_b200_chat_prompt": (C.c_int, [_VP, C.POINTER(C.c_char_p), C.POINTER(C.c_char_p), C.c_int, C.c_int, C.c_int,
                                       C.c_char_p, C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t)]),
    "soc_b200_tokenizer_check_model": (C.c_int, [_VP, C.c_longlong]),
    "soc_b200_manifest_generation_options": (C.c_int, [C.c_char_p, C.c_void_p]),
    "soc_b200_manifest_tokenizer_path": (C.c_int, [C.c_char_p, C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t)]),
    "soc_b200_sampler_check": (C.c_int, [C.c_float, C.c_size_t]),
    "soc_b200_set_sampler": (C.c_int, [_VP, C.c_float, C.c_size_t]),
    "soc_b200_validate_bundle": (C.c_int, [C.c_char_p]),
}


def lib() -> C.CDLL:
    """Load the in-tree CUDA library (raises if it was never built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(f"{LIB_PATH} is missing: run `python -m soc_b200.build` (no CPU fallback exists)")
        l = C.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGNATURES.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def _check(rc: int) -> None:
    if rc != OK:
        raise SocError(rc, lib().soc_b200_last_error().decode("utf-8", "replace"))


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int32)


def _ip(a: np.ndarray):
    return a.ctypes.data_as(_I32P)


def _fp(a: np.ndarray):
    return a.ctypes.data_as(_FP)


def kernel_launches() -> int:
    return int(lib().soc_b200_kernel_launches())


class Context:
    def __init__(self, device: int = 0):
        h = _VP()
        _check(lib().soc_b200_open(device, C.byref(h)))
        self.h = h
        self.device = device

    def close(self):
        if self.h:
            lib().soc_b200_close(self.h)
            self.h = None

    def synchronize(self):
        _check(lib().soc_b200_synchronize(self.h))

    @property
    def stream(self) -> int:
        return lib().soc_b200_stream(self.h) or 0

    def linear(self, weight_format, w_ptr, scales_ptr, out_features, in_features, x_ptr, rows, y_ptr, stream=None):
        """Kernel-level linear on device pointers (see ``soc_b200_linear``)."""
        _check(lib().soc_b200_linear(self.h, weight_format, w_ptr, scales_ptr, out_features, in_features, x_ptr,
                                     rows, y_ptr, stream))

    # ---- tensor parallelism (NCCL loaded at run time)
    @staticmethod
    def nccl_unique_id() -> bytes:
        buf = C.create_string_buffer(128)
        _check(lib().soc_b200_nccl_unique_id(buf))
        return buf.raw

    def nccl_comm_create(self, nranks: int, rank: int, uid: bytes):
        """Communicator of `nranks` ranks on this context's device (every rank calls it)."""
        buf = C.create_string_buffer(bytes(uid), 128)
        h = _VP()
        _check(lib().soc_b200_nccl_comm_create(self.h, nranks, rank, buf, C.byref(h)))
        return h

    @staticmethod
    def nccl_comm_destroy(comm):
        if comm:
            _check(lib().soc_b200_nccl_comm_destroy(comm))


def tensor_parallel_comm(ctx: "Context", group=None):
    """NCCL communicator over the ranks of an initialised torch.distributed group: rank 0's
    id reaches the others by broadcast_object_list."""
    import torch.distributed as dist
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    obj = [Context.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    return ctx.nccl_comm_create(world, rank, obj[0])


class Model:
    def __init__(self, ctx: Context, manifest_path, weight_format: int = WEIGHTS_NATIVE, tp_rank: int = 0,
                 tp_size: int = 1, comm=None):
        h = _VP()
        _check(lib().soc_b200_load_bundle(ctx.h, str(manifest_path).encode(), weight_format, tp_rank, tp_size, comm,
                                          C.byref(h)))
        self.ctx = ctx
        self.h = h
        self.top_k = 1  # the sampler's candidate count (set_sampler)
        info = ModelInfo()
        _check(lib().soc_b200_model_info(h, C.byref(info)))
        self.info = info
        self.vocab = info.vocab

    def free(self):
        if self.h:
            lib().soc_b200_free_model(self.h)
            self.h = None

    # QwenCausalLM::ForwardLogitsCached for one sequence, last row only.
    def forward_logits_cached(self, kv: "KVCache", seq: int, ids) -> tuple[np.ndarray, int]:
        ids = _i32(ids)
        logits = np.empty(self.vocab, dtype=np.float32)
        nid = np.zeros(1, dtype=np.int32)
        _check(lib().soc_b200_prefill(self.h, kv.h, seq, _ip(ids), ids.size, _fp(logits), _ip(nid)))
        return logits, int(nid[0])

    def decode(self, kv: "KVCache", seq_ids, last_ids, want_logits=True):
        seq_ids, last_ids = _i32(seq_ids), _i32(last_ids)
        n = seq_ids.size
        logits = np.empty((n, self.vocab), dtype=np.float32) if want_logits else None
        nxt = np.zeros(n, dtype=np.int32)
        _check(lib().soc_b200_decode(self.h, kv.h, n, _ip(seq_ids), _ip(last_ids),
                                     _fp(logits) if logits is not None else None, _ip(nxt)))
        return logits, nxt

    def set_sampler(self, temperature: float = 1.0, top_k: int = 1) -> None:
        """Sampler(SamplerConfig) for later picks: argmax of logit / temperature (``soc_b200_set_sampler``)."""
        _check(lib().soc_b200_set_sampler(self.h, float(temperature), int(top_k)))
        self.top_k = int(top_k)

    def decode_noalloc(self, kv: "KVCache", seq: int, last_id: int, want_logits=True):
        """One decode step that allocates no device memory (``soc_b200_decode_noalloc``):
        for hosts that cannot call cudaMalloc while serving."""
        logits = np.empty(self.vocab, dtype=np.float32) if want_logits else None
        nid = np.zeros(1, dtype=np.int32)
        _check(lib().soc_b200_decode_noalloc(self.h, kv.h, seq, int(last_id),
                                             _fp(logits) if logits is not None else None, _ip(nid)))
        return logits, int(nid[0])

    def topk(self, row: int, k: int) -> tuple[np.ndarray, np.ndarray]:
        """The sampler's k candidates of logits row `row` of the last prefill / decode call
        (``soc_b200_topk``): raw logits and token ids, larger logit / temperature first."""
        vals = np.empty(k, dtype=np.float32)
        ids = np.empty(k, dtype=np.int32)
        _check(lib().soc_b200_topk(self.h, row, k, _fp(vals), _ip(ids)))
        return vals, ids

    def generate(self, kv: "KVCache", seq: int, prompt, max_new: int, eos: int = -1) -> list[int]:
        prompt = _i32(prompt)
        out = np.zeros(max(max_new, 1), dtype=np.int32)
        n = C.c_int(0)
        _check(lib().soc_b200_generate(self.h, kv.h, seq, _ip(prompt), prompt.size, max_new, eos, _ip(out),
                                       C.byref(n)))
        return out[: n.value].tolist()

    def generate_device(self, kv: "KVCache", seq: int, d_prompt: int, n_prompt: int, max_new: int, d_out: int):
        _check(lib().soc_b200_generate_device(self.h, kv.h, seq, d_prompt, n_prompt, max_new, d_out))


class KVCache:
    def __init__(self, model: Model, max_seqs: int = 1, max_tokens: int = 4096, page_tokens: int = 16):
        h = _VP()
        _check(lib().soc_b200_kv_create(model.h, max_seqs, max_tokens, page_tokens, C.byref(h)))
        self.h = h
        self.model = model

    def free(self):
        if self.h:
            lib().soc_b200_free_kv(self.h)
            self.h = None

    def reset(self, seq: int = 0):
        _check(lib().soc_b200_kv_reset(self.h, seq))

    def length(self, seq: int = 0) -> int:
        r = lib().soc_b200_kv_length(self.h, seq)
        if r < 0:
            _check(r)
        return r

    def read(self, seq: int, layer: int, start: int, end: int):
        """K and V [end - start, kv heads held here, head_dim] (a tensor-parallel rank holds
        kv_heads / tp_size of them)."""
        i = self.model.info
        k = np.empty((end - start, i.kv_heads // i.tp_size, i.head_dim), dtype=np.float32)
        v = np.empty_like(k)
        _check(lib().soc_b200_kv_read(self.h, seq, layer, start, end, _fp(k), _fp(v)))
        return k, v

    def write(self, seq: int, layer: int, start: int, k, v):
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        _check(lib().soc_b200_kv_write(self.h, seq, layer, start, start + k.shape[0], _fp(k), _fp(v)))

    def fill_random(self, seq: int, n_tokens: int, seed: int):
        """Replace `seq` by n_tokens positions of seeded ~N(0, 1) fp16 K/V (soc_b200_kv_fill_random)."""
        _check(lib().soc_b200_kv_fill_random(self.h, seq, n_tokens, seed))


@dataclass
class GenerationStepResult:
    token_id: int
    logits: np.ndarray | None = None
    top_logits: np.ndarray | None = None     # the sampler's top_k candidates (generation_context.h:17-21)
    top_token_ids: np.ndarray | None = None


class GenerationContext:
    """The reference's ``GenerationContext`` shape over one sequence of a ``KVCache``
    (``Mac/gpu/include/runtime/generation_context.h:23-74``)."""

    def __init__(self, model: Model, max_sequence_length: int = 256, kv: KVCache | None = None, seq: int = 0):
        self.model = model
        self.max_sequence_length = max_sequence_length
        self.kv = kv or KVCache(model, 1, max_sequence_length)
        self.seq = seq
        self.prompt_token_ids: list[int] = []
        self.running_token_ids: list[int] = []
        self._last_logits: np.ndarray | None = None

    def prefill(self, token_ids) -> np.ndarray:
        """Reset, then run the prompt; returns the last row's logits (generation_context.cpp:17-59)."""
        if len(token_ids) == 0:
            raise SocError(ERR_INVALID, "GenerationContext prefill requires at least one token")
        self.reset()
        if len(token_ids) > self.max_sequence_length:
            raise SocError(ERR_CAPACITY, "GenerationContext sequence length would exceed max_sequence_length")
        self.prompt_token_ids = list(map(int, token_ids))
        self.running_token_ids = list(self.prompt_token_ids)
        logits, _ = self.model.forward_logits_cached(self.kv, self.seq, token_ids)
        self._last_logits = logits
        return logits

    def decode_next_token(self, last_token_id: int) -> GenerationStepResult:
        """generation_context.cpp:61-116 (tail check, length check, one step, greedy pick)."""
        if self.kv.length(self.seq) == 0:
            raise SocError(ERR_INVALID, "GenerationContext decode requires a prefilled KV cache")
        if not self.running_token_ids or self.running_token_ids[-1] != last_token_id:
            raise SocError(ERR_INVALID,
                           "GenerationContext decode requires last_token_id to match the current sequence tail")
        if len(self.running_token_ids) >= self.max_sequence_length:
            raise SocError(ERR_CAPACITY, "GenerationContext sequence length would exceed max_sequence_length")
        logits, nxt = self.model.decode(self.kv, [self.seq], [last_token_id])
        tok = int(nxt[0])
        top_vals, top_ids = self.model.topk(0, min(max(self.model.top_k, 1), 64))
        self.running_token_ids.append(tok)
        self._last_logits = logits[0]
        return GenerationStepResult(tok, logits[0], top_vals, top_ids)

    def generate(self, prompt_token_ids, max_new_tokens: int, eos_token_id: int = -1) -> list[int]:
        """generation_context.cpp:118-172, with the decode loop resident on the device."""
        if len(prompt_token_ids) + max(max_new_tokens - 1, 0) > self.max_sequence_length:
            raise SocError(ERR_CAPACITY, "GenerationContext sequence length would exceed max_sequence_length")
        self.reset()
        out = self.model.generate(self.kv, self.seq, prompt_token_ids, max_new_tokens, eos_token_id)
        self.prompt_token_ids = list(map(int, prompt_token_ids))
        self.running_token_ids = self.prompt_token_ids + out
        return out

    def reset(self):
        self.kv.reset(self.seq)
        self.prompt_token_ids = []
        self.running_token_ids = []
        self._last_logits = None


def header_functions() -> list[str]:
    """Names of every entry point declared in include/soc_b200.h."""
    import re
    text = HEADER.read_text()
    return re.findall(r"SOC_B200_API\s+[\w\s\*]+?\b(soc_b200_\w+)\s*\(", text)


class GenerationOptions(C.Structure):
    """``soc_generation_options``: RuntimeGenerationOptions (Mac/cpu/header/runtime_pipeline.h:12-17)."""
    _fields_ = [("max_new_tokens", C.c_size_t), ("temperature", C.c_float), ("top_k", C.c_size_t),
                ("eos_token_id", C.c_int), ("max_sequence_length", C.c_size_t)]

    @classmethod
    def from_manifest(cls, manifest_path) -> "GenerationOptions":
        """Defaults overridden by the manifest's generation_config
        (RuntimePipeline::GenerationOptionsFromManifest, Mac/cpu/src/runtime_pipeline.cpp:43-55)."""
        o = cls()
        _check(lib().soc_b200_manifest_generation_options(str(manifest_path).encode(), C.byref(o)))
        return o

    def check(self) -> None:
        """The sampler's argument checks (Mac/cpu/src/sampler.cpp:17-20)."""
        _check(lib().soc_b200_sampler_check(self.temperature, self.top_k))


def validate_bundle(manifest_path) -> None:
    """RuntimePipeline::LoadBundle's checks without a device (``soc_b200_validate_bundle``):
    raises SocError with the reference loader's message for the first problem found."""
    _check(lib().soc_b200_validate_bundle(str(manifest_path).encode()))


def manifest_tokenizer_path(manifest_path) -> str:
    """The manifest's tokenizer_runtime_file, resolved against the manifest's directory."""
    n = C.c_size_t(0)
    lib().soc_b200_manifest_tokenizer_path(str(manifest_path).encode(), None, 0, C.byref(n))
    buf = C.create_string_buffer(n.value + 1)
    _check(lib().soc_b200_manifest_tokenizer_path(str(manifest_path).encode(), buf, n.value + 1, C.byref(n)))
    return buf.value.decode()


class Tokenizer:
    """The bundle's tokenizer and Qwen3 chat template (host only; ``soc_b200_tokenizer_*``)."""

    def __init__(self, path):
        """`path`: a tokenizer_runtime.json, or a bundle's manifest.json (its tokenizer file is used)."""
        from pathlib import Path as _P
        p = _P(path)
        if p.name == "manifest.json":
            p = manifest_tokenizer_path(p)
        h = _VP()
        _check(lib().soc_b200_tokenizer_load(str(p).encode(), C.byref(h)))
        self.h = h

    def check_model(self, model_vocab_size: int) -> None:
        """StartupValidator::ValidateManifestAndTokenizer's vocab checks
        (Mac/cpu/src/startup_validator.cpp:77-101)."""
        _check(lib().soc_b200_tokenizer_check_model(self.h, int(model_vocab_size)))

    def free(self):
        if self.h:
            lib().soc_b200_tokenizer_free(self.h)
            self.h = None

    def encode(self, text: str | bytes) -> list[int]:
        data = text.encode("utf-8") if isinstance(text, str) else bytes(text)
        n = C.c_int(0)
        cap = max(16, len(data) + 16)
        ids = np.zeros(cap, dtype=np.int32)
        rc = lib().soc_b200_tokenizer_encode(self.h, data, len(data), _ip(ids), cap, C.byref(n))
        if rc == ERR_CAPACITY:
            ids = np.zeros(n.value, dtype=np.int32)
            rc = lib().soc_b200_tokenizer_encode(self.h, data, len(data), _ip(ids), n.value, C.byref(n))
        _check(rc)
        return ids[: n.value].tolist()

    def decode_bytes(self, ids) -> bytes:
        ids = _i32(ids)
        n = C.c_size_t(0)
        cap = max(64, 16 * ids.size)
        buf = C.create_string_buffer(cap)
        rc = lib().soc_b200_tokenizer_decode(self.h, _ip(ids), ids.size, buf, cap, C.byref(n))
        if rc == ERR_CAPACITY:
            buf = C.create_string_buffer(n.value)
            rc = lib().soc_b200_tokenizer_decode(self.h, _ip(ids), ids.size, buf, n.value, C.byref(n))
        _check(rc)
        return buf.raw[: n.value]

    def decode(self, ids) -> str:
        return self.decode_bytes(ids).decode("utf-8", errors="replace")

    def chat_prompt(self, messages, add_generation_prompt=True, enable_thinking=True, system_prompt="") -> str:
        """messages: [(role, content), ...] -> the Qwen3 template text."""
        n = len(messages)
        roles = (C.c_char_p * max(n, 1))(*[r.encode() for r, _ in messages])
        contents = (C.c_char_p * max(n, 1))(*[c.encode() for _, c in messages])
        ln = C.c_size_t(0)
        cap = 256 + sum(len(c.encode()) + len(r) + 32 for r, c in messages) + len(system_prompt.encode())
        buf = C.create_string_buffer(cap)
        _check(lib().soc_b200_chat_prompt(self.h, roles, contents, n, int(add_generation_prompt), int(enable_thinking),
                                          system_prompt.encode(), buf, cap, C.byref(ln)))
        return buf.raw[: ln.value].decode("utf-8")
