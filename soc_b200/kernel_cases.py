"""Small workloads that launch each kernel of the forward path a few times, for profiling.

    python -m soc_b200.kernel_cases linear    # k_linear / k_dequant / k_rows_to_half / k_gemm_tc / k_splitk_reduce
    python -m soc_b200.kernel_cases prefill   # a 2048-token prefill of a 2-layer Qwen3-0.6B-shape bundle
    python -m soc_b200.kernel_cases batched   # int8 decode of 32 sequences at contexts near 1,000 + top-k
    python -m soc_b200.kernel_cases decode    # the persistent batch-1 decode kernel (16-token prompt, 4 steps)

Every case runs on cuda:0 with seeded synthetic weights and inputs of the Qwen3-0.6B shapes and
holds well under 2 GB of device memory, so a profiler can replay its launches.  The case prints
`ok <case>` when it finishes.
"""
from __future__ import annotations

import sys
import tempfile
from pathlib import Path

import numpy as np

from . import runtime as R
from .bundle import QWEN3_0_6B, write_synthetic_bundle

# (out_features, in_features): the q projection and the tied lm_head of Qwen3-0.6B
LINEAR_SHAPES = ((2048, 1024), (151936, 1024))
LINEAR_ROWS = (1, 4, 16, 64)


def _quantise(torch, w32, fmt: str):
    """Group-wise symmetric quantisation as the bundle exporter does it (int8 g64 / int4 g32)."""
    out_f, in_f = w32.shape
    grp, qmax = (64, 127.0) if fmt == "int8" else (32, 7.0)
    wg = w32.view(out_f, in_f // grp, grp)
    sc = (wg.abs().amax(-1) / qmax).half().contiguous()
    q = torch.round(wg / sc.float()[..., None]).clamp(-qmax, qmax).to(torch.int8).view(out_f, in_f)
    if fmt == "int4":
        q = ((q[:, 0::2] & 0xF) | ((q[:, 1::2] & 0xF) << 4)).to(torch.uint8)
    code = R.WEIGHTS_INT8_G64 if fmt == "int8" else R.WEIGHTS_INT4_G32
    return q.contiguous(), sc, code


def case_linear(ctx) -> None:
    import torch
    st = torch.cuda.ExternalStream(ctx.stream)
    g = torch.Generator(device="cuda").manual_seed(2)
    for out_f, in_f in LINEAR_SHAPES:
        w32 = torch.randn(out_f, in_f, device="cuda", generator=g) * 0.02
        for fmt in ("fp16", "int8", "int4"):
            if fmt == "fp16":
                wq, sc, code = w32.half().contiguous(), None, R.WEIGHTS_F16
            else:
                wq, sc, code = _quantise(torch, w32, fmt)
            for rows in LINEAR_ROWS:
                x = torch.randn(rows, in_f, device="cuda", generator=g)
                y = torch.empty(rows, out_f, device="cuda")
                ctx.linear(code, wq.data_ptr(), sc.data_ptr() if sc is not None else None, out_f, in_f,
                           x.data_ptr(), rows, y.data_ptr(), st.cuda_stream)
            del wq, sc
        del w32
    ctx.synchronize()


def case_prefill(ctx, d: Path) -> None:
    p = write_synthetic_bundle(d / "b", dict(QWEN3_0_6B, num_hidden_layers=2), seed=0)
    m = R.Model(ctx, p)
    kv = R.KVCache(m, 1, 2100)
    prompt = np.random.default_rng(3).integers(0, QWEN3_0_6B["vocab_size"], 2048).astype(np.int32)
    m.forward_logits_cached(kv, 0, prompt)
    ctx.synchronize()
    kv.free()
    m.free()


def case_batched(ctx, d: Path) -> None:
    p = write_synthetic_bundle(d / "b", dict(QWEN3_0_6B, num_hidden_layers=2), seed=0)
    m = R.Model(ctx, p, weight_format=R.WEIGHTS_INT8_G64)
    n = 32
    kv = R.KVCache(m, n, 1100 * n)
    for s in range(n):
        kv.fill_random(s, 1000 + s, 100 + s)
    m.decode(kv, list(range(n)), np.arange(n, dtype=np.int32) * 7)
    m.topk(0, 8)
    ctx.synchronize()
    kv.free()
    m.free()


def case_decode(ctx, d: Path) -> None:
    p = write_synthetic_bundle(d / "b", dict(QWEN3_0_6B, num_hidden_layers=2), seed=0)
    m = R.Model(ctx, p)
    kv = R.KVCache(m, 1, 256)
    prompt = np.random.default_rng(1).integers(0, QWEN3_0_6B["vocab_size"], 16).astype(np.int32)
    m.generate(kv, 0, prompt, 5)
    ctx.synchronize()
    kv.free()
    m.free()


CASES = {"linear": case_linear, "prefill": case_prefill, "batched": case_batched, "decode": case_decode}


def main(argv: list[str]) -> int:
    if len(argv) != 1 or argv[0] not in CASES:
        print("usage: python -m soc_b200.kernel_cases {" + "|".join(CASES) + "}", file=sys.stderr)
        return 2
    ctx = R.Context(0)
    with tempfile.TemporaryDirectory() as tmp:
        fn = CASES[argv[0]]
        if argv[0] == "linear":
            fn(ctx)
        else:
            fn(ctx, Path(tmp))
    ctx.close()
    print("ok", argv[0])
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
