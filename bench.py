"""Benchmark of the B200 Qwen3 forward path (config 0 of the benchmark set).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl soc|reference]

Workload: Qwen3-0.6B architecture, random fp16 weights
N(0, 0.02) seed 0 in the reference bundle format, batch 1, a 16-token prompt of
ids uniform in [0, 151936) seed 1, prefill + 32 greedy decode steps.  One
"step" = that whole generation job (prefill 16 + 32 decode steps, 33 generated
ids).  Metric: decode tokens/s = generated ids per second of job time.

* value        device-timed (CUDA events on the library stream) with the prompt
               already resident in HBM (soc_b200_generate_device);
* e2e          the same job through the public C ABI with host buffers
               (soc_b200_generate: pinned prompt in, ids out, synchronous);
* roofline     the decode step, timed as (job - prefill-only job) / 32: algorithmic
               bytes = every weight byte read once + the KV bytes of the step;
* cpu_baseline the reference CPU runtime (oracle/_ref) on a bounded sample.

N > 1: one process per GPU (torchrun), each running its own replica of the job
("replicas only": batch-1 decode of one sequence does not shard); value sums all
ranks' ids over the max-over-ranks time.  The same line carries, under
"partitioned", the two paths that do split across the GPUs, measured in the same
run: config 3 (256 sequences sharded over the ranks, no collective) and config 4
(Qwen3-8B tensor-parallel over the ranks, NCCL all-reduce after o_proj and
down_proj), each with its own workload, value and roofline.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tokens/s (B=1 & batched) Qwen3-0.6B shape; HBM GB/s vs 8 TB/s"
PROMPT_LEN, NEW_TOKENS = 16, 33  # 1 id from the prefill + 32 decode steps
SPEC_HBM_GBS = 8000.0


def qwen06_bytes_per_decode_step(cfg: dict, ctx_len: int) -> float:
    """Algorithmic HBM bytes of one batch-1 decode step at context ctx_len (keys incl. the new one)."""
    H, I, L, D = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"], cfg["head_dim"]
    hq, hkv, V = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["vocab_size"]
    lin = L * (H * (hq + 2 * hkv) * D + H * hq * D + 3 * H * I)
    weights = 2 * (lin + V * H)                       # fp16 linears + tied lm_head
    norms = 4 * (L * (2 * H + 2 * D) + H)              # fp32 norm vectors
    kv_token = L * 2 * hkv * D * 2                     # fp16 K and V of one position, all layers
    return float(weights + norms + kv_token * ctx_len + kv_token)


def _find_number(d, key):
    """The number stored under `key` at any depth of a JSON object (first found), else None."""
    if isinstance(d, dict):
        v = d.get(key)
        if isinstance(v, (int, float)) and not isinstance(v, bool):
            return float(v)
        for sub in d.values():
            r = _find_number(sub, key)
            if r is not None:
                return r
    return None


def load_peaks() -> dict:
    """Roofline denominators: the driver-measured MEASURED_PEAKS.json when present and readable
    (copy bandwidth `hbm_gbs`, cuBLAS bf16 `bf16_tflops` burst / `bf16_tflops_sustained`), else the
    pool's earlier measurements (6,650 GB/s, 1,590 TFLOP/s), labelled "fallback"."""
    out = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
        except (OSError, ValueError):
            return out
        hbm = _find_number(d, "hbm_gbs")
        if hbm:
            out.update(hbm_gbs=hbm, source="measured")
            for k in ("bf16_tflops", "bf16_tflops_sustained"):
                v = _find_number(d, k)
                if v:
                    out[k] = v
    return out


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.path = Path(tempfile.mkstemp(prefix="clocks", suffix=".csv")[1])

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            self.proc.wait(timeout=10)

    def summary(self) -> dict:
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(parts)
            except ValueError:
                pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def config0_bundle(rank: int, world: int, barrier):
    from soc_b200.bundle import QWEN3_0_6B, cached_bundle
    if rank == 0:
        p = cached_bundle("config0", QWEN3_0_6B, seed=0, dtype="float16")
    barrier()
    if rank != 0:
        p = cached_bundle("config0", QWEN3_0_6B, seed=0, dtype="float16")
    return p


def prompt_ids(cfg) -> np.ndarray:
    return np.random.default_rng(1).integers(0, cfg["vocab_size"], PROMPT_LEN).astype(np.int32)


# ------------------------------------------------------------------ reference arm
def config0_config(world: int) -> dict:
    """The `config` object of the config-0 line (both arms print the same one)."""
    return {"workload": "config0: Qwen3-0.6B fp16 weights, batch 1, 16-token prompt + 32 greedy "
                        "decode steps (33 ids/job), ids seed 1, weights seed 0",
            "global_batch": world, "seq_len": PROMPT_LEN + NEW_TOKENS - 1,
            "parallelism": f"replicas{world}",
            "l2": "weights 1.19 GB per token > 126 MB L2; no flush needed"}


def run_reference(args, rank, world):
    """The reference CPU runtime (its sources compiled unchanged, oracle/_ref) on this host's
    cores, on the config-0 job counted as the GPU arm counts it: 33 ids per job of one
    16-token prefill plus 32 decode steps.  Every host thread runs its own copy of the job:
    the 16-token prefill once (timed; it also builds the thread's cache), then decode steps
    at the job's positions 16..47 (wrapping round to 16 when the warm-up and timed steps
    outrun the window, which rewrites the same cache positions at the same cost).  One timed
    step = one decode token on every thread.  value = threads x 33 / (prefill + 32 x mean
    decode step), the job rate of all threads together."""
    if rank != 0:
        return
    from oracle import oracle as O
    from soc_b200.bundle import QWEN3_0_6B, cached_bundle
    if not O.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libsocref.so was not built"}))
        return
    p = cached_bundle("config0", QWEN3_0_6B, seed=0, dtype="float16")
    cores = O.host_cores()
    threads = max(1, min(cores, int(os.environ.get("SOC_REF_THREADS", "32"))))
    models = [O.RefModel(p, 64) for _ in range(threads)]
    ids = prompt_ids(QWEN3_0_6B)
    toks = [0] * threads
    step_no = [0] * threads
    pf_s = [0.0] * threads
    decode_window = NEW_TOKENS - 1

    def prefill(i):
        t0 = time.perf_counter()
        lg = models[i].forward(ids, 0)
        toks[i] = models[i].sample(lg[-1])
        pf_s[i] = time.perf_counter() - t0

    def step(i):
        pos = PROMPT_LEN + step_no[i] % decode_window
        lg = models[i].forward([toks[i]], pos)
        toks[i] = models[i].sample(lg[0])
        step_no[i] += 1

    def parallel(fn):
        ts = [threading.Thread(target=fn, args=(i,)) for i in range(threads)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()

    parallel(prefill)
    for _ in range(args.warmup):
        parallel(step)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        parallel(step)
    dt = time.perf_counter() - t0
    dec_s = dt / args.steps
    job_s = max(pf_s) + decode_window * dec_s
    value = threads * NEW_TOKENS / job_s
    sample = (f"{threads} threads (of {cores} host cores), each its own config-0 job: the 16-token prefill timed "
              f"once ({max(pf_s):.1f} s, slowest thread), then {args.steps} timed decode steps (after "
              f"{args.warmup} warm-up) at the job's positions 16..47, every thread one token per step; "
              f"job = prefill + 32 x mean step")
    print(json.dumps({
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dec_s * 1000, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": config0_config(world),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "host_cores": cores,
                         "kind": "reference", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "job_s_per_thread": job_s, "prefill_s": max(pf_s), "decode_s_per_token": dec_s,
    }), flush=True)


def cpu_baseline_sample() -> dict:
    """Reference CPU runtime, 1 thread (it is single-threaded), on a bounded sample of
    the config-0 workload: 2-token prompt, then 3 timed decode steps."""
    from oracle import oracle as O
    from soc_b200.bundle import QWEN3_0_6B, cached_bundle
    if not O.ref_available():
        return {"value": None, "unit": "tokens/s", "cores": 1, "kind": "reference",
                "sample": "unavailable: oracle/_ref not built"}
    p = cached_bundle("config0", QWEN3_0_6B, seed=0, dtype="float16")
    rm = O.RefModel(p, 64)
    ids = prompt_ids(QWEN3_0_6B)[:2]
    tok = rm.sample(rm.forward(ids, 0)[-1])
    steps = 3
    t0 = time.perf_counter()
    for i in range(steps):
        tok = rm.sample(rm.forward([tok], 2 + i)[0])
    dt = time.perf_counter() - t0
    return {"value": steps / dt, "unit": "tokens/s", "cores": 1, "host_cores": O.host_cores(), "kind": "reference",
            "sample": f"{steps} decode steps after a 2-token prefill, 1 thread of {O.host_cores()} host cores "
                      f"(the reference runtime is single-threaded)"}


# ----------------------------------------------------------------------- our arm
def run_soc(args, rank, world, local):
    import torch
    import torch.distributed as dist
    from soc_b200 import runtime as R
    from soc_b200.bundle import QWEN3_0_6B

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=900), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    p = config0_bundle(rank, world, barrier)
    ctx = R.Context(local)
    model = R.Model(ctx, p)
    kv = R.KVCache(model, 1, 256)
    stream = torch.cuda.ExternalStream(ctx.stream)
    prompt = prompt_ids(QWEN3_0_6B)
    d_prompt = torch.from_numpy(prompt).cuda()
    d_out = torch.zeros(NEW_TOKENS, dtype=torch.int32, device="cuda")

    def job(max_new=NEW_TOKENS):
        model.generate_device(kv, 0, d_prompt.data_ptr(), PROMPT_LEN, max_new, d_out.data_ptr())

    torch.cuda.synchronize()
    for _ in range(max(args.warmup, 3)):
        job()
        job(1)
    ctx.synchronize()

    def timed(fn, reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        ctx.synchronize()
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        ctx.synchronize()
        torch.cuda.synchronize()
        barrier()
        return e0.elapsed_time(e1)

    launches0 = R.kernel_launches()
    with ClockSampler(local) as clk:
        ms_total = timed(job, args.steps)
    launches = R.kernel_launches() - launches0
    ms_prefill = timed(lambda: job(1), args.steps)
    if world > 1:
        t = torch.tensor([ms_total, ms_prefill], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total, ms_prefill = t.tolist()
    greedy = d_out.cpu().tolist()

    # e2e through the public ABI with host buffers (pinned prompt in, ids out).
    h_prompt = torch.from_numpy(prompt).pin_memory()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        out = model.generate(kv, 0, h_prompt.numpy(), NEW_TOKENS)
    e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = t.item()
    assert out == greedy[: len(out)], "e2e and device runs disagree"

    step_ms = ms_total / args.steps
    decode_ms = (ms_total - ms_prefill) / args.steps / (NEW_TOKENS - 1)
    cfg = QWEN3_0_6B
    ctx_lens = [PROMPT_LEN + i for i in range(NEW_TOKENS - 1)]
    alg_bytes = float(np.mean([qwen06_bytes_per_decode_step(cfg, c) for c in ctx_lens]))
    peaks = load_peaks()
    achieved = alg_bytes / (decode_ms * 1e-3) / 1e9
    traffic = None
    tf = ROOT / "profiles" / "decode_step_traffic.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get("dram_bytes_per_decode_step")

    result = None
    if rank == 0:
        cpu = cpu_baseline_sample() if world == 1 and not args.no_cpu_baseline else None
        result = {
            "metric": METRIC,
            "value": NEW_TOKENS * args.steps * world / (ms_total * 1e-3),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": step_ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f16w-f32a",
            "data": "synthetic",
            "impl": "soc_b200",
            "config": config0_config(world),
            "decode_ms_per_token": decode_ms,
            "prefill_ms": ms_prefill / args.steps,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / peaks["hbm_gbs"], "peak_source": peaks["source"],
                         "frac_of_8TBs": achieved / SPEC_HBM_GBS, "traffic": traffic,
                         "unit_of_work": "one batch-1 decode step (all 28 layers + lm_head + argmax)",
                         "algorithmic_bytes_per_step": alg_bytes},
            "e2e": {"value": NEW_TOKENS * args.steps * world / e2e_s, "unit": "tokens/s",
                    "h2d_bytes_per_step": PROMPT_LEN * 4, "d2h_bytes_per_step": NEW_TOKENS * 4},
            "gpu_launches": int(launches),
            "clocks": clk.summary(),
            "greedy_ids_head": greedy[:8],
        }
        if cpu is not None:
            result["cpu_baseline"] = cpu
    kv.free()
    model.free()
    ctx.close()
    if world > 1 and not args.no_partitioned:
        # The headline `value` above is config 0 (one sequence per GPU: replicas only).  The paths
        # that are partitioned across GPUs are measured in the same run and reported beside it:
        # config 3 with its 256 sequences sharded over the ranks, and config 4 tensor-parallel
        # over the ranks (when the ranks divide the Qwen3-8B heads).
        part = {}
        c3 = config3_measure(rank, world, local, PART_STEPS, 3, C3_SEQS)
        if rank == 0:
            part["config3_sequence_sharded"] = c3
        if 32 % world == 0 and 8 % world == 0:
            c4 = config4_measure(rank, world, local, PART_STEPS, 3)
            if rank == 0:
                part["config4_tensor_parallel"] = c4
        if rank == 0:
            result["partitioned"] = part
    if world > 1:
        dist.destroy_process_group()
    if result is not None:
        print(json.dumps(result), flush=True)


PART_STEPS = 16  # timed steps of each partitioned measurement beside the N > 1 headline


# ------------------------------------------------------------------- config 2
C2_PROMPT, C2_NEW = 2048, 129  # 1 id from the prefill + 128 decode steps


def config2_flops(cfg: dict, n: int) -> float:
    """Algorithmic FLOPs of an n-token causal prefill (linears, attention, last-row lm_head)."""
    H, I, L, D = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"], cfg["head_dim"]
    hq, hkv, V = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["vocab_size"]
    lin = L * (H * (hq + 2 * hkv) * D + H * hq * D + 3 * H * I)
    attn = L * hq * D * 2 * 2 * (n * (n + 1) / 2)  # QK^T and PV over the causal triangle
    return 2.0 * lin * n + attn + 2.0 * V * H


def run_config2(args):
    """Config 2: Qwen3-0.6B fp16 (weights as config 0), one 2048-token prompt (ids seed 3)
    prefilled, then 128 greedy decode steps against the 2048-entry KV cache.  Prints one JSON
    line: prefill time and its tensor-roofline fraction, decode tokens/s at context 2048-2176
    and its HBM-roofline fraction."""
    import torch
    from soc_b200 import runtime as R
    from soc_b200.bundle import QWEN3_0_6B
    torch.cuda.set_device(0)
    p = config0_bundle(0, 1, lambda: None)
    ctx = R.Context(0)
    model = R.Model(ctx, p)
    kv = R.KVCache(model, 1, C2_PROMPT + C2_NEW + 16)
    stream = torch.cuda.ExternalStream(ctx.stream)
    prompt = np.random.default_rng(3).integers(0, QWEN3_0_6B["vocab_size"], C2_PROMPT).astype(np.int32)
    d_prompt = torch.from_numpy(prompt).cuda()
    d_out = torch.zeros(C2_NEW, dtype=torch.int32, device="cuda")

    def job(max_new):
        model.generate_device(kv, 0, d_prompt.data_ptr(), C2_PROMPT, max_new, d_out.data_ptr())

    for _ in range(max(args.warmup, 3)):
        job(C2_NEW)
    ctx.synchronize()

    def timed(max_new, reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ctx.synchronize()
        e0.record(stream)
        for _ in range(reps):
            job(max_new)
        e1.record(stream)
        ctx.synchronize()
        return e0.elapsed_time(e1) / reps

    reps = max(1, min(args.steps, 10))
    launches0 = R.kernel_launches()
    with ClockSampler(0) as clk:
        ms_job = timed(C2_NEW, reps)
        ms_prefill = timed(1, reps)
    launches = (R.kernel_launches() - launches0) // (2 * reps)
    greedy = d_out.cpu().tolist()
    cfg = QWEN3_0_6B
    flops = config2_flops(cfg, C2_PROMPT)
    decode_ms = (ms_job - ms_prefill) / (C2_NEW - 1)
    alg_bytes = float(np.mean([qwen06_bytes_per_decode_step(cfg, C2_PROMPT + i) for i in range(C2_NEW - 1)]))
    peaks = load_peaks()
    tc_peak = peaks["bf16_tflops"]
    hbm = peaks["hbm_gbs"]
    print(json.dumps({
        "workload": "config2: Qwen3-0.6B fp16, prefill 2048 ids (seed 3) + 128 greedy decode steps",
        "prefill_ms": ms_prefill, "prefill_tokens_per_s": C2_PROMPT / (ms_prefill * 1e-3),
        "prefill_tflops": flops / (ms_prefill * 1e-3) / 1e12, "prefill_algorithmic_flop": flops,
        "prefill_frac_of_measured_bf16": flops / (ms_prefill * 1e-3) / 1e12 / tc_peak,
        "decode_ms_per_token": decode_ms, "decode_tokens_per_s": 1e3 / decode_ms,
        "decode_gbs": alg_bytes / (decode_ms * 1e-3) / 1e9,
        "decode_frac_of_measured_hbm": alg_bytes / (decode_ms * 1e-3) / 1e9 / hbm,
        "job_ms": ms_job, "kernels_per_job": int(launches), "clocks": clk.summary(),
        "greedy_ids_head": greedy[:8]}), flush=True)
    kv.free()
    model.free()
    ctx.close()


# ------------------------------------------------------------------- config 3
C3_SEQS, C3_STEPS = 256, 64


def config3_contexts() -> np.ndarray:
    return np.random.default_rng(4).integers(128, 4097, C3_SEQS)


def run_config3(args, rank, world, local):
    """Config 3 on its own (--workload config3): see config3_measure."""
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    result = config3_measure(rank, world, local, args.steps, args.warmup, min(C3_SEQS, args.c3_seqs))
    if world > 1:
        dist.destroy_process_group()
    if result is not None:
        print(json.dumps(result), flush=True)


def config3_measure(rank, world, local, steps, warmup, total):
    """Config 3: batched ragged decode, Qwen3-0.6B with int8 group-64 linears (the config-0
    fp16 weights quantised at load time; embeddings, norms and the tied lm_head stay fp16).
    256 sequences with contexts U[128, 4096] (seed 4) of seeded ~N(0, 1) fp16 KV written on
    the device (soc_b200_kv_fill_random, seed 4000 + sequence index), sequences placed on the
    ranks by soc_b200.sharding.balanced_shards (equal counts, balanced total context),
    `steps` greedy decode steps of every local sequence per timed run (one soc_b200_decode
    call per step: host ids in, host ids out).  Returns the JSON object (rank 0) with the
    max-over-ranks time; with world > 1 the process group must already be initialised."""
    import torch
    import torch.distributed as dist
    from soc_b200 import runtime as R
    from soc_b200.bundle import QWEN3_0_6B
    from soc_b200.sharding import balanced_shards

    def barrier():
        if world > 1:
            dist.barrier()

    cfg = QWEN3_0_6B
    p = config0_bundle(rank, world, barrier)
    ctx = R.Context(local)
    model = R.Model(ctx, p, weight_format=R.WEIGHTS_INT8_G64)
    ctxs = config3_contexts()
    # equal counts per rank and balanced total context (the KV read bounds each step)
    mine = balanced_shards(ctxs[:total], world)[rank]
    n = len(mine)
    warmup = max(warmup, 3)
    cap = int(sum(-(-(int(ctxs[g]) + steps + warmup + 1) // 16) * 16 for g in mine))
    kv = R.KVCache(model, n, cap)
    for i, g in enumerate(mine):
        kv.fill_random(i, int(ctxs[g]), 4000 + g)
    ctx.synchronize()
    toks = np.random.default_rng(5).integers(0, cfg["vocab_size"], C3_SEQS).astype(np.int32)[mine]
    seqs = list(range(n))
    for _ in range(warmup):
        _, toks = model.decode(kv, seqs, toks, want_logits=False)
    stream = torch.cuda.ExternalStream(ctx.stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx_before = np.array([kv.length(i) for i in seqs])
    barrier()
    ctx.synchronize()
    launches0 = R.kernel_launches()
    with ClockSampler(local) as clk:
        e0.record(stream)
        t0 = time.perf_counter()
        for _ in range(steps):
            _, toks = model.decode(kv, seqs, toks, want_logits=False)
        e1.record(stream)
        ctx.synchronize()
        wall = time.perf_counter() - t0
    launches = R.kernel_launches() - launches0
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms, wall], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, wall = t.tolist()
    # algorithmic bytes per step on this rank: int8 linears + fp16 lm_head + the KV read
    H, I, L, D = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"], cfg["head_dim"]
    hq, hkv, V = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["vocab_size"]
    lin = L * (H * (hq + 2 * hkv) * D + H * hq * D + 3 * H * I)
    kv_tok = L * 2 * hkv * D * 2
    mean_ctx = float(np.mean([c + 1 + i for c in ctx_before for i in range(steps)])) if n else 0.0
    bytes_step = lin * (1 + 2 / 64) + 2 * V * H + kv_tok * mean_ctx * n
    achieved = bytes_step * steps / (ms * 1e-3) / 1e9
    peaks = load_peaks()
    result = None
    if rank == 0:
        result = {
            "metric": METRIC, "value": total * steps / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
            "steps": steps, "warmup": warmup, "ms_per_step": ms / steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "i8w-f32a", "data": "synthetic", "impl": "soc_b200",
            "config": {"workload": "config3: 256 sequences, contexts U[128,4096] seed 4, random N(0,1) fp16 KV, "
                                   "Qwen3-0.6B int8 g64 linears, batched greedy decode",
                       "global_batch": total, "seq_len": int(ctxs.max()) + steps + warmup,
                       "parallelism": f"sequence-sharded{world}",
                       "l2": "KV 63 GB per step > 126 MB L2; no flush needed"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / peaks["hbm_gbs"], "peak_source": peaks["source"], "traffic": None,
                         "unit_of_work": "one batched decode step of this rank's sequences",
                         "algorithmic_bytes_per_step_rank0": bytes_step},
            "e2e": {"value": total * steps / wall, "unit": "tokens/s", "h2d_bytes_per_step": 8 * n,
                    "d2h_bytes_per_step": 4 * n},
            "gpu_launches": int(launches), "clocks": clk.summary(),
        }
    kv.free()
    model.free()
    ctx.close()
    return result


# ------------------------------------------------------------------- config 4
C4_BATCH, C4_CTX = 32, 2048


def run_config4(args, rank, world, local):
    """Config 4 on its own (--workload config4): see config4_measure."""
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    result = config4_measure(rank, world, local, args.steps, args.warmup)
    if world > 1:
        dist.destroy_process_group()
    if result is not None:
        print(json.dumps(result), flush=True)


def config4_measure(rank, world, local, steps, warmup):
    """Config 4: Qwen3-8B architecture, random bf16 weights N(0, 0.02) seed 5 (drawn by
    torch.randn on the GPU: 8.2 G values), tensor
    parallel over the ranks (TP = --gpus: heads and FFN columns sharded, all-reduce of the
    residual stream after o_proj and down_proj, vocab-parallel lm_head).  Batch 32 decode at
    context 2048 of seeded ~N(0, 1) KV (soc_b200_kv_fill_random, seed 5000 + sequence), one
    soc_b200_decode call per step.  Returns the JSON object (rank 0), max-over-ranks time; with
    world > 1 the process group must already be initialised."""
    import torch
    import torch.distributed as dist
    from soc_b200 import runtime as R
    from soc_b200.bundle import QWEN3_8B, cached_bundle

    def barrier():
        if world > 1:
            dist.barrier()

    cfg = QWEN3_8B
    if rank == 0:
        p = cached_bundle("config4_qwen3_8b_bf16", cfg, seed=5, dtype="bfloat16", torch_device="cuda")
    barrier()
    if rank != 0:
        p = cached_bundle("config4_qwen3_8b_bf16", cfg, seed=5, dtype="bfloat16", torch_device="cuda")
    ctx = R.Context(local)
    comm = R.tensor_parallel_comm(ctx) if world > 1 else None
    model = R.Model(ctx, p, tp_rank=rank, tp_size=world, comm=comm)
    warmup = max(warmup, 3)
    kv = R.KVCache(model, C4_BATCH, C4_BATCH * (C4_CTX + steps + warmup + 16))
    for s in range(C4_BATCH):
        kv.fill_random(s, C4_CTX, 5000 + s)
    ctx.synchronize()
    toks = np.random.default_rng(6).integers(0, cfg["vocab_size"], C4_BATCH).astype(np.int32)
    seqs = list(range(C4_BATCH))
    for _ in range(warmup):
        _, toks = model.decode(kv, seqs, toks, want_logits=False)
    stream = torch.cuda.ExternalStream(ctx.stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    ctx.synchronize()
    launches0 = R.kernel_launches()
    with ClockSampler(local) as clk:
        e0.record(stream)
        t0 = time.perf_counter()
        for _ in range(steps):
            _, toks = model.decode(kv, seqs, toks, want_logits=False)
        e1.record(stream)
        ctx.synchronize()
        wall = time.perf_counter() - t0
    launches = R.kernel_launches() - launches0
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms, wall], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, wall = t.tolist()
    H, I, L, D = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"], cfg["head_dim"]
    hq, hkv, V = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["vocab_size"]
    params = L * (H * (hq + 2 * hkv) * D + H * hq * D + 3 * H * I) + V * H
    mean_ctx = C4_CTX + warmup + (steps + 1) / 2
    bytes_rank = (2 * params + C4_BATCH * mean_ctx * L * 2 * hkv * D * 2) / world
    achieved = bytes_rank * steps / (ms * 1e-3) / 1e9
    peaks = load_peaks()
    result = None
    if rank == 0:
        result = {
            "metric": METRIC, "value": C4_BATCH * steps / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
            "steps": steps, "warmup": warmup, "ms_per_step": ms / steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16w-f32a", "data": "synthetic", "impl": "soc_b200",
            "config": {"workload": "config4: Qwen3-8B bf16 seed 5, batch 32 decode, context 2048 random N(0,1) KV",
                       "global_batch": C4_BATCH, "seq_len": C4_CTX + steps + warmup, "parallelism": f"tp{world}",
                       "l2": "weights 15.1 GB + KV 9.8 GB per step > 126 MB L2; no flush needed"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / peaks["hbm_gbs"], "peak_source": peaks["source"], "traffic": None,
                         "unit_of_work": "one batch-32 decode step, bytes held by one rank",
                         "algorithmic_bytes_per_step_per_rank": bytes_rank},
            "e2e": {"value": C4_BATCH * steps / wall, "unit": "tokens/s", "h2d_bytes_per_step": 8 * C4_BATCH,
                    "d2h_bytes_per_step": 4 * C4_BATCH},
            "gpu_launches": int(launches), "clocks": clk.summary(),
        }
    kv.free()
    model.free()
    R.Context.nccl_comm_destroy(comm)
    ctx.close()
    return result


# ------------------------------------------------------------- config 1 sweep
SWEEP_SHAPES = {"q_proj": (2048, 1024), "k_proj": (1024, 1024), "o_proj": (1024, 2048), "gate_proj": (3072, 1024),
                "down_proj": (1024, 3072), "lm_head": (151936, 1024)}
SWEEP_FORMATS = ("fp16", "int8_g64", "int4_g32")
SWEEP_BATCHES = (1, 4, 16, 64)


def run_linear_sweep(args):
    """Config 1: y = W x for every 0.6B linear shape x {fp16, int8 g64, int4 g32} x batch
    {1, 4, 16, 64}, x ~ N(0, 1) seed 2, W ~ N(0, 0.02).  One JSON line per case: device time
    of one soc_b200_linear launch (CUDA events over `steps` launches that rotate through
    enough weight copies to exceed the 126 MB L2) and its algorithmic bytes / time."""
    import torch
    from soc_b200 import runtime as R
    torch.cuda.set_device(0)
    ctx = R.Context(0)
    peaks = load_peaks()
    fmt_code = {"fp16": R.WEIGHTS_F16, "int8_g64": R.WEIGHTS_INT8_G64, "int4_g32": R.WEIGHTS_INT4_G32}
    g = torch.Generator(device="cuda").manual_seed(2)
    stream = torch.cuda.ExternalStream(ctx.stream)  # the library's stream: events and launches on it
    for name, (out_f, in_f) in SWEEP_SHAPES.items():
        w32 = torch.randn(out_f, in_f, device="cuda", generator=g) * 0.02
        for fmt in SWEEP_FORMATS:
            if fmt == "fp16":
                wq, sc = w32.half().view(torch.uint8), None
            else:
                grp, qmax = (64, 127.0) if fmt == "int8_g64" else (32, 7.0)
                wg = w32.view(out_f, in_f // grp, grp)
                sc = (wg.abs().amax(-1) / qmax).half()
                q = torch.round(wg / sc.float().clamp_min(1e-30)[..., None]).clamp(-qmax, qmax).to(torch.int8)
                q = q.view(out_f, in_f)
                if fmt == "int4_g32":
                    q = ((q[:, 0::2] & 0xF) | ((q[:, 1::2] & 0xF) << 4)).to(torch.uint8)
                wq = q.view(torch.uint8).contiguous()
            wbytes = wq.numel() + (sc.numel() * 2 if sc is not None else 0)
            copies = max(1, min(256, -(-(256 << 20) // wbytes)))
            ws = [wq.clone() for _ in range(copies)] if copies > 1 else [wq]
            ss = [sc.clone() for _ in range(copies)] if (sc is not None and copies > 1) else [sc] * len(ws)
            for batch in SWEEP_BATCHES:
                x = torch.randn(batch, in_f, device="cuda", generator=g)
                y = torch.empty(batch, out_f, device="cuda")

                def launch(i):
                    ctx.linear(fmt_code[fmt], ws[i % len(ws)].data_ptr(),
                               ss[i % len(ss)].data_ptr() if ss[0] is not None else None,
                               out_f, in_f, x.data_ptr(), batch, y.data_ptr(), stream.cuda_stream)

                for i in range(max(args.warmup, 3)):
                    launch(i)
                reps = max(args.steps, len(ws))
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                ctx.synchronize()
                with torch.cuda.stream(stream):
                    # keep the GPU busy while the host queues the launches, so the events
                    # time the kernels and not the host's launch rate
                    torch.cuda._sleep(4_000_000)
                    e0.record(stream)
                    for i in range(reps):
                        launch(i)
                    e1.record(stream)
                ctx.synchronize()
                us = e0.elapsed_time(e1) * 1e3 / reps
                alg = wbytes + 4 * batch * (in_f + out_f)
                gbs = alg / (us * 1e-6) / 1e9
                print(json.dumps({"workload": "config1-linear", "shape": name, "out": out_f, "in": in_f, "format": fmt,
                                  "batch": batch, "us": round(us, 3), "algorithmic_bytes": alg,
                                  "gbs": round(gbs, 1), "frac_of_measured_hbm": round(gbs / peaks["hbm_gbs"], 4),
                                  "gflops": round(2 * out_f * in_f * batch / (us * 1e-6) / 1e9, 1),
                                  "l2_rotation_copies": len(ws)}), flush=True)
            del ws, ss
        del w32
        torch.cuda.empty_cache()
    ctx.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="soc", choices=["soc", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-partitioned", action="store_true",
                    help="N > 1: skip the config-3 (sequence-sharded) and config-4 (tensor-parallel) measurements")
    ap.add_argument("--workload", default="config0", choices=["config0", "linear-sweep", "config2", "config3", "config4"],
                    help="config0 (the headline line), linear-sweep (config 1, one line per case), config2, "
                         "config3 (batched ragged decode, sequence-sharded over --gpus), "
                         "config4 (Qwen3-8B batch-32 decode, tensor-parallel over --gpus)")
    ap.add_argument("--c3-seqs", type=int, default=C3_SEQS,
                    help="config3: number of the 256 sequences to run (a smaller case for profiling)")
    args = ap.parse_args()
    rank, world, local = dist_env()
    if args.workload == "linear-sweep":
        run_linear_sweep(args)
        return
    if args.workload == "config2":
        run_config2(args)
        return
    if args.workload == "config3":
        run_config3(args, rank, world, local)
        return
    if args.workload == "config4":
        run_config4(args, rank, world, local)
        return
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_soc(args, rank, world, local)


if __name__ == "__main__":
    main()
