#!/usr/bin/env python3
"""Benchmark: Qwen2.5-1.5B W8 greedy decode tokens/s on B200 (28 layers, batch 1 per GPU,
512-token prompt of uniform-random ids, then greedy decode steps; synthetic seeded weights).

  python bench.py [--gpus N --steps K --warmup W] [--impl b200|reference]

One JSON line on rank 0. A "step" is one greedy decode step of the full model for the sequence each GPU
holds (embedding -> 28 decoder layers -> final norm -> LM head -> argmax); with N GPUs each rank decodes its
own independent sequence (weak scaling) and the next-token ids are all-gathered over NCCL every step.

value : device-resident decode loop (token ids stay on the GPU; one CUDA-graph launch per step), timed
        with CUDA events on the engine stream, max over ranks.
e2e   : the same steps through the engine's C-ABI call with host token buffers (H2D of the step's input
        token, D2H of the argmax inside the timed region).
With N GPUs the engines all-gather each step's next-token ids over NCCL from C++ (qwen_engine_gather_tokens_async, on a side stream beside the next step).

Sub-records, each with its own time and roofline (work counts from work_llm_accelerator_b200.performance_model):
  batched       config 3: 64 sequences x 2048-token history, greedy steps; 64/N sequences per GPU (strong scaling)
  prefill_4096  config 4: 8 prompts of 4096 tokens through 28 layers; 8/N per GPU (strong scaling), tensor roofline
  prefill_128   config 1's length through the 28-layer engine (one prompt per GPU)
  layer_abi     configs 0 and 1 through the drop-in C-ABI (qwen_decode_top_smoke_forward_w8 /
                qwen_prefill_top_smoke_forward_w8) with host buffers, plus config 0's device time with the
                28 layers' weights rotated (HBM, not L2)
The reference arm (--impl reference) times the reference's own host library (oracle/_ref, built from the
reference sources; int4 weights, its only format) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PROMPT = 512
SEED = 2024
HIDDEN, INTER, KV_WIDTH, LAYERS, VOCAB = 1536, 8960, 256, 28, 151936
METRIC = "Qwen2.5-1.5B W8 decode tok/s (bs1, bs64) & prefill tok/s; % of HBM roofline"


from work_llm_accelerator_b200 import performance_model as pm  # noqa: E402

DTYPE_W8 = ("f32 activations, each token row rounded to 24-bit fixed point (step * X, |X| <= 8355711, three "
            "int8 digit planes) for the int8 tensor cores; int8 weights; exact int32 accumulation; fp32/f64 epilogue")


def step_bytes(wbits: int, history: float) -> float:
    """Algorithmic HBM bytes of one batch-1 decode step (performance_model.decode_step_bytes)."""
    return pm.decode_step_bytes(wbits, history)


def layers_bytes(wbits: int, history: float) -> float:
    """Algorithmic HBM bytes of the 28-layer part of one batch-1 step (the persistent kernel)."""
    return pm.decode_layers_bytes(wbits, history)


def lm_head_bytes() -> float:
    """Algorithmic HBM bytes of the final norm + fp16 LM head + argmax (batch 1)."""
    return pm.lm_head_bytes()


def bench_config(world: int, warmup: int, steps: int, wbits: int) -> dict:
    """The workload both arms report: batch 1 per GPU after a 512-token prompt."""
    sb = step_bytes(wbits, PROMPT + warmup + steps / 2)
    return {"workload": "config2_decode_bs1", "model": "Qwen2.5-1.5B (28 layers, random init)",
            "global_batch": world, "seq_len": PROMPT, "prompt": PROMPT,
            "history_during_timing": [PROMPT + warmup, PROMPT + warmup + steps],
            "parallelism": f"dp{world} (independent sequences)",
            "l2": f"inputs larger than L2: {sb / 1e9:.2f} GB of weights/KV per step vs 126 MB L2",
            "wbits": wbits}


def peaks() -> tuple[float, str]:
    pk = pm.load_peaks()
    return pk.hbm_gbs, pk.source


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# --------------------------------------------------------------------------------------------------
# CPU legs (oracle / reference host library), imported only here and in tests
# --------------------------------------------------------------------------------------------------
def _ref_worker(args):
    """One process of the reference arm: `layers` layers of a W4 decode step through the reference's
    qwen_decode_top_smoke_forward, as the reference caller does it (verification/real_host_top_backend.py:
    290-336), repeated warmup + steps times; returns seconds per step."""
    layers, steps, warmup, proc = args
    sys.path.insert(0, str(ROOT / "oracle"))
    import qwen_oracle as qo

    ref = qo.RefLibs()
    ddrs = [qo.synth_layer(SEED, l, 4).ddr() for l in range(layers)]
    past = PROMPT
    kvs = []
    for l in range(layers):
        k = qo.synth(SEED + proc, qo.STREAM_ACT + 10 + 2 * l, past * KV_WIDTH)
        v = qo.synth(SEED + proc, qo.STREAM_ACT + 11 + 2 * l, past * KV_WIDTH)
        kvs.append((k, v))
    x = qo.synth(SEED + proc, qo.STREAM_ACT, HIDDEN)
    sram = qo.sram_ports()

    def one_step():
        h = x
        for l in range(layers):
            wd, sd = ddrs[l]
            kv_stride = (past + 1) * KV_WIDTH
            kv = np.zeros(2 * kv_stride, np.float32)
            kv[:past * KV_WIDTH] = kvs[l][0]
            kv[kv_stride:kv_stride + past * KV_WIDTH] = kvs[l][1]
            act = np.zeros(2 * HIDDEN, np.float32)
            act[:HIDDEN] = h
            st = ref.decode.qwen_decode_top_smoke_forward(l, past, 0, HIDDEN * 4, 0, 0, 0, kv_stride * 4, wd, sd, kv,
                                                          act, *sram)
            assert st == 0
            h = qo.round_bf16(act[HIDDEN:])

    for _ in range(warmup):
        one_step()
    t = time.perf_counter()
    for _ in range(steps):
        one_step()
    return (time.perf_counter() - t) / steps


def run_reference(args) -> dict:
    import multiprocessing as mp

    sys.path.insert(0, str(ROOT / "oracle"))
    import qwen_oracle as qo

    if not qo.REF_DECODE_LIB.exists():
        return {"impl": "reference", "unavailable": "reference host library not built (make -C oracle ref)"}
    cores = os.cpu_count() or 1
    # bounded sample: layers per step chosen so that the whole run stays near two minutes of wall time
    per_layer_s = 0.07
    layers = int(max(1, min(4, 120.0 / max(1, args.steps + args.warmup) / per_layer_s)))
    procs = cores
    ctx = mp.get_context("spawn")
    with ctx.Pool(procs) as pool:
        secs = pool.map(_ref_worker, [(layers, args.steps, args.warmup, p) for p in range(procs)])
    sec_sampled = statistics.median(secs)  # measured: `layers` layers of one decode step, per process
    sec_per_token = sec_sampled * LAYERS / layers
    value = procs / sec_per_token
    sample = (f"reference host library (oracle/_ref/libqwen_decode_stub.so, int4 weights: its only format), "
              f"{procs} concurrent single-threaded processes (all host cores), each one batch-1 sequence at history "
              f"{PROMPT}; each step times {layers} of 28 decoder layers through qwen_decode_top_smoke_forward; "
              f"value = aggregate tokens/s extrapolated to 28 layers (x{LAYERS / layers:g}); embedding/LM head "
              f"excluded")
    cfg = bench_config(args.gpus, args.warmup, args.steps, 4)
    cfg.update({"layers_timed_per_step": layers, "lm_head": "excluded", "embedding": "excluded",
                "processes": procs})
    return {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": sec_sampled * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 activations x int4 weights (fp32 serial sums)", "data": "synthetic",
        "config": cfg,
        "extrapolation": {"what": f"ms_per_step is the measured time of {layers} of the 28 layers of one decode "
                                  f"step (per process); value scales it to the 28-layer step",
                          "layers_timed": layers, "factor": LAYERS / layers,
                          "ms_per_token_extrapolated": sec_per_token * 1e3},
        "impl": "reference",
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": procs, "kind": "reference", "sample": sample},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def cpu_baseline_port(wbits: int, budget_s: float = 12.0) -> dict:
    """The oracle's C restatement (W8 codes, OpenMP over output rows, all cores) on a bounded sample:
    4 of the 28 decoder layers per step at history 512, scaled to 28, plus one LM head pass."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import qwen_oracle as qo

    layers = 4
    params = [qo.synth_layer(SEED, l, wbits) for l in range(layers)]
    past = PROMPT
    kvs = [(qo.synth(SEED, qo.STREAM_ACT + 10 + l, past * KV_WIDTH), qo.synth(SEED, qo.STREAM_ACT + 40 + l,
                                                                              past * KV_WIDTH)) for l in range(layers)]
    x = qo.synth(SEED, qo.STREAM_ACT, HIDDEN)

    def one():
        h = x
        for l in range(layers):
            kc = np.zeros((past + 1) * KV_WIDTH, np.float32)
            vc = kc.copy()
            kc[:past * KV_WIDTH] = kvs[l][0]
            vc[:past * KV_WIDTH] = kvs[l][1]
            st, out = qo.decode_layer(params[l], h, past, kc, vc)
            h = qo.round_bf16(out)
        return h

    one()
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 3:
        t = time.perf_counter()
        h = one()
        times.append(time.perf_counter() - t)
    embed = qo.synth_embedding(SEED)
    norm = qo.synth_final_norm(SEED)
    t = time.perf_counter()
    qo.lm_head_argmax(h, norm, embed)
    t_lm = time.perf_counter() - t
    sec = statistics.median(times) * LAYERS / layers + t_lm
    cores = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    return {"value": 1.0 / sec, "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"oracle C restatement, W{wbits} codes, OpenMP over output rows on {cores} threads; "
                      f"{len(times)} steps of 4 of 28 layers at history {PROMPT} (scaled x7) + 1 LM head pass"}


# --------------------------------------------------------------------------------------------------
# B200 arm
# --------------------------------------------------------------------------------------------------
def _events(torch):
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def sub_batched(host, torch, args, world, rank, local, clocks_on: bool) -> dict:
    """Config 3: 64 sequences with a 2048-token history, greedy steps; this rank decodes its share."""
    from work_llm_accelerator_b200.parallel import connect_engine, shard_range

    total_seqs, hist = 64, 2048
    a, b = shard_range(total_seqs, world, rank)
    n = b - a
    steps, warmup = args.steps, args.warmup
    eng = host.Engine(local, 8, max_seqs=n, max_len=hist + warmup + steps + 64)
    try:
        if world > 1:
            connect_engine(eng, world, rank, device=f"cuda:{local}")
        eng.init_synthetic(SEED)
        rng = np.random.default_rng(SEED + 1000 + a)
        eng.set_option("graphs", 0)  # history prefills run once each: no capture
        firsts = [eng.prefill(i, rng.integers(0, VOCAB, hist).astype(np.int32)) for i in range(n)]
        eng.set_option("graphs", 1)
        stream = torch.cuda.ExternalStream(eng.stream())
        slots = list(range(n))
        bufs = [torch.tensor(firsts, dtype=torch.int32, device="cuda"), torch.zeros(n, dtype=torch.int32, device="cuda")]
        gathered = torch.zeros(world * n, dtype=torch.int32, device="cuda")

        def step(i):
            eng.decode_device(slots, bufs[i % 2].data_ptr(), bufs[(i + 1) % 2].data_ptr())
            if world > 1:
                eng.gather_tokens(bufs[(i + 1) % 2].data_ptr(), n, gathered.data_ptr())

        with torch.cuda.stream(stream):
            for i in range(warmup):
                step(i)
            stream.synchronize()
            if world > 1:
                torch.distributed.barrier()
            clk = ClockSampler(local) if clocks_on else None
            if clk:
                clk.start()
                time.sleep(0.2)
            e0, e1 = _events(torch)
            e0.record(stream)
            for i in range(warmup, warmup + steps):
                step(i)
            e1.record(stream)
            e1.synchronize()
            clocks = clk.stop() if clk else None
        ms = e0.elapsed_time(e1) / steps
        kernels = eng.kernels_per_decode_step(n)
        torch.cuda.synchronize()
        del bufs, gathered, stream
    finally:
        eng.close()
    return {"ms": ms, "n_local": n, "history_mid": hist + warmup + steps / 2, "clocks": clocks, "kernels": kernels}


def sub_prefill(host, torch, local, seq_len: int, n_seqs: int, reps: int, seed: int) -> dict:
    """n_seqs prompts of seq_len tokens through the 28-layer engine, repeated `reps` times after one pass that
    captures each slot's CUDA graph; device time per repetition (CUDA events on the engine stream)."""
    eng = host.Engine(local, 8, max_seqs=n_seqs, max_len=seq_len + 8)
    try:
        eng.init_synthetic(SEED)
        rng = np.random.default_rng(seed)
        prompts = [rng.integers(0, VOCAB, seq_len).astype(np.int32) for _ in range(n_seqs)]

        def one_pass():
            for i in range(n_seqs):
                eng.reset(i)
                eng.prefill(i, prompts[i])

        one_pass()  # eager + capture per slot
        one_pass()  # warm replay
        stream = torch.cuda.ExternalStream(eng.stream())
        e0, e1 = _events(torch)
        e0.record(stream)
        for _ in range(reps):
            one_pass()
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / reps
        del stream
    finally:
        eng.close()
    return {"ms": ms}


def sub_layer_abi(host, reps: int) -> dict:
    """Configs 0 and 1 through the drop-in C-ABI with host DDR images (H2D of the layer's parameters and
    activations and D2H of the outputs inside every call), W8 codes."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import qwen_oracle as qo

    dec = host.load_decode_lib()
    pre = host.load_prefill_lib()
    p = qo.synth_layer(SEED, 0, 8)
    wd, sd = p.ddr()
    out = {}
    past = 128
    kv_stride = (past + 1) * KV_WIDTH
    kv = np.zeros(2 * kv_stride, np.float32)
    kv[:past * KV_WIDTH] = qo.synth(SEED, qo.STREAM_ACT + 1, past * KV_WIDTH)
    kv[kv_stride:kv_stride + past * KV_WIDTH] = qo.synth(SEED, qo.STREAM_ACT + 2, past * KV_WIDTH)
    act = np.zeros(2 * HIDDEN, np.float32)
    act[:HIDDEN] = qo.synth(SEED, qo.STREAM_ACT, HIDDEN)
    sram = qo.sram_ports()

    def dcall():
        st = dec.qwen_decode_top_smoke_forward_w8(0, past, 0, HIDDEN * 4, 0, 0, 0, kv_stride * 4, wd, sd, kv, act, *sram)
        assert st == 0, st

    for _ in range(3):
        dcall()
    t = time.perf_counter()
    for _ in range(reps):
        dcall()
    out["decode_ms"] = (time.perf_counter() - t) * 1e3 / reps
    # the bytes the call copies in: the layer's codes and fp32 vectors, the K/V history, the input row
    out["decode_h2d_bytes"] = int(pm.layer_param_bytes(8) + 2 * past * KV_WIDTH * 4 + HIDDEN * 4)
    S = 128
    acts = np.zeros(3 * S * HIDDEN, np.float32)
    acts[:S * HIDDEN] = qo.synth(SEED, qo.STREAM_ACT, S * HIDDEN)
    kvp = np.zeros(2 * S * KV_WIDTH, np.float32)

    def pcall():
        st = pre.qwen_prefill_top_smoke_forward_w8(0, S, *qo.tiles_tuple(), 0, S * HIDDEN * 4, 0, 0, 0,
                                                    S * KV_WIDTH * 4, wd, sd, kvp, acts, *sram)
        assert st == 0, st

    for _ in range(3):
        pcall()
    t = time.perf_counter()
    for _ in range(reps):
        pcall()
    out["prefill_ms"] = (time.perf_counter() - t) * 1e3 / reps
    out["prefill_h2d_bytes"] = int(pm.layer_param_bytes(8) + S * HIDDEN * 4)
    return out


def run_b200(args, world: int, rank: int, local: int) -> dict | None:
    import torch
    import torch.distributed as dist

    from work_llm_accelerator_b200 import host
    from work_llm_accelerator_b200.parallel import connect_engine, max_over_ranks, shard_range

    torch.cuda.set_device(local)
    os.environ["QWEN_B200_DEVICE"] = str(local)
    wbits = args.wbits
    total_steps = args.warmup + args.steps
    max_len = PROMPT + 2 * total_steps + 3 + 32 + 64  # device loop, e2e steps, per-kernel profile, margin
    eng = host.Engine(local, wbits, max_seqs=1, max_len=max_len)
    if world > 1:
        connect_engine(eng, world, rank, device=f"cuda:{local}")
    eng.init_synthetic(SEED)
    rng = np.random.default_rng(SEED + rank)
    prompt = rng.integers(0, VOCAB, PROMPT).astype(np.int32)
    first = eng.prefill(0, prompt)

    stream = torch.cuda.ExternalStream(eng.stream())
    bufs = [torch.tensor([first], dtype=torch.int32, device="cuda"), torch.zeros(1, dtype=torch.int32, device="cuda")]
    gathered = torch.zeros(world, dtype=torch.int32, device="cuda")


    def dev_step(i):
        eng.decode_device([0], bufs[i % 2].data_ptr(), bufs[(i + 1) % 2].data_ptr())
        if world > 1:  # the step's token ids of every rank, over NCCL from the engine (C++), on a side stream
            eng.gather_tokens_async(bufs[(i + 1) % 2].data_ptr(), 1, gathered.data_ptr())

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            dev_step(i)
        if world > 1:
            eng.gather_join()
        stream.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        clocks = ClockSampler(local)
        clocks.start()
        time.sleep(0.3)
        ev0, ev1 = _events(torch)
        ev0.record(stream)
        for i in range(args.warmup, args.warmup + args.steps):
            dev_step(i)
        if world > 1:  # the timed region ends after the last gather
            eng.gather_join()
        ev1.record(stream)
        ev1.synchronize()
        clk = clocks.stop()
    ms = ev0.elapsed_time(ev1) / args.steps
    history_mid = PROMPT + args.warmup + args.steps / 2

    # e2e: host token in, host argmax out, through the engine C-ABI (and the NCCL gather with N GPUs)
    cur = int(bufs[(args.warmup + args.steps) % 2].item())
    host_tok = torch.zeros(1, dtype=torch.int32).pin_memory()
    dev_tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    with torch.cuda.stream(stream):
        for _ in range(3):
            cur = int(eng.decode([0], [cur])[0])
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = _events(torch)
        e0.record(stream)
        for _ in range(args.steps):
            cur = int(eng.decode([0], [cur])[0])
            if world > 1:
                host_tok[0] = cur
                dev_tok.copy_(host_tok, non_blocking=True)
                eng.gather_tokens(dev_tok.data_ptr(), 1, gathered.data_ptr())
        e1.record(stream)
        e1.synchronize()
    ms_e2e = e0.elapsed_time(e1) / args.steps

    # per-kernel device time over the same histories: the 28-layer kernel and the LM head, each timed with
    # CUDA events on the engine stream (eager launches, otherwise the same work as one graph step)
    prof = eng.profile_decode(0, cur, max(8, min(args.steps, 32)))
    # config 0's device time: one decode layer's five kernels at history 128, the 28 layers' weights rotated
    # (so they stream from HBM); uses scratch positions of slot 0 after the timed steps
    layer_prof = eng.profile_kernels(1, 128, 56)
    kernels = eng.kernels_per_decode_step(1) + 1  # + the position-advance kernel
    # Tensors that were used on the engine's stream must be released while that stream still exists.
    torch.cuda.synchronize()
    del bufs, gathered, host_tok, dev_tok, stream
    import gc

    gc.collect()
    torch.cuda.synchronize()
    eng.close()

    # ---- sub-records (every rank runs the same steps) ----
    bat = sub_batched(host, torch, args, world, rank, local, clocks_on=True)
    a4, b4 = shard_range(8, world, rank)
    p4096 = sub_prefill(host, torch, local, 4096, b4 - a4, reps=max(1, min(args.steps, 4)), seed=SEED + 77 + a4)
    p128 = sub_prefill(host, torch, local, 128, 1, reps=max(4, min(args.steps, 16)), seed=SEED + 55 + rank)
    abi = sub_layer_abi(host, reps=max(5, min(args.steps, 20)))

    dev = f"cuda:{local}"
    ms, ms_e2e, bat_ms, p4096_ms, p128_ms = max_over_ranks([ms, ms_e2e, bat["ms"], p4096["ms"], p128["ms"]],
                                                           device=dev)
    if rank != 0:
        return None

    peak, peak_kind = peaks()
    pk = pm.load_peaks()
    hist_prof = history_mid + args.steps  # histories of the profiled steps (after the e2e steps)
    lb = layers_bytes(wbits, hist_prof)
    layers_achieved = lb / (prof["layers"] * 1e-3) / 1e9
    head_achieved = lm_head_bytes() / (prof["lm_head"] * 1e-3) / 1e9
    sb = step_bytes(wbits, history_mid)
    step_achieved = sb / (ms * 1e-3) / 1e9
    traffic = None
    tr = ROOT / "profiles" / "decode_bs1_w8_bs1_dram.json"
    if tr.exists() and wbits == 8:
        d = json.loads(tr.read_text())
        traffic = d.get("dram_bytes_per_launch")

    # batched: bytes of this rank's step (its sequences' KV, the replicated weights and LM head)
    bat_bytes = pm.decode_step_bytes(8, bat["history_mid"], bat["n_local"])
    ceiling = pm.decode_step_bytes(8, 2048, 64) / pm.decode_step_bytes(8, 2048, 8)
    batched = {
        "workload": "config3_decode_bs64_hist2048", "value": 64 / (bat_ms * 1e-3), "unit": "tok/s",
        "ms_per_step": bat_ms, "steps": args.steps, "warmup": args.warmup, "sequences": 64,
        "sequences_per_gpu": bat["n_local"], "scaling": "strong", "history_during_timing": [2048 + args.warmup,
                                                                                         2048 + args.warmup + args.steps],
        "l2": f"inputs larger than L2: {bat_bytes / 1e9:.2f} GB per step per GPU",
        "roofline": pm.roofline(bat_bytes, bat_ms * 1e-3, "hbm", pk),
        "hbm_scaling_ceiling_1_to_8": ceiling,
        "gpu_launches": bat["kernels"] * args.steps, "clocks": bat["clocks"],
    }
    batched["roofline"]["kernel"] = "whole step (one CUDA graph: many-token int8 tensor-core GEMMs, paged attention)"
    n4 = b4 - a4
    f4 = pm.prefill_flops(4096)["total"] * n4
    prefill_4096 = {
        "workload": "config4_prefill_4096", "value": 8 * 4096 / (p4096_ms * 1e-3), "unit": "tok/s",
        "ms_per_repetition": p4096_ms, "prompts": 8, "prompts_per_gpu": n4, "scaling": "strong",
        "roofline": pm.roofline(f4, p4096_ms * 1e-3, "tensor", pk, sustained=True),
        "flops_per_gpu": f4, "flops_counted": "2 per projection MAC + causal attention (QK^T and PV)",
    }
    prefill_4096["roofline"]["kernel"] = "28-layer prefill (CUDA graph)"
    b128 = pm.prefill_model_bytes(8, 128)
    prefill_128 = {
        "workload": "config1_length_128_through_28_layers", "value": world * 128 / (p128_ms * 1e-3),
        "unit": "tok/s", "ms_per_prefill": p128_ms, "scaling": "weak",
        "roofline": pm.roofline(b128, p128_ms * 1e-3, "hbm", pk),
        "tensor_roofline": pm.roofline(pm.prefill_flops(128)["total"], p128_ms * 1e-3, "tensor", pk),
    }
    prefill_128["roofline"]["kernel"] = "28-layer prefill (CUDA graph)"
    layer_dev_ms = sum(layer_prof[k] for k in ("qkv", "attention", "o", "gate_up", "down"))
    layer_abi = {
        "workload": "config0_decode_layer_hist128 / config1_prefill_layer_128 through the drop-in C-ABI",
        "decode_e2e": {"value": 1e3 / abi["decode_ms"], "unit": "layer-steps/s", "ms": abi["decode_ms"],
                       "h2d_bytes_per_call": abi["decode_h2d_bytes"], "d2h_bytes_per_call": HIDDEN * 4 + 2 * 1024,
                       "call": "qwen_decode_top_smoke_forward_w8, host DDR images"},
        "decode_device": {"ms": layer_dev_ms, "kernels_ms": {k: layer_prof[k] for k in
                                                            ("qkv", "attention", "o", "gate_up", "down")},
                          "weights": "28 layers rotated (HBM, not L2)",
                          "roofline": pm.roofline(pm.decode_layer_bytes(8, 128), layer_dev_ms * 1e-3, "hbm", pk)},
        "prefill_e2e": {"value": 128 / (abi["prefill_ms"] * 1e-3), "unit": "tok/s", "ms": abi["prefill_ms"],
                        "h2d_bytes_per_call": abi["prefill_h2d_bytes"],
                        "call": "qwen_prefill_top_smoke_forward_w8, host DDR images, 128 tokens"},
    }
    out = {
        "metric": METRIC,
        "value": world / (ms * 1e-3),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": DTYPE_W8 if wbits == 8 else "f32 activations x int4 weights",
        "data": "synthetic: seeded N(0,0.02) weights quantized per channel, uniform-random prompt ids",
        "config": bench_config(world, args.warmup, args.steps, wbits),
        "e2e": {"value": world / (ms_e2e * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": 12, "d2h_bytes_per_step": 4},
        "roofline": {"bound": "hbm",
                     "kernel": ("decode_bs1_kernel: persistent 28-layer W8 batch-1 decode step (1 launch per step)"
                                if wbits == 8 else "28 layers x 5 CUDA-core kernels (W4)"),
                     "achieved": layers_achieved, "peak": peak, "unit": "GB/s", "frac": layers_achieved / peak,
                     "traffic": traffic, "peak_source": peak_kind, "algorithmic_bytes_per_launch": lb,
                     "launch_ms": prof["layers"]},
        "lm_head_roofline": {"achieved": head_achieved, "frac": head_achieved / peak, "launch_ms": prof["lm_head"],
                             "algorithmic_bytes_per_launch": lm_head_bytes()},
        "step_roofline": {"achieved": step_achieved, "peak": peak, "unit": "GB/s", "frac": step_achieved / peak,
                          "algorithmic_bytes_per_step": sb},
        "kernel_ms": prof,
        "gpu_launches": kernels * args.steps,
        "clocks": clk,
        "batched": batched,
        "prefill_4096": prefill_4096,
        "prefill_128": prefill_128,
        "layer_abi": layer_abi,
    }
    if world == 1 and not args.no_cpu_baseline:
        try:
            out["cpu_baseline"] = cpu_baseline_port(wbits)
        except Exception as exc:  # the CPU leg must not hide the GPU number
            out["cpu_baseline"] = {"value": None, "unavailable": str(exc)}
    return out


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--wbits", type=int, default=8, choices=[4, 8])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    world, rank, local = dist_setup()
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args)), flush=True)
        return 0
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    try:
        out = run_b200(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
    if out is not None:
        print(json.dumps(out), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
