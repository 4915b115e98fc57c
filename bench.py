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


def layer_weight_bytes(wbits: int) -> int:
    return (2 * HIDDEN * HIDDEN + 2 * KV_WIDTH * HIDDEN + 3 * INTER * HIDDEN) * wbits // 8


LAYER_FLOAT_BYTES = (2 * HIDDEN + (HIDDEN + 2 * KV_WIDTH) + (3 * HIDDEN + 2 * KV_WIDTH + 2 * INTER)) * 4


def step_bytes(wbits: int, history: float) -> float:
    """Algorithmic HBM bytes of one batch-1 decode step: every layer's codes + fp32 scale/bias/norm
    vectors, the attention's K/V read over `history`+1 rows and the new row written, the fp16 LM head."""
    per_layer = layer_weight_bytes(wbits) + LAYER_FLOAT_BYTES + (history + 1) * 2 * KV_WIDTH * 4 + 2 * KV_WIDTH * 4
    return LAYERS * per_layer + VOCAB * HIDDEN * 2 + HIDDEN * 4


def layers_bytes(wbits: int, history: float) -> float:
    """Algorithmic HBM bytes of the 28-layer part of one batch-1 decode step (the persistent kernel): every
    layer's weight codes and fp32 vectors, the K/V history read and the new K/V row written."""
    per_layer = layer_weight_bytes(wbits) + LAYER_FLOAT_BYTES + (history + 1) * 2 * KV_WIDTH * 4 + 2 * KV_WIDTH * 4
    return LAYERS * per_layer


def lm_head_bytes() -> float:
    """Algorithmic HBM bytes of the final norm + fp16 LM head + argmax (batch 1)."""
    return VOCAB * HIDDEN * 2 + HIDDEN * 4


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
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


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
    sec_per_token = statistics.median(secs) * LAYERS / layers
    value = procs / sec_per_token
    sample = (f"reference host library (oracle/_ref/libqwen_decode_stub.so, int4 weights: its only format), "
              f"{procs} concurrent single-threaded processes (all host cores), each one batch-1 sequence at history "
              f"{PROMPT}; value = their aggregate tokens/s; each step times {layers} of 28 decoder layers through "
              f"qwen_decode_top_smoke_forward (scaled x{LAYERS / layers:.0f}); embedding/LM head excluded")
    return {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": sec_per_token * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 activations x int4 weights", "data": "synthetic",
        "config": bench_config(args.gpus, args.warmup, args.steps, args.wbits),
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
def run_b200(args, world: int, rank: int, local: int) -> dict | None:
    import torch
    import torch.distributed as dist

    from work_llm_accelerator_b200 import host

    torch.cuda.set_device(local)
    os.environ["QWEN_B200_DEVICE"] = str(local)
    wbits = args.wbits
    total_steps = args.warmup + args.steps
    max_len = PROMPT + 2 * total_steps + 3 + 32 + 64  # device loop, e2e steps, per-kernel profile, margin
    eng = host.Engine(local, wbits, max_seqs=1, max_len=max_len)
    eng.init_synthetic(SEED)
    rng = np.random.default_rng(SEED + rank)
    prompt = rng.integers(0, VOCAB, PROMPT).astype(np.int32)
    first = eng.prefill(0, prompt)

    stream = torch.cuda.ExternalStream(eng.stream())
    bufs = [torch.tensor([first], dtype=torch.int32, device="cuda"), torch.zeros(1, dtype=torch.int32, device="cuda")]
    gathered = torch.zeros(world, dtype=torch.int32, device="cuda")

    def dev_step(i):
        eng.decode_device([0], bufs[i % 2].data_ptr(), bufs[(i + 1) % 2].data_ptr())
        if world > 1:
            dist.all_gather_into_tensor(gathered, bufs[(i + 1) % 2])

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            dev_step(i)
        stream.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        clocks = ClockSampler(local)
        clocks.start()
        time.sleep(0.3)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for i in range(args.warmup, args.warmup + args.steps):
            dev_step(i)
        ev1.record(stream)
        ev1.synchronize()
        clk = clocks.stop()
    ms = ev0.elapsed_time(ev1) / args.steps
    history_mid = PROMPT + args.warmup + args.steps / 2

    # e2e: host token in, host argmax out, through the engine C-ABI
    cur = int(bufs[(args.warmup + args.steps) % 2].item())
    host_tok = torch.zeros(1, dtype=torch.int32).pin_memory()
    with torch.cuda.stream(stream):
        for _ in range(3):
            cur = int(eng.decode([0], [cur])[0])
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            cur = int(eng.decode([0], [cur])[0])
            if world > 1:
                host_tok[0] = cur
                dist.all_gather_into_tensor(gathered, host_tok.cuda(non_blocking=True))
        e1.record(stream)
        e1.synchronize()
    ms_e2e = e0.elapsed_time(e1) / args.steps

    # per-kernel device time over the same histories: the 28-layer kernel and the LM head, each timed with
    # CUDA events on the engine stream (eager launches, otherwise the same work as one graph step)
    prof = eng.profile_decode(0, cur, max(8, min(args.steps, 32)))

    t = torch.tensor([ms, ms_e2e], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, ms_e2e = float(t[0]), float(t[1])
    kernels = eng.kernels_per_decode_step(1) + 1  # + the position-advance kernel
    # Tensors that were used on the engine's stream (and on NCCL's) must be released while that stream
    # still exists: free them, then let the engine destroy its stream.
    torch.cuda.synchronize()
    del bufs, gathered, host_tok, t, stream
    import gc

    gc.collect()
    torch.cuda.synchronize()
    eng.close()
    if rank != 0:
        return None

    peak, peak_kind = peaks()
    hist_prof = history_mid + args.steps  # histories of the profiled steps (after the e2e steps)
    lb = layers_bytes(wbits, hist_prof)
    layers_achieved = lb / (prof["layers"] * 1e-3) / 1e9
    head_achieved = lm_head_bytes() / (prof["lm_head"] * 1e-3) / 1e9
    sb = step_bytes(wbits, history_mid)
    step_achieved = sb / (ms * 1e-3) / 1e9
    traffic = None
    tr = ROOT / "profiles" / "decode_stack_w8_bs1_dram.json"
    if tr.exists() and wbits == 8:
        d = json.loads(tr.read_text())
        traffic = d.get("dram_bytes_per_launch")
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
        "dtype": "f32 activations x int8 weights (fp32 accumulate)" if wbits == 8 else "f32 x int4",
        "data": "synthetic: seeded N(0,0.02) weights quantized per channel, uniform-random prompt ids",
        "config": bench_config(world, args.warmup, args.steps, wbits),
        "e2e": {"value": world / (ms_e2e * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": 12, "d2h_bytes_per_step": 4},
        "roofline": {"bound": "hbm",
                     "kernel": ("decode_stack_kernel: persistent 28-layer W8 decode step (1 launch per step)"
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
