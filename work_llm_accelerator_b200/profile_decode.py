"""Small, self-contained decode workloads for kernel profiling (one GPU, synthetic weights).

    python -m work_llm_accelerator_b200.profile_decode kernels --wbits 8 --iters 2
        times each decode kernel of one layer in isolation (engine profile_kernels) and prints the
        per-kernel microseconds: a capture of a single kernel (`ncu -k regex:<name> -c 1`) stays small.
    python -m work_llm_accelerator_b200.profile_decode steps --wbits 8 --prompt 512 --steps 3
        prefills one sequence and runs full 28-layer decode steps (CUDA graphs by default): the launch
        list of a whole step.
    python -m work_llm_accelerator_b200.profile_decode prefill --wbits 8 --prompt 4096 --steps 2
        times full 28-layer prefills of one sequence (CUDA events on the engine stream) and prints
        tokens/s.
    python -m work_llm_accelerator_b200.profile_decode batched --batch 64 --prompt 2048 --steps 8
        prefills `batch` sequences, then times device-resident greedy decode steps of all of them
        together (the batched W8 path) and prints tokens/s.
    python -m work_llm_accelerator_b200.profile_decode trace --wbits 8 --prompt 512 --steps 6
        runs W8 batch-1 decode steps with the engine's "trace" option and prints the persistent kernel's
        per-layer timeline of the last step: for each stage the time (us, latest CTA) at which its inputs
        were held, its digits built and its results published, median over layers 1-26, from the moment the
        last q|k|v CTA held its inputs.

The modes hold about 2.2 GB (W8) of weights on the device plus the KV pool of their sequences.
--profile-range brackets the timed part with cudaProfilerStart/Stop, so that
`ncu --profile-from-start off ...` captures only those launches (not the weight synthesis or the history
prefills before them).
"""
from __future__ import annotations

import argparse
import json

import numpy as np

from . import host


# Trace slots of the persistent kernels (decode_stack.h kTrace*): per stage i (0 q|k|v, 1 attention, 2 o_proj,
# 3 gate|up, 4 down) inputs held (0 + i), digits built (5 + i) and done (10 + i); attention: q ready (34),
# chunk partial stored (35), group merged (36).
_TRACE_EVENTS = {"qkv_inputs": 0, "qkv_built": 5, "qkv_done": 10, "attn_q": 34, "attn_chunk": 35,
                 "attn_merged": 36, "o_built": 7, "o_done": 12, "gate_up_inputs": 3, "gate_up_built": 8,
                 "gate_up_done": 13, "down_inputs": 4, "down_built": 9, "down_done": 14}


def trace_timeline(eng, prompt_len: int, steps: int) -> dict:
    """Per-layer stage timeline of one traced W8 batch-1 decode step (the last of `steps`)."""
    eng.set_option("trace", 1)
    prompt = np.random.default_rng(1).integers(0, 151936, prompt_len).astype(np.int32)
    tok = eng.prefill(0, prompt)
    for _ in range(steps):
        tok = int(eng.decode([0], [tok])[0])
    tr = eng.read_trace(148).astype(np.int64)  # [ctas][28][slots], global-timer ns, 0 = not stamped
    layers = []
    for l in range(tr.shape[1]):
        t = tr[:, l, :]
        latest = {k: int(t[:, slot].max()) for k, slot in _TRACE_EVENTS.items()}
        layers.append(latest)
    out = {}
    for k in _TRACE_EVENTS:
        vals = [(layers[l][k] - layers[l]["qkv_inputs"]) / 1e3 for l in range(1, tr.shape[1] - 1) if layers[l][k] > 0]
        if vals:
            out[k] = round(float(np.median(vals)), 2)
    per_layer = [(layers[l + 1]["qkv_inputs"] - layers[l]["qkv_inputs"]) / 1e3 for l in range(1, tr.shape[1] - 2)]
    out["layer_us"] = round(float(np.median(per_layer)), 2)
    return {"prompt": prompt_len, "steps": steps, "median_us_from_qkv_inputs": out}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("mode", choices=["kernels", "steps", "prefill", "batched", "trace"])
    ap.add_argument("--batch", type=int, default=64, help="batched: sequences decoded together")
    ap.add_argument("--wbits", type=int, default=8, choices=[4, 8])
    ap.add_argument("--seed", type=int, default=7)
    ap.add_argument("--iters", type=int, default=2, help="kernels: launches of each kernel")
    ap.add_argument("--past", type=int, default=512, help="kernels: history length of the attention launch")
    ap.add_argument("--prompt", type=int, default=512, help="steps: prompt length")
    ap.add_argument("--steps", type=int, default=3, help="steps: decode steps")
    ap.add_argument("--graphs", type=int, default=1, help="steps: 1 = CUDA graphs, 0 = eager launches")
    ap.add_argument("--option", action="append", default=[], metavar="NAME=VALUE",
                    help="engine option (e.g. qgemm=0, prefetch=0, pdl=0)")
    ap.add_argument("--profile-range", action="store_true",
                    help="bracket the timed part with cudaProfilerStart/Stop (ncu --profile-from-start off)")
    a = ap.parse_args(argv)

    def profiler(on: bool) -> None:
        if a.profile_range:
            import torch

            (torch.cuda.cudart().cudaProfilerStart if on else torch.cuda.cudart().cudaProfilerStop)()

    max_seqs = a.batch if a.mode == "batched" else 1
    eng = host.Engine(0, a.wbits, max_seqs=max_seqs, max_len=max(1024, a.prompt + 2 * a.steps + 16))
    try:
        eng.init_synthetic(a.seed)
        for opt in a.option:
            name, value = opt.split("=", 1)
            eng.set_option(name, int(value))
        if a.mode == "prefill":
            import torch

            prompt = np.random.default_rng(1).integers(0, 151936, a.prompt).astype(np.int32)
            stream = torch.cuda.ExternalStream(eng.stream())
            eng.prefill(0, prompt)  # warm-up (allocations, first launches)
            times = []
            profiler(True)
            for _ in range(a.steps):
                eng.reset(0)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                eng.prefill(0, prompt)
                e1.record(stream)
                e1.synchronize()
                times.append(e0.elapsed_time(e1))
            profiler(False)
            ms = min(times)
            print(json.dumps({"prompt": a.prompt, "ms": ms, "tok_per_s": a.prompt / (ms * 1e-3)}))
        elif a.mode == "batched":
            rng = np.random.default_rng(1)
            first = []
            for i in range(a.batch):
                first.append(eng.prefill(i, rng.integers(0, 151936, a.prompt).astype(np.int32)))
            profiler(True)
            ms = eng.bench_decode(list(range(a.batch)), first, a.steps, 2)
            profiler(False)
            cats = eng.profile_batched(list(range(a.batch)), first, 2)
            print(json.dumps({"batch": a.batch, "history": a.prompt, "ms_per_step": ms,
                              "tok_per_s": a.batch / (ms * 1e-3), "ms_by_group": cats}))
        elif a.mode == "kernels":
            us = eng.profile_kernels(1, a.past, iters=a.iters)
            print(json.dumps({k: round(v * 1000.0, 3) for k, v in us.items()}))
        elif a.mode == "trace":
            print(json.dumps(trace_timeline(eng, a.prompt, a.steps)))
        else:
            eng.set_option("graphs", a.graphs)
            prompt = np.random.default_rng(1).integers(0, 151936, a.prompt).astype(np.int32)
            tok = eng.prefill(0, prompt)
            profiler(True)
            ms = eng.bench_decode([0], [tok], a.steps, 1)
            profiler(False)
            print(json.dumps({"ms_per_step": ms}))
    finally:
        eng.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
