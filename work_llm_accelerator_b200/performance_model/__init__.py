"""B200 roofline model of the quantized Qwen2.5-1.5B decoder path.

This is the B200 counterpart of the reference's ASIC budget estimator
(performance_model/estimate_qwen_prefill_decode.py:10-200). It keeps that estimator's model description and
MAC accounting: ModelSpec, param_breakdown, decode_macs_per_token, prefill_macs and the decode/prefill
bandwidth reports. In place of a MAC array and an SRAM budget it rates each workload against the B200's
measured HBM copy bandwidth and dense tensor-core throughput (MEASURED_PEAKS.json at the repository root,
written on this pool's B200s; fallback 6650 GB/s and 1590 TFLOP/s).

The algorithmic work of each benchmark configuration:
- config 0: one decode step of one layer, history 128;
- config 1: a 128-token prefill of one layer;
- config 2: a 28-layer batch-1 decode step;
- config 3: a 28-layer batched decode step;
- config 4: a 4096-token 28-layer prefill.

Work counts what the computation must move or perform: every weight code once per step, the fp32 norm, bias
and scale vectors, the K/V rows read and written, and the fp16 LM head; FLOPs are 2 per multiply-accumulate of
the projections, plus the causal attention products. bench.py takes its roofline figures from here, so the two
cannot drift apart.

  python -m work_llm_accelerator_b200.performance_model [--json] [--wbits 8]
"""
from __future__ import annotations

import json
import math
from dataclasses import asdict, dataclass
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


@dataclass(frozen=True)
class ModelSpec:
    """Qwen2.5-1.5B (reference performance_model/estimate_qwen_prefill_decode.py:10-24)."""

    hidden_size: int = 1536
    intermediate_size: int = 8960
    num_hidden_layers: int = 28
    num_attention_heads: int = 12
    num_key_value_heads: int = 2
    vocab_size: int = 151936

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @property
    def kv_width(self) -> int:
        return self.num_key_value_heads * self.head_dim


SPEC = ModelSpec()


def param_breakdown(spec: ModelSpec = SPEC) -> dict[str, int]:
    """Weight counts (reference :27-52, same keys)."""
    h, i, kv = spec.hidden_size, spec.intermediate_size, spec.kv_width
    attention = 2 * h * h + 2 * h * kv
    mlp = 3 * h * i
    norms = 2 * h
    per_layer = attention + mlp + norms
    embed = spec.vocab_size * h
    return {"attention_per_layer": attention, "mlp_per_layer": mlp, "norms_per_layer": norms,
            "per_layer": per_layer, "layers_total": per_layer * spec.num_hidden_layers, "embed_or_lm_head": embed,
            "model_total": per_layer * spec.num_hidden_layers + embed}


def projection_macs_per_token(spec: ModelSpec = SPEC) -> int:
    """Multiply-accumulates of the seven projections of one layer for one token (46,792,704)."""
    p = param_breakdown(spec)
    return p["attention_per_layer"] + p["mlp_per_layer"]


# ---------------------------------------------------------------------------------------------------------
# bytes
# ---------------------------------------------------------------------------------------------------------
def layer_weight_bytes(wbits: int, spec: ModelSpec = SPEC) -> int:
    """Weight codes of one layer: 46,792,704 codes at 4 or 8 bits."""
    return projection_macs_per_token(spec) * wbits // 8


def layer_vector_bytes(spec: ModelSpec = SPEC) -> int:
    """fp32 vectors of one layer: two norm weights, q|k|v biases, seven per-channel scale vectors."""
    h, i, kv = spec.hidden_size, spec.intermediate_size, spec.kv_width
    return (2 * h + (h + 2 * kv) + (3 * h + 2 * kv + 2 * i)) * 4


def layer_param_bytes(wbits: int, spec: ModelSpec = SPEC) -> int:
    """One layer's parameters in the reference's DDR layout (W4: 23,508,992 B; W8: 46,905,344 B)."""
    return layer_weight_bytes(wbits, spec) + layer_vector_bytes(spec)


def kv_row_bytes(spec: ModelSpec = SPEC) -> int:
    """fp32 K and V rows of one token in one layer (the reference caches fp32, llm_memory_layout.h:53)."""
    return 2 * spec.kv_width * 4


def lm_head_bytes(spec: ModelSpec = SPEC, rows: int = 1) -> int:
    """Final norm weight + the tied fp16 LM head table (read once for all rows of a step)."""
    return spec.vocab_size * spec.hidden_size * 2 + spec.hidden_size * 4


def decode_layers_bytes(wbits: int, history: float, n_seqs: int = 1, spec: ModelSpec = SPEC) -> float:
    """The 28-layer part of one decode step: every layer's parameters once, and per sequence the K/V read over
    history + 1 rows (the new row included) and the new row written."""
    per_layer = layer_param_bytes(wbits, spec) + n_seqs * ((history + 1) * kv_row_bytes(spec) + kv_row_bytes(spec))
    return spec.num_hidden_layers * per_layer


def decode_step_bytes(wbits: int, history: float, n_seqs: int = 1, spec: ModelSpec = SPEC) -> float:
    """One greedy decode step of n_seqs sequences at `history`: the layers, then the LM head read once."""
    return decode_layers_bytes(wbits, history, n_seqs, spec) + lm_head_bytes(spec)


def decode_layer_bytes(wbits: int, history: int, spec: ModelSpec = SPEC) -> float:
    """Config 0: one layer's decode step (history rows read, one written) plus its in/out activations."""
    return (layer_param_bytes(wbits, spec) + (history + 1) * kv_row_bytes(spec) + kv_row_bytes(spec)
            + 2 * spec.hidden_size * 4)


def prefill_layer_bytes(wbits: int, seq_len: int, spec: ModelSpec = SPEC) -> float:
    """Config 1: one layer's prefill through the top wrapper: parameters, the activation DDR window (input,
    output, scratch: 3 S H fp32) and the K/V rows written."""
    return layer_param_bytes(wbits, spec) + 3 * seq_len * spec.hidden_size * 4 + seq_len * kv_row_bytes(spec)


def prefill_model_bytes(wbits: int, seq_len: int, spec: ModelSpec = SPEC) -> float:
    """A 28-layer prefill: every layer's parameters once, the K/V rows written, the embedding rows gathered and
    the LM head for the last token."""
    return (spec.num_hidden_layers * (layer_param_bytes(wbits, spec) + seq_len * kv_row_bytes(spec))
            + seq_len * spec.hidden_size * 2 + lm_head_bytes(spec))


# ---------------------------------------------------------------------------------------------------------
# FLOPs (2 per multiply-accumulate)
# ---------------------------------------------------------------------------------------------------------
def decode_macs_per_token(context_len: int, spec: ModelSpec = SPEC) -> dict[str, int]:
    """Reference :55-66 accounting (QK and PV over the context, LM head), projections without norms."""
    dense = projection_macs_per_token(spec) * spec.num_hidden_layers
    attn = 2 * spec.num_hidden_layers * spec.num_attention_heads * spec.head_dim * context_len
    lm = param_breakdown(spec)["embed_or_lm_head"]
    return {"dense_stack": dense, "lm_head": lm, "attention_context": attn, "total": dense + lm + attn}


def prefill_flops(seq_len: int, layers: int | None = None, spec: ModelSpec = SPEC) -> dict[str, float]:
    """Projections 2 * 46.79 M * S per layer plus causal attention 4 * heads * head_dim * S(S+1)/2 per layer
    (QK^T and PV over the key <= query pairs)."""
    layers = spec.num_hidden_layers if layers is None else layers
    dense = 2.0 * projection_macs_per_token(spec) * seq_len * layers
    pairs = seq_len * (seq_len + 1) / 2
    attn = 4.0 * spec.num_attention_heads * spec.head_dim * pairs * layers
    return {"dense": dense, "attention": attn, "total": dense + attn}


# ---------------------------------------------------------------------------------------------------------
# peaks and roofline
# ---------------------------------------------------------------------------------------------------------
@dataclass(frozen=True)
class Peaks:
    hbm_gbs: float
    bf16_tflops: float
    bf16_tflops_sustained: float
    source: str  # "measured" (MEASURED_PEAKS.json) or "fallback"


def load_peaks(path: Path | None = None) -> Peaks:
    p = path or ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return Peaks(float(d["hbm_gbs"]), float(d["bf16_tflops"]),
                     float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured")
    return Peaks(FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, FALLBACK_BF16_TFLOPS, "fallback")


def roofline(work: float, seconds: float, bound: str, peaks: Peaks | None = None, sustained: bool = False,
             traffic: float | None = None) -> dict:
    """Achieved rate of `work` (bytes for bound "hbm", FLOPs for "tensor") in `seconds`, against the peak."""
    peaks = peaks or load_peaks()
    if bound == "hbm":
        achieved, peak, unit = work / seconds / 1e9, peaks.hbm_gbs, "GB/s"
    elif bound == "tensor":
        achieved = work / seconds / 1e12
        peak = peaks.bf16_tflops_sustained if sustained else peaks.bf16_tflops
        unit = "TFLOP/s"
    else:
        raise ValueError(f"unknown bound {bound!r}")
    return {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak,
            "traffic": traffic, "peak_source": peaks.source}


def lower_bound_seconds(bytes_: float, flops: float, peaks: Peaks | None = None) -> float:
    """Time no implementation can beat: the slower of streaming the bytes and doing the FLOPs."""
    peaks = peaks or load_peaks()
    return max(bytes_ / (peaks.hbm_gbs * 1e9), flops / (peaks.bf16_tflops * 1e12))


# ---------------------------------------------------------------------------------------------------------
# reports (the reference's decode_bandwidth_report / prefill_bandwidth_report, rated on B200)
# ---------------------------------------------------------------------------------------------------------
def decode_report(wbits: int, history: int, n_seqs: int = 1, peaks: Peaks | None = None,
                  spec: ModelSpec = SPEC) -> dict:
    peaks = peaks or load_peaks()
    b = decode_step_bytes(wbits, history, n_seqs, spec)
    macs = decode_macs_per_token(history + 1, spec)
    flops = 2.0 * (n_seqs * (macs["dense_stack"] + macs["attention_context"]) + n_seqs * macs["lm_head"])
    t = lower_bound_seconds(b, flops, peaks)
    return {"wbits": wbits, "history": history, "n_seqs": n_seqs, "bytes_per_step": b, "flops_per_step": flops,
            "weight_bytes_per_step": spec.num_hidden_layers * layer_param_bytes(wbits, spec) + lm_head_bytes(spec),
            "kv_bytes_per_step": n_seqs * spec.num_hidden_layers * (history + 2) * kv_row_bytes(spec),
            "bound": "hbm" if b / (peaks.hbm_gbs * 1e9) >= flops / (peaks.bf16_tflops * 1e12) else "tensor",
            "min_ms_per_step": t * 1e3, "max_tok_s": n_seqs / t}


def prefill_report(wbits: int, seq_len: int, peaks: Peaks | None = None, spec: ModelSpec = SPEC) -> dict:
    peaks = peaks or load_peaks()
    b = prefill_model_bytes(wbits, seq_len, spec)
    f = prefill_flops(seq_len, spec=spec)
    t = lower_bound_seconds(b, f["total"], peaks)
    return {"wbits": wbits, "seq_len": seq_len, "bytes": b, "flops": f,
            "bound": "hbm" if b / (peaks.hbm_gbs * 1e9) >= f["total"] / (peaks.bf16_tflops * 1e12) else "tensor",
            "min_ms": t * 1e3, "max_tok_s": seq_len / t}


def baseline_configs_report(wbits: int = 8, peaks: Peaks | None = None) -> dict:
    """Lower bounds of the five benchmark configurations on one B200."""
    peaks = peaks or load_peaks()
    c0_bytes = decode_layer_bytes(wbits, 128)
    c1_bytes = prefill_layer_bytes(wbits, 128)
    c1_flops = prefill_flops(128, layers=1)["total"]
    return {
        "peaks": asdict(peaks),
        "model": asdict(SPEC),
        "params": param_breakdown(),
        "config0_decode_layer_hist128": {"bytes": c0_bytes,
                                         "min_us": lower_bound_seconds(c0_bytes, 0.0, peaks) * 1e6},
        "config1_prefill_layer_128": {"bytes": c1_bytes, "flops": c1_flops,
                                      "min_us": lower_bound_seconds(c1_bytes, c1_flops, peaks) * 1e6},
        "config2_decode_bs1_hist512": decode_report(wbits, 512, 1, peaks),
        "config3_decode_bs64_hist2048": decode_report(wbits, 2048, 64, peaks),
        "config4_prefill_4096": prefill_report(wbits, 4096, peaks),
    }


def main(argv: list[str] | None = None) -> int:
    import argparse

    ap = argparse.ArgumentParser(description="B200 roofline of the Qwen2.5-1.5B decoder path (benchmark configs)")
    ap.add_argument("--wbits", type=int, default=8, choices=[4, 8])
    ap.add_argument("--json", action="store_true")
    args = ap.parse_args(argv)
    rep = baseline_configs_report(args.wbits)
    if args.json:
        print(json.dumps(rep, indent=1))
        return 0
    pk = rep["peaks"]
    print(f"B200 peaks ({pk['source']}): HBM {pk['hbm_gbs']:.0f} GB/s, bf16 {pk['bf16_tflops']:.0f} TFLOP/s")
    print(f"config 0 (decode layer, hist 128): {rep['config0_decode_layer_hist128']['bytes'] / 1e6:.2f} MB, "
          f">= {rep['config0_decode_layer_hist128']['min_us']:.2f} us")
    c1 = rep["config1_prefill_layer_128"]
    print(f"config 1 (prefill layer, 128): {c1['bytes'] / 1e6:.2f} MB, {c1['flops'] / 1e9:.2f} GFLOP, "
          f">= {c1['min_us']:.2f} us")
    for k in ("config2_decode_bs1_hist512", "config3_decode_bs64_hist2048"):
        d = rep[k]
        print(f"{k}: {d['bytes_per_step'] / 1e9:.3f} GB/step ({d['bound']}), >= {d['min_ms_per_step']:.3f} ms, "
              f"<= {d['max_tok_s']:.0f} tok/s")
    p = rep["config4_prefill_4096"]
    print(f"config4_prefill_4096: {p['flops']['total'] / 1e12:.2f} TFLOP ({p['bound']}), >= {p['min_ms']:.2f} ms, "
          f"<= {p['max_tok_s']:.0f} tok/s")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
