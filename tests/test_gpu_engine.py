"""GPU parity of the full 28-layer model against the full-model oracle harness (oracle/qwen_full_model.py:
the reference caller's flow with the reference's per-layer math, itself pinned by the `full_model_w4`
golden case to the reference's own host libraries).

Criterion (north_star: per-layer hidden states within 1e-3 relative L2): checked layer-wise -- every
GPU layer is fed the oracle's input for that layer (and the oracle's KV history) and must reproduce the
oracle's output. Free-running comparisons are not a valid criterion on this synthetic model: with random
N(0, 0.02) weights, the attention residual dropped (as in the reference) and bf16 rounding between layers,
a perturbation grows ~1.3x per layer, so ~1e-6 arithmetic differences flip some bf16 roundings in the first
layers and the final hidden states differ completely (measured: layer-0 1.9e-4 -> layer-27 0.78 rel-L2).
Greedy-token identity therefore requires bit-identical arithmetic; the engine tests below check the engine's
own invariants (graph == eager == device API, batch == single, LM head + argmax == oracle on the same
hidden state, device weight synthesis == host generator).
"""
from __future__ import annotations

import numpy as np
import pytest

import qwen_oracle as qo
from qwen_full_model import OracleModel

pytestmark = pytest.mark.gpu

HIDDEN_TOL = 1e-3


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def host(built_libs, gpu_available):
    if not gpu_available:
        pytest.fail("no CUDA device: the -m gpu suite must run on a B200")
    from work_llm_accelerator_b200 import host as h

    return h


@pytest.mark.parametrize("wbits", [4, 8])
def test_device_synthesis_matches_host_generator(host, wbits):
    eng = host.Engine(0, wbits, max_seqs=1, max_len=256)
    try:
        eng.init_synthetic(5)
        for layer in (0, 27):
            w_dev, s_dev = eng.read_layer(layer)
            w_host, s_host = qo.synth_layer(5, layer, wbits).ddr()
            assert np.array_equal(w_dev, w_host)
            assert np.array_equal(s_dev[:s_host.size], s_host)
    finally:
        eng.close()


@pytest.mark.parametrize("wbits", [4, 8])
def test_full_model_layerwise_parity(host, golden, wbits):
    """All 28 layers, prefill (8-token prompt) then 3 decode steps of the oracle's own greedy run: each GPU
    layer (drop-in ABI) on the oracle's layer input and KV history."""
    seed = 31
    case = next(c for c in golden["cases"] if c["kind"] == "full_model_w4")
    prompt = case["prompt"]
    ora = OracleModel(seed, wbits)
    dec = host.load_decode_lib()
    pre = host.load_prefill_lib()
    S = len(prompt)
    # prefill, layer by layer
    x = ora.embed_rows(prompt).reshape(-1)
    worst = 0.0
    for l in range(qo.LAYERS):
        p = ora.params[l]
        k_o, v_o = np.zeros(S * qo.KV_WIDTH, np.float32), np.zeros(S * qo.KV_WIDTH, np.float32)
        st, out_o = qo.prefill_layer(p, x, S, k_o, v_o)
        k_g, v_g, out_g = np.zeros_like(k_o), np.zeros_like(v_o), np.zeros_like(out_o)
        fn = pre.qwen_prefill_layer_smoke_forward if wbits == 4 else pre.qwen_prefill_layer_smoke_forward_w8
        assert fn(x, S, *qo.tiles_tuple(), *layer_args(p), k_g, v_g, out_g) == 0
        worst = max(worst, rel_l2(out_g, out_o), rel_l2(k_g, k_o), rel_l2(v_g, v_o))
        ora.k[l], ora.v[l] = k_o, v_o
        x = qo.round_bf16(out_o)
    ora.len = S
    tok = qo.lm_head_argmax(x.reshape(S, qo.HIDDEN)[-1], ora.final_norm, ora.embed)
    for _ in range(3):
        x = ora.embed_rows([tok]).reshape(-1)
        past = ora.len
        for l in range(qo.LAYERS):
            p = ora.params[l]
            kc = np.zeros((past + 1) * qo.KV_WIDTH, np.float32)
            vc = kc.copy()
            kc[:past * qo.KV_WIDTH], vc[:past * qo.KV_WIDTH] = ora.k[l], ora.v[l]
            kg, vg = kc.copy(), vc.copy()
            st, out_o = qo.decode_layer(p, x, past, kc, vc)
            out_g = np.zeros(qo.HIDDEN, np.float32)
            fn = dec.qwen_decode_layer_smoke_forward if wbits == 4 else dec.qwen_decode_layer_smoke_forward_w8
            assert fn(x, past, *layer_args(p), kg, vg, out_g) == 0
            row = slice(past * qo.KV_WIDTH, (past + 1) * qo.KV_WIDTH)
            worst = max(worst, rel_l2(out_g, out_o), rel_l2(kg[row], kc[row]), rel_l2(vg[row], vc[row]))
            ora.k[l], ora.v[l] = kc, vc
            x = qo.round_bf16(out_o)
        ora.len = past + 1
        tok = qo.lm_head_argmax(x, ora.final_norm, ora.embed)
    assert worst <= HIDDEN_TOL
    assert worst <= 1e-4  # observed ~2e-6; the tighter bound catches real regressions


def layer_args(p):
    return (p["input_layernorm"], p["post_attention_layernorm"], p["q_w"], p["k_w"], p["v_w"], p["o_w"], p["gate_w"],
            p["up_w"], p["down_w"], p["q_bias"], p["k_bias"], p["v_bias"], p["q_s"], p["k_s"], p["v_s"], p["o_s"],
            p["gate_s"], p["up_s"], p["down_s"])


def test_engine_first_layer_and_lm_head_match_oracle(host):
    """Engine prefill/decode: layer 0 (identical embedding input) within 1e-3; LM head + argmax on the engine's
    own final hidden state equal the oracle's LM head on that same state."""
    seed = 31
    prompt = [5, 77, 1234, 99999, 151935, 0, 42, 8]
    ora = OracleModel(seed, 8)
    eng = host.Engine(0, 8, max_seqs=1, max_len=256)
    try:
        eng.init_synthetic(seed)
        eng.set_option("dump_hidden", 1)
        eng.set_option("logits", 1)
        tok_e = eng.prefill(0, prompt)
        ora.prefill(prompt)
        hid = eng.read_hidden(1)
        assert rel_l2(hid[0, 0], ora.hidden_trace[0]) <= HIDDEN_TOL
        logits = eng.read_logits(1)[0]
        tok_o, logits_o = qo.lm_head_argmax(hid[27, 0], ora.final_norm, ora.embed, want_logits=True)
        assert rel_l2(logits, logits_o) <= 1e-5
        assert tok_e == tok_o
        nxt = int(eng.decode([0], [tok_e])[0])
        hid = eng.read_hidden(1)
        tok_o2 = qo.lm_head_argmax(hid[27, 0], ora.final_norm, ora.embed)
        assert nxt == tok_o2
    finally:
        eng.close()


def test_graph_and_eager_paths_agree(host):
    """CUDA-graph + PDL decode steps, eager launches, the host-token API and the device-token API give
    the same tokens."""
    import torch

    seed = 9
    prompt = [11, 22, 33, 44, 55]
    outs = []
    for graphs, pdl in ((1, 1), (0, 0), (1, 0)):
        eng = host.Engine(0, 8, max_seqs=1, max_len=256)
        eng.init_synthetic(seed)
        eng.set_option("graphs", graphs)
        eng.set_option("pdl", pdl)
        toks = [eng.prefill(0, prompt)]
        for _ in range(6):
            toks.append(int(eng.decode([0], [toks[-1]])[0]))
        outs.append(toks)
        eng.close()
    assert outs[0] == outs[1] == outs[2]
    eng = host.Engine(0, 8, max_seqs=1, max_len=256)
    try:
        eng.init_synthetic(seed)
        first = eng.prefill(0, prompt)
        assert first == outs[0][0]
        cur = torch.tensor([first], dtype=torch.int32, device="cuda")
        nxt = torch.zeros(1, dtype=torch.int32, device="cuda")
        toks = [first]
        for _ in range(6):
            eng.decode_device([0], cur.data_ptr(), nxt.data_ptr())
            torch.cuda.synchronize()
            toks.append(int(nxt.item()))
            cur.copy_(nxt)
        assert toks == outs[0]
    finally:
        eng.close()


@pytest.mark.parametrize("wbits", [4, 8])
def test_prefill_graph_replay_matches_eager(host, wbits):
    """A prefill of a length seen before replays its captured CUDA graph: same next token and the same K/V
    rows, bit for bit, as the eager first call; a different slot gets its own graph."""
    prompt = [int(x) for x in np.random.default_rng(3).integers(0, 151936, 37)]
    eng = host.Engine(0, wbits, max_seqs=2, max_len=256)
    try:
        eng.init_synthetic(4)
        first = eng.prefill(0, prompt)  # eager pass + capture
        k0, v0 = eng.read_kv(0, 27, len(prompt))
        for _ in range(2):
            eng.reset(0)
            assert eng.prefill(0, prompt) == first  # graph replay
            k, v = eng.read_kv(0, 27, len(prompt))
            assert np.array_equal(k, k0) and np.array_equal(v, v0)
        assert eng.prefill(1, prompt) == first  # other slot: eager + capture, same values
        k1, v1 = eng.read_kv(1, 27, len(prompt))
        assert np.array_equal(k1, k0) and np.array_equal(v1, v0)
        eng.set_option("graphs", 0)
        eng.reset(0)
        assert eng.prefill(0, prompt) == first
    finally:
        eng.close()


def test_batched_decode_matches_single(host):
    """Four sequences decoded together equal the same sequences decoded one by one."""
    seed = 12
    prompts = [[1, 2, 3], [7, 8, 9, 10], [100, 200], [5000, 6000, 7000, 8000, 9000]]
    eng = host.Engine(0, 8, max_seqs=4, max_len=256)
    try:
        eng.init_synthetic(seed)
        single = []
        for i, p in enumerate(prompts):
            toks = [eng.prefill(i, p)]
            for _ in range(3):
                toks.append(int(eng.decode([i], [toks[-1]])[0]))
            single.append(toks)
            eng.reset(i)
        cur = [eng.prefill(i, p) for i, p in enumerate(prompts)]
        batched = [[c] for c in cur]
        for _ in range(3):
            cur = [int(t) for t in eng.decode([0, 1, 2, 3], cur)]
            for i, t in enumerate(cur):
                batched[i].append(t)
        assert batched == single
    finally:
        eng.close()


def _decode_trace(host, seed, prompt, steps, max_len=256, **options):
    eng = host.Engine(0, 8, max_seqs=1, max_len=max_len)
    try:
        eng.init_synthetic(seed)
        for name, value in options.items():
            eng.set_option(name, value)
        eng.set_option("dump_hidden", 1)
        toks = [eng.prefill(0, prompt)]
        hidden = []
        for _ in range(steps):
            toks.append(int(eng.decode([0], [toks[-1]])[0]))
            hidden.append(eng.read_hidden(1).copy())
        return toks, hidden
    finally:
        eng.close()


@pytest.mark.parametrize("prompt_len", [5, 130, 600])
def test_persistent_step_kernels_match_separate_kernels(host, prompt_len):
    """The single-launch decode steps (decode_bs1.cu: batch 1 on the CUDA cores with self-validating
    cross-CTA words; decode_stack.cu: the tensor-core persistent kernel) and the five-launches-per-layer
    tensor-core path do the same arithmetic in the same order: every layer's hidden state and every token
    are bit-identical. 130 prompt tokens give three 64-key attention chunks (cross-CTA chunk merge), 5 give
    one, 600 give ten (one merge batch of the batch-1 kernel; the 2500-token test below needs four)."""
    rng = np.random.default_rng(prompt_len)
    prompt = [int(t) for t in rng.integers(0, qo.VOCAB, prompt_len)]
    host.kernel_error(reset=True)
    toks_1, hid_1 = _decode_trace(host, 21, prompt, 4, max_len=1024, stack=1, bs1=1)
    assert host.kernel_error(reset=True) == 0
    toks_s, hid_s = _decode_trace(host, 21, prompt, 4, max_len=1024, stack=1, bs1=0)
    assert host.kernel_error(reset=True) == 0
    toks_k, hid_k = _decode_trace(host, 21, prompt, 4, max_len=1024, stack=0)
    assert toks_1 == toks_s == toks_k
    for step, (a, b, c) in enumerate(zip(hid_1, hid_s, hid_k)):
        assert np.array_equal(a, c), ("bs1", step, rel_l2(a, c))
        assert np.array_equal(b, c), ("stack", step, rel_l2(b, c))


def test_batch1_kernel_long_history(host):
    """A 2500-token history gives 40 attention chunks: 160 chunk items for 148 CTAs, so some CTAs run two
    items (a merging item waits only on items of lower index) and the merge's running-max scan spans two
    32-chunk windows. Every layer's output equals the separate kernels' over three steps."""
    rng = np.random.default_rng(2500)
    prompt = [int(t) for t in rng.integers(0, qo.VOCAB, 2500)]
    host.kernel_error(reset=True)
    toks_1, hid_1 = _decode_trace(host, 9, prompt, 3, max_len=2600, stack=1, bs1=1)
    assert host.kernel_error(reset=True) == 0
    toks_k, hid_k = _decode_trace(host, 9, prompt, 3, max_len=2600, stack=0)
    assert toks_1 == toks_k
    for step, (a, b) in enumerate(zip(hid_1, hid_k)):
        assert np.array_equal(a, b), (step, rel_l2(a, b))


def test_batch1_kernel_cta_count_does_not_change_results(host):
    """Option "bs1_ctas": the batch-1 kernel's default schedule over 144 CTAs (the fewest: one down_proj item
    per CTA) gives the same layers and tokens as over 146 CTAs and over every SM of a B200 (148)."""
    rng = np.random.default_rng(144)
    prompt = [int(t) for t in rng.integers(0, qo.VOCAB, 200)]
    toks_a, hid_a = _decode_trace(host, 4, prompt, 3, max_len=512, stack=1, bs1=1)
    for ctas in (146, 148):
        toks_b, hid_b = _decode_trace(host, 4, prompt, 3, max_len=512, stack=1, bs1=1, bs1_ctas=ctas)
        assert host.kernel_error(reset=True) == 0
        assert toks_a == toks_b
        for step, (a, b) in enumerate(zip(hid_a, hid_b)):
            assert np.array_equal(a, b), (ctas, step, rel_l2(a, b))


def test_batch1_kernel_bounded_waits_end_a_broken_step(host):
    """Failure path of the batch-1 kernel without a GPU fault: option "bs1_poison" fills the launch's packed
    split-K words with counts no producer can complete, so its consumers wait out their bounded waits (~1 s),
    raise the abort flag (every other wait then ends at once) and set the kernel error flag. The step returns
    within seconds, the next launch (the other launch parity, zeroed by the broken one) completes without an
    error, and after a fresh prefill the kernel again equals the separate kernels."""
    import time

    rng = np.random.default_rng(31)
    prompt = [int(t) for t in rng.integers(0, qo.VOCAB, 40)]
    eng = host.Engine(0, 8, max_seqs=1, max_len=256)
    try:
        eng.init_synthetic(31)
        host.kernel_error(reset=True)
        tok = eng.prefill(0, prompt)
        tok = int(eng.decode([0], [tok])[0])
        assert host.kernel_error(reset=True) == 0
        eng.set_option("bs1_poison", 1)
        t0 = time.time()
        eng.decode([0], [tok])
        assert time.time() - t0 < 30.0
        assert host.kernel_error(reset=True) == 1  # a bounded wait gave up
        eng.decode([0], [tok])
        assert host.kernel_error(reset=True) == 0
        eng.reset(0)
        eng.set_option("dump_hidden", 1)
        toks, hid = [eng.prefill(0, prompt)], []
        for _ in range(3):
            toks.append(int(eng.decode([0], [toks[-1]])[0]))
            hid.append(eng.read_hidden(1).copy())
        assert host.kernel_error(reset=True) == 0
    finally:
        eng.close()
    toks_k, hid_k = _decode_trace(host, 31, prompt, 3, max_len=256, stack=0)
    assert toks == toks_k
    for step, (a, b) in enumerate(zip(hid, hid_k)):
        assert np.array_equal(a, b), (step, rel_l2(a, b))


def test_batch1_kernel_over_many_launches(host):
    """The batch-1 persistent kernel keeps launch-parity words (zeroed by the following launch) and tagged
    words (launch epoch and layer in the tag): 40 consecutive steps with the trace option on, each equal
    to the separate kernels' step from the same state."""
    rng = np.random.default_rng(77)
    prompt = [int(t) for t in rng.integers(0, qo.VOCAB, 70)]
    toks_1, hid_1 = _decode_trace(host, 5, prompt, 40, max_len=256, stack=1, bs1=1, trace=1)
    assert host.kernel_error(reset=True) == 0
    toks_k, hid_k = _decode_trace(host, 5, prompt, 40, max_len=256, stack=0)
    assert toks_1 == toks_k
    for step, (a, b) in enumerate(zip(hid_1, hid_k)):
        assert np.array_equal(a, b), (step, rel_l2(a, b))


@pytest.mark.parametrize("n", [5, 12, 40])  # 40: 64-token padding (CTA-pair GEMM tiles)
def test_batched_w8_decode_matches_single(host, n):
    """More than four sequences per step take the batched path (every projection of all tokens in one
    many-token tensor-core GEMM, paged attention over all tokens); it performs the same per-token
    arithmetic as the persistent single-sequence kernel, so tokens and every layer's output are identical."""
    rng = np.random.default_rng(100 + n)
    prompts = [[int(t) for t in rng.integers(0, qo.VOCAB, int(rng.integers(3, 90)))] for _ in range(n)]
    steps = 3
    eng = host.Engine(0, 8, max_seqs=n, max_len=256)
    try:
        eng.init_synthetic(17)
        eng.set_option("dump_hidden", 1)
        single_tok, single_hid = [], []
        for i, p in enumerate(prompts):
            toks, hids = [eng.prefill(i, p)], []
            for _ in range(steps):
                toks.append(int(eng.decode([i], [toks[-1]])[0]))
                hids.append(eng.read_hidden(1)[:, 0].copy())
            single_tok.append(toks)
            single_hid.append(hids)
            eng.reset(i)
        cur = [eng.prefill(i, p) for i, p in enumerate(prompts)]
        batched = [[c] for c in cur]
        for step in range(steps):
            cur = [int(t) for t in eng.decode(list(range(n)), cur)]
            hid = eng.read_hidden(n)
            for i, t in enumerate(cur):
                batched[i].append(t)
                assert np.array_equal(hid[:, i], single_hid[i][step]), (i, step, rel_l2(hid[:, i], single_hid[i][step]))
        assert batched == single_tok
        assert host.kernel_error(reset=True) == 0
    finally:
        eng.close()


def test_decode_attention_grid_does_not_change_results(host):
    """The separate decode attention kernel is persistent: its CTAs walk contiguous ranges of the
    (token, KV head, 64-key chunk) items, so one CTA may finish one (token, head) and start the next; a
    follow-up kernel merges each (token, head)'s chunks in order. Every grid size (option "attn_ctas", down
    to one CTA doing everything) gives bit-identical layer outputs, equal to the persistent single-sequence
    kernel's; the histories are ragged (1 to 5 chunks, a chunk holding only the new row)."""
    rng = np.random.default_rng(77)
    lens = (3, 64, 65, 200, 257, 130)
    prompts = [[int(t) for t in rng.integers(0, qo.VOCAB, n)] for n in lens]
    eng = host.Engine(0, 8, max_seqs=len(lens), max_len=512)
    try:
        eng.init_synthetic(23)
        eng.set_option("dump_hidden", 1)
        single_tok, single_hid = [], []
        for i, p in enumerate(prompts):
            first = eng.prefill(i, p)
            single_tok.append(int(eng.decode([i], [first])[0]))
            single_hid.append(eng.read_hidden(1)[:, 0].copy())
            eng.reset(i)
        for ctas in (0, 1, 5, 16):
            eng.set_option("attn_ctas", ctas)
            cur = [eng.prefill(i, p) for i, p in enumerate(prompts)]
            out = [int(t) for t in eng.decode(list(range(len(lens))), cur)]
            hid = eng.read_hidden(len(lens))
            for i in range(len(lens)):
                assert np.array_equal(hid[:, i], single_hid[i]), (ctas, i, rel_l2(hid[:, i], single_hid[i]))
            assert out == single_tok, ctas
            for i in range(len(lens)):
                eng.reset(i)
        assert host.kernel_error(reset=True) == 0
    finally:
        eng.close()


def test_tensor_core_lm_head_matches_cuda_core_head(host):
    """The tensor-core LM head (fp16 table x two fp16 planes of the normalised activations, 22 significant
    bits; tensor-core fp32 accumulation) and the CUDA-core GEMV head give the same greedy tokens and logits
    within 1e-5 relative L2, the tolerance the LM head has against the oracle (1 and 9 rows)."""
    rng = np.random.default_rng(3)
    prompts = [[int(t) for t in rng.integers(0, qo.VOCAB, 6)] for _ in range(9)]
    eng = host.Engine(0, 8, max_seqs=9, max_len=64)
    try:
        eng.init_synthetic(23)
        eng.set_option("logits", 1)
        out = {}
        for lm_tc in (1, 0):
            eng.set_option("lm_tc", lm_tc)
            toks = [eng.prefill(i, p) for i, p in enumerate(prompts)]
            l1 = eng.read_logits(1).copy()
            nxt = [int(t) for t in eng.decode(list(range(9)), toks)]
            l9 = eng.read_logits(9).copy()
            out[lm_tc] = (toks, nxt, l1, l9)
            for i in range(9):
                eng.reset(i)
        assert out[1][0] == out[0][0] and out[1][1] == out[0][1]
        assert rel_l2(out[1][2], out[0][2]) <= 1e-5
        assert rel_l2(out[1][3], out[0][3]) <= 1e-5
        assert host.kernel_error(reset=True) == 0
    finally:
        eng.close()


def test_hf_cache_export_and_import(host):
    """The engine's KV rows in the Hugging Face per-layer layout the reference caller converts to and from
    (verification/real_host_top_backend.py:199-206): read_kv_hf is the head-major transpose of read_kv,
    write_kv_hf stores what read_kv_hf returns, and EngineBackend.hf_cache gives 28 (k, v) pairs of
    [1][2][seq][128]."""
    prompt = [int(t) for t in np.random.default_rng(8).integers(0, qo.VOCAB, 70)]
    eng = host.Engine(0, 8, max_seqs=2, max_len=128)
    try:
        eng.init_synthetic(6)
        be = host.EngineBackend(eng, slot=0)
        res = be.prefill(prompt)
        be.decode_step([int(np.argmax(res.logits[0]))], res.cache)
        n = eng.seq_len(0)
        assert n == 71
        cache = be.hf_cache(res.cache)
        assert len(cache) == qo.LAYERS and cache[0][0].shape == (1, 2, n, 128)
        for layer in (0, 13, 27):
            k, v = eng.read_kv(0, layer, n)
            assert np.array_equal(cache[layer][0][0], k.reshape(n, 2, 128).transpose(1, 0, 2))
            assert np.array_equal(cache[layer][1][0], v.reshape(n, 2, 128).transpose(1, 0, 2))
        # import into the other slot, every layer, then read back token-major
        for layer in range(qo.LAYERS):
            eng.write_kv_hf(1, layer, cache[layer][0], cache[layer][1])
        assert eng.seq_len(1) == n
        for layer in (0, 27):
            k0, v0 = eng.read_kv(0, layer, n)
            k1, v1 = eng.read_kv(1, layer, n)
            assert np.array_equal(k0, k1) and np.array_equal(v0, v1)
        # both slots continue identically from the same cache
        t = int(np.argmax(eng.read_logits(1)[0]))
        assert int(eng.decode([0], [t])[0]) == int(eng.decode([1], [t])[0])
    finally:
        eng.close()


@pytest.mark.parametrize("wbits", [4, 8])
def test_chunked_prefill_matches_whole_prompt(host, wbits):
    """qwen_engine_prefill_chunk: a prompt prefilled in chunks (the second and third continuing the slot's cached
    rows, with boundaries off the 64-token pages and 128-query tiles) gives the whole-prompt prefill's next token
    and K/V rows. The tensor-core path reorders fp32 sums by tile, so rows agree within 1e-5; the "exact" option
    computes per output in a fixed order, so there the rows, the last hidden state and the token are identical."""
    prompt = [int(t) for t in np.random.default_rng(17).integers(0, qo.VOCAB, 200)]
    cuts = [(0, 130), (130, 131), (131, 200)]
    for exact in (0, 1):
        eng = host.Engine(0, wbits, max_seqs=2, max_len=256)
        try:
            eng.init_synthetic(12)
            eng.set_option("exact", exact)
            eng.set_option("dump_hidden", 1)
            whole = eng.prefill(0, prompt)
            h_whole = eng.read_hidden(1)[:, 0].copy()
            for a, b in cuts:
                part = eng.prefill_chunk(1, prompt[a:b])
            h_chunk = eng.read_hidden(1)[:, 0].copy()
            assert eng.seq_len(1) == len(prompt)
            assert part == whole
            for layer in (0, 27):
                k0, v0 = eng.read_kv(0, layer, len(prompt))
                k1, v1 = eng.read_kv(1, layer, len(prompt))
                if exact:
                    assert np.array_equal(k0, k1) and np.array_equal(v0, v1), layer
                else:
                    # layer 0's rows come from identical inputs; later layers inherit attention reordering
                    assert rel_l2(k1, k0) <= 1e-5 and rel_l2(v1, v0) <= 1e-5, layer
            if exact:
                assert np.array_equal(h_chunk, h_whole)
            # both slots continue with the same greedy step
            assert int(eng.decode([0], [whole])[0]) == int(eng.decode([1], [whole])[0])
        finally:
            eng.close()
