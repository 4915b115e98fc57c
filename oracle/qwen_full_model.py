"""Full-model oracle harness: the reference caller's flow (verification/real_host_top_backend.py:208-351)
on synthetic parameters, with every layer computed either by the C restatement (libqwen_oracle.so) or
by the reference's own host libraries through their top-wrapper ABI.

TEST INFRASTRUCTURE ONLY (tests/, smoke(), bench.py CPU legs).

Per layer: prefill via `qwen_prefill_top_smoke_forward` semantics (activation DDR = input | output |
scratch), decode via `qwen_decode_top_smoke_forward` semantics; hidden states are rounded to bf16 after
every layer (:260, :334); KV is kept in the reference's token-major layout. Embedding, final RMSNorm and
the tied fp16 LM head are the harness definitions in qwen_oracle.c (`oracle_lm_head_argmax`), since the
Hugging Face modules the reference uses are not available.
"""
from __future__ import annotations

import numpy as np

import qwen_oracle as qo


class OracleModel:
    def __init__(self, seed: int, wbits: int = 4, layers: int = qo.LAYERS, use_reference_libs: bool = False,
                 ref_prefill_path=None):
        self.seed = seed
        self.wbits = wbits
        self.n_layers = layers
        self.params = [qo.synth_layer(seed, l, wbits) for l in range(layers)]
        self.embed = qo.synth_embedding(seed)
        self.final_norm = qo.synth_final_norm(seed)
        self.ref = None
        if use_reference_libs:
            if wbits != 4:
                raise ValueError("the reference libraries only take int4 weights")
            self.ref = qo.RefLibs(prefill_path=ref_prefill_path or qo.REF_PREFILL_LIB)
            self.ddr = [p.ddr() for p in self.params]
        self.k = [None] * layers  # per layer flat [len][256]
        self.v = [None] * layers
        self.len = 0
        self.hidden_trace: list[np.ndarray] = []

    def embed_rows(self, tokens) -> np.ndarray:
        return self.embed[np.asarray(tokens, dtype=np.int64)].view(np.float16).astype(np.float32)

    def _prefill_layer(self, l: int, x: np.ndarray, S: int):
        kc = np.zeros(S * qo.KV_WIDTH, np.float32)
        vc = np.zeros(S * qo.KV_WIDTH, np.float32)
        if self.ref is None:
            st, out = qo.prefill_layer(self.params[l], x, S, kc, vc)
            assert st == 0, st
            return out, kc, vc
        wd, sd = self.ddr[l]
        act = np.zeros(3 * S * qo.HIDDEN, np.float32)
        act[:S * qo.HIDDEN] = x.reshape(-1)
        kv = np.zeros(2 * S * qo.KV_WIDTH, np.float32)
        st = self.ref.prefill.qwen_prefill_top_smoke_forward(
            l, S, *qo.tiles_tuple(), 0, S * qo.HIDDEN * 4, 0, 0, 0, S * qo.KV_WIDTH * 4, wd, sd, kv, act,
            *qo.sram_ports())
        assert st == 0, st
        return act[S * qo.HIDDEN:2 * S * qo.HIDDEN].copy(), kv[:S * qo.KV_WIDTH].copy(), kv[S * qo.KV_WIDTH:].copy()

    def _decode_layer(self, l: int, x: np.ndarray, past: int):
        kc = np.zeros((past + 1) * qo.KV_WIDTH, np.float32)
        vc = np.zeros((past + 1) * qo.KV_WIDTH, np.float32)
        kc[:past * qo.KV_WIDTH] = self.k[l]
        vc[:past * qo.KV_WIDTH] = self.v[l]
        if self.ref is None:
            st, out = qo.decode_layer(self.params[l], x, past, kc, vc)
            assert st == 0, st
            return out, kc, vc
        wd, sd = self.ddr[l]
        act = np.zeros(2 * qo.HIDDEN, np.float32)
        act[:qo.HIDDEN] = x
        kv = np.concatenate([kc, vc])
        st = self.ref.decode.qwen_decode_top_smoke_forward(l, past, 0, qo.HIDDEN * 4, 0, 0, 0, kc.size * 4, wd, sd,
                                                           kv, act, *qo.sram_ports())
        assert st == 0, st
        return act[qo.HIDDEN:].copy(), kv[:kc.size].copy(), kv[kc.size:].copy()

    def prefill(self, tokens) -> int:
        S = len(tokens)
        x = self.embed_rows(tokens).reshape(-1)
        self.hidden_trace = []
        for l in range(self.n_layers):
            out, kc, vc = self._prefill_layer(l, x, S)
            x = qo.round_bf16(out)
            self.k[l], self.v[l] = kc, vc
            self.hidden_trace.append(x.reshape(S, qo.HIDDEN)[-1].copy())
        self.len = S
        return qo.lm_head_argmax(x.reshape(S, qo.HIDDEN)[-1], self.final_norm, self.embed)

    def decode(self, token: int) -> int:
        x = self.embed_rows([token]).reshape(-1)
        past = self.len
        self.hidden_trace = []
        for l in range(self.n_layers):
            out, kc, vc = self._decode_layer(l, x, past)
            x = qo.round_bf16(out)
            self.k[l], self.v[l] = kc, vc
            self.hidden_trace.append(x.copy())
        self.len = past + 1
        return qo.lm_head_argmax(x, self.final_norm, self.embed)

    def logits(self, hidden: np.ndarray) -> np.ndarray:
        return qo.lm_head_argmax(hidden, self.final_norm, self.embed, want_logits=True)[1]
