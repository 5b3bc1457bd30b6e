"""Single-token decode of a Qwen2-shaped model on the CPU oracle -- TEST
INFRASTRUCTURE ONLY (imported by tests/ and bench.py's CPU legs, never by the
product package).

Restates the reference's fast single-token decode path,
``src/inference/cpu_engine.rs:2819-3064`` (``spec_len == 0`` branch), for a
dense (non-MoE) model:

    x = embed[token % vocab]                                          :2821-2825
    per layer:
      h = rms_norm(x, input_layernorm)                                :2866
      q, k, v = W_q h, W_k h, W_v h (+ biases)                        :2873-2897
      rope(q, pos), rope(k, pos)                                      :2902-2903
      append k, v to the layer's cache                                :2909
      a = attention(q, cache[0..pos])                                 :2913-2921
      x += W_o a (+ bias)                                             :2927-2939
      h2 = rms_norm(x, post_attention_layernorm)                      :2944
      x += W_down (silu(W_gate h2) * W_up h2)                         :2950-2968 (run_mlp_into :1990-2031)
    logits = W_lm rms_norm(x, norm)                                   :2974-2976
    token = argmax(penalise(logits, generated))                       :2985-3031

The linears use the oracle's restatement of ``matvec_mul_into``
(cpu_engine.rs:1307-1444) on the quantized weights; the other operations the C
restatements in ``bramha_oracle.c``.  Whole-model parity is not pinned by the
reference's own tests (its golden test is tautological); this restatement is the
checker.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

import oracle


@dataclass
class Qwen2Config:
    layers: int = 24
    hidden: int = 896
    heads: int = 14
    kv_heads: int = 2
    head_dim: int = 64
    intermediate: int = 4864
    vocab: int = 151936
    eps: float = 1e-6
    rope_theta: float = 1e6


@dataclass
class Linear:
    fmt: str
    n: int
    k: int
    q: np.ndarray
    s: np.ndarray

    def __call__(self, h: np.ndarray) -> np.ndarray:
        return oracle.matvec_mul_into(self.fmt, np.ascontiguousarray(h, np.float32), self.q, self.s, self.n)


@dataclass
class Layer:
    ln1: np.ndarray
    q: Linear
    k: Linear
    v: Linear
    bq: np.ndarray
    bk: np.ndarray
    bv: np.ndarray
    o: Linear
    ln2: np.ndarray
    gate: Linear
    up: Linear
    down: Linear


@dataclass
class Model:
    cfg: Qwen2Config
    embed: np.ndarray          # [vocab][hidden] f32
    layers: list
    norm: np.ndarray
    lm_head: Linear
    k_cache: list = field(default_factory=list)   # per layer: [t][kv_heads * head_dim]
    v_cache: list = field(default_factory=list)

    def reset(self):
        self.k_cache = [[] for _ in self.layers]
        self.v_cache = [[] for _ in self.layers]

    def forward(self, token: int, pos: int) -> np.ndarray:
        """Logits for `token` at position `pos` (the cache must hold positions < pos)."""
        c = self.cfg
        x = self.embed[token % c.vocab].astype(np.float32).copy()
        for li, L in enumerate(self.layers):
            h = oracle.rms_norm(x, L.ln1, c.eps)
            q = (L.q(h) + L.bq).astype(np.float32)
            k = (L.k(h) + L.bk).astype(np.float32)
            v = (L.v(h) + L.bv).astype(np.float32)
            oracle.rope_(q, pos, c.heads, c.head_dim, c.rope_theta)
            oracle.rope_(k, pos, c.kv_heads, c.head_dim, c.rope_theta)
            self.k_cache[li].append(k)
            self.v_cache[li].append(v)
            kv_len = len(self.k_cache[li])
            a = oracle.attention(q, np.stack(self.k_cache[li]), np.stack(self.v_cache[li]), kv_len, c.heads,
                                 c.kv_heads, c.head_dim)
            x = (x + L.o(a)).astype(np.float32)
            h2 = oracle.rms_norm(x, L.ln2, c.eps)
            m = oracle.silu_mul(L.gate(h2), L.up(h2))
            x = (x + L.down(m)).astype(np.float32)
        hf = oracle.rms_norm(x, self.norm, c.eps)
        return self.lm_head(hf)
