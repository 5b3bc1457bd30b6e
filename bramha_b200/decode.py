"""Single-token decode of a dense Qwen2-shaped model on the GPU.

The step restates the reference's fast decode path
(src/inference/cpu_engine.rs:2819-3064, ``spec_len == 0``):

    x = embed[token]; per layer: h = norm(x); q|k|v = W h (+ bias); RoPE;
    KV append; a = attention(q); x += W_o a; h = norm(x);
    x += W_down (silu(W_gate h) * W_up h); then logits = W_lm norm(x),
    repetition penalty 1.15 and greedy argmax.

The linears are the GEMVs of the quantized formats (q|k|v and gate|up each
one launch), SiLU * up formed by the down GEMV (``bramha_cuda_gemv_swiglu_dev``);
everything else is the ``bramha_cuda_op_*`` kernels (bias + RoPE + KV append
fused into the attention launch).  With ``fuse_norm`` each pre-norm block's
residual add + RMSNorm is formed by the GEMV that reads it instead
(``bramha_cuda_gemv_rmsnorm_dev``: one launch when the CUDA-core GEMV takes
the weights; the residual stream is double-buffered so the GEMV's CTAs can
write the new residual while others still read the old).  That saves two
launches per layer but is not the default: measured on the Qwen2-0.5B step,
2.31 ms per token fused against 2.25 with the separate RMSNorm kernel (whose
launch overlaps the previous kernel; the fused GEMV does the whole-vector
reduction after its dependency wait, in every CTA).  Token id and position live in device
memory, so a step is captured once in a CUDA graph and replayed token after
token with no host work: ``greedy`` steps pick the next token on the device,
teacher-forced steps (prompt prefill, parity checks) take a token the host
writes before the replay.  torch supplies device memory and streams only.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Sequence

from ._lib import check, lib
from .plane import CudaComputePlane, Weight


# formats whose down GEMV forms silu(gate) * up itself (bramha_cuda_gemv_swiglu_dev)
_FUSED_SWIGLU = ("log4", "w4zp8", "w8")
_SLICE = {"log4": 32, "w4zp8": 32, "w8": 64}  # packed bytes per row per 64-column block


def _norm_one_launch(ws) -> bool:
    """Whether bramha_cuda_gemv_rmsnorm_dev runs `ws` as one launch: the
    CUDA-core GEMV's default choice (tiled format, K <= 1024 and even, at most
    8 MB of packed tiles) -- otherwise it runs the RMSNorm kernel first."""
    fmt, k = ws[0].fmt, ws[0].K
    if fmt not in _SLICE or k > 1024 or k % 2:
        return False
    tiles = sum((w.N + 127) // 128 for w in ws)
    return tiles * ((k + 63) // 64) * 128 * _SLICE[fmt] <= (8 << 20)


@dataclass
class DecodeConfig:
    layers: int = 24
    hidden: int = 896
    heads: int = 14
    kv_heads: int = 2
    head_dim: int = 64
    intermediate: int = 4864
    vocab: int = 151936
    eps: float = 1e-6
    rope_theta: float = 1e6
    rep_penalty: float = 1.15  # cpu_engine.rs:2985


@dataclass
class DecodeLayer:
    """One decoder layer: norm weights and biases as torch CUDA f32 tensors
    (biases may be None), linears as registered :class:`Weight` objects."""
    ln1: object
    q: Weight
    k: Weight
    v: Weight
    bq: Optional[object]
    bk: Optional[object]
    bv: Optional[object]
    o: Weight
    ln2: object
    gate: Weight
    up: Weight
    down: Weight


def _p(t) -> Optional[int]:
    return None if t is None else t.data_ptr()


class DecodeModel:
    """Holds the activations, KV cache and token state of one decode stream."""

    def __init__(self, plane: CudaComputePlane, cfg: DecodeConfig, layers: Sequence[DecodeLayer], embed, norm,
                 lm_head: Weight, max_ctx: int = 1024, max_generated: int = 4096, stream=None,
                 fuse_norm=False):
        import torch

        c = self.cfg = cfg
        self.plane, self.layers, self.embed, self.norm, self.lm_head = plane, list(layers), embed, norm, lm_head
        self.max_ctx, self.max_generated = max_ctx, max_generated
        dev = embed.device
        self.stream = stream if stream is not None else torch.cuda.Stream(device=dev)
        f32, i32 = torch.float32, torch.int32
        qd, kvd = c.heads * c.head_dim, c.kv_heads * c.head_dim
        if len(self.layers) != c.layers:
            raise ValueError(f"{len(self.layers)} layers given, config has {c.layers}")
        if max_ctx > 51200:
            raise ValueError("max_ctx above the attention kernel's limit (51200)")
        # which residual adds + RMSNorms the GEMV that reads them forms: True (both
        # of a layer), "mlp" (the one before gate|up) or False (none)
        if fuse_norm not in (True, False, "mlp"):
            raise ValueError(f"fuse_norm must be True, False or 'mlp' (got {fuse_norm!r})")
        self.fuse_norm = fuse_norm
        self.residual = None
        self.x = torch.zeros(c.hidden, dtype=f32, device=dev)
        self.x2 = torch.zeros(c.hidden, dtype=f32, device=dev)  # the other residual buffer (fused norms)
        self.h = torch.zeros(c.hidden, dtype=f32, device=dev)
        self.qkv = torch.zeros(qd + 2 * kvd, dtype=f32, device=dev)
        self.q, self.k, self.v = self.qkv[:qd], self.qkv[qd:qd + kvd], self.qkv[qd + kvd:]
        self.attn = torch.zeros(qd, dtype=f32, device=dev)
        self.o = torch.zeros(c.hidden, dtype=f32, device=dev)
        self.gu = torch.zeros(2 * c.intermediate, dtype=f32, device=dev)
        self.g, self.u = self.gu[:c.intermediate], self.gu[c.intermediate:]
        self.m = torch.zeros(c.intermediate, dtype=f32, device=dev)
        self.d = torch.zeros(c.hidden, dtype=f32, device=dev)
        self.logits = torch.zeros(c.vocab, dtype=f32, device=dev)
        self.k_cache = torch.zeros((c.layers, max_ctx, kvd), dtype=f32, device=dev)
        self.v_cache = torch.zeros((c.layers, max_ctx, kvd), dtype=f32, device=dev)
        self.token = torch.zeros(1, dtype=i32, device=dev)
        self.pos = torch.zeros(1, dtype=i32, device=dev)
        self.generated = torch.zeros(max_generated, dtype=i32, device=dev)
        self.count = torch.zeros(1, dtype=i32, device=dev)
        self._graphs = {}

    # ------------------------------------------------------------- state
    def reset(self):
        """Position 0, no generated tokens (the caches are overwritten as it advances)."""
        with self._on_stream():
            self.pos.zero_()
            self.count.zero_()

    def set_token(self, token: int):
        with self._on_stream():
            self.token.fill_(int(token))

    def position(self) -> int:
        self.stream.synchronize()
        return int(self.pos.item())

    def last_token(self) -> int:
        self.stream.synchronize()
        return int(self.token.item())

    def generated_tokens(self):
        self.stream.synchronize()
        return self.generated[: int(self.count.item())].cpu().tolist()

    def _on_stream(self):
        import torch
        return torch.cuda.stream(self.stream)

    # ------------------------------------------------------------- step
    def _launch_step(self, greedy: bool):
        """The launch sequence of one token (on self.stream)."""
        c, L, P = self.cfg, lib(), self.plane
        ctx, st = P.ctx, self.stream.cuda_stream
        check(L.bramha_cuda_op_embed(ctx, self.embed.data_ptr(), c.vocab, c.hidden, self.token.data_ptr(),
                                     self.x.data_ptr(), st))
        delta = None
        cur, other = self.x, self.x2  # the residual stream lives in `cur`
        fuse_attn, fuse_mlp = self.fuse_norm is True, self.fuse_norm in (True, "mlp")
        for li, lw in enumerate(self.layers):
            if fuse_attn:  # other = cur + delta; q|k|v = W norm(other)
                P.gemv_rmsnorm_dev([lw.q, lw.k, lw.v], cur, delta, lw.ln1, c.eps, other,
                                   [self.q, self.k, self.v], stream=self.stream)
                cur, other = other, cur
            else:
                check(L.bramha_cuda_op_rmsnorm(ctx, cur.data_ptr(), _p(delta), lw.ln1.data_ptr(), c.hidden,
                                               c.eps, self.h.data_ptr(), st))
                P.gemv_multi_dev([lw.q, lw.k, lw.v], self.h, [self.q, self.k, self.v], stream=self.stream)
            kc, vc = self.k_cache[li], self.v_cache[li]
            check(L.bramha_cuda_op_rope_attention(ctx, self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(),
                                                  _p(lw.bq), _p(lw.bk), _p(lw.bv), c.heads, c.kv_heads, c.head_dim,
                                                  c.rope_theta, self.pos.data_ptr(), self.max_ctx, kc.data_ptr(),
                                                  vc.data_ptr(), self.attn.data_ptr(), st))
            P.gemv_multi_dev([lw.o], self.attn, [self.o], stream=self.stream)
            if fuse_mlp:  # other = cur + o; gate|up = W norm(other)
                P.gemv_rmsnorm_dev([lw.gate, lw.up], cur, self.o, lw.ln2, c.eps, other, [self.g, self.u],
                                   stream=self.stream)
                cur, other = other, cur
            else:
                check(L.bramha_cuda_op_rmsnorm(ctx, cur.data_ptr(), self.o.data_ptr(), lw.ln2.data_ptr(),
                                               c.hidden, c.eps, self.h.data_ptr(), st))
                P.gemv_multi_dev([lw.gate, lw.up], self.h, [self.g, self.u], stream=self.stream)
            if lw.down.fmt in _FUSED_SWIGLU:  # silu(g) * u formed by the down GEMV itself
                P.gemv_swiglu_dev(lw.down, self.g, self.u, self.d, stream=self.stream)
            else:
                check(L.bramha_cuda_op_silu_mul(ctx, self.g.data_ptr(), self.u.data_ptr(), c.intermediate,
                                                self.m.data_ptr(), st))
                P.gemv_multi_dev([lw.down], self.m, [self.d], stream=self.stream)
            delta = self.d
        check(L.bramha_cuda_op_rmsnorm(ctx, cur.data_ptr(), _p(delta), self.norm.data_ptr(), c.hidden, c.eps,
                                       self.h.data_ptr(), st))
        self.residual = cur  # where the residual stream ends (x, or x2 after an odd number of swaps)
        P.gemv_multi_dev([self.lm_head], self.h, [self.logits], stream=self.stream)
        check(L.bramha_cuda_op_select(ctx, self.logits.data_ptr(), c.vocab, self.generated.data_ptr(),
                                      self.count.data_ptr(), self.max_generated, c.rep_penalty, 1 if greedy else 0,
                                      self.token.data_ptr(), self.pos.data_ptr(), st))

    def kernel_launches_per_step(self) -> int:
        """Launches of this library's kernels in one step: the embedding, per layer
        4 GEMVs, the attention and two RMSNorms (none where the GEMV forms them;
        a SiLU when the down weight is f32), then
        the final norm, lm_head and selection (device-to-device copies not counted)."""
        n = 1 + 3
        for lw in self.layers:
            n += 5 + (0 if lw.down.fmt in _FUSED_SWIGLU else 1)
            for ws, fused in (([lw.q, lw.k, lw.v], self.fuse_norm is True),
                              ([lw.gate, lw.up], self.fuse_norm in (True, "mlp"))):
                n += 0 if fused and _norm_one_launch(ws) else 1
        return n

    def step(self, greedy: bool = True):
        """One token: eagerly launched, or replayed from the captured graph."""
        g = self._graphs.get(bool(greedy))
        if g is not None:
            with self._on_stream():
                g.replay()
        else:
            self._launch_step(greedy)

    def capture(self):
        """Captures the greedy and the teacher-forced step in CUDA graphs.  Runs
        one eager step of each first (kernel set-up outside the capture) and
        leaves the state as it found it."""
        import torch

        pos0 = self.pos.clone()
        cnt0 = self.count.clone()
        tok0 = self.token.clone()
        for greedy in (False, True):
            self._launch_step(greedy)
            with self._on_stream():
                self.pos.copy_(pos0)
                self.count.copy_(cnt0)
                self.token.copy_(tok0)
        self.stream.synchronize()
        for greedy in (False, True):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=self.stream):
                self._launch_step(greedy)
            self._graphs[greedy] = g
        self.stream.synchronize()

    def release(self):
        self._graphs.clear()

    def sync(self):
        """Waits for the stream; raises if a kernel recorded a device-side failure."""
        self.plane.stream_sync(self.stream)
