"""Device-resident decode step of a Llama-shaped model (the reference's
Context::forward for one token, src/core/context.cpp:84-282), built on the
library's kernels:

  embed -> per layer [rms_norm -> QKV GEMV -> rope + fp16 KV append ->
  attention -> O GEMV -> residual add -> rms_norm -> gate|up GEMV ->
  silu*mul -> down GEMV -> residual add] -> rms_norm -> output GEMV -> argmax

Q, K, V share one weight (rows stacked: the GEMV reads the activation once),
and so do gate and up.  The token and position live on the device and argmax
advances them, so a step is captured once as a CUDA graph and replayed per
token with no host work; the generated tokens are recorded on the device.

Differences from the reference, by design: the KV cache is fp16 (the
reference keeps fp32, context.cpp:55-56), and attention covers positions
0..pos of the cache (the reference's causal mask uses the query's index
within the current chunk, cpu_backend.cpp:576-582, so a single decode token
attends only to position 0).
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass, field
from typing import Optional

from . import (ACT_Q8, FLAG_PDL, ODI_DTYPE_Q4_K, ODI_DTYPE_Q6_K, DeviceWeight, _ptr, check, lib, quantize_weight,
               repack)


class DecodeState(ctypes.Structure):
    """odi_cuda_decode_state (include/odi_cuda.h)."""

    _fields_ = [("token", ctypes.c_int32), ("pos", ctypes.c_int32), ("step", ctypes.c_int32),
                ("reserved", ctypes.c_int32)]


@dataclass
class LlamaConfig:
    layers: int = 32
    hidden: int = 4096
    heads: int = 32
    kv_heads: int = 32
    head_dim: int = 128
    ffn: int = 11008
    vocab: int = 32000
    ctx: int = 4096
    eps: float = 1e-5
    theta: float = 10000.0
    attn_dtype: int = ODI_DTYPE_Q4_K   # Q, K, V, O and gate/up
    down_dtype: int = ODI_DTYPE_Q6_K   # down and output
    act_mode: int = ACT_Q8

    @property
    def qkv_rows(self) -> int:
        return (self.heads + 2 * self.kv_heads) * self.head_dim

    def weight_bytes(self) -> int:
        """Packed weight bytes streamed per token (GGUF sizes)."""
        from . import gguf_bytes

        E, F = self.hidden, self.ffn
        per_layer = (gguf_bytes(self.attn_dtype, self.qkv_rows, E) + gguf_bytes(self.attn_dtype, E, self.heads * self.head_dim)
                     + gguf_bytes(self.attn_dtype, 2 * F, E) + gguf_bytes(self.down_dtype, E, F))
        return self.layers * per_layer + gguf_bytes(self.down_dtype, self.vocab, E)

    def kv_bytes(self, kv_len: int) -> int:
        """fp16 K and V bytes read per token at kv_len cached positions."""
        return self.layers * 2 * self.kv_heads * kv_len * self.head_dim * 2


@dataclass
class LayerWeights:
    attn_norm: object
    wqkv: DeviceWeight
    wo: DeviceWeight
    ffn_norm: object
    wgu: DeviceWeight
    wdown: DeviceWeight


@dataclass
class ModelWeights:
    token_embd: object           # fp32 [vocab, hidden]
    layers: list = field(default_factory=list)
    out_norm: object = None
    output: Optional[DeviceWeight] = None


def _seeded_quant(dtype: int, N: int, K: int, gen, device, std: float = 0.02) -> DeviceWeight:
    import torch

    w = torch.empty((N, K), dtype=torch.float32, device=device).normal_(0.0, std, generator=gen)
    blocks = quantize_weight(dtype, w)
    del w
    tiled = repack(dtype, blocks, N, K)
    del blocks
    return DeviceWeight.from_tiled(dtype, N, K, tiled)


def seeded_model(cfg: LlamaConfig, seed: int = 0, device=None) -> ModelWeights:
    """A random-init model of the given shape: weights N(0, 0.02) quantised on
    the device (attention and gate/up cfg.attn_dtype, down and output
    cfg.down_dtype), norm weights 1 + N(0, 0.02), embeddings N(0, 1)."""
    import torch

    device = device or torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    E, F = cfg.hidden, cfg.ffn

    def norm():
        return 1.0 + torch.empty(E, dtype=torch.float32, device=device).normal_(0.0, 0.02, generator=gen)

    mw = ModelWeights(token_embd=torch.empty((cfg.vocab, E), dtype=torch.float32, device=device)
                      .normal_(0.0, 1.0, generator=gen))
    for _ in range(cfg.layers):
        mw.layers.append(LayerWeights(
            attn_norm=norm(),
            wqkv=_seeded_quant(cfg.attn_dtype, cfg.qkv_rows, E, gen, device),
            wo=_seeded_quant(cfg.attn_dtype, E, cfg.heads * cfg.head_dim, gen, device),
            ffn_norm=norm(),
            wgu=_seeded_quant(cfg.attn_dtype, 2 * F, E, gen, device),
            wdown=_seeded_quant(cfg.down_dtype, E, F, gen, device)))
    mw.out_norm = norm()
    mw.output = _seeded_quant(cfg.down_dtype, cfg.vocab, E, gen, device)
    return mw


class DecodeModel:
    """One sequence decoded on the device.  ``step()`` enqueues one token's
    forward pass (embed .. argmax) on ``stream``; ``capture()`` records it as
    a CUDA graph that ``generate`` replays."""

    def __init__(self, cfg: LlamaConfig, weights: ModelWeights, device=None, max_record: int = 4096,
                 fused: bool = True, records: bool = True):
        import torch

        self.cfg, self.w = cfg, weights
        # fused: RMSNorm, SwiGLU and the residual adds run inside the GEMVs
        # (odi_cuda_matmul_fused); otherwise as separate kernels
        self.fused = fused
        # records (with fused): every GEMV input is quantized once into Q8
        # records -- by a small kernel that also applies RMSNorm / SwiGLU, or
        # by the attention itself -- instead of by every CTA of the GEMV
        self.records = fused and records and cfg.act_mode == ACT_Q8
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        dev, f32 = self.device, torch.float32
        E, F, H, hd = cfg.hidden, cfg.ffn, cfg.heads, cfg.head_dim
        self.x = torch.zeros(E, dtype=f32, device=dev)
        self.h = torch.zeros(E, dtype=f32, device=dev)
        self.qkv = torch.zeros(cfg.qkv_rows, dtype=f32, device=dev)
        self.attn = torch.zeros(H * hd, dtype=f32, device=dev)
        self.o = torch.zeros(E, dtype=f32, device=dev)
        self.gu = torch.zeros(2 * F, dtype=f32, device=dev)
        self.a = torch.zeros(F, dtype=f32, device=dev)
        self.logits = torch.zeros(cfg.vocab, dtype=f32, device=dev)
        # sums of squares of x per 64 values, left by x's writer (embed or a
        # residual GEMV) for the next fused RMSNorm
        self.ssq_slots = (E + 63) // 64
        self.ssq = torch.zeros(self.ssq_slots, dtype=f32, device=dev)
        rb = lib().odi_cuda_q8_records_bytes
        self.rec_e = torch.zeros(rb(1, E), dtype=torch.uint8, device=dev)        # x (normalised)
        self.rec_a = torch.zeros(rb(1, H * hd), dtype=torch.uint8, device=dev)   # attention output
        self.rec_f = torch.zeros(rb(1, F), dtype=torch.uint8, device=dev)        # SwiGLU output
        self.kc = torch.zeros((cfg.layers, cfg.kv_heads, cfg.ctx, hd), dtype=torch.float16, device=dev)
        self.vc = torch.zeros_like(self.kc)
        sb = lib().odi_cuda_attention_scratch_bytes(H, hd, cfg.ctx)
        self.att_scratch = torch.zeros(max(sb, 16) // 4 + 1, dtype=f32, device=dev)
        self.state = torch.zeros(4, dtype=torch.int32, device=dev)  # odi_cuda_decode_state
        self.max_record = max_record
        self.record = torch.full((max_record,), -1, dtype=torch.int32, device=dev)
        self.stream = torch.cuda.Stream(device=dev)
        self.graph = None
        self._host_state = torch.zeros(4, dtype=torch.int32).pin_memory()
        # every GEMV's workspace (error word), allocated before any capture
        for lw in self.w.layers:
            for dw in (lw.wqkv, lw.wo, lw.wgu, lw.wdown):
                dw._ws_for(1, cfg.act_mode, dev)
        self.w.output._ws_for(1, cfg.act_mode, dev)
        # error words of every kernel with bounded waits (the GEMV workspaces'
        # and the attention scratch's first int), gathered in one read
        words = [self.att_scratch.view(torch.int32)[:1]]
        for lw in self.w.layers:
            for dw in (lw.wqkv, lw.wo, lw.wgu, lw.wdown):
                words.append(dw._ws.view(torch.int32)[:1])
        words.append(self.w.output._ws.view(torch.int32)[:1])
        self._err_words = words
        # the buffers and the weights were filled on the current stream: the
        # model's own stream must not run ahead of those fills
        self.stream.wait_stream(torch.cuda.current_stream(dev))

    def status(self) -> int:
        """OR of the device error words (0: no bounded wait gave up)."""
        import torch

        self.stream.synchronize()
        with torch.cuda.stream(self.stream):
            words = torch.cat(self._err_words).cpu().tolist()
        v = 0
        for x in words:
            v |= x
        return v

    def _check_status(self) -> None:
        st = self.status()
        if st:
            raise RuntimeError(f"decode step: a bounded device wait gave up (error word {st:#x})")

    # ---- one step ----------------------------------------------------------
    def _gemv(self, dw: DeviceWeight, x, y, s):
        ws = dw._ws
        check(lib().odi_cuda_matmul(dw.dtype, dw.data_ptr, _ptr(x), _ptr(y), 1, dw.N, dw.K, self.cfg.act_mode,
                                    _ptr(ws), ws.numel(), FLAG_PDL, s))

    def _gemv_fused(self, dw: DeviceWeight, x, y, s, norm=None, swiglu=False, accumulate=False):
        """norm: RMSNorm of x from the sums of squares its writer left in
        self.ssq; accumulate: y += product, leaving y's sums of squares."""
        from . import MatmulOpts

        ssq = _ptr(self.ssq)
        o = MatmulOpts(_ptr(norm) if norm is not None else None, self.cfg.eps, 1 if swiglu else 0,
                       1 if accumulate else 0, ssq if norm is not None else None, self.ssq_slots,
                       ssq if accumulate else None)
        ws = dw._ws
        check(lib().odi_cuda_matmul_fused(dw.dtype, dw.data_ptr, _ptr(x), _ptr(y), 1, dw.N, dw.K, self.cfg.act_mode,
                                          _ptr(ws), ws.numel(), FLAG_PDL, ctypes.byref(o), s))

    def _opts(self, norm=None, swiglu=False, accumulate=False):
        from . import MatmulOpts

        ssq = _ptr(self.ssq)
        return MatmulOpts(_ptr(norm) if norm is not None else None, self.cfg.eps, 1 if swiglu else 0,
                          1 if accumulate else 0, ssq if norm is not None else None, self.ssq_slots,
                          ssq if accumulate else None)

    def _records(self, x, K, rec, s, norm=None, swiglu=False):
        o = self._opts(norm=norm, swiglu=swiglu)
        check(lib().odi_cuda_quantize_records(_ptr(x), 1, K, ctypes.byref(o), _ptr(rec), FLAG_PDL, s))

    def _gemv_rec(self, dw: DeviceWeight, rec, y, s, accumulate=False):
        o = self._opts(accumulate=accumulate)
        ws = dw._ws
        check(lib().odi_cuda_matmul_q8rec(dw.dtype, dw.data_ptr, _ptr(rec), _ptr(y), 1, dw.N, dw.K, _ptr(ws),
                                          ws.numel(), FLAG_PDL, ctypes.byref(o), s))

    def step(self) -> None:
        if self.records:
            self._step_records()
        elif self.fused:
            self._step_fused()
        else:
            self._step_unfused()

    def _step_records(self) -> None:
        """8 launches per layer, every GEMV on pre-quantized records: records
        of RMSNorm(x), QKV GEMV, attention (rope and the KV append fused in,
        writing the O GEMV's records), O GEMV (+= x), records of RMSNorm(x),
        gate|up GEMV, records of SwiGLU(gate|up), down GEMV (+= x)."""
        cfg, L, s = self.cfg, lib(), self.stream.cuda_stream
        E, F, H, KV, hd = cfg.hidden, cfg.ffn, cfg.heads, cfg.kv_heads, cfg.head_dim
        st = _ptr(self.state)
        q = _ptr(self.qkv)
        k = q + H * hd * 4
        v = k + KV * hd * 4
        scale = 1.0 / math.sqrt(hd)
        check(L.odi_cuda_embed(_ptr(self.w.token_embd), cfg.vocab, E, st, _ptr(self.x), _ptr(self.ssq), s))
        for li, lw in enumerate(self.w.layers):
            kc, vc = _ptr(self.kc[li]), _ptr(self.vc[li])
            self._records(self.x, E, self.rec_e, s, norm=lw.attn_norm)
            self._gemv_rec(lw.wqkv, self.rec_e, self.qkv, s)
            check(L.odi_cuda_rope_attention(q, k, v, kc, vc, _ptr(self.attn), _ptr(self.rec_a), st, H, KV, hd,
                                            cfg.ctx, cfg.theta, scale, _ptr(self.att_scratch),
                                            self.att_scratch.numel() * 4, s))
            self._gemv_rec(lw.wo, self.rec_a, self.x, s, accumulate=True)
            self._records(self.x, E, self.rec_e, s, norm=lw.ffn_norm)
            self._gemv_rec(lw.wgu, self.rec_e, self.gu, s)
            self._records(self.gu, F, self.rec_f, s, swiglu=True)
            self._gemv_rec(lw.wdown, self.rec_f, self.x, s, accumulate=True)
        self._records(self.x, E, self.rec_e, s, norm=self.w.out_norm)
        self._gemv_rec(self.w.output, self.rec_e, self.logits, s)
        check(L.odi_cuda_argmax(_ptr(self.logits), cfg.vocab, st, _ptr(self.record), self.max_record, s))

    def _step_fused(self) -> None:
        """5 launches per layer: QKV GEMV (RMSNorm fused), attention (rope and
        the KV append fused), O GEMV (+= x), gate|up GEMV (RMSNorm fused),
        down GEMV (SwiGLU fused, += x)."""
        cfg, L, s = self.cfg, lib(), self.stream.cuda_stream
        H, KV, hd = cfg.heads, cfg.kv_heads, cfg.head_dim
        st = _ptr(self.state)
        q = _ptr(self.qkv)
        k = q + H * hd * 4
        v = k + KV * hd * 4
        scale = 1.0 / math.sqrt(hd)
        check(L.odi_cuda_embed(_ptr(self.w.token_embd), cfg.vocab, cfg.hidden, st, _ptr(self.x), _ptr(self.ssq), s))
        for li, lw in enumerate(self.w.layers):
            kc, vc = _ptr(self.kc[li]), _ptr(self.vc[li])
            self._gemv_fused(lw.wqkv, self.x, self.qkv, s, norm=lw.attn_norm)
            check(L.odi_cuda_rope_attention(q, k, v, kc, vc, _ptr(self.attn), None, st, H, KV, hd, cfg.ctx,
                                            cfg.theta, scale, _ptr(self.att_scratch), self.att_scratch.numel() * 4,
                                            s))
            self._gemv_fused(lw.wo, self.attn, self.x, s, accumulate=True)
            self._gemv_fused(lw.wgu, self.x, self.gu, s, norm=lw.ffn_norm)
            self._gemv_fused(lw.wdown, self.gu, self.x, s, swiglu=True, accumulate=True)
        self._gemv_fused(self.w.output, self.x, self.logits, s, norm=self.w.out_norm)
        check(L.odi_cuda_argmax(_ptr(self.logits), cfg.vocab, st, _ptr(self.record), self.max_record, s))

    def _step_unfused(self) -> None:
        cfg, L, s = self.cfg, lib(), self.stream.cuda_stream
        E, F, H, KV, hd = cfg.hidden, cfg.ffn, cfg.heads, cfg.kv_heads, cfg.head_dim
        st = _ptr(self.state)
        q = _ptr(self.qkv)
        k = q + H * hd * 4
        v = k + KV * hd * 4
        scale = 1.0 / math.sqrt(hd)
        check(L.odi_cuda_embed(_ptr(self.w.token_embd), cfg.vocab, E, st, _ptr(self.x), None, s))
        for li, lw in enumerate(self.w.layers):
            kc, vc = _ptr(self.kc[li]), _ptr(self.vc[li])
            check(L.odi_cuda_rms_norm(_ptr(self.x), _ptr(lw.attn_norm), _ptr(self.h), 1, E, cfg.eps, s))
            self._gemv(lw.wqkv, self.h, self.qkv, s)
            check(L.odi_cuda_rope_kv(q, k, v, kc, vc, st, H, KV, hd, cfg.ctx, cfg.theta, s))
            check(L.odi_cuda_attention_decode(q, kc, vc, _ptr(self.attn), st, H, KV, hd, cfg.ctx, scale,
                                              _ptr(self.att_scratch), self.att_scratch.numel() * 4, s))
            self._gemv(lw.wo, self.attn, self.o, s)
            check(L.odi_cuda_add(_ptr(self.x), _ptr(self.o), E, s))
            check(L.odi_cuda_rms_norm(_ptr(self.x), _ptr(lw.ffn_norm), _ptr(self.h), 1, E, cfg.eps, s))
            self._gemv(lw.wgu, self.h, self.gu, s)
            check(L.odi_cuda_silu_mul(_ptr(self.gu), _ptr(self.a), F, s))
            self._gemv(lw.wdown, self.a, self.o, s)
            check(L.odi_cuda_add(_ptr(self.x), _ptr(self.o), E, s))
        check(L.odi_cuda_rms_norm(_ptr(self.x), _ptr(self.w.out_norm), _ptr(self.h), 1, E, cfg.eps, s))
        self._gemv(self.w.output, self.h, self.logits, s)
        check(L.odi_cuda_argmax(_ptr(self.logits), cfg.vocab, st, _ptr(self.record), self.max_record, s))

    def launches_per_step(self) -> int:
        if self.records:
            return 1 + 8 * self.cfg.layers + 3  # embed, per layer, records + output GEMV + argmax
        if self.fused:
            return 1 + 5 * self.cfg.layers + 2  # embed, per layer, output GEMV + argmax
        return 1 + 10 * self.cfg.layers + 3  # embed, per layer, final norm + output GEMV + argmax

    def capture(self) -> None:
        """Record one step as a CUDA graph (after one eager step has run)."""
        import torch

        with torch.cuda.stream(self.stream):
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=self.stream):
                self.step()
        self.stream.synchronize()

    def _run(self) -> None:
        import torch

        with torch.cuda.stream(self.stream):
            if self.graph is not None:
                self.graph.replay()
            else:
                self.step()

    # ---- sequences ---------------------------------------------------------
    def clear_cache(self) -> None:
        """Zero the KV cache (a new sequence)."""
        import torch

        with torch.cuda.stream(self.stream):
            self.kc.zero_()
            self.vc.zero_()

    def reset(self, token: int, pos: int = 0) -> None:
        """Next step consumes `token` at position `pos`; the record restarts."""
        import torch

        if not 0 <= token < self.cfg.vocab:
            raise ValueError(f"token {token} outside the vocabulary")
        if not 0 <= pos < self.cfg.ctx:
            raise ValueError(f"position {pos} outside the context of {self.cfg.ctx}")
        self._host_state.copy_(torch.tensor([token, pos, 0, 0], dtype=torch.int32))
        with torch.cuda.stream(self.stream):
            self.state.copy_(self._host_state, non_blocking=True)
            self.record.fill_(-1)

    def prefill(self, tokens) -> None:
        """Run the prompt through the cache one token at a time (each step's
        own argmax is overwritten by the next prompt token)."""
        import torch

        if len(tokens) >= self.cfg.ctx:
            raise ValueError("prompt longer than the context")
        host = torch.tensor([[t, i, 0, 0] for i, t in enumerate(tokens)], dtype=torch.int32).pin_memory()
        for i in range(len(tokens)):
            with torch.cuda.stream(self.stream):
                self.state.copy_(host[i], non_blocking=True)
            self._run()
        self._check_status()

    def generate(self, n: int) -> list:
        """n greedy steps from the current state; returns the n tokens."""
        import torch

        self.stream.synchronize()
        cur = self.state.cpu()
        if int(cur[1]) + n > self.cfg.ctx:
            raise ValueError("generation would run past the context")
        start = int(cur[2])
        for _ in range(n):
            self._run()
        self._check_status()
        return self.record[start:start + n].cpu().tolist()
