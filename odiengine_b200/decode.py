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
    # gate|up rows interleaved by 32 in every 64-row tile (interleave_gate_up):
    # the gate|up GEMV can then hand the down GEMV its SwiGLU records
    gu_interleaved: bool = False


def gate_up_order(F: int):
    """Row order of an interleaved gate|up weight: row p of the stored weight
    is row gate_up_order(F)[p] of the [gate F | up F] weight.  Every 64-row
    tile holds 32 gate rows and the 32 matching up rows (F % 32 == 0)."""
    import numpy as np

    if F % 32:
        raise ValueError("interleaving gate|up needs F % 32 == 0")
    p = np.arange(2 * F)
    t, i = p // 64, p % 64
    return np.where(i < 32, 32 * t + i, F + 32 * t + (i - 32))


def interleave_gate_up(blocks, F: int, row_bytes: int):
    """GGUF block rows of a [gate F | up F] weight (device uint8 tensor) in
    the interleaved order."""
    import torch

    idx = torch.as_tensor(gate_up_order(F), device=blocks.device)
    return blocks.view(2 * F, row_bytes).index_select(0, idx).reshape(-1)


def _seeded_quant(dtype: int, N: int, K: int, gen, device, std: float = 0.02, interleave: bool = False) -> DeviceWeight:
    import torch

    from . import gguf_bytes

    w = torch.empty((N, K), dtype=torch.float32, device=device).normal_(0.0, std, generator=gen)
    blocks = quantize_weight(dtype, w)
    del w
    if interleave:
        blocks = interleave_gate_up(blocks, N // 2, gguf_bytes(dtype, 1, K))
    tiled = repack(dtype, blocks, N, K)
    del blocks
    return DeviceWeight.from_tiled(dtype, N, K, tiled)


def seeded_model(cfg: LlamaConfig, seed: int = 0, device=None, interleave_gate_up: bool = True) -> ModelWeights:
    """A random-init model of the given shape: weights N(0, 0.02) quantised on
    the device (attention and gate/up cfg.attn_dtype, down and output
    cfg.down_dtype), norm weights 1 + N(0, 0.02), embeddings N(0, 1).  The
    same seed gives the same model whether or not the gate|up rows are
    interleaved (only their order in HBM differs)."""
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
            wgu=_seeded_quant(cfg.attn_dtype, 2 * F, E, gen, device, interleave=interleave_gate_up),
            wdown=_seeded_quant(cfg.down_dtype, E, F, gen, device)))
    mw.out_norm = norm()
    mw.output = _seeded_quant(cfg.down_dtype, cfg.vocab, E, gen, device)
    mw.gu_interleaved = interleave_gate_up
    return mw


class DecodeModel:
    """One sequence decoded on the device.  ``step()`` enqueues one token's
    forward pass (embed .. argmax) on ``stream``; ``capture()`` records it as
    a CUDA graph that ``generate`` replays."""

    MODES = ("epilogue", "records", "fused", "separate")

    def __init__(self, cfg: LlamaConfig, weights: ModelWeights, device=None, max_record: int = 4096,
                 mode: str = "auto", fused: bool = True, records: bool = True):
        """mode:
          epilogue  every GEMV runs on Q8 records written by the kernel before
                    it (the embedding, the attention, the residual and gate|up
                    GEMVs' epilogues): 5 launches per layer.  Needs Q8
                    activations and interleaved gate|up weights.
          records   every GEMV runs on Q8 records made by a small kernel that
                    applies RMSNorm / SwiGLU (the attention writes its own):
                    8 launches per layer.
          fused     RMSNorm, SwiGLU and the residual adds fused into the GEMVs,
                    activations staged and quantized by every GEMV CTA.
          separate  every operation its own kernel.
          auto      epilogue when the weights allow it, else records (Q8
                    activations) or fused (fp32 activations).
        (fused=False / records=False select separate / fused.)"""
        import torch

        self.cfg, self.w = cfg, weights
        q8 = cfg.act_mode == ACT_Q8
        if mode == "auto":
            mode = ("separate" if not fused else "fused" if not (records and q8)
                    else "epilogue" if weights.gu_interleaved else "records")
        if mode not in self.MODES:
            raise ValueError(f"unknown decode mode {mode!r}")
        if (mode == "epilogue") != weights.gu_interleaved:
            raise ValueError(f"mode {mode!r} needs gate|up weights {'interleaved' if mode == 'epilogue' else 'in [gate | up] order'}"
                             " (seeded_model / load_llama interleave_gate_up)")
        if mode in ("epilogue", "records") and not q8:
            raise ValueError(f"mode {mode!r} runs on Q8 activations (cfg.act_mode = ACT_Q8)")
        self.mode = mode
        self.fused = mode != "separate"
        self.records = mode == "records"
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
        self._q8rec(dw, rec, y, s, accumulate=accumulate)

    def step(self) -> None:
        {"epilogue": self._step_epilogue, "records": self._step_records, "fused": self._step_fused,
         "separate": self._step_unfused}[self.mode]()

    def _q8rec(self, dw: DeviceWeight, rec, y, s, accumulate=False, norm=False, out_rec=None, out_norm=None,
               out_swiglu=False):
        from . import Q8RecOpts

        ssq = _ptr(self.ssq)
        o = Q8RecOpts(1 if accumulate else 0, ssq if accumulate else None, ssq if norm else None, self.ssq_slots,
                      self.cfg.eps, _ptr(out_rec) if out_rec is not None else None,
                      _ptr(out_norm) if out_norm is not None else None, 1 if out_swiglu else 0)
        ws = dw._ws
        check(lib().odi_cuda_matmul_q8rec(dw.dtype, dw.data_ptr, _ptr(rec), _ptr(y), 1, dw.N, dw.K, _ptr(ws),
                                          ws.numel(), FLAG_PDL, ctypes.byref(o), s))

    def _step_epilogue(self) -> None:
        """5 launches per layer, each GEMV on the Q8 records its producer wrote:
        QKV GEMV (records of x * attn_norm, scaled by 1/rms from the slots),
        attention (rope and the KV append fused in; writes the O GEMV's
        records), O GEMV (+= x, slots, records of x * ffn_norm), gate|up GEMV
        (scaled records; writes SwiGLU records), down GEMV (+= x, slots,
        records of x * the next norm's weights)."""
        cfg, L, s = self.cfg, lib(), self.stream.cuda_stream
        E, H, KV, hd = cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim
        st = _ptr(self.state)
        q = _ptr(self.qkv)
        k = q + H * hd * 4
        v = k + KV * hd * 4
        scale = 1.0 / math.sqrt(hd)
        layers = self.w.layers
        check(L.odi_cuda_embed(_ptr(self.w.token_embd), cfg.vocab, E, st, _ptr(self.x), _ptr(self.ssq),
                               _ptr(layers[0].attn_norm), _ptr(self.rec_e), s))
        for li, lw in enumerate(layers):
            nxt = layers[li + 1].attn_norm if li + 1 < len(layers) else self.w.out_norm
            kc, vc = _ptr(self.kc[li]), _ptr(self.vc[li])
            self._q8rec(lw.wqkv, self.rec_e, self.qkv, s, norm=True)
            check(L.odi_cuda_rope_attention(q, k, v, kc, vc, _ptr(self.attn), _ptr(self.rec_a), st, H, KV, hd,
                                            cfg.ctx, cfg.theta, scale, _ptr(self.att_scratch),
                                            self.att_scratch.numel() * 4, s))
            self._q8rec(lw.wo, self.rec_a, self.x, s, accumulate=True, out_rec=self.rec_e, out_norm=lw.ffn_norm)
            self._q8rec(lw.wgu, self.rec_e, self.gu, s, norm=True, out_rec=self.rec_f, out_swiglu=True)
            self._q8rec(lw.wdown, self.rec_f, self.x, s, accumulate=True, out_rec=self.rec_e, out_norm=nxt)
        self._q8rec(self.w.output, self.rec_e, self.logits, s, norm=True)
        check(L.odi_cuda_argmax(_ptr(self.logits), cfg.vocab, st, _ptr(self.record), self.max_record, s))

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
        check(L.odi_cuda_embed(_ptr(self.w.token_embd), cfg.vocab, E, st, _ptr(self.x), _ptr(self.ssq), None, None,
                               s))
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
        check(L.odi_cuda_embed(_ptr(self.w.token_embd), cfg.vocab, cfg.hidden, st, _ptr(self.x), _ptr(self.ssq),
                               None, None, s))
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
        check(L.odi_cuda_embed(_ptr(self.w.token_embd), cfg.vocab, E, st, _ptr(self.x), None, None, None, s))
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
        if self.mode == "epilogue":
            return 1 + 5 * self.cfg.layers + 2  # embed, per layer, output GEMV + argmax
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


class DecoderConfig(ctypes.Structure):
    """odi_cuda_decoder_config (include/odi_cuda.h)."""

    _fields_ = [(n, ctypes.c_int) for n in ("layers", "hidden", "heads", "kv_heads", "head_dim", "ffn", "vocab",
                                             "ctx")] + [("eps", ctypes.c_float), ("theta", ctypes.c_float),
                                                        ("attn_dtype", ctypes.c_int), ("down_dtype", ctypes.c_int)]


class DecoderLayer(ctypes.Structure):
    """odi_cuda_decoder_layer (include/odi_cuda.h)."""

    _fields_ = [(n, ctypes.c_void_p) for n in ("attn_norm", "wqkv", "wo", "ffn_norm", "wgu", "wdown")]


class CDecoder:
    """The decode step driven by the library itself (odi_cuda_decoder_*):
    the same step as DecodeModel's epilogue mode, captured and replayed by
    the C ABI, the way a C++ engine calls it -- one call per batch of tokens,
    no Python per step.  The weights stay ``weights``' device tensors (with
    gate|up interleaved)."""

    def __init__(self, cfg: LlamaConfig, weights: ModelWeights, max_record: int = 4096):
        if not weights.gu_interleaved:
            raise ValueError("the library's decoder needs gate|up interleaved (seeded_model / load_llama default)")
        self.cfg, self.w = cfg, weights
        c = DecoderConfig(cfg.layers, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab, cfg.ctx,
                          cfg.eps, cfg.theta, cfg.attn_dtype, cfg.down_dtype)
        layers = (DecoderLayer * cfg.layers)(*[
            DecoderLayer(_ptr(lw.attn_norm), lw.wqkv.data_ptr, lw.wo.data_ptr, _ptr(lw.ffn_norm), lw.wgu.data_ptr,
                         lw.wdown.data_ptr) for lw in weights.layers])
        h = ctypes.c_void_p()
        check(lib().odi_cuda_decoder_create(ctypes.byref(c), _ptr(weights.token_embd), layers, _ptr(weights.out_norm),
                                            weights.output.data_ptr, max_record, ctypes.byref(h)))
        self.h = h

    def reset(self, token: int, pos: int = 0, clear_cache: bool = False) -> None:
        check(lib().odi_cuda_decoder_reset(self.h, token, pos, 1 if clear_cache else 0))

    def prefill(self, tokens, pos0: int = 0) -> None:
        arr = (ctypes.c_int32 * len(tokens))(*tokens)
        check(lib().odi_cuda_decoder_prefill(self.h, arr, len(tokens), pos0))

    def generate(self, n: int) -> list:
        out = (ctypes.c_int32 * n)()
        check(lib().odi_cuda_decoder_generate(self.h, n, out))
        return list(out)

    def time(self, n: int) -> float:
        """Milliseconds of n greedy steps on the device (CUDA events)."""
        ms = ctypes.c_float()
        check(lib().odi_cuda_decoder_time(self.h, n, ctypes.byref(ms)))
        return ms.value

    def tokens(self, start: int, n: int) -> list:
        out = (ctypes.c_int32 * n)()
        check(lib().odi_cuda_decoder_tokens(self.h, start, n, out))
        return list(out)

    def logits(self):
        import numpy as np

        v = np.zeros(self.cfg.vocab, np.float32)
        check(lib().odi_cuda_decoder_logits(self.h, v.ctypes.data))
        return v

    def launches_per_step(self) -> int:
        return int(lib().odi_cuda_decoder_launches_per_step(self.h))

    def free(self) -> None:
        if getattr(self, "h", None):
            check(lib().odi_cuda_decoder_free(self.h))
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
