"""Incremental Qwen3-Omni code2wav: streams' new codec frames decoded from per-stream slots.

Drop-in for Qwen3OmniIncrementalCodec.decode_slots and CodecStatePool
(sglang_omni/models/qwen3_omni/components/code2wav.py:378-460, incremental_codec.py,
codec_state_pool.py): a stream's frames decoded in any split give the waveform the
whole-sequence Qwen3OmniMoeCode2Wav forward gives on all of them at once.

The network (transformers' Qwen3OmniMoeCode2Wav, whose weights this module reads):
code embeddings averaged over the quantizers -> a pre-transformer of sliding-window
causal attention (window 72) -> two upsampling stages (transposed conv, ConvNeXt block)
-> a causal conv -> four decoder blocks (SnakeBeta, transposed conv, three residual
units of SnakeBeta / dilated causal conv / SnakeBeta / 1x1 conv) -> SnakeBeta -> a
causal conv to one channel, clamped to [-1, 1].

What a slot carries between decodes:
- the pre-transformer's K/V of its last `window - 1` frames, in a ring of `ring_frames`
  rows per slot and layer (position p at row slot * ring_frames + p % ring_frames);
- each causal conv's last (taps - 1) x dilation input samples (its history), exchanged
  in place with the padded input by `history_exchange`;
- each transposed conv's samples past the ones it emitted (stride of them), which the
  next frames' outputs add to, exchanged by `overlap_exchange`; transposed-conv biases
  are added after the overlap so that overlapped samples carry them once.
A stream's first decode reads no state and drops each transposed conv's left pad, as
the whole-sequence forward trims it.

Activations stay channels last ([rows, samples, channels]).  The dilated 7-tap convs of
the decoder's residual units run on the implicit-GEMM tcgen05 kernel (omni_conv1d_gemm: no
window is materialised) with the SnakeBeta that follows them (bias and residual adds
included) in its epilogue, writing straight into the next conv's padded input.  The 1x1
convs, the first conv and the transposed convs' taps run as cuBLAS GEMMs (over a gathered
window where taps > 1), each followed by the separate `fused_bias_snake_beta` kernel: for
those shapes that measured faster (`_implicit`).  The last conv is the clamped
single-output-channel kernel.  The ConvNeXt depthwise conv is a cuDNN call, its pointwise
layers and the pre-transformer's projections cuBLAS GEMMs, and the windowed attention an
SDPA call.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from types import SimpleNamespace

import torch
import torch.nn.functional as F


def default_kernels() -> SimpleNamespace:
    """The library's CUDA kernels (raises when libomni_b200.so is missing)."""
    from omni_b200 import _lib
    from omni_b200.kernels.bias_snake_beta import SnakeBetaCoefficients, fused_bias_snake_beta
    from omni_b200.kernels.codec_state import history_exchange, overlap_exchange
    from omni_b200.kernels.conv_window import conv_window_gather
    from omni_b200.kernels.single_output_conv import clamped_single_output_conv

    _lib.load()
    from omni_b200.ops import conv1d_gemm

    return SimpleNamespace(coefficients=SnakeBetaCoefficients.from_activation, snake=fused_bias_snake_beta,
                           history_exchange=history_exchange, overlap_exchange=overlap_exchange,
                           single_output_conv=clamped_single_output_conv, conv_windows=conv_window_gather,
                           conv_gemm=conv1d_gemm)


@dataclass(frozen=True)
class _CausalConv:
    key: str
    conv: torch.nn.Conv1d
    history: int          # (taps - 1) x dilation samples in front of the new ones


@dataclass(frozen=True)
class _TransConv:
    key: str
    conv: torch.nn.ConvTranspose1d
    stride: int
    overlap: int          # samples past the emitted ones (= the whole forward's right trim)
    left_trim: int


def _causal(module, key: str) -> _CausalConv:
    conv = module.conv
    if conv.stride != (1,):
        raise ValueError("code2wav causal convs are stride one")
    return _CausalConv(key, conv, int(module.padding))


def _trans(module, key: str) -> _TransConv:
    conv = module.conv
    return _TransConv(key, conv, int(conv.stride[0]), int(module.right_pad), int(module.left_pad))


class CodecStateLayout:
    """The code2wav's per-slot state in decode order: causal-conv histories and
    transposed-conv overlaps (zero-length ones kept out of the pool), and the K/V ring
    shape (code2wav.py:378-410, incremental_codec.py:31-57)."""

    def __init__(self, codec) -> None:
        self.upsample = []            # [(transconv, dwconv history, ConvNeXt block)]
        for i, (trans, convnext) in enumerate(codec.upsample):
            self.upsample.append((_trans(trans, f"upsample.{i}.transconv"),
                                  _causal(convnext.dwconv, f"upsample.{i}.convnext.dwconv"), convnext))
        self.decoder_in = _causal(codec.decoder[0], "decoder.0")
        self.blocks = []              # [(snake in front, transconv, [(snake1, conv1, snake2, conv2)])]
        for b, block in enumerate(codec.decoder[1:-2], start=1):
            units = []
            for u, unit in enumerate(block.block[2:]):
                key = f"decoder.{b}.residual.{u}"
                units.append((unit.act1, _causal(unit.conv1, f"{key}.conv1"), unit.act2,
                              _causal(unit.conv2, f"{key}.conv2")))
            self.blocks.append((block.block[0], _trans(block.block[1], f"decoder.{b}.transconv"), units))
        self.final_snake = codec.decoder[-2]
        self.final = _causal(codec.decoder[-1], "decoder.final")
        convs = [c for _, c, _ in self.upsample] + [self.decoder_in]
        for _, _, units in self.blocks:
            for _, c1, _, c2 in units:
                convs += [c1, c2]
        convs.append(self.final)
        self.histories = [(c.key, c.conv.in_channels, c.history) for c in convs]
        self.overlaps = [(t.key, t.conv.out_channels, t.overlap)
                         for t in [t for t, _, _ in self.upsample] + [t for _, t, _ in self.blocks]]
        tr = codec.pre_transformer
        cfg = tr.config
        self.num_layers = len(tr.layers)
        self.num_heads = cfg.num_attention_heads
        self.num_kv_heads = cfg.num_key_value_heads
        self.head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        self.window = int(cfg.sliding_window)
        self.retained = self.window - 1


class CodecStatePool:
    """Per-slot code2wav state where the decode's kernels read and write it: one history
    pool per causal conv, one overlap pool per transposed conv, per-layer K/V rings and
    each slot's next frame position (codec_state_pool.py:64-145)."""

    def __init__(self, layout: CodecStateLayout, *, num_slots: int, ring_frames: int, device, dtype) -> None:
        if ring_frames <= layout.retained:
            raise ValueError("a ring holds the retained window and the new frames")
        self.num_slots = num_slots
        self.ring_frames = ring_frames
        self.retained_frames = layout.retained
        self.free_slots = list(range(num_slots - 1, -1, -1))
        self.histories = {k: torch.zeros(num_slots, n, c, device=device, dtype=dtype)
                          for k, c, n in layout.histories if n}
        self.overlaps = {k: torch.zeros(num_slots, n, c, device=device, dtype=dtype)
                         for k, c, n in layout.overlaps if n}
        width = layout.num_kv_heads * layout.head_dim
        self.keys = [torch.zeros(num_slots * ring_frames, width, device=device, dtype=dtype)
                     for _ in range(layout.num_layers)]
        self.values = [torch.zeros_like(k) for k in self.keys]
        self.frame_positions = torch.zeros(num_slots, device=device, dtype=torch.int64)
        self.bytes_per_slot = dtype.itemsize * (
            sum(p[0].numel() for p in self.histories.values()) + sum(p[0].numel() for p in self.overlaps.values())
            + 2 * layout.num_layers * ring_frames * width)

    def available_size(self) -> int:
        return len(self.free_slots)

    def acquire(self) -> int | None:
        return self.free_slots.pop() if self.free_slots else None

    def release(self, slot: int) -> None:
        self.free_slots.append(slot)

    def zero_slots(self, slots: torch.Tensor) -> None:
        for pool in (*self.histories.values(), *self.overlaps.values()):
            pool.index_fill_(0, slots, 0)
        for ring in (*self.keys, *self.values):
            ring.view(self.num_slots, self.ring_frames, -1).index_fill_(0, slots, 0)
        self.frame_positions.index_fill_(0, slots, 0)


def _rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return weight * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


class Qwen3OmniIncrementalCodec:
    """decode_slots over a CodecStatePool (code2wav.py:378-460)."""

    def __init__(self, codec, kernels: SimpleNamespace | None = None) -> None:
        self.codec = codec
        self.k = kernels if kernels is not None else default_kernels()
        self.layout = CodecStateLayout(codec)
        tr = codec.pre_transformer
        self.eps = float(tr.config.rms_norm_eps)
        self.inv_freq = tr.rotary_emb.inv_freq.float()
        acts = [a for a, _, _ in self.layout.blocks] + [self.layout.final_snake]
        for _, _, units in self.layout.blocks:
            for s1, _, s2, _ in units:
                acts += [s1, s2]
        self.snake = {id(a): self.k.coefficients(a) for a in acts}
        self._weights: dict[int, torch.Tensor] = {}

    def make_pool(self, *, num_slots: int, ring_frames: int, device=None, dtype=None) -> CodecStatePool:
        p = next(self.codec.parameters())
        return CodecStatePool(self.layout, num_slots=num_slots, ring_frames=ring_frames,
                              device=device or p.device, dtype=dtype or p.dtype)

    # -- pre-transformer over the K/V rings ----------------------------------------
    def _transformer(self, x: torch.Tensor, pool: CodecStatePool, slots: torch.Tensor, start: torch.Tensor):
        B, T, _ = x.shape
        L, R = self.layout, pool.ring_frames
        dev = x.device
        qpos = start[:, None] + torch.arange(T, device=dev)                       # [B, T]
        wstart = (start - L.retained).clamp(min=0)
        kpos = wstart[:, None] + torch.arange(R, device=dev)                       # [B, R]
        write_rows = (slots[:, None] * R + qpos % R).reshape(-1)
        window_rows = (slots[:, None] * R + kpos % R).reshape(-1)
        mask = (kpos[:, None, :] <= qpos[:, :, None]) & (kpos[:, None, :] > qpos[:, :, None] - L.window)
        freqs = qpos.float()[..., None] * self.inv_freq.to(dev)
        emb = torch.cat((freqs, freqs), dim=-1)
        cos, sin = emb.cos().to(x.dtype)[:, :, None, :], emb.sin().to(x.dtype)[:, :, None, :]
        H, KV, D = L.num_heads, L.num_kv_heads, L.head_dim
        for i, layer in enumerate(self.codec.pre_transformer.layers):
            att = layer.self_attn
            h = _rms_norm(x, layer.input_layernorm.weight, self.eps)
            q = F.linear(h, att.q_proj.weight, att.q_proj.bias).view(B, T, H, D)
            k = F.linear(h, att.k_proj.weight, att.k_proj.bias).view(B, T, KV, D)
            v = F.linear(h, att.v_proj.weight, att.v_proj.bias).view(B, T, KV, D)
            q = q * cos + _rotate_half(q) * sin
            k = k * cos + _rotate_half(k) * sin
            pool.keys[i].index_copy_(0, write_rows, k.reshape(B * T, KV * D))
            pool.values[i].index_copy_(0, write_rows, v.reshape(B * T, KV * D))
            kw = pool.keys[i].index_select(0, window_rows).view(B, R, KV, D).transpose(1, 2)
            vw = pool.values[i].index_select(0, window_rows).view(B, R, KV, D).transpose(1, 2)
            o = F.scaled_dot_product_attention(q.transpose(1, 2), kw, vw, attn_mask=mask[:, None],
                                               scale=att.scaling, enable_gqa=H != KV)
            o = o.transpose(1, 2).reshape(B, T, H * D)
            x = x + layer.self_attn_layer_scale.scale * F.linear(o, att.o_proj.weight, att.o_proj.bias)
            h = _rms_norm(x, layer.post_attention_layernorm.weight, self.eps)
            mlp = layer.mlp
            g = F.silu(F.linear(h, mlp.gate_proj.weight)) * F.linear(h, mlp.up_proj.weight)
            x = x + layer.mlp_layer_scale.scale * F.linear(g, mlp.down_proj.weight)
        return _rms_norm(x, self.codec.pre_transformer.norm.weight, self.eps)

    # -- conv stack over the histories and overlaps --------------------------------
    def _padded(self, c: _CausalConv, rows: int, length: int, like: torch.Tensor):
        buf = like.new_empty(rows, c.history + length, c.conv.in_channels)
        return buf, buf[:, c.history:]

    def _gemm_weight(self, conv) -> torch.Tensor:
        """A conv's weight as the [taps x C_in, C_out] (causal conv) or [C_in, taps x
        C_out] (transposed conv) matrix of its GEMM form, made once."""
        w = self._weights.get(id(conv))
        if w is None:
            if isinstance(conv, torch.nn.ConvTranspose1d):      # [C_in, C_out, taps]
                w = conv.weight.permute(0, 2, 1).reshape(conv.in_channels, -1).contiguous()
            else:                                               # [C_out, C_in, taps]
                w = conv.weight.permute(2, 1, 0).reshape(-1, conv.out_channels).contiguous()
            self._weights[id(conv)] = w
        return w

    def _conv_weight(self, conv) -> torch.Tensor:
        """A causal conv's weight as the [C_out, taps x C_in] matrix of the implicit GEMM."""
        key = ("implicit", id(conv))
        w = self._weights.get(key)
        if w is None:
            w = conv.weight.permute(0, 2, 1).reshape(conv.out_channels, -1).contiguous()
            self._weights[key] = w
        return w

    @staticmethod
    def _implicit(conv) -> bool:
        """Which convs take the implicit-GEMM kernel: the dilated multi-tap convs of at most
        768 channels, where (with the next SnakeBeta in its epilogue) it measured faster on a
        B200 than the gathered window + cuBLAS GEMM + separate SnakeBeta (64 streams x 10
        frames, per conv: 768 ch 196 vs 224 us, 384 ch 315 vs 384, 192 ch 437 vs 673, 96 ch
        903 vs 993); the 1x1 convs (whose epilogue outweighs their short K loop: 384 ch 273
        vs 123 us), the transposed convs' GEMMs and the first 1024 -> 1536 conv are faster
        on cuBLAS."""
        return (conv.groups == 1 and conv.kernel_size[0] > 1 and conv.in_channels <= 768
                and conv.in_channels % 32 == 0 and conv.out_channels % 32 == 0)

    def _conv(self, c: _CausalConv, padded: torch.Tensor, pool, slots, length: int, cold: bool, snake=None):
        """The causal conv's [rows, length, C_out] outputs without bias, its padded input's
        history exchanged with the slots first.  Ungrouped convs run as the implicit-GEMM
        tcgen05 kernel (conv_gemm: the taps' windows are TMA boxes of the channels-last
        input, nothing is gathered); kernel sets without it (the tests' oracle kernels)
        take one GEMM over the gathered taps-wide window.
        snake = (bias, SnakeBeta coefficients, dest, residual, sum_out): instead of
        returning the conv, write SnakeBeta(conv + bias [+ residual]) to dest (and the sum
        to sum_out) — fused into the conv's epilogue when the kernel is conv_gemm."""
        if c.history:
            self.k.history_exchange(padded, pool.histories[c.key], slots, new_samples=length, is_cold=cold)
        conv = c.conv
        rows, taps = padded.shape[0], conv.kernel_size[0]
        gemm = getattr(self.k, "conv_gemm", None)
        if conv.groups != 1:
            y = F.conv1d(padded.transpose(1, 2), conv.weight, None, 1, 0, conv.dilation, conv.groups)
            y = y.transpose(1, 2).contiguous()
        elif (gemm is not None and self._implicit(conv) and padded.dtype is torch.bfloat16
              and conv.weight.dtype is torch.bfloat16):
            w = self._conv_weight(conv)
            if snake is None:
                y = padded.new_empty(rows, length, conv.out_channels)
                gemm(padded, w, taps=taps, dilation=conv.dilation[0], length=length, out=y)
                return y
            bias, coeff, dest, residual, sum_out = snake
            gemm(padded, w, taps=taps, dilation=conv.dilation[0], length=length, out=dest, bias=bias,
                 alpha_scale=coeff.alpha_scale, inverse_beta=coeff.inverse_beta, residual=residual,
                 sum_out=sum_out)
            return None
        else:
            window = padded if taps == 1 else self.k.conv_windows(padded, length, taps, conv.dilation[0])
            y = (window.reshape(rows * length, -1) @ self._gemm_weight(conv)).view(rows, length, conv.out_channels)
        if snake is None:
            return y
        bias, coeff, dest, residual, sum_out = snake
        self.k.snake(y, bias, coeff, dest, residual=residual, sum_out=sum_out)
        return None

    def _transconv(self, t: _TransConv, frames: torch.Tensor, pool, slots, cold: bool):
        """The transposed conv's emitted samples without bias: the slots' overlap added in
        front, the samples past the emitted ones kept, the left pad dropped on a first decode.
        One GEMM gives every input frame's taps x C_out contributions; with taps = 2 x stride
        frame i writes output blocks i (first stride taps) and i + 1 (the rest); the two
        contributions are added once, in the activations' dtype (torch adds bf16 in fp32
        and rounds once)."""
        rows, n, _ = frames.shape
        conv, s = t.conv, t.stride
        taps, cout = conv.kernel_size[0], conv.out_channels
        z = (frames.reshape(rows * n, -1) @ self._gemm_weight(conv)).view(rows, n, taps, cout)
        if taps == s:
            y = z.reshape(rows, n * s, cout)
        elif taps == 2 * s:
            y = z.new_empty(rows, n + 1, s, cout)
            y[:, :n].copy_(z[:, :, :s])
            y[:, n].zero_()
            y[:, 1:].add_(z[:, :, s:])
            y = y.view(rows, (n + 1) * s, cout)
        else:
            raise ValueError("code2wav transposed convs have taps = stride or 2 x stride")
        emitted = n * s
        if t.overlap:
            self.k.overlap_exchange(y, pool.overlaps[t.key], slots, emitted_samples=emitted, is_cold=cold)
        return y[:, (t.left_trim if cold else 0):emitted]

    def _conv_stack(self, x: torch.Tensor, pool, slots, cold: bool) -> torch.Tensor:
        L, k = self.layout, self.k
        rows = x.shape[0]
        for trans, dw, convnext in L.upsample:
            frames = self._transconv(trans, x, pool, slots, cold)
            n = frames.shape[1]
            padded, body = self._padded(dw, rows, n, frames)
            torch.add(frames, trans.conv.bias, out=body)
            residual = body
            y = self._conv(dw, padded, pool, slots, n, cold) + dw.conv.bias
            y = convnext.norm(y)
            y = convnext.pwconv2(convnext.act(convnext.pwconv1(y)))
            x = residual + convnext.gamma * y
        n = x.shape[1]
        padded, body = self._padded(L.decoder_in, rows, n, x)
        body.copy_(x)
        # the conv whose output feeds the next SnakeBeta: run by that SnakeBeta's caller,
        # so that the two fuse (conv + bias [+ residual] -> SnakeBeta in the conv epilogue)
        pending = (L.decoder_in, padded, n)
        bias = L.decoder_in.conv.bias
        residual = None
        channels = L.decoder_in.conv.out_channels
        for act, trans, units in L.blocks:
            activated = x.new_empty(rows, n, channels)
            pc, ppad, pn = pending
            self._conv(pc, ppad, pool, slots, pn, cold, snake=(bias, self.snake[id(act)], activated, residual, None))
            frames = self._transconv(trans, activated, pool, slots, cold)
            n = frames.shape[1]
            channels = frames.shape[2]
            # unit input = out + bias (+ the previous unit's input): SnakeBeta of it into
            # conv1's padded input, the sum itself kept as the residual (one buffer a block,
            # read and rewritten element by element)
            residual = frames.new_empty(frames.shape)
            s1, c1 = units[0][0], units[0][1]
            padded1, body1 = self._padded(c1, rows, n, frames)
            k.snake(frames, trans.conv.bias, self.snake[id(s1)], body1, residual=None, sum_out=residual)
            for ui, (_, c1, s2, c2) in enumerate(units):
                padded2, body2 = self._padded(c2, rows, n, frames)
                self._conv(c1, padded1, pool, slots, n, cold,
                           snake=(c1.conv.bias, self.snake[id(s2)], body2, None, None))
                if ui + 1 < len(units):
                    s1n, c1n = units[ui + 1][0], units[ui + 1][1]
                    padded1, body1 = self._padded(c1n, rows, n, frames)
                    self._conv(c2, padded2, pool, slots, n, cold,
                               snake=(c2.conv.bias, self.snake[id(s1n)], body1, residual, residual))
                else:
                    pending = (c2, padded2, n)
                    bias = c2.conv.bias
        padded, body = self._padded(L.final, rows, n, x)
        pc, ppad, pn = pending
        self._conv(pc, ppad, pool, slots, pn, cold, snake=(bias, self.snake[id(L.final_snake)], body, residual, None))
        if L.final.history:
            k.history_exchange(padded, pool.histories[L.final.key], slots, new_samples=n, is_cold=cold)
        return k.single_output_conv(padded, L.final.conv, n)

    @torch.no_grad()
    def decode_slots(self, codes: torch.Tensor, pool: CodecStatePool, slot_index: torch.Tensor, *,
                     first_decode: bool) -> torch.Tensor:
        """The [rows, 1, samples] waveform of the [rows, Q, T] codes after the frames the
        rows' slots hold; the slots' state advances in place.  A first decode starts every
        row's stream and reads no slot state."""
        T = codes.shape[-1]
        if T + (0 if first_decode else pool.retained_frames) > pool.ring_frames:
            raise ValueError("a decode's window and new frames must fit the ring")
        slots = slot_index.to(torch.int64)
        start = torch.zeros_like(slots) if first_decode else pool.frame_positions.index_select(0, slots)
        codec = self.codec
        x = codec.code_embedding(codes + codec.code_offset).mean(1)
        x = self._transformer(x, pool, slots, start)
        wav = self._conv_stack(x, pool, slots, first_decode)
        pool.frame_positions.index_copy_(0, slots, start + T)
        return wav

    def samples_per_frame(self) -> int:
        return int(math.prod(self.codec.config.upsample_rates + self.codec.config.upsampling_ratios))
