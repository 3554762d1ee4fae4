"""The talker model object with the reference's call signatures.

The reference's ModelRunner calls its talker model object through
``forward(input_ids, positions, forward_batch, input_embeds=None,
input_embeds_are_projected=False, omni_prefill_rids=None) -> LogitsProcessorOutput``
(Qwen3OmniTalker.forward, sglang_omni/models/qwen3_omni/components/talker.py:1259-1340;
Qwen3TTSTalker.forward, sglang_omni/models/qwen3_tts/sglang_model.py:1273-1302) and
``code_predictor_forward(layer0_codes, talker_hidden, semantic_positions=None)``
(sglang_model.py:1317-1346; talker.py:1907-1918).  ``TalkerModel`` gives the B200
runner's components (omni_b200.talker.DenseTalker, omni_b200.predictor.CodePredictor)
exactly that surface:

- decode: the rows' input embeddings (``input_embeds`` [B, H], or the codec embedding
  of ``input_ids``) through the talker layers over the paged KV cache, the final
  RMSNorm, the codec head in fp32; returns next_token_logits [B, V0] fp32 and
  hidden_states [B, H] bf16 (normalized).  With the Qwen3-Omni flavor the decode forward
  also draws the layer-0 codes and runs code_predictor_forward, as the reference's Omni
  talker does (its output lands in output_codes / output_embeds);
- extend / mixed: decode rows first, then every new stream's prompt rows
  (``input_embeds`` covers both), written into the paged pool; the logits of the decode
  rows and of each stream's last prompt row (manual_extend_logits, talker.py:1344-1360);
- code_predictor_forward: the residual codebooks of one frame from the normalized talker
  hidden states.

The runner's fused decode step (TalkerDecodeRunner.custom_decode_forward) skips the
separate final-norm launch by folding the norm into the predictor's first kernel; this
object keeps the reference's boundary, where the hidden state handed over is already
normalized.
"""

from __future__ import annotations

import enum
from dataclasses import dataclass

import torch

from omni_b200 import ops
from omni_b200.staging import OMNI, TalkerRequest
from omni_b200.talker import DecodeForwardBatch, ExtendForwardBatch


class ForwardMode(enum.IntEnum):
    DECODE = 1
    EXTEND = 2
    MIXED = 3

    def is_decode(self) -> bool:
        return self is ForwardMode.DECODE

    def is_extend(self) -> bool:
        return self is not ForwardMode.DECODE


@dataclass
class ForwardBatch:
    """The device-side batch description of one forward (sglang's ForwardBatch fields that
    this path reads): the decode part (packed by omni_decode_prepare) and, in an extend or
    mixed batch, the extend part (packed by omni_extend_prepare) with every row's position
    and KV slot and the rows whose logits are returned."""

    forward_mode: ForwardMode
    batch_size: int                       # decode rows
    positions: torch.Tensor               # i64 [rows]
    decode: DecodeForwardBatch
    extend: ExtendForwardBatch | None = None
    row_positions: torch.Tensor | None = None   # i64 [decode rows + extend rows]
    row_cache_loc: torch.Tensor | None = None   # i64 [decode rows + extend rows]
    select: torch.Tensor | None = None          # i64 [decode rows + streams]: rows that produce logits


@dataclass
class LogitsProcessorOutput:
    next_token_logits: torch.Tensor
    hidden_states: torch.Tensor


class TalkerModel:
    """Reference-shaped talker model object over a TalkerDecodeRunner's components."""

    def __init__(self, runner):
        self.runner = runner
        self.cfg = runner.cfg
        self.talker = runner.talker
        self.predictor = runner.predictor
        B = runner.max_batch
        H = self.cfg.hidden_size
        self.input_rows = torch.zeros(B, H, dtype=torch.bfloat16, device=runner.device)
        # the reference talker's persistent output buffers
        self.output_codes = self.predictor.output_codes
        self.output_embeds = self.predictor.output_embeds
        self.sampled_token_ids = self.talker.sampled_token_ids

    # ------------------------------------------------------------------
    def prepare_decode_buffers(self, requests: list[TalkerRequest]) -> None:
        """Stage the batch's per-row sampling state (omni_b200.staging)."""
        self.runner.stage(requests)

    def forward(self, input_ids: torch.Tensor | None, positions: torch.Tensor, forward_batch: ForwardBatch,
                input_embeds: torch.Tensor | None = None, input_embeds_are_projected: bool = False,
                omni_prefill_rids=None) -> LogitsProcessorOutput:
        del positions, input_embeds_are_projected, omni_prefill_rids  # positions come with the batch
        fb = forward_batch
        t, cfg = self.talker, self.cfg
        B = fb.batch_size
        H = cfg.hidden_size
        if fb.forward_mode.is_decode():
            if input_embeds is None:
                if input_ids is None:
                    raise ValueError("decode needs input_ids or input_embeds")
                rows = self.input_rows[:B]
                torch.index_select(t.w["codec_embedding"], 0, input_ids.reshape(-1), out=rows)
            else:
                rows = input_embeds.reshape(-1, H)
                if rows.shape[0] != B:
                    raise ValueError("input_embeds rows differ from the batch size")
            logits = t.forward(rows, None, fb.decode)
            hidden = t.hidden[:B]
            ops.rmsnorm(t.h[:B], t.w["norm"], cfg.rms_norm_eps, out=hidden)
            if self.runner.flavor == OMNI:
                c0 = t.sample_decode_tokens(logits, fb.decode)
                self.code_predictor_forward(c0.unsqueeze(1), hidden.unsqueeze(1), fb.decode.positions)
            return LogitsProcessorOutput(next_token_logits=logits, hidden_states=hidden)
        if fb.extend is None or input_embeds is None or fb.select is None:
            raise ValueError("an extend batch needs its extend part, input_embeds and the selected rows")
        ext = fb.extend
        rows = input_embeds.reshape(-1, H)
        if rows.shape[0] != B + ext.tokens:
            raise ValueError("input_embeds must hold the decode rows then the prompt rows")
        logits = t.forward_mixed(rows[:B], None, fb.decode, rows[B:], ext, fb.row_positions, fb.row_cache_loc,
                                 fb.select)
        n = fb.select.shape[0]
        hidden = t.hidden[:n]
        ops.rmsnorm(t.h_sel[:n], t.w["norm"], cfg.rms_norm_eps, out=hidden)
        return LogitsProcessorOutput(next_token_logits=logits, hidden_states=hidden)

    def sample_decode_tokens(self, logits: torch.Tensor, forward_batch: ForwardBatch) -> torch.Tensor:
        """Repetition penalty, suppression and the seeded layer-0 draw (talker.py:1376-1412)."""
        return self.talker.sample_decode_tokens(logits, forward_batch.decode)

    def code_predictor_forward(self, layer0_codes: torch.Tensor, talker_hidden: torch.Tensor,
                               semantic_positions: torch.Tensor | None = None):
        """(layer0_codes [B, 1] i64, talker_hidden [B, 1, H] bf16 normalized, semantic_positions
        [B] or None) -> (codes [B, G, 1] i64, summed [B, 1, H] bf16)."""
        return self.predictor.code_predictor_forward(layer0_codes, talker_hidden, semantic_positions)
