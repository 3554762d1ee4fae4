"""Per-request staging of the decode step's sampling state (prepare_decode_buffers).

The reference builds each row's layer-0 and residual sampling state on the host
from the request objects and copies it into fixed device buffers before a decode
step; this module is that host logic, for both talkers of the reference:

- Qwen3-Omni (``Qwen3OmniTalker.prepare_decode_buffers``,
  sglang_omni/models/qwen3_omni/components/talker.py:1065-1215): the row's
  repetition penalty, temperature, top-p, top-k, min-p and seed; the repetition
  mask = the unique prior output ids inside the vocabulary, only for rows whose
  penalty is not 1; the suppress mask = the request's suppress tokens (the data's
  own list when non-empty, else the request's codec suppress list) inside the
  vocabulary; the seed = the request's sampling seed masked to a positive int32,
  or for an unseeded row ``derive_sampling_seed("sglang-omni-unseeded-row", rid)``.
- Qwen3-TTS: seeds from the public request seed,
  ``derive_sampling_seed("qwen3-tts", seed & 0x7FFFFFFF, "semantic" | "subtalker")``
  (qwen3_tts/request_builders.py:94-124, 1778-1788; fresh random seeds for an
  unseeded request); the codec control suppression of
  ``Qwen3TTSModelRunner.apply_codec_suppress_tokens`` (qwen3_tts/model_runner.py:155-198):
  the last 1024 ids of the configured vocabulary except the codec EOS, plus the
  silence ids for a cold-start clone (mask_leading_silence) while it has emitted
  fewer than ``leading_silence_mask_frames`` frames; and the subtalker rows of
  ``Qwen3TTSTalker.prepare_decode_buffers`` (sglang_model.py:1162-1270): a greedy
  row is staged as temperature 1, top-p 1, top-k 1; a sampled row's temperature
  is clamped to at least 1e-5; the batch signature (ladder width, top-p flag) comes
  from the sampled rows only.

Everything here returns numpy arrays; the runners copy them into their device
tensors (one host-to-device copy per admission, none per step).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Sequence

import numpy as np

from omni_b200.config import SamplingParams
from omni_b200.seed import SAMPLING_SEED_MASK, derive_sampling_seed, new_random_sampling_seed, resolve_row_seed

OMNI = "omni"
TTS = "tts"

# the residual sampler's top-k ladder (sampling_kernels.py:792-800)
TOP_K_LADDER = (4, 8, 16, 32, 50, 64, 128, 256, 512, 1024)


def unseeded_row_seed(request_id: str | None, row: int) -> int:
    """Rank-shared seed of an unseeded row in a seeded batch (model_runner/base.py:86-88)."""
    return derive_sampling_seed("sglang-omni-unseeded-row", request_id or f"row-{row}")


def omni_row_seed(sampling_seed: int | None, rid: str) -> int:
    """The Qwen3-Omni talker's layer-0 seed of a row (talker.py:1106-1114)."""
    if sampling_seed is None:
        return derive_sampling_seed("sglang-omni-unseeded-row", rid)
    if not 0 <= int(sampling_seed) <= SAMPLING_SEED_MASK:
        return resolve_row_seed(int(sampling_seed))
    return int(sampling_seed)


def normalize_qwen3_tts_seed(seed: object) -> int:
    """An integral request seed masked to a positive int32 (request_builders.py:94-110)."""
    if isinstance(seed, bool):
        raise ValueError("Qwen3-TTS seed must be an integer")
    if isinstance(seed, float) and not seed.is_integer():
        raise ValueError("Qwen3-TTS seed must be an integer")
    try:
        value = int(seed)
    except (TypeError, ValueError) as exc:
        raise ValueError("Qwen3-TTS seed must be an integer") from exc
    return value & SAMPLING_SEED_MASK


def qwen3_tts_sampling_seeds(seed: object | None) -> tuple[int, int]:
    """(semantic, subtalker) seeds of a Qwen3-TTS request; fresh random ones when unseeded."""
    if seed is None:
        return new_random_sampling_seed(), new_random_sampling_seed()
    s = normalize_qwen3_tts_seed(seed)
    return derive_sampling_seed("qwen3-tts", s, "semantic"), derive_sampling_seed("qwen3-tts", s, "subtalker")


@dataclass(frozen=True)
class CodecControl:
    """Qwen3-TTS codec-control suppression (apply_codec_suppress_tokens)."""

    codec_eos_token_id: int = 2150
    leading_silence_mask_frames: int = 2
    silence_codec_ids: tuple[int, ...] = ()
    control_ids: int = 1024  # the last ids of the configured vocabulary


@dataclass
class TalkerRequest:
    """The request state that staging reads (the fields of the reference's request
    objects that prepare_decode_buffers and the codec suppression look at)."""

    rid: str
    seed: int | None = None
    sampling: SamplingParams = field(default_factory=SamplingParams)
    output_ids: Sequence[int] | None = None     # layer-0 codes emitted so far
    suppress_tokens: Sequence[int] | None = None  # the data's own list
    codec_suppress_tokens: Sequence[int] | None = None  # the request's codec list
    mask_leading_silence: bool = False
    # Qwen3-TTS seeds, derived once per request (fresh random when unseeded)
    semantic_seed: int | None = None
    subtalker_seed: int | None = None

    def tts_seeds(self) -> tuple[int, int]:
        if self.semantic_seed is None or self.subtalker_seed is None:
            self.semantic_seed, self.subtalker_seed = qwen3_tts_sampling_seeds(self.seed)
        return self.semantic_seed, self.subtalker_seed

    @property
    def frames(self) -> int:
        return len(self.output_ids) if self.output_ids else 0


@dataclass
class DecodeStaging:
    """Host arrays of one batch's staged rows."""

    repetition_penalties: np.ndarray  # f32 [B]
    temperatures: np.ndarray          # f32 [B]
    top_ps: np.ndarray                # f32 [B]
    top_ks: np.ndarray                # i64 [B]
    min_ps: np.ndarray                # f32 [B]
    seeds: np.ndarray                 # i64 [B] layer-0 seeds
    repetition_mask: np.ndarray       # u8 [B, V0]
    suppress_mask: np.ndarray         # u8 [B, V0] (with the leading-silence ids)
    base_suppress_mask: np.ndarray    # u8 [B, V0] (without them)
    sub_temperatures: np.ndarray      # f32 [B]
    sub_top_ps: np.ndarray            # f32 [B]
    sub_top_ks: np.ndarray            # i64 [B]
    sub_seeds: np.ndarray             # i64 [B]
    sub_do_sample: np.ndarray         # u8 [B]
    silence_rows: np.ndarray          # bool [B]: rows whose silence ids are still masked
    signature: dict                   # predictor batch signature (sampled rows only)


def predictor_signature(sampled_top_ks: Sequence[int], sampled_top_ps: Sequence[float], vocab: int) -> dict:
    """The residual sampler's batch signature (predictor_signature_terms,
    sglang_model.py:154-187): the smallest ladder width covering the largest bounded
    top-k, whether any sampled row uses top-p, whether a top-k is unbounded."""
    bounded = [int(k) for k in sampled_top_ks if 0 < int(k) < vocab]
    has_top_p = any(0.0 < float(p) < 1.0 for p in sampled_top_ps)
    unbounded = len(bounded) != len(sampled_top_ks)
    max_top_k = 0
    widest = max(bounded, default=0)
    if widest > 0 and not unbounded:
        step = next((w for w in TOP_K_LADDER if w >= widest), None)
        if step is None or step >= vocab:
            unbounded = True
        else:
            max_top_k = step
    return {"max_top_k": max_top_k, "has_top_p": has_top_p, "has_unbounded_top_k": unbounded}


def codec_control_mask(vocab: int, control: CodecControl) -> np.ndarray:
    """u8 [vocab]: the control range [vocab - control_ids, vocab) but the codec EOS."""
    m = np.zeros(vocab, dtype=np.uint8)
    lo = max(0, vocab - control.control_ids)
    m[lo:vocab] = 1
    if lo <= control.codec_eos_token_id < vocab:
        m[control.codec_eos_token_id] = 0
    return m


def stage_decode_buffers(requests: Sequence[TalkerRequest], *, flavor: str, vocab: int, predictor_vocab: int,
                         control: CodecControl | None = None) -> DecodeStaging:
    """Stage rows 0..len(requests)-1 of a decode batch.

    flavor OMNI: layer-0 seeds per omni_row_seed, suppress = the per-request tokens.
    flavor TTS: layer-0 (semantic) and subtalker seeds per qwen3_tts_sampling_seeds,
    suppress = the per-request tokens, the codec control range and, for cold-start
    clones, the silence ids.  Both flavors build the repetition mask from the prior
    output ids of rows whose penalty is not 1."""
    if flavor not in (OMNI, TTS):
        raise ValueError(f"unknown talker flavor {flavor!r}")
    control = control or CodecControl()
    B = len(requests)
    f32 = dict(dtype=np.float32)
    st = DecodeStaging(
        repetition_penalties=np.ones(B, **f32), temperatures=np.ones(B, **f32), top_ps=np.ones(B, **f32),
        top_ks=np.ones(B, dtype=np.int64), min_ps=np.zeros(B, **f32), seeds=np.zeros(B, dtype=np.int64),
        repetition_mask=np.zeros((B, vocab), dtype=np.uint8), suppress_mask=np.zeros((B, vocab), dtype=np.uint8),
        base_suppress_mask=np.zeros((B, vocab), dtype=np.uint8), sub_temperatures=np.ones(B, **f32),
        sub_top_ps=np.ones(B, **f32), sub_top_ks=np.ones(B, dtype=np.int64), sub_seeds=np.zeros(B, dtype=np.int64),
        sub_do_sample=np.zeros(B, dtype=np.uint8), silence_rows=np.zeros(B, dtype=bool), signature={})
    ctl = codec_control_mask(vocab, control) if flavor == TTS else None
    silence = np.array([t for t in control.silence_codec_ids if 0 <= t < vocab], dtype=np.int64)
    sampled: list[int] = []
    for i, rq in enumerate(requests):
        sp = rq.sampling
        st.repetition_penalties[i] = sp.repetition_penalty
        st.temperatures[i] = sp.temperature
        st.top_ps[i] = sp.top_p
        st.top_ks[i] = sp.top_k
        st.min_ps[i] = sp.min_p
        if flavor == OMNI:
            st.seeds[i] = omni_row_seed(rq.seed, rq.rid)
            sub_seed = derive_sampling_seed("subtalker", int(st.seeds[i]))
        else:
            st.seeds[i], sub_seed = rq.tts_seeds()
        if float(sp.repetition_penalty) != 1.0 and rq.output_ids:
            ids = np.unique(np.asarray([int(t) for t in rq.output_ids], dtype=np.int64))
            ids = ids[(ids >= 0) & (ids < vocab)]
            st.repetition_mask[i, ids] = 1
        sup = rq.suppress_tokens or rq.codec_suppress_tokens
        if sup:
            ids = np.asarray([int(t) for t in sup], dtype=np.int64)
            st.base_suppress_mask[i, ids[(ids >= 0) & (ids < vocab)]] = 1
        if ctl is not None:
            st.base_suppress_mask[i] |= ctl
        st.suppress_mask[i] = st.base_suppress_mask[i]
        if (flavor == TTS and rq.mask_leading_silence and control.leading_silence_mask_frames > 0
                and rq.frames < control.leading_silence_mask_frames and silence.size):
            st.suppress_mask[i, silence] = 1
            st.silence_rows[i] = True
        # residual (subtalker) rows
        ds = bool(sp.subtalker_dosample)
        st.sub_do_sample[i] = ds
        st.sub_temperatures[i] = max(float(sp.subtalker_temperature), 1e-5) if ds else 1.0
        st.sub_top_ps[i] = sp.subtalker_top_p if ds else 1.0
        st.sub_top_ks[i] = sp.subtalker_top_k if ds else 1
        st.sub_seeds[i] = sub_seed
        if ds:
            sampled.append(i)
    st.signature = predictor_signature([int(st.sub_top_ks[i]) for i in sampled],
                                       [float(st.sub_top_ps[i]) for i in sampled], predictor_vocab)
    st.signature["has_sampled_rows"] = bool(sampled)
    st.signature["has_argmax_rows"] = len(sampled) < B
    return st


def layer0_top_k_width(top_ks: Sequence[int]) -> int:
    """The layer-0 sampler's ladder width for a batch of top-k values."""
    widest = max((int(k) for k in top_ks), default=4)
    for w in TOP_K_LADDER:
        if w >= widest:
            return w
    return TOP_K_LADDER[-1]


def synthetic_requests(n: int, *, seed: int, sampling: SamplingParams = SamplingParams(), prefix: str = "req",
                       first: int = 0) -> list[TalkerRequest]:
    """Seeded benchmark requests: request i has id f"{prefix}{first + i}" and public seed
    seed * 1_000_003 + first + i (no prior output, no suppress list)."""
    return [TalkerRequest(rid=f"{prefix}{first + i}", seed=seed * 1_000_003 + first + i, sampling=sampling)
            for i in range(n)]
