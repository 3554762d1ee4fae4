"""The B200 talker model runner: one continuous-batching decode step as a single
CUDA graph.

Plugs in where the reference's ModelRunner hook protocol lets a subclass own
the forward (sglang_omni/model_runner/base.py:839-1020):
``custom_decode_forward(forward_batch, schedule_batch, requests)`` returns the
batch result (next_token_ids, logits, hidden) and leaves the frame's codes and
summed embeddings in ``output_codes`` / ``output_embeds`` as the reference's
talkers do (sglang_model.py:1023-1160).

One step on the device, in order:
  1. omni_decode_prepare: seq_lens += 1, page/slot allocation, positions, page
     table and the attention work list (prepare_for_decode + build_forward_batch);
  2. talker forward over the decode rows, input = previous frame's summed codec
     embeddings + the text row (write_feedback_buffers); dense SwiGLU or, with
     cfg.moe, the block-FP8 MoE block per layer;
  3. layer-0 codec draw (repetition penalty, suppression, seeded top-k/top-p);
  4. the code predictor: G - 1 residual codebooks, each fused sample + gather.
The host touches nothing inside the step: it copies the text rows in and the
codes out around the graph replay.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from omni_b200 import ops
from omni_b200.config import SamplingParams, TalkerConfig
from omni_b200.kv_cache import PageAllocator, PagedKVPool, ReqToTokenPool
from omni_b200.predictor import CodePredictor, init_predictor_weights
from omni_b200.staging import OMNI, TTS, CodecControl, TalkerRequest, layer0_top_k_width, stage_decode_buffers, \
    synthetic_requests
from omni_b200.talker import DecodeForwardBatch, DenseTalker, ExtendForwardBatch, init_talker_weights


@dataclass
class GenerationBatchResult:
    """What custom_decode_forward hands back (base.py:879-890, 649-655)."""

    next_token_ids: torch.Tensor   # layer-0 codes [B]
    next_token_logits: torch.Tensor  # fp32 [B, V0]
    hidden_states: torch.Tensor    # [B, H]
    codes: torch.Tensor            # [B, G] all codebooks of the frame
    summed_embeds: torch.Tensor    # [B, H] feedback for the next frame


class TalkerDecodeRunner:
    def __init__(self, cfg: TalkerConfig, *, max_batch: int, num_pages: int, seed: int = 0, device="cuda",
                 pages_per_chunk: int = 32, weights: dict | None = None, predictor_weights: dict | None = None,
                 expert_parallel: bool = False, max_prefill_tokens: int = 0, flavor: str | None = None,
                 codec_control: CodecControl | None = None):
        """max_batch: streams in a step (decode + newly admitted); max_prefill_tokens: extend rows of
        a mixed step (0 = decode only).  flavor: how requests are staged (omni_b200.staging):
        "tts" (Qwen3-TTS seeds and codec-control suppression; the default for the dense
        talker) or "omni" (Qwen3-Omni seeds; the default for the MoE talker)."""
        self.cfg = cfg
        self.flavor = flavor or (TTS if cfg.moe is None else OMNI)
        self.codec_control = codec_control or CodecControl()
        # host mirror of the staged requests of rows [0, len(requests))
        self.requests: list[TalkerRequest] = []
        self.silence_rows = np.zeros(0, dtype=bool)
        self.base_suppress: np.ndarray | None = None
        self.device = torch.device(device)
        self.max_batch = max_batch
        self.pages_per_chunk = pages_per_chunk
        self.w = weights if weights is not None else init_talker_weights(cfg, seed=seed, device=self.device)
        pw = predictor_weights if predictor_weights is not None else init_predictor_weights(
            cfg.predictor, seed=seed + 1, device=self.device)
        self.kv = PagedKVPool(num_layers=cfg.num_hidden_layers, num_pages=num_pages, page_size=cfg.page_size,
                              num_kv_heads=cfg.num_key_value_heads, head_dim=cfg.head_dim, device=self.device)
        self.r2t = ReqToTokenPool(max_reqs=max_batch, max_context=cfg.max_context, device=self.device)
        self.talker = DenseTalker(cfg, self.w, max_batch=max_batch, device=self.device, kv_pool=self.kv,
                                  expert_parallel=expert_parallel, max_rows=max_batch + max_prefill_tokens)
        self.predictor = CodePredictor(cfg.predictor, pw, max_batch=max_batch, device=self.device,
                                       layer0_embedding=self.w["codec_embedding"])
        B = max_batch
        i64 = dict(dtype=torch.long, device=self.device)
        i32 = dict(dtype=torch.int32, device=self.device)
        self.seq_lens = torch.zeros(B, **i64)
        self.req_pool_indices = torch.arange(B, **i64)
        # positions / slots of every row of a step: decode rows first, then extend rows
        R = B + max_prefill_tokens
        self.row_positions = torch.zeros(R, **i64)
        self.row_cache_loc = torch.zeros(R, **i64)
        self.out_cache_loc = self.row_cache_loc[:B]
        self.positions = self.row_positions[:B]
        self.max_prefill_tokens = max_prefill_tokens
        self.extend: ExtendForwardBatch | None = None
        self.page_indptr = torch.zeros(B + 1, **i32)
        self.page_indices = torch.zeros(num_pages + B, **i32)
        self.work_indptr = torch.zeros(B + 1, **i32)
        # attention partial segments: one per (row, CTA page range) piece, at most rows + CTAs
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.work_capacity = max((num_pages + pages_per_chunk - 1) // pages_per_chunk, sms) + B
        self.status = torch.zeros(1, **i32)
        self.text_embeds = torch.zeros(B, cfg.hidden_size, dtype=torch.bfloat16, device=self.device)
        self.allocator: PageAllocator | None = None
        self.batch_size = 0
        self.host_seq_lens: list[int] = []
        self.graph: torch.cuda.CUDAGraph | None = None
        self.talker.ensure_attention_workspace(self.work_capacity)

    # ------------------------------------------------------------------
    # request admission (synthetic prefill: random KV contents)
    # ------------------------------------------------------------------
    def admit(self, context_lens: list[int], *, sampling: SamplingParams = SamplingParams(), seed: int = 0,
              requests: list[TalkerRequest] | None = None, fill_kv: bool = True) -> None:
        """Admit len(context_lens) streams whose first context_lens[i] tokens are in the
        KV pool (pages randomly permuted in the pool), with seeded random KV contents.
        Their sampling state is staged from `requests` (default: seeded synthetic requests
        with `sampling`, omni_b200.staging.synthetic_requests)."""
        cfg = self.cfg
        B = len(context_lens)
        if B > self.max_batch:
            raise RuntimeError("batch exceeds max_batch")
        if requests is not None and len(requests) != B:
            raise ValueError("one request per admitted stream")
        P = cfg.page_size
        rng = np.random.default_rng(seed)
        num_pages = self.kv.num_pages
        perm = torch.from_numpy(rng.permutation(num_pages).astype(np.int32))
        self.allocator = PageAllocator(perm, self.device)
        need = [(L + P - 1) // P for L in context_lens]
        r2t = torch.zeros(B, cfg.max_context, dtype=torch.int32)
        pages = self.allocator.alloc_prefix(sum(need)).cpu()
        off = 0
        for i, (L, n) in enumerate(zip(context_lens, need)):
            if L + 1 > cfg.max_context:
                raise ValueError("context exceeds max_context")
            pg = pages[off: off + n].long()
            off += n
            slots = (pg[:, None] * P + torch.arange(P)[None, :]).reshape(-1)[:L]
            r2t[i, :L] = slots.to(torch.int32)
        self.r2t.req_to_token[:B].copy_(r2t.to(self.device))
        self.seq_lens[:B].copy_(torch.tensor(context_lens, dtype=torch.long))
        self.host_seq_lens = list(context_lens)
        self.batch_size = B
        if fill_kv:
            g = torch.Generator(device=self.device).manual_seed(seed + 7)
            for li in range(cfg.num_hidden_layers):
                self.kv.k_buffer[li].normal_(generator=g)
                self.kv.v_buffer[li].normal_(generator=g)
        self.requests = []
        self.stage(requests if requests is not None else synthetic_requests(B, seed=seed, sampling=sampling))
        self.predictor.output_embeds[:B].zero_()
        self.graph = None

    def stage(self, requests: list[TalkerRequest], *, row0: int = 0) -> None:
        """prepare_decode_buffers for rows row0 .. row0 + len(requests): per-row layer-0
        sampling parameters, seeds, repetition mask (prior output ids), suppress mask
        (request tokens; for the TTS flavor the codec control range and leading silence)
        and the residual sampling rows, per omni_b200.staging."""
        n = len(requests)
        if row0 + n > self.max_batch:
            raise RuntimeError("staged rows exceed max_batch")
        st = self.stage_requests(requests)
        self.write_staging(st, row0=row0)
        # host mirrors: the requests and the rows whose leading-silence ids are still masked
        self.requests = self.requests[:row0] + list(requests)
        V = self.cfg.vocab_size
        base = np.zeros((row0 + n, V), dtype=np.uint8)
        sil = np.zeros(row0 + n, dtype=bool)
        if row0 > 0 and self.base_suppress is not None:
            k = min(row0, self.base_suppress.shape[0])
            base[:k] = self.base_suppress[:k]
            sil[:k] = self.silence_rows[:k]
        base[row0:] = st.base_suppress_mask
        sil[row0:] = st.silence_rows
        self.base_suppress, self.silence_rows = base, sil

    def stage_requests(self, requests: list[TalkerRequest]):
        """The host staging of `requests` under this runner's flavor (omni_b200.staging)."""
        return stage_decode_buffers(requests, flavor=self.flavor, vocab=self.cfg.vocab_size,
                                    predictor_vocab=self.cfg.predictor.vocab_size, control=self.codec_control)

    def write_staging(self, st, *, row0: int = 0) -> None:
        """Copy staged rows (omni_b200.staging.DecodeStaging) into rows row0.. of the
        step's sampling tensors."""
        n = st.seeds.shape[0]
        t = self.talker
        rows = slice(row0, row0 + n)

        def put(dst, arr):
            dst[rows].copy_(torch.from_numpy(np.ascontiguousarray(arr)).to(dst.dtype).view(dst[rows].shape),
                            non_blocking=False)

        put(t.repetition_penalties, st.repetition_penalties)
        put(t.sampling_temperatures, st.temperatures)
        put(t.sampling_top_ps, st.top_ps)
        put(t.sampling_top_ks, st.top_ks)
        put(t.sampling_min_ps, st.min_ps)
        put(t.sampling_seeds, st.seeds)
        put(t.repetition_mask, st.repetition_mask)
        put(t.suppress_mask, st.suppress_mask)
        widths = [int(k) for k in st.top_ks] + ([t.max_top_k] if row0 > 0 else [])
        t.max_top_k = layer0_top_k_width(widths)
        self.predictor.set_sampling(
            temperature=st.sub_temperatures, top_k=st.sub_top_ks, top_p=st.sub_top_ps, seeds=st.sub_seeds,
            do_sample=st.sub_do_sample, batch=n, row0=row0)

    def note_frames(self, layer0_codes: np.ndarray) -> None:
        """Host bookkeeping after a step: append each row's layer-0 code to its request's
        output ids and lift the leading-silence mask of rows that have now emitted
        leading_silence_mask_frames frames (apply_codec_suppress_tokens masks the silence
        ids while fewer frames exist)."""
        lim = self.codec_control.leading_silence_mask_frames
        for i, c in enumerate(np.asarray(layer0_codes).reshape(-1).tolist()[: len(self.requests)]):
            rq = self.requests[i]
            rq.output_ids = list(rq.output_ids or []) + [int(c)]
            if self.silence_rows.size > i and self.silence_rows[i] and rq.frames >= lim:
                self.talker.suppress_mask[i].copy_(torch.from_numpy(self.base_suppress[i]))
                self.silence_rows[i] = False

    # ------------------------------------------------------------------
    def forward_batch(self) -> DecodeForwardBatch:
        B = self.batch_size
        return DecodeForwardBatch(
            batch_size=B, positions=self.positions[:B], seq_lens=self.seq_lens[:B],
            out_cache_loc=self.out_cache_loc[:B], req_pool_indices=self.req_pool_indices[:B],
            page_indptr=self.page_indptr[: B + 1], page_indices=self.page_indices, work_indptr=self.work_indptr[: B + 1],
            work_capacity=self.work_capacity, pages_per_chunk=self.pages_per_chunk)

    def prepare_decode(self) -> DecodeForwardBatch:
        """Device-side prepare_for_decode + ForwardBatch packing."""
        B = self.batch_size
        ops.decode_prepare(seq_lens=self.seq_lens[:B], req_pool_indices=self.req_pool_indices[:B],
                           req_to_token=self.r2t.req_to_token, page_size=self.cfg.page_size,
                           free_pages=self.allocator.free_pages, free_head=self.allocator.free_head,
                           out_cache_loc=self.out_cache_loc[:B], positions=self.positions[:B],
                           page_indptr=self.page_indptr[: B + 1], page_indices=self.page_indices,
                           work_indptr=self.work_indptr[: B + 1], pages_per_chunk=self.pages_per_chunk,
                           status=self.status)
        return self.forward_batch()

    def build_forward_batch(self):
        """Host page bookkeeping and the device packing of the next step (prepare_for_decode
        + build_forward_batch, and prepare_for_extend when new streams are admitted) as the
        ForwardBatch that omni_b200.talker_model.TalkerModel.forward takes."""
        from omni_b200.talker_model import ForwardBatch, ForwardMode

        self._host_reserve()
        fb = self.prepare_decode()
        B = fb.batch_size
        if self.extend is None:
            return ForwardBatch(ForwardMode.DECODE, B, fb.positions, fb)
        ext = self.prepare_extend()
        R = B + ext.tokens
        return ForwardBatch(ForwardMode.MIXED, B, self.row_positions[:R], fb, ext, self.row_positions,
                            self.row_cache_loc, self.select)

    def run_step(self) -> None:
        """The whole decode step on the current stream (capturable); a mixed step when
        extend streams are admitted."""
        fb = self.prepare_decode()
        if self.extend is not None:
            self.custom_mixed_forward(fb)
        else:
            self.custom_decode_forward(fb, None, None)

    def custom_decode_forward(self, forward_batch: DecodeForwardBatch, schedule_batch, requests):
        """The hook that owns the decode forward (base.py:879-890)."""
        B = forward_batch.batch_size
        # the previous frame's summed codec embeddings are this frame's feedback input
        feedback = self.predictor.output_embeds[:B]
        logits = self.talker.forward(feedback, self.text_embeds[:B], forward_batch)
        c0 = self.talker.sample_decode_tokens(logits, forward_batch)
        t = self.talker
        codes, summed = self.predictor.code_predictor_forward(
            c0, t.h[:B], forward_batch.positions, final_norm=t.w["norm"], final_ss=t.ss, final_eps=self.cfg.rms_norm_eps,
            hidden_out=t.hidden[:B])
        return GenerationBatchResult(next_token_ids=c0, next_token_logits=logits, hidden_states=self.talker.hidden[:B],
                                     codes=codes[:, :, 0], summed_embeds=summed[:, 0])

    # ------------------------------------------------------------------
    # mixed step: new streams prefilled in the same forward as the decode rows
    # ------------------------------------------------------------------
    def admit_prefill(self, prompt_lens: list[int], *, seed: int = 0,
                      sampling: SamplingParams = SamplingParams(),
                      requests: list[TalkerRequest] | None = None) -> None:
        """Admit len(prompt_lens) new streams (rows after the decode streams) whose prompts
        (seeded N(0, 1) embeddings, the rows compose_prefill_embeds would produce) are
        prefilled by every following step's fused forward, their slots reserved in
        req_to_token (prepare_for_extend).  Each step then samples the layer-0 token of each
        new stream from its last prompt row and runs the predictor for it."""
        cfg, P = self.cfg, self.cfg.page_size
        Bd, n = self.batch_size, len(prompt_lens)
        if Bd + n > self.max_batch:
            raise RuntimeError("decode + new streams exceed max_batch")
        T = int(sum(prompt_lens))
        if T > self.max_prefill_tokens:
            raise RuntimeError("prompts exceed max_prefill_tokens")
        if max(prompt_lens) >= cfg.max_context:
            raise ValueError("prompt exceeds max_context")
        dev = self.device
        i64 = dict(dtype=torch.long, device=dev)
        i32 = dict(dtype=torch.int32, device=dev)
        need = [(L + P - 1) // P for L in prompt_lens]
        pages = self.allocator.alloc_prefix(sum(need)).cpu()
        r2t = torch.zeros(n, cfg.max_context, dtype=torch.int32)
        off = 0
        for i, (L, k) in enumerate(zip(prompt_lens, need)):
            pg = pages[off: off + k].long()
            off += k
            r2t[i, :L] = (pg[:, None] * P + torch.arange(P)[None, :]).reshape(-1)[:L].to(torch.int32)
        self.r2t.req_to_token[Bd: Bd + n].copy_(r2t.to(dev))
        self.ext_req = torch.arange(Bd, Bd + n, **i64)
        self.ext_prefix = torch.zeros(n, **i64)
        self.ext_lens = torch.tensor(prompt_lens, **i64)
        self.ext_seq_lens = torch.zeros(n, **i64)
        self.ext_qo = torch.zeros(n + 1, **i32)
        self.ext_page_indptr = torch.zeros(n + 1, **i32)
        self.ext_page_indices = torch.zeros(sum(need) + 1, **i32)
        self.ext_tiles = torch.zeros(n + 1, **i32)
        max_tiles = sum((L + ops.PREFILL_Q_TILE - 1) // ops.PREFILL_Q_TILE for L in prompt_lens)
        g = torch.Generator(device=dev).manual_seed(seed + 13)
        self.prompt_embeds = torch.randn(T, cfg.hidden_size, generator=g, device=dev).to(torch.bfloat16)
        last = np.cumsum(prompt_lens) - 1
        self.select = torch.tensor(list(range(Bd)) + [Bd + int(x) for x in last], **i64)
        self.extend = ExtendForwardBatch(streams=n, tokens=T, qo_indptr=self.ext_qo, seq_lens=self.ext_seq_lens,
                                         page_indptr=self.ext_page_indptr, page_indices=self.ext_page_indices,
                                         tile_indptr=self.ext_tiles, max_tiles=max_tiles)
        self.sel_positions = torch.zeros(Bd + n, **i64)
        # per-stream sampling state of the new rows
        self.stage(requests if requests is not None else
                   synthetic_requests(n, seed=seed, sampling=sampling, prefix="new"), row0=Bd)
        self.graph = None

    def prepare_extend(self) -> ExtendForwardBatch:
        """Device-side prepare_for_extend packing of the admitted new streams."""
        Bd = self.batch_size
        T = self.extend.tokens
        ops.extend_prepare(prefix_lens=self.ext_prefix, extend_lens=self.ext_lens, req_pool_indices=self.ext_req,
                           req_to_token=self.r2t.req_to_token, page_size=self.cfg.page_size,
                           seq_lens=self.ext_seq_lens, qo_indptr=self.ext_qo,
                           out_cache_loc=self.row_cache_loc[Bd: Bd + T], positions=self.row_positions[Bd: Bd + T],
                           page_indptr=self.ext_page_indptr, page_indices=self.ext_page_indices,
                           tile_indptr=self.ext_tiles, status=self.status)
        return self.extend

    def custom_mixed_forward(self, fb: DecodeForwardBatch):
        """custom_prefill_forward for a mixed batch (model_runner/base.py:866-877): decode rows and
        the new streams' prompts in one forward, then the layer-0 draw and the code predictor for
        every stream of the step (the decode rows and each new stream's first frame)."""
        ext = self.prepare_extend()
        Bd, n = fb.batch_size, self.select.shape[0]
        t = self.talker
        feedback = self.predictor.output_embeds[:Bd]
        logits = t.forward_mixed(feedback, self.text_embeds[:Bd], fb, self.prompt_embeds, ext, self.row_positions,
                                 self.row_cache_loc, self.select)
        torch.index_select(self.row_positions, 0, self.select, out=self.sel_positions)
        sel_fb = DecodeForwardBatch(batch_size=n, positions=self.sel_positions, seq_lens=fb.seq_lens,
                                    out_cache_loc=fb.out_cache_loc, req_pool_indices=fb.req_pool_indices,
                                    page_indptr=fb.page_indptr, page_indices=fb.page_indices,
                                    work_indptr=fb.work_indptr, work_capacity=fb.work_capacity,
                                    pages_per_chunk=fb.pages_per_chunk)
        c0 = t.sample_decode_tokens(logits, sel_fb)
        codes, summed = self.predictor.code_predictor_forward(
            c0, t.h_sel[:n], self.sel_positions, final_norm=t.w["norm"], final_ss=t.ss_sel,
            final_eps=self.cfg.rms_norm_eps, hidden_out=t.hidden[:n])
        return GenerationBatchResult(next_token_ids=c0, next_token_logits=logits, hidden_states=t.hidden[:n],
                                     codes=codes[:, :, 0], summed_embeds=summed[:, 0])

    # ------------------------------------------------------------------
    def _host_reserve(self) -> None:
        self.allocator.reserve_host(self.host_seq_lens, self.cfg.page_size)
        self.host_seq_lens = [L + 1 for L in self.host_seq_lens]
        if max(self.host_seq_lens) >= self.cfg.max_context:
            raise RuntimeError("a stream reached max_context")

    def step(self, use_graph: bool = True) -> None:
        """One decode step on device-resident inputs (text rows already in text_embeds)."""
        self._host_reserve()
        if use_graph:
            if self.graph is None:
                raise RuntimeError("capture() first")
            self.graph.replay()
        else:
            self.run_step()

    def capture(self, warmup: int = 1) -> None:
        """Warm up eagerly (consuming `warmup` steps) and capture one step as a CUDA graph."""
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self._host_reserve()
                self.run_step()
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        # recording executes nothing: the device state is unchanged by capture
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self.run_step()
        torch.cuda.synchronize(self.device)
        self.graph = g

    # ------------------------------------------------------------------
    # public end-to-end API: host text rows in, host codes out
    # ------------------------------------------------------------------
    def decode(self, text_embeds_host: torch.Tensor, codes_host: torch.Tensor | None = None) -> torch.Tensor:
        """One frame for every live stream: copy the text rows in (pinned host -> HBM),
        replay the step graph, copy the frame's codes out.  Returns codes [B, G] on the host
        (in a mixed step also the new streams' first frames, after the decode rows)."""
        B = self.batch_size
        n = B + (self.extend.streams if self.extend is not None else 0)  # + the new streams' first frames
        self.text_embeds[:B].copy_(text_embeds_host, non_blocking=True)
        self.step(use_graph=self.graph is not None)
        if codes_host is None:
            codes_host = torch.empty((n, self.cfg.predictor.num_code_groups), dtype=torch.long, pin_memory=True)
        codes_host.copy_(self.predictor.output_codes[:n], non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        if self.silence_rows.any():
            self.note_frames(codes_host[:, 0].numpy())
        return codes_host
