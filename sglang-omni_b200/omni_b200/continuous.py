"""Continuous batching of talker streams on one GPU: the talker stage's event
loop (sglang_omni/scheduling/omni_scheduler.py:3616-3653) over the B200 decode
step.

Each iteration asks the C++ scheduler (omni_b200.scheduler) for a plan, then
  1. applies the plan's row moves to every per-row state tensor in one launch
     (omni_move_rows: sampling parameters and seeds, repetition / suppress masks,
     the predictor's summed-embedding feedback, seq_lens, req_pool_indices), so
     the live streams stay rows [0, B);
  2. DECODE: stages the pages the decode rows open (the step's
     omni_decode_prepare takes them in row order), pads the batch to the decode
     graph bucket (generation_batch_policy.py:57-74; padding rows attend to two
     tokens of the reserved page 0 under a reserved request slot and are never
     read back), copies the text rows in and replays that bucket's CUDA graph
     (recorded the first time the bucket runs; the first run is eager);
     MIXED: writes the admitted streams' req_to_token rows, seq_len and slot
     (omni_admit_streams) and their sampling state, copies their prompt rows
     in, and runs the fused decode + prefill forward eagerly
     (custom_mixed_forward): the decode rows take a frame and every admitted
     stream its first frame;
  3. copies the step's codes out and hands the frames to process_batch_result,
     which finishes streams (max_frames or the codec EOS), frees their pages and,
     with emit_messages, queues the frames for the vocoder stage in the talker's
     coalesced chunks (pop_messages).
Streams are independent rows: for one bucket size a stream's results do not
depend on its row or on the other rows, which the GPU tests check by moving
streams between rows.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from omni_b200 import ops
from omni_b200.config import SamplingParams
from omni_b200.kv_cache import PageAllocator
from omni_b200.model_runner import TalkerDecodeRunner
from omni_b200.scheduler import DECODE, MIXED, OmniScheduler, StepPlan
from omni_b200.staging import TalkerRequest
from omni_b200.talker import ExtendForwardBatch


def decode_graph_buckets(max_bs: int) -> list[int]:
    """The decode CUDA-graph batch ladder (build_default_cuda_graph_bs,
    sglang_omni/scheduling/generation_batch_policy.py:57-74)."""
    values = [1, 2, 4, 8, 12] + list(range(16, 257, 8)) + list(range(272, 512, 16)) + list(
        range(512, max_bs + 1, 32))
    values = [b for b in values if b <= max_bs]
    if not values or values[-1] != max_bs:
        values.append(max_bs)
    return values


def poisson_arrival_trace(total: int, world: int, steady_per_gpu: int, frames_range: tuple[int, int],
                          seed: int = 4242):
    """The config-4 stream set (synthetic, seeded): `total` streams with config-1/3
    contexts as prompts (lognormal(6, 0.8) clipped to [16, 8192]), frame counts
    U[frames_range], and
    Poisson arrivals in step time at the rate that keeps `steady_per_gpu` streams live
    per GPU (Little's law: rate = world x steady / mean frames).  Returns
    [(rid, arrival_step, prompt_len, frames)]."""
    rng = np.random.default_rng(seed)
    prompts = np.clip(np.round(np.exp(rng.normal(6.0, 0.8, total))), 16, 8192).astype(int)
    lo, hi = frames_range
    frames = rng.integers(lo, hi + 1, total)
    rate = world * steady_per_gpu / ((lo + hi) / 2.0)
    out, rid, step = [], 0, 0
    while rid < total:
        for _ in range(int(rng.poisson(rate))):
            if rid < total:
                out.append((rid, step, int(prompts[rid]), int(frames[rid])))
                rid += 1
        step += 1
    return out


@dataclass
class StepOutput:
    mode: int
    rids: list           # stream of each row of the step (decode rows, then admitted)
    codes: np.ndarray    # [rows, G] int64, this step's frame of every row
    finished: list       # streams that ended with this step


class ContinuousTalkerRunner:
    def __init__(self, runner: TalkerDecodeRunner, sched: OmniScheduler, *, sampling: SamplingParams = SamplingParams(),
                 seed: int = 0, use_graphs: bool = True, prompt_pool_rows: int = 0):
        sc = sched.cfg
        if runner.max_batch < sc.max_batch + 1:
            raise ValueError("the runner needs one request slot more than the scheduler's max_batch")
        if runner.max_prefill_tokens < sc.max_prefill_tokens:
            raise ValueError("the runner's max_prefill_tokens is below the scheduler's")
        if runner.kv.num_pages != sc.num_pages or runner.cfg.page_size != sc.page_size:
            raise ValueError("scheduler and KV pool disagree on pages")
        if runner.r2t.req_to_token.shape[1] < sc.max_context:
            raise ValueError("req_to_token rows are shorter than the scheduler's max_context")
        self.runner, self.sched = runner, sched
        self.sampling, self.seed, self.use_graphs = sampling, seed, use_graphs
        cfg, dev = runner.cfg, runner.device
        self.device = dev
        B = sc.max_batch
        self.buckets = decode_graph_buckets(B)
        H = cfg.hidden_size
        G = cfg.predictor.num_code_groups
        i64 = dict(dtype=torch.long, device=dev)
        i32 = dict(dtype=torch.int32, device=dev)
        pin = dict(pin_memory=True)
        # request slot sc.max_batch is the padding rows' slot: tokens 0, 1 of page 0
        self.dummy_slot = sc.max_batch
        runner.r2t.req_to_token[self.dummy_slot].zero_()
        runner.r2t.req_to_token[self.dummy_slot, 1] = 1
        # the step's opened pages, staged from the host (the device allocator of decode_prepare)
        runner.allocator = PageAllocator(torch.zeros(B, dtype=torch.int32), dev)
        self.pages_h = torch.zeros(B, dtype=torch.int32, **pin)
        self.zero_h = torch.zeros(1, dtype=torch.long, **pin)
        self.pad_seq_h = torch.ones(B, dtype=torch.long, **pin)
        self.pad_slot_h = torch.full((B,), self.dummy_slot, dtype=torch.long, **pin)
        # synthetic inputs on the host: the streams' text rows and prompt rows
        g = torch.Generator().manual_seed(seed + 101)
        # each stream's text rows (the thinker's chunk embeddings): a row of this pool
        # chosen by the stream id, gathered into the step's staging rows
        self.text_pool_h = torch.randn(4096, H, generator=g).to(torch.bfloat16)
        self.text_h = torch.zeros(B, H, dtype=torch.bfloat16, **pin)
        P = max(prompt_pool_rows, sc.max_prefill_tokens + 4096)
        self.prompt_h = torch.randn(P, H, generator=g).to(torch.bfloat16).pin_memory()
        self.codes_h = torch.zeros(B, G, dtype=torch.long, **pin)
        # admission staging (host pinned -> device)
        self.adm = {
            "rows": (torch.zeros(B, dtype=torch.int32, **pin), torch.zeros(B, **i32)),
            "slots": (torch.zeros(B, dtype=torch.int32, **pin), torch.zeros(B, **i32)),
            "slots64": (torch.zeros(B, dtype=torch.long, **pin), torch.zeros(B, **i64)),
            "lens": (torch.zeros(B, dtype=torch.long, **pin), torch.zeros(B, **i64)),
            "indptr": (torch.zeros(B + 1, dtype=torch.int32, **pin), torch.zeros(B + 1, **i32)),
            "pages": (torch.zeros(sc.num_pages, dtype=torch.int32, **pin), torch.zeros(sc.num_pages, **i32)),
            "select": (torch.zeros(B, dtype=torch.long, **pin), torch.zeros(B, **i64)),
            "seeds": (torch.zeros(B, dtype=torch.long, **pin), torch.zeros(B, **i64)),
        }
        self.prompt_dev = torch.zeros(sc.max_prefill_tokens, H, dtype=torch.bfloat16, device=dev)
        self.ext_prefix = torch.zeros(B, **i64)
        self.ext_seq_lens = torch.zeros(B, **i64)
        self.ext_qo = torch.zeros(B + 1, **i32)
        self.ext_page_indptr = torch.zeros(B + 1, **i32)
        self.ext_page_indices = torch.zeros(sc.num_pages + B, **i32)
        self.ext_tiles = torch.zeros(B + 1, **i32)
        self.sel_positions = torch.zeros(B, **i64)
        # every per-row state tensor that follows a stream when it changes rows
        t, p = runner.talker, runner.predictor
        self.row_state = ops.RowTensors([
            runner.seq_lens, runner.req_pool_indices,
            t.repetition_penalties, t.repetition_mask, t.suppress_mask, t.sampling_temperatures,
            t.sampling_top_ks, t.sampling_top_ps, t.sampling_min_ps, t.sampling_seeds,
            p.output_embeds, p.sub_temperature_tensor, p.sub_top_k_tensor, p.sub_top_p_tensor,
            p.sub_sampling_seed_tensor, p.sub_do_sample_tensor,
        ])
        # the batch-wide sampler flags of every row (the per-row tensors are restaged at
        # admission): the padding rows of a bucket carry this configuration too
        runner.stage([TalkerRequest(rid=f"pad{i}", seed=0, sampling=sampling) for i in range(runner.max_batch)])
        runner.requests = []
        # per-stream request state by stream id: seeds, the layer-0 output ids so far (the
        # repetition mask of a retracted stream's re-admission carries them), the suppress
        # row without the leading-silence ids and whether those are still masked
        self.streams: dict[int, TalkerRequest] = {}
        self.base_suppress: dict[int, np.ndarray] = {}
        self.silenced: set[int] = set()
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.graph_pool = None
        self.eager_steps = 0
        self.graph_steps = 0
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        runner.graph = None
        runner.extend = None
        runner.batch_size = 0

    # ------------------------------------------------------------------
    def bucket(self, rows: int) -> int:
        for b in self.buckets:
            if b >= rows:
                return b
        raise RuntimeError("batch above the largest decode bucket")

    def request(self, rid: int) -> TalkerRequest:
        """The request state of stream `rid` (synthetic: public seed seed * 1_000_003 + rid)."""
        rq = self.streams.get(rid)
        if rq is None:
            rq = TalkerRequest(rid=f"req{rid}", seed=self.seed * 1_000_003 + rid, sampling=self.sampling, output_ids=[])
            self.streams[rid] = rq
        return rq

    def _after_step(self, rids: list[int], codes: np.ndarray, finished) -> None:
        """Output-id history, leading-silence release and the end of finished streams."""
        lim = self.runner.codec_control.leading_silence_mask_frames
        release = []
        for row, rid in enumerate(rids):
            rq = self.request(int(rid))
            rq.output_ids = list(rq.output_ids or []) + [int(codes[row, 0])]
            if int(rid) in self.silenced and rq.frames >= lim:
                release.append((row, int(rid)))
        for row, rid in release:
            self.runner.talker.suppress_mask[row].copy_(torch.from_numpy(self.base_suppress[rid]))
            self.silenced.discard(rid)
        for rid in finished:
            rid = int(rid)
            self.streams.pop(rid, None)
            self.base_suppress.pop(rid, None)
            self.silenced.discard(rid)

    def _stage_text(self, rids: list[int]) -> None:
        n = len(rids)
        if n:
            idx = torch.tensor([rid % self.text_pool_h.shape[0] for rid in rids], dtype=torch.long)
            torch.index_select(self.text_pool_h, 0, idx, out=self.text_h[:n])

    def _stage_pages(self, pages: np.ndarray) -> None:
        al = self.runner.allocator
        k = int(pages.shape[0])
        if k:
            self.pages_h[:k].copy_(torch.from_numpy(pages))
            al.free_pages[:k].copy_(self.pages_h[:k], non_blocking=True)
            self.h2d_bytes += 4 * k
        al.free_head.copy_(self.zero_h, non_blocking=True)
        self.h2d_bytes += 8

    def _h2d(self, key: str, values, n: int) -> torch.Tensor:
        host, dev = self.adm[key]
        host[:n].copy_(torch.as_tensor(np.asarray(values), dtype=host.dtype))
        dev[:n].copy_(host[:n], non_blocking=True)
        self.h2d_bytes += n * host.element_size()
        return dev[:n]

    def _admit(self, plan: StepPlan) -> None:
        """Device state of the admitted streams and the extend batch of the mixed step."""
        r, t, p = self.runner, self.runner.talker, self.runner.predictor
        sp = self.sampling
        Bd, n, T = plan.decode_rows, plan.new_rows, plan.new_tokens
        lens = plan.new_prompt_len
        rows = self._h2d("rows", np.arange(Bd, Bd + n, dtype=np.int32), n)
        slots = self._h2d("slots", plan.new_slot, n)
        slots64 = self._h2d("slots64", plan.new_slot.astype(np.int64), n)
        lens_d = self._h2d("lens", lens, n)
        indptr = self._h2d("indptr", plan.new_page_indptr, n + 1)
        npg = int(plan.new_page_indptr[n])
        pages = self._h2d("pages", plan.new_pages, npg)
        ops.admit_streams(rows=rows, slots=slots, prompt_lens=lens_d, page_indptr=indptr, pages=pages,
                          req_to_token=r.r2t.req_to_token, page_size=r.cfg.page_size, seq_lens=r.seq_lens,
                          req_pool_indices=r.req_pool_indices, status=r.status)
        # sampling state of the new rows (prepare_decode_buffers): a re-admitted (retracted)
        # stream's repetition mask carries its whole output history
        reqs = [self.request(int(rid)) for rid in plan.new_rid]
        st = r.stage_requests(reqs)
        r.write_staging(st, row0=Bd)
        self.h2d_bytes += n * (2 * r.cfg.vocab_size + 48)
        for i, rid in enumerate(plan.new_rid.tolist()):
            self.base_suppress[int(rid)] = st.base_suppress_mask[i].copy()
            if st.silence_rows[i]:
                self.silenced.add(int(rid))
        # prompt rows of the new streams (compose_prefill_embeds): each stream's rows
        # start at an offset of the host pool chosen by its id
        off = 0
        pool = self.prompt_h.shape[0]
        for rid, L in zip(plan.new_rid.tolist(), lens.tolist()):
            start = (int(rid) * 7919) % (pool - int(L) + 1)
            self.prompt_dev[off: off + L].copy_(self.prompt_h[start: start + L], non_blocking=True)
            off += L
        self.h2d_bytes += T * self.prompt_dev.shape[1] * 2
        # the extend batch (prepare_for_extend): prefix 0, extend = prompt
        last = np.cumsum(lens) - 1
        sel = self._h2d("select", np.concatenate([np.arange(Bd), Bd + last]).astype(np.int64), Bd + n)
        r.ext_req = slots64
        r.ext_prefix = self.ext_prefix[:n]
        r.ext_lens = lens_d
        r.ext_seq_lens = self.ext_seq_lens[:n]
        r.ext_qo = self.ext_qo[: n + 1]
        r.ext_page_indptr = self.ext_page_indptr[: n + 1]
        r.ext_page_indices = self.ext_page_indices
        r.ext_tiles = self.ext_tiles[: n + 1]
        max_tiles = int(sum((int(L) + ops.PREFILL_Q_TILE - 1) // ops.PREFILL_Q_TILE for L in lens))
        r.prompt_embeds = self.prompt_dev[:T]
        r.select = sel
        r.sel_positions = self.sel_positions[: Bd + n]
        r.extend = ExtendForwardBatch(streams=n, tokens=T, qo_indptr=r.ext_qo, seq_lens=r.ext_seq_lens,
                                      page_indptr=r.ext_page_indptr, page_indices=r.ext_page_indices,
                                      tile_indptr=r.ext_tiles, max_tiles=max_tiles)

    def _decode(self, B: int) -> None:
        r = self.runner
        b = self.bucket(B)
        if b > B:
            r.seq_lens[B:b].copy_(self.pad_seq_h[: b - B], non_blocking=True)
            r.req_pool_indices[B:b].copy_(self.pad_slot_h[: b - B], non_blocking=True)
            self.h2d_bytes += 16 * (b - B)
        r.text_embeds[:b].copy_(self.text_h[:b], non_blocking=True)
        self.h2d_bytes += b * self.text_h.shape[1] * 2
        r.batch_size = b
        r.extend = None
        g = self.graphs.get(b)
        if g is not None:
            g.replay()
            self.graph_steps += 1
            return
        r.run_step()
        self.eager_steps += 1
        if self.use_graphs:
            s = torch.cuda.Stream(self.device)
            s.wait_stream(torch.cuda.current_stream(self.device))
            if self.graph_pool is None:
                self.graph_pool = torch.cuda.graph_pool_handle()
            g = torch.cuda.CUDAGraph()
            # recording executes nothing: the device state is unchanged by capture
            with torch.cuda.graph(g, stream=s, pool=self.graph_pool):
                r.run_step()
            torch.cuda.current_stream(self.device).wait_stream(s)
            self.graphs[b] = g

    def capture_buckets(self, up_to: int | None = None) -> None:
        """Record the decode graph of every bucket up to `up_to` rows before serving (the
        reference's decode graph runner captures its buckets at start-up): each bucket
        runs once eagerly over padding rows only, then is recorded.  Only while no
        stream is live."""
        if self.sched.stats()["running"]:
            raise RuntimeError("capture_buckets while streams are running")
        r = self.runner
        top = self.buckets[-1] if up_to is None else self.bucket(up_to)
        self._stage_pages(np.zeros(0, dtype=np.int32))
        for b in self.buckets:
            if b > top:
                break
            if b in self.graphs:
                continue
            r.seq_lens[:b].copy_(self.pad_seq_h[:b], non_blocking=True)
            r.req_pool_indices[:b].copy_(self.pad_slot_h[:b], non_blocking=True)
            self._decode(b)
        torch.cuda.current_stream(self.device).synchronize()
        r.batch_size = 0
        self.eager_steps = self.graph_steps = self.h2d_bytes = self.d2h_bytes = 0

    # ------------------------------------------------------------------
    def step(self, now_us: int | None = None, ready=None) -> StepOutput | None:
        """One iteration of the event loop; None when there was nothing to run.

        ready(plan) -> bool is the talker's is_batch_ready_to_run
        (talker_scheduler.py:159-171): a decode batch whose inputs are not ready is
        rolled back (rollback_decode_prep_after_skip) and nothing runs."""
        plan = self.sched.get_next_batch_to_run(now_us)
        if plan.is_idle():
            return None
        r = self.runner
        if plan.moves_src.size:
            ops.move_rows(self.row_state, plan.moves_src, plan.moves_dst)
        if plan.mode == DECODE and ready is not None and not ready(plan):
            self.sched.rollback_decode_prep_after_skip()
            return None
        self._stage_pages(plan.decode_pages)
        Bd = plan.decode_rows
        rids = self.sched.row_rids()
        self._stage_text(rids[:Bd])
        if plan.mode == MIXED:
            self._admit(plan)
            r.text_embeds[:Bd].copy_(self.text_h[:Bd], non_blocking=True)
            self.h2d_bytes += Bd * self.text_h.shape[1] * 2
            r.batch_size = Bd
            r.run_step()
            self.eager_steps += 1
            r.extend = None
            rows = Bd + plan.new_rows
        else:
            assert plan.mode == DECODE
            self._decode(Bd)
            rows = Bd
        r.batch_size = rows
        self.codes_h[:rows].copy_(r.predictor.output_codes[:rows], non_blocking=True)
        self.d2h_bytes += rows * self.codes_h.shape[1] * 8
        torch.cuda.current_stream(self.device).synchronize()
        rids = rids[:rows]
        codes = self.codes_h[:rows].numpy().copy()
        finished = self.sched.process_batch_result(codes)
        self._after_step(rids, codes, finished)
        return StepOutput(plan.mode, rids, codes, finished)

    def forward_messages(self, relay, backlog: list | None = None) -> list:
        """Hand the ready code chunks to the vocoder stage through a CodecRelay
        (omni_b200.relay), oldest first; what does not fit in the ring stays in the
        returned backlog for the next call (the talker never blocks on the vocoder)."""
        backlog = list(backlog or []) + self.pop_messages()
        sent = 0
        for m in backlog:
            if not relay.push(*m):
                break
            sent += 1
        return backlog[sent:]

    def pop_messages(self) -> list[tuple[int, int, np.ndarray, bool]]:
        """The code chunks ready for the vocoder stage (scheduler emit_messages on):
        (rid, first frame, codes [frames, G], final), in emission order."""
        return self.sched.pop_messages(self.runner.cfg.predictor.num_code_groups)

    def device_status(self) -> int:
        """The packing kernels' sticky status (0 = no page shortfall or bad length)."""
        return int(self.runner.status.item())
