"""Generates tests/golden/*.json by executing the reference's own pure-torch code.

Run in a container where the reference checkout is present (its path is the
first argument, default: the REFERENCE_ROOT environment variable).  The
reference cannot be imported whole (its pinned sglang is absent), so this
script loads single functions from their source files:

- ``murmur_hash32_pytorch`` (sglang_omni/models/qwen3_tts/sampling_kernels.py:633-677),
  imported as a module with ``sglang_omni.platforms`` stubbed;
- ``Qwen3TTSTalker.sample_subtalker_token_seeded`` (sglang_model.py:1954-2034),
  whose torch fallback runs on CPU; its last step calls sglang's
  ``multinomial_with_seed``, which is not in the reference tree and is
  restated here from the reference's own description of it
  (sampling_kernels.py:67-78: u = h / (2^32 - 1) in float64, log u clamped to
  [-DBL_MAX, -2^-32], g = -log(-log u), argmax of logprob + g, first maximum);
- ``Qwen3OmniTalker.sample_decode_tokens`` (talker.py:1376-1412) for the
  repetition-penalty / suppression known answer of test_talker.py:2587-2627;
- ``QwenTalkerScheduler.rollback_decode_prep_after_skip``
  (talker_scheduler.py:198-225) for the known answer of test_talker.py:1118-1134.

A second pass (``main_staging``) writes ``staging_golden.json`` and
``sampler_scale_golden.npz`` from more reference code executed the same way:

- ``derive_sampling_seed`` / ``resolve_row_seed`` (sglang_omni/sampling/seed.py:24-48),
  ``derive_qwen3_tts_sampling_seeds`` (qwen3_tts/request_builders.py:94-124) and
  ``rank_shared_unseeded_sampling_seed`` (model_runner/base.py:86-88): seed triples;
- ``Qwen3OmniTalker.prepare_decode_buffers`` (talker.py:1065-1215) on a fake request
  set: repetition / suppress masks and the staged sampling rows;
- ``Qwen3TTSModelRunner.apply_codec_suppress_tokens`` (qwen3_tts/model_runner.py:155-198):
  the control-range and leading-silence masks;
- ``Qwen3TTSTalker.prepare_decode_buffers`` (sglang_model.py:1162-1270): the staged
  subtalker rows and the batch signature;
- the residual sampler's torch fallback on 12 000 rows per case of untied random bf16
  logits at the config-0 and config-3 sampling parameters (tests/golden/scale_inputs.py):
  the tokens only (the logits are regenerated from their seed by the tests).

The outputs are small fixtures; tests read only the fixtures.
"""

from __future__ import annotations

import ast
import base64
import importlib.util
import json
import os
import sys
import types
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _stub_platforms() -> None:
    plat = types.ModuleType("sglang_omni.platforms")
    plat.current_platform = SimpleNamespace(is_npu=lambda: False, is_cuda=lambda: False)
    pkg = types.ModuleType("sglang_omni")
    pkg.__path__ = []
    sys.modules.setdefault("sglang_omni", pkg)
    sys.modules["sglang_omni.platforms"] = plat


def _load_module(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _load_method(path: Path, cls: str, method: str, namespace: dict):
    tree = ast.parse(path.read_text())
    for node in tree.body:
        if isinstance(node, ast.ClassDef) and node.name == cls:
            for item in node.body:
                if isinstance(item, ast.FunctionDef) and item.name == method:
                    item.decorator_list = []
                    mod = ast.Module(body=[item], type_ignores=[])
                    code = compile(mod, str(path), "exec")
                    ns = dict(namespace)
                    exec(code, ns)
                    return ns[method]
    raise LookupError(f"{cls}.{method} not found in {path}")


def main(ref: Path) -> None:
    _stub_platforms()
    sk = _load_module(ref / "sglang_omni/models/qwen3_tts/sampling_kernels.py", "ref_sampling_kernels")
    mh = sk.murmur_hash32_pytorch

    # ---- hash table + endpoints --------------------------------------------------
    cases = [(0, 1_707_985_137), (0x804B40E3, 0), (0x572AB199, 0), (17, 3), (123456789, 42), (2**31 - 1, 2**31 + 5),
             (-1, 7), (0x7FFFFFFF, 0), (5, 2**40 + 9)]
    hashes = []
    for seed, pos in cases:
        h = mh(torch.tensor([seed]), torch.tensor([pos]), 64)[0].tolist()
        hashes.append({"seed": seed, "position": pos, "hash": [int(x) for x in h]})

    # ---- restated multinomial_with_seed (float64 Gumbel-max, first maximum) --------
    def multinomial_with_seed(logprobs, seeds, positions):
        h = mh(seeds, positions, logprobs.shape[1]).to(torch.float64)
        u = h / 4294967295.0
        lu = torch.log(u).clamp(min=torch.finfo(torch.float64).min, max=-(2.0**-32))
        g = -torch.log(-lu)
        return torch.argmax(logprobs.to(torch.float64) + g, dim=1, keepdim=True)

    def sample_seeded_categorical(logprobs, seeds, positions):
        return multinomial_with_seed(logprobs, seeds, positions).view(-1)

    ns = {
        "torch": torch,
        "sample_from_logits_with_seed_top_k_top_p": sk.sample_from_logits_with_seed_top_k_top_p,
        "sample_from_sorted_logprobs_with_seed_small_k": sk.sample_from_sorted_logprobs_with_seed_small_k,
        "sample_seeded_categorical": sample_seeded_categorical,
    }
    sampler = _load_method(ref / "sglang_omni/models/qwen3_tts/sglang_model.py", "Qwen3TTSTalker",
                           "sample_subtalker_token_seeded", ns)

    # ---- residual sampler cases: distinct bf16 logits (torch CPU topk breaks ties
    # differently from the CUDA network, so ties are covered by the GPU tests) -------
    sampler_cases = []
    gen = torch.Generator().manual_seed(0)
    for case_id, (rows, vocab, max_top_k, has_top_p, temp) in enumerate(
        [(6, 2048, 50, True, 0.9), (6, 2048, 50, False, 0.9), (5, 2048, 32, True, 0.7), (5, 2048, 16, False, 1.0),
         (4, 2048, 4, True, 1.3), (4, 2048, 64, True, 0.9), (4, 2048, 128, True, 0.5), (3, 1024, 256, True, 0.9),
         (3, 2048, 1024, True, 1.0), (4, 1024, 8, True, 0.9)]
    ):
        perm = torch.stack([torch.randperm(vocab, generator=gen) for _ in range(rows)])
        # distinct bf16 values: consecutive bf16 magnitudes below 8 with both signs
        first = 0x3D00 if vocab == 2048 else 0x3F00
        mags = (torch.arange(first, first + vocab // 2, dtype=torch.int32) << 16).view(torch.float32)
        base = torch.cat([mags, -mags])
        logits = base[perm].to(torch.bfloat16)
        assert all(len(set(r.tolist())) == vocab for r in logits.float())
        temps = torch.full((rows,), temp, dtype=torch.float32)
        top_ks = torch.randint(1, max_top_k + 1, (rows,), generator=gen).long()
        top_ks[0] = max_top_k
        top_ps = torch.tensor([0.8, 1.0, 0.5, 0.95, 0.3, 0.0][:rows] + [0.8] * max(0, rows - 6), dtype=torch.float32)
        seeds = torch.randint(0, 2**31 - 1, (rows,), generator=gen).long()
        positions = torch.randint(0, 10_000, (rows,), generator=gen).long()
        self_ns = SimpleNamespace(
            sub_temperature_tensor=temps,
            sub_top_k_tensor=top_ks,
            sub_top_p_tensor=top_ps,
            sub_sampling_seed_tensor=seeds,
            sub_sampled_max_top_k=max_top_k,
            sub_sampled_has_unbounded_top_k=False,
            sub_sampled_has_top_p=has_top_p,
        )
        tokens = sampler(self_ns, logits, sub_positions=positions)
        sampler_cases.append({
            "id": case_id,
            "logits_bf16_b64": base64.b64encode(logits.view(torch.int16).numpy().astype("<u2").tobytes()).decode(),
            "shape": [rows, vocab],
            "temperatures": temps.tolist(),
            "top_ks": top_ks.tolist(),
            "top_ps": top_ps.tolist(),
            "seeds": seeds.tolist(),
            "positions": positions.tolist(),
            "max_top_k": max_top_k,
            "has_top_p": has_top_p,
            "tokens": tokens.tolist(),
        })

    # ---- sorted Gumbel sampler endpoints (test_sampling_kernels.py:73-148) -----------
    sorted_cases = []
    for seed, other, endpoint, pos in [(0x804B40E3, -100.0, 0.0, 0), (0x572AB199, 0.0, -100.0, 0),
                                       (0, -100.0, 0.0, 1_707_985_137)]:
        lp = torch.full((1, 50), other, dtype=torch.float32)
        lp[:, -1] = endpoint
        idx = torch.arange(50).view(1, -1)
        rank = multinomial_with_seed(lp, torch.tensor([seed]), torch.tensor([pos]))
        sorted_cases.append({"logprobs": lp.tolist(), "sorted_idx": idx.tolist(), "seed": seed, "position": pos,
                             "token": int(idx.gather(1, rank).item())})
    lp = torch.tensor([[-100.0, 0.0]])
    rank = multinomial_with_seed(lp, torch.tensor([0]), torch.tensor([1_707_985_137]))
    sorted_cases.append({"logprobs": lp.tolist(), "sorted_idx": [[7, 9]], "seed": 0, "position": 1_707_985_137,
                         "token": [7, 9][int(rank.item())]})

    # ---- layer-0 penalty / suppression known answer (test_talker.py:2587-2627) ----
    seen = {}

    def fake_sampler(logits_output, *args):
        seen["logits"] = logits_output.next_token_logits.clone()
        return logits_output.next_token_logits.argmax(dim=-1)

    talker_ns = {"torch": torch, "LogitsProcessorOutput": lambda **kw: SimpleNamespace(**kw)}
    sample_decode = _load_method(ref / "sglang_omni/models/qwen3_omni/components/talker.py", "Qwen3OmniTalker",
                                 "sample_decode_tokens", talker_ns)
    logits = torch.tensor([[2.0, -1.0, 0.5, 1.9], [0.1, 0.2, 0.3, -3.0]])
    fake = SimpleNamespace(
        repetition_penalties=torch.tensor([[1.05], [2.0]]),
        repetition_mask=torch.zeros(2, 4, dtype=torch.bool),
        suppress_mask=torch.zeros(2, 4, dtype=torch.bool),
        sampler=fake_sampler,
        build_static_sampling_info=lambda batch_size: None,
    )
    fake.repetition_mask[0, 0] = True
    fake.repetition_mask[1, 3] = True
    fake.suppress_mask[1, 2] = True
    toks = sample_decode(fake, logits, SimpleNamespace(positions=None))
    penalty = {
        "logits": logits.tolist(),
        "penalties": [1.05, 2.0],
        "rep_mask": fake.repetition_mask.to(torch.uint8).tolist(),
        "suppress_mask": fake.suppress_mask.to(torch.uint8).tolist(),
        "processed": [[float(x) if np.isfinite(x) else None for x in row] for row in seen["logits"].tolist()],
        "argmax_tokens": toks.tolist(),
    }

    # ---- rollback known answer (test_talker.py:1118-1134) --------------------------
    freed = []
    rollback = _load_method(ref / "sglang_omni/models/qwen3_omni/talker_scheduler.py", "QwenTalkerScheduler",
                            "rollback_decode_prep_after_skip", {"torch": torch})
    sched = SimpleNamespace(token_to_kv_pool_allocator=SimpleNamespace(
        page_size=4, free=lambda indices: freed.append(indices.tolist())))
    batch = SimpleNamespace(
        forward_mode=SimpleNamespace(is_decode=lambda: True), reqs=[],
        out_cache_loc=torch.tensor([16, 22]), seq_lens=torch.tensor([5, 7]), seq_lens_cpu=torch.tensor([5, 7]),
        orig_seq_lens=torch.tensor([5, 7]), req_pool_indices=torch.tensor([0, 1]),
        req_to_token_pool=SimpleNamespace(req_to_token=torch.ones(2, 8, dtype=torch.int32)))
    rollback(sched, batch)
    rollback_golden = {"page_size": 4, "seq_lens": [5, 7], "out_cache_loc": [16, 22], "req_pool_indices": [0, 1],
                       "freed": freed, "seq_lens_after": batch.seq_lens.tolist(),
                       "req_to_token_after": batch.req_to_token_pool.req_to_token.tolist()}

    out = {
        "source": "executed reference functions; see tests/golden/make_golden.py",
        "hashes": hashes,
        "residual_sampler": sampler_cases,
        "sorted_sampler": sorted_cases,
        "layer0_penalty": penalty,
        "rollback": rollback_golden,
    }
    (HERE / "reference_golden.json").write_text(json.dumps(out))
    print("wrote", HERE / "reference_golden.json")


def _load_function(path: Path, name: str, namespace: dict):
    tree = ast.parse(path.read_text())
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name == name:
            node.decorator_list = []
            ns = dict(namespace)
            exec(compile(ast.Module(body=[node], type_ignores=[]), str(path), "exec"), ns)
            return ns[name]
    raise LookupError(f"{name} not found in {path}")


def _residual_sampler(ref: Path):
    """The reference's sample_subtalker_token_seeded with its torch fallback (see main)."""
    _stub_platforms()
    sk = _load_module(ref / "sglang_omni/models/qwen3_tts/sampling_kernels.py", "ref_sampling_kernels2")
    mh = sk.murmur_hash32_pytorch

    def multinomial_with_seed(logprobs, seeds, positions):
        h = mh(seeds, positions, logprobs.shape[1]).to(torch.float64)
        u = h / 4294967295.0
        lu = torch.log(u).clamp(min=torch.finfo(torch.float64).min, max=-(2.0**-32))
        g = -torch.log(-lu)
        return torch.argmax(logprobs.to(torch.float64) + g, dim=1, keepdim=True)

    ns = {
        "torch": torch,
        "sample_from_logits_with_seed_top_k_top_p": sk.sample_from_logits_with_seed_top_k_top_p,
        "sample_from_sorted_logprobs_with_seed_small_k": sk.sample_from_sorted_logprobs_with_seed_small_k,
        "sample_seeded_categorical": lambda lp, s, p: multinomial_with_seed(lp, s, p).view(-1),
    }
    return _load_method(ref / "sglang_omni/models/qwen3_tts/sglang_model.py", "Qwen3TTSTalker",
                        "sample_subtalker_token_seeded", ns)


def main_staging(ref: Path) -> None:
    seed_mod = _load_module(ref / "sglang_omni/sampling/seed.py", "ref_seed")
    seed_ns = {"derive_sampling_seed": seed_mod.derive_sampling_seed, "resolve_row_seed": seed_mod.resolve_row_seed,
               "SAMPLING_SEED_MASK": seed_mod.SAMPLING_SEED_MASK, "new_random_sampling_seed": seed_mod.new_random_sampling_seed,
               "_QWEN3_TTS_SAMPLING_SEED_MASK": seed_mod.SAMPLING_SEED_MASK}
    rb = ref / "sglang_omni/models/qwen3_tts/request_builders.py"
    normalize = _load_function(rb, "normalize_qwen3_tts_seed", seed_ns)
    seed_ns["normalize_qwen3_tts_seed"] = normalize
    child = _load_function(rb, "derive_qwen3_tts_child_seed", seed_ns)
    seed_ns["derive_qwen3_tts_child_seed"] = child
    tts_seeds = _load_function(rb, "derive_qwen3_tts_sampling_seeds", seed_ns)
    unseeded = _load_function(ref / "sglang_omni/model_runner/base.py", "rank_shared_unseeded_sampling_seed", seed_ns)

    derive_cases = [("qwen3-tts", 0, "semantic"), ("qwen3-tts", 0, "subtalker"), ("qwen3-tts", 42, "semantic"),
                    ("sglang-omni-unseeded-row", "req-7", None), ("sglang-omni-unseeded-row", "", None),
                    ("ns", 2**40 + 3, "x"), ("ns", -5, None), ("ünïcode", "päth", "λ")]
    derive = [{"namespace": n, "seed": sd, "label": lb, "value": seed_mod.derive_sampling_seed(n, sd, lb)}
              for n, sd, lb in derive_cases]
    tts = [{"seed": sd, "semantic_subtalker": list(tts_seeds(sd))}
           for sd in (0, 1, 42, 2**31 - 1, 2**31, 2**40 + 5, -7, 123456789, 7.0)]
    resolve = [{"seed": sd, "value": seed_mod.resolve_row_seed(sd)} for sd in (0, 5, 2**31 - 1, 2**31, -1, 2**63 - 1)]
    rows_unseeded = [{"rid": rid, "row": i, "value": unseeded(SimpleNamespace(request_id=rid), i)}
                     for i, rid in enumerate(["a", "req-12", None, "ß"])]

    # ---- Qwen3OmniTalker.prepare_decode_buffers on a fake request set ------------------
    B, V = 6, 64
    omni_prep = _load_method(ref / "sglang_omni/models/qwen3_omni/components/talker.py", "Qwen3OmniTalker",
                             "prepare_decode_buffers", {"torch": torch, **seed_ns})
    fake = SimpleNamespace(
        reuse_decode_buffers=lambda reqs: False, sampling_staging_event=None,
        repetition_mask=torch.zeros(B, V, dtype=torch.bool), suppress_mask=torch.zeros(B, V, dtype=torch.bool),
        sampling_staging_cpu=torch.zeros(6, B, dtype=torch.int64), sampling_staging_gpu=torch.zeros(6, B, dtype=torch.int64),
        repetition_penalties=torch.ones(B, 1), sampling_temperatures=torch.ones(B, 1), sampling_top_ps=torch.ones(B),
        sampling_min_ps=torch.zeros(B), sampling_top_ks=torch.ones(B, dtype=torch.int32),
        sampling_seeds=torch.zeros(B, dtype=torch.int64))
    omni_reqs = [
        dict(rid="r0", penalty=1.05, temperature=0.9, top_p=0.8, top_k=50, min_p=0.0, seed=None,
             output_ids=[3, 3, 17, 63, 64, 100, -1], suppress=[5, 70, 63], codec_suppress=None),
        dict(rid="r1", penalty=1.0, temperature=0.7, top_p=1.0, top_k=20, min_p=0.05, seed=12345,
             output_ids=[1, 2, 3], suppress=None, codec_suppress=[0, 1]),
        dict(rid="r2", penalty=2.0, temperature=1.0, top_p=0.95, top_k=64, min_p=0.0, seed=2**31 + 9,
             output_ids=[], suppress=[], codec_suppress=None),
        dict(rid="r3", penalty=1.3, temperature=0.5, top_p=0.5, top_k=1, min_p=0.1, seed=-3,
             output_ids=[10, 11, 10, 12], suppress=[7], codec_suppress=[8]),
        dict(rid="", penalty=1.1, temperature=1.2, top_p=0.9, top_k=40, min_p=0.0, seed=None,
             output_ids=None, suppress=None, codec_suppress=None),
        dict(rid="r5", penalty=0.9, temperature=0.9, top_p=0.8, top_k=50, min_p=0.0, seed=0,
             output_ids=[60, 61, 62, 63], suppress=[60, 61, 62, 63], codec_suppress=None),
    ]

    def omni_request(d):
        sp = SimpleNamespace(repetition_penalty=d["penalty"], temperature=d["temperature"], top_p=d["top_p"],
                             top_k=d["top_k"], min_p=d["min_p"], sampling_seed=d["seed"])
        req = SimpleNamespace(rid=d["rid"], sampling_params=sp, output_ids=d["output_ids"],
                              _codec_suppress_tokens=d["codec_suppress"])
        return SimpleNamespace(data=SimpleNamespace(req=req, suppress_tokens=d["suppress"]))

    omni_prep(fake, [omni_request(d) for d in omni_reqs])
    omni_golden = {
        "vocab": V, "requests": omni_reqs,
        "repetition_mask": fake.repetition_mask.to(torch.uint8).tolist(),
        "suppress_mask": fake.suppress_mask.to(torch.uint8).tolist(),
        "repetition_penalties": fake.repetition_penalties[:, 0].tolist(),
        "temperatures": fake.sampling_temperatures[:, 0].tolist(), "top_ps": fake.sampling_top_ps.tolist(),
        "min_ps": fake.sampling_min_ps.tolist(), "top_ks": fake.sampling_top_ks.tolist(),
        "seeds": fake.sampling_seeds.tolist(),
    }

    # ---- Qwen3TTSModelRunner.apply_codec_suppress_tokens ---------------------------------
    supp = _load_method(ref / "sglang_omni/models/qwen3_tts/model_runner.py", "Qwen3TTSModelRunner",
                        "apply_codec_suppress_tokens", {"torch": torch})
    tts_rows = [(False, 0), (True, 0), (True, 1), (True, 2), (True, 5), (False, 3)]
    silence = [4, 9, 2047, 100]
    runner = SimpleNamespace(model=SimpleNamespace(config=SimpleNamespace(vocab_size=3072, codec_eos_token_id=2150)),
                             leading_silence_mask_frames=2, silence_codec_ids=torch.tensor(silence))
    lo = SimpleNamespace(next_token_logits=torch.zeros(len(tts_rows), 3072))
    supp(runner, lo, [SimpleNamespace(data=SimpleNamespace(mask_leading_silence=m, output_codes=[0] * f))
                      for m, f in tts_rows])
    masked = torch.isinf(lo.next_token_logits)
    tts_suppress = {"vocab": 3072, "codec_eos_token_id": 2150, "leading_silence_mask_frames": 2,
                    "silence_codec_ids": silence, "rows": [{"mask_leading_silence": m, "frames": f} for m, f in tts_rows],
                    "masked": [torch.nonzero(r).view(-1).tolist() for r in masked]}

    # ---- Qwen3TTSTalker.prepare_decode_buffers (subtalker staging) ------------------------
    sm = ref / "sglang_omni/models/qwen3_tts/sglang_model.py"
    ladder_ns = {}
    tree = ast.parse(sm.read_text())
    for node in tree.body:
        if isinstance(node, ast.Assign) and any(getattr(t, "id", "") == "_PREDICTOR_TOP_K_LADDER" for t in node.targets):
            exec(compile(ast.Module(body=[node], type_ignores=[]), str(sm), "exec"), ladder_ns)
    qtk = _load_function(sm, "quantize_predictor_top_k", ladder_ns)
    pst = _load_function(sm, "predictor_signature_terms", {"quantize_predictor_top_k": qtk})
    tts_prep = _load_method(sm, "Qwen3TTSTalker", "prepare_decode_buffers",
                            {"torch": torch, "predictor_signature_terms": pst, "is_pin_memory_available": lambda d: False})
    Bt = 5
    tfake = SimpleNamespace(
        sub_temperature_tensor=torch.zeros(Bt), sub_top_p_tensor=torch.zeros(Bt),
        sub_top_k_tensor=torch.zeros(Bt, dtype=torch.int64), sub_sampling_seed_tensor=torch.zeros(Bt, dtype=torch.int64),
        sub_do_sample_tensor=torch.zeros(Bt, dtype=torch.bool), semantic_sampling_seed_tensor=torch.zeros(Bt, dtype=torch.int64),
        decode_prep_rids=None, decode_prep_epoch=0,
        config=SimpleNamespace(code_predictor_config=SimpleNamespace(vocab_size=2048)))
    tts_reqs = [dict(seed=0, dosample=True, temperature=0.9, top_p=0.8, top_k=50),
                dict(seed=77, dosample=False, temperature=0.0, top_p=0.3, top_k=-1),
                dict(seed=2**33, dosample=True, temperature=0.0, top_p=1.0, top_k=7),
                dict(seed=5, dosample=True, temperature=1.3, top_p=0.95, top_k=120),
                dict(seed=6, dosample=False, temperature=0.9, top_p=0.8, top_k=0)]

    def tts_request(d):
        sem, sub = tts_seeds(d["seed"])
        return SimpleNamespace(request_id=None, data=SimpleNamespace(
            semantic_sampling_seed=sem, subtalker_dosample=d["dosample"], subtalker_temperature=d["temperature"],
            subtalker_top_p=d["top_p"], subtalker_top_k=d["top_k"], subtalker_sampling_seed=sub,
            decode_prep_epoch=None))

    tts_prep(tfake, [tts_request(d) for d in tts_reqs])
    tts_staging = {"requests": tts_reqs, "predictor_vocab": 2048,
                   "semantic_seeds": tfake.semantic_sampling_seed_tensor.tolist(),
                   "temperatures": tfake.sub_temperature_tensor.tolist(), "top_ps": tfake.sub_top_p_tensor.tolist(),
                   "top_ks": tfake.sub_top_k_tensor.tolist(), "seeds": tfake.sub_sampling_seed_tensor.tolist(),
                   "do_sample": tfake.sub_do_sample_tensor.tolist(),
                   "max_top_k": tfake.sub_sampled_max_top_k, "has_top_p": tfake.sub_sampled_has_top_p,
                   "has_sampled_rows": tfake.sub_has_sampled_rows, "has_argmax_rows": tfake.sub_has_argmax_rows,
                   "has_unbounded_top_k": tfake.sub_sampled_has_unbounded_top_k}

    out = {"source": "executed reference functions; see tests/golden/make_golden.py (main_staging)",
           "derive": derive, "tts_seeds": tts, "resolve_row_seed": resolve, "unseeded_rows": rows_unseeded,
           "omni_prepare_decode_buffers": omni_golden, "tts_codec_suppress": tts_suppress,
           "tts_prepare_decode_buffers": tts_staging}
    (HERE / "staging_golden.json").write_text(json.dumps(out))
    print("wrote", HERE / "staging_golden.json")

    # ---- the residual sampler at scale ------------------------------------------------------
    sys.path.insert(0, str(HERE))
    from scale_inputs import SCALE_CASES, scale_case

    sampler = _residual_sampler(ref)
    arrays = {}
    for name, *_ in SCALE_CASES:
        bits, temps, top_ks, top_ps, seeds, positions, max_top_k = scale_case(name)
        logits = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16)
        self_ns = SimpleNamespace(
            sub_temperature_tensor=torch.from_numpy(temps), sub_top_k_tensor=torch.from_numpy(top_ks),
            sub_top_p_tensor=torch.from_numpy(top_ps), sub_sampling_seed_tensor=torch.from_numpy(seeds),
            sub_sampled_max_top_k=max_top_k, sub_sampled_has_unbounded_top_k=False, sub_sampled_has_top_p=True)
        toks = []
        for r0 in range(0, bits.shape[0], 2000):
            sl = slice(r0, r0 + 2000)
            sub = SimpleNamespace(**{k: (v[sl] if isinstance(v, torch.Tensor) else v) for k, v in vars(self_ns).items()})
            toks.append(sampler(sub, logits[sl], sub_positions=torch.from_numpy(positions[sl])))
        arrays[name] = torch.cat(toks).numpy().astype(np.int16)
    np.savez_compressed(HERE / "sampler_scale_golden.npz", **arrays)
    print("wrote", HERE / "sampler_scale_golden.npz")


if __name__ == "__main__":
    root = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("REFERENCE_ROOT", "/nonexistent"))
    if not root.exists():
        raise SystemExit(f"reference checkout not found at {root}")
    main(root)
    main_staging(root)
