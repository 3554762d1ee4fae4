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

The outputs are small JSON fixtures; tests read only the fixtures.
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


if __name__ == "__main__":
    root = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("REFERENCE_ROOT", "/nonexistent"))
    if not root.exists():
        raise SystemExit(f"reference checkout not found at {root}")
    main(root)
