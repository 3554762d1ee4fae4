"""ctypes binding of the C oracle (omni_oracle.c) — test infrastructure only.

Every function takes and returns numpy arrays; see omni_oracle.c for the
reference file:line each one restates.
"""

from __future__ import annotations

import ctypes
import numpy as np

from oracle import build as _build

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = _build.build()
        l = ctypes.CDLL(str(path))
        l.orc_hash.restype = ctypes.c_uint32
        l.orc_hash.argtypes = [_I64, _I64, ctypes.c_uint32]
        l.orc_expf.restype = ctypes.c_float
        l.orc_expf.argtypes = [ctypes.c_float]
        l.orc_logf.restype = ctypes.c_float
        l.orc_logf.argtypes = [ctypes.c_float]
        l.orc_log.restype = ctypes.c_double
        l.orc_log.argtypes = [ctypes.c_double]
        l.orc_gumbel.restype = ctypes.c_double
        l.orc_gumbel.argtypes = [ctypes.c_uint32]
        l.orc_sample_topk_topp.argtypes = [_P, _I64, _I64, _I64, _P, _P, _P, _P, _P, ctypes.c_int, ctypes.c_int, _P]
        l.orc_sample_sorted.argtypes = [_P, _P, _I64, _I64, _P, _P, _P]
        l.orc_codebook_step.argtypes = [_P, _I64, _I64, _P, _I64, _P, _I64, _P, _P]
        l.orc_gather_add.argtypes = [_P, _I64, _P, _I64, _P, _P]
        l.orc_layer0_sample.argtypes = [_P, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_int, _P, _P]
        l.orc_decode_prepare.argtypes = [_I64, _P, _P, _P, _I64, _I64, _P, _I64, _P, _P, _P, _P, _P, _P, _P]
        l.orc_decode_rollback.restype = _I64
        l.orc_decode_rollback.argtypes = [_I64, _P, _P, _P, _I64, _I64, _P, _P]
        l.orc_moe_route.argtypes = [_P, _I64, _I64, _I64, ctypes.c_int, _P, _P]
        l.orc_moe_permute.argtypes = [_P, _I64, _I64, _I64, _P, _P]
        l.orc_e4m3_from_f32.restype = ctypes.c_uint8
        l.orc_e4m3_from_f32.argtypes = [ctypes.c_float]
        l.orc_e4m3_to_f32.restype = ctypes.c_float
        l.orc_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        l.orc_quant_fp8_group.argtypes = [_P, _I64, _I64, _I64, _P, _P]
        l.orc_extend_prepare.argtypes = [_I64, _P, _P, _P, _P, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _P]
        _lib = l
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


def _c(a, dtype):
    return None if a is None else np.ascontiguousarray(a, dtype=dtype)


def murmur_hash(seed: int, position: int, column: int) -> int:
    return int(lib().orc_hash(int(seed), int(position), int(column)))


def expf(x: float) -> float:
    return float(lib().orc_expf(float(x)))


def logf(x: float) -> float:
    return float(lib().orc_logf(float(x)))


def log64(x: float) -> float:
    return float(lib().orc_log(float(x)))


def gumbel(h: int) -> float:
    return float(lib().orc_gumbel(int(h)))


def sample_topk_topp(logits_bf16_bits: np.ndarray, temperatures, top_ks, top_ps, seeds, positions, *,
                     max_top_k: int, has_top_p: bool) -> np.ndarray:
    """logits as uint16 bf16 bit patterns [rows, vocab]."""
    lg = _c(logits_bf16_bits, np.uint16)
    rows, vocab = lg.shape
    out = np.zeros(rows, np.int64)
    args = [_c(temperatures, np.float32), _c(top_ks, np.int64), _c(top_ps, np.float32), _c(seeds, np.int64),
            _c(positions, np.int64)]
    rc = lib().orc_sample_topk_topp(_p(lg), rows, vocab, vocab, *map(_p, args), int(max_top_k), int(has_top_p),
                                    _p(out))
    if rc != 0:
        raise ValueError("oracle: unsupported sampler contract")
    return out


def sample_sorted(logprobs, sorted_idx, seeds, positions) -> np.ndarray:
    lp = _c(logprobs, np.float32)
    idx = _c(sorted_idx, np.int64)
    rows, cols = lp.shape
    out = np.zeros(rows, np.int64)
    sd = _c(seeds, np.int64)
    ps = _c(positions, np.int64)
    rc = lib().orc_sample_sorted(_p(lp), _p(idx), rows, cols, _p(sd), _p(ps), _p(out))
    if rc != 0:
        raise ValueError("oracle: unsupported")
    return out


def codebook_step(logits_bf16_bits, table_bits, summed_bits=None, with_gathered=True):
    lg = _c(logits_bf16_bits, np.uint16)
    tb = _c(table_bits, np.uint16)
    rows, vocab = lg.shape
    hidden = tb.shape[1]
    codes = np.zeros(rows, np.int64)
    gathered = np.zeros((rows, hidden), np.uint16) if with_gathered else None
    summed = None if summed_bits is None else _c(summed_bits, np.uint16).copy()
    lib().orc_codebook_step(_p(lg), rows, vocab, _p(tb), hidden, _p(codes), 1, _p(gathered), _p(summed))
    return codes, gathered, summed


def gather_add(tokens, table_bits, summed_bits):
    tk = _c(tokens, np.int64)
    tb = _c(table_bits, np.uint16)
    rows = tk.shape[0]
    hidden = tb.shape[1]
    gathered = np.zeros((rows, hidden), np.uint16)
    summed = _c(summed_bits, np.uint16).copy()
    lib().orc_gather_add(_p(tk), rows, _p(tb), hidden, _p(gathered), _p(summed))
    return gathered, summed


def layer0_sample(logits, penalties, rep_mask, suppress_mask, temperatures, top_ks, top_ps, min_ps, seeds,
                  positions, *, max_top_k: int, return_processed: bool = False):
    lg = _c(logits, np.float32)
    rows, vocab = lg.shape
    out = np.zeros(rows, np.int64)
    processed = np.zeros((rows, vocab), np.float32) if return_processed else None
    keep = [_c(penalties, np.float32), _c(rep_mask, np.uint8), _c(suppress_mask, np.uint8),
            _c(temperatures, np.float32), _c(top_ks, np.int64), _c(top_ps, np.float32), _c(min_ps, np.float32),
            _c(seeds, np.int64), _c(positions, np.int64)]
    rc = lib().orc_layer0_sample(_p(lg), rows, vocab, *map(_p, keep), int(max_top_k), _p(out), _p(processed))
    if rc != 0:
        raise ValueError("oracle: unsupported layer-0 contract")
    return (out, processed) if return_processed else out


def decode_prepare(seq_lens, req_pool_indices, req_to_token, page_size, free_pages, free_head=0):
    """Returns (seq_lens, req_to_token, out_cache_loc, positions, kv_indptr, kv_indices,
    page_indptr, page_indices, free_head) after one prepare_for_decode."""
    sl = _c(seq_lens, np.int64).copy()
    rp = _c(req_pool_indices, np.int64)
    r2t = _c(req_to_token, np.int32).copy()
    fp = _c(free_pages, np.int32)
    rows = sl.shape[0]
    max_ctx = r2t.shape[1]
    head = np.array([free_head], np.int64)
    out_loc = np.zeros(rows, np.int64)
    pos = np.zeros(rows, np.int64)
    total = int(sl.sum()) + rows
    kv_indptr = np.zeros(rows + 1, np.int32)
    kv_indices = np.zeros(max(total, 1), np.int32)
    page_indptr = np.zeros(rows + 1, np.int32)
    page_indices = np.zeros(max(total, 1), np.int32)
    rc = lib().orc_decode_prepare(rows, _p(sl), _p(rp), _p(r2t), max_ctx, int(page_size), _p(fp), fp.shape[0],
                                  _p(head), _p(out_loc), _p(pos), _p(kv_indptr), _p(kv_indices),
                                  _p(page_indptr), _p(page_indices))
    if rc != 0:
        raise RuntimeError("oracle: KV capacity exceeded")
    return (sl, r2t, out_loc, pos, kv_indptr, kv_indices[: kv_indptr[-1]], page_indptr,
            page_indices[: page_indptr[-1]], int(head[0]))


def decode_rollback(seq_lens, req_pool_indices, req_to_token, page_size, out_cache_loc):
    sl = _c(seq_lens, np.int64).copy()
    r2t = _c(req_to_token, np.int32).copy()
    freed = np.zeros(sl.shape[0], np.int64)
    rp = _c(req_pool_indices, np.int64)
    loc = _c(out_cache_loc, np.int64)
    n = lib().orc_decode_rollback(sl.shape[0], _p(sl), _p(rp), _p(r2t), r2t.shape[1], int(page_size), _p(loc),
                                  _p(freed))
    return sl, r2t, freed[:n]


def extend_prepare(prefix_lens, extend_lens, req_pool_indices, req_to_token, page_size, q_tile=128):
    """Returns (seq_lens, qo_indptr, out_cache_loc, positions, page_indptr, page_indices, tile_indptr)."""
    pre = _c(prefix_lens, np.int64)
    ext = _c(extend_lens, np.int64)
    rp = _c(req_pool_indices, np.int64)
    r2t = _c(req_to_token, np.int32)
    rows = pre.shape[0]
    total = int(ext.sum())
    sl = np.zeros(rows, np.int64)
    qo = np.zeros(rows + 1, np.int32)
    loc = np.zeros(max(total, 1), np.int64)
    pos = np.zeros(max(total, 1), np.int64)
    pgp = np.zeros(rows + 1, np.int32)
    npages = int(sum((pre + ext + page_size - 1) // page_size))
    pgi = np.zeros(max(npages, 1), np.int32)
    tp = np.zeros(rows + 1, np.int32)
    if lib().orc_extend_prepare(rows, _p(pre), _p(ext), _p(rp), _p(r2t), r2t.shape[1], int(page_size), int(q_tile),
                                _p(sl), _p(qo), _p(loc), _p(pos), _p(pgp), _p(pgi), _p(tp)) != 0:
        raise ValueError("oracle: extend exceeds max_ctx")
    return sl, qo, loc[:total], pos[:total], pgp, pgi[:npages], tp


def moe_route(router_logits, top_k: int, renormalize: bool = True):
    lg = _c(router_logits, np.float32)
    tokens, experts = lg.shape
    ids = np.zeros((tokens, top_k), np.int32)
    w = np.zeros((tokens, top_k), np.float32)
    rc = lib().orc_moe_route(_p(lg), tokens, experts, int(top_k), int(renormalize), _p(ids), _p(w))
    if rc != 0:
        raise ValueError("oracle: unsupported routing contract")
    return ids, w


def moe_permute(topk_ids, experts: int):
    ids = _c(topk_ids, np.int32)
    tokens, k = ids.shape
    offsets = np.zeros(experts + 1, np.int32)
    pairs = np.zeros(tokens * k, np.int32)
    lib().orc_moe_permute(_p(ids), tokens, k, experts, _p(offsets), _p(pairs))
    return offsets, pairs


def e4m3_from_f32(x) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    f = lib().orc_e4m3_from_f32
    return np.array([f(float(v)) for v in x], np.uint8)


_E4M3_TABLE = None


def e4m3_to_f32(b) -> np.ndarray:
    """Decodes e4m3 bytes through the oracle's decoder (as a 256-entry table)."""
    global _E4M3_TABLE
    if _E4M3_TABLE is None:
        f = lib().orc_e4m3_to_f32
        _E4M3_TABLE = np.array([f(i) for i in range(256)], np.float32)
    return _E4M3_TABLE[np.asarray(b, np.uint8)]


def quant_fp8_group(x, group: int = 128):
    """Per-row, per-group e4m3 quantisation: returns (q uint8 [rows, cols], scales f32 [rows, cols/group])."""
    xs = _c(x, np.float32)
    rows, cols = xs.shape
    q = np.zeros((rows, cols), np.uint8)
    sc = np.zeros((rows, cols // group), np.float32)
    if lib().orc_quant_fp8_group(_p(xs), rows, cols, int(group), _p(q), _p(sc)) != 0:
        raise ValueError("oracle: group must divide the row length")
    return q, sc


# ---------------------------------------------------------------------------
# bf16 helpers (numpy)
# ---------------------------------------------------------------------------
def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7F800000) == 0x7F800000
    nan &= (u & 0x007FFFFF) != 0
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


