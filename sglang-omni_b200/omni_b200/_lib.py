"""ctypes binding of libomni_b200.so (the C ABI declared in include/omni_b200.h).

The library is the only compute path: if it is missing or fails to load on a
machine with a GPU, every op raises.  There is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libomni_b200.so"

OMNI_OK = 0
OMNI_ERR_UNSUPPORTED = 1
OMNI_ERR_INVALID = 2
OMNI_ERR_CAPACITY = 3
OMNI_ERR_CUDA = 4

# status word of omni_device_status (include/omni_b200.h OMNI_DEV_*)
OMNI_DEV_TIMEOUT_TMA = 0x100
OMNI_DEV_TIMEOUT_MMA = 0x200
OMNI_DEV_BAD_INDEX = 0x300
OMNI_DEV_TIMEOUT_FLAG = 0x400

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_F32 = ctypes.c_float
_U32 = ctypes.c_uint32

# name -> argument types (all entry points return int unless listed in _RESTYPES)
SIGNATURES: dict[str, list] = {
    "omni_version": [],
    "omni_last_error": [],
    "omni_device_status": [ctypes.c_int],
    "omni_sample_topk_topp": [_P, _I64, _I64, _I64, _P, _P, _P, _P, _P, _I32, _I32, _P, _P],
    "omni_predictor_sample_step": [_P, _I64, _I64, _I64, _P, _P, _P, _P, _P, _I64, _I64, _P, _I32, _I32, _I32,
                                   _P, _I64, _P, _I64, _P, _P, _P, _P],
    "omni_sample_sorted_seeded": [_P, _P, _I64, _I64, _P, _P, _P, _P],
    "omni_codebook_step": [_P, _I64, _I64, _I64, _P, _I64, _P, _I64, _P, _P, _P],
    "omni_gather_embedding_add": [_P, _I32, _I64, _P, _I64, _P, _P, _P, _I64, _P, _P],
    "omni_layer0_sample": [_P, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I32, _P, _P, _P],
    "omni_predictor_pair_inputs": [_P, _P, _I64, _P, _P, _I32, _I64, _F32, _P, _P, _I64, _I64, _P, _P, _P, _P, _I64,
                                   _P],
    "omni_add_sumsq": [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _I64, _P],
    "omni_linear_fused": [_P, _P],
    "omni_linear_workspace_bytes": [_I64, _I64, _I64, _I32, _I32],
    "omni_linear": [_P, _I64, _I64, _I64, _P, _I64, _I32, _P, _I64, _P, _I64, _P, _I64, _I32, _P],
    "omni_rmsnorm": [_P, _I64, _P, _I64, _P, _I64, _P, _F32, _P, _I64, _I64, _I64, _P],
    "omni_qknorm_rope_store": [_P, _I64, _I64, _I32, _I32, _I32, _P, _P, _F32, _P, _I64, _P, _P, _I32, _I32, _I32,
                               _P, _I64, _P, _P, _P],
    "omni_paged_attention_workspace_bytes": [_I64, _I32, _I64],
    "omni_paged_decode_attention": [_P, _I64, _P, _P, _P, _P, _P, _P, _I64, _I32, _I32, _I32, _I32, _I32, _I64, _F32,
                                    _P, _I64, _P, _I64, _I32, _P],
    "omni_paged_decode_attention_noalloc": [_P, _I64, _P, _P, _P, _P, _P, _P, _I64, _I32, _I32, _I32, _I32, _I32,
                                            _I64, _F32, _P, _I64, _I32, _P],
    "omni_predictor_attention": [_P, _I64, _P, _P, _I64, _I32, _I32, _I32, _I32, _I32, _I32, _F32, _P, _I64, _P],
    "omni_decode_prepare": [_I64, _P, _P, _P, _I64, _I32, _P, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _I32, _P, _P],
    "omni_decode_rollback": [_I64, _P, _P, _P, _I64, _I32, _P, _P, _P, _P, _P],
    "omni_move_rows": [_P, _P, _P, _I32, _P, _P, _I32, _P],
    "omni_admit_streams": [_I64, _P, _P, _P, _P, _P, _P, _I64, _I32, _P, _P, _P, _P],
    # host-only continuous-batching scheduler (include/omni_sched.h)
    "omni_sched_create": [_P],
    "omni_sched_destroy": [_P],
    "omni_sched_add_request": [_P, _I64, _I64, _I64],
    "omni_sched_abort": [_P, _I64],
    "omni_sched_schedule": [_P, _I64, _P],
    "omni_sched_commit": [_P, _P, _I64, _I32, _P, _P],
    "omni_sched_pop_message": [_P, _P, _P, _P, _P, _P, _I64],
    "omni_sched_rollback": [_P],
    "omni_sched_stats": [_P, _P, _I32],
    "omni_sched_row_rids": [_P, _P, _I64, _P],
    "omni_sched_request_state": [_P, _I64, _P, _P, _P, _I64, _P],
    "omni_sched_check": [_P],
    # host-only codec-frame relay (include/omni_relay.h)
    "omni_relay_open": [ctypes.c_char_p, _I64, _I32],
    "omni_relay_close": [_P, _I32],
    "omni_relay_push": [_P, _I64, _I64, _I32, _I32, _I32, _P],
    "omni_relay_pop": [_P, _P, _P, _P, _P, _P, _P, _I64],
    "omni_relay_stats": [_P, _P, _I32],
    "omni_moe_rmsnorm_quant": [_P, _I64, _P, _I32, _I64, _P, _F32, _I64, _I32, _P, _I64, _P, _P, _P],
    "omni_moe_chunk_capacity": [_I64, _I32, _I32],
    "omni_moe_align_gather": [_P, _I64, _I32, _I32, _P, _P, _I32, _P, _P, _P, _P, _P, _I64, _P, _P],
    "omni_moe_gate_up_fp8": [_P, _P, _I64, _I32, _P, _P, _I32, _I32, _P, _P, _P, _P, _P],
    "omni_moe_down_fp8": [_P, _P, _I64, _I32, _P, _P, _I32, _I32, _P, _P, _P, _I64, _P],
    "omni_moe_combine": [_P, _I64, _P, _P, _I32, _P, _I64, _P, _P, _I64, _P, _I64, _P, _I64, _I64, _I32, _P],
    "omni_moe_align_gather_strided": [_P, _I64, _I64, _I32, _I32, _P, _I64, _P, _I64, _I32, _P, _P, _P, _P, _P, _I64,
                                      _P, _P],
    "omni_moe_ep_pack": [_P, _P, _I64, _I32, _P, _I64, _P, _I64, _I32, _I32, _I32, _I64, _P, _I64, _P, _P],
    "omni_moe_partial_sum": [_P, _I64, _P, _P, _I64, _I32, _I64, _I32, _P, _I64, _P],
    "omni_moe_combine_parts": [_P, _I64, _P, _I32, _P, _I64, _P, _P, _I64, _P, _I64, _P, _I64, _I64, _I32, _P],
    "omni_extend_prepare": [_I64, _P, _P, _P, _P, _I64, _I32, _P, _P, _P, _P, _P, _P, _P, _I32, _P, _P],
    "omni_prefill_attention": [_P, _I64, _I64, _P, _P, _I64, _P, _P, _P, _P, _P, _I64, _I64, _I32, _I32, _I32,
                               _I32, _F32, _P, _I64, _P],
    "omni_bias_snake_beta": [_P, _I64, _P, _P, _P, _P, _I64, _P, _P, _I64, _I64, _I64, _I32, _P],
    "omni_clamped_single_output_conv": [_P, _I64, _P, _I64, _I64, _P, _P, _I64, _I64, _I64, _I32, _I32, _P],
    "omni_conv1d_gemm": [_P, _I64, _I64, _I32, _P, _I32, _I32, _I32, _I64, _P, _I64, _P, _P, _P, _P, _P, _P],
    "omni_conv_window_gather": [_P, _I64, _I64, _I64, _I64, _I32, _I32, _I32, _I32, _P, _P],
    "omni_history_exchange": [_P, _I64, _I64, _I64, _P, _I64, _I64, _I64, _P, _I64, _I32, _I32, _I32, _I32, _I32,
                              _I32, _P],
    "omni_gemm_wait_probe": [_P, _I64, _I64, _P, _I64, _P, _I32, _U32, _P],
    "omni_overlap_exchange": [_P, _I64, _I64, _I64, _P, _I64, _I64, _I64, _P, _I64, _I32, _I32, _I32, _I32, _I32,
                              _P],
}
_RESTYPES = {
    "omni_version": ctypes.c_char_p,
    "omni_last_error": ctypes.c_char_p,
    "omni_device_status": ctypes.c_uint,
    "omni_linear_workspace_bytes": ctypes.c_int64,
    "omni_paged_attention_workspace_bytes": ctypes.c_int64,
    "omni_moe_chunk_capacity": ctypes.c_int64,
    "omni_sched_create": ctypes.c_void_p,
    "omni_sched_destroy": None,
    "omni_relay_open": ctypes.c_void_p,
    "omni_relay_close": None,
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class OmniUnsupported(Exception):
    """The call is outside the kernel's contract (the reference returns None/False)."""


def load() -> ctypes.CDLL:
    """Load the CUDA library; raise if it is absent (no fallback path exists)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            if os.environ.get("OMNI_B200_AUTOBUILD", "1") != "0":
                import importlib.util

                spec = importlib.util.spec_from_file_location(
                    "omni_b200_build", LIB_PATH.parent.parent / "build.py"
                )
                mod = importlib.util.module_from_spec(spec)
                spec.loader.exec_module(mod)
                mod.build()
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"omni_b200 CUDA library not found at {LIB_PATH}; build it with "
                    "`python sglang-omni_b200/build.py`"
                )
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, argtypes in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = _RESTYPES.get(name, ctypes.c_int)
        _lib = lib
        return lib


def exported_symbols() -> list[str]:
    return list(SIGNATURES)


def last_error() -> str:
    return load().omni_last_error().decode()


def check(rc: int, name: str) -> None:
    """Raise the Python exception matching an OMNI_* return code."""
    if rc == OMNI_OK:
        return
    msg = f"{name}: {last_error()}"
    if rc == OMNI_ERR_UNSUPPORTED:
        raise OmniUnsupported(msg)
    if rc == OMNI_ERR_INVALID:
        raise ValueError(msg)
    if rc == OMNI_ERR_CAPACITY:
        raise RuntimeError(msg)
    raise RuntimeError(f"CUDA error in {msg}")


# Entry points that launch kernels (counted by launch_count()), one kernel each but
# the paged decode attention (the attention and the merge of split rows).
_HOST_ONLY = ("omni_version", "omni_last_error", "omni_device_status")
_LAUNCHERS = {n for n in SIGNATURES
              if not n.endswith("_bytes") and not n.startswith(("omni_sched_", "omni_relay_")) and n not in _HOST_ONLY}
_KERNELS_PER_CALL = {"omni_paged_decode_attention": 2, "omni_paged_decode_attention_noalloc": 2}
_launches = 0


def launch_count() -> int:
    """Number of kernels launched through the C-ABI by this process so far."""
    return _launches


def call(name: str, *args) -> None:
    global _launches
    check(getattr(load(), name)(*args), name)
    if name in _LAUNCHERS:
        _launches += _KERNELS_PER_CALL.get(name, 1)


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def device_status(reset: bool = False) -> int:
    return int(load().omni_device_status(1 if reset else 0))
