"""Kernels of the streaming vocoder step, with the call signatures of sglang_omni/kernels."""
