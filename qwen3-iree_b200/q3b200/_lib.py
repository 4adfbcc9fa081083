"""ctypes binding of libq3b200.so (include/q3b200.h).  No PyTorch.

The CUDA path is the only path: importing this module fails loudly when the
shared library is missing, and every non-zero status raises Q3Error.
"""
from __future__ import annotations

import ctypes
import os

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.environ.get("Q3B200_LIB", os.path.join(PKG_DIR, "lib", "libq3b200.so"))

Q3_OK = 0
STATUS_NAMES = {1: "Q3_ERR_INVALID", 2: "Q3_ERR_CUDA", 3: "Q3_ERR_DEVICE", 4: "Q3_ERR_NOMEM",
                5: "Q3_ERR_STATE", 6: "Q3_ERR_UNSUPPORTED"}


class Q3Error(RuntimeError):
    def __init__(self, status: int, where: str, detail: str):
        self.status = status
        super().__init__(f"{where}: {STATUS_NAMES.get(status, status)}: {detail}")


class Weights(ctypes.Structure):
    """struct q3_weights -- device pointers in the reference's parameter layout."""
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "token_embd", "output_norm", "output_T", "attn_norm", "ffn_norm", "attn_q_norm",
        "attn_k_norm", "q8_attn_q", "q8_attn_k", "q8_attn_v", "q8_attn_output", "q8_ffn_gate_up",
        "q8_ffn_down")]


P, I, I64, U32, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_uint32, ctypes.c_size_t
PP = ctypes.POINTER(ctypes.c_void_p)
PI64 = ctypes.POINTER(ctypes.c_int64)

# name -> argtypes (all return int status unless listed in _RESTYPE)
SIGNATURES = {
    "q3_abi_version": [],
    "q3_device_count": [ctypes.POINTER(ctypes.c_int)],
    "q3_set_device": [I],
    "q3_device_info": [I, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                       ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_size_t)],
    "q3_device_malloc": [PP, SZ],
    "q3_device_free": [P],
    "q3_host_malloc": [PP, SZ],
    "q3_host_free": [P],
    "q3_memcpy_htod": [P, P, SZ, P],
    "q3_memcpy_dtoh": [P, P, SZ, P],
    "q3_memcpy_dtod": [P, P, SZ, P],
    "q3_memset": [P, I, SZ, P],
    "q3_stream_create": [PP],
    "q3_stream_destroy": [P],
    "q3_stream_synchronize": [P],
    "q3_graph_capture_begin": [P],
    "q3_graph_capture_end": [P, PP],
    "q3_graph_launch": [P, P],
    "q3_graph_destroy": [P],
    "q3_event_create": [PP],
    "q3_event_destroy": [P],
    "q3_event_record": [P, P],
    "q3_event_synchronize": [P],
    "q3_event_elapsed_ms": [P, P, ctypes.POINTER(ctypes.c_float)],
    "q3_rope_table": [I64, P, P],
    "q3_quantize_q8_0": [P, I64, P],
    "q3_gemv_q8": [P, P, P, I, I, P],
    "q3_gemv_q8_cuda_order": [P, P, P, I, I, P],
    "q3_gemv_q8_overlapped": [P, P, P, I, I, P],
    "q3_gemv_q8_layers": [P, I64, P, P, I, I, I, P],
    "q3_gemv_q8_norm": [P, P, P, P, I, I, P],
    "q3_gemv_q8_resid": [P, P, P, P, I, I, P],
    "q3_gemv_q8_swiglu": [P, P, P, P, I, I, P],
    "q3_vocab_argmax_workspace_bytes": [],
    "q3_vocab_argmax": [P, P, P, P, P, P, I, I, P],
    "q3_attention_workspace_bytes": [I64],
    "q3_decode_attention": [P, P, P, P, P, I64, P, P, I64, I64, P, P, P, P],
    "q3_decode_attention_noalloc": [P, P, P, P, P, I64, P, P, I64, I64, P, P, P],
    "q3_iree_dispatch_3": [P, P, P, U32, U32, P],
    "q3_iree_dispatch_4": [P, P, P, U32, U32, U32, P],
    "q3_iree_dispatch_12": [P, P, P, U32, U32, P],
    "q3_iree_dispatch_18": [P, P, P, U32, U32, P],
    "q3_iree_dispatch_20": [P, P, P, U32, U32, P],
    "q3_iree_dispatch_24": [P, P, P, U32, P],
    "q3_fused_layer_workspace_bytes": [],
    "q3_fused_layer": [ctypes.POINTER(Weights), I, P, P, P, P, I64, P, P, P, P, I, P],
    "q3_model_create": [ctypes.POINTER(Weights), I64, P, PP],
    "q3_model_destroy": [P],
    "q3_model_stream": [P],
    "q3_run": [P, P, I64, I64, I64, P, PI64],
    "q3_decode": [P, I64, I64, P, PI64],
    "q3_init_chat": [P, I64],
    "q3_chat_turn": [P, P, I64, I64, I64, P, PI64],
    "q3_generate_begin": [P, P, I64, I64, I64],
    "q3_generate_steps": [P, I64],
    "q3_generate_end": [P, P, PI64],
    "q3_model_launches_per_step": [P, PI64],
    "q3_model_device_error": [P, ctypes.POINTER(ctypes.c_int)],
    "q3_model_poke": [P, I, I64, I64],
    "q3_selftest_bounded_wait": [P, I, I64, P, P],
    "q3_check_error_word": [P, P],
    "q3_model_profile_steps": [P, I64, P, P, I64],
    "q3_model_set_engine": [P, I],
    "q3_model_engine": [P, ctypes.POINTER(ctypes.c_int)],
    "q3_model_set_prefill": [P, I],
    "q3_model_prefill_mode": [P, ctypes.POINTER(ctypes.c_int)],
    "q3_model_prefill": [P, P, I64, I64],
    "q3_model_kernel_launches": [P, PI64],
    "q3_model_trace_steps": [P, I64, I64, P, I64, ctypes.POINTER(ctypes.c_int),
                             ctypes.POINTER(ctypes.c_int)],
    "q3_bgemm_q8": [P, I64, I64, P, P, P, I, I, I, I, I, P],
    "q3_bvocab_workspace_bytes": [],
    "q3_bvocab_argmax": [P, I, P, I, P, P, P, P],
    "q3_batch_create": [ctypes.POINTER(Weights), I, I64, P, PP],
    "q3_batch_destroy": [P],
    "q3_batch_stream": [P],
    "q3_batch_begin": [P, I, P, I64, P],
    "q3_batch_begin_random": [P, I, P, P, ctypes.c_uint64],
    "q3_batch_steps": [P, I64],
    "q3_batch_read": [P, P, P, ctypes.POINTER(ctypes.c_int)],
    "q3_batch_read_argmax": [P, P],
    "q3_model_trace_kernels": [P, I64, P, P, I64, PI64],
    "q3_model_trace_phases": [P, I64, P, I64, PI64, ctypes.POINTER(ctypes.c_int),
                              ctypes.POINTER(ctypes.c_int)],
    "q3_batch_trace_kernels": [P, I64, P, P, I64, PI64],
    "q3_batch_attention_workspace_bytes": [I64, I],
    "q3_batch_attention": [P, P, P, P, P, I64, P, P, I, I64, I, P, P, P, P],
    "q3_batch_profile_steps": [P, I64, P, P, I64, PI64],
    "q3_batch_trace_phases": [P, I64, P, P, I64, PI64],
    "q3_batch_kernel_launches": [P, PI64],
    "q3_strerror": [I],
    "q3_last_error": [],
}
_RESTYPE = {
    "q3_strerror": ctypes.c_char_p,
    "q3_last_error": ctypes.c_char_p,
    "q3_vocab_argmax_workspace_bytes": SZ,
    "q3_attention_workspace_bytes": SZ,
    "q3_fused_layer_workspace_bytes": SZ,
    "q3_model_stream": P,
    "q3_bvocab_workspace_bytes": SZ,
    "q3_batch_attention_workspace_bytes": SZ,
    "q3_batch_stream": P,
}

_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"libq3b200.so not found at {LIB_PATH}; build it with "
                "`python __graft_entry__.py build` or `make -C qwen3-iree_b200`")
        L = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = _RESTYPE.get(name, ctypes.c_int)
        _lib = L
    return _lib


def check(status: int, where: str) -> None:
    if status != Q3_OK:
        raise Q3Error(status, where, lib().q3_last_error().decode(errors="replace"))


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)
