"""ctypes binding of include/zealot_attn.h (libzealot_attn.so).

This is the Python twin of the `extern "C"` block a Rust host would write
for the same header. It loads the in-tree library and declares every entry
point; nothing here computes.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libzealot_attn.so")

c_int, c_int64, c_uint64, c_float, c_size_t = (ctypes.c_int, ctypes.c_int64, ctypes.c_uint64,
                                               ctypes.c_float, ctypes.c_size_t)
c_void_p, c_char_p = ctypes.c_void_p, ctypes.c_char_p
P = ctypes.POINTER


class zl_ctx_cfg(ctypes.Structure):
    _fields_ = [("device", c_int), ("workspace_bytes", c_size_t)]


class zl_block_handle(ctypes.Structure):
    _fields_ = [("block_id", c_uint64), ("generation", c_uint64)]


class zl_runner_cfg(ctypes.Structure):
    _fields_ = [("hidden_dim", c_int), ("num_heads", c_int), ("num_kv_heads", c_int),
                ("head_dim", c_int), ("num_layers", c_int), ("vocab_size", c_int),
                ("num_gpu_blocks", c_uint64), ("block_size", c_int),
                ("max_blocks_per_seq", c_int), ("gqa_map", c_int)]


class zl_runner_weights(ctypes.Structure):
    _fields_ = [(n, P(c_float)) for n in ("embedding", "q_proj", "k_proj", "v_proj",
                                          "attn_proj", "lm_head")]


class zl_seq_input(ctypes.Structure):
    _fields_ = [("request_id", c_char_p), ("tokens", P(c_int64)), ("num_tokens", c_int),
                ("is_prefill", c_int), ("prefill_pos", c_int)]


class zl_layer_weights(ctypes.Structure):
    _fields_ = [(n, c_void_p) for n in ("attn_norm", "wq", "wk", "wv", "wo", "mlp_norm",
                                        "w_gate_up", "w_down")]


class zl_decoder(ctypes.Structure):
    _fields_ = [("num_layers", c_int), ("hidden", c_int), ("num_heads", c_int),
                ("num_kv_heads", c_int), ("head_dim", c_int), ("intermediate", c_int),
                ("vocab", c_int64), ("rms_eps", c_float), ("embed", c_void_p),
                ("layers", P(zl_layer_weights)), ("final_norm", c_void_p), ("lm_head", c_void_p)]


class zl_step_batch(ctypes.Structure):
    _fields_ = [("tokens", c_void_p), ("slot_mapping", c_void_p), ("cu_prefill", c_void_p),
                ("num_prefill", c_int), ("max_prefill_len", c_int), ("prefill_tokens", c_int64),
                ("block_tables", c_void_p), ("seq_lens", c_void_p), ("num_decode", c_int),
                ("max_blocks_per_seq", c_int), ("last_rows", c_void_p), ("num_last", c_int)]


class zl_sampling_params(ctypes.Structure):
    _fields_ = [("temperature", c_float), ("top_k", c_int), ("top_p", c_float),
                ("repetition_penalty", c_float), ("frequency_penalty", c_float),
                ("presence_penalty", c_float)]


# name -> (restype, argtypes); every symbol declared in include/zealot_attn.h
SIGNATURES = {
    "zl_ctx_create": (c_int, [P(zl_ctx_cfg), P(c_void_p)]),
    "zl_ctx_set_flags": (c_int, [c_void_p, ctypes.c_uint32]),
    "zl_ctx_destroy": (c_int, [c_void_p]),
    "zl_last_error": (c_char_p, []),
    "zl_status_string": (c_char_p, [c_int]),
    "zl_abi_version": (c_int, []),
    "zl_check_status": (c_int, [c_void_p, c_void_p]),
    "zl_launch_count": (c_uint64, [c_void_p]),
    "zl_selftest_wait_timeout": (c_int, [c_void_p, c_void_p]),
    "zl_reshape_and_cache": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                     c_int64, c_int, c_int, c_int, c_int64, c_int, c_void_p]),
    "zl_paged_decode": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int64,
                                c_float, c_int, c_int, c_int, c_void_p]),
    "zl_paged_decode_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                        c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
                                        c_int, c_int64, c_float, c_void_p]),
    "zl_paged_decode_partial": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                        c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                                        c_int, c_int, c_int, c_int, c_int, c_int64, c_float, c_int,
                                        c_int, c_void_p]),
    "zl_merge_partials": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int64, c_int,
                                  c_void_p, c_int, c_void_p]),
    "zl_prefill_varlen": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                  c_int64, c_void_p, c_int, c_int, c_int, c_float, c_int, c_int,
                                  c_int, c_void_p]),
    "zl_nccl_get_unique_id": (c_int, [c_void_p]),
    "zl_nccl_init": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int64, c_int, c_int]),
    "zl_nccl_merge": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p,
                              c_int, c_void_p]),
    "zl_nccl_wait": (c_int, [c_void_p, c_int]),
    "zl_nccl_abort": (c_int, [c_void_p]),
    "zl_nccl_finalize": (c_int, [c_void_p]),
    "zl_block_manager_create": (c_int, [c_uint64, c_uint64, P(c_void_p)]),
    "zl_block_manager_destroy": (c_int, [c_void_p]),
    "zl_block_manager_try_allocate": (c_int, [c_void_p, P(zl_block_handle)]),
    "zl_block_manager_try_free": (c_int, [c_void_p, P(zl_block_handle)]),
    "zl_block_manager_try_reference": (c_int, [c_void_p, P(zl_block_handle)]),
    "zl_block_manager_available": (c_uint64, [c_void_p]),
    "zl_kv_cache_create": (c_int, [c_void_p, c_uint64, c_int, c_int, c_int, c_int, c_int,
                                   P(c_void_p)]),
    "zl_kv_cache_destroy": (c_int, [c_void_p]),
    "zl_kv_cache_register_seq": (c_int, [c_void_p, c_char_p, c_int]),
    "zl_kv_cache_alloc_block": (c_int, [c_void_p, c_char_p, c_void_p, P(zl_block_handle)]),
    "zl_kv_cache_release_seq": (c_int, [c_void_p, c_char_p]),
    "zl_kv_cache_store_kv": (c_int, [c_void_p, c_int, c_char_p, c_void_p, c_void_p, c_uint64,
                                     c_uint64, c_void_p]),
    "zl_kv_cache_append_kv": (c_int, [c_void_p, c_int, c_char_p, c_void_p, c_void_p, c_void_p]),
    "zl_kv_cache_cached_tokens": (c_int, [c_void_p, c_char_p, P(c_uint64)]),
    "zl_kv_cache_block_table_ptr": (c_void_p, [c_void_p, c_char_p]),
    "zl_kv_cache_k_pool_ptr": (c_void_p, [c_void_p, c_int]),
    "zl_kv_cache_v_pool_ptr": (c_void_p, [c_void_p, c_int]),
    "zl_runner_create": (c_int, [c_void_p, P(zl_runner_cfg), P(zl_runner_weights), P(c_void_p)]),
    "zl_runner_destroy": (c_int, [c_void_p]),
    "zl_runner_step": (c_int, [c_void_p, P(zl_seq_input), c_int, P(c_float)]),
    "zl_runner_drop_state": (c_int, [c_void_p, c_char_p]),
    "zl_sample": (c_int, [c_void_p, c_void_p, c_int, c_int64, c_void_p, c_void_p, c_void_p, c_int64,
                          c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p,
                          c_void_p, c_void_p, c_void_p]),
    "zl_decode_graph_create": (c_int, [c_void_p, P(zl_decoder), P(c_void_p), P(c_void_p), c_int64, c_int,
                                       c_int, c_int, c_int, P(c_void_p)]),
    "zl_decode_graph_destroy": (c_int, [c_void_p]),
    "zl_decode_graph_set_row": (c_int, [c_void_p, c_int, P(ctypes.c_int32), c_int, c_int, c_int64,
                                        P(zl_sampling_params), P(c_int64), c_int]),
    "zl_decode_graph_clear_row": (c_int, [c_void_p, c_int]),
    "zl_decode_graph_rows_needing_block": (c_int, [c_void_p, P(ctypes.c_int32), P(c_int)]),
    "zl_decode_graph_step": (c_int, [c_void_p, P(ctypes.c_int32), c_int, P(c_float), c_void_p]),
    "zl_decode_graph_tokens": (c_int, [c_void_p, P(c_int64), P(c_float)]),
    "zl_decode_graph_logits": (c_int, [c_void_p, P(c_float)]),
    "zl_decode_graph_num_kernels": (c_int, [c_void_p]),
    "zl_linear_swiglu": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int, c_void_p]),
    "zl_decoder_step": (c_int, [c_void_p, P(zl_decoder), P(c_void_p), P(c_void_p), c_int64, c_int,
                                P(zl_step_batch), c_void_p, c_void_p]),
}

_lib = None


def load(path: str = LIB_PATH):
    """Loads libzealot_attn.so and declares its signatures. Raises if the
    library has not been built: there is no Python fallback."""
    global _lib
    if _lib is None:
        if not os.path.exists(path):
            raise ImportError(f"{path} is missing: build it with `python zealot_b200/build.py`")
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib
