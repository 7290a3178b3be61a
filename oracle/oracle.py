"""numpy front end of the CPU oracle (oracle/zl_oracle.c).

TEST INFRASTRUCTURE ONLY: the checker for the CUDA path. Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline / reference arm import
this module. Each wrapper names the reference function it restates
(`path:line` inside the reference Rust project 0xnicholas/Zealot).

Besides the C restatement, this file holds the two pieces of host logic the
oracle needs in Python: the BlockManager model (src/block_manager.rs:88-165)
and the Sequence.step_input rule (src/scheduler.rs:88-101).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libzl_oracle.so")
_lib = None

GQA_GROUPED = 0
GQA_MODULO = 1

_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i32p = ctypes.POINTER(ctypes.c_int32)
_i64p = ctypes.POINTER(ctypes.c_int64)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_sz = ctypes.c_size_t


def build() -> str:
    """Compile the oracle with make (gcc -ffp-contract=off, see oracle/Makefile)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.zlo_matmul.argtypes = [_f32p, _f32p, _f32p, _sz, _sz, _sz]
        L.zlo_cpu_attention_forward.argtypes = [_f32p, _sz, _f32p, _sz, _f32p, _sz, _f32p, _sz, _sz, _sz, _sz]
        L.zlo_cpu_attention_forward.restype = ctypes.c_int
        L.zlo_repeat_interleave_kv.argtypes = [_f32p, _f32p, _sz, _sz, _sz, _sz]
        L.zlo_runner_step.argtypes = [_f32p, _sz, _f32p, _f32p, _f32p, _f32p, _f32p, _sz, _sz, _sz, _sz, _sz, _i64p, _sz, _f32p]
        L.zlo_runner_step.restype = ctypes.c_int
        L.zlo_store_kv.argtypes = [_u8p, _u8p, _u8p, _u8p, _i64p, _sz, _sz, _sz, _sz, _sz, _sz, _sz]
        L.zlo_store_kv.restype = ctypes.c_int
        L.zlo_reshape_and_cache.argtypes = [_u8p, _u8p, _u8p, _u8p, _i64p, _sz, _sz, _sz, _sz, _sz, _sz]
        L.zlo_reshape_and_cache.restype = ctypes.c_int
        L.zlo_paged_decode.argtypes = [_f32p, _f32p, _f32p, _i32p, _i32p, _f32p, _sz, _sz, _sz, _sz, _sz, _sz, _sz, ctypes.c_float, ctypes.c_int, ctypes.c_int]
        L.zlo_paged_decode.restype = ctypes.c_int
        L.zlo_paged_decode_partial.argtypes = [_f32p, _f32p, _f32p, _i32p, _i32p, _i32p, _f32p, _f32p, _f32p, _sz, _sz, _sz, _sz, _sz, _sz, _sz, ctypes.c_float, ctypes.c_int]
        L.zlo_paged_decode_partial.restype = ctypes.c_int
        L.zlo_merge_partials.argtypes = [_f32p, _f32p, _f32p, _f32p, _sz, _sz, _sz]
        L.zlo_prefill_varlen.argtypes = [_f32p, _f32p, _f32p, _i32p, _sz, _f32p, _sz, _sz, _sz, ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.zlo_prefill_varlen.restype = ctypes.c_int
        L.zlo_prefill_varlen_rows.argtypes = [_f32p, _f32p, _f32p, _i32p, _sz, _i64p, _sz, _f32p, _sz, _sz, _sz, ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.zlo_prefill_varlen_rows.restype = ctypes.c_int
        L.zlo_argmax.argtypes = [_f32p, _sz]
        L.zlo_argmax.restype = ctypes.c_int64
        L.zlo_f32_to_bf16.argtypes = [_f32p, _u16p, _sz]
        L.zlo_bf16_to_f32.argtypes = [_u16p, _f32p, _sz]
        _f = ctypes.c_float
        L.zlo_sample.argtypes = [_f32p, _sz, _i64p, _sz, _f, ctypes.c_uint32, _f, _f, _f, _f, _u8p, _sz,
                                 _f, ctypes.c_int, _i64p, _f32p, ctypes.POINTER(ctypes.c_double)]
        L.zlo_sample.restype = ctypes.c_int
        L.zlo_softmax_probs.argtypes = [_f32p, _f32p, _sz]
        _lib = L
    return _lib


class OracleError(RuntimeError):
    """The restated reference returned its error path."""


def _p(a: np.ndarray, t):
    assert a.flags["C_CONTIGUOUS"], "oracle buffers must be C-contiguous"
    return a.ctypes.data_as(t)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def default_scale(head_dim: int) -> float:
    """`1.0_f32 / (d_head as f32).sqrt()` (src/attention/mod.rs:53), in fp32."""
    return float(np.float32(1.0) / np.sqrt(np.float32(head_dim)))


# --------------------------------------------------------------- restatements

def matmul(a, b, m: int, k: int, n: int) -> np.ndarray:
    """src/attention/mod.rs:105-115."""
    a = _f32(a).reshape(-1)
    b = _f32(b).reshape(-1)
    c = np.empty(m * n, np.float32)
    lib().zlo_matmul(_p(a, _f32p), _p(b, _f32p), _p(c, _f32p), m, k, n)
    return c


def cpu_attention_forward(q, k, v, num_seqs, num_heads, head_dim, max_seq_len) -> np.ndarray:
    """src/attention/mod.rs:31-103 (raises OracleError on the dimension mismatch of :39-48)."""
    q, k, v = (_f32(x).reshape(-1) for x in (q, k, v))
    n = num_seqs * num_heads * head_dim * max_seq_len
    out = np.empty(max(n, 1), np.float32)
    rc = lib().zlo_cpu_attention_forward(_p(q, _f32p), q.size, _p(k, _f32p), k.size, _p(v, _f32p), v.size,
                                         _p(out, _f32p), num_seqs, num_heads, head_dim, max_seq_len)
    if rc != 0:
        raise OracleError(f"dimension mismatch: expected {n}, got q={q.size} k={k.size} v={v.size}")
    return out[:n]


def repeat_interleave_kv(src, kv_heads, num_heads, seq_len, head_dim) -> np.ndarray:
    """src/model_runner_cpu.rs:286-304."""
    src = _f32(src).reshape(-1)
    out = np.empty(num_heads * seq_len * head_dim, np.float32)
    lib().zlo_repeat_interleave_kv(_p(src, _f32p), _p(out, _f32p), kv_heads, num_heads, seq_len, head_dim)
    return out


def runner_step(w: dict, token_ids) -> np.ndarray:
    """src/model_runner_cpu.rs:172-276 for one sequence; w holds the layer-0
    weights ([in,out] row-major) and the shape fields of CpuModelRunner."""
    ids = np.ascontiguousarray(token_ids, dtype=np.int64)
    logits = np.empty(w["vocab_size"], np.float32)
    emb = _f32(w["embedding"]).reshape(-1)
    mats = [_f32(w[n]).reshape(-1) for n in ("q_proj", "k_proj", "v_proj", "attn_proj", "lm_head")]
    rc = lib().zlo_runner_step(_p(emb, _f32p), emb.size, *(_p(m, _f32p) for m in mats),
                               w["hidden_dim"], w["num_heads"], w["num_kv_heads"], w["head_dim"],
                               w["vocab_size"], _p(ids, _i64p), ids.size, _p(logits, _f32p))
    if rc != 0:
        raise OracleError("runner step failed")
    return logits


def store_kv(k_pool: np.ndarray, v_pool: np.ndarray, k, v, block_ids, start_token, n_tokens,
             num_kv_heads, head_dim, block_size) -> None:
    """src/kv_cache.rs:212-276, in place on byte-viewable pools."""
    k = np.ascontiguousarray(k)
    v = np.ascontiguousarray(v)
    ids = np.ascontiguousarray(block_ids, dtype=np.int64)
    es = k_pool.itemsize
    rc = lib().zlo_store_kv(_p(k_pool.view(np.uint8), _u8p), _p(v_pool.view(np.uint8), _u8p),
                            _p(k.view(np.uint8), _u8p), _p(v.view(np.uint8), _u8p), _p(ids, _i64p),
                            ids.size, start_token, n_tokens, num_kv_heads, head_dim, block_size, es)
    if rc != 0:
        raise OracleError("KVCache store_kv: block_idx OOB")


def reshape_and_cache(k_pool, v_pool, k, v, slot_mapping, num_kv_heads, head_dim, block_size, num_blocks) -> int:
    """Slot-mapping scatter with the offset arithmetic of src/kv_cache.rs:241-247."""
    k = np.ascontiguousarray(k)
    v = np.ascontiguousarray(v)
    sm = np.ascontiguousarray(slot_mapping, dtype=np.int64)
    return lib().zlo_reshape_and_cache(_p(k_pool.view(np.uint8), _u8p), _p(v_pool.view(np.uint8), _u8p),
                                       _p(k.view(np.uint8), _u8p), _p(v.view(np.uint8), _u8p),
                                       _p(sm, _i64p), sm.size, num_kv_heads, head_dim, block_size,
                                       num_blocks, k_pool.itemsize)


def paged_decode(q, k_pool, v_pool, block_tables, seq_lens, num_heads, num_kv_heads, head_dim,
                 block_size, num_blocks, scale=None, gqa_map=GQA_GROUPED, num_threads=1) -> np.ndarray:
    """Decode attention: block-table gather (paged_attention.cu:65-73 layout
    rules) + the CpuAttention row math (src/attention/mod.rs:64-97)."""
    q = _f32(q)
    kp = _f32(k_pool).reshape(-1)
    vp = _f32(v_pool).reshape(-1)
    bt = np.ascontiguousarray(block_tables, dtype=np.int32)
    sl = np.ascontiguousarray(seq_lens, dtype=np.int32)
    B = sl.size
    max_blocks = bt.shape[1] if bt.ndim == 2 else (bt.size // max(B, 1))
    out = np.empty((B, num_heads, head_dim), np.float32)
    if scale is None:
        scale = default_scale(head_dim)
    rc = lib().zlo_paged_decode(_p(q, _f32p), _p(kp, _f32p), _p(vp, _f32p), _p(bt, _i32p), _p(sl, _i32p),
                                _p(out, _f32p), B, num_heads, num_kv_heads, head_dim, block_size,
                                max_blocks, num_blocks, scale, gqa_map, num_threads)
    if rc != 0:
        raise OracleError("block id outside the pool / table overflow")
    return out


def paged_decode_partial(q, k_pool, v_pool, block_tables, tok_begin, tok_end, num_heads, num_kv_heads,
                         head_dim, block_size, num_blocks, scale=None, gqa_map=GQA_GROUPED):
    q = _f32(q)
    kp = _f32(k_pool).reshape(-1)
    vp = _f32(v_pool).reshape(-1)
    bt = np.ascontiguousarray(block_tables, dtype=np.int32)
    tb = np.ascontiguousarray(tok_begin, dtype=np.int32)
    te = np.ascontiguousarray(tok_end, dtype=np.int32)
    B = te.size
    m = np.empty((B, num_heads), np.float32)
    l = np.empty((B, num_heads), np.float32)
    o = np.empty((B, num_heads, head_dim), np.float32)
    if scale is None:
        scale = default_scale(head_dim)
    rc = lib().zlo_paged_decode_partial(_p(q, _f32p), _p(kp, _f32p), _p(vp, _f32p), _p(bt, _i32p),
                                        _p(tb, _i32p), _p(te, _i32p), _p(m, _f32p), _p(l, _f32p),
                                        _p(o, _f32p), B, num_heads, num_kv_heads, head_dim, block_size,
                                        bt.shape[1], num_blocks, scale, gqa_map)
    if rc != 0:
        raise OracleError("block id outside the pool")
    return m, l, o


def merge_partials(m, l, o) -> np.ndarray:
    m = _f32(m)
    l = _f32(l)
    o = _f32(o)
    P = m.shape[0]
    rows = m[0].size
    d = o.shape[-1]
    out = np.empty((rows, d), np.float32)
    lib().zlo_merge_partials(_p(m, _f32p), _p(l, _f32p), _p(o, _f32p), _p(out, _f32p), P, rows, d)
    return out


def prefill_varlen(q, k, v, cu_seqlens, num_heads, num_kv_heads, head_dim, causal=True, scale=None,
                   gqa_map=GQA_GROUPED, num_threads=1) -> np.ndarray:
    q, k, v = _f32(q), _f32(k), _f32(v)
    cu = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
    T = int(cu[-1])
    out = np.empty((T, num_heads, head_dim), np.float32)
    if scale is None:
        scale = default_scale(head_dim)
    rc = lib().zlo_prefill_varlen(_p(q, _f32p), _p(k, _f32p), _p(v, _f32p), _p(cu, _i32p), cu.size - 1,
                                  _p(out, _f32p), num_heads, num_kv_heads, head_dim, scale, int(causal),
                                  gqa_map, num_threads)
    if rc != 0:
        raise OracleError("bad cu_seqlens")
    return out


def prefill_varlen_rows(q, k, v, cu_seqlens, rows, num_heads, num_kv_heads, head_dim, causal=True,
                        scale=None, gqa_map=GQA_GROUPED, num_threads=1) -> np.ndarray:
    q, k, v = _f32(q), _f32(k), _f32(v)
    cu = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
    r = np.ascontiguousarray(rows, dtype=np.int64)
    out = np.empty((r.size, num_heads, head_dim), np.float32)
    if scale is None:
        scale = default_scale(head_dim)
    rc = lib().zlo_prefill_varlen_rows(_p(q, _f32p), _p(k, _f32p), _p(v, _f32p), _p(cu, _i32p), cu.size - 1,
                                       _p(r, _i64p), r.size, _p(out, _f32p), num_heads, num_kv_heads,
                                       head_dim, scale, int(causal), gqa_map, num_threads)
    if rc != 0:
        raise OracleError("bad cu_seqlens")
    return out


def argmax(x) -> int:
    """src/sampling.rs:233-243: first maximum wins."""
    x = _f32(x).reshape(-1)
    return int(lib().zlo_argmax(_p(x, _f32p), x.size))


def softmax(scores) -> np.ndarray:
    """src/sampling.rs:254-273."""
    x = _f32(scores).reshape(-1)
    out = np.empty_like(x)
    lib().zlo_softmax_probs(_p(x, _f32p), _p(out, _f32p), x.size)
    return out


EMPTY_LOGITS, ALL_TOKENS_MASKED = 1, 2  # SamplingError (src/sampling.rs:15-20)


def sample(logits, prev=(), temperature=1.0, top_k=0, top_p=0.0, repetition_penalty=1.0,
           frequency_penalty=0.0, presence_penalty=0.0, mask=None, r=0.5, exact=False):
    """src/sampling.rs:77-230 (Sampler::sample_with_mask) with `r` the rng draw.
    Returns (status, token, logprob, margin): status 0, EMPTY_LOGITS or
    ALL_TOKENS_MASKED; margin = the closest a float decision came to flipping.
    exact=True: the same decisions with every sum in double (see zl_oracle.h)."""
    x = _f32(logits).reshape(-1)
    pv = np.ascontiguousarray(prev, dtype=np.int64).reshape(-1)
    if pv.size == 0:
        pv = np.zeros(1, np.int64)
        n_prev = 0
    else:
        n_prev = pv.size
    if x.size == 0:
        x = np.zeros(1, np.float32)
        n = 0
    else:
        n = x.size
    if mask is None:
        mp, mlen = ctypes.POINTER(ctypes.c_uint8)(), 0
    else:
        m = np.ascontiguousarray(mask, dtype=np.uint8).reshape(-1)
        if m.size == 0:
            m = np.zeros(1, np.uint8)
            mlen = 0
        else:
            mlen = m.size
        mp = _p(m, _u8p)
    tok = np.zeros(1, np.int64)
    lp = np.zeros(1, np.float32)
    margin = ctypes.c_double()
    rc = lib().zlo_sample(_p(x, _f32p), n, _p(pv, _i64p), n_prev, temperature, top_k, top_p,
                          repetition_penalty, frequency_penalty, presence_penalty, mp, mlen, r,
                          int(exact), _p(tok, _i64p), _p(lp, _f32p), ctypes.byref(margin))
    return rc, int(tok[0]), float(lp[0]), float(margin.value)


def f32_to_bf16_bits(x) -> np.ndarray:
    x = _f32(x)
    out = np.empty(x.shape, np.uint16)
    lib().zlo_f32_to_bf16(_p(x.reshape(-1), _f32p), _p(out.reshape(-1), _u16p), x.size)
    return out


def bf16_bits_to_f32(b) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    out = np.empty(b.shape, np.float32)
    lib().zlo_bf16_to_f32(_p(b.reshape(-1), _u16p), _p(out.reshape(-1), _f32p), b.size)
    return out


def round_bf16(x) -> np.ndarray:
    """fp32 values rounded to the nearest bf16 (what a bf16 kernel reads), as fp32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


# ------------------------------------------------------------ host-logic model

class OracleBlockManager:
    """src/block_manager.rs:88-165: LIFO free list (ids 0,1,2,... from a fresh
    pool), refcount, per-block generation starting at 1, stale-handle check."""

    def __init__(self, num_gpu_blocks: int, block_size: int):
        if block_size == 0:
            raise ValueError("InvalidBlockSize")
        self.num_gpu_blocks = num_gpu_blocks
        self.block_size = block_size
        self.free_list = list(range(num_gpu_blocks))[::-1]
        self.refcount = [0] * num_gpu_blocks
        self.generation = [1] * num_gpu_blocks

    def try_allocate(self):
        if not self.free_list:
            raise MemoryError("OutOfBlocks")
        bid = self.free_list.pop()
        self.refcount[bid] = 1
        return (bid, self.generation[bid])

    def _check(self, h):
        bid, gen = h
        if bid >= self.num_gpu_blocks:
            raise KeyError("BlockNotAllocated")
        if gen != self.generation[bid]:
            raise LookupError("StaleHandle")

    def try_free(self, h):
        self._check(h)
        bid = h[0]
        prev = self.refcount[bid]
        self.refcount[bid] = prev - 1
        if prev == 1:
            self.generation[bid] += 1
            self.free_list.append(bid)

    def try_reference(self, h):
        self._check(h)
        self.refcount[h[0]] += 1

    def available(self) -> int:
        return len(self.free_list)


def step_input(prompt, outputs, prefill_pending: bool, prefill_pos: int, chunk_size: int):
    """src/scheduler.rs:88-101."""
    if prefill_pending:
        end = min(prefill_pos + chunk_size, len(prompt))
        return list(prompt[prefill_pos:end]) + list(outputs)
    return [outputs[-1]]
