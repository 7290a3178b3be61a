"""Host-side layout of a decoder engine step (no GPU): the row order, slot mapping
and last rows StepBatch.build gives zl_decoder_step, following the slot
arithmetic of KVCache::append_kv (src/kv_cache.rs:212-357) and the step input of
Sequence::step_input (src/scheduler.rs:88-113)."""
import numpy as np


def test_step_batch_layout():
    from zealot_b200.decoder import StepBatch
    b = StepBatch.build([np.arange(20), np.arange(5)], [7, 8],
                        np.array([[3, -1], [4, 5]], np.int32), [10, 17], [[0, 1], [2]], 16,
                        device="cpu")
    assert b.prefill_tokens == 25 and b.num_prefill == 2 and b.num_decode == 2
    assert b.cu_prefill.tolist() == [0, 20, 25]
    assert b.tokens.tolist() == list(range(20)) + list(range(5)) + [7, 8]
    # prefill rows: block ids from their tables; decode rows: position seq_len - 1
    assert b.slot_mapping.tolist() == list(range(20)) + [32, 33, 34, 35, 36, 3 * 16 + 9, 5 * 16 + 0]
    assert b.last_rows.tolist() == [19, 24, 25, 26]
    assert b.max_blocks_per_seq == 2 and b.max_prefill_len == 20


def test_step_batch_one_kind_only():
    from zealot_b200.decoder import StepBatch
    p = StepBatch.build([np.arange(33)], [], None, [], [[4, 9, 2]], 16, device="cpu")
    assert p.num_decode == 0 and p.num_last == 1 and p.last_rows.tolist() == [32]
    assert p.slot_mapping[-1].item() == 2 * 16 + 0
    d = StepBatch.build([], [1, 2], [[9], [8]], [3, 16], [], 16, device="cpu")
    assert d.prefill_tokens == 0 and d.cu_prefill.tolist() == [0]
    assert d.slot_mapping.tolist() == [9 * 16 + 2, 8 * 16 + 15]
    assert d.last_rows.tolist() == [0, 1]


def test_mistral_shapes():
    from zealot_b200.decoder import DecoderConfig
    c = DecoderConfig.mistral_7b()
    s = c.layer_shapes()
    params = sum(int(np.prod(v)) for v in s.values())
    assert s["w_gate_up"] == (2 * 14336, 4096) and s["wk"] == (1024, 4096)
    assert params == 218112000  # 4096*(4096+1024+1024+4096+3*14336) + 2*4096
