"""Host-side behaviour of flash_evict.streaming_adapter (no GPU).

Argument checks and messages follow the reference's streaming adapter
(flash_evict/streaming_adapter.py:18-24,34-47); the controller installs and
removes its attention forward; chunk_mlp bounds the feed-forward chunk size
without changing the result; decoding attention masks only the new tokens
among themselves.  Prefill through the controller needs the CUDA library, so
on CPU tensors it raises instead of falling back.
"""
import pytest
import torch

from flash_evict.streaming_adapter import StreamingController, _decode_attention, chunk_mlp


def tiny_model():
    from transformers import Qwen2Config, Qwen2ForCausalLM
    torch.manual_seed(0)
    cfg = Qwen2Config(vocab_size=64, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=32, max_position_embeddings=256)
    return Qwen2ForCausalLM(cfg).eval()


def test_controller_argument_checks():
    m = tiny_model()
    with pytest.raises(ValueError, match="Unsupported backend"):
        StreamingController(m, backend="h2o")
    for bad in (0, -3, 2.5, True, "8"):
        with pytest.raises(ValueError, match="Positive integer budget required"):
            StreamingController(m, budget=bad)


def test_controller_installs_and_restores_forwards():
    m = tiny_model()
    attns = [layer.self_attn for layer in m.model.layers]
    before = [a.forward for a in attns]
    ctl = StreamingController(m, backend="snap", budget=16, scoring={"recency_decay": 0.1})
    assert ctl.mode == "prefill" and ctl.scoring == {"recency_decay": 0.1}
    assert all(a.forward.__func__.__name__ == "_forward" for a in attns)
    ctl.finish_prefill()
    assert ctl.mode == "decode"
    ctl.reset()
    assert ctl.mode == "prefill" and ctl.states == {}
    ctl.restore()
    assert [a.forward for a in attns] == before
    assert not any(hasattr(a, "_kv_controller") for a in attns)


def test_prefill_on_cpu_raises_instead_of_falling_back():
    m = tiny_model()
    ctl = StreamingController(m, backend="fused", budget=8)
    try:
        with torch.no_grad(), pytest.raises(ValueError):
            m(torch.zeros(1, 12, dtype=torch.long), use_cache=False)
    finally:
        ctl.restore()


def test_batched_prompt_is_rejected():
    m = tiny_model()
    ctl = StreamingController(m, backend="full", budget=8)
    try:
        with torch.no_grad(), pytest.raises(ValueError, match="one unpadded prompt"):
            m(torch.zeros(2, 12, dtype=torch.long), use_cache=False)
    finally:
        ctl.restore()


def test_chunk_mlp_same_result_and_restore():
    m = tiny_model()
    ids = torch.randint(0, 64, (1, 40), generator=torch.Generator().manual_seed(2))
    with torch.no_grad():
        ref = m(ids, use_cache=False).logits
        restore = chunk_mlp(m, 7)
        got = m(ids, use_cache=False).logits
        restore()
        again = m(ids, use_cache=False).logits
    torch.testing.assert_close(got, ref, atol=1e-5, rtol=1e-5)
    assert torch.equal(again, ref)


def test_chunk_mlp_checks():
    m = tiny_model()
    for bad in (0, -1, 1.5, True):
        with pytest.raises(ValueError, match="chunk_size must be a positive integer"):
            chunk_mlp(m, bad)
    restore = chunk_mlp(m, 4)
    try:
        with pytest.raises(RuntimeError, match="inference-only"):
            m(torch.zeros(1, 9, dtype=torch.long), use_cache=False)
    finally:
        restore()


def test_decode_attention_masks_only_new_tokens():
    g = torch.Generator().manual_seed(3)
    q = torch.randn(1, 4, 3, 16, generator=g)
    k = torch.randn(1, 2, 10, 16, generator=g)
    v = torch.randn(1, 2, 10, 16, generator=g)
    got = _decode_attention(q, k, v, 0.25)
    kk, vv = k.repeat_interleave(2, 1), v.repeat_interleave(2, 1)
    s = (q @ kk.transpose(-1, -2)) * 0.25
    allowed = torch.arange(10)[None, :] <= torch.arange(7, 10)[:, None]
    ref = torch.softmax(s.masked_fill(~allowed, float("-inf")), -1) @ vv
    torch.testing.assert_close(got, ref, atol=1e-5, rtol=1e-5)
    one = _decode_attention(q[:, :, -1:], k, v, 0.25)
    torch.testing.assert_close(one, ref[:, :, -1:], atol=1e-5, rtol=1e-5)
