"""The reference's per-layer prefill-and-compact flow, run on this package.

Restates one attention layer of flash_evict/streaming_adapter.py:57-87 (and
the fused prefill of flash_evict/kv_distill_adapter.py:49-71) without its
kv_distill dependency or model weights: a Qwen2-shaped layer with random
projections, rotary embeddings from transformers (apply_rotary_pos_emb, as
the adapter imports it), q/k/v as [B,N,H,D]-transposed views, then
  fused: prefill -> select_tokens -> gather_tokens(k), gather_tokens(v)
  snap:  flash_attention -> snap_scores -> snap_select -> gather
with the compacted cache checked bitwise against torch.gather and the layer
output against the oracle attention on the same rotated inputs.
"""
import numpy as np
import pytest
import torch

from common import selection_mismatch
from flash_evict import gather_tokens, prefill, select_and_gather, select_tokens
from flash_evict.baselines import flash_attention, snap_scores, snap_select
from oracle import restate as O

pytestmark = pytest.mark.gpu

HIDDEN, HEADS, KV_HEADS, HEAD_DIM, N = 1024, 8, 2, 128, 2000


def make_layer(seed):
    from transformers import Qwen2Config
    from transformers.models.qwen2.modeling_qwen2 import Qwen2RotaryEmbedding
    g = torch.Generator().manual_seed(seed)
    w = lambda o, i: (torch.randn(o, i, generator=g) * i ** -0.5).to(torch.bfloat16).cuda()
    cfg = Qwen2Config(hidden_size=HIDDEN, num_attention_heads=HEADS, num_key_value_heads=KV_HEADS,
                      head_dim=HEAD_DIM, max_position_embeddings=4 * N)
    rot = Qwen2RotaryEmbedding(cfg, device="cuda")
    return dict(q=w(HEADS * HEAD_DIM, HIDDEN), k=w(KV_HEADS * HEAD_DIM, HIDDEN), v=w(KV_HEADS * HEAD_DIM, HIDDEN),
                o=w(HIDDEN, HEADS * HEAD_DIM), rot=rot)


def project(layer, hidden):
    # streaming_adapter.py:72-77: projections viewed as [B,N,H,D] then transposed, RoPE applied
    from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb
    b, n, _ = hidden.shape
    q = (hidden @ layer["q"].T).view(b, n, HEADS, HEAD_DIM).transpose(1, 2)
    k = (hidden @ layer["k"].T).view(b, n, KV_HEADS, HEAD_DIM).transpose(1, 2)
    v = (hidden @ layer["v"].T).view(b, n, KV_HEADS, HEAD_DIM).transpose(1, 2)
    pos = torch.arange(n, device="cuda")[None]
    cos, sin = layer["rot"](v, pos)
    q, k = apply_rotary_pos_emb(q, k, cos, sin)
    return q, k, v


@pytest.mark.parametrize("backend", ["fused", "snap"])
def test_layer_prefill_and_compaction(backend):
    torch.manual_seed(0)
    layer = make_layer(3)
    hidden = torch.randn(1, N, HIDDEN, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16).cuda()
    q, k, v = project(layer, hidden)
    budget, reserved = 256, 64
    if backend == "fused":
        # kv_distill_adapter.py:63 then streaming_adapter.py:63-65
        out, importance = prefill(q, k, v, recency_decay=0.1)
        idx, keep = select_tokens(importance, budget, reserved_recent=reserved)
        k_kept, v_kept = gather_tokens(k, idx), gather_tokens(v, idx)
        # the same step in one launch
        idx2, keep2, k2, v2 = select_and_gather(importance, budget, k, v, reserved_recent=reserved)
        assert torch.equal(idx2, idx) and torch.equal(keep2, keep) and torch.equal(k2, k_kept)
        assert torch.equal(v2, v_kept)
        ref_out, ref_imp = O.materialized(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                          v.float().cpu().numpy(), recency_decay=0.1)
        np.testing.assert_allclose(importance.cpu().numpy(), ref_imp, atol=3e-3, rtol=3e-4)
        _, ref_keep = O.select_tokens(ref_imp, budget, reserved_recent=reserved)
        _, ok = selection_mismatch(keep.cpu().numpy(), ref_keep, importance.cpu().numpy(), ref_imp, 3e-3, 3e-4)
        assert ok
    else:
        # streaming_adapter.py:78-83
        out = flash_attention(q, k, v)
        scores = snap_scores(q, k, 32)
        idx, keep = snap_select(scores, budget, 32)
        k_kept, v_kept = gather_tokens(k, idx), gather_tokens(v, idx)
        ref_out, _ = O.materialized(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy())
        ref_s = O.snap_scores(q.float().cpu().numpy(), k.float().cpu().numpy(), 32, "bfloat16")
        rel = np.abs(scores.cpu().numpy() - ref_s) / (np.abs(ref_s) + 1e-6)
        assert np.quantile(rel, 0.99) < 1e-4
    np.testing.assert_allclose(out.float().cpu().numpy(), ref_out, atol=0.012, rtol=0.006)
    gather = lambda x: x.gather(2, idx[..., None].expand(-1, -1, -1, HEAD_DIM))
    assert torch.equal(k_kept, gather(k)) and torch.equal(v_kept, gather(v))
    assert k_kept.shape == (1, KV_HEADS, budget, HEAD_DIM)
    assert not keep[..., -32:].logical_not().any()  # the recent suffix is always kept
    # streaming_adapter.py:84-85: the dense output feeds o_proj for the next layer
    y = out.transpose(1, 2).contiguous().reshape(1, N, HIDDEN if HEADS * HEAD_DIM == HIDDEN else HEADS * HEAD_DIM)
    y = y @ layer["o"].T
    ref_y = torch.from_numpy(ref_out).to(torch.bfloat16).cuda().transpose(1, 2).reshape(1, N, -1) @ layer["o"].T
    torch.testing.assert_close(y.float(), ref_y.float(), atol=0.05, rtol=0.02)
