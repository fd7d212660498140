"""StreamingController on a whole (small, random-init) transformers Qwen2 model.

The reference's streaming adapter (flash_evict/streaming_adapter.py:17-31,
57-87) compacts every layer's K/V during prefill while the dense attention
output feeds the next layer.  Checked here on a 2-layer Qwen2 (4 query heads,
2 KV heads, head_dim 128) with a ragged 1500-token prompt:
  * backend 'full' reproduces the uncompressed transformers model (prefill
    logits and decoding over its own cache);
  * 'fused' and 'snap' give the same prefill logits bit for bit as 'full'
    (only the stored K/V differ), and every layer stores exactly the rows of
    its K/V that the library's selection of that layer's scores keeps;
  * decoding then grows each compacted cache by one row per token.
"""
import numpy as np
import pytest
import torch

from common import selection_mismatch
from flash_evict import prefill, select_tokens, gather_tokens
from flash_evict.baselines import snap_scores, snap_select
from flash_evict.streaming_adapter import StreamingController
from oracle import restate as O

pytestmark = pytest.mark.gpu

N, LAYERS, HEADS, KV_HEADS, HEAD_DIM = 1500, 2, 4, 2, 128


@pytest.fixture(scope="module")
def model():
    from transformers import Qwen2Config, Qwen2ForCausalLM
    torch.manual_seed(0)
    cfg = Qwen2Config(vocab_size=512, hidden_size=HEADS * HEAD_DIM, intermediate_size=1024,
                      num_hidden_layers=LAYERS, num_attention_heads=HEADS, num_key_value_heads=KV_HEADS,
                      head_dim=HEAD_DIM, max_position_embeddings=4 * N, initializer_range=0.1)
    m = Qwen2ForCausalLM(cfg).to(torch.bfloat16).cuda().eval()
    return m


@pytest.fixture(scope="module")
def prompt():
    g = torch.Generator().manual_seed(1)
    return torch.randint(0, 512, (1, N), generator=g).cuda()


def _qkv(attn, kw):
    # The projections of the patched forward, recomputed from a hook's inputs.
    from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb
    h = kw["hidden_states"]
    b, n, _ = h.shape
    q = attn.q_proj(h).view(b, n, HEADS, HEAD_DIM).transpose(1, 2)
    k = attn.k_proj(h).view(b, n, KV_HEADS, HEAD_DIM).transpose(1, 2)
    v = attn.v_proj(h).view(b, n, KV_HEADS, HEAD_DIM).transpose(1, 2)
    cos, sin = kw["position_embeddings"]
    q, k = apply_rotary_pos_emb(q, k, cos, sin)
    return q, k, v


def _run(model, prompt, decode_tokens=(), capture=False, **ctl_kwargs):
    ctl = StreamingController(model, **ctl_kwargs)
    captured, hooks = {}, []
    if capture:
        for layer in model.model.layers:
            attn = layer.self_attn

            def hook(mod, args, kwargs, output, attn=attn):
                if ctl.mode == "prefill":
                    captured[attn.layer_idx] = _qkv(attn, kwargs)
            hooks.append(attn.register_forward_hook(hook, with_kwargs=True))
    try:
        with torch.no_grad():
            logits = [model(prompt, use_cache=False).logits[:, -1].float()]
            ctl.finish_prefill()
            for i, tok in enumerate(decode_tokens):
                pos = torch.tensor([[N + i]], device=prompt.device)
                logits.append(model(tok.view(1, 1), position_ids=pos, use_cache=False).logits[:, -1].float())
                for state in ctl.states.values():
                    assert state["k"].shape[2] == state["v"].shape[2]
        states = {i: dict(s) for i, s in ctl.states.items()}
    finally:
        for hnd in hooks:
            hnd.remove()
        ctl.restore()
    return logits, states, captured


def test_full_backend_matches_the_uncompressed_model(model, prompt):
    with torch.no_grad():
        out = model(prompt, use_cache=True)
        ref = [out.logits[:, -1].float()]
        past = out.past_key_values
        toks = []
        for i in range(4):
            tok = ref[-1].argmax(-1)
            toks.append(tok)
            step = model(tok.view(1, 1), past_key_values=past, use_cache=True)
            past = step.past_key_values
            ref.append(step.logits[:, -1].float())
    got, states, _ = _run(model, prompt, decode_tokens=toks, backend="full", budget=4 * N)
    scale = ref[0].abs().max().item()
    for a, b in zip(got, ref):
        torch.testing.assert_close(a, b, atol=0.03 * scale, rtol=0.03)
    assert all(s["k"].shape[2] == N + 4 for s in states.values())


@pytest.mark.parametrize("backend", ["fused", "snap"])
def test_compacting_backends(model, prompt, backend):
    budget, reserved = 256, 64
    full_logits, full_states, captured = _run(model, prompt, capture=True, backend="full", budget=4 * N)
    toks = [full_logits[0].argmax(-1)] * 3
    scoring = {"recency_decay": 0.1} if backend == "fused" else {}
    got, states, _ = _run(model, prompt, decode_tokens=toks, backend=backend, budget=budget,
                          reserved_recent=reserved, scoring=scoring)
    # Dense outputs feed the next layer: prefill logits equal bit for bit.
    assert torch.equal(got[0], full_logits[0])
    for layer, (q, k, v) in captured.items():
        state = states[layer]
        if backend == "fused":
            _, imp = prefill(q, k, v, **scoring)
            idx, keep = select_tokens(imp, budget, reserved_recent=reserved)
            if layer == 0:
                ref_out, ref_imp = O.materialized(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                                  v.float().cpu().numpy(), recency_decay=0.1)
                np.testing.assert_allclose(imp.cpu().numpy(), ref_imp, atol=3e-3, rtol=3e-4)
                _, ref_keep = O.select_tokens(ref_imp, budget, reserved_recent=reserved)
                _, ok = selection_mismatch(keep.cpu().numpy(), ref_keep, imp.cpu().numpy(), ref_imp, 3e-3, 3e-4)
                assert ok
        else:
            idx, _ = snap_select(snap_scores(q, k, 32), budget, 32)
        assert torch.equal(state["indices"], idx)
        assert torch.all(idx[..., -32:] == torch.arange(N - 32, N, device=idx.device))
        kept = state["k"].shape[2]
        assert kept == budget + len(toks)
        assert torch.equal(state["k"][:, :, :budget], gather_tokens(full_states[layer]["k"], idx))
        assert torch.equal(state["v"][:, :, :budget], gather_tokens(full_states[layer]["v"], idx))
    assert all(torch.isfinite(x).all() for x in got)


def test_budget_at_prompt_length_decodes_like_the_dense_model(model, prompt):
    # With nothing evicted the compacted cache is the whole cache: decoding
    # must agree with the uncompressed model.
    full, _, _ = _run(model, prompt, decode_tokens=[torch.tensor([7], device="cuda")] * 2, backend="full",
                      budget=4 * N)
    got, states, _ = _run(model, prompt, decode_tokens=[torch.tensor([7], device="cuda")] * 2, backend="fused",
                          budget=N, reserved_recent=64)
    for a, b in zip(got, full):
        assert torch.equal(a, b)
    assert all(s["k"].shape[2] == N + 2 for s in states.values())
