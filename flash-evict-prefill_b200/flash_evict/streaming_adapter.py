"""Per-layer prefill-and-compact on a transformers Qwen2 model.

Mirrors the reference's streaming adapter (flash_evict/streaming_adapter.py:
`StreamingController` :17-31, `chunk_mlp` :34-54, the patched attention
forward :57-87) for the Qwen2 attention modules of the installed transformers
(5.x, where the decoder layer hands each attention module its rotary
`position_embeddings`).  The reference builds on the external kv_distill
Controller (its prefill/decode modes, per-layer `states`, and decoding over
the compacted cache); that package is not available, so this controller keeps
those pieces itself:

* prefill (``mode == 'prefill'``), one unpadded prompt, no external cache:
  each layer projects q/k/v, views them ``[B,N,H,D]`` and transposes them
  (no copy; the kernels read the strided views), applies RoPE, and then
    - ``'fused'``: ``prefill(q, k, v, **scoring)`` for the dense output and the
      importance, then one launch that selects ``min(N, budget)`` tokens with
      ``reserved_recent`` pinned and ``pool_kernel`` pooling and gathers the
      kept K/V rows (streaming_adapter.py:61-66,86);
    - ``'snap'``: dense attention, SnapKV window-32 scores and selection, gather
      (streaming_adapter.py:78-83,86);
    - ``'full'``: dense attention, the whole K/V kept.
  The dense attention output always feeds ``o_proj``: only the stored K/V are
  compacted, so the next layer sees exactly the uncompressed model's input.
* decode (after ``finish_prefill()``): every new token's K/V is appended to its
  layer's stored K/V and its query attends to all of them (plus the new tokens
  before it); positions continue from the caller's ``position_ids``.  Decode
  attention is torch's ``scaled_dot_product_attention`` (a library call: one
  query row per step is not this package's hot path).

The model is called with ``use_cache=False``; the controller owns the cache
(``states[layer_idx] = {'k', 'v', 'indices'}``).
"""
import types

import torch
import torch.nn.functional as F

from .baselines import flash_attention, snap_scores, snap_select
from .compact import gather_tokens, select_and_gather
from .prefill import prefill

__all__ = ["StreamingController", "chunk_mlp"]


def _attention_modules(model):
    return [layer.self_attn for layer in model.model.layers]


class StreamingController:
    """Compact every layer's K/V cache during prefill (streaming_adapter.py:17-31).

    Same keyword arguments, defaults and ValueErrors as the reference's
    ``StreamingController``.  ``scoring`` is passed to ``prefill`` as keyword
    arguments (e.g. ``{'recency_decay': 0.1}``).  ``restore()`` puts the
    model's original attention forwards back.
    """

    def __init__(self, model, *, backend="fused", budget=1024, scoring=None, reserved_recent=64, pool_kernel=1):
        if backend not in ("fused", "snap", "full"):
            raise ValueError("Unsupported backend")
        if isinstance(budget, bool) or not isinstance(budget, int) or budget < 1:
            raise ValueError("Positive integer budget required")
        self.model = model
        self.prefill_backend = backend
        self.cache_budget = budget
        self.scoring = {} if scoring is None else dict(scoring)
        self.reserved_recent = reserved_recent
        self.pool_kernel = pool_kernel
        self.mode = "prefill"
        self.states = {}
        self.originals = [(attn, attn.forward) for attn in _attention_modules(model)]
        for attn, _ in self.originals:
            attn._kv_controller = self
            attn.forward = types.MethodType(_forward, attn)

    def finish_prefill(self):
        """Switch to decoding over the compacted caches (streaming_adapter.py:29-30)."""
        self.mode = "decode"

    def reset(self):
        """Drop every cache and return to prefill mode for the next prompt."""
        self.mode = "prefill"
        self.states = {}

    def restore(self):
        """Give the attention modules their original forward back."""
        for attn, original in self.originals:
            attn.forward = original
            if hasattr(attn, "_kv_controller"):
                del attn._kv_controller
        self.originals = []


def chunk_mlp(model, chunk_size):
    """Run every layer's feed-forward block on at most ``chunk_size`` tokens at a time.

    Bounds the activation memory of inference on long prompts; returns a
    function that restores the original MLP forwards (streaming_adapter.py:34-54).
    The GEMM shapes change, so results may differ in the last bits.
    """
    if isinstance(chunk_size, bool) or not isinstance(chunk_size, int) or chunk_size < 1:
        raise ValueError("chunk_size must be a positive integer")
    saved = []

    def chunked_forward(original):
        def run(hidden):
            if torch.is_grad_enabled():
                raise RuntimeError("Chunked MLP is inference-only")
            n = hidden.shape[1]
            if n <= chunk_size:
                return original(hidden)
            out = torch.empty_like(hidden)
            for start in range(0, n, chunk_size):
                out[:, start:start + chunk_size] = original(hidden[:, start:start + chunk_size])
            return out
        return run

    for layer in model.model.layers:
        saved.append((layer.mlp, layer.mlp.forward))
        layer.mlp.forward = chunked_forward(layer.mlp.forward)

    def restore():
        for mlp, original in saved:
            mlp.forward = original

    return restore


def _decode_attention(q, k, v, scale):
    # q [B,Hq,n,D] are the newest n positions of the Hkv-headed k/v [B,Hkv,L,D].
    n, total = q.shape[2], k.shape[2]
    mask = None
    if n > 1:
        qpos = torch.arange(total - n, total, device=q.device)[:, None]
        mask = torch.arange(total, device=q.device)[None, :] <= qpos
    return F.scaled_dot_product_attention(q, k, v, attn_mask=mask, scale=scale, enable_gqa=True)


def _forward(self, hidden_states, position_embeddings=None, attention_mask=None, past_key_values=None, **kwargs):
    """Attention forward installed by StreamingController (streaming_adapter.py:57-87)."""
    ctl = self._kv_controller
    b, n, _ = hidden_states.shape
    if b != 1 or past_key_values is not None or kwargs.get("output_attentions"):
        raise ValueError("Streaming adapter expects one unpadded prompt and an empty external cache")
    if position_embeddings is None:
        raise ValueError("Streaming adapter needs the rotary position_embeddings of the decoder layer")
    from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb

    hq, hk, d = self.config.num_attention_heads, self.config.num_key_value_heads, self.head_dim
    q = self.q_proj(hidden_states).view(b, n, hq, d).transpose(1, 2)
    k = self.k_proj(hidden_states).view(b, n, hk, d).transpose(1, 2)
    v = self.v_proj(hidden_states).view(b, n, hk, d).transpose(1, 2)
    cos, sin = position_embeddings
    q, k = apply_rotary_pos_emb(q, k, cos, sin)

    if ctl.mode == "prefill":
        budget = min(n, ctl.cache_budget)
        if ctl.prefill_backend == "fused":
            out, importance = prefill(q, k, v, **ctl.scoring)
            idx, _, k_kept, v_kept = select_and_gather(importance, budget, k, v,
                                                       reserved_recent=min(budget, ctl.reserved_recent),
                                                       pool_kernel=ctl.pool_kernel)
        elif ctl.prefill_backend == "snap":
            out = flash_attention(q, k, v)
            idx, _ = snap_select(snap_scores(q, k, 32), budget, 32)
            k_kept, v_kept = gather_tokens(k, idx), gather_tokens(v, idx)
        else:
            out = flash_attention(q, k, v)
            idx, k_kept, v_kept = None, k, v
        ctl.states[self.layer_idx] = {"k": k_kept, "v": v_kept, "indices": idx}
    else:
        state = ctl.states[self.layer_idx]
        state["k"] = torch.cat([state["k"], k], dim=2)
        state["v"] = torch.cat([state["v"], v], dim=2)
        out = _decode_attention(q, state["k"], state["v"], self.scaling)
    out = out.transpose(1, 2).reshape(b, n, hq * d)
    return self.o_proj(out), None
