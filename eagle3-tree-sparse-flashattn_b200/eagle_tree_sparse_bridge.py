"""Drop-in for the reference module ``eagle_tree_sparse_bridge``.

* ``extract_tree_mask_from_attention_mask``  (bridge.py:24-70)
* ``run_tree_sparse_kernel``                 (bridge.py:76-159) -- the entry
  point of the verify-step attention; one dispatcher op
  (``torch.ops.tsfa.run_tree_sparse``, libtsfa ``tsfa_run_tree_sparse``)
  builds the block-CSR metadata on the GPU and runs the forward on the
  current stream, with no host round trip; torch.compile traces it as one op.
* ``patch_llama_flex_attention`` / ``patch_llama_attention`` /
  ``inject_tree_sparse_bridge`` / ``_fallback_to_original``
  (bridge.py:162-421) -- forward replacements for a user's EAGLE-3 Llama
  module that route the verify phase (q_len > 1 and a tree mask recoverable
  from the 4-D attention mask) to ``run_tree_sparse_kernel`` and leave every
  other path on the module's own code.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

import tsfa_native as _native
from tree_sparse_flashattn import block_sparse_tree_fwd_kernel, prepare_tree_sparse_metadata  # noqa: F401


# -----------------------------------------------------------------------------
# attention_mask [B, 1, Q, KV] -> tree_mask [Q, Q]
# -----------------------------------------------------------------------------
def extract_tree_mask_from_attention_mask(
    attention_mask: Optional[torch.Tensor],
    q_len: int,
    kv_len: int,
    *,
    batch_idx: int = 0,
) -> Optional[torch.Tensor]:
    """Tree-only bool mask (True = visible) from an HF/EAGLE 4-D mask.

    The last q_len key columns ``[kv_len - q_len, kv_len)`` of batch
    ``batch_idx`` are the tree part.  Floating masks are additive (0 visible,
    -inf hidden): visible = finite and >= 0.  Integer / bool masks: nonzero is
    visible.  Returns None when no tree mask can be recovered: no mask,
    q_len <= 1, not 4-D, too small, or kv_len < q_len.
    """
    if attention_mask is None or q_len <= 1 or attention_mask.ndim != 4:
        return None
    if attention_mask.shape[2] < q_len or attention_mask.shape[3] < kv_len:
        return None
    prefix_len = kv_len - q_len
    if prefix_len < 0:
        return None
    cols = attention_mask[batch_idx, 0, :q_len, :kv_len][:, prefix_len:prefix_len + q_len]
    if cols.shape != (q_len, q_len):
        return None
    if torch.is_floating_point(cols):
        visible = torch.isfinite(cols) & (cols >= 0)
    else:
        visible = cols.to(torch.bool)
    return visible.contiguous()


def extract_tree_masks_per_batch(
    attention_mask: Optional[torch.Tensor],
    q_len: int,
    kv_len: int,
) -> Optional[torch.Tensor]:
    """``extract_tree_mask_from_attention_mask`` for every batch element:
    a [B, q_len, q_len] bool mask (True = visible), element b from batch b of
    the 4-D mask.  No reference counterpart (the reference keeps batch 0's
    tree only).  None in the same cases as the single-tree extractor."""
    if attention_mask is None or q_len <= 1 or attention_mask.ndim != 4:
        return None
    if attention_mask.shape[2] < q_len or attention_mask.shape[3] < kv_len:
        return None
    prefix_len = kv_len - q_len
    if prefix_len < 0:
        return None
    cols = attention_mask[:, 0, :q_len, :kv_len][:, :, prefix_len:prefix_len + q_len]
    if cols.shape[1:] != (q_len, q_len):
        return None
    if torch.is_floating_point(cols):
        visible = torch.isfinite(cols) & (cols >= 0)
    else:
        visible = cols.to(torch.bool)
    return visible.contiguous()


# -----------------------------------------------------------------------------
# the verify-step attention
# -----------------------------------------------------------------------------
def _kernel_ready(t: torch.Tensor) -> torch.Tensor:
    """Unit stride on head_dim, 16-byte aligned rows (else one contiguous copy)."""
    ok = t.stride(-1) == 1 and all(s % 8 == 0 for s in t.stride()[:-1]) and t.data_ptr() % 16 == 0
    return t if ok else t.contiguous()


def run_tree_sparse_kernel(
    query_states: torch.Tensor,  # [B, Hq, Q, D]
    key_states: torch.Tensor,  # [B, Hkv, KV, D]
    value_states: torch.Tensor,  # [B, Hkv, KV, D]
    tree_mask: torch.Tensor,  # [Q, Q], nonzero = visible
    *,
    block_m: int,
    block_n: int,
) -> torch.Tensor:
    """softmax(Q K^T / sqrt(D)) V where each tree token sees the whole prefix
    [0, KV - Q) and the tree keys its row of ``tree_mask`` marks visible.
    Returns a new [B, Hq, Q, D] tensor in the query's dtype (bf16 or fp16)."""
    assert query_states.is_cuda and key_states.is_cuda and value_states.is_cuda
    bsz, num_heads, q_len, head_dim = query_states.shape
    b2, num_kv_heads, kv_len, d2 = key_states.shape
    assert bsz == b2 and head_dim == d2
    assert value_states.shape == key_states.shape
    assert num_heads % num_kv_heads == 0  # kv_h = h // G (bridge.py:115)
    for t in (query_states, key_states, value_states):
        _native.qkv_dtype_code(t)  # TypeError unless bf16 / fp16

    prefix_len = kv_len - q_len
    if prefix_len < 0:
        raise ValueError(f"Invalid lengths: kv_len={kv_len}, q_len={q_len}")
    if tree_mask.ndim != 2 or tree_mask.shape[0] != tree_mask.shape[1]:
        raise ValueError("tree_mask must be shape [q_len, q_len].")
    if tree_mask.shape[0] != q_len:
        raise ValueError(f"tree_mask is {tuple(tree_mask.shape)} but q_len={q_len}")
    if block_m <= 0 or block_n <= 0:
        raise ValueError("BLOCK_M and BLOCK_N must be positive.")

    device = query_states.device
    if tree_mask.device != device:
        tree_mask = tree_mask.to(device, non_blocking=True)
    q, k, v = query_states, key_states, value_states  # the op copies views TMA cannot read
    # one dispatcher op (libtsfa_torch.so over tsfa_run_tree_sparse): metadata
    # build + forward on the current stream; out = a new contiguous tensor, as
    # empty_like(q) at bridge.py:108
    return _native.load_torch_op().run_tree_sparse(q, k, v, tree_mask, prefix_len, block_m, block_n,
                                                   1.0 / math.sqrt(head_dim))


def run_tree_sparse_kernel_per_batch(
    query_states: torch.Tensor,  # [B, Hq, Q, D]
    key_states: torch.Tensor,  # [B, Hkv, KV, D]
    value_states: torch.Tensor,  # [B, Hkv, KV, D]
    tree_masks: torch.Tensor,  # [B, Q, Q], nonzero = visible
    *,
    block_m: int,
    block_n: int,
) -> torch.Tensor:
    """``run_tree_sparse_kernel`` with tree_masks[b] applied to batch element
    b (each request of a batch verifies its own draft tree).  No reference
    counterpart: the reference runs batch 0's tree for every element.  Same
    arguments, checks and exceptions otherwise."""
    assert query_states.is_cuda and key_states.is_cuda and value_states.is_cuda
    bsz, num_heads, q_len, head_dim = query_states.shape
    b2, num_kv_heads, kv_len, d2 = key_states.shape
    assert bsz == b2 and head_dim == d2
    assert value_states.shape == key_states.shape

    prefix_len = kv_len - q_len
    if prefix_len < 0:
        raise ValueError(f"Invalid lengths: kv_len={kv_len}, q_len={q_len}")
    if tree_masks.ndim != 3 or tree_masks.shape[1] != tree_masks.shape[2]:
        raise ValueError("tree_masks must be shape [batch, q_len, q_len].")
    if tree_masks.shape[0] != bsz or tree_masks.shape[1] != q_len:
        raise ValueError(f"tree_masks is {tuple(tree_masks.shape)} but batch={bsz}, q_len={q_len}")
    if block_m <= 0 or block_n <= 0:
        raise ValueError("BLOCK_M and BLOCK_N must be positive.")

    device = query_states.device
    if tree_masks.device != device:
        tree_masks = tree_masks.to(device, non_blocking=True)
    q = _kernel_ready(query_states)
    k = _kernel_ready(key_states)
    v = _kernel_ready(value_states)
    out = torch.empty_like(q, memory_format=torch.contiguous_format)
    with torch.cuda.device(device):
        _native.run_tree_sparse_batched(q, k, v, tree_masks, out, prefix_len=prefix_len, block_m=block_m,
                                        block_n=block_n, sm_scale=1.0 / math.sqrt(head_dim))
    return out


def run_tree_sparse_kernel_paged(
    query_states: torch.Tensor,  # [B, Hq, Q, D]
    k_pages: torch.Tensor,  # [num_pages, page_size, Hkv, D]
    v_pages: torch.Tensor,  # [num_pages, page_size, Hkv, D]
    page_indptr: torch.Tensor,  # [B + 1] int32
    page_indices: torch.Tensor,  # [page_indptr[B]] int32
    tree_mask: torch.Tensor,  # [Q, Q], nonzero = visible
    *,
    kv_len: int,
    block_m: int,
    block_n: int,
) -> torch.Tensor:
    """``run_tree_sparse_kernel`` over a paged K/V cache: key n of batch
    element b is token n % page_size of page
    page_indices[page_indptr[b] + n // page_size] of the pools, the last
    Q = tree_mask.shape[0] keys being the tree.  FlashInfer's
    [pages, 2, page_size, Hkv, D] cache is ``kv_cache[:, 0]`` / ``kv_cache[:, 1]``.
    page_size must be a power of two >= 8.  No reference counterpart: the
    reference concatenates the cache into contiguous K/V every step."""
    assert query_states.is_cuda and k_pages.is_cuda and v_pages.is_cuda
    bsz, num_heads, q_len, head_dim = query_states.shape
    assert k_pages.ndim == 4 and k_pages.shape == v_pages.shape and k_pages.shape[3] == head_dim
    assert page_indptr.shape == (bsz + 1,) and page_indptr.dtype == torch.int32 and page_indptr.is_cuda
    assert page_indices.dtype == torch.int32 and page_indices.is_cuda
    prefix_len = kv_len - q_len
    if prefix_len < 0:
        raise ValueError(f"Invalid lengths: kv_len={kv_len}, q_len={q_len}")
    if tree_mask.ndim != 2 or tree_mask.shape[0] != tree_mask.shape[1]:
        raise ValueError("tree_mask must be shape [q_len, q_len].")
    if tree_mask.shape[0] != q_len:
        raise ValueError(f"tree_mask is {tuple(tree_mask.shape)} but q_len={q_len}")
    if block_m <= 0 or block_n <= 0:
        raise ValueError("BLOCK_M and BLOCK_N must be positive.")
    device = query_states.device
    if tree_mask.device != device:
        tree_mask = tree_mask.to(device, non_blocking=True)
    q = _kernel_ready(query_states)
    out = torch.empty_like(q, memory_format=torch.contiguous_format)
    with torch.cuda.device(device):
        _native.run_tree_sparse_paged(q, k_pages, v_pages, page_indptr, page_indices, tree_mask, out,
                                      kv_len=kv_len, prefix_len=prefix_len, block_m=block_m, block_n=block_n,
                                      sm_scale=1.0 / math.sqrt(head_dim))
    return out


# -----------------------------------------------------------------------------
# forward patches for a user's EAGLE-3 Llama module
# -----------------------------------------------------------------------------
def _fallback_to_original(orig_forward, self, **kwargs):
    return orig_forward(self, **kwargs)


def _split_heads(x: torch.Tensor, bsz: int, q_len: int, heads: int, head_dim: int) -> torch.Tensor:
    return x.view(bsz, q_len, heads, head_dim).transpose(1, 2)


def _project(self, hidden_states: torch.Tensor):
    bsz, q_len, _ = hidden_states.size()
    q = _split_heads(self.q_proj(hidden_states), bsz, q_len, self.num_heads, self.head_dim)
    k = _split_heads(self.k_proj(hidden_states), bsz, q_len, self.num_key_value_heads, self.head_dim)
    v = _split_heads(self.v_proj(hidden_states), bsz, q_len, self.num_key_value_heads, self.head_dim)
    return q, k, v


def _rotate(self, llama_module, q, k, position_ids, offset: int, q_len: int):
    """RoPE as the host module applies it; returns (q, k, cos, sin)."""
    if isinstance(self.rotary_emb, llama_module.LlamaMutiRotaryEmbedding):
        cos, sin = self.rotary_emb(q, position_ids + offset)
        cos, sin = cos.to(q.device), sin.to(q.device)
        q, k = llama_module.apply_multimodal_rotary_pos_emb(q, k, cos, sin, self.config.rope_scaling["mrope_section"])
    else:
        cos, sin = self.rotary_emb(q, seq_len=q_len + offset)
        cos, sin = cos.to(q.device), sin.to(q.device)
        q, k = llama_module.apply_rotary_pos_emb(q, k, cos, sin, position_ids + offset)
    return q, k, cos, sin


def _merge_heads(self, attn: torch.Tensor, bsz: int, q_len: int) -> torch.Tensor:
    attn = attn.transpose(1, 2).contiguous().reshape(bsz, q_len, self.head_dim * self.num_heads)
    return self.o_proj(attn)


def _tree_dispatch(q, k_full, v_full, attention_mask, q_len: int, block_m: int, block_n: int,
                   per_batch_trees: bool = False):
    """run_tree_sparse_kernel on the verify phase, else None.  With
    per_batch_trees, every batch element's own tree from the 4-D mask
    (run_tree_sparse_kernel_per_batch); otherwise batch 0's, as the
    reference does."""
    kv_len = k_full.shape[-2]
    if per_batch_trees:
        tree_masks = extract_tree_masks_per_batch(attention_mask, q_len, kv_len)
        if q_len > 1 and tree_masks is not None and tree_masks.shape[0] == q.shape[0]:
            return run_tree_sparse_kernel_per_batch(q.contiguous(), k_full, v_full, tree_masks, block_m=block_m,
                                                    block_n=block_n)
        return None
    tree_mask = extract_tree_mask_from_attention_mask(attention_mask, q_len, kv_len)
    if q_len > 1 and tree_mask is not None:
        return run_tree_sparse_kernel(q.contiguous(), k_full, v_full, tree_mask, block_m=block_m, block_n=block_n)
    return None


def patch_llama_flex_attention(llama_module, *, block_m: int = 64, block_n: int = 64,
                               per_batch_trees: bool = False):
    """Route ``llama_module.LlamaFlexAttention.forward``'s verify phase to the
    tree-sparse kernel; other calls keep the module's flex_attention path.
    Idempotent."""
    cls = llama_module.LlamaFlexAttention
    if hasattr(cls, "_orig_forward_tree_sparse_bridge"):
        return
    cls._orig_forward_tree_sparse_bridge = cls.forward

    def forward(self, hidden_states, cache_hidden=None, attention_mask=None, position_ids=None,
                past_key_values=None, output_attentions=False, use_cache=False):
        bsz, q_len, _ = hidden_states.size()
        seen = past_key_values.get_seq_length() if past_key_values is not None else 0
        q, k, v = _project(self, hidden_states)
        lck = seen // q_len
        q, k, cos, sin = _rotate(self, llama_module, q, k, position_ids, lck, q_len)
        cache_position = torch.arange(seen, seen + q_len, device=hidden_states.device)
        key_cache, value_cache = past_key_values.update(
            k, v, layer_idx=0, cache_kwargs={"sin": sin, "cos": cos, "cache_position": cache_position})
        key_cache = key_cache.contiguous()
        value_cache = value_cache.contiguous()
        attn = _tree_dispatch(q, key_cache, value_cache, attention_mask, q_len, block_m, block_n, per_batch_trees)
        if attn is None:  # the module's own flex-attention path
            kv_len = key_cache.shape[-2]
            seq_lengths = attention_mask.sum(dim=-1)
            seq_lengths -= lck
            if q_len <= 128:
                make_mask, flex = llama_module.create_block_mask, llama_module.flex_attention
            else:
                make_mask = llama_module.compile_friendly_create_block_mask
                flex = llama_module.compile_friendly_flex_attention
            block_mask = make_mask(
                mask_mod=llama_module.generate_eagle3_mask(seq_lengths=seq_lengths, Q_LEN=q_len, KV_LEN=kv_len,
                                                           lck=lck),
                B=bsz, H=1, Q_LEN=q_len, KV_LEN=kv_len, device=q.device)
            attn = flex(query=q, key=key_cache, value=value_cache, block_mask=block_mask, enable_gqa=True)
        return _merge_heads(self, attn, bsz, q_len)

    cls.forward = forward


def patch_llama_attention(llama_module, *, block_m: int = 64, block_n: int = 64, per_batch_trees: bool = False):
    """Route ``llama_module.LlamaAttention.forward``'s cache_hidden branch to the
    tree-sparse kernel on the verify phase.  Idempotent.

    The module caches K/V after ``repeat_kv`` (copy r of kv-head h at head
    h * G + r, as transformers' repeat_kv lays them out), so its cache holds
    every kv-head G times.  The kernel is given one copy per group -- the
    strided view ``[:, ::G]`` of each cached step, concatenated -- and folds
    the G query heads of a kv-head as usual: G times fewer K/V bytes read and
    copied than handing it the repeated heads (the reference concatenates and
    reads all of them, bridge.py:357-373)."""
    cls = llama_module.LlamaAttention
    if hasattr(cls, "_orig_forward_tree_sparse_bridge"):
        return
    cls._orig_forward_tree_sparse_bridge = cls.forward

    def forward(self, hidden_states, cache_hidden=None, attention_mask=None, position_ids=None,
                past_key_values=None, output_attentions=False, use_cache=False):
        if cache_hidden is None:
            return _fallback_to_original(
                cls._orig_forward_tree_sparse_bridge, self, hidden_states=hidden_states, cache_hidden=cache_hidden,
                attention_mask=attention_mask, position_ids=position_ids, past_key_values=past_key_values,
                output_attentions=output_attentions, use_cache=use_cache)
        bsz, q_len, _ = hidden_states.size()
        q, k, v = _project(self, hidden_states)
        lck = len(cache_hidden[0])
        q, k, _, _ = _rotate(self, llama_module, q, k, position_ids, lck, q_len)
        k = llama_module.repeat_kv(k, self.num_key_value_groups)
        v = llama_module.repeat_kv(v, self.num_key_value_groups)
        cache_hidden[0] = cache_hidden[0] + [k]
        cache_hidden[1] = cache_hidden[1] + [v]
        groups = self.num_key_value_groups
        full_k = torch.cat([c[:, ::groups] for c in cache_hidden[0]], dim=2)
        full_v = torch.cat([c[:, ::groups] for c in cache_hidden[1]], dim=2)
        attn = _tree_dispatch(q, full_k, full_v, attention_mask, q_len, block_m, block_n, per_batch_trees)
        if attn is None:  # the module's own manual softmax over cached steps
            scale = math.sqrt(self.head_dim)
            k0, v0 = cache_hidden[0][0], cache_hidden[1][0]
            weights = torch.matmul(q, k0.transpose(2, 3)) / scale
            if attention_mask is not None:
                weights = weights + attention_mask
            steps = len(cache_hidden[0])
            extra = [((q * cache_hidden[0][i]).sum(-1) / scale)[..., None] for i in range(1, steps)]
            if extra:
                weights = torch.cat([weights, *extra], dim=-1)
            weights = torch.nn.functional.softmax(weights, dim=-1, dtype=torch.float32).to(q.dtype)
            attn = torch.matmul(weights[..., :q_len], v0)
            for i in range(1, steps):
                attn = attn + weights[..., q_len + i - 1][..., None] * cache_hidden[1][i]
        return _merge_heads(self, attn, bsz, q_len)

    cls.forward = forward


def inject_tree_sparse_bridge(llama_module, *, block_m: int = 64, block_n: int = 64, per_batch_trees: bool = False):
    """Install both patches (LlamaFlexAttention and LlamaAttention).
    per_batch_trees (an extension; default off, the reference's behaviour):
    each batch element verifies its own tree from the 4-D attention mask."""
    patch_llama_flex_attention(llama_module, block_m=block_m, block_n=block_n, per_batch_trees=per_batch_trees)
    patch_llama_attention(llama_module, block_m=block_m, block_n=block_n, per_batch_trees=per_batch_trees)
