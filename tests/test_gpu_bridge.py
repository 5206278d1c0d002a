"""The patched EAGLE-3 attention forward end to end on a GPU: a stand-in
module with real bf16 projections and transformers-style repeat_kv (the host
module itself is not part of the reference), its verify step routed to the
kernel with the repeated kv-heads deduplicated, against a dense fp32
attention over the same cache and tree -- one tree for the batch (the
reference's behaviour) and one tree per batch element."""

import math
import types

import numpy as np
import pytest
import torch

import eagle_tree_sparse_bridge as br
import tsfa_trees as trees
from gpu_helpers import ATOL, OUT_REL

pytestmark = pytest.mark.gpu


def _module(hidden, Hq, Hkv, D):
    m = types.SimpleNamespace()

    class LlamaMutiRotaryEmbedding:  # not used: the plain rotary path below
        pass

    class Rotary:
        def __call__(self, x, seq_len=None):
            return torch.ones(1, device=x.device), torch.zeros(1, device=x.device)

    def apply_rotary_pos_emb(q, k, cos, sin, pos):
        return q, k  # identity position encoding: the test is about the attention

    def repeat_kv(x, n):  # transformers' layout: copy r of kv-head h at head h * n + r
        b, h, s, d = x.shape
        return x[:, :, None].expand(b, h, n, s, d).reshape(b, h * n, s, d)

    g = torch.Generator(device="cuda").manual_seed(7)

    def lin(i, o):
        w = (torch.randn((o, i), generator=g, device="cuda") / math.sqrt(i)).to(torch.bfloat16)
        return lambda x: x @ w.t()

    class Attn:
        def __init__(self):
            self.num_heads, self.num_key_value_heads, self.head_dim = Hq, Hkv, D
            self.num_key_value_groups = Hq // Hkv
            self.q_proj, self.k_proj, self.v_proj = lin(hidden, Hq * D), lin(hidden, Hkv * D), lin(hidden, Hkv * D)
            self.o_proj = lambda x: x  # the merged heads themselves are compared
            self.rotary_emb = Rotary()

        def forward(self, **kw):
            raise AssertionError("the verify step must not reach the module's own forward")

    m.LlamaMutiRotaryEmbedding = LlamaMutiRotaryEmbedding
    m.apply_rotary_pos_emb = apply_rotary_pos_emb
    m.repeat_kv = repeat_kv
    m.LlamaAttention = Attn
    return m


def _dense(q, k_full, v_full, add_mask):
    """fp32 softmax(q k^T / sqrt(D) + mask) v, heads merged: [B, Q, Hq * D]."""
    D = q.shape[-1]
    w = q.float() @ k_full.float().transpose(2, 3) / math.sqrt(D) + add_mask.float()
    o = torch.softmax(w, dim=-1) @ v_full.float()
    return o.transpose(1, 2).reshape(q.shape[0], q.shape[2], -1)


@pytest.mark.parametrize("per_batch", [False, True])
def test_patched_llama_attention_verify_step(per_batch):
    B, hidden, Hq, Hkv, D, prev, q_len = 2, 256, 8, 2, 128, 200, 24
    m = _module(hidden, Hq, Hkv, D)
    br.patch_llama_attention(m, block_m=16, block_n=16, per_batch_trees=per_batch)
    attn = m.LlamaAttention()
    g = torch.Generator(device="cuda").manual_seed(11)
    k0 = torch.randn((B, Hkv, prev, D), generator=g, device="cuda").to(torch.bfloat16)
    v0 = torch.randn((B, Hkv, prev, D), generator=g, device="cuda").to(torch.bfloat16)
    G = Hq // Hkv
    cache = [[m.repeat_kv(k0, G)], [m.repeat_kv(v0, G)]]
    h = torch.randn((B, q_len, hidden), generator=g, device="cuda").to(torch.bfloat16)
    masks = np.stack([trees.random_tree(q_len, 5, 3, seed=20 + b) for b in range(B)])
    if not per_batch:
        masks[1] = masks[0]  # one tree for the batch: the reference's case
    add = torch.zeros((B, 1, q_len, prev + q_len), device="cuda")
    add[:, 0, :, prev:] = torch.where(torch.from_numpy(masks).cuda(), 0.0, float("-inf"))

    out = attn.forward(hidden_states=h, cache_hidden=cache, attention_mask=add,
                       position_ids=torch.arange(q_len, device="cuda")[None])
    torch.cuda.synchronize()

    q = attn.q_proj(h).view(B, q_len, Hq, D).transpose(1, 2)
    k = attn.k_proj(h).view(B, q_len, Hkv, D).transpose(1, 2)
    v = attn.v_proj(h).view(B, q_len, Hkv, D).transpose(1, 2)
    k_full = torch.cat([m.repeat_kv(k0, G), m.repeat_kv(k, G)], dim=2)
    v_full = torch.cat([m.repeat_kv(v0, G), m.repeat_kv(v, G)], dim=2)
    want = _dense(q, k_full, v_full, add)
    assert out.shape == (B, q_len, Hq * D) and out.dtype == torch.bfloat16
    err = (out.float() - want).abs()
    tol = ATOL + OUT_REL[torch.bfloat16] * want.abs()
    assert bool((err <= tol).all()), f"max |err| {float(err.max()):.3e}"
    assert len(cache[0]) == 2 and cache[0][1].shape == (B, Hq, q_len, D)  # the module's cache layout is kept
