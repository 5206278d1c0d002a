"""Host-side behaviour of the drop-in modules (no GPU): argument validation,
the attention-mask helper, and the forward patches' dispatch on a mock module."""

import types

import numpy as np
import pytest
import torch

import eagle_tree_sparse_bridge as br
import tree_sparse_flashattn as tsfa
from conftest import load_npz


def test_constants_and_fields():
    assert tsfa.FULL_BLOCK == 0 and tsfa.MIXED_BLOCK == 1
    fields = [f for f in tsfa.TreeSparseMetadata.__dataclass_fields__]
    assert fields == ["row_ptr", "col_idx", "blk_type", "mixed_mask_payload", "mixed_mask_offset",
                      "n_q_blocks", "n_tree_blocks", "block_m", "block_n", "prefix_len"]


@pytest.mark.parametrize("shape", [(3, 4), (3,), (2, 2, 2)])
def test_prepare_rejects_non_square(shape):
    with pytest.raises(ValueError, match=r"tree_mask must be shape \[q_len, q_len\]"):
        tsfa.prepare_tree_sparse_metadata(torch.ones(shape, dtype=torch.bool), 0, 16, 16)


@pytest.mark.parametrize("bm,bn", [(0, 16), (16, 0), (-4, 4)])
def test_prepare_rejects_bad_blocks(bm, bn):
    with pytest.raises(ValueError, match="BLOCK_M and BLOCK_N must be positive"):
        tsfa.prepare_tree_sparse_metadata(torch.ones(4, 4, dtype=torch.bool), 0, bm, bn)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU error path")
def test_no_cpu_fallback():
    with pytest.raises(RuntimeError, match="CUDA"):
        tsfa.prepare_tree_sparse_metadata(torch.ones(4, 4, dtype=torch.bool), 0, 4, 4)
    with pytest.raises(RuntimeError, match="CUDA"):
        tsfa._pack_block_mask_to_int32(torch.ones(4, 4, dtype=torch.bool))


def test_run_requires_cuda_tensors():
    q = torch.zeros(1, 2, 4, 64, dtype=torch.bfloat16)
    with pytest.raises(AssertionError):
        br.run_tree_sparse_kernel(q, q, q, torch.ones(4, 4, dtype=torch.bool), block_m=4, block_n=4)


def test_extract_tree_mask_matches_reference():
    g = load_npz("extract_golden.npz")
    names = sorted({k.split(".")[0] for k in g.files})
    for n in names:
        got = br.extract_tree_mask_from_attention_mask(torch.from_numpy(g[f"{n}.in"]), int(g[f"{n}.q_len"]),
                                                       int(g[f"{n}.kv_len"]))
        if bool(g[f"{n}.none"]):
            assert got is None, n
        else:
            assert got.dtype == torch.bool and np.array_equal(got.numpy(), g[f"{n}.out"]), n
    assert br.extract_tree_mask_from_attention_mask(None, 4, 8) is None


# ---------------------------------------------------------------- patches
class _Linear:
    def __init__(self, n_out):
        self.n_out = n_out

    def __call__(self, x):
        return torch.zeros(*x.shape[:-1], self.n_out)


def _mock_module(calls):
    m = types.SimpleNamespace()

    class LlamaMutiRotaryEmbedding:  # never instantiated here
        pass

    class Rotary:
        def __call__(self, x, seq_len=None):
            return torch.ones(1), torch.zeros(1)

    def apply_rotary_pos_emb(q, k, cos, sin, pos):
        calls.append("rope")
        return q, k

    def repeat_kv(x, n):
        return x.repeat_interleave(n, dim=1)

    class Attn:
        def __init__(self):
            self.num_heads, self.num_key_value_heads, self.head_dim = 4, 2, 8
            self.num_key_value_groups = 2
            self.q_proj, self.k_proj, self.v_proj = _Linear(32), _Linear(16), _Linear(16)
            self.o_proj = lambda x: x
            self.rotary_emb = Rotary()

        def forward(self, **kw):
            calls.append("original")
            return "orig"

    m.LlamaMutiRotaryEmbedding = LlamaMutiRotaryEmbedding
    m.apply_rotary_pos_emb = apply_rotary_pos_emb
    m.repeat_kv = repeat_kv
    m.LlamaAttention = Attn
    m.LlamaFlexAttention = type("LlamaFlexAttention", (Attn,), {})
    return m


def test_patches_are_idempotent_and_keep_fallback(monkeypatch):
    calls = []
    m = _mock_module(calls)
    orig = m.LlamaAttention.forward
    br.inject_tree_sparse_bridge(m, block_m=16, block_n=16)
    patched = m.LlamaAttention.forward
    br.inject_tree_sparse_bridge(m)  # second install is a no-op
    assert m.LlamaAttention.forward is patched
    assert m.LlamaAttention._orig_forward_tree_sparse_bridge is orig
    # no cache_hidden -> the module's own forward
    out = m.LlamaAttention().forward(hidden_states=torch.zeros(1, 3, 32))
    assert out == "orig" and calls == ["original"]


def test_patch_routes_verify_phase_to_kernel(monkeypatch):
    calls = []
    m = _mock_module(calls)
    br.patch_llama_attention(m, block_m=16, block_n=32)
    seen = {}

    def fake_kernel(q, k, v, tree_mask, *, block_m, block_n):
        seen.update(q=q.shape, k=k.shape, k_prefix=k[:, :, :5].clone(), v_prefix=v[:, :, :5].clone(),
                    mask=tree_mask.clone(), bm=block_m, bn=block_n)
        return torch.zeros_like(q)

    monkeypatch.setattr(br, "run_tree_sparse_kernel", fake_kernel)
    q_len, prev = 3, 5
    attn = m.LlamaAttention()
    g = torch.Generator().manual_seed(0)
    k0 = torch.randn((1, 2, prev, 8), generator=g)
    v0 = torch.randn((1, 2, prev, 8), generator=g)
    cache = [[m.repeat_kv(k0, 2)], [m.repeat_kv(v0, 2)]]
    tree = torch.tensor([[1, 0, 0], [1, 1, 0], [1, 0, 1]], dtype=torch.bool)
    am = torch.full((1, 1, q_len, prev + q_len), float("-inf"))
    am[..., :prev] = 0
    am[0, 0, :, prev:] = torch.where(tree, 0.0, float("-inf"))
    out = attn.forward(hidden_states=torch.zeros(1, q_len, 32), cache_hidden=cache, attention_mask=am,
                       position_ids=torch.arange(q_len)[None])
    assert out.shape == (1, q_len, 32)
    # the kernel gets one copy of each repeated kv-head: G = 2, Hkv = 2
    assert seen["q"] == (1, 4, 3, 8) and seen["k"] == (1, 2, prev + q_len, 8)
    assert torch.equal(seen["k_prefix"], k0) and torch.equal(seen["v_prefix"], v0)
    assert torch.equal(seen["mask"], tree) and (seen["bm"], seen["bn"]) == (16, 32)


def test_extract_tree_masks_per_batch_matches_single_extractor():
    """Every batch element's tree, each equal to the single-tree extractor's
    answer for that batch index; None in the same cases."""
    B, T, P = 3, 12, 5
    g = torch.Generator().manual_seed(3)
    vis = torch.rand((B, T, T), generator=g) > 0.5
    add = torch.zeros((B, 1, T, P + T))
    add[:, 0, :, P:] = torch.where(vis, 0.0, float("-inf"))
    got = br.extract_tree_masks_per_batch(add, T, P + T)
    assert got.shape == (B, T, T) and got.dtype == torch.bool
    for b in range(B):
        assert torch.equal(got[b], br.extract_tree_mask_from_attention_mask(add, T, P + T, batch_idx=b))
    ints = add.isfinite().to(torch.int32)
    assert torch.equal(br.extract_tree_masks_per_batch(ints, T, P + T)[:, :, :], ints[:, 0, :T, P:].to(torch.bool))
    assert br.extract_tree_masks_per_batch(None, T, P + T) is None
    assert br.extract_tree_masks_per_batch(add, 1, P + 1) is None
    assert br.extract_tree_masks_per_batch(add[:, 0], T, P + T) is None
    assert br.extract_tree_masks_per_batch(add, T, T - 1) is None
