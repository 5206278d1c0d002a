"""Generate the golden fixtures by running the reference implementation itself.

Run in a container where the reference checkout is available:

    python tests/golden/gen_golden.py --reference <path to the reference checkout>

It imports the reference's ``tree_sparse_flashattn.prepare_tree_sparse_metadata``
/ ``_pack_block_mask_to_int32`` (tsfa.py:44-160), ``benchmark.torch_baseline_tree_attention``
(benchmark.py:8-35) and ``eagle_tree_sparse_bridge.extract_tree_mask_from_attention_mask``
(bridge.py:24-70), runs them on CPU on seeded inputs and writes
``tests/golden/*.npz``.  The fixtures are committed; the tests and the GPU box
never need the reference.
"""

from __future__ import annotations

import argparse
import hashlib
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "eagle3-tree-sparse-flashattn_b200"))
import tsfa_trees as trees  # noqa: E402


def _load(ref_dir: str, name: str):
    """Import a reference module under its own name (benchmark.py imports
    tree_sparse_flashattn by name)."""
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    return importlib.import_module(name)


def meta_cases():
    """(case_id, mask ndarray, BM, BN, prefix_len)."""
    cases = []
    c2 = trees.CONFIGS["cfg2_llama3_8b"]
    c3 = trees.CONFIGS["cfg3_serving_70b"]
    c4 = trees.CONFIGS["cfg4_long_ctx"]
    t2 = trees.config_tree(c2, seed=0)
    for bm, bn in [(64, 64), (16, 16), (32, 32), (128, 128), (16, 64), (64, 16)]:
        cases.append((f"cfg2_tree_{bm}x{bn}", t2, bm, bn, 4096))
    cases.append(("cfg3_tree_64x64", trees.config_tree(c3, seed=0), 64, 64, 8192))
    cases.append(("cfg3_tree_16x16", trees.config_tree(c3, seed=0), 16, 16, 8192))
    cases.append(("cfg4_tree_64x64", trees.config_tree(c4, seed=0), 64, 64, 32768))
    cases.append(("cfg1_tree_64x64", trees.config_tree(trees.CONFIGS["cfg1_cpu"], seed=0), 64, 64, 512))
    for T in (64, 100):
        for bm, bn in [(16, 16), (64, 64), (16, 32), (32, 16)]:
            cases.append((f"chain{T}_{bm}x{bn}", trees.chain_tree(T), bm, bn, 7))
    cases.append(("star64_16x16", trees.star_tree(64), 16, 16, 0))
    cases.append(("star100_32x32", trees.star_tree(100), 32, 32, 3))
    cases.append(("ones40_16x16", np.ones((40, 40), np.bool_), 16, 16, 5))      # FULL + clipped, no MIXED
    cases.append(("ones64_64x64", np.ones((64, 64), np.bool_), 64, 64, 5))
    cases.append(("eye50_8x8", np.eye(50, dtype=np.bool_), 8, 8, 1))
    cases.append(("zeros20_8x8", np.zeros((20, 20), np.bool_), 8, 8, 1))      # nnz == 0
    cases.append(("single_64x64", np.ones((1, 1), np.bool_), 64, 64, 9))
    cases.append(("empty_0", np.zeros((0, 0), np.bool_), 16, 16, 4))
    cases.append(("chain9_4x4", trees.chain_tree(9), 4, 4, 2))                 # W = 1, bits < 32
    cases.append(("tree13_3x5", trees.random_tree(13, 4, 3, seed=3), 3, 5, 2))
    cases.append(("tree10_1x1", trees.random_tree(10, 4, 3, seed=4), 1, 1, 0))
    cases.append(("tree21_2x8", trees.random_tree(21, 5, 2, seed=5), 2, 8, 0))
    cases.append(("tree37_8x4", trees.random_tree(37, 5, 3, seed=6), 8, 4, 0))
    cases.append(("tree40_5x7", trees.random_tree(40, 6, 3, seed=7), 5, 7, 0))
    cases.append(("causal_sparse64_16x16", trees.random_causal_sparse(64, seed=42), 16, 16, 1024))
    cases.append(("causal_sparse64_64x64", trees.random_causal_sparse(64, seed=43), 64, 64, 1024))
    for T, bm in [(512, 32), (512, 128), (1024, 16), (1024, 64)]:
        cases.append((f"tree{T}_{bm}x{bm}", trees.random_tree(T, 10, 6, seed=T + bm), bm, bm, 1024))
        cases.append((f"chain{T}_{bm}x{bm}", trees.chain_tree(T), bm, bm, 0))
        cases.append((f"star{T}_{bm}x{bm}", trees.star_tree(T), bm, bm, 16384))
    return cases


def typed_mask_cases():
    """Non-bool masks: the reference converts with .to(torch.bool) (tsfa.py:90)."""
    base = trees.random_tree(48, 5, 3, seed=11)
    rng = np.random.default_rng(12)
    out = []
    vals = rng.integers(1, 100, size=base.shape).astype(np.int32) * base
    out.append(("int32_48_16x16", vals.astype(np.int32), 16, 16))
    f = np.where(base, rng.standard_normal(base.shape) + 3.0, 0.0).astype(np.float32)
    f[0, 5] = -0.0             # negative zero is invisible
    f[7, 9] = np.nan           # NaN is visible
    out.append(("float32_48_16x16", f, 16, 16))
    out.append(("int64_48_32x32", base.astype(np.int64) * -5, 32, 32))
    out.append(("uint8_48_64x64", base.astype(np.uint8) * 255, 64, 64))
    return out


def attn_cases():
    """(case_id, B, Hq, Hkv, D, P, mask)."""
    return [
        ("small_tree", 1, 4, 2, 64, 32, trees.random_tree(16, 4, 3, seed=1)),
        ("gqa4_star", 2, 8, 2, 128, 70, trees.star_tree(24)),
        ("tree_only_chain", 1, 4, 1, 64, 0, trees.chain_tree(16)),
        ("g1_causal_sparse", 1, 2, 2, 64, 128, trees.random_causal_sparse(33, seed=9)),
        ("gqa8_tree40", 1, 16, 2, 128, 200, trees.random_tree(40, 6, 4, seed=2)),
    ]


def metadata_digest(arrays) -> bytes:
    """SHA-256 over the five metadata arrays in the reference's order
    (row_ptr, col_idx, blk_type, mixed_mask_payload, mixed_mask_offset), each
    preceded by its length and its dtype: equal digests mean equal values,
    dtypes and shapes.  The GPU and oracle tests hash their output the same way."""
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(np.array([a.size], np.int64).tobytes())
        h.update(str(a.dtype).encode())
        h.update(a.tobytes())
    return h.digest()


def mask_digest(mask) -> bytes:
    m = np.ascontiguousarray(np.asarray(mask, dtype=np.bool_))
    return hashlib.sha256(np.array(m.shape, np.int64).tobytes() + m.tobytes()).digest()


def sweep5(ref) -> dict:
    """Reference metadata digests at every (tree size, tree, BLOCK_M, BLOCK_N)
    point of the sparsity / tiling sweep."""
    out = {}
    ids = []
    s = trees.SWEEP5
    for T in s["T"]:
        for kind in trees.SWEEP5_TREES:
            mask = trees.sweep5_tree(kind, T)
            out[f"T{T}_{kind}.mask_sha256"] = np.frombuffer(mask_digest(mask), np.uint8)
            out[f"T{T}_{kind}.visible_fraction"] = np.array(float(mask.mean()))
            for bm in s["BLOCKS"]:
                for bn in s["BLOCKS"]:
                    md = ref.prepare_tree_sparse_metadata(torch.from_numpy(mask), 0, bm, bn)
                    cid = f"T{T}_{kind}_{bm}x{bn}"
                    ids.append(cid)
                    arrs = [getattr(md, f).numpy() for f in ("row_ptr", "col_idx", "blk_type", "mixed_mask_payload",
                                                              "mixed_mask_offset")]
                    out[f"{cid}.sha256"] = np.frombuffer(metadata_digest(arrs), np.uint8)
                    n_mixed = int((arrs[2] == 1).sum())
                    out[f"{cid}.counts"] = np.array([arrs[1].size, n_mixed, md.n_q_blocks, md.n_tree_blocks], np.int64)
    out["__ids__"] = np.array(ids)
    return out


def bf16_randn(shape, gen):
    return torch.randn(shape, generator=gen, dtype=torch.float32).to(torch.bfloat16).to(torch.float32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--parts", default="all", help="comma list of: core (the original fixtures), sweep5")
    args = ap.parse_args()
    parts = {"core", "sweep5"} if args.parts == "all" else set(args.parts.split(","))
    ref = _load(args.reference, "tree_sparse_flashattn")
    bm_mod = _load(args.reference, "benchmark")
    bridge = _load(args.reference, "eagle_tree_sparse_bridge")

    if "sweep5" in parts:
        np.savez_compressed(os.path.join(HERE, "sweep5_golden.npz"), **sweep5(ref))
    if "core" not in parts:
        print("wrote fixtures to", HERE)
        return

    # -- metadata ---------------------------------------------------------
    blob = {}
    ids = []
    for cid, mask, bm, bn, P in meta_cases() + [(c, m, a, b, 3) for c, m, a, b in typed_mask_cases()]:
        md = ref.prepare_tree_sparse_metadata(torch.from_numpy(np.ascontiguousarray(mask)), P, bm, bn)
        ids.append(cid)
        blob[f"{cid}.mask"] = mask
        blob[f"{cid}.params"] = np.array([bm, bn, P, md.n_q_blocks, md.n_tree_blocks], np.int64)
        for f in ("row_ptr", "col_idx", "blk_type", "mixed_mask_payload", "mixed_mask_offset"):
            t = getattr(md, f)
            blob[f"{cid}.{f}"] = t.numpy()
        h = hashlib.sha256()
        for f in ("row_ptr", "col_idx", "blk_type", "mixed_mask_payload", "mixed_mask_offset"):
            h.update(getattr(md, f).numpy().tobytes())
        blob[f"{cid}.sha256"] = np.frombuffer(h.digest(), np.uint8)
    blob["__ids__"] = np.array(ids)
    np.savez_compressed(os.path.join(HERE, "meta_golden.npz"), **blob)

    # -- bit packing of single tiles (tsfa.py:44-64) ---------------------------
    rng = np.random.default_rng(5)
    pack = {}
    for i, (r, c) in enumerate([(1, 1), (4, 4), (3, 5), (8, 4), (16, 16), (64, 64), (1, 31), (1, 33), (2, 32)]):
        tile = rng.random((r, c)) > 0.5
        if i == 4:
            tile[:] = True  # every bit set: bit 31 words become -1
        pack[f"t{i}.tile"] = tile
        pack[f"t{i}.words"] = ref._pack_block_mask_to_int32(torch.from_numpy(tile)).numpy()
    np.savez_compressed(os.path.join(HERE, "pack_golden.npz"), **pack)

    # -- dense attention (benchmark.py:8-35) ------------------------------------
    attn = {}
    aids = []
    for i, (cid, B, Hq, Hkv, D, P, mask) in enumerate(attn_cases()):
        T = mask.shape[0]
        gen = torch.Generator().manual_seed(1000 + i)
        q = bf16_randn((B, Hq, T, D), gen)
        k = bf16_randn((B, Hkv, P + T, D), gen)
        v = bf16_randn((B, Hkv, P + T, D), gen)
        out = bm_mod.torch_baseline_tree_attention(q, k, v, torch.from_numpy(mask), P)
        aids.append(cid)
        # Inputs are regenerated from the seed by the tests (torch's CPU
        # generator is deterministic); only their shapes and the seed are kept.
        attn[f"{cid}.seed"] = np.array(1000 + i)
        attn[f"{cid}.shape"] = np.array([B, Hq, Hkv, D, P, T])
        attn[f"{cid}.mask"] = mask
        attn[f"{cid}.prefix_len"] = np.array(P)
        attn[f"{cid}.out"] = out.numpy()
    # A tree-only row that sees nothing -> NaN (tsfa.py:329 has no l == 0 guard).
    mask = trees.chain_tree(12)
    mask[5, :] = False
    gen = torch.Generator().manual_seed(77)
    q = bf16_randn((1, 2, 12, 64), gen)
    k = bf16_randn((1, 1, 12, 64), gen)
    v = bf16_randn((1, 1, 12, 64), gen)
    out = bm_mod.torch_baseline_tree_attention(q, k, v, torch.from_numpy(mask), 0)
    aids.append("empty_row_nan")
    attn["empty_row_nan.seed"] = np.array(77)
    attn["empty_row_nan.shape"] = np.array([1, 2, 1, 64, 0, 12])
    attn["empty_row_nan.out"] = out.numpy()
    attn["empty_row_nan.mask"] = mask
    attn["empty_row_nan.prefix_len"] = np.array(0)
    attn["__ids__"] = np.array(aids)
    np.savez_compressed(os.path.join(HERE, "attn_golden.npz"), **attn)

    # -- config 1 output on a strided sample ---------------
    c1 = trees.CONFIGS["cfg1_cpu"]
    mask = trees.config_tree(c1, seed=0)
    gen = torch.Generator().manual_seed(1)
    q = bf16_randn((c1["B"], c1["Hq"], c1["T"], c1["D"]), gen)
    k = bf16_randn((c1["B"], c1["Hkv"], c1["P"] + c1["T"], c1["D"]), gen)
    v = bf16_randn((c1["B"], c1["Hkv"], c1["P"] + c1["T"], c1["D"]), gen)
    out = bm_mod.torch_baseline_tree_attention(q, k, v, torch.from_numpy(mask), c1["P"]).numpy()
    np.savez_compressed(os.path.join(HERE, "cfg1_golden.npz"), mask=mask, out_sample=out.reshape(-1)[::17],
                        q_sum=np.array(q.double().sum().item()), seed=np.array(1))

    # -- 4D attention mask -> tree mask (bridge.py:24-70) ------------------------
    ext = {}
    T, P = 10, 6
    tm = trees.random_tree(T, 4, 3, seed=8)
    add = np.zeros((2, 1, T, P + T), np.float32)
    add[:, 0, :, P:] = np.where(tm, 0.0, -np.inf)
    add[1, 0, :, P:] = np.where(trees.chain_tree(T), 0.0, -np.inf)  # batch 1 differs, ignored
    cases = {
        "float_additive": (add, T, P + T),
        "bool": (np.concatenate([np.ones((2, 1, T, P), np.bool_), np.broadcast_to(tm, (2, 1, T, T))], -1), T, P + T),
        "int": (np.concatenate([np.ones((1, 1, T, P), np.int64), tm[None, None].astype(np.int64) * 3], -1), T, P + T),
        "q1": (add, 1, P + 1),
        "not4d": (add[0], T, P + T),
        "short_kv": (add, T, P + T + 1),
        "neg_prefix": (add, T, T - 1),
        "bigger_mask": (np.pad(add, ((0, 0), (0, 0), (0, 2), (0, 3)), constant_values=-np.inf), T, P + T),
    }
    for name, (m, ql, kl) in cases.items():
        res = bridge.extract_tree_mask_from_attention_mask(torch.from_numpy(np.ascontiguousarray(m)), ql, kl)
        ext[f"{name}.in"] = m
        ext[f"{name}.q_len"] = np.array(ql)
        ext[f"{name}.kv_len"] = np.array(kl)
        ext[f"{name}.none"] = np.array(res is None)
        ext[f"{name}.out"] = np.zeros((0, 0), np.bool_) if res is None else res.numpy()
    np.savez_compressed(os.path.join(HERE, "extract_golden.npz"), **ext)
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
