"""Drop-in for the reference module ``tree_sparse_flashattn`` (metadata protocol
and forward kernel), backed by libtsfa.so on B200.

Public surface, same names and argument meaning as the reference
(tree_sparse_flashattn.py):

* ``FULL_BLOCK`` / ``MIXED_BLOCK``                  (tsfa.py:11-12)
* ``TreeSparseMetadata``                            (tsfa.py:15-41)
* ``_pack_block_mask_to_int32(mask_2d)``            (tsfa.py:44-64)
* ``prepare_tree_sparse_metadata(tree_mask, prefix_len, BLOCK_M, BLOCK_N)``
                                                    (tsfa.py:67-160)
* ``block_sparse_tree_fwd_kernel[grid](...)``       (tsfa.py:163-339): a
  launcher object taking the reference's 35 positional arguments plus the
  BLOCK_M / BLOCK_N / BLOCK_D constexprs; ``grid``, ``num_warps`` and
  ``num_stages`` are accepted and ignored (the native kernel plans its own
  launch).

The metadata is built on the GPU (kernel K1 in libtsfa.so) and is bit-exact
with the reference builder.  Tensors come back on the mask's device: a CPU mask
is copied to the current CUDA device, processed there, and the result copied
back, so CPU callers see the reference's CPU tensors.  Without a CUDA device
these functions raise; nothing here computes on the CPU.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

import tsfa_native as _native

FULL_BLOCK = 0
MIXED_BLOCK = 1


@dataclass
class TreeSparseMetadata:
    """Block-CSR description of the tree part of the mask.

    row_ptr            int32 [n_q_blocks + 1]  CSR row pointer over q-blocks
    col_idx            int32 [nnz]             tree block column of each entry
    blk_type           int8  [nnz]             FULL_BLOCK (0) or MIXED_BLOCK (1)
    mixed_mask_payload int32 [n_mixed * W]     row-major bitsets of MIXED tiles
    mixed_mask_offset  int32 [nnz]             payload offset per entry (0 for
                                               FULL); empty when n_mixed == 0
    n_q_blocks, n_tree_blocks, block_m, block_n, prefix_len  (ints)
    """

    row_ptr: torch.Tensor
    col_idx: torch.Tensor
    blk_type: torch.Tensor
    mixed_mask_payload: torch.Tensor
    mixed_mask_offset: torch.Tensor
    n_q_blocks: int
    n_tree_blocks: int
    block_m: int
    block_n: int
    prefix_len: int


def _on_cuda(t: torch.Tensor) -> tuple[torch.Tensor, torch.device | None]:
    """(tensor on a CUDA device, original device if it had to move)."""
    if t.is_cuda:
        _native.require_cuda(t.device)
        return t, None
    dev = _native.require_cuda(None)
    return t.to(dev), t.device


def _pack_block_mask_to_int32(mask_2d: torch.Tensor) -> torch.Tensor:
    """Pack a [BLOCK_M, BLOCK_N] mask into int32 words, row-major: bit i % 32
    of word i // 32 is flat[i] with i = r * BLOCK_N + c (bit 31 is the sign)."""
    tile, back = _on_cuda(mask_2d)
    out = _native.pack_tile_device(tile)
    return out.to(back) if back is not None else out


def prepare_tree_sparse_metadata(
    tree_mask: torch.Tensor,
    prefix_len: int,
    BLOCK_M: int,
    BLOCK_N: int,
) -> TreeSparseMetadata:
    """CSR + tri-state (ZERO dropped / FULL / MIXED) metadata of a [q_len, q_len]
    tree mask tiled in BLOCK_M x BLOCK_N blocks.  Any nonzero mask value is
    visible.  Raises ValueError for a non-square mask or a non-positive block
    size, like the reference."""
    if tree_mask.ndim != 2 or tree_mask.shape[0] != tree_mask.shape[1]:
        raise ValueError("tree_mask must be shape [q_len, q_len].")
    if BLOCK_M <= 0 or BLOCK_N <= 0:
        raise ValueError("BLOCK_M and BLOCK_N must be positive.")
    mask, back = _on_cuda(tree_mask)
    d = _native.meta_dims(mask.shape[0], BLOCK_M, BLOCK_N)
    # K1 through the dispatcher op (fixed-capacity buffers, counts on the
    # device), then one device -> host read of (nnz, n_mixed) to cut the
    # tensors to the reference's exact sizes
    row_ptr, col_idx, blk_type, payload, offset, counts = _native.load_torch_op().build_metadata(
        mask, BLOCK_M, BLOCK_N)
    nnz, n_mixed = (int(x) for x in counts.tolist())
    W = int(d.words_per_tile)
    col_idx = col_idx[:nnz]
    blk_type = blk_type[:nnz]
    if n_mixed:
        payload = payload[: n_mixed * W]
        offset = offset[:nnz]
    else:  # the reference returns empty payload AND empty offsets here (tsfa.py:145-147)
        payload = payload[:0]
        offset = offset[:0]
    fields = [row_ptr, col_idx, blk_type, payload, offset]
    if back is not None:
        fields = [f.to(back) for f in fields]
    return TreeSparseMetadata(*fields, n_q_blocks=int(d.n_q_blocks), n_tree_blocks=int(d.n_tree_blocks),
                              block_m=BLOCK_M, block_n=BLOCK_N, prefix_len=prefix_len)


class _Meta:
    __slots__ = ("row_ptr", "col_idx", "blk_type", "mixed_mask_payload", "mixed_mask_offset",
                 "n_q_blocks", "n_tree_blocks", "block_m", "block_n")


class _BlockSparseTreeFwdKernel:
    """``block_sparse_tree_fwd_kernel[grid](*args, BLOCK_M=, BLOCK_N=, BLOCK_D=)``.

    Accepts the reference's launch (tsfa.py:164-203; benchmark.py:183-194):
    q, k, v, o, the five metadata tensors, 16 element strides, sm_scale,
    batch_size, num_heads, num_kv_heads, q_len, kv_len, prefix_len,
    n_q_blocks, n_tree_blocks, gqa_group_size.  Runs the native forward on the
    current stream of q's device.
    """

    def __getitem__(self, grid):
        return self._launch

    @staticmethod
    def _launch(q_ptr, k_ptr, v_ptr, o_ptr, row_ptr_ptr, col_idx_ptr, blk_type_ptr,
                mixed_mask_payload_ptr, mixed_mask_offset_ptr,
                stride_qb, stride_qh, stride_qm, stride_qd,
                stride_kb, stride_kh, stride_kn, stride_kd,
                stride_vb, stride_vh, stride_vn, stride_vd,
                stride_ob, stride_oh, stride_om, stride_od,
                sm_scale, batch_size, num_heads, num_kv_heads, q_len, kv_len, prefix_len,
                n_q_blocks, n_tree_blocks, gqa_group_size,
                BLOCK_M=None, BLOCK_N=None, BLOCK_D=None, num_warps=None, num_stages=None, **_unused):
        for t in (q_ptr, k_ptr, v_ptr, o_ptr):
            assert t.is_cuda
        if BLOCK_M is None or BLOCK_N is None or BLOCK_D is None:
            raise TypeError("BLOCK_M, BLOCK_N and BLOCK_D are required")
        if int(BLOCK_D) != q_ptr.shape[-1]:
            raise ValueError(f"BLOCK_D={BLOCK_D} must equal head_dim={q_ptr.shape[-1]}")
        if int(gqa_group_size) * int(num_kv_heads) != int(num_heads):
            raise ValueError("gqa_group_size * num_kv_heads must equal num_heads")
        if o_ptr.dtype != q_ptr.dtype:
            raise TypeError("output must have the dtype of the query")
        m = _Meta()
        m.row_ptr, m.col_idx, m.blk_type = row_ptr_ptr, col_idx_ptr, blk_type_ptr
        m.mixed_mask_payload, m.mixed_mask_offset = mixed_mask_payload_ptr, mixed_mask_offset_ptr
        m.n_q_blocks, m.n_tree_blocks, m.block_m, m.block_n = int(n_q_blocks), int(n_tree_blocks), int(BLOCK_M), int(BLOCK_N)
        a = _native.fwd_args(q_ptr, k_ptr, v_ptr, o_ptr, prefix_len=int(prefix_len), sm_scale=float(sm_scale), meta=m)
        a.q_stride[:] = (stride_qb, stride_qh, stride_qm, stride_qd)
        a.k_stride[:] = (stride_kb, stride_kh, stride_kn, stride_kd)
        a.v_stride[:] = (stride_vb, stride_vh, stride_vn, stride_vd)
        a.o_stride[:] = (stride_ob, stride_oh, stride_om, stride_od)
        a.batch, a.num_heads, a.num_kv_heads = int(batch_size), int(num_heads), int(num_kv_heads)
        a.q_len, a.kv_len = int(q_len), int(kv_len)
        _native.launch_fwd_args(a, q_ptr.device)


block_sparse_tree_fwd_kernel = _BlockSparseTreeFwdKernel()
