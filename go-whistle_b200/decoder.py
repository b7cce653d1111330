"""The decoder head's scale and greedy choice on the B200 library:
``logits`` (internal/decoder/decoder.go:508-523, the head scale) and
``argmax`` (internal/decoder/greedy.go:182) for rows of vocabulary logits in
device memory, so a greedy decode step brings back one token id per stream.
"""

from __future__ import annotations

import ctypes

from ._lib import Panic, WC_ERR_INVALID, check, lib

__all__ = ["HeadArgmax"]


def HeadArgmax(y, rows: int, vocab: int, head: float = 1.0, logits=None, idx=None):
    """idx[r] = argmax over row r of y·head (y·head only when head != 1; the
    first index of the largest value, a NaN at 0 gives 0). y, logits (None,
    or y itself for the reference's in-place scale) and idx are CUDA tensors
    (float32 [rows·vocab], int32 [rows]); returns idx."""
    import torch

    if rows < 0 or vocab < 0 or y.numel() != rows * vocab:
        raise Panic(WC_ERR_INVALID, f"decoder: head of {rows} rows of {vocab} logits on {y.numel()} values")
    for t in (y, logits):
        if t is not None and (not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous()):
            raise Panic(WC_ERR_INVALID, "decoder: logits must be contiguous float32 CUDA tensors")
    if idx is None:
        idx = torch.empty(rows, dtype=torch.int32, device=y.device)
    if logits is not None and logits.numel() != rows * vocab:
        raise Panic(WC_ERR_INVALID, f"decoder: {logits.numel()} logits for {rows} rows of {vocab}")
    if idx.numel() != rows or idx.dtype != torch.int32 or not idx.is_cuda:
        raise Panic(WC_ERR_INVALID, "decoder: idx must be an int32 CUDA tensor of one entry per row")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    check(lib().wc_head_argmax(ctypes.c_void_p(y.data_ptr()), rows, vocab, float(head),
                               ctypes.c_void_p(logits.data_ptr()) if logits is not None else None,
                               ctypes.c_void_p(idx.data_ptr()), stream))
    return idx
