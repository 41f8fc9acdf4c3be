"""Ragged GQA decode attention straight from the KV pool, as a torch custom op.

Drop-in for the reference's ``cardgym.nn.cuda_decode`` (cardgym/nn/cuda_decode.py:172-202):
``decode_attention(q, k_cache, v_cache, rows, key_lengths, span, scale)`` with q
[B, H, T, D], k/v [R, KVH, L, D]; query t of row b sees keys < key_lengths[b] + t
(capped at ``span``). Returns [B, H, T, D] in the cache's dtype, like the reference.
Beyond the reference's head_dim 32 / span 64 limits (cuda_decode.py:31-32,184-185),
this op takes head_dim up to 128, any span up to L, fp16/bf16/fp32 caches.
"""

from __future__ import annotations

import torch

from . import _native as nat


@torch.library.custom_op("cardgym_b200::decode_attention", mutates_args=())
def _decode_attention(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, rows: torch.Tensor, lengths: torch.Tensor, span: int, scale: float
) -> torch.Tensor:
    if k.stride() != v.stride() or k.stride(3) != 1:
        raise ValueError("k and v must share strides with a contiguous head dimension")
    if rows.dtype != torch.int64 or lengths.dtype != torch.int64:
        raise ValueError("rows and lengths must be int64")
    out = torch.empty_like(q)
    batch, heads, steps, dim = q.shape
    nat.call(
        "cg_decode_attention", nat.ptr(q), nat.DTYPE_CODES[q.dtype], nat.ptr(k), nat.ptr(v), nat.DTYPE_CODES[k.dtype],
        k.stride(0), k.stride(1), k.stride(2), nat.ptr(rows.contiguous()), nat.ptr(lengths.contiguous()), batch, heads,
        k.shape[1], steps, dim, int(span), float(scale), nat.ptr(out), nat.DTYPE_CODES[out.dtype],
        nat.stream_handle(q.device),
    )
    return out


@_decode_attention.register_fake
def _(q, k, v, rows, lengths, span, scale):
    return torch.empty_like(q)


def supported(head_dim: int, span: int, queries: int) -> bool:
    """Shapes this op takes (reference: head_dim 32 and span <= 64 only)."""

    return head_dim <= 128 and span >= 0


def decode_attention(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    rows: torch.Tensor,
    key_lengths: torch.Tensor,
    span: int,
    scale: float,
) -> torch.Tensor:
    """q [B, H, T, D] against cache rows ``rows`` [B] of k/v [R, KVH, L, D]; returns [B, H, T, D] in the cache dtype."""

    return _decode_attention(q.to(k_cache.dtype).contiguous(), k_cache, v_cache, rows, key_lengths, span, scale)
