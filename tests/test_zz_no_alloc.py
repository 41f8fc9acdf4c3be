"""The allocation-free KV row copy, checked against the workspace-based one (B200 only).

cg_kv_copy_rows_noalloc serves callers that cannot allocate device memory around a copy
(a collector loop that must not synchronize the device through cudaMalloc, or a host that
drives the C ABI without an allocator of its own): it stages rows through a fixed buffer
inside the library. This file is collected last so that a stop-at-first-failure run has
already run every other test when it reaches these.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from card_playing_gym_b200 import _native as nat
from card_playing_gym_b200.kv_cache import KVCache

pytestmark = pytest.mark.gpu


def noalloc_copy(cache: KVCache, sources: torch.Tensor, targets: torch.Tensor, length: int) -> None:
    nat.call(
        "cg_kv_copy_rows_noalloc", nat.ptr(cache.k_pool), nat.ptr(cache.v_pool), nat.DTYPE_CODES[cache.dtype],
        cache.n_layers, cache.capacity, cache.kv_heads, cache.max_len, cache.head_dim, nat.ptr(sources),
        nat.ptr(targets), int(sources.shape[0]), int(length), nat.stream_handle(cache.device),
    )


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_noalloc_copy_matches_the_workspace_copy_twice_in_a_row(dtype):
    layers, kv_heads, head_dim, capacity, max_len = 4, 2, 24, 40, 33
    generator = torch.Generator(device="cuda").manual_seed(5)
    reference = KVCache(n_layers=layers, kv_heads=kv_heads, head_dim=head_dim, capacity=capacity, max_len=max_len,
                        device="cuda", dtype=dtype)
    reference.k_pool.normal_(generator=generator)
    reference.v_pool.normal_(generator=generator)
    mine = KVCache(n_layers=layers, kv_heads=kv_heads, head_dim=head_dim, capacity=capacity, max_len=max_len,
                   device="cuda", dtype=dtype)
    mine.k_pool.copy_(reference.k_pool)
    mine.v_pool.copy_(reference.v_pool)
    # Two calls in a row; the first slides survivors down (a row is both a source and a
    # target), the second moves rows the other way with another length.
    plans = [([3, 7, 8, 12], [2, 3, 4, 5], 17), ([30, 2, 9], [31, 20, 10], 33)]
    for sources, targets, length in plans:
        src = torch.tensor(sources, dtype=torch.int64, device="cuda")
        dst = torch.tensor(targets, dtype=torch.int64, device="cuda")
        reference.copy_rows(src, dst, length)
        noalloc_copy(mine, src, dst, length)
        torch.cuda.synchronize()
        assert torch.equal(mine.k_pool, reference.k_pool)
        assert torch.equal(mine.v_pool, reference.v_pool)


def test_noalloc_copy_rejects_copies_above_its_fixed_buffer():
    limit = nat.query("cg_kv_copy_rows_noalloc_max_bytes")
    assert limit == 16 << 20
    cache = KVCache(n_layers=16, kv_heads=2, head_dim=24, capacity=64, max_len=257, device="cuda",
                    dtype=torch.float16)
    cache.k_pool.normal_()
    cache.v_pool.normal_()
    rows = torch.arange(64, dtype=torch.int64, device="cuda")
    # 64 rows x 257 positions x 16 layers x 2 (K, V) x 2 heads x 24 x 2 bytes = 50.5 MB > 16 MiB
    with pytest.raises(nat.NativeError, match="split the copy"):
        noalloc_copy(cache, rows, rows.flip(0), 257)
    noalloc_copy(cache, rows[:4], rows[4:8], 257)  # 3.2 MB: within the limit
    torch.cuda.synchronize()
    assert torch.equal(cache.k_pool[:, 4:8], cache.k_pool[:, :4])
    assert torch.equal(cache.v_pool[:, 4:8], cache.v_pool[:, :4])
