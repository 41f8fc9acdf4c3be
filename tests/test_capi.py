"""The C ABI boundary without a GPU: the library loads, exports what include/cg_b200.h declares,
answers its pure-host queries, rejects bad arguments with a message, and refuses CPU tensors."""

from __future__ import annotations

import ctypes
import re

import pytest
import torch

from card_playing_gym_b200 import _native as nat
from card_playing_gym_b200.config import RL_V6
from tests.conftest import ROOT


@pytest.fixture(scope="module", autouse=True)
def library():
    if not nat.LIBRARY.exists():
        from card_playing_gym_b200.build import build

        build()
    return nat.lib()


def declared() -> list[str]:
    header = (ROOT / "include" / "cg_b200.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:const char\*|int64_t|int)\s+(cg_[a-z0-9_]+)\s*\(", header, re.M)))


def test_every_declared_entry_point_is_exported_and_bound():
    names = declared()
    assert len(names) >= 25
    lib = ctypes.CDLL(str(nat.LIBRARY))
    for name in names:
        assert hasattr(lib, name), name
    assert sorted(nat.declared_symbols()) == names


def test_version_and_pure_host_queries():
    from card_playing_gym_b200.trunk import trunk_dims

    assert nat.lib().cg_version() >= 1
    dims = trunk_dims(RL_V6.trunk())
    total = nat.query("cg_trunk_blob_bytes", dims)
    offsets = []
    for part in range(14):
        for layer in range(16 if part >= nat.CG_PART_LN_ATTN_W else 1):
            offset = nat.lib().cg_trunk_part_offset(dims, part, layer)
            if offset >= 0:
                offsets.append(offset)
                assert offset % 256 == 0
                assert offset < total
    assert len(set(offsets)) == len(offsets)
    # bf16 rollout workspace of the bench configuration: 16,384 rows, one token each
    assert nat.query("cg_plump_step_workspace_bytes", dims, 16384, 1, nat.CG_PREC_BF16) > 0
    assert nat.query("cg_ppo_objective_workspace_bytes", 262144) > 0


def test_bad_arguments_return_a_message():
    status = nat.lib().cg_decode_attention(None, 0, None, None, 0, 0, 0, 0, None, None, 4, 10, 3, 1, 24, 8, 1.0,
                                           None, 0, None)
    assert status == 1  # CG_ERR_ARGUMENT
    assert b"kv_heads" in nat.lib().cg_last_error()
    with pytest.raises(nat.NativeError, match="width"):
        nat.call("cg_masked_sample", None, None, None, 4, 0, None, None, None)


def test_cpu_tensors_are_refused():
    from card_playing_gym_b200.cuda_decode import decode_attention

    q = torch.zeros(2, 10, 1, 24)
    k = torch.zeros(2, 2, 8, 24)
    with pytest.raises(ValueError, match="CUDA"):
        decode_attention(q, k, k, torch.zeros(2, dtype=torch.int64), torch.ones(2, dtype=torch.int64), 8, 0.2)


def test_a_replaced_workspace_stays_alive():
    """A captured graph keeps the address of the workspace it ran with; growing the workspace must not free it."""

    device = torch.device("cpu", 0)
    small = nat.Workspace.get(device, 1000, "test-retire")
    address = small.data_ptr()
    del small
    large = nat.Workspace.get(device, 5000, "test-retire")
    assert large.numel() >= 5000 and large.data_ptr() != address
    assert any(t.data_ptr() == address for t in nat.Workspace._retired)
    assert nat.Workspace.get(device, 4000, "test-retire").data_ptr() == large.data_ptr()
