"""ctypes binding of the C ABI in include/cg_b200.h (libcg_b200.so, built in-tree).

The product path has no fallback: a missing library, a CPU tensor or a failed
kernel raises. ``lib()`` loads the library once per process.
"""

from __future__ import annotations

import ctypes
from functools import lru_cache
from pathlib import Path

import torch

LIBRARY = Path(__file__).resolve().parent / "libcg_b200.so"

CG_F32, CG_F16, CG_BF16 = 0, 1, 2
CG_I16, CG_I32, CG_I64 = 16, 32, 64
CG_PREC_FP32, CG_PREC_BF16 = 0, 1
(CG_PART_INPUT_NORM, CG_PART_PLE_CONTEXT, CG_PART_FINAL_W, CG_PART_FINAL_B, CG_PART_LN_ATTN_W, CG_PART_LN_ATTN_B,
 CG_PART_QKV, CG_PART_OUT, CG_PART_LN_MLP_W, CG_PART_LN_MLP_B, CG_PART_UP, CG_PART_UP_B, CG_PART_DOWN,
 CG_PART_DOWN_B) = range(14)

DTYPE_CODES = {torch.float32: CG_F32, torch.float16: CG_F16, torch.bfloat16: CG_BF16}
INDEX_CODES = {torch.int16: CG_I16, torch.int32: CG_I32, torch.int64: CG_I64}
PRECISIONS = {"fp32": CG_PREC_FP32, "bf16": CG_PREC_BF16}

_p = ctypes.c_void_p
_i32 = ctypes.c_int
_i64 = ctypes.c_int64
_f32 = ctypes.c_float
_f64 = ctypes.c_double


class TrunkDims(ctypes.Structure):
    _fields_ = [
        ("d_model", ctypes.c_int32), ("n_layers", ctypes.c_int32), ("n_heads", ctypes.c_int32),
        ("n_kv_heads", ctypes.c_int32), ("d_ff", ctypes.c_int32), ("per_layer_dim", ctypes.c_int32),
        ("input_norm", ctypes.c_int32), ("reserved", ctypes.c_int32), ("value_layers", ctypes.c_uint64),
    ]


class PlumpSchemaC(ctypes.Structure):
    _fields_ = [
        ("field_count", ctypes.c_int32), ("field_slots", ctypes.c_int32 * 16), ("field_offsets", ctypes.c_int32 * 16),
        ("field_na", ctypes.c_int32 * 16), ("field_rows", ctypes.c_int32), ("pattern_rows", ctypes.c_int32),
        ("token_width", ctypes.c_int32), ("slot_type", ctypes.c_int32), ("slot_pattern", ctypes.c_int32),
        ("slot_hand", ctypes.c_int32), ("hand_slots", ctypes.c_int32), ("trick_win_type", ctypes.c_int32),
        ("rank_offset", ctypes.c_int32), ("suit_offset", ctypes.c_int32), ("num_cards", ctypes.c_int32),
        ("num_ranks", ctypes.c_int32),
    ]


class HeadsDesc(ctypes.Structure):
    _fields_ = [
        ("d_model", ctypes.c_int32), ("n_policy", ctypes.c_int32), ("value_outputs", ctypes.c_int32),
        ("max_width", ctypes.c_int32), ("width", ctypes.c_int32 * 8), ("weight_offset", ctypes.c_int64 * 8),
        ("bias_offset", ctypes.c_int64 * 8), ("value_w1", ctypes.c_int64), ("value_b1", ctypes.c_int64),
        ("value_w2", ctypes.c_int64), ("value_b2", ctypes.c_int64),
    ]


class CardScorerWeights(ctypes.Structure):
    _fields_ = [
        ("d_model", ctypes.c_int32), ("card_width", ctypes.c_int32), ("dim", ctypes.c_int32), ("cards", ctypes.c_int32),
        ("query_w", ctypes.c_void_p), ("query_b", ctypes.c_void_p), ("card_w", ctypes.c_void_p),
        ("card_id", ctypes.c_void_p), ("norm_w", ctypes.c_void_p), ("norm_b", ctypes.c_void_p),
        ("hidden_w", ctypes.c_void_p), ("hidden_b", ctypes.c_void_p), ("out_w", ctypes.c_void_p),
        ("out_b", ctypes.c_void_p),
    ]


class CandidateScorerWeights(ctypes.Structure):
    _fields_ = [
        ("d_model", ctypes.c_int32), ("card_width", ctypes.c_int32), ("dim", ctypes.c_int32), ("cards", ctypes.c_int32),
        ("kinds", ctypes.c_int32), ("sizes", ctypes.c_int32),
    ] + [(name, ctypes.c_void_p) for name in (
        "query_w", "query_b", "card_w", "target_w", "taken_w", "card_id", "target_id", "taken_id", "kind_emb",
        "size_emb", "norm_w", "norm_b", "hidden_w", "hidden_b", "out_w", "out_b")]


class CardGridWeights(ctypes.Structure):
    _fields_ = [
        ("width", ctypes.c_int32), ("hidden", ctypes.c_int32), ("kernel", ctypes.c_int32), ("blocks", ctypes.c_int32),
        ("codes", ctypes.c_int32), ("ranks", ctypes.c_int32), ("circular", ctypes.c_int32),
        ("code_emb", ctypes.c_void_p), ("rank_emb", ctypes.c_void_p),
    ] + [(name, ctypes.c_void_p * 4) for name in ("norm_w", "conv_w", "conv_b", "across_w", "out_w", "out_b")] + [
        ("final_norm", ctypes.c_void_p),
    ]


_SIGNATURES: dict[str, tuple[type, list]] = {
    "cg_last_error": (ctypes.c_char_p, []),
    "cg_version": (_i32, []),
    "cg_fault_status": (_i32, [ctypes.POINTER(_i32)]),
    "cg_launch_count": (_i64, []),
    "cg_attention_profiling": (_i32, [_i32, _i32]),
    "cg_attention_timings": (_i32, [ctypes.POINTER(_f32), _i32]),
    "cg_dense_profiling": (_i32, [_i32, _i32]),
    "cg_dense_timings": (_i32, [ctypes.POINTER(_f32), _i32]),
    "cg_decode_attention": (_i32, [_p, _i32, _p, _p, _i32, _i64, _i64, _i64, _p, _p, _i64, _i32, _i32, _i32, _i32, _i32,
                                   _f32, _p, _i32, _p]),
    "cg_kv_write_step": (_i32, [_p, _p, _i32, _i64, _i32, _i32, _i32, _p, _p, _i64, _i32, _p, _p, _i32, _p]),
    "cg_kv_copy_rows_workspace_bytes": (_i64, [_i32, _i32, _i32, _i32, _i32, _i64]),
    "cg_kv_copy_rows": (_i32, [_p, _p, _i32, _i32, _i64, _i32, _i32, _i32, _p, _p, _i64, _i32, _p, _i64, _p]),
    "cg_kv_copy_rows_noalloc_max_bytes": (_i64, []),
    "cg_kv_copy_rows_noalloc": (_i32, [_p, _p, _i32, _i32, _i64, _i32, _i32, _i32, _p, _p, _i64, _i32, _p]),
    "cg_trunk_blob_bytes": (_i64, [ctypes.POINTER(TrunkDims)]),
    "cg_trunk_part_offset": (_i64, [ctypes.POINTER(TrunkDims), _i32, _i32]),
    "cg_trunk_prepare": (_i32, [ctypes.POINTER(TrunkDims), _p, _p]),
    "cg_plump_embed": (_i32, [ctypes.POINTER(PlumpSchemaC), _p, _i32, _p, _i32, _i64, _p, _p]),
    "cg_onehot_bags": (_i32, [_p, _i32, _i64, _i64, _i32, ctypes.POINTER(_i64), _p, _i32, _i64, _i32, _p, _p]),
    "cg_bags_forward_ragged": (_i32, [ctypes.POINTER(TrunkDims), _p, _p, _i32, _i64, _i32, ctypes.POINTER(_i64), _p,
                                      _i64, _p, _i64, _i32, _p, _p, _p, _i32, _p, _p, _i32, _i64, _i32, _i32, _p, _i64,
                                      _p, _p]),
    "cg_card_grid": (_i32, [ctypes.POINTER(CardGridWeights), _p, _i32, _i64, _i64, _p, _p]),
    "cg_card_scorer": (_i32, [ctypes.POINTER(CardScorerWeights), _p, _i64, _p, _i32, _p, _p]),
    "cg_candidate_scorer": (_i32, [ctypes.POINTER(CandidateScorerWeights), _p, _i64, _i32, _i32, _p, _i32, _p, _p, _p,
                                   _p, _p, _p]),
    "cg_trunk_step_workspace_bytes": (_i64, [ctypes.POINTER(TrunkDims), _i64, _i32, _i32]),
    "cg_trunk_forward_ragged": (_i32, [ctypes.POINTER(TrunkDims), _p, _p, _p, _p, _i64, _i32, _p, _p, _p, _i32, _p, _p,
                                       _i32, _i64, _i32, _i32, _p, _i64, _p, _p]),
    "cg_plump_step_workspace_bytes": (_i64, [ctypes.POINTER(TrunkDims), _i64, _i32, _i32]),
    "cg_plump_forward_ragged": (_i32, [ctypes.POINTER(TrunkDims), _p, ctypes.POINTER(PlumpSchemaC), _p, _p, _i32, _i64,
                                       _i32, _p, _p, _p, _i32, _p, _p, _i32, _i64, _i32, _i32, _p, _i64, _p, _p]),
    "cg_trunk_condition": (_i32, [ctypes.POINTER(TrunkDims), _p, _p, _i64, _p, _p, _p, _i32, _p]),
    "cg_plump_decide": (_i32, [ctypes.POINTER(HeadsDesc), _p, _p, _p, _i64, _p, _p, _p, _p, _p, _p, _p, _p]),
    "cg_masked_sample": (_i32, [_p, _p, _p, _i64, _i32, _p, _p, _p]),
    "cg_gae_segments": (_i32, [_p, _i32, _p, _p, _i64, _p, _f64, _p, _p]),
    "cg_weighted_sums_workspace_bytes": (_i64, [_i64]),
    "cg_weighted_sums": (_i32, [_p, _p, _i64, _f64, _p, _p, _i64, _p]),
    "cg_normalize": (_i32, [_p, _i64, _f64, _f64, _p]),
    "cg_weighted_sums_shifted": (_i32, [_p, _p, _i64, _p, _p, _p, _i64, _p]),
    "cg_normalize_from_sums": (_i32, [_p, _i64, _p, _p, _p]),
    "cg_ppo_objective_workspace_bytes": (_i64, [_i64]),
    "cg_ppo_objective": (_i32, [_p, _p, _i64, _i32, _i64, _p, _p, _p, _f32, _f32, _p, _p, _p, _p, _i64, _p]),
    "cg_value_loss_workspace_bytes": (_i64, [_i64]),
    "cg_value_loss": (_i32, [_p, _p, _p, _p, _i64, _i32, _f32, _p, _p, _p, _i64, _p]),
    "cg_seat_values": (_i32, [_p, _i64, _i32, _p, _p, _p, _p, _i64, _i32, _p, _p, _p]),
    "cg_center_zero_sum": (_i32, [_p, _p, _i64, _i32, _p, _p]),
}


class NativeError(RuntimeError):
    """A C ABI call returned an error status."""


@lru_cache(maxsize=1)
def lib() -> ctypes.CDLL:
    if not LIBRARY.exists():
        raise RuntimeError(
            f"{LIBRARY} is missing: build it with `python -m card_playing_gym_b200.build` "
            "(the B200 path has no CPU fallback)"
        )
    handle = ctypes.CDLL(str(LIBRARY))
    for name, (restype, argtypes) in _SIGNATURES.items():
        fn = getattr(handle, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return handle


def declared_symbols() -> list[str]:
    return list(_SIGNATURES)


def call(name: str, *args) -> int:
    status = getattr(lib(), name)(*args)
    if status != 0:
        message = lib().cg_last_error().decode(errors="replace")
        raise NativeError(f"{name} failed ({status}): {message}")
    return status


def query(name: str, *args) -> int:
    value = getattr(lib(), name)(*args)
    if value < 0:
        raise NativeError(f"{name} rejected its arguments: {lib().cg_last_error().decode(errors='replace')}")
    return value


def fault_status() -> int:
    code = _i32(0)
    call("cg_fault_status", ctypes.byref(code))
    return code.value


def launch_count() -> int:
    return int(lib().cg_launch_count())


def attention_profiling(enable: bool, capacity: int = 4096) -> None:
    call("cg_attention_profiling", 1 if enable else 0, capacity)


def attention_timings(max_count: int = 1 << 16) -> list[float]:
    buffer = (_f32 * max_count)()
    count = lib().cg_attention_timings(buffer, max_count)
    if count < 0:
        raise NativeError("cg_attention_timings failed")
    return [buffer[i] for i in range(count)]


def dense_profiling(enable: bool, capacity: int = 4096) -> None:
    call("cg_dense_profiling", 1 if enable else 0, capacity)


def dense_timings(max_count: int = 1 << 16) -> list[float]:
    buffer = (_f32 * max_count)()
    count = lib().cg_dense_timings(buffer, max_count)
    if count < 0:
        raise NativeError("cg_dense_timings failed")
    return [buffer[i] for i in range(count)]


def ptr(tensor: torch.Tensor | None) -> int | None:
    if tensor is None:
        return None
    if not tensor.is_cuda:
        raise ValueError("card_playing_gym_b200 kernels take CUDA tensors only (there is no CPU path)")
    return tensor.data_ptr()


def stream_handle(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class Workspace:
    """A grow-only device scratch buffer per (device, purpose).

    A buffer that a larger one replaces is kept alive, not freed: a CUDA graph captured while it
    was current holds its address, and the next capture's ``empty_cache`` would otherwise return
    it to the driver, so that graph's replay would touch freed memory. Growth is geometric, so
    the retired buffers add up to less than the current one.
    """

    _buffers: dict[tuple[int, str], torch.Tensor] = {}
    _retired: list[torch.Tensor] = []

    @classmethod
    def get(cls, device: torch.device, nbytes: int, purpose: str = "step") -> torch.Tensor:
        index = device.index if device.index is not None else torch.cuda.current_device()
        key = (index, purpose)
        buffer = cls._buffers.get(key)
        if buffer is None or buffer.numel() < nbytes:
            size = max(int(nbytes), 256)
            if buffer is not None:
                cls._retired.append(buffer)
                size = max(size, 2 * buffer.numel())
            buffer = torch.empty(size, dtype=torch.uint8, device=device)
            cls._buffers[key] = buffer
        return buffer
