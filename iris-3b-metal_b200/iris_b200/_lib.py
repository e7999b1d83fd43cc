"""ctypes binding of ``libiris_b200.so`` (the C ABI in ``include/iris_b200.h``).

Loading fails loudly: there is no CPU or library fallback behind these
symbols. ``call`` raises ``ValueError`` for a rejected argument
(``IRIS_EINVAL``) and ``RuntimeError`` for a CUDA failure.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent / "libiris_b200.so"

IRIS_OK, IRIS_EINVAL, IRIS_ECUDA = 0, 1, 2
F32, BF16, F16 = 0, 1, 2
EPI_STORE, EPI_SWIGLU, EPI_GATE, EPI_HEADS, EPI_ADD, EPI_SILU = 0, 1, 2, 3, 4, 5
HEADS_LOCAL, HEADS_PEER_SCATTER, HEADS_PEER_BROADCAST_KV = 0, 1, 2
MAX_PEERS = 8  # IRIS_MAX_PEERS
IPC_HANDLE_BYTES = 64
NEXT_NONE, NEXT_NORM_MODULATE, NEXT_SILU_ADD = 0, 1, 2

P, I64, I32, F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float

# name -> argument types, in the order of include/iris_b200.h
SIGNATURES: dict[str, list] = {
    "iris_device_error": [I32, ctypes.POINTER(ctypes.c_uint), P],
    "iris_rms_norm_modulate": [P, I32, I64, I64, I64, P, I32, P, P, P, I64, I64, I64, I64, F, P],
    "iris_gated_residual_rms_norm": [
        P, I64, I64, I64, P, I32, I64, I64, I64, P, P, I64, I64, I64, I64, F, I32, P, P, P, I64, P, I32, I64, I64, I64, P
    ],
    "iris_rms_norm_add_rows": [P, P, P, I64, I64, I64, F, P],
    "iris_qk_norm_rope": [P, I32, I64, I64, I64, I64, I64, P, P, P, F, P, I32, I64, I64, P],
    "iris_qkv_heads": [P, I64, I64, I64, I64, I64, P, P, P, P, F, P, P, P, I64, I64, I64, I32, P],
    "iris_gemm_bf16": [P, I64, P, I64, P, I32, I64, I64, I64, I64, I32, P, P, I64, I64, I64, I64, I64, I64, I64, P],
    "iris_flash_attn_fwd": [P, P, P, P, I64, I64, I64, I64, I64, F, I64, P],
    "iris_pixel_rms_norm": [P, I32, P, P, I64, F, P],
    "iris_pixel_mlp": [P, I32, P, P, P, P, P, P, P, P, P, I64, F, P],
    "iris_pixel_mlp_head": [P, I32, P, P, P, P, P, P, P, P, P, P, P, I64, I64, I64, I64, I64, I64, F, P],
    "iris_pixel_embed": [P, P, P, P, P, I32, P, P, F, I64, I64, I64, I64, I64, I64, I64, P],
    "iris_patchify": [P, P, I64, I64, I64, I64, I64, I64, I64, P],
    "iris_block_copy": [P, I64, I64, I64, P, I64, I64, I64, I64, I64, I64, I64, P],
    "iris_unpatchify": [P, P, I64, I64, I64, I64, I64, P],
    "iris_timestep_embedding": [P, P, I64, I64, F, P],
    "iris_gemv": [P, I64, I64, P, I32, P, P, I64, I32, I32, P],
    "iris_add_bias_rows": [P, P, P, I64, I64, I64, P],
    "iris_cfg_euler": [P, P, P, I64, I64, F, F, F, I32, P],
    "iris_dpm_update": [P, P, P, P, P, I64, I64, F, I32, F, I32, F, F, F, P],
    "iris_all_finite": [P, I64, P, P],
    "iris_poison_on_error": [P, I64, ctypes.c_uint, P],
    "iris_small_attention": [P, I64, I64, I64, I64, I64, P, P, F, P, F, P, I64, P],
    "iris_layer_pool": [P, I64, I64, I64, P, P, P, P],
    "iris_tile_crop": [P, I64, I64, I64, I64, I64, I64, P, P],
    "iris_tile_accumulate": [P, I64, I64, I64, P, I64, P, I64, I64, F, P, P, P],
    "iris_tile_normalize": [P, P, I64, I64, I64, P],
}

class HeadsEpilogue(ctypes.Structure):
    """``iris_heads_epilogue`` of include/iris_b200.h."""

    _fields_ = [
        ("q_out", P), ("k_out", P), ("v_out", P), ("q_weight", P), ("k_weight", P), ("cos", P), ("sin", P),
        ("eps", F), ("head_major", I32), ("heads_q", I64), ("heads_kv", I64), ("tokens", I64), ("batch", I64),
        ("n_out", I64), ("n_out_kv", I64), ("peer_mode", I32), ("world", I32), ("token_offset", I64),
        ("n_dest", I64), ("q_peer", P * MAX_PEERS), ("k_peer", P * MAX_PEERS), ("v_peer", P * MAX_PEERS),
    ]  # fmt: skip


class GemmProblem(ctypes.Structure):
    """``iris_gemm_problem`` of include/iris_b200.h."""

    _fields_ = [
        ("a", P), ("lda", I64), ("w", P), ("ldw", I64), ("out", P), ("out_dtype", I32), ("ldc", I64),
        ("M", I64), ("N", I64), ("K", I64), ("epilogue", I32), ("bias", P), ("aux", P), ("ldaux", I64),
        ("out_seg_rows", I64), ("out_seg_stride", I64), ("out_seg_offset", I64),
        ("aux_seg_rows", I64), ("aux_seg_stride", I64), ("aux_seg_offset", I64),
        ("heads", ctypes.POINTER(HeadsEpilogue)),
    ]  # fmt: skip


class ResidualProblem(ctypes.Structure):
    """``iris_residual_problem`` of include/iris_b200.h."""

    _fields_ = [
        ("residual", P), ("res_seg_rows", I64), ("res_seg_stride", I64), ("res_seg_offset", I64),
        ("branch", P), ("br_seg_rows", I64), ("br_seg_stride", I64), ("br_seg_offset", I64),
        ("weight", P), ("gate", P), ("mod_stride", I64), ("rows", I64), ("rows_per_batch", I64),
        ("next_mode", I32), ("next_weight", P), ("next_shift", P), ("next_scale", P), ("next_mod_stride", I64),
        ("next_out", P), ("nx_seg_rows", I64), ("nx_seg_stride", I64), ("nx_seg_offset", I64),
    ]  # fmt: skip


SIGNATURES["iris_gated_residual_rms_norm_grouped"] = [ctypes.POINTER(ResidualProblem), I32, I32, I32, I64, F, P]
SIGNATURES["iris_gemm_bf16_grouped"] = [ctypes.POINTER(GemmProblem), I32, P]
SIGNATURES["iris_flash_attn_fwd_peers"] = [P, P, P, I64, I64, I64, I64, I64, I64, F, F, P, I32, I64, I64, I64, P]
SIGNATURES["iris_ipc_export"] = [P, P, ctypes.POINTER(I64)]
SIGNATURES["iris_ipc_import"] = [P, ctypes.POINTER(P)]
SIGNATURES["iris_ipc_close"] = [P]
SIGNATURES["iris_peer_barrier"] = [P, P, I32, I32, ctypes.c_uint, I64, P]
SIGNATURES["iris_flash_attn_fwd_split"] = [P, P, P, I64, I64, I64, I64, I64, I64, F, F, I64, P, P, P, P, I64, P]

_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """The loaded library; raises if it was not built."""
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            raise RuntimeError(
                f"{LIBRARY.name} is not built; run `python -m iris_b200.build` (needs nvcc) -- "
                "there is no CPU fallback for the B200 kernels"
            )
        lib = ctypes.CDLL(str(LIBRARY))
        lib.iris_last_error.restype = ctypes.c_char_p
        lib.iris_last_error.argtypes = []
        lib.iris_abi_version.restype = ctypes.c_int
        for name, argtypes in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = ctypes.c_int
        _lib = lib
    return _lib


_launches = 0
# kernels each entry point enqueues (1 unless listed)
_KERNELS_PER_CALL = {"iris_device_error": 0, "iris_all_finite": 2, "iris_ipc_export": 0, "iris_ipc_import": 0,
                     "iris_ipc_close": 0}


def launch_count() -> int:
    """Kernels of this library enqueued so far by this process (replays of a
    captured CUDA graph count the library kernels the graph holds)."""
    return _launches


def count_launches(n: int) -> None:
    """Adjust the count for kernels enqueued other than through :func:`call`
    (a CUDA graph replay) or counted while being captured rather than run."""
    global _launches
    _launches += n


def call(name: str, *args) -> None:
    global _launches
    status = getattr(load(), name)(*args)
    if status == IRIS_OK:
        _launches += _KERNELS_PER_CALL.get(name, 1)
        return
    message = load().iris_last_error().decode(errors="replace")
    if status == IRIS_EINVAL:
        raise ValueError(message)
    raise RuntimeError(f"{name}: {message}")


def exported_symbols() -> list[str]:
    return ["iris_last_error", "iris_abi_version", *SIGNATURES]
