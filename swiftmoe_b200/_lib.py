"""ctypes binding of libswiftmoe.so (the C ABI in include/swiftmoe.h).

The library is loaded from this package directory.  There is no fallback: if the
shared object is missing or a call fails, an exception is raised.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libswiftmoe.so"

SMOE_OK = 0
SMOE_F32, SMOE_F16, SMOE_BF16 = 0, 1, 2
SMOE_F32_SPLITW = 16   # layer dtype: fp32 with routed expert weights split for the tf32 tensor cores
SMOE_EXPERT_LINEAR, SMOE_EXPERT_SWIGLU = 0, 1
SMOE_EPI_STORE, SMOE_EPI_SWIGLU, SMOE_EPI_GATEUP = 0, 1, 3

DTYPE_CODE = {torch.float32: SMOE_F32, torch.float16: SMOE_F16, torch.bfloat16: SMOE_BF16}

_vp, _i32, _i64, _sz = C.c_void_p, C.c_int, C.c_int64, C.c_size_t


class LayerArgs(C.Structure):
    """Mirror of ``smoe_layer_args``."""
    _fields_ = [
        ("tokens", C.c_int32), ("d_model", C.c_int32), ("num_experts", C.c_int32), ("top_k", C.c_int32),
        ("expert_type", C.c_int32), ("d_ff", C.c_int32), ("dtype", C.c_int32), ("capacity", C.c_int32),
        ("num_shared", C.c_int32), ("d_ff_shared", C.c_int32),
        ("x", _vp), ("gate_w", _vp), ("logit_bias", _vp), ("w1", _vp), ("w3", _vp), ("w2", _vp),
        ("w_lin", _vp), ("sw1", _vp), ("sw3", _vp), ("sw2", _vp), ("out", _vp),
        ("topk_idx", _vp), ("topk_w", _vp), ("expert_counts", _vp),
        ("workspace", _vp), ("workspace_bytes", _sz),
        ("stage_events", _vp * 6),
    ]


class LayerBwdArgs(C.Structure):
    """Mirror of ``smoe_layer_bwd_args``."""
    _fields_ = [
        ("tokens", C.c_int32), ("d_model", C.c_int32), ("num_experts", C.c_int32), ("top_k", C.c_int32),
        ("d_ff", C.c_int32), ("dtype", C.c_int32), ("capacity", C.c_int32),
        ("num_shared", C.c_int32), ("d_ff_shared", C.c_int32),
        ("x", _vp), ("dout", _vp), ("gate_w", _vp), ("logit_bias", _vp),
        ("w1", _vp), ("w3", _vp), ("w2t", _vp), ("w13t", _vp),
        ("sw1", _vp), ("sw3", _vp), ("sw2t", _vp), ("sw13t", _vp),
        ("dx", _vp), ("dgate", _vp), ("dw13", _vp), ("dw2", _vp), ("dsw13", _vp), ("dsw2", _vp),
        ("workspace", _vp), ("workspace_bytes", _sz),
        ("expert_type", C.c_int32), ("dw_lin_transposed", C.c_int32), ("w_lin_t", _vp), ("dw_lin", _vp),
    ]


# name -> (restype, argtypes)
SIGNATURES = {
    "smoe_version": (C.c_char_p, []),
    "smoe_status_string": (C.c_char_p, [_i32]),
    "smoe_device_sm_count": (_i32, []),
    "smoe_read_device_error": (_i32, [C.POINTER(C.c_int), _vp]),
    "smoe_selftest_wait_timeout": (_i32, [C.c_uint64, _vp, _vp]),
    "smoe_router_fwd": (_i32, [_vp, _vp, _i32, _vp, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _sz, _vp]),
    "smoe_router_workspace_size": (_sz, [_i32, _i32, _i32, _i32]),
    "smoe_topk_from_logits": (_i32, [_vp, _i32, _i32, _i32, _vp, _vp, _vp]),
    "smoe_plan_workspace_size": (_sz, [_i32, _i32, _i32]),
    "smoe_plan_rows_cap": (_i64, [_i32, _i32, _i32, _i32, _i32]),
    "smoe_dispatch_plan": (_i32, [_vp, _i32, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _i64, _vp, _sz, _vp]),
    "smoe_dispatch_plan_noalloc": (_i32, [_vp, _i32, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _i64, _vp]),
    "smoe_permute_rows": (_i32, [_vp, _i32, _i32, _i32, _vp, _vp, _i32, _i64, _vp, _vp]),
    "smoe_combine": (_i32, [_vp, _i32, _vp, _vp, _i32, _i32, _i32, _vp, _vp, _vp]),
    "smoe_grouped_gemm": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp, _vp, _i32, _i64, _i32, _i32, _vp]),
    "smoe_grouped_gemm_rows": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp, _vp, _i32, _i64, _i32, _i32, _vp]),
    "smoe_transpose_batched": (_i32, [_vp, _vp, _i32, _i32, _i32, _i32, _vp]),
    "smoe_tf32_split_weights": (_i32, [_vp, _vp, _i64, _i32, _vp]),
    "smoe_gather_rows": (_i32, [_vp, _i32, _i32, _vp, _i64, _vp, _vp]),
    "smoe_ep_regroup_workspace_size": (_sz, [_i32, _i32]),
    "smoe_ep_regroup_plan": (_i32, [_vp, _i32, _i32, _i32, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "smoe_ep_return_rows": (_i32, [_vp, _vp, _i32, _vp, _i64, _vp, _i32, _i64, _vp, _i64, _vp]),
    "smoe_ep_dedup_ranks": (_i32, [_vp, _i64, _i32, _i32, _i32, _i32, _vp, _vp]),
    "smoe_ep_dedup_meta": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _vp, _vp, _vp, _vp]),
    "smoe_ep_layout": (_i32, [_vp, _i32, _i32, _i32, _i32, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _i32, _vp]),
    "smoe_ep_clear_tail": (_i32, [_vp, _vp, _i64, _i32, _vp]),
    "smoe_store_rows": (_i32, [_vp, _i64, _vp, _i64, _vp]),
    "smoe_copy_rows_count": (_i32, [_vp, _vp, _i64, _vp, _i64, _vp]),
    "smoe_ep_send_rows": (_i32, [_vp, _i64, _vp, _vp, _i32, _i32, _i32, _vp, _vp, _i64, _vp]),
    "smoe_ep_drop_slots": (_i32, [_vp, _i64, _vp, _i32, _vp, _vp, _vp]),
    "smoe_ep_buffer_create": (_i32, [_sz, C.POINTER(_vp), _vp]),
    "smoe_ep_buffer_destroy": (_i32, [_vp]),
    "smoe_ep_peer_open": (_i32, [_vp, C.POINTER(_vp)]),
    "smoe_ep_peer_close": (_i32, [_vp]),
    "smoe_copy_segments": (_i32, [C.POINTER(_vp), C.POINTER(_vp), C.POINTER(_sz), _i32, _vp]),
    "smoe_event_create": (_i32, [C.POINTER(_vp)]),
    "smoe_event_destroy": (_i32, [_vp]),
    "smoe_event_record": (_i32, [_vp, _vp]),
    "smoe_event_elapsed": (_i32, [_vp, _vp, C.POINTER(C.c_float)]),
    "smoe_layer_workspace_size": (_sz, [C.POINTER(LayerArgs)]),
    "smoe_layer_fwd": (_i32, [C.POINTER(LayerArgs), _vp]),
    "smoe_layer_bwd_workspace_size": (_sz, [C.POINTER(LayerBwdArgs)]),
    "smoe_layer_bwd": (_i32, [C.POINTER(LayerBwdArgs), _vp]),
    "smoe_wgrad_gemm": (_i32, [_vp, _i64, _vp, _i64, _i32, _vp, _i32, _i32, _i32, _i64, _vp, _vp]),
    "smoe_wgrad_gemm_rows": (_i32, [_vp, _i64, _vp, _i64, _i32, _vp, _i32, _i32, _i32, _i64, _vp, _vp]),
    "smoe_swiglu_bwd": (_i32, [_vp, _vp, _vp, _vp, _i64, _i32, _i32, _vp, _vp]),
    "smoe_linear_bwd": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i32, _i32, _vp, _vp]),
    "smoe_moe_bwd_dx": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _vp]),
    "smoe_router_dwg_workspace_size": (_sz, [_i32, _i32]),
    "smoe_router_dwg": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp, _vp, _sz, _vp]),
}

_lock = threading.Lock()
_lib = None


class SwiftMoEError(RuntimeError):
    pass


def load() -> C.CDLL:
    """Load libswiftmoe.so (raises if it has not been built)."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise SwiftMoEError(
                    f"{LIB_PATH} is missing: build it with `python -m swiftmoe_b200.build` "
                    "(no CPU fallback exists)")
            lib = C.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(status: int, what: str) -> None:
    if status != SMOE_OK:
        msg = load().smoe_status_string(status).decode()
        raise SwiftMoEError(f"{what} failed: {msg} (status {status})")


def ptr(t) -> int | None:
    if t is None:
        return None
    return t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dt: torch.dtype) -> int:
    try:
        return DTYPE_CODE[dt]
    except KeyError:
        raise SwiftMoEError(f"unsupported dtype {dt}") from None


class StageEvents:
    """Six library-side CUDA events for ``smoe_layer_args.stage_events``."""

    def __init__(self):
        lib = load()
        self.handles = []
        for _ in range(6):
            h = C.c_void_p()
            check(lib.smoe_event_create(C.byref(h)), "smoe_event_create")
            self.handles.append(h.value)

    def attach(self, args: "LayerArgs"):
        for i, h in enumerate(self.handles):
            args.stage_events[i] = h

    def elapsed(self, i: int, j: int) -> float:
        ms = C.c_float()
        check(load().smoe_event_elapsed(self.handles[i], self.handles[j], C.byref(ms)), "smoe_event_elapsed")
        return float(ms.value)

    def __del__(self):
        try:
            lib = load()
            for h in self.handles:
                lib.smoe_event_destroy(h)
        except Exception:
            pass
